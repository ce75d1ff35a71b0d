"""Model shapes for the StripedHyena2 target and the γ-parallel drafter.

The target's dense-block code lives in the absent ``vortex`` runtime, so the
conventions below are chosen here and implemented identically by the CUDA
kernels and the CPU oracle:

* block wiring: pre-norm RMSNorm → mixer → out-projection + residual, then
  RMSNorm → SwiGLU MLP ``w3(silu(w1 x) * w2 x)`` + residual; residual stream
  kept in fp32, GEMM inputs and mixer activations in the data dtype;
* no biases in the dense projections; final RMSNorm; tied unembedding
  (logits = norm(x) @ embed.T, fp32 out);
* Hyena mixer: in-projection ``d → 3d``, outer causal FIR K=3 over all 3d
  channels, de-interleave (channel 3h+j → group j) into ``x2, x1, v``
  (evspark/specdec/block/chunk.py:202-211), inner FIR (SE K=7 unflipped, MR
  K=128 flipped + gated bias D) or modal IIR (LI, real poles);
* MHA: fused qkv projection ``[q | k | v]``, rotate-half RoPE (base 10000),
  softmax(q·k/√Dh) causal, bottom-right aligned.

Block pattern: MHA at every 8th block (index % 8 == 7), the other blocks cycle
SE, MR, LI in order.  The tiny config is the fixed pattern [SE, MR, LI, MHA].
"""

from __future__ import annotations

from dataclasses import dataclass, field, replace

VOCAB_SIZE = 512
MASK_ID = 256
HEAD_DIM_DRAFTER = 64

HCS, HCM, HCL, MHA = "hcs", "hcm", "hcl", "mha"
LAYER_KINDS = (HCS, HCM, HCL, MHA)
#: integer codes used across the C ABI (include/evspark_sm100.h: EVS_LAYER_*)
LAYER_CODE = {HCS: 0, HCM: 1, HCL: 2, MHA: 3}


def striped_pattern(n_layers: int, attn_every: int = 8) -> tuple[str, ...]:
    """MHA at ``i % attn_every == attn_every-1``; other blocks cycle SE, MR, LI."""
    out = []
    n = 0
    for i in range(n_layers):
        if i % attn_every == attn_every - 1:
            out.append(MHA)
        else:
            out.append((HCS, HCM, HCL)[n % 3])
            n += 1
    return tuple(out)


@dataclass(frozen=True)
class TargetConfig:
    name: str
    d_model: int
    n_layers: int
    layer_types: tuple[str, ...]
    n_heads: int
    head_dim: int
    mlp_inner: int
    vocab_size: int = VOCAB_SIZE
    state_size: int = 16
    short_filter_length: int = 3
    hcs_filter_length: int = 7
    hcm_filter_length: int = 128
    eps: float = 1e-6
    rope_base: float = 10000.0
    dtype: str = "bf16"  # data dtype: "bf16" or "fp32"
    max_batch_size: int = 1

    def __post_init__(self):
        if len(self.layer_types) != self.n_layers:
            raise ValueError(f"layer_types has {len(self.layer_types)} entries, n_layers={self.n_layers}")
        bad = [t for t in self.layer_types if t not in LAYER_KINDS]
        if bad:
            raise ValueError(f"unknown layer kinds {bad}")
        if self.n_heads * self.head_dim != self.d_model:
            raise ValueError("n_heads * head_dim must equal d_model")
        if self.dtype not in ("bf16", "fp32"):
            raise ValueError(f"dtype must be bf16 or fp32, got {self.dtype}")

    def layer_idxs(self, kind: str) -> list[int]:
        return [i for i, t in enumerate(self.layer_types) if t == kind]

    def filter_length(self, kind: str) -> int | None:
        return {HCS: self.hcs_filter_length, HCM: self.hcm_filter_length}.get(kind)

    def get(self, key, default=None):
        return getattr(self, key, default)

    def with_(self, **kw) -> "TargetConfig":
        return replace(self, **kw)


@dataclass(frozen=True)
class DrafterConfig:
    d_model: int
    gamma: int
    inject_layers: tuple[str, ...]
    target_hidden: int
    n_layers: int = 2
    vocab_size: int = VOCAB_SIZE
    mask_id: int = MASK_ID
    ctx_window: int = 64
    mlp_mult: int = 4
    n_heads: int | None = None

    @property
    def heads(self) -> int:
        return self.n_heads if self.n_heads is not None else max(1, self.d_model // HEAD_DIM_DRAFTER)

    @property
    def n_inject(self) -> int:
        return len(self.inject_layers)


TINY = TargetConfig(
    name="tiny", d_model=256, n_layers=4, layer_types=(HCS, HCM, HCL, MHA),
    n_heads=8, head_dim=32, mlp_inner=704, dtype="fp32",
)
EVO2_7B = TargetConfig(
    name="evo2_7b", d_model=4096, n_layers=32, layer_types=striped_pattern(32),
    n_heads=32, head_dim=128, mlp_inner=11008, dtype="bf16",
)
EVO2_40B = TargetConfig(
    name="evo2_40b", d_model=8192, n_layers=50, layer_types=striped_pattern(50),
    n_heads=64, head_dim=128, mlp_inner=22528, dtype="bf16",
)
#: 7B-width, four blocks (one of each kind): full-width parity case that fits a CPU oracle run
EVO2_7B_SLICE = EVO2_7B.with_(name="evo2_7b_slice", n_layers=4, layer_types=(HCS, HCM, HCL, MHA))

TARGETS = {c.name: c for c in (TINY, EVO2_7B, EVO2_40B, EVO2_7B_SLICE)}

DRAFTERS = {
    "tiny": DrafterConfig(d_model=128, gamma=12, inject_layers=("blocks.2",), target_hidden=256),
    "evo2_7b": DrafterConfig(d_model=1024, gamma=12, inject_layers=("blocks.27",), target_hidden=4096),
    "evo2_40b": DrafterConfig(d_model=1024, gamma=12, inject_layers=("blocks.45",), target_hidden=8192),
    "evo2_7b_slice": DrafterConfig(d_model=1024, gamma=12, inject_layers=("blocks.2",), target_hidden=4096),
}


def target_config(name: str) -> TargetConfig:
    try:
        return TARGETS[name]
    except KeyError:
        raise ValueError(f"unknown model_name {name!r}; known: {sorted(TARGETS)}") from None
