"""Seeded random initialisation of the target and drafter weights.

Real Evo2 / drafter checkpoints are not available, so every run uses
random-init weights of the configured shape.  Each tensor is drawn from its own
``torch.Generator`` (seed derived from the model seed and the tensor index), so
a given (config, seed, device type) always yields the same weights.

Distributions: dense input projections and the (tied) embedding N(0, 0.02²);
residual out-projections (Hyena ``w_out``, attention ``w_o``, MLP ``w3``)
N(0, 1/fan_in); norm scales 1 + N(0, 0.1²) (the final norm included); FIR taps
N(0, 1/K); IIR real poles |p| ~ U(0.9, 0.999) stored as ``log_poles``;
residues N(0, 1/S); D N(0, 0.5²).  The logits have a standard deviation of
0.02 * sqrt(d) (1.3 at Evo2-7B width).  Out-projections of N(0, 1/fan_in)
keep the blocks' contributions well above the embedding row in the residual
stream; with the GPT-style 0.02 / sqrt(2 n_layers) instead, the 4-block
tiny model's greedy argmax repeats its input token at 92 % of positions.
"""

from __future__ import annotations

import math

import torch

from .config import HCL, HCM, HCS, MHA, DrafterConfig, TargetConfig

_DT = {"bf16": torch.bfloat16, "fp32": torch.float32}


def data_dtype(cfg: TargetConfig) -> torch.dtype:
    return _DT[cfg.dtype]


def target_weight_specs(cfg: TargetConfig) -> list[tuple[str, tuple[int, ...], str, str]]:
    """``(name, shape, init kind, storage)`` in a fixed order; storage 'data' or 'fp32'."""
    d, F, S = cfg.d_model, cfg.mlp_inner, cfg.state_size
    specs: list[tuple[str, tuple[int, ...], str, str]] = [("embed", (cfg.vocab_size, d), "embed", "data")]
    for i, kind in enumerate(cfg.layer_types):
        p = f"blocks.{i}."
        specs.append((p + "pre_norm", (d,), "norm", "fp32"))
        if kind == MHA:
            specs.append((p + "w_qkv", (3 * d, d), "dense", "data"))
            specs.append((p + "w_o", (d, d), "dense_out", "data"))
        else:
            specs.append((p + "w_in", (3 * d, d), "dense", "data"))
            specs.append((p + "short_w", (3 * d, cfg.short_filter_length), "fir", "fp32"))
            if kind in (HCS, HCM):
                specs.append((p + "inner_w", (d, cfg.filter_length(kind)), "fir", "fp32"))
            if kind in (HCM, HCL):
                specs.append((p + "D", (d,), "dvec", "fp32"))
            if kind == HCL:
                specs.append((p + "log_poles", (d, S), "poles", "fp32"))
                specs.append((p + "residues", (d, S), "residues", "fp32"))
            specs.append((p + "w_out", (d, d), "dense_out", "data"))
        specs.append((p + "post_norm", (d,), "norm", "fp32"))
        specs.append((p + "w1", (F, d), "dense", "data"))
        specs.append((p + "w2", (F, d), "dense", "data"))
        specs.append((p + "w3", (d, F), "dense_out", "data"))
    specs.append(("final_norm", (d,), "final_norm", "fp32"))
    return specs


def _draw(kind: str, shape, gen: torch.Generator, device, cfg: TargetConfig) -> torch.Tensor:
    f32 = torch.float32
    if kind in ("dense", "embed"):
        return torch.randn(shape, generator=gen, device=device, dtype=f32) * 0.02
    if kind == "dense_out":
        return torch.randn(shape, generator=gen, device=device, dtype=f32) / math.sqrt(shape[1])
    if kind in ("norm", "final_norm"):
        return 1.0 + 0.1 * torch.randn(shape, generator=gen, device=device, dtype=f32)
    if kind == "fir":
        return torch.randn(shape, generator=gen, device=device, dtype=f32) / math.sqrt(shape[-1])
    if kind == "dvec":
        return 0.5 * torch.randn(shape, generator=gen, device=device, dtype=f32)
    if kind == "poles":
        u = torch.rand(shape, generator=gen, device=device, dtype=torch.float64)
        return torch.log(0.9 + 0.099 * u).to(f32)
    if kind == "residues":
        return torch.randn(shape, generator=gen, device=device, dtype=f32) / math.sqrt(shape[-1])
    raise ValueError(kind)


def init_target_weights(cfg: TargetConfig, seed: int = 20260820, device="cpu") -> dict[str, torch.Tensor]:
    """Seeded target weights; data-dtype GEMM weights, fp32 filter/norm parameters."""
    device = torch.device(device)
    out: dict[str, torch.Tensor] = {}
    for idx, (name, shape, kind, storage) in enumerate(target_weight_specs(cfg)):
        gen = torch.Generator(device=device)
        gen.manual_seed(int(seed) * 1_000_003 + idx)
        t = _draw(kind, shape, gen, device, cfg)
        out[name] = t.to(data_dtype(cfg) if storage == "data" else torch.float32).contiguous()
    return out


def init_target_tensor(cfg: TargetConfig, name: str, seed: int = 20260820, device="cpu") -> torch.Tensor:
    """One named tensor of ``init_target_weights(cfg, seed, device)``, drawn alone (same bits)."""
    device = torch.device(device)
    for idx, (nm, shape, kind, storage) in enumerate(target_weight_specs(cfg)):
        if nm == name:
            gen = torch.Generator(device=device)
            gen.manual_seed(int(seed) * 1_000_003 + idx)
            t = _draw(kind, shape, gen, device, cfg)
            return t.to(data_dtype(cfg) if storage == "data" else torch.float32).contiguous()
    raise KeyError(name)


def drafter_weight_specs(dcfg: DrafterConfig) -> list[tuple[str, tuple[int, ...], str]]:
    """Parameter names follow the reference ``Drafter`` module (evspark/train/drafter.py:274-336)."""
    d, H, V = dcfg.d_model, dcfg.target_hidden, dcfg.vocab_size
    hid = dcfg.mlp_mult * d
    specs = [
        ("embed.weight", (V, H), "embed"),
        ("in_proj.weight", (d, H), "lin"), ("in_proj.bias", (d,), "bias"),
        ("out_proj.weight", (H, d), "out"), ("out_proj.bias", (H,), "zero"),
        ("pos.weight", (dcfg.gamma, d), "pos"),
    ]
    if dcfg.n_inject > 0:
        specs += [("ctx_proj.weight", (d, dcfg.n_inject * H), "lin"), ("ctx_proj.bias", (d,), "bias"),
                  ("ctx_norm.scale", (d,), "one")]
    for l in range(dcfg.n_layers):
        p = f"layers.{l}."
        specs += [(p + "ln1.scale", (d,), "one")]
        for nm in ("q_proj", "k_proj", "v_proj", "o_proj"):
            specs.append((p + nm + ".weight", (d, d), "lin"))
        specs += [(p + "ln2.scale", (d,), "one"),
                  (p + "mlp.0.weight", (hid, d), "lin"), (p + "mlp.0.bias", (hid,), "bias"),
                  (p + "mlp.2.weight", (d, hid), "lin"), (p + "mlp.2.bias", (d,), "bias")]
    specs += [("final_ln.scale", (d,), "one"), ("markov", (V, V), "markov"),
              ("conf_w.weight", (1, 2 * d), "lin"), ("conf_w.bias", (1,), "bias")]
    return specs


def init_drafter_weights(dcfg: DrafterConfig, seed: int = 20260830, device="cpu",
                         embed: torch.Tensor | None = None) -> dict[str, torch.Tensor]:
    """Seeded fp32 drafter weights (nn.Linear-style uniform init, Markov bias 0.5·N(0,1)).

    ``embed`` (the target's embedding) is copied into the frozen drafter
    embedding when given, as the reference training does (drafter.py:338-345).
    """
    device = torch.device(device)
    out: dict[str, torch.Tensor] = {}
    for idx, (name, shape, kind) in enumerate(drafter_weight_specs(dcfg)):
        gen = torch.Generator(device=device)
        gen.manual_seed(int(seed) * 1_000_003 + idx)
        f32 = torch.float32
        if kind == "lin":
            bound = 1.0 / math.sqrt(shape[-1])
            t = (torch.rand(shape, generator=gen, device=device, dtype=f32) * 2 - 1) * bound
        elif kind == "bias":
            t = (torch.rand(shape, generator=gen, device=device, dtype=f32) * 2 - 1) * 0.02
        elif kind == "out":
            t = torch.randn(shape, generator=gen, device=device, dtype=f32) * 0.02
        elif kind == "zero":
            t = torch.zeros(shape, device=device, dtype=f32)
        elif kind == "one":
            t = torch.ones(shape, device=device, dtype=f32)
        elif kind == "pos":
            t = torch.randn(shape, generator=gen, device=device, dtype=f32)
        elif kind == "embed":
            t = torch.randn(shape, generator=gen, device=device, dtype=f32) * (2.0 / math.sqrt(shape[-1]))
        elif kind == "markov":
            t = 0.5 * torch.randn(shape, generator=gen, device=device, dtype=f32)
        else:
            raise ValueError(kind)
        out[name] = t.contiguous()
    if embed is not None:
        if tuple(embed.shape) != tuple(out["embed.weight"].shape):
            raise ValueError(f"embedding shape {tuple(embed.shape)} != {tuple(out['embed.weight'].shape)}")
        out["embed.weight"] = embed.detach().to(device=device, dtype=torch.float32).contiguous()
    return out
