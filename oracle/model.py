"""StripedHyena2 target restated on CPU — the parity oracle (TEST INFRASTRUCTURE ONLY).

Semantics follow the reference where it defines them:

* outer short FIR (K=3, unflipped) and inner FIR (SE K=7 unflipped; MR K=128
  flipped with gated bias ``D·x1v``): full window = causal correlation over
  ``[state | x]``; a state shorter than K-1 grows token by token and uses the
  *first* c+1 taps (unflipped) or the *last* c+1 taps of the flipped kernel
  (evspark/specdec/block/chunk.py:88-159);
* de-interleave + split into ``x2, x1, v`` (chunk.py:202-211), ``x1v = x1*v``
  in the data dtype, ``y = x2 * z`` (chunk.py:221-248);
* modal IIR: ``s_j = p∘s_{j-1} + x1v_j`` from the injected ``s0``, every
  per-position state kept, ``y = x2∘(Σ_s R s_j + D x1v_j)`` (chunk.py:251-295);
  computed here by the recurrence in the oracle's compute dtype (the reference
  evaluates the same sums with one FFT);
* rollback to block index k: FIR window ``cat[max(0,S+k+1-(K-1)) : S+k+1]``,
  ragged widths left-zero-padded for flipped filters and refused otherwise,
  IIR ``s_all[..., k]``, lengths ``L0 + k + 1`` (evspark/specdec/block/slice.py:70-191).

Prefill (an empty state, vortex's parallel path) uses the zero-padded causal
convolution and stores the last ``min(L, K-1)`` inputs as the FIR state.

The dense conventions (pre-norm blocks, SwiGLU, rotate-half RoPE, tied
unembedding) are the ones documented in ``evspark_b200.config``.

Modes: ``compute=torch.float64, emulate=False`` is the reference arithmetic; ``emulate=True``
rounds at every point where the device stores the data dtype (bf16 / fp32)
and keeps the residual stream in fp32, like the CUDA path.
"""

from __future__ import annotations

import copy
from dataclasses import dataclass, field

import numpy as np
import torch

from evspark_b200.config import HCL, HCM, HCS, MHA, TargetConfig


@dataclass
class OracleState:
    """Per-sequence caches in the reference's (vortex) layout."""

    batch: int
    max_seqlen: int
    lengths: np.ndarray  # int64 [B]: tokens consumed per row
    outer: dict = field(default_factory=dict)  # layer -> [B, 3d, S<=2]
    inner: dict = field(default_factory=dict)  # layer -> [B, d, S<=K-1]
    iir: dict = field(default_factory=dict)  # layer -> [B, d, state_size]
    kv: dict = field(default_factory=dict)  # layer -> [B, Lmax, 2, H, Dh]

    def clone(self) -> "OracleState":
        return copy.deepcopy(self)


@dataclass
class OracleStash:
    """Per-position intermediates of one chunk forward (slice.py:33-52)."""

    L0: np.ndarray
    chunk_len: int
    cat_u: dict = field(default_factory=dict)
    k_outer: dict = field(default_factory=dict)
    x1v_cat: dict = field(default_factory=dict)
    k_inner: dict = field(default_factory=dict)
    s_all: dict = field(default_factory=dict)


def fir_chunk(state: torch.Tensor, x: torch.Tensor, w: torch.Tensor, K: int, *, flip: bool,
              gated: torch.Tensor | None):
    """Chunk FIR over ``[state | x]`` with the step path's growing-state tap rule.

    state [B,C,S] (S<=K-1), x [B,C,T], w [C,K]; returns (z [B,C,T], new_state, cat).
    """
    B, C, S = state.shape
    T = x.shape[-1]
    if S > K - 1:
        raise ValueError(f"FIR state width {S} > K-1={K - 1}")
    cat = torch.cat([state, x], dim=-1)
    z = torch.empty_like(x)
    for t in range(T):
        c = min(S + t, K - 1)
        cache = cat[..., S + t - c: S + t]  # oldest first, width c
        if flip:
            # y = sum_a w[a] x_{t-a}; the cache entry i has age c-i
            taps = w[:, :c + 1].flip(-1)  # [C, c+1], aligned oldest..newest
        else:
            taps = w[:, :c + 1]  # first c+1 taps: w[c] on the newest input
        win = torch.cat([cache, x[..., t:t + 1]], dim=-1)
        z[..., t] = (win * taps).sum(-1)
    if gated is not None:
        z = z + gated[None, :, None] * x
    new_state = cat[..., -min(S + T, K - 1):] if min(S + T, K - 1) > 0 else cat[..., :0]
    return z, new_state.contiguous(), cat


def fir_prefill(x: torch.Tensor, w: torch.Tensor, K: int, *, flip: bool, gated: torch.Tensor | None):
    """Zero-padded causal convolution from an empty state (parallel prefill)."""
    B, C, T = x.shape
    wo = w.flip(-1) if flip else w  # correlation taps: wo[j] multiplies x_{t-(K-1)+j}
    xp = torch.cat([x.new_zeros(B, C, K - 1), x], dim=-1)
    z = torch.zeros_like(x)
    for j in range(K):
        z = z + wo[None, :, j:j + 1] * xp[..., j:j + T]
    if gated is not None:
        z = z + gated[None, :, None] * x
    return z, x[..., -min(T, K - 1):].contiguous(), None


def fir_window(cat: torch.Tensor, kk: int, s: int, K: int) -> torch.Tensor:
    end = s + int(kk) + 1
    return cat[..., max(0, end - (K - 1)):end]


def gather_fir_windows(cat: torch.Tensor, ks: np.ndarray, s: int, K: int) -> torch.Tensor:
    if bool(np.all(ks == ks[0])):
        return fir_window(cat, int(ks[0]), s, K)
    wins = [fir_window(cat[b], int(ks[b]), s, K) for b in range(cat.shape[0])]
    widths = {int(w.shape[-1]) for w in wins}
    if len(widths) == 1:
        return torch.stack(wins, 0)
    if K < 128:
        raise ValueError("ragged slice would give different FIR state widths for an unflipped filter")
    width = max(widths)
    out = cat.new_zeros(*cat.shape[:-1], width)
    for b, w in enumerate(wins):
        out[b, ..., width - w.shape[-1]:] = w
    return out


class OracleTarget:
    """CPU StripedHyena2 with the conventions shared with the CUDA path."""

    def __init__(self, cfg: TargetConfig, weights: dict, compute=torch.float64, emulate: bool = False):
        self.cfg = cfg
        self.ct = compute
        self.emulate = emulate
        self.data_torch = torch.bfloat16 if cfg.dtype == "bf16" else torch.float32
        self.w = {k: v.detach().to("cpu").to(compute) for k, v in weights.items()}
        self.poles = {}
        for i, kind in enumerate(cfg.layer_types):
            if kind == HCL:
                lp = weights[f"blocks.{i}.log_poles"].detach().to("cpu")
                # the device computes p = exp(log_p) once in fp32
                p = torch.exp(lp.to(torch.float32)) if emulate else torch.exp(lp.to(torch.float64))
                self.poles[i] = p.to(compute)
        half = cfg.head_dim // 2
        self.inv_freq = torch.tensor(
            [cfg.rope_base ** (-2.0 * j / cfg.head_dim) for j in range(half)], dtype=torch.float64)

    # -- rounding points -----------------------------------------------------
    def q(self, x: torch.Tensor) -> torch.Tensor:
        """Storage in the data dtype."""
        return x.to(self.data_torch).to(self.ct) if self.emulate else x

    def r32(self, x: torch.Tensor) -> torch.Tensor:
        """Storage in fp32 (residual stream, logits, FIR/IIR states)."""
        return x.to(torch.float32).to(self.ct) if self.emulate else x

    # -- state ---------------------------------------------------------------
    def init_state(self, batch: int, max_seqlen: int) -> OracleState:
        cfg = self.cfg
        d = cfg.d_model
        st = OracleState(batch=batch, max_seqlen=max_seqlen, lengths=np.zeros(batch, dtype=np.int64))
        for i, kind in enumerate(cfg.layer_types):
            if kind == MHA:
                st.kv[i] = torch.zeros(batch, max_seqlen, 2, cfg.n_heads, cfg.head_dim, dtype=self.ct)
            else:
                st.outer[i] = torch.zeros(batch, 3 * d, 0, dtype=self.ct)
                if kind in (HCS, HCM):
                    st.inner[i] = torch.zeros(batch, d, 0, dtype=self.ct)
                else:
                    st.iir[i] = torch.zeros(batch, d, cfg.state_size, dtype=self.ct)
        return st

    # -- ops -----------------------------------------------------------------
    def rmsnorm(self, x, scale):
        ms = (x * x).mean(-1, keepdim=True)
        return x * torch.rsqrt(ms + self.cfg.eps) * scale

    def rope(self, x: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        """Rotate-half RoPE; x [..., T, H, Dh], pos [T] absolute positions."""
        ang = pos.to(torch.float64)[:, None] * self.inv_freq[None, :]  # [T, half]
        cos = torch.cos(ang).to(self.ct)[:, None, :]
        sin = torch.sin(ang).to(self.ct)[:, None, :]
        if self.emulate:
            cos, sin = self.r32(cos), self.r32(sin)
        half = self.cfg.head_dim // 2
        x1, x2 = x[..., :half], x[..., half:]
        return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)

    def _mha(self, i: int, a: torch.Tensor, st: OracleState) -> torch.Tensor:
        cfg = self.cfg
        B, T, d = a.shape
        H, Dh = cfg.n_heads, cfg.head_dim
        qkv = self.q(a @ self.w[f"blocks.{i}.w_qkv"].T).view(B, T, 3, H, Dh)
        out = torch.empty(B, T, H, Dh, dtype=self.ct)
        cache = st.kv[i]
        for b in range(B):
            L0 = int(st.lengths[b])
            if L0 + T > st.max_seqlen:
                raise ValueError(f"KV cache overflow: {L0 + T} > {st.max_seqlen}")
            pos = torch.arange(L0, L0 + T)
            qh = self.q(self.rope(qkv[b, :, 0], pos))
            kh = self.q(self.rope(qkv[b, :, 1], pos))
            cache[b, L0:L0 + T, 0] = kh
            cache[b, L0:L0 + T, 1] = qkv[b, :, 2]
            keys = cache[b, :L0 + T, 0]  # [L, H, Dh]
            vals = cache[b, :L0 + T, 1]
            sc = torch.einsum("thd,lhd->htl", qh, keys) * (Dh ** -0.5)
            mask = torch.arange(L0 + T)[None, :] > pos[:, None]  # [T, L]
            sc = sc.masked_fill(mask[None], float("-inf"))
            p = torch.softmax(sc, dim=-1)
            out[b] = torch.einsum("htl,lhd->thd", p, vals)
        return self.q(out.reshape(B, T, d))

    def _hyena(self, i: int, kind: str, u: torch.Tensor, st: OracleState, prefill: bool,
               stash: OracleStash | None) -> torch.Tensor:
        cfg = self.cfg
        K0 = cfg.short_filter_length
        xo = u.transpose(1, 2)  # [B, 3d, T]
        w_short = self.w[f"blocks.{i}.short_w"]
        if prefill:
            zo, new_o, _ = fir_prefill(xo, w_short, K0, flip=False, gated=None)
            cat = None
        else:
            zo, new_o, cat = fir_chunk(st.outer[i], xo, w_short, K0, flip=False, gated=None)
        st.outer[i] = self.r32(new_o)
        if stash is not None:
            stash.cat_u[i] = cat
            stash.k_outer[i] = K0
        zq = self.q(zo)
        x2, x1, v = zq[:, 0::3], zq[:, 1::3], zq[:, 2::3]
        x1v = self.q(x1 * v)
        if kind in (HCS, HCM):
            K = cfg.filter_length(kind)
            flip = kind == HCM
            gated = self.w[f"blocks.{i}.D"] if kind == HCM else None
            w_in = self.w[f"blocks.{i}.inner_w"]
            if prefill:
                z, new_i, cat_i = fir_prefill(x1v, w_in, K, flip=flip, gated=gated)
            else:
                z, new_i, cat_i = fir_chunk(st.inner[i], x1v, w_in, K, flip=flip, gated=gated)
            st.inner[i] = self.r32(new_i)
            if stash is not None:
                stash.x1v_cat[i] = cat_i
                stash.k_inner[i] = K
            y = self.q(x2 * self.q(self.r32(z)))
        else:
            p = self.poles[i]  # [d, S]
            R = self.w[f"blocks.{i}.residues"]
            D = self.w[f"blocks.{i}.D"]
            s = st.iir[i]
            T = x1v.shape[-1]
            s_all = torch.empty(*s.shape, T, dtype=self.ct)
            for t in range(T):
                s = self.r32(p[None] * s + x1v[..., t:t + 1])
                s_all[..., t] = s
            st.iir[i] = s.contiguous()
            if stash is not None:
                stash.s_all[i] = s_all
            res = (R[None, :, :, None] * s_all).sum(2)  # [B, d, T]
            y = self.q(x2 * self.r32(res + D[None, :, None] * x1v))
        return y.transpose(1, 2)

    def embed(self, ids) -> torch.Tensor:
        """Embedding lookup: the residual stream entering block 0, ``[B, T, d]``."""
        ids = torch.as_tensor(np.asarray(ids), dtype=torch.long)
        return self.w["embed"][ids[None] if ids.dim() == 1 else ids]

    def block(self, i: int, x: torch.Tensor, st: OracleState, *, prefill: bool = False,
              stash: OracleStash | None = None) -> torch.Tensor:
        """Block ``i`` on the residual stream ``x [B, T, d]`` (returned updated).

        Advances the layer's FIR/IIR/KV state; ``st.lengths`` (the tokens consumed before this
        chunk) is read, not advanced.
        """
        kind = self.cfg.layer_types[i]
        a = self.q(self.rmsnorm(x, self.w[f"blocks.{i}.pre_norm"]))
        if kind == MHA:
            o = self._mha(i, a, st)
            x = self.r32(x + o @ self.w[f"blocks.{i}.w_o"].T)
        else:
            u = self.q(a @ self.w[f"blocks.{i}.w_in"].T)
            y = self._hyena(i, kind, u, st, prefill, stash)
            x = self.r32(x + y @ self.w[f"blocks.{i}.w_out"].T)
        bn = self.q(self.rmsnorm(x, self.w[f"blocks.{i}.post_norm"]))
        g1 = bn @ self.w[f"blocks.{i}.w1"].T
        g2 = bn @ self.w[f"blocks.{i}.w2"].T
        g = self.q(g1 * torch.sigmoid(g1) * g2)
        return self.r32(x + g @ self.w[f"blocks.{i}.w3"].T)

    def head(self, x: torch.Tensor) -> torch.Tensor:
        """Final RMSNorm and tied unembedding: fp32 logits ``[B, T, V]``."""
        h = self.q(self.rmsnorm(x, self.w["final_norm"]))
        return self.r32(h @ self.w["embed"].T)

    def forward(self, ids, st: OracleState, *, prefill: bool = False, retain: bool = False,
                capture_layers: tuple[int, ...] = ()):
        """Run ``ids [B,T]`` through the model from ``st`` (advanced in place).

        ``prefill=True`` requires an empty state.  Returns ``(logits [B,T,V],
        stash or None, captured {layer: [B,T,d]})``.
        """
        cfg = self.cfg
        x = self.embed(ids)
        B, T = x.shape[:2]
        if B != st.batch:
            raise ValueError(f"batch {B} != state batch {st.batch}")
        if prefill and np.any(st.lengths != 0):
            raise ValueError("prefill requires an empty state")
        stash = OracleStash(L0=st.lengths.copy(), chunk_len=T) if retain else None
        captured = {}
        for i in range(cfg.n_layers):
            x = self.block(i, x, st, prefill=prefill, stash=stash)
            if i in capture_layers:
                captured[i] = x.clone()
        logits = self.head(x)
        st.lengths = st.lengths + T
        return logits, stash, captured

    def step_reference(self, ids, st: OracleState):
        """Token-by-token path; row i = logits after consuming ids[:, i]."""
        ids = np.asarray(ids)
        if ids.ndim == 1:
            ids = ids[None]
        outs = [self.forward(ids[:, t:t + 1], st)[0] for t in range(ids.shape[1])]
        return torch.cat(outs, dim=1)

    def slice(self, st: OracleState, stash: OracleStash, k) -> None:
        """Roll the state back to block index ``k`` (scalar or per-row)."""
        ks = np.asarray(k, dtype=np.int64).ravel()
        if ks.size == 1:
            ks = np.full(st.batch, int(ks[0]), dtype=np.int64)
        if ks.size != st.batch:
            raise ValueError(f"k has {ks.size} entries for batch {st.batch}")
        if np.any(ks < 0) or np.any(ks >= stash.chunk_len):
            raise ValueError(f"k={ks.tolist()} outside [0, {stash.chunk_len - 1}]")
        for i, cat in stash.cat_u.items():
            K = stash.k_outer[i]
            s = cat.shape[-1] - stash.chunk_len
            st.outer[i] = gather_fir_windows(cat, ks, s, K).clone()
        for i, cat in stash.x1v_cat.items():
            K = stash.k_inner[i]
            s = cat.shape[-1] - stash.chunk_len
            st.inner[i] = gather_fir_windows(cat, ks, s, K).clone()
        for i, s_all in stash.s_all.items():
            st.iir[i] = torch.stack([s_all[b, ..., int(ks[b])] for b in range(st.batch)], 0)
        st.lengths = stash.L0 + ks + 1


def block_over_segments(cfg: TargetConfig, i: int, layer_weights: dict, xs: list, *, compute=torch.float64,
                        emulate: bool = False) -> list:
    """Block ``i`` alone, from an empty state, over consecutive chunks of its input stream.

    ``layer_weights`` maps the block's slot names (``w_in``, ``pre_norm``, ...) to tensors and
    ``xs`` is a list of residual-stream chunks ``[B, T_j, d]``: the first is prefilled (the
    parallel path of an empty state), each later one runs as a chunk forward on the state the
    earlier ones left.  Returns the block's output for every chunk.  One block's weights are held
    at a time, so models of any depth fit host memory when run block by block.
    """
    kind = cfg.layer_types[i]
    sub = cfg.with_(name=f"{cfg.name}.block{i}", n_layers=1, layer_types=(kind,))
    o = OracleTarget(sub, {f"blocks.0.{k}": v for k, v in layer_weights.items()}, compute=compute, emulate=emulate)
    B = xs[0].shape[0]
    st = o.init_state(B, sum(int(x.shape[1]) for x in xs))
    outs = []
    for j, x in enumerate(xs):
        outs.append(o.block(0, x.to(compute), st, prefill=(j == 0)))
        st.lengths = st.lengths + int(x.shape[1])
    return outs
