"""Stub ``vortex.model.model``: the oracle StripedHyena2 in vortex's shape.

TEST INFRASTRUCTURE ONLY.  ``HyenaCascade.forward`` implements the two paths
the reference leaves to vortex — the parallel prefill (empty state) and the
single-token step — with ``oracle.model``'s math; the γ-token chunk path is the
reference's own ``hyena_chunk_forward`` once ``install_chunk_forward()`` has
patched this class (evspark/specdec/block/chunk.py:55-75).
"""

from __future__ import annotations

import torch
import torch.nn as nn

from oracle.model import OracleTarget, fir_chunk, fir_prefill
from evspark_b200.config import HCL, HCM, HCS, MHA

from .utils import dotdict, interleave


class InferenceParams:
    """Attention cache container (vortex layout ``[B, Lmax, 2, H, Dh]``)."""

    def __init__(self, max_seqlen, max_batch_size, seqlen_offset=0):
        self.max_seqlen = max_seqlen
        self.max_batch_size = max_batch_size
        self.seqlen_offset = seqlen_offset
        self.batch_size_offset = 0
        self.key_value_memory_dict = {}
        self.lengths_per_sample = None


class RecurrentInferenceParams:
    """Hyena state container: FIR tails and IIR states per layer."""

    def __init__(self, fir_filter_length, state_dim, seqlen_offset=0):
        self.fir_filter_length = fir_filter_length
        self.state_dim = state_dim
        self.seqlen_offset = seqlen_offset
        self.fir_state_dict = {}
        self.fir_inner_state_dict = {}
        self.state_dict = {}


class HyenaCascade(nn.Module):
    def __init__(self, oracle: OracleTarget, layer_idx: int, kind: str, config):
        super().__init__()
        cfg = oracle.cfg
        self.oracle = oracle
        self.kind = kind
        self.config = config
        self.layer_idx = layer_idx
        self.hidden_size = cfg.d_model
        self.data_dtype = None
        self.short_filter_length = cfg.short_filter_length
        self.short_filter_weight = oracle.w[f"blocks.{layer_idx}.short_w"]
        self.short_filter_bias = None
        self.column_split_hyena = False
        self.num_attention_heads = cfg.n_heads
        self.hidden_size_per_attention_head = cfg.head_dim
        self.hyena_flip_x1x2 = False
        self.hyena_filter_groups = 1
        self.fir_inner_filter_length = cfg.filter_length(kind)
        self.h = oracle.w.get(f"blocks.{layer_idx}.inner_w")
        self.D = oracle.w.get(f"blocks.{layer_idx}.D")
        lp = oracle.w.get(f"blocks.{layer_idx}.log_poles")
        self.log_poles = None if lp is None else lp[..., None]  # [G=d, S, 1]
        self.residues = oracle.w.get(f"blocks.{layer_idx}.residues")

    def forward(self, u, inference_params=None, padding_mask=None, *args, **kwargs):
        """Prefill (offset 0) or a single-token step; u [B, T, 3H] -> y [B, T, H]."""
        if self.data_dtype is None:
            self.data_dtype = u.dtype
        ip = inference_params
        i = self.layer_idx
        prefill = ip is None or ip.seqlen_offset == 0 or i not in ip.fir_state_dict
        T = u.shape[1]
        if not prefill and T != 1:
            raise RuntimeError("stub vortex: multi-token forward on a filled state needs the chunk path")
        K0 = self.short_filter_length
        xo = u.permute(0, 2, 1).to(torch.float32)
        w_short = self.short_filter_weight.to(torch.float32)
        if prefill:
            zo, new_o, _ = fir_prefill(xo, w_short, K0, flip=False, gated=None)
        else:
            zo, new_o, _ = fir_chunk(ip.fir_state_dict[i], xo, w_short, K0, flip=False, gated=None)
        if ip is not None:
            ip.fir_state_dict[i] = new_o
        z = interleave(zo.to(u.dtype))
        H = self.hidden_size
        x2, x1, v = z.split([H, H, H], dim=1)
        x1v = x1 * v
        if self.kind in (HCS, HCM):
            K = self.fir_inner_filter_length
            flip = K >= 128
            gated = self.D.to(torch.float32) if flip else None
            w = self.h.to(torch.float32)
            if prefill:
                zi, new_i, _ = fir_prefill(x1v.to(torch.float32), w, K, flip=flip, gated=gated)
            else:
                zi, new_i, _ = fir_chunk(ip.fir_inner_state_dict[i], x1v.to(torch.float32), w, K,
                                         flip=flip, gated=gated)
            if ip is not None:
                ip.fir_inner_state_dict[i] = new_i
            y = x2 * zi.to(u.dtype)
        else:
            p = torch.exp(self.log_poles[..., 0].to(torch.float32))  # [H, S]
            if prefill:
                s = x1v.new_zeros(u.shape[0], H, p.shape[-1], dtype=torch.float32)
            else:
                s = ip.state_dict[i].to(torch.float32)
            xv = x1v.to(torch.float32)
            res = torch.empty_like(xv)
            for t in range(T):
                s = p[None] * s + xv[..., t:t + 1]
                res[..., t] = (self.residues.to(torch.float32)[None] * s).sum(-1)
            if ip is not None:
                ip.state_dict[i] = s
            y = (x2.to(torch.float32) * (res + self.D.to(torch.float32)[None, :, None] * xv)).to(u.dtype)
        return y.permute(0, 2, 1), inference_params


class _HyenaBlock(nn.Module):
    def __init__(self, oracle, i, kind, config):
        super().__init__()
        self.o, self.i, self.kind = oracle, i, kind
        self.filter = HyenaCascade(oracle, i, kind, config)

    def forward(self, x, ip_dict=None):
        o, i = self.o, self.i
        a = o.rmsnorm(x, o.w[f"blocks.{i}.pre_norm"])
        u = a @ o.w[f"blocks.{i}.w_in"].T
        ip = None if ip_dict is None else ip_dict[self.kind]
        y, _ = self.filter(u, inference_params=ip)
        x = x + y @ o.w[f"blocks.{i}.w_out"].T
        return _mlp(o, i, x), None


class _MHABlock(nn.Module):
    def __init__(self, oracle, i):
        super().__init__()
        self.o, self.i = oracle, i

    def forward(self, x, ip_dict=None):
        o, i = self.o, self.i
        cfg = o.cfg
        B, T, d = x.shape
        H, Dh = cfg.n_heads, cfg.head_dim
        a = o.rmsnorm(x, o.w[f"blocks.{i}.pre_norm"])
        qkv = (a @ o.w[f"blocks.{i}.w_qkv"].T).view(B, T, 3, H, Dh)
        off = 0 if ip_dict is None else int(ip_dict["mha"].seqlen_offset)
        pos = torch.arange(off, off + T)
        qh = o.rope(qkv[:, :, 0], pos)
        kh = o.rope(qkv[:, :, 1], pos)
        vh = qkv[:, :, 2]
        if ip_dict is not None:
            mha = ip_dict["mha"]
            cache = mha.key_value_memory_dict.get(i)
            if cache is None:
                cache = torch.zeros(mha.max_batch_size, mha.max_seqlen, 2, H, Dh, dtype=x.dtype)
                mha.key_value_memory_dict[i] = cache
            cache[:B, off:off + T, 0] = kh
            cache[:B, off:off + T, 1] = vh
            keys, vals = cache[:B, :off + T, 0], cache[:B, :off + T, 1]
        else:
            keys, vals = kh, vh
        sc = torch.einsum("bthd,blhd->bhtl", qh, keys) * (Dh ** -0.5)
        mask = torch.arange(off + T)[None, :] > pos[:, None]
        sc = sc.masked_fill(mask[None, None], float("-inf"))
        out = torch.einsum("bhtl,blhd->bthd", torch.softmax(sc, -1), vals).reshape(B, T, d)
        x = x + out @ o.w[f"blocks.{i}.w_o"].T
        return _mlp(o, i, x), None


def _mlp(o, i, x):
    b = o.rmsnorm(x, o.w[f"blocks.{i}.post_norm"])
    g1 = b @ o.w[f"blocks.{i}.w1"].T
    g = g1 * torch.sigmoid(g1) * (b @ o.w[f"blocks.{i}.w2"].T)
    return x + g @ o.w[f"blocks.{i}.w3"].T


class StripedHyena(nn.Module):
    """``model(ids, inference_params_dict) -> (logits, None)`` over the oracle weights."""

    def __init__(self, oracle: OracleTarget, max_batch_size: int = 1):
        super().__init__()
        cfg = oracle.cfg
        self.oracle = oracle
        self.config = dotdict(
            hidden_size=cfg.d_model, vocab_size=cfg.vocab_size, max_batch_size=max_batch_size,
            use_flash_attn=False, interleave=True, state_size=cfg.state_size,
        )
        blocks = []
        for i, kind in enumerate(cfg.layer_types):
            blocks.append(_MHABlock(oracle, i) if kind == MHA else _HyenaBlock(oracle, i, kind, self.config))
        self.blocks = nn.ModuleList(blocks)

    def initialize_inference_params(self, max_seqlen=None):
        cfg = self.oracle.cfg
        max_seqlen = int(max_seqlen)
        out = {"mha": InferenceParams(max_seqlen, int(self.config.max_batch_size))}
        for kind in (HCL, HCM, HCS):
            out[kind] = RecurrentInferenceParams(cfg.filter_length(kind) or cfg.short_filter_length,
                                                 cfg.state_size)
        return out

    def forward(self, ids, inference_params_dict=None, padding_mask=None):
        o = self.oracle
        x = o.w["embed"][ids.long()]
        for blk in self.blocks:
            x, _ = blk(x, inference_params_dict)
        h = o.rmsnorm(x, o.w["final_norm"])
        return h @ o.w["embed"].T, None
