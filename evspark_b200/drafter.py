"""γ-parallel neural drafter on the device (the reference ``Drafter``, evspark/train/drafter.py:274-409).

``DeviceDrafter`` holds the fp32 drafter parameters in HBM (same names as the reference module's
state_dict) and one ``evs_drafter`` handle; ``propose`` runs trunk + serial Markov head +
confidence head for a batch of rows in one ``evs_draft_propose`` call, reading the injected
hidden-state context straight from the target state's capture ring.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _native as N
from .checkpoint import SCHEME_LAYERS, read_drafter_checkpoint  # noqa: F401  (SCHEME_LAYERS re-exported)
from .config import DrafterConfig
from .weights import drafter_weight_specs, init_drafter_weights


def layer_index(name: str) -> int:
    if not name.startswith("blocks."):
        raise ValueError(f"injection layer must be 'blocks.N', got {name!r}")
    return int(name.split(".")[1])


class DeviceDrafter:
    def __init__(self, dcfg: DrafterConfig, weights: dict[str, torch.Tensor], *, device="cuda:0",
                 max_batch: int = 1):
        self.cfg = dcfg
        self.device = torch.device(device)
        self.gamma = int(dcfg.gamma)
        self.ctx_window = int(dcfg.ctx_window)
        self.max_batch = int(max_batch)
        names = [n for n, _, _ in drafter_weight_specs(dcfg)]
        missing = [n for n in names if n not in weights]
        if missing:
            raise ValueError(f"drafter weights missing {missing[:4]}")
        self.weights = {n: weights[n].detach().to(self.device, torch.float32).contiguous() for n in names}
        c = N.DrafterConfig()
        c.d_model, c.n_layers, c.n_heads, c.gamma = dcfg.d_model, dcfg.n_layers, dcfg.heads, dcfg.gamma
        c.n_inject, c.target_hidden, c.vocab_size, c.mask_id = dcfg.n_inject, dcfg.target_hidden, dcfg.vocab_size, dcfg.mask_id
        c.ctx_window, c.mlp_mult = dcfg.ctx_window, dcfg.mlp_mult
        h = C.c_void_p()
        with torch.cuda.device(self.device):
            N.check(N.lib().evs_drafter_create(C.byref(c), self.max_batch, C.byref(h)), "evs_drafter_create")
            self._h = h
            for n, t in self.weights.items():
                N.check(N.lib().evs_drafter_set_tensor(h, N.drafter_tensor_id(n), t.data_ptr(), t.numel()), n)
            N.check(N.lib().evs_drafter_finalize(h), "evs_drafter_finalize")

    @classmethod
    def random(cls, dcfg: DrafterConfig, seed: int = 20260830, *, embed: torch.Tensor | None = None,
               device="cuda:0", max_batch: int = 1, init_on: str = "cpu"):
        w = init_drafter_weights(dcfg, seed=seed, device=device if init_on == "cuda" else "cpu",
                                 embed=None if embed is None else embed.float())
        return cls(dcfg, w, device=device, max_batch=max_batch)

    def propose(self, ip, anchors: torch.Tensor, gamma: int, greedy: bool, *, temperature: float = 1.0,
                top_k: int | None = 4, uniforms: torch.Tensor | None = None, forced: torch.Tensor | None = None,
                want_U: bool = False):
        """anchors int64 [B] (device).  Returns device (tokens [B,γ'], q fp64 [B,γ',V], conf [B,γ'], U|None)."""
        B = int(anchors.shape[0])
        V = self.cfg.vocab_size
        dev = self.device
        toks = torch.empty(B, gamma, dtype=torch.int64, device=dev)
        q = torch.empty(B, gamma, V, dtype=torch.float64, device=dev)
        conf = torch.empty(B, gamma, dtype=torch.float32, device=dev)
        U = torch.empty(B, gamma, V, dtype=torch.float32, device=dev) if want_U else None
        k = 0 if top_k is None else int(top_k)
        N.check(N.lib().evs_draft_propose(self._h, ip.handle, anchors.data_ptr(), B, int(gamma), int(greedy),
                                          float(temperature), k, N.ptr(uniforms), N.ptr(forced), toks.data_ptr(),
                                          q.data_ptr(), conf.data_ptr(), N.ptr(U), N.stream_ptr()),
                "evs_draft_propose")
        return toks, q, conf, U

    def propose_into(self, ip, anchors: torch.Tensor, gamma: int, greedy: bool, toks: torch.Tensor,
                     q: torch.Tensor, conf: torch.Tensor, *, temperature: float = 1.0, top_k: int | None = 4,
                     uniforms: torch.Tensor | None = None, forced: torch.Tensor | None = None) -> None:
        """``propose`` into caller-owned outputs (tokens int64 [B,γ'], q fp64 [B,γ',V], conf fp32 [B,γ']):
        a fixed sequence of launches over fixed buffers, which a CUDA graph can capture and replay."""
        B = int(anchors.shape[0])
        V = self.cfg.vocab_size
        if (toks.shape != (B, gamma) or q.shape != (B, gamma, V) or conf.shape != (B, gamma)
                or toks.dtype != torch.int64 or q.dtype != torch.float64 or conf.dtype != torch.float32):
            raise ValueError("propose_into: outputs must be int64 [B,γ'], fp64 [B,γ',V] and fp32 [B,γ']")
        k = 0 if top_k is None else int(top_k)
        N.check(N.lib().evs_draft_propose(self._h, ip.handle, anchors.data_ptr(), B, int(gamma), int(greedy),
                                          float(temperature), k, N.ptr(uniforms), N.ptr(forced), toks.data_ptr(),
                                          q.data_ptr(), conf.data_ptr(), None, N.stream_ptr()),
                "evs_draft_propose")

    def close(self):
        if getattr(self, "_h", None):
            N.lib().evs_drafter_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def load_checkpoint(path: str, target_hidden: int, *, device="cuda:0", max_batch: int = 1) -> tuple:
    """Drafter .pt of the reference schema {scheme, d_model, gamma, state_dict, ...}
    (evspark/train/train_drafter.py:557-571) -> (DeviceDrafter, layer_names, meta)."""
    dcfg, sd, layers, meta = read_drafter_checkpoint(path, target_hidden)
    return DeviceDrafter(dcfg, sd, device=device, max_batch=max_batch), layers, meta
