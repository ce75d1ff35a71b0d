"""Replay-free state-slice rollback (evspark/specdec/block/slice.py:33-191).

Block index k in [0, chunk_len-1] is the last consumed token of the chunk ``[y, x_1..x_γ]``.
The device keeps every per-position state of the last retained forward (FIR inputs in
position-indexed rings, IIR states in per-position slots, KV rows in place), so rolling back
moves no data: ``evs_rollback`` rewrites each row's length and IIR slot index.  Argument
checks and error messages follow the reference (message fragments the reference tests match
are kept verbatim).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from evspark_b200.config import HCS


@dataclass
class ChunkStash:
    """Handle on the per-position states kept by one retained ``block_forward``."""

    L0: int
    chunk_len: int
    flash_attn: bool = True
    lengths_before: torch.Tensor | None = None
    model: object = field(default=None, repr=False)
    uid: int = 0

    @property
    def k_outer(self) -> dict:
        cfg = self.model.cfg
        return {i: cfg.short_filter_length for i, t in enumerate(cfg.layer_types) if t != "mha"}

    @property
    def k_inner(self) -> dict:
        cfg = self.model.cfg
        return {i: cfg.filter_length(t) for i, t in enumerate(cfg.layer_types) if t in ("hcs", "hcm")}

    @property
    def cat_u(self) -> dict:
        return dict.fromkeys(self.k_outer, "device")

    @property
    def x1v_cat(self) -> dict:
        return dict.fromkeys(self.k_inner, "device")

    @property
    def s_all(self) -> dict:
        cfg = self.model.cfg
        return dict.fromkeys(cfg.layer_idxs("hcl"), "device")


def _as_k_array(k, chunk_len: int, batch: int) -> np.ndarray:
    arr = np.asarray(k, dtype=np.int64).ravel()
    if arr.size == 1:
        arr = np.full(batch, int(arr[0]), dtype=np.int64)
    if arr.size != batch:
        raise ValueError(f"k has {arr.size} entries but the stash batch is {batch}")
    if np.any(arr < 0) or np.any(arr >= chunk_len):
        raise ValueError(f"k={arr.tolist()} outside the block indices [0, {chunk_len - 1}] (slice)")
    return arr


def slice_states_to_accept(ip_dict, stash: ChunkStash, k) -> None:
    if not isinstance(stash, ChunkStash):
        raise TypeError(f"stash must be a ChunkStash, got {type(stash)!r}")
    ip = ip_dict
    if stash.uid == 0 or stash.uid != ip.retained_uid:
        raise ValueError("stale ChunkStash: slice right after the retained block_forward of this state")
    batch = ip.batch
    ks = _as_k_array(k, stash.chunk_len, batch)
    uniform = bool(np.all(ks == ks[0]))
    if not uniform and not stash.flash_attn:
        raise ValueError("ragged slicing needs the flash_attn kvcache path (per-sample lengths); "
                         "collapse to one sequence first")
    L0 = ip.retained_len0[:batch]
    if not uniform:
        cfg = ip.model.cfg
        for kind, K in (("outer", cfg.short_filter_length), (HCS, cfg.hcs_filter_length)):
            if kind == HCS and not cfg.layer_idxs(HCS):
                continue
            widths = {int(min(L0[b] + ks[b] + 1, K - 1)) for b in range(batch)}
            if len(widths) > 1:
                raise ValueError("ragged slice below the HCS/outer FIR window gives 不同 FIR 状态长度 "
                                 f"(different FIR state widths) {sorted(widths)}; collapse first or use a longer prefix")
    ip.rollback(ks)
