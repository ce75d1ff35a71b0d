"""CPU: host side of the channel-sharded (tensor-parallel) target.

* sharding a model's weights and putting the shards back together is the identity, for 2 and 4
  ranks, and drawing a rank's shard directly equals sharding the full draw;
* the column-/row-parallel split computes the same projections as the full weights: the in-
  projection rows of a rank are the interleaved x2/x1/v triplets of its channels, the q/k/v rows
  of its heads, and the row-parallel partial sums of all ranks add up to the full product;
* the shared-region handles are exchanged in rank order over a world_size-2 gloo group.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from evspark_b200.config import TINY
from evspark_b200.tp import (connect_state, init_target_weights_sharded, shard_target_weights, shard_tensor,
                             unshard_target_weights)
from evspark_b200.weights import init_target_weights

# a bf16-free 7B-like miniature: 4 blocks, d = 512 so that d / 4 is still a multiple of 128
CFG = TINY.with_(name="tp_mini", d_model=512, n_heads=4, head_dim=128, mlp_inner=1024)


@pytest.mark.parametrize("world", [2, 4])
def test_shard_unshard_roundtrip(world):
    w = init_target_weights(CFG, seed=3)
    shards = [shard_target_weights(CFG, w, r, world) for r in range(world)]
    back = unshard_target_weights(CFG, shards)
    assert back.keys() == w.keys()
    for k in w:
        assert torch.equal(back[k], w[k]), k
    for r in range(world):
        direct = init_target_weights_sharded(CFG, r, world, seed=3)
        for k in w:
            assert torch.equal(direct[k], shards[r][k]), (r, k)


def test_parallel_projections_match_full():
    world = 2
    w = init_target_weights(CFG, seed=5)
    d, F = CFG.d_model, CFG.mlp_inner
    x = torch.randn(7, d, dtype=torch.float64)
    # Hyena in-projection: rank r's rows are the interleaved (x2, x1, v) triplets of its channels
    win = w["blocks.0.w_in"].double()
    full = (x @ win.T).reshape(7, d, 3)
    for r in range(world):
        loc = x @ shard_tensor(CFG, "blocks.0.w_in", win, r, world).T
        torch.testing.assert_close(loc.reshape(7, d // world, 3), full[:, r * d // world:(r + 1) * d // world])
    # attention q/k/v rows of the local heads, in [q | k | v] order as the kernels expect
    wq = w["blocks.3.w_qkv"].double()
    fq = x @ wq.T
    for r in range(world):
        loc = x @ shard_tensor(CFG, "blocks.3.w_qkv", wq, r, world).T
        dl = d // world
        for j in range(3):
            torch.testing.assert_close(loc[:, j * dl:(j + 1) * dl], fq[:, j * d + r * dl:j * d + (r + 1) * dl])
    # row-parallel: the partial sums of the ranks add up to the full product
    for name, width in (("blocks.0.w_out", d), ("blocks.3.w_o", d), ("blocks.1.w3", F)):
        W = w[name].double()
        z = torch.randn(7, width, dtype=torch.float64)
        k = width // world
        total = sum(z[:, r * k:(r + 1) * k] @ shard_tensor(CFG, name, W, r, world).T for r in range(world))
        torch.testing.assert_close(total, z @ W.T)


class _FakeLib:
    def __init__(self, rank):
        self.rank, self.got = rank, None

    def evs_state_tp_handle(self, h, buf):
        for i in range(64):
            buf[i] = bytes([(self.rank * 64 + i) % 251])
        return 0

    def evs_state_tp_connect(self, h, buf, world):
        self.got = bytes(buf)
        return 0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _exchange_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lib = _FakeLib(rank)
        connect_state(None, lib, world, "cpu")
        want = b"".join(bytes((r * 64 + i) % 251 for i in range(64)) for r in range(world))
        assert lib.got == want
        open(os.path.join(out, f"ok{rank}"), "w").close()
    finally:
        dist.destroy_process_group()


def test_handle_exchange_in_rank_order_gloo(tmp_path):
    mp.start_processes(_exchange_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    assert (tmp_path / "ok0").exists() and (tmp_path / "ok1").exists()
