"""CPU: host logic of the multi-GPU paths, run as world_size-2 gloo process groups.

* streams are partitioned over ranks contiguously, disjointly and completely;
* the bench's timing combine takes the max of the ranks' device times and the sum of their tokens;
* a batched multi-stream run, with its streams split over two ranks, emits for every stream the
  tokens that stream emits when one process decodes all of them (CPU oracle model and drafter).
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from evspark_b200.ranks import combine_timing, stream_partition


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(fn, world, *args):
    port = _free_port()
    mp.start_processes(fn, args=(world, port) + args, nprocs=world, join=True, start_method="spawn")


def test_stream_partition_covers_every_stream_once():
    for total in (0, 1, 7, 64):
        for world in (1, 2, 3, 8):
            seen = []
            for r in range(world):
                first, count = stream_partition(total, world, r)
                seen.extend(range(first, first + count))
            assert seen == list(range(total))
    with pytest.raises(ValueError):
        stream_partition(4, 2, 2)


def _timing_worker(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ms, tok = combine_timing(10.0 + rank, 3.0 * (rank + 1))
        assert ms == 10.0 + world - 1
        assert tok == 3.0 * world * (world + 1) / 2
    finally:
        dist.destroy_process_group()


def test_combine_timing_two_ranks_gloo():
    _run(_timing_worker, 2)
    assert combine_timing(5.0, 2.0) == (5.0, 2.0)  # no process group: identity


def _streams_worker(rank, world, port, prompts, n_tok, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle.loop import oracle_streams

        first, count = stream_partition(len(prompts), world, rank)
        em = oracle_streams(prompts[first:first + count], n_tok, seeds=list(range(first, first + count)))
        gathered = [None] * world
        dist.all_gather_object(gathered, (first, em))
        if rank == 0:
            np.save(os.path.join(out_dir, "sharded.npy"), np.stack([e for _, part in gathered for e in part]))
    finally:
        dist.destroy_process_group()


def test_streams_split_over_two_gloo_ranks_match_one_process(tmp_path):
    from oracle.loop import oracle_streams

    prompts = np.stack([np.random.default_rng(40 + b).choice([65, 67, 71, 84], size=24) for b in range(3)])
    n_tok = 6
    whole = np.stack(oracle_streams(prompts, n_tok, seeds=[0, 1, 2]))
    _run(_streams_worker, 2, prompts, n_tok, str(tmp_path))
    np.testing.assert_array_equal(np.load(tmp_path / "sharded.npy"), whole)
