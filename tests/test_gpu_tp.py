"""GPU (2 GPUs): the channel-sharded target, two ranks in two processes.

The 7B-width 4-block model is split over two GPUs (half the Hyena channels, attention heads and
MLP features per rank; the row-parallel partial sums are added across the ranks inside the
residual + RMSNorm over NVLink).  Checks:

* both ranks produce bit-identical logits (everything after the cross-rank sum is replicated);
* the 13-token block forward equals 13 native T=1 steps bit for bit on the sharded model;
* every block and the logits agree with the bf16-emulating oracle of the full (unsharded) model
  on the device's own residual stream, within the single-GPU bounds (tests/_parity.py);
* greedy speculative decoding equals native greedy decoding on the sharded model.

Skipped when fewer than two GPUs are visible.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    rng = np.random.default_rng(3)
    prompt = rng.choice([65, 67, 71, 84], size=40)
    chunk = rng.choice([65, 67, 71, 84], size=13)
    return prompt, chunk


def _tp_worker(rank, world, port, out_dir):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from evspark_b200.config import EVO2_7B_SLICE
        from evspark_b200.model import TargetModel
        from evspark_b200.specdec.block import block_forward, clone_inference_params, prefill, step_forward_reference
        from evspark_b200.specdec.block.loop import native_greedy_reference, speculative_generate
        from evspark_b200.tp import init_target_weights_sharded
        from oracle.loop import IdentityDraft
        from tests import _parity

        dev = torch.device("cuda", rank)
        model = TargetModel.random(EVO2_7B_SLICE, seed=7, device=dev, init_on="cpu", tp=(rank, world))
        prompt, chunk = _inputs()
        ip = model.initialize_inference_params(128)
        prefill(model, torch.tensor(prompt)[None], ip)
        ip2 = clone_inference_params(ip)
        block = block_forward(model, torch.tensor(chunk)[None], ip)[0].cpu().double().numpy()
        step = step_forward_reference(model, torch.tensor(chunk)[None], ip2)[0].cpu().double().numpy()
        ip.close()
        ip2.close()
        pr = torch.tensor(prompt[:32])[None]
        nat, ipn, _ = native_greedy_reference(model, pr, 24)
        ipn.close()
        spec = speculative_generate(model, IdentityDraft(), pr, 24, 12, greedy=True, rng=np.random.default_rng(0))
        spec.inference_params_dict.close()
        model.close()
        # residual streams of every block (the capture ring holds the full, replicated stream)
        ws = init_target_weights_sharded(EVO2_7B_SLICE, rank, world, seed=7, device="cpu")
        xs, pre, blk = _parity.device_block_outputs(EVO2_7B_SLICE, ws, prompt, chunk, dev, tp=(rank, world))
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), block=block, step=step, nat=nat, spec=spec.emitted_ids,
                 xs=xs.numpy(), pre=pre.numpy(), blk=blk.numpy())
    finally:
        dist.destroy_process_group()


def test_two_rank_channel_sharded_7b_width(tmp_path):
    if not torch.cuda.is_available() or torch.cuda.device_count() < WORLD:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    mp.start_processes(_tp_worker, args=(WORLD, _free_port(), str(tmp_path)), nprocs=WORLD, join=True,
                       start_method="spawn")
    r = [np.load(tmp_path / f"rank{k}.npz") for k in range(WORLD)]
    for k in range(1, WORLD):
        assert np.array_equal(r[0]["block"], r[k]["block"]), "ranks disagree on the logits"
        assert np.array_equal(r[0]["spec"], r[k]["spec"])
    assert np.array_equal(r[0]["block"], r[0]["step"]), "sharded block forward != native T=1 steps"
    np.testing.assert_array_equal(r[0]["spec"], r[0]["nat"])

    from evspark_b200.config import EVO2_7B_SLICE
    from evspark_b200.weights import init_target_weights
    from tests import _parity

    for k in range(1, WORLD):
        assert np.array_equal(r[0]["xs"], r[k]["xs"]), "ranks disagree on the residual stream"
    assert np.array_equal(r[0]["blk"], r[0]["block"])
    cfg = EVO2_7B_SLICE
    w = init_target_weights(cfg, seed=7)
    prompt, chunk = _inputs()
    rep = _parity.teacher_forced_report(cfg, w, np.concatenate([prompt, chunk]), len(prompt),
                                        torch.as_tensor(r[0]["xs"]), torch.as_tensor(r[0]["pre"]),
                                        torch.as_tensor(r[0]["blk"]), free_running=True)
    _parity.assert_teacher_forced(rep)
