"""CPU: the block-by-block bf16 parity harness (tests/_parity.py) is exact and has teeth.

The oracle itself stands in for the device: its fp32-compute run plays the device, its fp64
run is the reference, and a copy with one planted mistake must fail the bounds.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from evspark_b200.config import HCL, HCM, HCS, MHA, TargetConfig
from evspark_b200.weights import init_target_weights
from oracle.model import OracleTarget, block_over_segments
from tests import _parity

CFG = TargetConfig(name="bf16_small", d_model=512, n_layers=4, layer_types=(HCS, HCM, HCL, MHA), n_heads=4,
                   head_dim=128, mlp_inner=1024, dtype="bf16")


@pytest.fixture(scope="module")
def setup():
    w = init_target_weights(CFG, seed=11)
    rng = np.random.default_rng(4)
    prompt = rng.choice([65, 67, 71, 84], size=24)
    chunk = rng.choice([65, 67, 71, 84], size=13)
    return w, prompt, chunk


def _stand_in_device(w, prompt, chunk, compute):
    """(xs [n_layers, P, d], prefill logits, block logits) of the oracle run as a device would."""
    o = OracleTarget(CFG, w, compute=compute, emulate=True)
    st = o.init_state(1, 64)
    pre, _, cap1 = o.forward(prompt[None], st, prefill=True, capture_layers=tuple(range(CFG.n_layers)))
    blk, _, cap2 = o.forward(chunk[None], st, capture_layers=tuple(range(CFG.n_layers)))
    xs = torch.stack([torch.cat([cap1[i], cap2[i]], 1)[0].to(torch.float32) for i in range(CFG.n_layers)])
    return xs, pre[0].float(), blk[0].float()


def test_block_over_segments_equals_full_forward_bitwise(setup):
    w, prompt, chunk = setup
    xs, pre, blk = _stand_in_device(w, prompt, chunk, torch.float64)
    rep = _parity.teacher_forced_report(CFG, w, np.concatenate([prompt, chunk]), len(prompt), xs, pre, blk,
                                        free_running=True)
    # fp64 reference on the fp64 run's own residual streams: the same arithmetic, block by block
    assert all(b["rel_max"] == 0.0 for b in rep["blocks"]), rep["blocks"]
    assert rep["logits_err"] < 1e-6 and rep["free_running_err"] < 1e-6


def test_fp32_compute_passes_the_bounds(setup):
    w, prompt, chunk = setup
    xs, pre, blk = _stand_in_device(w, prompt, chunk, torch.float32)
    rep = _parity.teacher_forced_report(CFG, w, np.concatenate([prompt, chunk]), len(prompt), xs, pre, blk)
    _parity.assert_teacher_forced(rep)


@pytest.mark.parametrize("slot,scale", [("w_in", 1.02), ("inner_w", 1.05), ("residues", 1.05), ("w_o", 1.03)])
def test_planted_mistake_fails(setup, slot, scale):
    """A stand-in device whose one block computes with a slightly wrong weight fails the bounds."""
    w, prompt, chunk = setup
    layer = {"w_in": 0, "inner_w": 1, "residues": 2, "w_o": 3}[slot]
    bad = dict(w)
    bad[f"blocks.{layer}.{slot}"] = (w[f"blocks.{layer}.{slot}"].float() * scale).to(w[f"blocks.{layer}.{slot}"].dtype)
    xs, pre, blk = _stand_in_device(bad, prompt, chunk, torch.float32)
    rep = _parity.teacher_forced_report(CFG, w, np.concatenate([prompt, chunk]), len(prompt), xs, pre, blk)
    with pytest.raises(AssertionError):
        _parity.assert_teacher_forced(rep)
    others = [b for b in rep["blocks"] if b["block"] != layer]
    assert all(b["rel_max"] <= _parity.TOL_BLOCK_MAX for b in others)


def test_block_over_segments_matches_chunked_forward():
    """Prefill then a chunk, block by block, equals the whole model's prefill then chunk."""
    w = init_target_weights(CFG, seed=12)
    rng = np.random.default_rng(9)
    ids = rng.choice([65, 67, 71, 84], size=30)
    o = OracleTarget(CFG, w)
    st = o.init_state(1, 64)
    o.forward(ids[None, :17], st, prefill=True)
    ref, _, _ = o.forward(ids[None, 17:], st)
    x = o.embed(ids[None])
    segs = [x[:, :17], x[:, 17:]]
    for i in range(CFG.n_layers):
        lw = {k.split(".", 2)[2]: v for k, v in w.items() if k.startswith(f"blocks.{i}.")}
        segs = block_over_segments(CFG, i, lw, segs)
    got = o.head(segs[1])
    assert torch.equal(got, ref)
