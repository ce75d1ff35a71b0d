"""GPU parity at full size: the whole 32-block Evo2-7B shape, the Evo2-40B width and the 7B drafter.

* Evo2-7B shape (32 blocks: 10 SE, 9 MR, 9 LI, 4 MHA; d = 4096, 32 heads, F = 11008), bf16:
  every block and the logits of a prefill + γ+1 verify block against the bf16-emulating oracle on
  the device's residual stream (tests/_parity.py), plus block == native steps bit for bit.  The
  oracle runs one block at a time, so host memory holds one block's weights.
* Evo2-40B width (d = 8192, 64 heads, F = 22528), its first 8 blocks (SE, MR, LI, ..., MHA at 7).
* The drafter at 7B width (d = 1024, 16 heads, context rows 4096 wide as from block 27) against the
  reference ``Drafter`` outputs (tests/golden/drafter_7b.npz).
"""

from __future__ import annotations

import gc

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from evspark_b200 import _native as N

    N.call("evs_device_check")
    return torch.device("cuda:0")


def _inputs(seed):
    from evspark_b200.workload import markov_prompt

    prompt = markov_prompt(40, seed)
    chunk = np.concatenate([prompt[-1:], np.random.default_rng(seed + 1).choice([65, 67, 71, 84], size=12)])
    return prompt, chunk


def _run(cfg, seed, cuda, free_running):
    from evspark_b200.model import TargetModel
    from evspark_b200.specdec.block import block_forward, clone_inference_params, prefill, step_forward_reference
    from evspark_b200.weights import init_target_weights
    from tests import _parity

    w = init_target_weights(cfg, seed=seed, device=cuda)
    prompt, chunk = _inputs(seed)
    model = TargetModel(cfg, w, device=cuda, max_chunk=64)
    ip = model.initialize_inference_params(128, max_chunk=64)
    prefill(model, torch.tensor(prompt)[None], ip)
    ip2 = clone_inference_params(ip)
    logits = block_forward(model, torch.tensor(chunk)[None], ip)[0]
    step = step_forward_reference(model, torch.tensor(chunk)[None], ip2)[0]
    assert torch.equal(logits, step), "block forward != native T=1 steps"
    ip.close()
    ip2.close()
    model.close()
    xs, pre, blk = _parity.device_block_outputs(cfg, w, prompt, chunk, cuda)
    assert torch.equal(blk, logits.cpu())
    rep = _parity.teacher_forced_report(cfg, w, np.concatenate([prompt, chunk]), len(prompt), xs, pre, blk,
                                        free_running=free_running)
    del w, xs
    gc.collect()
    torch.cuda.empty_cache()
    return rep


def test_evo2_7b_full_depth_bf16_vs_oracle(cuda):
    from evspark_b200.config import EVO2_7B
    from tests import _parity

    rep = _run(EVO2_7B, 31, cuda, free_running=True)
    _parity.assert_teacher_forced(rep)


def test_evo2_40b_width_bf16_vs_oracle(cuda):
    from evspark_b200.config import EVO2_40B
    from tests import _parity

    cfg = EVO2_40B.with_(name="evo2_40b_first8", n_layers=8, layer_types=EVO2_40B.layer_types[:8])
    assert cfg.layer_types == ("hcs", "hcm", "hcl", "hcs", "hcm", "hcl", "hcs", "mha")
    rep = _run(cfg, 41, cuda, free_running=False)
    _parity.assert_teacher_forced(rep)


@pytest.mark.parametrize("T", [0, 64])
def test_device_drafter_7b_width_matches_reference(golden, cuda, T):
    from evspark_b200.config import DRAFTERS, EVO2_7B, EVO2_7B_SLICE
    from evspark_b200.drafter import DeviceDrafter
    from evspark_b200.model import TargetModel
    from evspark_b200.weights import init_drafter_weights, init_target_tensor

    d = golden("drafter_7b.npz")
    dcfg = DRAFTERS["evo2_7b"]
    dw = init_drafter_weights(dcfg, seed=20260830, embed=init_target_tensor(EVO2_7B, "embed", seed=20260820))
    dr = DeviceDrafter(dcfg, dw, device=cuda)
    # a 7B-width target state whose capture ring carries the context rows
    model = TargetModel.random(EVO2_7B_SLICE, seed=3, device=cuda, init_on="cuda", capture_layers=(2,))
    ip = model.initialize_inference_params(256)
    if T:
        ip.prefill(torch.full((1, T), 65, dtype=torch.long))
        ptr, ring_len = ip.capture_ring(0)

        class _Ring:  # the ring [max_batch, ring_len, d] as a CUDA array view
            __cuda_array_interface__ = {"shape": (ip.max_batch, ring_len, 4096), "typestr": "<f4",
                                        "data": (int(ptr), False), "version": 3, "strides": None}

        view = torch.as_tensor(_Ring(), device=cuda)
        # the context rows are the injection-layer outputs at positions len-T .. len-1 (= 0 .. T-1)
        view[0, torch.arange(T, device=cuda) % ring_len] = torch.as_tensor(d[f"ctx{T}/h_raw"], device=cuda)
    anchor = torch.tensor([67], device=cuda)
    toks, q, conf, U = dr.propose(ip, anchor, dcfg.gamma, True, want_U=True)
    err = (U[0].cpu() - torch.as_tensor(d[f"ctx{T}/U"])).abs().max().item()
    print(f"[drafter 7B] ctx={T} U max-abs {err:.2e}")
    np.testing.assert_allclose(U[0].cpu().numpy(), d[f"ctx{T}/U"], atol=2e-5, rtol=1e-4)
    np.testing.assert_array_equal(toks[0].cpu().numpy(), d[f"ctx{T}/greedy_tokens"])
    np.testing.assert_allclose(q[0].cpu().numpy(), d[f"ctx{T}/greedy_q"], atol=1e-6)
    np.testing.assert_allclose(conf[0].double().cpu().numpy(), d[f"ctx{T}/greedy_conf"], atol=1e-5)
    u = torch.as_tensor(np.random.default_rng(11).random(dcfg.gamma), device=cuda)[None]
    toks, q, conf, _ = dr.propose(ip, anchor, dcfg.gamma, False, temperature=1.0, top_k=4, uniforms=u)
    np.testing.assert_array_equal(toks[0].cpu().numpy(), d[f"ctx{T}/sample_tokens"])
    np.testing.assert_allclose(q[0].cpu().numpy(), d[f"ctx{T}/sample_q"], atol=1e-6)
    ip.close()
    dr.close()
    model.close()
