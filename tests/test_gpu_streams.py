"""GPU: multi-stream speculative decoding (B streams per GPU in lockstep batched rounds).

A stream decoded inside a batch must emit exactly the tokens of the same stream decoded alone:
greedy streams equal native greedy decoding of their own prompt, and seeded sampling streams
equal the single-stream speculative loop with the same generator seed.  The bf16 7B-width case
runs the batched projections on the 64- and 128-token MMA tiles.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ACGT = [65, 67, 71, 84]


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from evspark_b200 import _native as N

    N.call("evs_device_check")
    return torch.device("cuda:0")


def _prompts(B, L, seed):
    return np.stack([np.random.default_rng(seed + b).choice(ACGT, size=L) for b in range(B)]).astype(np.int64)


def test_tiny_streams_equal_single_stream_runs(cuda):
    from evspark_b200.config import DRAFTERS, TINY
    from evspark_b200.drafter import DeviceDrafter
    from evspark_b200.model import TargetModel
    from evspark_b200.specdec.block.loop import native_greedy_reference, speculative_generate
    from evspark_b200.specdec.block.neural_draft import NeuralDraftModel
    from evspark_b200.specdec.block.streams import speculative_generate_streams
    from evspark_b200.weights import init_target_weights

    w = init_target_weights(TINY, seed=20260820)
    model = TargetModel(TINY, w, device=cuda, capture_layers=(2,))
    dr = DeviceDrafter.random(DRAFTERS["tiny"], embed=w["embed"], device=cuda, max_batch=3)
    nd = NeuralDraftModel(model, dr, ("blocks.2",))
    B, n = 3, 40
    prompts = _prompts(B, 120, 100)

    res = speculative_generate_streams(model, nd, prompts, n, 12, True, [np.random.default_rng(0)] * B)
    for b in range(B):
        nat, ipn, _ = native_greedy_reference(model, torch.as_tensor(prompts[b])[None], n)
        ipn.close()
        np.testing.assert_array_equal(res.emitted[b], nat, err_msg=f"greedy stream {b}")
    res.inference_params_dict.close()

    nd.capture_reset()
    seeds = [7, 8, 9]
    res = speculative_generate_streams(model, nd, prompts, n, 12, False, [np.random.default_rng(s) for s in seeds])
    assert res.rounds >= int(res.active_rounds.max())
    for b in range(B):
        nd.capture_reset()
        one = speculative_generate(model, nd, torch.as_tensor(prompts[b])[None], n, 12, greedy=False,
                                   rng=np.random.default_rng(seeds[b]))
        np.testing.assert_array_equal(res.emitted[b], one.emitted_ids, err_msg=f"sampled stream {b}")
        one.inference_params_dict.close()
    res.inference_params_dict.close()
    nd.close()
    model.close()


def test_7b_width_bf16_streams_greedy_equal_native(cuda):
    from evspark_b200.config import DRAFTERS, EVO2_7B_SLICE
    from evspark_b200.drafter import DeviceDrafter, layer_index
    from evspark_b200.model import TargetModel
    from evspark_b200.specdec.block.loop import native_greedy_reference
    from evspark_b200.specdec.block.neural_draft import NeuralDraftModel
    from evspark_b200.specdec.block.streams import speculative_generate_streams

    dcfg = DRAFTERS["evo2_7b_slice"]
    model = TargetModel.random(EVO2_7B_SLICE, seed=11, device=cuda, init_on="cuda",
                               capture_layers=tuple(layer_index(x) for x in dcfg.inject_layers))
    dr = DeviceDrafter.random(dcfg, embed=model.weights["embed"], device=cuda, max_batch=6, init_on="cuda")
    nd = NeuralDraftModel(model, dr, dcfg.inject_layers)
    B, n = 6, 24  # M = 78 token rows per verify forward: 128-token tiles; prefill chunks M = 192
    prompts = _prompts(B, 80, 300)
    res = speculative_generate_streams(model, nd, prompts, n, 12, True, [np.random.default_rng(0)] * B)
    for b in range(B):
        nat, ipn, _ = native_greedy_reference(model, torch.as_tensor(prompts[b])[None], n)
        ipn.close()
        np.testing.assert_array_equal(res.emitted[b], nat, err_msg=f"stream {b}")
    res.inference_params_dict.close()
    nd.close()
    model.close()
