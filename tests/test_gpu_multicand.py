"""GPU: SpecInfer multi-candidate verification (``n_candidates > 1``).

* ``evs_verify_multicand`` equals the restated ``verify_round_multicand`` /
  ``verify_round_greedy_multicand`` (evspark/specdec/verifier.py:212-319) on seeded cases: same
  tokens, accepted length, winner, residual/fallback flags and number of uniforms consumed.
* Greedy speculative decoding with 3 candidates per round (neural drafter: top-3 first tokens)
  equals native greedy decoding; sampled multi-candidate decoding runs and keeps its state
  consistent with the emitted tokens.
"""

from __future__ import annotations

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


class _Counting:
    def __init__(self, seed):
        self.rng = np.random.default_rng(seed)
        self.n = 0

    def random(self, *a):
        self.n += 1
        return self.rng.random(*a)


def _case(seed, B, g, V=512):
    rng = np.random.default_rng(seed)
    logits = rng.normal(size=(B, g + 1, V)) * 3.0
    p = np.exp(logits - logits.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    ql = logits[:, :g] + rng.normal(size=(B, g, V)) * 1.5
    q = np.exp(ql - ql.max(-1, keepdims=True))
    q /= q.sum(-1, keepdims=True)
    x = np.empty((B, g), dtype=np.int64)
    for b in range(B):
        for i in range(g):
            x[b, i] = rng.choice(V, p=q[b, i])
        if b > 0 and rng.random() < 0.6:  # candidates that share a prefix with candidate 0
            cut = int(rng.integers(1, g))
            x[b, :cut] = x[0, :cut]
    return p, q, x


@pytest.mark.parametrize("seed,B", [(1, 2), (2, 3), (3, 4), (4, 2), (5, 3), (6, 4), (7, 2), (8, 3)])
def test_multicand_verify_matches_oracle(cuda, seed, B):
    from evspark_b200.specdec.verifier import verify_device_multicand
    from oracle.specdec import verify_round_greedy_multicand, verify_round_multicand

    g = 12
    p, q, x = _case(seed, B, g)
    cnt = _Counting(100 + seed)
    ref = verify_round_multicand(x, q, p, cnt)
    u = np.random.default_rng(100 + seed).random(g * B + 1)
    t = lambda a: torch.as_tensor(a, device=cuda)
    toks, info = verify_device_multicand(t(p), t(q), t(x), t(u), greedy=False)
    info = info.cpu().numpy()
    k = int(info[0])
    assert k == ref.accepted_len
    np.testing.assert_array_equal(toks.cpu().numpy()[:k + 1], ref.tokens)
    assert (bool(info[1]), bool(info[2]), int(info[3]), int(info[4])) == (ref.from_residual, ref.fallback, cnt.n,
                                                                          ref.winner)
    gref = verify_round_greedy_multicand(x, np.log(p))
    gt, gi = verify_device_multicand(t(np.log(p)), None, t(x), None, greedy=True)
    gi = gi.cpu().numpy()
    assert int(gi[0]) == gref.accepted_len and int(gi[4]) == gref.winner
    np.testing.assert_array_equal(gt.cpu().numpy()[:int(gi[0]) + 1], gref.tokens)


def test_multicand_loop_greedy_equals_native(cuda):
    from evspark_b200.config import DRAFTERS, TINY
    from evspark_b200.drafter import DeviceDrafter
    from evspark_b200.model import TargetModel
    from evspark_b200.specdec.block.loop import native_greedy_reference, speculative_generate
    from evspark_b200.specdec.block.neural_draft import NeuralDraftModel
    from evspark_b200.weights import init_target_weights

    w = init_target_weights(TINY, seed=20260820)
    model = TargetModel(TINY, w, device=cuda, capture_layers=(2,))
    dr = DeviceDrafter.random(DRAFTERS["tiny"], embed=w["embed"], device=cuda, max_batch=3)
    nd = NeuralDraftModel(model, dr, ("blocks.2",))
    prompt = torch.tensor(np.random.default_rng(21).choice([65, 67, 71, 84], size=150))[None]
    spec = speculative_generate(model, nd, prompt, 48, 12, greedy=True, rng=np.random.default_rng(0), n_candidates=3)
    nat, ipn, _ = native_greedy_reference(model, prompt, 48)
    np.testing.assert_array_equal(spec.emitted_ids, nat)
    assert all(r.n_candidates == 3 for r in spec.rounds_log)
    ipn.close()
    spec.inference_params_dict.close()
    nd.capture_reset()
    spec = speculative_generate(model, nd, prompt, 40, 12, greedy=False, rng=np.random.default_rng(4),
                                n_candidates=3)
    assert spec.emitted_ids.shape == (40,)
    ip = spec.inference_params_dict
    assert ip.batch == 1 and ip.offset == 150 + 40 - 1
    spec.inference_params_dict.close()
    nd.close()
    model.close()
