"""GPU: speculative loop, native references and the device drafter against the reference.

* The loop with the identity drafter reproduces, token for token, the reference's own
  ``speculative_generate`` outputs on the same model and seeds (golden fixtures), in greedy and
  in seeded-sampling mode, with the same per-round accepted lengths.
* Greedy speculative decoding equals native decoding exactly (fp32 tiny and bf16 7B-width).
* The device drafter (trunk + serial Markov head + confidence) matches the reference ``Drafter``.
"""

from __future__ import annotations

import ctypes
import glob
import os

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


@pytest.fixture(scope="module")
def tiny(cuda):
    from evspark_b200.config import TINY
    from evspark_b200.model import TargetModel
    from evspark_b200.weights import init_target_weights

    w = init_target_weights(TINY, seed=20260820)
    return TargetModel(TINY, w, device=cuda, capture_layers=(2,)), w


def _cudart():
    import torch as _t

    roots = [os.path.dirname(_t.__file__)] + [p for p in __import__("sys").path if "site-packages" in p]
    for r in roots:
        hits = glob.glob(os.path.join(r, "**", "libcudart.so*"), recursive=True)
        if hits:
            lib = ctypes.CDLL(sorted(hits)[0])
            lib.cudaMemcpy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]
            return lib
    pytest.skip("libcudart not found for raw device copies")


def test_tiny_loop_identity_matches_reference_golden(golden, tiny):
    from evspark_b200.specdec.block.loop import native_greedy_reference, speculative_generate
    from oracle.loop import IdentityDraft

    model, _ = tiny
    g = golden("tiny_model.npz")
    prompt = torch.tensor(g["loop/prompt"])[None]
    n = len(g["loop/native_greedy"])
    nat, ip, _ = native_greedy_reference(model, prompt, n)
    np.testing.assert_array_equal(nat, g["loop/native_greedy"])
    for gamma in (4, 12):
        spec = speculative_generate(model, IdentityDraft(), prompt, n, gamma, greedy=True, rng=np.random.default_rng(0))
        np.testing.assert_array_equal(spec.emitted_ids, g[f"loop/spec_greedy_g{gamma}"])
        assert [r.k for r in spec.rounds_log] == g[f"loop/spec_greedy_g{gamma}_ks"].tolist()
        rng = np.random.default_rng(7)
        spec = speculative_generate(model, IdentityDraft(), prompt, n, gamma, greedy=False, rng=rng,
                                    temperature=1.0, top_k=4)
        np.testing.assert_array_equal(spec.emitted_ids, g[f"loop/spec_sample_g{gamma}"])
        assert [r.k for r in spec.rounds_log] == g[f"loop/spec_sample_g{gamma}_ks"].tolist()


def test_tiny_loop_end_state_equals_teacher_forced(golden, tiny):
    from evspark_b200.specdec.block import diff_states, snapshot_states
    from evspark_b200.specdec.block.loop import spec_end_kv_len, speculative_generate, teacher_force_to_spec_state
    from oracle.loop import IdentityDraft

    model, _ = tiny
    g = golden("tiny_model.npz")
    prompt = torch.tensor(g["loop/prompt"])[None]
    for rollback in ("slice", "snapshot"):
        spec = speculative_generate(model, IdentityDraft(), prompt, 40, 8, greedy=True, rng=np.random.default_rng(0),
                                    rollback=rollback)
        assert any(r.k < 8 for r in spec.rounds_log)
        kv = spec_end_kv_len(prompt.shape[1], 40)
        assert spec.inference_params_dict.offset == kv
        ref = teacher_force_to_spec_state(model, prompt, spec.emitted_ids)
        d = diff_states(snapshot_states(spec.inference_params_dict, kv_len=kv), snapshot_states(ref, kv_len=kv))
        assert max(v["max_abs"] for v in d.values()) == 0.0


def test_truncation_round(golden, tiny):
    from evspark_b200.specdec.block.loop import native_greedy_reference, speculative_generate

    model, _ = tiny
    g = golden("tiny_model.npz")
    prompt = torch.tensor(g["loop/prompt"])[None]
    nat, _, _ = native_greedy_reference(model, prompt, 10)

    class Oracle:
        def probs(self, prefix):
            out = np.zeros(512)
            i = len(prefix) - prompt.shape[1]
            out[int(nat[i]) if 0 <= i < len(nat) else 65] = 1.0
            return out

    spec = speculative_generate(model, Oracle(), prompt, 10, 8, greedy=True, rng=np.random.default_rng(0))
    np.testing.assert_array_equal(spec.emitted_ids, nat)
    assert any(r.n_emitted < r.k + 1 for r in spec.rounds_log)
    assert spec.inference_params_dict.offset == prompt.shape[1] + 10 - 1


@pytest.mark.parametrize("T", [0, 9, 64])
def test_device_drafter_matches_reference_drafter(golden, tiny, T):
    from evspark_b200.config import DRAFTERS
    from evspark_b200.drafter import DeviceDrafter
    from evspark_b200.weights import init_drafter_weights

    model, w = tiny
    d = golden("drafter_tiny.npz")
    dcfg = DRAFTERS["tiny"]
    dw = init_drafter_weights(dcfg, seed=20260830, embed=w["embed"])
    dr = DeviceDrafter(dcfg, dw, device=model.device)
    ip = model.initialize_inference_params(256)
    if T:
        ip.prefill(torch.full((1, T), 65, dtype=torch.long))
        ring, ring_len = ip.capture_ring(0)
        h_raw = np.ascontiguousarray(d[f"ctx{T}/h_raw"].astype(np.float32))
        rt = _cudart()
        H = model.cfg.d_model
        torch.cuda.synchronize()
        for j in range(T):  # context rows live at positions len-T .. len-1
            dst = ring + (j % ring_len) * H * 4
            assert rt.cudaMemcpy(dst, h_raw[j].ctypes.data, H * 4, 1) == 0
    anchor = torch.tensor([71], device=model.device)
    toks, q, conf, U = dr.propose(ip, anchor, dcfg.gamma, True, want_U=True)
    np.testing.assert_allclose(U[0].cpu().numpy(), d[f"ctx{T}/U"], atol=2e-5, rtol=1e-4)
    np.testing.assert_array_equal(toks[0].cpu().numpy(), d[f"ctx{T}/greedy_tokens"])
    np.testing.assert_allclose(q[0].cpu().numpy(), d[f"ctx{T}/greedy_q"], atol=1e-6)
    np.testing.assert_allclose(conf[0].double().cpu().numpy(), d[f"ctx{T}/greedy_conf"], atol=1e-5)
    u = torch.as_tensor(np.random.default_rng(11).random(dcfg.gamma), device=model.device)[None]
    toks, q, conf, _ = dr.propose(ip, anchor, dcfg.gamma, False, temperature=1.0, top_k=4, uniforms=u)
    np.testing.assert_array_equal(toks[0].cpu().numpy(), d[f"ctx{T}/sample_tokens"])
    np.testing.assert_allclose(q[0].cpu().numpy(), d[f"ctx{T}/sample_q"], atol=1e-6)
    # decode γ' < training γ is an exact prefix computation
    toks5, _, _, U5 = dr.propose(ip, anchor, 5, True, want_U=True)
    np.testing.assert_allclose(U5[0].cpu().numpy(), d[f"ctx{T}/U_g5"], atol=2e-5, rtol=1e-4)
    with pytest.raises(ValueError, match="γ"):
        dr.propose(ip, anchor, dcfg.gamma + 1, True)
    ip.close()
    dr.close()


def test_neural_loop_greedy_equals_native(tiny):
    from evspark_b200.config import DRAFTERS
    from evspark_b200.drafter import DeviceDrafter
    from evspark_b200.specdec.block.loop import native_greedy_reference, speculative_generate
    from evspark_b200.specdec.block.neural_draft import NeuralDraftModel

    model, w = tiny
    dr = DeviceDrafter.random(DRAFTERS["tiny"], embed=w["embed"], device=model.device)
    nd = NeuralDraftModel(model, dr, ("blocks.2",))
    prompt = torch.tensor(np.random.default_rng(5).choice([65, 67, 71, 84], size=200))[None]
    spec = speculative_generate(model, nd, prompt, 64, 12, greedy=True, rng=np.random.default_rng(0))
    nat, _, _ = native_greedy_reference(model, prompt, 64)
    np.testing.assert_array_equal(spec.emitted_ids, nat)
    assert all(r.conf is not None and len(r.conf) == 12 for r in spec.rounds_log)
    assert nd.capture_buffer_len() == spec.inference_params_dict.offset
    nd.capture_reset()
    spec = speculative_generate(model, nd, prompt, 64, 12, greedy=False, rng=np.random.default_rng(3))
    assert spec.emitted_ids.shape == (64,)
    with pytest.raises(ValueError, match="slice"):
        speculative_generate(model, nd, prompt, 4, 12, greedy=True, rng=np.random.default_rng(0),
                             rollback="snapshot")
    nd.close()


def test_7b_width_bf16_greedy_spec_equals_native(cuda):
    from evspark_b200.config import EVO2_7B_SLICE
    from evspark_b200.model import TargetModel
    from evspark_b200.specdec.block.loop import native_greedy_reference, speculative_generate
    from oracle.loop import IdentityDraft

    model = TargetModel.random(EVO2_7B_SLICE, seed=11, device=cuda, init_on="cuda")
    prompt = torch.tensor(np.random.default_rng(9).choice([65, 67, 71, 84], size=96))[None]
    nat, _, _ = native_greedy_reference(model, prompt, 48)
    spec = speculative_generate(model, IdentityDraft(), prompt, 48, 12, greedy=True, rng=np.random.default_rng(0))
    np.testing.assert_array_equal(spec.emitted_ids, nat)
    model.close()


def test_single_sync_round_equals_general_round(tiny):
    """The device round (pinned uniform buffers, rollback index taken from the device verification,
    one host synchronisation) emits the same tokens and leaves the same state as the general round."""
    from evspark_b200.config import DRAFTERS
    from evspark_b200.drafter import DeviceDrafter
    from evspark_b200.specdec.block.loop import speculative_generate
    from evspark_b200.specdec.block.neural_draft import NeuralDraftModel

    model, w = tiny
    dr = DeviceDrafter.random(DRAFTERS["tiny"], embed=w["embed"], device=model.device)
    nd = NeuralDraftModel(model, dr, ("blocks.2",))
    prompt = torch.tensor(np.random.default_rng(31).choice([65, 67, 71, 84], size=120))[None]
    for greedy, seed in ((True, 0), (False, 5), (False, 6)):
        outs = []
        for timing in (True, False):
            nd.capture_reset()
            spec = speculative_generate(model, nd, prompt, 37, 12, greedy=greedy, rng=np.random.default_rng(seed),
                                        timing=timing)
            ip = spec.inference_params_dict
            outs.append((spec.emitted_ids, [r.k for r in spec.rounds_log], ip.offset, ip.export(0, 0), ip.export(2, 2)))
            ip.close()
        (e1, k1, o1, f1, s1), (e2, k2, o2, f2, s2) = outs
        np.testing.assert_array_equal(e1, e2)
        assert k1 == k2 and o1 == o2
        assert torch.equal(f1, f2) and torch.equal(s1, s2)
    nd.close()


def test_evspark_generate_reuses_its_decode_state(tiny):
    """EvSpark keeps one decode state across generate calls: it resets it to length 0 and
    allocates a larger one when a call needs more positions.  Every call emits exactly the tokens
    that speculative_generate emits with a fresh state of its own, when sampling and greedy."""
    from evspark_b200.api import EvSpark, ids_to_text
    from evspark_b200.config import DRAFTERS
    from evspark_b200.drafter import DeviceDrafter
    from evspark_b200.specdec.block.loop import speculative_generate
    from evspark_b200.specdec.block.neural_draft import NeuralDraftModel

    model, w = tiny
    dr = DeviceDrafter.random(DRAFTERS["tiny"], embed=w["embed"], device=model.device)
    nd = NeuralDraftModel(model, dr, ("blocks.2",))
    es = EvSpark(model, nd, str(model.device), state_seqlen=300)
    rng = np.random.default_rng(7)
    p1 = ids_to_text(rng.choice([65, 67, 71, 84], size=200))
    p2 = ids_to_text(rng.choice([65, 67, 71, 84], size=260))  # 260 + 48 + 14 > 300: a larger state
    state0 = es._state
    for prompt, n, greedy, seed in ((p1, 48, False, 5), (p1, 48, False, 5), (p1, 40, True, 0), (p2, 48, False, 9)):
        got = es.generate(prompt, n_tokens=n, greedy=greedy, seed=seed)
        nd.capture_reset()
        ids = torch.as_tensor(np.frombuffer(prompt.encode("ascii"), dtype=np.uint8).astype(np.int64))[None]
        ref = speculative_generate(model, nd, ids, n, 12, greedy=greedy, rng=np.random.default_rng(seed),
                                   temperature=1.0, top_k=4)
        ref.inference_params_dict.close()
        np.testing.assert_array_equal(got.ids, ref.emitted_ids)
    assert es._state is not state0 and es._state.max_seqlen >= 260 + 48 + 14
    es._state.close()  # not es.close(): the model belongs to the module fixture
    es._state = None
    nd.close()


def test_drafter_context_cache_equals_a_fresh_drafter(tiny):
    """The drafter projects each context position once and keeps its k/v rows for later calls
    (valid while the capture ring row it came from is unchanged).  Every proposal of a speculative
    run, with rollbacks that rewrite positions, and of a second run on a reset state, equals the
    proposal of a freshly built drafter (no cached rows) on the same state, bit for bit."""
    from evspark_b200.config import DRAFTERS
    from evspark_b200.drafter import DeviceDrafter
    from evspark_b200.specdec.block.loop import speculative_generate
    from evspark_b200.specdec.block.neural_draft import NeuralDraftModel
    from evspark_b200.weights import init_drafter_weights

    model, w = tiny
    dcfg = DRAFTERS["tiny"]
    dw = init_drafter_weights(dcfg, seed=20260830, embed=w["embed"])

    class CheckedDraft(NeuralDraftModel):
        checked = 0

        def propose_device(self, anchor, gamma, greedy, rng, *, temperature=1.0, top_k=4,
                           inference_params_dict=None):
            ip = inference_params_dict
            u = None if greedy else torch.as_tensor(rng.random(int(gamma)), device=model.device)[None]
            got = self.drafter.propose(ip, anchor.reshape(1), int(gamma), greedy, temperature=temperature,
                                       top_k=top_k, uniforms=u)
            fresh = DeviceDrafter(dcfg, dw, device=model.device)
            ref = fresh.propose(ip, anchor.reshape(1), int(gamma), greedy, temperature=temperature, top_k=top_k,
                                uniforms=u)
            torch.cuda.synchronize()
            fresh.close()
            for a, b in zip(got[:3], ref[:3]):
                assert torch.equal(a, b)
            CheckedDraft.checked += 1
            return got[0], got[1], got[2]

    nd = CheckedDraft(model, DeviceDrafter(dcfg, dw, device=model.device), ("blocks.2",))
    rng = np.random.default_rng(41)
    for L, greedy, seed in ((150, False, 3), (90, True, 0), (200, False, 8)):
        prompt = torch.tensor(rng.choice([65, 67, 71, 84], size=L))[None]
        nd.capture_reset()
        spec = speculative_generate(model, nd, prompt, 30, 12, greedy=greedy, rng=np.random.default_rng(seed))
        assert any(r.k < 12 for r in spec.rounds_log)
        spec.inference_params_dict.close()
    assert CheckedDraft.checked >= 30
    nd.close()
