"""CPU: the oracle reproduces the reference's own outputs (golden fixtures).

The fixtures were produced by the reference implementation itself
(tests/golden/make_golden.py): block_forward / slice_states_to_accept /
speculative_generate on the tiny config, the verifier and sampling transform,
and the drafter trunk + serial head.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from evspark_b200.config import DRAFTERS, TINY
from evspark_b200.weights import init_drafter_weights, init_target_weights
from oracle import loop as oloop
from oracle import specdec as sd
from oracle.model import OracleTarget

# fp64 oracle vs the reference's fp32 chunk path (FFT-based IIR, fp32 FIR): fp32 noise
TOL_LOGITS = 2e-5
TOL_STATE = 2e-5


@pytest.fixture(scope="module")
def tiny_weights():
    return init_target_weights(TINY, seed=20260820)


@pytest.fixture(scope="module")
def oracle64(tiny_weights):
    return OracleTarget(TINY, tiny_weights)


def test_weights_are_the_fixture_weights(golden, tiny_weights):
    from tests.golden.make_golden import weights_digest

    assert str(golden("tiny_model.npz")["weights_sha256"]) == weights_digest(tiny_weights)


def _states_of(st, layer_types):
    out = {}
    for i, kind in enumerate(layer_types):
        if kind == "mha":
            continue
        out[f"fir_state_dict/{i}"] = st.outer[i][0:].numpy()
        if kind in ("hcs", "hcm"):
            out[f"fir_inner_state_dict/{i}"] = st.inner[i].numpy()
        else:
            out[f"state_dict/{i}"] = st.iir[i].numpy()
    return out


def _check_states(g, prefix, st):
    ours = _states_of(st, TINY.layer_types)
    keys = [k[len(prefix) + 1:] for k in g if k.startswith(prefix + "/") and not k.endswith("offset")]
    assert sorted(keys) == sorted(ours), (sorted(keys), sorted(ours))
    for k in keys:
        ref = g[f"{prefix}/{k}"]
        assert ref.shape == ours[k].shape, (k, ref.shape, ours[k].shape)
        np.testing.assert_allclose(ours[k], ref, atol=TOL_STATE * max(1.0, np.abs(ref).max()), rtol=0, err_msg=k)
    assert int(g[f"{prefix}/offset"]) == int(st.lengths.max())


@pytest.mark.parametrize("case", ["full", "short"])
def test_oracle_block_and_slices_match_reference(golden, oracle64, case):
    g = golden("tiny_model.npz")
    prompt, chunk = g[f"{case}/prompt"], g[f"{case}/chunk"]
    st = oracle64.init_state(1, len(prompt) + 64)
    pre, _, _ = oracle64.forward(prompt[None, :-1], st, prefill=True)
    np.testing.assert_allclose(pre[0, -1].numpy(), g[f"{case}/prefill_last_logits"], atol=TOL_LOGITS * 30, rtol=0)
    _check_states(g, f"{case}/after_prefill", st)
    st_step = st.clone()
    step = oracle64.step_reference(chunk[None], st_step)
    logits, stash, _ = oracle64.forward(chunk[None], st, retain=True)
    scale = np.abs(g[f"{case}/block_logits"]).max()
    np.testing.assert_allclose(logits[0].numpy(), g[f"{case}/block_logits"], atol=TOL_LOGITS * scale, rtol=0)
    np.testing.assert_allclose(step[0].numpy(), g[f"{case}/step_logits"], atol=TOL_LOGITS * scale, rtol=0)
    ks = sorted(int(k.split("slice_k")[1].split("/")[0]) for k in g
                if k.startswith(f"{case}/slice_k") and k.endswith("offset"))
    assert ks
    for k in ks:
        stk = st.clone()
        oracle64.slice(stk, stash, k)
        _check_states(g, f"{case}/slice_k{k}", stk)


def test_oracle_ragged_slice_matches_reference(golden, oracle64):
    g = golden("tiny_model.npz")
    prompt, chunks, ks = g["ragged/prompt"], g["ragged/chunks"], g["ragged/ks"]
    st = oracle64.init_state(1, len(prompt) + 64)
    oracle64.forward(prompt[None, :-1], st, prefill=True)
    st2 = oracle64.init_state(2, len(prompt) + 64)
    for name in ("outer", "inner", "iir", "kv"):
        for i, t in getattr(st, name).items():
            getattr(st2, name)[i] = t.expand(2, *t.shape[1:]).clone()
    st2.lengths = np.repeat(st.lengths, 2)
    logits, stash, _ = oracle64.forward(chunks, st2, retain=True)
    np.testing.assert_allclose(logits.numpy(), g["ragged/block_logits"], atol=TOL_LOGITS * 30, rtol=0)
    oracle64.slice(st2, stash, ks)
    _check_states(g, "ragged/slice", st2)


def test_oracle_ragged_slice_refuses_unflipped_width_mismatch(oracle64):
    rng = np.random.default_rng(5)
    st = oracle64.init_state(2, 64)
    oracle64.forward(rng.choice([65, 67, 71, 84], size=(2, 3)), st, prefill=True)
    _, stash, _ = oracle64.forward(rng.choice([65, 67, 71, 84], size=(2, 5)), st, retain=True)
    with pytest.raises(ValueError, match="FIR state widths"):
        oracle64.slice(st, stash, np.array([0, 2]))


def test_oracle_loop_matches_reference_loop(golden, oracle64):
    g = golden("tiny_model.npz")
    prompt = g["loop/prompt"]
    n = len(g["loop/native_greedy"])
    nat, _ = oloop.native_greedy(oracle64, prompt, n)
    np.testing.assert_array_equal(nat, g["loop/native_greedy"])
    for gamma in (4, 12):
        ids, ks, _ = oloop.speculative_generate(oracle64, oloop.IdentityDraft(), prompt, n, gamma, True,
                                                np.random.default_rng(0))
        np.testing.assert_array_equal(ids, g[f"loop/spec_greedy_g{gamma}"])
        assert ks == g[f"loop/spec_greedy_g{gamma}_ks"].tolist()
        ids, ks, _ = oloop.speculative_generate(oracle64, oloop.IdentityDraft(), prompt, n, gamma, False,
                                                np.random.default_rng(7))
        np.testing.assert_array_equal(ids, g[f"loop/spec_sample_g{gamma}"])
        assert ks == g[f"loop/spec_sample_g{gamma}_ks"].tolist()


def test_transform_and_qprime_kat(golden):
    k = golden("verify_kat.npz")
    for key in [x for x in k if x.startswith("transform/T")]:
        T, topk = key.split("/")[1][1:].split("_k")
        got = np.stack([sd.apply_transform(r, float(T), int(topk)) for r in k["transform/logits"]])
        np.testing.assert_allclose(got, k[key], atol=1e-15, rtol=1e-12, err_msg=key)
    got = np.stack([sd.q_prime_from_raw(r, 1.0, 4) for r in k["qprime/raw"]])
    np.testing.assert_allclose(got, k["qprime/out"], atol=1e-15, rtol=1e-12)


def test_verify_kat(golden):
    k = golden("verify_kat.npz")
    for c, seed in enumerate(k["verify/seeds"]):
        vr = sd.verify_round(k["verify/tokens"][c], k["verify/q"][c].astype(np.float64),
                             k["verify/p"][c].astype(np.float64), np.random.default_rng(int(seed)))
        want = k["verify/result"][c]
        got = [vr.accepted_len, int(vr.from_residual), int(vr.fallback)] + vr.tokens.tolist()
        assert got == [int(v) for v in want[: len(got)]], (c, got, want)
    vg = sd.verify_round_greedy(k["greedy/x"], k["greedy/p"])
    assert [vg.accepted_len] + vg.tokens.tolist() == k["greedy/result"].tolist()
    vmg = sd.verify_round_greedy_multicand(k["mc_greedy/x"], np.stack([k["greedy/p"]] * 2))
    assert [vmg.accepted_len, vmg.winner] + vmg.tokens.tolist() == k["mc_greedy/result"].tolist()
    vm = sd.verify_round_multicand(k["mc/x"], k["mc/q"], k["mc/p"], np.random.default_rng(4242))
    assert [vm.accepted_len, vm.winner, int(vm.fallback)] + vm.tokens.tolist() == k["mc/result"].tolist()


def test_sampling_contract_one_uniform_inverse_cdf(golden):
    k = golden("verify_kat.npz")
    for s in k["choice/seeds"]:
        s = int(s)
        p = sd.as_prob_row(k["verify/p"][s % 200][s % 13].astype(np.float64))
        rng = np.random.default_rng(s)
        assert sd.inverse_cdf(p, float(rng.random())) == int(k["choice/draws"][s])


@pytest.mark.parametrize("T", [0, 9, 64])
def test_oracle_drafter_matches_reference(golden, tiny_weights, T):
    d = golden("drafter_tiny.npz")
    dcfg = DRAFTERS["tiny"]
    dw = init_drafter_weights(dcfg, seed=20260830, embed=tiny_weights["embed"])
    from tests.golden.make_golden import weights_digest

    assert str(d["drafter_sha256"]) == weights_digest(dw)
    h_raw = torch.from_numpy(d[f"ctx{T}/h_raw"])
    with torch.no_grad():
        U, h = sd.drafter_trunk(dw, dcfg, 71, h_raw if T else None, T)
        Ug, _ = sd.drafter_trunk(dw, dcfg, 71, h_raw if T else None, T, gamma=5)
    np.testing.assert_allclose(U.numpy(), d[f"ctx{T}/U"], atol=2e-5, rtol=1e-4)
    np.testing.assert_allclose(h.numpy(), d[f"ctx{T}/h"], atol=2e-5, rtol=1e-4)
    np.testing.assert_allclose(Ug.numpy(), d[f"ctx{T}/U_g5"], atol=2e-5, rtol=1e-4)
    U_ref, h_ref = torch.from_numpy(d[f"ctx{T}/U"]), torch.from_numpy(d[f"ctx{T}/h"])
    tg, qg, cg = sd.drafter_serial(dw, U_ref, h_ref, 71, True, np.random.default_rng(0))
    np.testing.assert_array_equal(tg, d[f"ctx{T}/greedy_tokens"])
    np.testing.assert_allclose(qg, d[f"ctx{T}/greedy_q"], atol=1e-7)
    np.testing.assert_allclose(cg, d[f"ctx{T}/greedy_conf"], atol=1e-6)
    ts, qs, cs = sd.drafter_serial(dw, U_ref, h_ref, 71, False, np.random.default_rng(11))
    np.testing.assert_array_equal(ts, d[f"ctx{T}/sample_tokens"])
    np.testing.assert_allclose(qs, d[f"ctx{T}/sample_q"], atol=1e-7)


@pytest.mark.parametrize("T", [0, 64])
def test_oracle_drafter_7b_width_matches_reference(golden, T):
    """The drafter at Evo2-7B width (d=1024, 16 heads, 4096-wide context rows from block 27) against
    the reference ``Drafter`` / ``trunk_forward`` / ``serial_sample`` (evspark/train/drafter.py:54-409,
    evspark/specdec/block/neural_draft.py:157-259)."""
    from evspark_b200.config import EVO2_7B
    from evspark_b200.weights import init_target_tensor
    from tests.golden.make_golden import weights_digest

    d = golden("drafter_7b.npz")
    dcfg = DRAFTERS["evo2_7b"]
    dw = init_drafter_weights(dcfg, seed=20260830, embed=init_target_tensor(EVO2_7B, "embed", seed=20260820))
    assert str(d["drafter_sha256"]) == weights_digest(dw)
    h_raw = torch.from_numpy(d[f"ctx{T}/h_raw"])
    with torch.no_grad():
        U, h = sd.drafter_trunk(dw, dcfg, 67, h_raw if T else None, T)
    np.testing.assert_allclose(U.numpy(), d[f"ctx{T}/U"], atol=2e-5, rtol=1e-4)
    np.testing.assert_allclose(h.numpy(), d[f"ctx{T}/h"], atol=2e-5, rtol=1e-4)
    U_ref, h_ref = torch.from_numpy(d[f"ctx{T}/U"]), torch.from_numpy(d[f"ctx{T}/h"])
    tg, qg, cg = sd.drafter_serial(dw, U_ref, h_ref, 67, True, np.random.default_rng(0))
    np.testing.assert_array_equal(tg, d[f"ctx{T}/greedy_tokens"])
    np.testing.assert_allclose(qg, d[f"ctx{T}/greedy_q"], atol=1e-7)
    np.testing.assert_allclose(cg, d[f"ctx{T}/greedy_conf"], atol=1e-6)
    ts, qs, cs = sd.drafter_serial(dw, U_ref, h_ref, 67, False, np.random.default_rng(11))
    np.testing.assert_array_equal(ts, d[f"ctx{T}/sample_tokens"])
    np.testing.assert_allclose(qs, d[f"ctx{T}/sample_q"], atol=1e-7)
