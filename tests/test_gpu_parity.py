"""GPU parity of the CUDA path against the oracle and the reference's golden vectors.

Every test here calls libevspark_sm100 through its C ABI (ctypes) and compares with
* the golden fixtures produced by the reference implementation (tests/golden/*.npz),
* the CPU oracle (oracle/model.py) on the same seeded inputs.

Tolerances (north star): fp32 logits within 1e-5 max-abs of the fp64 oracle and of the
reference's own fp32 outputs; bf16 logits within 2e-2 max-abs of the bf16-emulating oracle, block
by block on the device's own residual stream (tests/_parity.py says why end-to-end bf16 runs
cannot be compared at that bound); state slices, accepted lengths, greedy tokens and acceptance
decisions exact.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL_FP32 = 1e-5  # max-abs logits, fp32 device vs the fp64 oracle / the reference's fp32 outputs


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


@pytest.fixture(scope="module")
def oracle_tiny(tiny):
    from oracle.model import OracleTarget
    from evspark_b200.config import TINY

    return OracleTarget(TINY, tiny[1])


# ---------------------------------------------------------------------------
# tcgen05 GEMM
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("N_,K,M", [(256, 1024, 1), (512, 512, 13), (384, 4096, 16), (256, 640, 40),
                                    (512, 1024, 200)])
def test_gemm_bf16_tcgen05_vs_torch(cuda, N_, K, M):
    from evspark_b200 import _native as N

    g = torch.Generator(device=cuda).manual_seed(N_ + K + M)
    W = torch.randn(N_, K, device=cuda, generator=g).to(torch.bfloat16)
    X = torch.randn(M, K, device=cuda, generator=g).to(torch.bfloat16)
    out = torch.empty(M, N_, device=cuda)
    N.call("evs_gemm_bf16", W.data_ptr(), X.data_ptr(), out.data_ptr(), N_, K, M, 1, N.stream_ptr())
    ref = X.float() @ W.float().T
    torch.cuda.synchronize()
    err = (out - ref).abs().max().item()
    assert err <= 2e-3 * ref.abs().max().item(), err
    # a token row's result does not depend on the other rows of the tile
    out1 = torch.empty(1, N_, device=cuda)
    N.call("evs_gemm_bf16", W.data_ptr(), X[M - 1:].contiguous().data_ptr(), out1.data_ptr(), N_, K, 1, 1,
           N.stream_ptr())
    assert torch.equal(out1[0], out[M - 1])


def test_gemm_token_tile_widths_agree_bitwise(cuda):
    """Batched streams use 64- and 128-token MMA tiles; a token row must come out bit-identical
    to the 16-token tile a single stream uses, so batching never changes a stream's logits."""
    from evspark_b200 import _native as N

    N_, K = 768, 2048
    g = torch.Generator(device=cuda).manual_seed(11)
    W = torch.randn(N_, K, device=cuda, generator=g).to(torch.bfloat16)
    X = torch.randn(300, K, device=cuda, generator=g).to(torch.bfloat16)
    outs = {}
    for M in (13, 60, 300):  # 16-, 64- and 128-token tiles
        out = torch.empty(M, N_, device=cuda)
        N.call("evs_gemm_bf16", W.data_ptr(), X[:M].contiguous().data_ptr(), out.data_ptr(), N_, K, M, 1,
               N.stream_ptr())
        outs[M] = out
    torch.cuda.synchronize()
    assert torch.equal(outs[13], outs[60][:13])
    assert torch.equal(outs[13], outs[300][:13])
    assert torch.equal(outs[60], outs[300][:60])


# ---------------------------------------------------------------------------
# tiny fp32 model vs golden + oracle
# ---------------------------------------------------------------------------

def _hyena_states(ip, cfg):
    out = {}
    for i, kind in enumerate(cfg.layer_types):
        if kind == "mha":
            continue
        out[f"fir_state_dict/{i}"] = ip.export(i, 0).cpu().numpy()
        if kind in ("hcs", "hcm"):
            out[f"fir_inner_state_dict/{i}"] = ip.export(i, 1).cpu().numpy()
        else:
            out[f"state_dict/{i}"] = ip.export(i, 2).cpu().numpy()
    return out


def _check_states(g, prefix, ip, cfg, tol=2e-5):
    ours = _hyena_states(ip, cfg)
    for k, v in ours.items():
        ref = g[f"{prefix}/{k}"]
        assert ref.shape == v.shape, (k, ref.shape, v.shape)
        np.testing.assert_allclose(v, ref, atol=tol * max(1.0, np.abs(ref).max()), rtol=0, err_msg=f"{prefix} {k}")
    assert int(g[f"{prefix}/offset"]) == ip.offset


@pytest.mark.parametrize("case", ["full", "short"])
def test_tiny_block_slice_vs_golden_and_oracle(golden, tiny, oracle_tiny, case):
    from evspark_b200.specdec.block import block_forward, clone_inference_params, prefill, slice_states_to_accept

    model, _ = tiny
    cfg = model.cfg
    g = golden("tiny_model.npz")
    prompt, chunk = g[f"{case}/prompt"], g[f"{case}/chunk"]
    ip = model.initialize_inference_params(len(prompt) + 64)
    pre = prefill(model, torch.tensor(prompt[:-1])[None], ip)
    np.testing.assert_allclose(pre[0, -1].cpu().numpy(), g[f"{case}/prefill_last_logits"], atol=TOL_FP32, rtol=0)
    _check_states(g, f"{case}/after_prefill", ip, cfg)
    # oracle (fp64) on the same inputs
    st = oracle_tiny.init_state(1, len(prompt) + 64)
    oracle_tiny.forward(prompt[None, :-1], st, prefill=True)
    ref_logits, _, _ = oracle_tiny.forward(chunk[None], st, retain=True)
    logits, stash = block_forward(model, torch.tensor(chunk)[None], ip, retain=True)
    got = logits[0].cpu().double()
    err = (got - ref_logits[0]).abs().max().item()
    print(f"[fp32 parity] {case}: max-abs {err:.3e} (max|logit| {ref_logits.abs().max().item():.2f})")
    assert err <= TOL_FP32, f"block logits vs fp64 oracle: {err:.3e}"
    np.testing.assert_allclose(got.numpy(), g[f"{case}/block_logits"], atol=TOL_FP32, rtol=0)
    ks = sorted(int(k.split("slice_k")[1].split("/")[0]) for k in g
                if k.startswith(f"{case}/slice_k") and k.endswith("offset"))
    for k in ks:
        ipk = clone_inference_params(ip)
        slice_states_to_accept(ipk, stash, k)
        _check_states(g, f"{case}/slice_k{k}", ipk, cfg)
        ipk.close()


def test_tiny_block_equals_step_bitwise(tiny, golden):
    """Row invariance: the γ+1 block forward and the native T=1 steps give identical bits."""
    from evspark_b200.specdec.block import block_forward, clone_inference_params, prefill, step_forward_reference

    model, _ = tiny
    g = golden("tiny_model.npz")
    prompt, chunk = g["full/prompt"], g["full/chunk"]
    ip = model.initialize_inference_params(len(prompt) + 64)
    prefill(model, torch.tensor(prompt[:-1])[None], ip)
    ip2 = clone_inference_params(ip)
    step = step_forward_reference(model, torch.tensor(chunk)[None], ip2)
    blk = block_forward(model, torch.tensor(chunk)[None], ip)
    assert torch.equal(step, blk), (step - blk).abs().max().item()
    for i, kind in enumerate(model.cfg.layer_types):
        if kind != "mha":
            assert torch.equal(ip.export(i, 0), ip2.export(i, 0))
            which = 2 if kind == "hcl" else 1
            assert torch.equal(ip.export(i, which), ip2.export(i, which))


def _prefill_then_block(model, prompt, chunk, max_chunk):
    from evspark_b200.specdec.block import block_forward, prefill

    ip = model.initialize_inference_params(len(prompt) + 64, max_chunk=max_chunk)
    pre = prefill(model, torch.tensor(prompt)[None], ip)
    blk = block_forward(model, torch.tensor(chunk)[None], ip)
    ip.close()
    return pre, blk


@pytest.mark.parametrize("which", ["tiny", "7b_slice"])
def test_prefill_chunking_invariant_bitwise(cuda, tiny, which):
    """Prefilling in 16-token chunks (split-KV attention) and in 64-token chunks (fused attention)
    gives the same bits at every position, and the same verify block afterwards: the fused kernel
    reproduces the split-KV partials and their fold exactly, and nothing else depends on chunking."""
    if which == "tiny":
        model, _ = tiny
    else:
        from evspark_b200.config import EVO2_7B_SLICE
        from evspark_b200.model import TargetModel

        model = TargetModel.random(EVO2_7B_SLICE, seed=5, device=cuda, init_on="cuda")
    rng = np.random.default_rng(17)
    prompt = rng.choice([65, 67, 71, 84], size=150)
    chunk = rng.choice([65, 67, 71, 84], size=13)
    pre16, blk16 = _prefill_then_block(model, prompt, chunk, 16)
    pre64, blk64 = _prefill_then_block(model, prompt, chunk, 64)
    assert torch.equal(pre16, pre64), (pre16 - pre64).abs().max().item()
    assert torch.equal(blk16, blk64)
    if which != "tiny":
        model.close()


@pytest.mark.parametrize("which,L", [("tiny", 20000), ("7b_slice", 6000), ("7b_slice", 2500)])
def test_long_context_multi_block_split_kv_bitwise(cuda, tiny, which, L):
    """At contexts long enough that each split-KV CTA walks several key blocks (the grid keeps about
    16 CTAs per SM), prefilling in 16-token chunks (split-KV + combine) and in 64-token chunks (fused
    kernel) still gives the same bits at every position and for the verify block afterwards.  At
    2,500 keys (40 blocks, one per CTA) the combine kernel folds both levels itself."""
    if which == "tiny":
        model, _ = tiny
    else:
        from evspark_b200.config import EVO2_7B_SLICE
        from evspark_b200.model import TargetModel

        model = TargetModel.random(EVO2_7B_SLICE, seed=9, device=cuda, init_on="cuda")
    n_sm = torch.cuda.get_device_properties(cuda).multi_processor_count
    kv_blocks = (L + 13 + 63) // 64
    blocks_per_cta = -(-kv_blocks * model.cfg.n_heads // (16 * n_sm))
    if L >= 6000:
        assert blocks_per_cta > 1, "the context must be long enough for several key blocks per CTA"
    else:
        assert 16 < kv_blocks <= 64, "a context of a few 16-block groups"
    rng = np.random.default_rng(23)
    prompt = rng.choice([65, 67, 71, 84], size=L)
    chunk = rng.choice([65, 67, 71, 84], size=13)
    pre16, blk16 = _prefill_then_block(model, prompt, chunk, 16)
    pre64, blk64 = _prefill_then_block(model, prompt, chunk, 64)
    assert torch.equal(pre16, pre64), (pre16 - pre64).abs().max().item()
    assert torch.equal(blk16, blk64)
    if which != "tiny":
        model.close()


def test_long_context_group_fold_in_cta_bitwise(cuda):
    """Eight rows of 6,000 keys give the split-KV kernel enough key blocks per CTA to walk whole
    16-block groups and fold them in the CTA; one row alone gives per-block partials, the group
    fold kernel and the combine.  Every row's verify block agrees bit for bit between the two."""
    from evspark_b200.config import EVO2_7B_SLICE
    from evspark_b200.model import TargetModel
    from evspark_b200.specdec.block import block_forward, prefill

    model = TargetModel.random(EVO2_7B_SLICE, seed=9, device=cuda, init_on="cuda")
    n_sm = torch.cuda.get_device_properties(cuda).multi_processor_count
    B, L, H = 8, 6000, model.cfg.n_heads
    kv_blocks = (L + 13 + 63) // 64

    def blocks_per_cta(rows):
        return -(-kv_blocks * H * rows // (16 * n_sm))

    assert blocks_per_cta(B) >= 8 > blocks_per_cta(1), "one path each: in-CTA group fold, per-block partials"
    rng = np.random.default_rng(29)
    prompts = rng.choice([65, 67, 71, 84], size=(B, L))
    chunks = rng.choice([65, 67, 71, 84], size=(B, 13))
    ip = model.initialize_inference_params(L + 64, max_batch=B, max_chunk=1024)
    prefill(model, torch.tensor(prompts), ip)
    blk = block_forward(model, torch.tensor(chunks), ip)
    ip.close()
    for r in range(B):
        ip1 = model.initialize_inference_params(L + 64, max_chunk=1024)
        prefill(model, torch.tensor(prompts[r])[None], ip1)
        one = block_forward(model, torch.tensor(chunks[r])[None], ip1)
        ip1.close()
        assert torch.equal(blk[r], one[0]), (r, (blk[r] - one[0]).abs().max().item())
    model.close()


TOL_FP32_2K = 2e-5  # max-abs logits after a 2048-token context (8x the 256-token prompt of the tiny
                    # workload): the fp32 recurrences over 2048 positions (poles up to 0.999) and the
                    # softmax over 2k keys grow fp32 rounding noise; the oracle itself, run in fp32,
                    # is 6.1e-6 from fp64 on this case


def test_tiny_long_prefill_vs_oracle(tiny, oracle_tiny):
    """2048-token prompt prefilled in 256-token chunks (IIR over long chunks, MR tail carry across
    chunks, fused attention over 2 k keys), then a verify block: fp64 oracle agreement."""
    from evspark_b200.specdec.block import block_forward, prefill

    model, _ = tiny
    rng = np.random.default_rng(23)
    prompt = rng.choice([65, 67, 71, 84], size=2048)
    chunk = rng.choice([65, 67, 71, 84], size=13)
    ip = model.initialize_inference_params(2048 + 64, max_chunk=256)
    pre = prefill(model, torch.tensor(prompt)[None], ip)
    got = block_forward(model, torch.tensor(chunk)[None], ip)[0].cpu().double()
    st = oracle_tiny.init_state(1, 2048 + 64)
    ref_pre, _, _ = oracle_tiny.forward(prompt[None], st, prefill=True)
    ref, _, _ = oracle_tiny.forward(chunk[None], st)
    err_pre = (pre[0, -1].cpu().double() - ref_pre[0, -1].double()).abs().max().item()
    err = (got - ref[0].double()).abs().max().item()
    print(f"[fp32 parity] 2048-token context: prefill {err_pre:.3e}, verify block {err:.3e}")
    assert err_pre <= TOL_FP32_2K, err_pre
    assert err <= TOL_FP32_2K, err
    ip.close()


def test_tiny_slice_equals_replay_bitwise(tiny, golden):
    """Rollback to k gives exactly the state of replaying the first k+1 chunk tokens."""
    from evspark_b200.specdec.block import (block_forward, clone_inference_params, prefill, slice_states_to_accept,
                                            snapshot_states)

    model, _ = tiny
    g = golden("tiny_model.npz")
    prompt, chunk = g["full/prompt"], g["full/chunk"]
    ip0 = model.initialize_inference_params(len(prompt) + 64)
    prefill(model, torch.tensor(prompt[:-1])[None], ip0)
    ipf = clone_inference_params(ip0)
    _, stash = block_forward(model, torch.tensor(chunk)[None], ipf, retain=True)
    for k in range(len(chunk)):
        ips = clone_inference_params(ipf)
        slice_states_to_accept(ips, stash, k)
        ipr = clone_inference_params(ip0)
        block_forward(model, torch.tensor(chunk[: k + 1])[None], ipr)
        kv = ip0.offset + k + 1
        a, b = snapshot_states(ips, kv_len=kv), snapshot_states(ipr, kv_len=kv)
        from evspark_b200.specdec.block import diff_states

        worst = max(v["max_abs"] for v in diff_states(a, b).values())
        assert worst == 0.0, (k, worst)
        ips.close()
        ipr.close()


def test_tiny_ragged_slice_vs_golden(golden, tiny):
    from evspark_b200.specdec.block import block_forward, expand_inference_params, prefill, slice_states_to_accept

    model, _ = tiny
    g = golden("tiny_model.npz")
    prompt, chunks, ks = g["ragged/prompt"], g["ragged/chunks"], g["ragged/ks"]
    model.config.max_batch_size = 2
    try:
        ip = model.initialize_inference_params(len(prompt) + 64)
    finally:
        model.config.max_batch_size = 1
    prefill(model, torch.tensor(prompt[:-1])[None], ip)
    expand_inference_params(ip, 2)
    lg, stash = block_forward(model, torch.tensor(chunks), ip, retain=True)
    np.testing.assert_allclose(lg.cpu().numpy(), g["ragged/block_logits"], atol=TOL_FP32, rtol=0)
    slice_states_to_accept(ip, stash, ks)
    for i, kind in enumerate(model.cfg.layer_types):
        if kind == "mha":
            continue
        names = [("fir_state_dict", 0)] + ([("fir_inner_state_dict", 1)] if kind != "hcl" else [("state_dict", 2)])
        for nm, which in names:
            ref = g[f"ragged/slice/{nm}/{i}"]
            got = ip.export(i, which, rows=2).cpu().numpy()
            np.testing.assert_allclose(got, ref, atol=2e-5 * max(1.0, np.abs(ref).max()), rtol=0, err_msg=f"{nm}/{i}")


# ---------------------------------------------------------------------------
# verification and transform known answers
# ---------------------------------------------------------------------------

def test_verify_kat_identical_decisions(cuda, golden):
    from evspark_b200.specdec.verifier import verify_round, verify_round_greedy

    k = golden("verify_kat.npz")
    for c, seed in enumerate(k["verify/seeds"]):
        rng = np.random.default_rng(int(seed))
        vr = verify_round(k["verify/tokens"][c], k["verify/q"][c].astype(np.float64),
                          k["verify/p"][c].astype(np.float64), rng)
        got = [vr.accepted_len, int(vr.from_residual), int(vr.fallback)] + vr.tokens.tolist()
        want = [int(v) for v in k["verify/result"][c][: len(got)]]
        assert got == want, (c, got, want)
        # the generator advanced by exactly the uniforms the reference consumed
        ref_rng = np.random.default_rng(int(seed))
        from oracle import specdec as sd

        sd.verify_round(k["verify/tokens"][c], k["verify/q"][c].astype(np.float64),
                        k["verify/p"][c].astype(np.float64), ref_rng)
        assert rng.random() == ref_rng.random()
    vg = verify_round_greedy(k["greedy/x"], k["greedy/p"])
    assert [vg.accepted_len] + vg.tokens.tolist() == k["greedy/result"].tolist()


def test_transform_kat(cuda, golden):
    from evspark_b200.specdec.transforms import apply_transform

    k = golden("verify_kat.npz")
    for key in [x for x in k if x.startswith("transform/T")]:
        T, topk = key.split("/")[1][1:].split("_k")
        got = np.stack([apply_transform(r, float(T), int(topk)) for r in k["transform/logits"][:16]])
        np.testing.assert_allclose(got, k[key][:16], atol=1e-15, rtol=1e-13, err_msg=key)


# ---------------------------------------------------------------------------
# 7B-width bf16 model (4 blocks) vs the bf16-emulating oracle
# ---------------------------------------------------------------------------

def test_7b_width_bf16_block_vs_oracle(cuda):
    """Evo2-7B width, four blocks (SE, MR, LI, MHA): block == native steps bit for bit, and every
    block plus the head within the bf16 bounds of the oracle on the device's residual stream."""
    from evspark_b200.config import EVO2_7B_SLICE
    from evspark_b200.model import TargetModel
    from evspark_b200.specdec.block import block_forward, prefill, step_forward_reference, clone_inference_params
    from evspark_b200.weights import init_target_weights
    from tests import _parity

    cfg = EVO2_7B_SLICE
    w = init_target_weights(cfg, seed=7)
    model = TargetModel(cfg, w, device=cuda)
    rng = np.random.default_rng(3)
    prompt = rng.choice([65, 67, 71, 84], size=40)
    chunk = rng.choice([65, 67, 71, 84], size=13)
    ip = model.initialize_inference_params(128)
    prefill(model, torch.tensor(prompt)[None], ip)
    ip2 = clone_inference_params(ip)
    logits = block_forward(model, torch.tensor(chunk)[None], ip)[0].cpu().double()
    step = step_forward_reference(model, torch.tensor(chunk)[None], ip2)[0].cpu().double()
    assert torch.equal(logits, step), "bf16 block forward must equal the native T=1 path bit for bit"
    ip.close()
    ip2.close()
    xs, pre, blk = _parity.device_block_outputs(cfg, model.weights, prompt, chunk, cuda)
    assert torch.equal(blk.double(), logits)
    rep = _parity.teacher_forced_report(cfg, w, np.concatenate([prompt, chunk]), len(prompt), xs, pre, blk,
                                        free_running=True)
    _parity.assert_teacher_forced(rep)
    model.close()


@pytest.mark.parametrize("n_prompt", [700, 832])
def test_serial_split_prefill_equals_split_k_bitwise(cuda, n_prompt):
    """A prefill chunk of >= 512 tokens runs the large projections with every split of the fixed
    split plan in one CTA, storing the splits' running sum as a single split (96- and 128-token
    tiles at 700 tokens, 96-token tiles at 832).  Its logits at every position, and the verify
    block after it, equal a prefill in 64-token chunks (per-split partial sums added by the
    consumers) bit for bit."""
    from evspark_b200.config import EVO2_7B_SLICE
    from evspark_b200.model import TargetModel

    model = TargetModel.random(EVO2_7B_SLICE, seed=13, device=cuda, init_on="cuda")
    rng = np.random.default_rng(31)
    prompt = rng.choice([65, 67, 71, 84], size=n_prompt)
    chunk = rng.choice([65, 67, 71, 84], size=13)
    pre_one, blk_one = _prefill_then_block(model, prompt, chunk, 1024)
    pre64, blk64 = _prefill_then_block(model, prompt, chunk, 64)
    assert torch.equal(pre_one, pre64), (pre_one - pre64).abs().max().item()
    assert torch.equal(blk_one, blk64)
    model.close()
