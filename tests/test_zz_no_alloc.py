"""GPU: the no-allocation projection entry point agrees with the regular one.

``evs_gemm_bf16_noalloc`` exists for callers that cannot allocate device memory at call time
(a host that owns all device memory through its own pool, code running during stream capture,
plugins not allowed to allocate after start-up).  It keeps its split-K partial sums in a fixed
file-scope device array.  This file is collected last so that a failure here cannot stop the
rest of the GPU suite; it passes alone in a fresh process and after the other tests.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

TOL_REL = 2e-3  # same bound as the tcgen05 GEMM test against torch


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from evspark_b200 import _native as N

    N.call("evs_device_check")
    return torch.device("cuda:0")


@pytest.mark.parametrize("N_,K,M", [(12288, 4096, 13), (4096, 11008, 13), (512, 4096, 16), (256, 640, 40)])
def test_noalloc_matches_regular_entry_point_twice(cuda, N_, K, M):
    from evspark_b200 import _native as N

    g = torch.Generator(device=cuda).manual_seed(N_ * 7 + K + M)
    W = torch.randn(N_, K, device=cuda, generator=g).to(torch.bfloat16)
    X = torch.randn(M, K, device=cuda, generator=g).to(torch.bfloat16)
    ref = torch.empty(M, N_, device=cuda)
    N.call("evs_gemm_bf16", W.data_ptr(), X.data_ptr(), ref.data_ptr(), N_, K, M, 1, N.stream_ptr())
    outs = []
    for _ in range(2):  # the shared scratch keeps the previous call's partials: results must not depend on it
        out = torch.full((M, N_), float("nan"), device=cuda)
        N.call("evs_gemm_bf16_noalloc", W.data_ptr(), X.data_ptr(), out.data_ptr(), N_, K, M, N.stream_ptr())
        torch.cuda.synchronize()
        outs.append(out)
    scale = ref.abs().max().item()
    exact = X.float() @ W.float().T
    for out in outs:
        assert torch.isfinite(out).all()
        err = (out - ref).abs().max().item()
        assert err <= TOL_REL * scale, (err, scale)
        err = (out - exact).abs().max().item()
        assert err <= TOL_REL * exact.abs().max().item(), err
    # the partial sums are added in fixed split order: the same bits on every call
    assert torch.equal(outs[0], outs[1])


def _noalloc_splits(N_, K):
    """The entry point's K split: the smallest count that gives at least 148 CTAs, at most K / 64."""
    tiles, splits = N_ // 128, 1
    while tiles * splits < 148 and splits < K // 64:
        splits += 1
    return splits


def test_noalloc_at_the_scratch_limit(cuda):
    """splits * M * N exactly at the 1,048,576-value limit runs and matches the fp32 product; one
    token row more is rejected."""
    from evspark_b200 import _native as N

    N_, K, M = 16384, 512, 32
    splits = _noalloc_splits(N_, K)
    assert splits * M * N_ == 1 << 20
    g = torch.Generator(device=cuda).manual_seed(5)
    W = torch.randn(N_, K, device=cuda, generator=g).to(torch.bfloat16)
    X = torch.randn(M + 1, K, device=cuda, generator=g).to(torch.bfloat16)
    out = torch.full((M, N_), float("nan"), device=cuda)
    N.call("evs_gemm_bf16_noalloc", W.data_ptr(), X.data_ptr(), out.data_ptr(), N_, K, M, N.stream_ptr())
    exact = X[:M].float() @ W.float().T
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    assert (out - exact).abs().max().item() <= TOL_REL * exact.abs().max().item()
    out1 = torch.empty(M + 1, N_, device=cuda)
    with pytest.raises(ValueError, match="scratch"):
        N.call("evs_gemm_bf16_noalloc", W.data_ptr(), X.data_ptr(), out1.data_ptr(), N_, K, M + 1, N.stream_ptr())


def test_noalloc_rejects_sizes_beyond_the_fixed_scratch(cuda):
    from evspark_b200 import _native as N

    W = torch.zeros(12288, 4096, device=cuda, dtype=torch.bfloat16)
    X = torch.zeros(512, 4096, device=cuda, dtype=torch.bfloat16)
    out = torch.empty(512, 12288, device=cuda)
    with pytest.raises(ValueError, match="scratch"):
        N.call("evs_gemm_bf16_noalloc", W.data_ptr(), X.data_ptr(), out.data_ptr(), 12288, 4096, 512,
               N.stream_ptr())


def test_noalloc_on_a_second_device(cuda):
    """The shared-memory opt-in, the scratch array and the error word are per device: a call on a
    second GPU after calls on the first gives the same bits as on the first."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")
    from evspark_b200 import _native as N

    N_, K, M = 4096, 4096, 13
    outs = []
    for dev in (0, 1, 0):
        d = torch.device("cuda", dev)
        with torch.cuda.device(d):
            g = torch.Generator(device=d).manual_seed(5)
            W = torch.randn(N_, K, device=d, generator=g).to(torch.bfloat16)
            X = torch.randn(M, K, device=d, generator=g).to(torch.bfloat16)
            out = torch.full((M, N_), float("nan"), device=d)
            N.call("evs_gemm_bf16_noalloc", W.data_ptr(), X.data_ptr(), out.data_ptr(), N_, K, M,
                   torch.cuda.current_stream(d).cuda_stream)
            torch.cuda.synchronize(d)
            exact = X.float() @ W.float().T
            assert (out - exact).abs().max().item() <= TOL_REL * exact.abs().max().item()
            outs.append(out.cpu())
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])
