"""CPU: the C-ABI library loads, exports every symbol include/evspark_sm100.h declares, and
refuses to run without an sm_100 device (no compute call is made here)."""

from __future__ import annotations

import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols() -> set[str]:
    text = (ROOT / "include" / "evspark_sm100.h").read_text()
    return set(re.findall(r"^EVS_API\s+[\w\s\*]+?\b(evs_\w+)\(", text, flags=re.M))


def test_library_builds_and_exports_every_declared_symbol():
    from evspark_b200.build import build

    lib_path = build()
    import ctypes

    h = ctypes.CDLL(str(lib_path))
    decl = declared_symbols()
    assert len(decl) >= 30
    missing = [s for s in sorted(decl) if not hasattr(h, s)]
    assert not missing, missing


def test_bindings_cover_the_header():
    from evspark_b200 import _native as N

    assert declared_symbols() == set(N.exported_symbols())


def test_device_check_without_gpu_reports_enodev():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from evspark_b200 import _native as N

    assert N.lib().evs_device_check() == N.EVS_ENODEV
    assert b"device" in N.lib().evs_last_error()
    with pytest.raises(RuntimeError):
        N.call("evs_device_check")


def test_product_fails_loudly_without_gpu():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from evspark_b200.config import TINY
    from evspark_b200.model import TargetModel

    with pytest.raises(RuntimeError, match="CUDA|device"):
        TargetModel.random(TINY, device="cuda:0")


def test_verify_device_rejects_mismatched_result_buffers():
    """The device round hands verify_device views of one result buffer; a view of the wrong dtype,
    shape or layout is refused on the host, before any device call."""
    import torch

    from evspark_b200.specdec.verifier import verify_device

    B, g, V = 1, 12, 512
    p = torch.zeros(B, g + 1, V, dtype=torch.float64)
    x = torch.zeros(B, g, dtype=torch.int64)
    good = (torch.zeros(B, dtype=torch.int32), torch.zeros(B, g + 1, dtype=torch.int64),
            torch.zeros(B, 3, dtype=torch.int32))
    bad = [
        (good[0].long(), good[1], good[2]),                                   # accepted not int32
        (good[0], torch.zeros(B, g, dtype=torch.int64), good[2]),             # tokens one short
        (good[0], good[1], torch.zeros(B, 4, dtype=torch.int32)),             # flags of the wrong width
        (good[0], torch.zeros(g + 1, 2, dtype=torch.int64).t()[:1], good[2]),  # tokens not contiguous
    ]
    for out in bad:
        with pytest.raises(ValueError, match="out must be"):
            verify_device(p, None, x, None, greedy=True, out=out)
