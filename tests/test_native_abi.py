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
