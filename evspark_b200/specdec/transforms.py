"""Sampling transform on the device (evspark/specdec/transforms.py:18-64).

``apply_transform(logits, temperature, top_k)``: logits/T -> max-subtracted softmax -> keep the
top-k by (-p, index) -> renormalise; T <= 0 gives the one-hot argmax (lowest index on ties).
Computed in fp64 by ``evs_transform``.
"""

from __future__ import annotations

import numpy as np
import torch

from evspark_b200 import _native as N

DEFAULT_TEMPERATURE = 1.0
DEFAULT_TOP_K = 4


def device() -> torch.device:
    if not torch.cuda.is_available():
        raise RuntimeError("evspark_b200 runs on the B200; no CUDA device is available")
    return torch.device("cuda", torch.cuda.current_device())


def transform_rows(logits: torch.Tensor, temperature: float, top_k: int | None) -> torch.Tensor:
    """Device logits [R, V] (fp32 or fp64) -> device fp64 probabilities [R, V]."""
    if logits.dtype not in (torch.float32, torch.float64):
        logits = logits.to(torch.float32)
    lg = logits.contiguous()
    R, V = lg.shape
    out = torch.empty(R, V, dtype=torch.float64, device=lg.device)
    k = 0 if top_k is None else int(top_k)
    N.check(N.lib().evs_transform(lg.data_ptr(), int(lg.dtype == torch.float64), R, V, float(temperature), k,
                                  out.data_ptr(), N.stream_ptr()), "evs_transform")
    return out


def apply_transform(logits, temperature: float = DEFAULT_TEMPERATURE, top_k: int | None = DEFAULT_TOP_K) -> np.ndarray:
    x = np.asarray(logits, dtype=np.float64)
    if x.ndim != 1:
        raise ValueError(f"logits must be a 1-D [V] row, got shape={x.shape}")
    if x.shape[0] == 0:
        raise ValueError("empty vocabulary")
    out = transform_rows(torch.as_tensor(x, device=device())[None], temperature, top_k)
    return out[0].cpu().numpy()
