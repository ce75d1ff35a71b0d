"""Rejection-sampling verifier on the device (evspark/specdec/verifier.py:18-176).

Same names, arguments, results and errors as the reference.  The decision math runs in fp64
inside ``evs_verify`` / ``evs_sample``; the host only moves the rows and keeps the random
stream exact: a round pre-draws its worst-case γ+1 uniforms from ``rng`` and then rewinds the
generator to just after the uniforms the device actually consumed, so the numpy generator
advances exactly as the reference's sequential ``rng.random()`` / ``rng.choice`` calls do
(``Generator.choice(V, p=...)`` consumes one uniform: an inverse-CDF draw).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from evspark_b200 import _native as N
from evspark_b200.specdec.transforms import device


@dataclass
class VerifyResult:
    tokens: np.ndarray
    accepted_len: int
    accepted_mask: np.ndarray
    from_residual: bool
    fallback: bool
    winner: int = 0


def _rows(x, shape_msg) -> torch.Tensor:
    return torch.as_tensor(np.ascontiguousarray(np.asarray(x, dtype=np.float64)), device=device())


def sample_categorical(probs, rng: np.random.Generator) -> int:
    """One draw from ``probs`` (clipped at 0, normalised; uniform if the mass is 0/non-finite)."""
    p = np.asarray(probs, dtype=np.float64).ravel()
    dev = device()
    rows = torch.as_tensor(p, device=dev)[None]
    u = torch.tensor([float(rng.random())], dtype=torch.float64, device=dev)
    out = torch.empty(1, dtype=torch.int64, device=dev)
    N.check(N.lib().evs_sample(rows.data_ptr(), 1, p.shape[0], u.data_ptr(), out.data_ptr(), N.stream_ptr()),
            "evs_sample")
    return int(out.item())


def draw_uniforms(rng: np.random.Generator, n: int):
    """Pre-draw ``n`` uniforms; returns (values, saved generator state)."""
    state = rng.bit_generator.state
    return rng.random(n), state


def rewind_uniforms(rng: np.random.Generator, state, consumed: int) -> None:
    """Leave ``rng`` exactly ``consumed`` uniforms past ``state``."""
    rng.bit_generator.state = state
    if consumed > 0:
        rng.random(int(consumed))


def verify_device(p: torch.Tensor, q: torch.Tensor | None, x: torch.Tensor, u: torch.Tensor | None, greedy: bool,
                  out: tuple | None = None):
    """Batched device verification: p [B, γ+1, V] fp64, q [B, γ, V] fp64, x [B, γ] int64,
    u [B, γ+1] fp64.  Returns device (accepted [B], tokens [B, γ+1], info [B, 3]), written into
    ``out`` = (int32 [B], int64 [B, γ+1], int32 [B, 3]) contiguous tensors when given."""
    B, g1, V = p.shape
    g = g1 - 1
    dev = p.device
    if out is not None:
        acc, toks, info = out
        if (acc.dtype != torch.int32 or toks.dtype != torch.int64 or info.dtype != torch.int32
                or acc.numel() != B or toks.shape != (B, g + 1) or info.shape != (B, 3)
                or not (acc.is_contiguous() and toks.is_contiguous() and info.is_contiguous())):
            raise ValueError("verify_device: out must be contiguous int32 [B], int64 [B, γ+1] and int32 [B, 3]")
    else:
        acc = torch.empty(B, dtype=torch.int32, device=dev)
        toks = torch.empty(B, g + 1, dtype=torch.int64, device=dev)
        info = torch.empty(B, 3, dtype=torch.int32, device=dev)
    N.check(N.lib().evs_verify(p.data_ptr(), N.ptr(q), x.data_ptr(), N.ptr(u), B, g, V, int(greedy),
                               acc.data_ptr(), toks.data_ptr(), info.data_ptr(), N.stream_ptr()), "evs_verify")
    return acc, toks, info


def verify_device_multicand(p: torch.Tensor, q: torch.Tensor | None, x: torch.Tensor, u: torch.Tensor | None,
                            greedy: bool):
    """SpecInfer verification of B candidate drafts of one stream on the device:
    p [B, γ+1, V] fp64 (greedy: raw logits), q [B, γ, V] fp64, x [B, γ] int64, u [γB+1] fp64.
    Returns device (tokens [γ+1], info [5] = accepted, from_residual, fallback, consumed, winner)."""
    B, g1, V = p.shape
    g = g1 - 1
    toks = torch.empty(g + 1, dtype=torch.int64, device=p.device)
    info = torch.empty(5, dtype=torch.int32, device=p.device)
    N.check(N.lib().evs_verify_multicand(p.contiguous().data_ptr(), N.ptr(q), x.contiguous().data_ptr(), N.ptr(u), B, g,
                                         V, int(greedy), toks.data_ptr(), info.data_ptr(), N.stream_ptr()),
            "evs_verify_multicand")
    return toks, info


def _result(acc: int, toks: np.ndarray, info: np.ndarray, gamma: int) -> VerifyResult:
    mask = np.zeros(gamma, dtype=bool)
    mask[:acc] = True
    return VerifyResult(tokens=toks[: acc + 1].astype(np.int64), accepted_len=int(acc), accepted_mask=mask,
                        from_residual=bool(info[0]), fallback=bool(info[1]))


def verify_round(draft_tokens, draft_probs, target_probs, rng: np.random.Generator) -> VerifyResult:
    draft_tokens = np.asarray(draft_tokens, dtype=np.int64).ravel()
    q = np.asarray(draft_probs, dtype=np.float64)
    p = np.asarray(target_probs, dtype=np.float64)
    gamma = int(draft_tokens.shape[0])
    if q.ndim != 2 or p.ndim != 2:
        raise ValueError(f"draft_probs/target_probs must be 2-D, got {q.shape} / {p.shape}")
    if q.shape[0] != gamma:
        raise ValueError(f"draft_probs rows must equal γ={gamma}, got {q.shape[0]}")
    if p.shape[0] != gamma + 1:
        raise ValueError(f"target_probs rows must equal γ+1={gamma + 1}, got {p.shape[0]}")
    if q.shape[1] != p.shape[1]:
        raise ValueError(f"vocabulary mismatch: q V={q.shape[1]} vs p V={p.shape[1]}")
    dev = device()
    pt = torch.as_tensor(np.ascontiguousarray(p), device=dev)[None]
    qt = torch.as_tensor(np.ascontiguousarray(q), device=dev)[None]
    xt = torch.as_tensor(draft_tokens, device=dev)[None]
    uv, state = draw_uniforms(rng, gamma + 1)
    ut = torch.as_tensor(uv, device=dev)[None]
    acc, toks, info = verify_device(pt, qt, xt, ut, greedy=False)
    acc_h, toks_h, info_h = int(acc[0].item()), toks[0].cpu().numpy(), info[0].cpu().numpy()
    rewind_uniforms(rng, state, int(info_h[2]))
    return _result(acc_h, toks_h, info_h, gamma)


def verify_round_greedy(draft_tokens, target_probs) -> VerifyResult:
    draft_tokens = np.asarray(draft_tokens, dtype=np.int64).ravel()
    p = np.asarray(target_probs, dtype=np.float64)
    gamma = int(draft_tokens.shape[0])
    if p.ndim != 2:
        raise ValueError(f"target_probs must be 2-D, got {p.shape}")
    if p.shape[0] != gamma + 1:
        raise ValueError(f"target_probs rows must equal γ+1={gamma + 1}, got {p.shape[0]}")
    dev = device()
    pt = torch.as_tensor(np.ascontiguousarray(p), device=dev)[None]
    xt = torch.as_tensor(draft_tokens, device=dev)[None]
    acc, toks, info = verify_device(pt, None, xt, None, greedy=True)
    return _result(int(acc[0].item()), toks[0].cpu().numpy(), info[0].cpu().numpy(), gamma)
