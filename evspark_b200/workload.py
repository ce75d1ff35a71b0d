"""Seeded synthetic prompts standing in for the reference's evaluation prompt pack.

Order-3 Markov chain over the ACGT byte ids {65, 67, 71, 84}: a 64-context x 4 transition table
drawn from Dirichlet(1), G/C columns rescaled so that the chain's stationary GC fraction is
0.50 (to 1e-3), then L tokens sampled from the stationary start.  Config 1 uses iid ACGT.
"""

from __future__ import annotations

import numpy as np

ACGT = np.array([65, 67, 71, 84], dtype=np.int64)
_GC = np.array([False, True, True, False])


def _stationary_gc(P: np.ndarray) -> tuple[float, np.ndarray]:
    # 64 contexts (x_{t-3}, x_{t-2}, x_{t-1}); next context = (x_{t-2}, x_{t-1}, x_t)
    n = 64
    M = np.zeros((n, n))
    for c in range(n):
        for a in range(4):
            M[c, (c * 4 + a) % n] += P[c, a]
    pi = np.full(n, 1.0 / n)
    for _ in range(2000):
        pi = pi @ M
    pi /= pi.sum()
    return float((pi[:, None] * P)[:, _GC].sum()), pi


def markov_prompt(length: int, seed: int, gc: float = 0.5) -> np.ndarray:
    rng = np.random.default_rng(seed)
    base = rng.dirichlet(np.ones(4), size=64)
    lo, hi = 1e-3, 1e3
    for _ in range(100):
        f = np.sqrt(lo * hi)
        P = base.copy()
        P[:, _GC] *= f
        P /= P.sum(1, keepdims=True)
        g, pi = _stationary_gc(P)
        if abs(g - gc) < 1e-3:
            break
        lo, hi = (f, hi) if g < gc else (lo, f)
    ctx = int(rng.choice(64, p=pi))
    out = np.empty(length, dtype=np.int64)
    for t in range(length):
        a = int(rng.choice(4, p=P[ctx]))
        out[t] = ACGT[a]
        ctx = (ctx * 4 + a) % 64
    return out


def iid_prompt(length: int, seed: int) -> np.ndarray:
    return np.random.default_rng(seed).choice(ACGT, size=length)


def to_text(ids: np.ndarray) -> str:
    return bytes(np.asarray(ids, dtype=np.uint8).tolist()).decode("ascii")
