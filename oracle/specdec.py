"""Verifier, sampling transform and neural drafter restated on CPU (TEST INFRASTRUCTURE ONLY).

* ``apply_transform`` — evspark/specdec/transforms.py:18-64: fp64 softmax of
  logits/T (max-subtracted), top-k kept by (-p, index) order, renormalised;
  T<=0 gives a one-hot argmax (lowest index on ties).
* ``q_prime_from_raw`` — evspark/specdec/block/loop.py:111-128: log(q) through
  the same transform.
* ``sample_categorical`` — evspark/specdec/verifier.py:28-40: clip to >=0,
  normalise (uniform if the mass is 0 / non-finite), one uniform ``u`` and the
  first index whose normalised cumulative sum exceeds ``u`` (the inverse-CDF
  draw numpy's ``Generator.choice(V, p=...)`` performs with one uniform).
* ``verify_round`` / ``verify_round_greedy`` / the multi-candidate variants —
  verifier.py:43-319 (Leviathan accept test, residual resampling, p fallback on
  residual underflow, bonus token).
* ``drafter_trunk`` / ``drafter_serial`` — evspark/specdec/block/neural_draft.py:157-259
  and evspark/train/drafter.py:54-409, written functionally over a weight dict.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch


# ---------------------------------------------------------------------------
# sampling primitives
# ---------------------------------------------------------------------------

def as_prob_row(p) -> np.ndarray:
    p = np.maximum(np.asarray(p, dtype=np.float64).ravel(), 0.0)
    s = float(p.sum())
    if s <= 0.0 or not np.isfinite(s):
        return np.full(p.shape[0], 1.0 / p.shape[0])
    return p / s


def inverse_cdf(p: np.ndarray, u: float) -> int:
    """Index drawn by uniform ``u`` from the normalised row ``p``."""
    cdf = np.cumsum(p)
    cdf = cdf / cdf[-1]
    return int(np.searchsorted(cdf, u, side="right"))


def sample_categorical(p, rng: np.random.Generator) -> int:
    return inverse_cdf(as_prob_row(p), float(rng.random()))


def accept_prob(p_x: float, q_x: float) -> float:
    if q_x > 0.0:
        r = p_x / q_x
        if not np.isfinite(r):
            return 0.0
        return 1.0 if r >= 1.0 else float(r)
    return 1.0 if p_x > 0.0 else 0.0


def apply_transform(logits, temperature: float = 1.0, top_k: int | None = 4) -> np.ndarray:
    x = np.asarray(logits, dtype=np.float64)
    if x.ndim != 1 or x.shape[0] == 0:
        raise ValueError(f"logits must be a non-empty [V] row, got {x.shape}")
    V = x.shape[0]
    if temperature <= 0.0:
        out = np.zeros(V)
        out[int(np.argmax(x))] = 1.0
        return out
    e = np.exp(x / float(temperature) - np.max(x / float(temperature)))
    z = float(e.sum())
    probs = np.full(V, 1.0 / V) if (z <= 0.0 or not np.isfinite(z)) else e / z
    if top_k is None or top_k <= 0 or top_k >= V:
        return probs
    keep = np.lexsort((np.arange(V), -probs))[: int(top_k)]
    out = np.zeros(V)
    out[keep] = probs[keep]
    s = float(out.sum())
    if s <= 0.0 or not np.isfinite(s):
        out[keep] = 1.0 / float(top_k)
        return out
    return out / s


def q_prime_from_raw(q, temperature: float, top_k: int | None) -> np.ndarray:
    q = np.asarray(q, dtype=np.float64).ravel()
    lg = np.full(q.shape[0], -np.inf)
    pos = q > 0.0
    if np.any(pos):
        lg[pos] = np.log(q[pos])
    else:
        lg[:] = 0.0
    return apply_transform(lg, temperature, top_k)


# ---------------------------------------------------------------------------
# verification
# ---------------------------------------------------------------------------

@dataclass
class Verdict:
    tokens: np.ndarray
    accepted_len: int
    accepted_mask: np.ndarray
    from_residual: bool
    fallback: bool
    winner: int = 0


def verify_round(draft_tokens, draft_probs, target_probs, rng) -> Verdict:
    x = np.asarray(draft_tokens, dtype=np.int64).ravel()
    q = np.asarray(draft_probs, dtype=np.float64)
    p = np.asarray(target_probs, dtype=np.float64)
    g = x.shape[0]
    if q.shape[0] != g or p.shape[0] != g + 1 or q.shape[1] != p.shape[1]:
        raise ValueError(f"shape mismatch q {q.shape} p {p.shape} gamma {g}")
    mask = np.zeros(g, dtype=bool)
    acc: list[int] = []
    for i in range(g):
        r = float(rng.random())
        if r < accept_prob(float(p[i, x[i]]), float(q[i, x[i]])):
            mask[i] = True
            acc.append(int(x[i]))
            continue
        res = np.maximum(p[i] - q[i], 0.0)
        m = float(res.sum())
        fb = m <= 0.0 or not np.isfinite(m)
        y = sample_categorical(p[i] if fb else res, rng)
        return Verdict(np.asarray(acc + [y], dtype=np.int64), len(acc), mask, True, fb)
    y = sample_categorical(p[g], rng)
    return Verdict(np.asarray(acc + [y], dtype=np.int64), g, mask, False, False)


def verify_round_greedy(draft_tokens, target_probs) -> Verdict:
    x = np.asarray(draft_tokens, dtype=np.int64).ravel()
    p = np.asarray(target_probs, dtype=np.float64)
    g = x.shape[0]
    if p.shape[0] != g + 1:
        raise ValueError(f"target rows {p.shape[0]} != gamma+1")
    mask = np.zeros(g, dtype=bool)
    acc: list[int] = []
    for i in range(g):
        t = int(np.argmax(p[i]))
        if int(x[i]) == t:
            mask[i] = True
            acc.append(t)
            continue
        return Verdict(np.asarray(acc + [t], dtype=np.int64), len(acc), mask, True, False)
    return Verdict(np.asarray(acc + [int(np.argmax(p[g]))], dtype=np.int64), g, mask, False, False)


def verify_round_greedy_multicand(draft_tokens, target_probs) -> Verdict:
    x = np.asarray(draft_tokens, dtype=np.int64)
    p = np.asarray(target_probs, dtype=np.float64)
    if x.ndim == 1:
        x = x[None]
    if p.ndim == 2:
        p = p[None]
    B, g = x.shape
    mask = np.zeros(g, dtype=bool)
    acc: list[int] = []
    live = list(range(B))
    for i in range(g):
        t = int(np.argmax(p[live[0], i]))
        m = [b for b in live if int(x[b, i]) == t]
        if not m:
            return Verdict(np.asarray(acc + [t], dtype=np.int64), len(acc), mask, True, False, live[0])
        mask[i] = True
        acc.append(t)
        live = m
    return Verdict(np.asarray(acc + [int(np.argmax(p[live[0], g]))], dtype=np.int64), g, mask, False,
                   False, live[0])


def verify_round_multicand(draft_tokens, draft_probs, target_probs, rng) -> Verdict:
    x = np.asarray(draft_tokens, dtype=np.int64)
    q = np.asarray(draft_probs, dtype=np.float64)
    p = np.asarray(target_probs, dtype=np.float64)
    if x.ndim == 1:
        x = x[None]
    if q.ndim == 2:
        q = q[None]
    if p.ndim == 2:
        p = p[None]
    B, g = x.shape
    mask = np.zeros(g, dtype=bool)
    acc: list[int] = []
    live = list(range(B))
    fb = False
    for i in range(g):
        p_i = as_prob_row(p[live[0], i])
        q_i = as_prob_row(q[live[0], i])
        chosen = None
        work = p_i
        for b in live:
            xx = int(x[b, i])
            r = float(rng.random())
            if r < accept_prob(float(work[xx]), float(q_i[xx])):
                chosen = xx
                break
            res = np.maximum(work - q_i, 0.0)
            m = float(res.sum())
            if m <= 0.0 or not np.isfinite(m):
                fb = True
                work = as_prob_row(p_i)
                break
            work = res / m
        if chosen is None:
            y = sample_categorical(work, rng)
            return Verdict(np.asarray(acc + [y], dtype=np.int64), len(acc), mask, True, fb, live[0])
        mask[i] = True
        acc.append(chosen)
        live = [b for b in live if int(x[b, i]) == chosen]
    y = sample_categorical(as_prob_row(p[live[0], g]), rng)
    return Verdict(np.asarray(acc + [y], dtype=np.int64), g, mask, False, False, live[0])


# ---------------------------------------------------------------------------
# drafter
# ---------------------------------------------------------------------------

def _rms(x, scale, eps=1e-6):
    return scale * (x / x.pow(2).mean(-1, keepdim=True).add(eps).sqrt())


def drafter_trunk(w: dict, dcfg, anchor: int, h_raw: torch.Tensor | None, ctx_len: int,
                  gamma: int | None = None):
    """γ-parallel trunk for one stream; returns (U [γ', V], h [γ', d]) in fp32."""
    gamma = dcfg.gamma if gamma is None else int(gamma)
    if not 1 <= gamma <= dcfg.gamma:
        raise ValueError(f"decode γ'={gamma} must satisfy 1 <= γ' <= training γ={dcfg.gamma}")
    d, H = dcfg.d_model, dcfg.heads
    hd = d // H
    ids = torch.full((gamma,), dcfg.mask_id, dtype=torch.long)
    ids[0] = int(anchor)
    h = w["embed.weight"][ids] @ w["in_proj.weight"].T + w["in_proj.bias"]
    h = h + w["pos.weight"][:gamma]
    if dcfg.n_inject > 0 and h_raw is not None and h_raw.shape[0] > 0:
        ctx = _rms(h_raw.float() @ w["ctx_proj.weight"].T + w["ctx_proj.bias"], w["ctx_norm.scale"])
    else:
        ctx = h.new_zeros(0, d)
    Tc = ctx.shape[0]
    t = torch.arange(Tc)
    ctx_ok = (t < ctx_len) & (t >= max(0, ctx_len - dcfg.ctx_window))
    causal = torch.arange(gamma)[None, :] <= torch.arange(gamma)[:, None]
    mask = torch.cat([ctx_ok[None, :].expand(gamma, Tc), causal], dim=1)  # [γ, Tc+γ]
    for l in range(dcfg.n_layers):
        p = f"layers.{l}."
        x = _rms(h, w[p + "ln1.scale"])
        q = (x @ w[p + "q_proj.weight"].T).view(gamma, H, hd).transpose(0, 1)
        kin = torch.cat([ctx, x], 0)
        k = (kin @ w[p + "k_proj.weight"].T).view(-1, H, hd).transpose(0, 1)
        v = (kin @ w[p + "v_proj.weight"].T).view(-1, H, hd).transpose(0, 1)
        sc = (q @ k.transpose(-1, -2)) * hd ** -0.5
        sc = sc.masked_fill(~mask[None], torch.finfo(sc.dtype).min)
        y = (torch.softmax(sc, -1) @ v).transpose(0, 1).reshape(gamma, d)
        h = h + y @ w[p + "o_proj.weight"].T
        m = _rms(h, w[p + "ln2.scale"]) @ w[p + "mlp.0.weight"].T + w[p + "mlp.0.bias"]
        m = torch.nn.functional.silu(m) @ w[p + "mlp.2.weight"].T + w[p + "mlp.2.bias"]
        h = h + m
    h = _rms(h, w["final_ln.scale"])
    U = ((h @ w["out_proj.weight"].T + w["out_proj.bias"]) @ w["embed.weight"].T) * dcfg.target_hidden ** -0.5
    return U, h


def drafter_serial(w: dict, U: torch.Tensor, h: torch.Tensor, anchor: int, greedy: bool, rng,
                   temperature: float = 1.0, top_k: int | None = 4, forced=None):
    """Serial Markov head: q_k = softmax(U_k + B[x_{k-1}]); returns (tokens, q_rows, conf)."""
    g = U.shape[0]
    V = U.shape[1]
    toks = np.empty(g, dtype=np.int64)
    rows = np.empty((g, V))
    prev = int(anchor)
    for k in range(g):
        qk = torch.softmax((U[k] + w["markov"][prev]).float(), -1).numpy().astype(np.float64)
        if greedy:
            tok = int(np.argmax(qk))
            row = qk
        else:
            row = q_prime_from_raw(qk, temperature, top_k)
            tok = sample_categorical(row, rng)
        if forced is not None:
            tok = int(forced[k])
        toks[k] = tok
        rows[k] = row
        prev = tok
    prev_ids = torch.tensor([int(anchor)] + toks[:-1].tolist(), dtype=torch.long)
    pe = w["embed.weight"][prev_ids] @ w["in_proj.weight"].T + w["in_proj.bias"]
    conf = torch.sigmoid(torch.cat([h, pe], -1) @ w["conf_w.weight"].T + w["conf_w.bias"])[:, 0]
    return toks, rows, conf.double().numpy()
