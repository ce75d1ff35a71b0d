"""Speculative loop restated over the oracle model (TEST INFRASTRUCTURE ONLY).

Follows evspark/specdec/block/loop.py:258-581 (anchor protocol, slice rollback,
truncation round) and the native references at loop.py:584-658.  Drafts come
from a ``probs(prefix)`` model (e.g. the identity drafter,
evspark/specdec/drafts.py:16-36) proposed token by token (loop.py:131-162).
"""

from __future__ import annotations

import numpy as np

from . import specdec as sd
from .model import OracleTarget

VOCAB = 512
MASS_IDS = (65, 67, 71, 84, 78)


class IdentityDraft:
    """q(·|prefix) = one-hot of the last token; empty prefix -> uniform over ACGTN."""

    def probs(self, prefix) -> np.ndarray:
        out = np.zeros(VOCAB)
        prefix = np.asarray(prefix, dtype=np.int64).ravel()
        if prefix.size and 0 <= int(prefix[-1]) < VOCAB:
            out[int(prefix[-1])] = 1.0
        else:
            out[list(MASS_IDS)] = 1.0 / len(MASS_IDS)
        return out


def _propose(draft, seen, gamma, greedy, rng, temperature, top_k):
    toks = np.empty(gamma, dtype=np.int64)
    rows = np.empty((gamma, VOCAB))
    buf = list(seen)
    for i in range(gamma):
        q = np.asarray(draft.probs(np.asarray(buf)), dtype=np.float64)
        if not greedy:
            q = sd.q_prime_from_raw(q, temperature, top_k)
        rows[i] = q
        t = int(np.argmax(q)) if greedy else sd.sample_categorical(q, rng)
        toks[i] = t
        buf.append(t)
    return toks, rows


def speculative_generate(model: OracleTarget, draft, prompt, n_tokens: int, gamma: int, greedy: bool,
                         rng, temperature: float = 1.0, top_k: int | None = 4):
    """Returns (emitted ids, per-round accepted lengths, final state)."""
    prompt = np.asarray(prompt, dtype=np.int64).ravel()
    L = prompt.size
    st = model.init_state(1, L + n_tokens + gamma + 2)
    model.forward(prompt[None, :-1], st, prefill=True)
    y = int(prompt[-1])
    seen = prompt.copy()
    emitted: list[int] = []
    ks: list[int] = []
    while len(emitted) < n_tokens:
        remaining = n_tokens - len(emitted)
        toks, q = _propose(draft, seen, gamma, greedy, rng, temperature, top_k)
        chunk = np.concatenate([[y], toks])[None]
        logits, stash, _ = model.forward(chunk, st, retain=True)
        rows = logits[0].double().numpy()
        if greedy:
            res = sd.verify_round_greedy(toks, rows)
        else:
            p = np.stack([sd.apply_transform(r, temperature, top_k) for r in rows])
            res = sd.verify_round(toks, q, p, rng)
        k = res.accepted_len
        take = min(len(res.tokens), remaining)
        taken = res.tokens[:take]
        if not (k == gamma and take == k + 1):
            model.slice(st, stash, take - 1)
        emitted.extend(int(t) for t in taken)
        seen = np.concatenate([seen, taken])
        y = int(taken[-1])
        ks.append(k)
    return np.asarray(emitted[:n_tokens], dtype=np.int64), ks, st


def native_greedy(model: OracleTarget, prompt, n_tokens: int):
    prompt = np.asarray(prompt, dtype=np.int64).ravel()
    st = model.init_state(1, prompt.size + n_tokens + 2)
    logits, _, _ = model.forward(prompt[None], st, prefill=True)
    last = logits[0, -1].double().numpy()
    out = []
    for i in range(n_tokens):
        t = int(np.argmax(last))
        out.append(t)
        if i + 1 < n_tokens:
            last = model.forward(np.array([[t]]), st)[0][0, -1].double().numpy()
    return np.asarray(out, dtype=np.int64), st


def oracle_streams(prompts, n_tokens: int, seeds, gamma: int = 4):
    """Independent streams on the tiny oracle model (seeded weights), each with its own
    generator: the per-stream result a multi-stream decoder must reproduce, however the streams
    are grouped into batches or spread over ranks (scripts/regulatory_design/generation.py:
    196-277 runs streams independently)."""
    import torch

    from evspark_b200.config import TINY
    from evspark_b200.weights import init_target_weights

    model = OracleTarget(TINY, init_target_weights(TINY, seed=20260820), compute=torch.float64)
    out = []
    for p, s in zip(np.asarray(prompts, dtype=np.int64), seeds):
        em, _, _ = speculative_generate(model, IdentityDraft(), p, n_tokens, gamma, False, np.random.default_rng(s))
        out.append(em)
    return out
