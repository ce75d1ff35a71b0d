"""Multi-stream speculative decoding: B independent streams advance in lockstep, one batched round
at a time, on one GPU.

This is the batched form of the anchor loop in evspark/specdec/block/loop.py:381-570, with the
per-row bookkeeping of the reference's batched generator (scripts/regulatory_design/
generation.py:196-277): every stream keeps its own numpy generator, anchor, emitted tokens and
state row, and the rows of one round may accept different lengths.  The device work of a round
is one batched drafter call (``evs_draft_propose`` over B anchors), one retained verify forward
of the chunk ``[B, γ+1]`` (``evs_forward``, M = B(γ+1) token rows), one transform and
verification of the B(γ+1) target rows (``evs_transform`` + ``evs_verify``) and one per-row
rollback (``evs_rollback`` with a k per row, no data movement).  The host reads back one small
array per round.

Every kernel computes a row with the same arithmetic whatever the batch size, and each stream
consumes its own generator exactly as a single-stream run does (γ uniforms for sampled drafting,
then the verifier's draws), so a stream decoded inside a batch emits the same tokens as the same
stream decoded alone with the same seed.  A stream that has reached ``n_tokens`` stays in the
batch until the slowest one finishes: it accepts nothing further (its state keeps only the anchor
each round) and its tokens are not reported.
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field

import numpy as np
import torch

from evspark_b200.specdec.block.driver import prefill
from evspark_b200.specdec.transforms import transform_rows
from evspark_b200.specdec.verifier import draw_uniforms, rewind_uniforms, verify_device


@dataclass
class StreamsResult:
    emitted: list[np.ndarray]          # per stream, n_tokens each
    rounds: int
    accepted: np.ndarray               # per stream: drafts accepted in the rounds it was active
    active_rounds: np.ndarray          # per stream: rounds in which it still emitted tokens
    wall_s: float
    inference_params_dict: object = field(repr=False, default=None)

    @property
    def mean_tau(self) -> np.ndarray:
        """Tokens emitted per active round, per stream."""
        return np.array([len(e) for e in self.emitted]) / np.maximum(self.active_rounds, 1)


class StreamBatch:
    """Device state and host bookkeeping of B streams between rounds."""

    def __init__(self, model, draft, prompts, n_tokens: int, gamma: int, greedy: bool, rngs, *,
                 temperature: float = 1.0, top_k: int | None = 4, max_seqlen: int | None = None):
        prompts = np.asarray(prompts, dtype=np.int64)
        if prompts.ndim != 2:
            raise ValueError("prompts must be [B, L] (every stream the same length)")
        B, L = prompts.shape
        if L < 2:
            raise ValueError(f"prompt length must be >= 2 (the first round needs an anchor), got {L}")
        if len(rngs) != B:
            raise ValueError(f"need one generator per stream: {len(rngs)} for {B} streams")
        if gamma < 1:
            raise ValueError("gamma must be >= 1")
        drafter = getattr(draft, "drafter", None)
        if drafter is None:
            raise ValueError("multi-stream decoding needs the device drafter (NeuralDraftModel)")
        if int(gamma) > draft.gamma:
            raise ValueError(f"decode γ={gamma} > drafter training γ={draft.gamma}")
        self.model, self.draft, self.drafter = model, draft, drafter
        self.B, self.L, self.gamma, self.greedy = B, L, int(gamma), bool(greedy)
        self.n_tokens = int(n_tokens)
        self.rngs = list(rngs)
        self.temperature, self.top_k = float(temperature), top_k
        dev = model.device
        # an active stream gains >= 1 token per round, a finished one consumes 1 position per round
        ms = max_seqlen or L + 2 * self.n_tokens + self.gamma + 2
        self.ip = model.initialize_inference_params(max_seqlen=ms, max_batch=B)
        draft.capture_begin()
        prefill(model, torch.as_tensor(prompts[:, :-1], device=dev), self.ip)
        draft.capture_commit(L - 1)
        self.anchors = torch.as_tensor(prompts[:, -1].copy(), device=dev)
        self.emitted = [[] for _ in range(B)]
        self.accepted = np.zeros(B, dtype=np.int64)
        self.active_rounds = np.zeros(B, dtype=np.int64)
        self.rounds = 0

    @property
    def done(self) -> bool:
        return all(len(e) >= self.n_tokens for e in self.emitted)

    def round(self) -> None:
        """One lockstep round over all B streams."""
        B, g, dev = self.B, self.gamma, self.model.device
        V = self.model.cfg.vocab_size
        u_draft = None
        if not self.greedy:
            u_draft = torch.as_tensor(np.stack([r.random(g) for r in self.rngs]), device=dev)
        toks, q, _, _ = self.drafter.propose(self.ip, self.anchors, g, self.greedy, temperature=self.temperature,
                                             top_k=self.top_k, uniforms=u_draft)
        chunk = torch.cat([self.anchors[:, None], toks], dim=1)
        logits = self.ip.forward(chunk, retain=True)
        states = None
        if self.greedy:
            acc, tv, info = verify_device(logits.double(), None, toks, None, greedy=True)
        else:
            p = transform_rows(logits.reshape(B * (g + 1), V), self.temperature, self.top_k).reshape(B, g + 1, V)
            draws = [draw_uniforms(r, g + 1) for r in self.rngs]
            states = [s for _, s in draws]
            u = torch.as_tensor(np.stack([v for v, _ in draws]), device=dev)
            acc, tv, info = verify_device(p, q, toks, u, greedy=False)
        res = torch.cat([acc.to(torch.int64)[:, None], info.to(torch.int64), tv], dim=1).cpu().numpy()
        j_star = np.zeros(B, dtype=np.int64)
        anchors = np.empty(B, dtype=np.int64)
        for b in range(B):
            k, consumed = int(res[b, 0]), int(res[b, 3])
            tokens = res[b, 4:4 + k + 1]
            if states is not None:
                rewind_uniforms(self.rngs[b], states[b], consumed)
            remaining = self.n_tokens - len(self.emitted[b])
            if remaining > 0:
                take = min(k + 1, remaining)
                self.emitted[b].extend(int(t) for t in tokens[:take])
                self.accepted[b] += take - 1
                self.active_rounds[b] += 1
                j_star[b] = take - 1
                anchors[b] = tokens[take - 1]
            else:
                j_star[b] = 0
                anchors[b] = tokens[0]
        self.ip.rollback(j_star)
        self.anchors = torch.as_tensor(anchors, device=dev)
        self.rounds += 1

    def result(self, wall_s: float = 0.0) -> StreamsResult:
        return StreamsResult([np.asarray(e[: self.n_tokens], dtype=np.int64) for e in self.emitted], self.rounds,
                             self.accepted.copy(), self.active_rounds.copy(), wall_s, self.ip)


def speculative_generate_streams(model, draft, prompts, n_tokens: int, gamma: int, greedy: bool, rngs, *,
                                 temperature: float = 1.0, top_k: int | None = 4,
                                 max_seqlen: int | None = None) -> StreamsResult:
    """Decode B streams of ``n_tokens`` each in lockstep batched rounds (see the module doc)."""
    sb = StreamBatch(model, draft, prompts, n_tokens, gamma, greedy, rngs, temperature=temperature, top_k=top_k,
                     max_seqlen=max_seqlen)
    t0 = time.perf_counter()
    while not sb.done:
        sb.round()
    if model.device.type == "cuda":
        torch.cuda.synchronize(model.device)
    return sb.result(time.perf_counter() - t0)


__all__ = ["StreamBatch", "StreamsResult", "speculative_generate_streams"]
