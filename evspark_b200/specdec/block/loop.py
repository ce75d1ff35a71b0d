"""End-to-end speculative loop on the device path (mirror of evspark/specdec/block/loop.py).

Anchor protocol (loop.py:1-19): the prompt's first L-1 tokens are prefilled, the last one is the
anchor y; each round drafts γ tokens, verifies the chunk ``[y, x_1..x_γ]`` in one retained block
forward (row i of the logits is p_{i+1}), accepts ``k`` drafts, emits ``k+1`` tokens, and rolls
the state back to block index ``j* = take-1`` (skipped when all drafts are accepted and the round
is not truncated).  The new anchor is the last emitted token.

Per round on the device: drafting (neural drafter: one ``evs_draft_propose``), the block forward
(``evs_forward``), the transform of the γ+1 target rows and verification (``evs_transform`` +
``evs_verify``, fp64), and rollback (``evs_rollback``, zero data movement).  The host sees only
the accepted length and tokens (one small copy per round).  The numpy generator advances exactly
as in the reference: γ uniforms for sampled drafting, then the verifier's own draws.
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field

import numpy as np
import torch

from evspark_b200 import _native as N
from evspark_b200.specdec.block.driver import block_forward, prefill, step_forward_reference
from evspark_b200.specdec.block.slice import slice_states_to_accept
from evspark_b200.specdec.transforms import apply_transform, transform_rows
from evspark_b200.specdec.verifier import (draw_uniforms, rewind_uniforms, sample_categorical, verify_device,
                                           verify_device_multicand)

VOCAB_SIZE = 512
# tokens per forward when a prompt is prefilled: the whole prompt up to this many per forward
# (chunking does not change any result bit; fewer forwards stream the weights fewer times)
PREFILL_CHUNK_MAX = 1024


def _prefill_chunk(model, L: int) -> int:
    return int(min(PREFILL_CHUNK_MAX, max(int(model.max_chunk), int(L))))


@dataclass
class RoundLog:
    k: int
    replay_len: int
    t_draft: float
    t_block: float
    t_verify: float
    t_restore_replay: float
    from_residual: bool = False
    fallback: bool = False
    n_emitted: int = 0
    t_snapshot: float = 0.0
    t_slice: float = 0.0
    conf: list[float] | None = None
    n_candidates: int = 1
    winner: int = 0


@dataclass
class SpecGenerateResult:
    emitted_ids: np.ndarray
    rounds_log: list[RoundLog]
    inference_params_dict: object = field(repr=False)
    anchor: int = -1
    emitted_logits: np.ndarray | None = None
    rollback: str = "slice"

    def __iter__(self):
        yield self.emitted_ids
        yield self.rounds_log


def _as_prompt_ids(prompt_ids, device) -> torch.Tensor:
    t = torch.as_tensor(prompt_ids).long()
    if t.ndim == 1:
        t = t[None]
    if t.ndim != 2 or t.shape[0] != 1:
        raise ValueError(f"prompt_ids must be [1, L] (independent streams use the batched API), got {tuple(t.shape)}")
    return t.to(device)


def _prompt_host(prompt_ids) -> np.ndarray:
    """The prompt's ids on the host (read back from the device only when given there)."""
    if isinstance(prompt_ids, torch.Tensor) and prompt_ids.device.type != "cpu":
        out = prompt_ids.reshape(-1).cpu().numpy().astype(np.int64)
        N.note_transfer(d2h=out.nbytes)
        return out
    return np.asarray(prompt_ids, dtype=np.int64).reshape(-1)


def _q_prime_from_raw(q: np.ndarray, temperature: float, top_k: int | None) -> np.ndarray:
    """Draft distribution -> the target's sampling transform applied to log(q) (loop.py:111-128)."""
    q = np.asarray(q, dtype=np.float64).ravel()
    lg = np.full(q.shape[0], -np.inf)
    pos = q > 0.0
    if np.any(pos):
        lg[pos] = np.log(q[pos])
    else:
        lg[:] = 0.0
    return apply_transform(lg, temperature=temperature, top_k=top_k)


def _propose_draft(draft, prefix: np.ndarray, gamma: int, greedy: bool, rng, *, temperature=1.0, top_k=4):
    """``probs(prefix)`` drafters (identity, lookup, Markov): token by token (loop.py:131-162)."""
    toks = np.empty(gamma, dtype=np.int64)
    rows = np.empty((gamma, VOCAB_SIZE), dtype=np.float64)
    buf = list(np.asarray(prefix, dtype=np.int64))
    for i in range(gamma):
        q = np.asarray(draft.probs(np.asarray(buf, dtype=np.int64)), dtype=np.float64).ravel()
        if q.shape[0] != VOCAB_SIZE:
            raise ValueError(f"draft.probs must return [{VOCAB_SIZE}], got {q.shape}")
        if not greedy:
            q = _q_prime_from_raw(q, temperature, top_k)
        rows[i] = q
        t = int(np.argmax(q)) if greedy else sample_categorical(q, rng)
        toks[i] = t
        buf.append(t)
    return toks, rows


def _sync(device) -> None:
    torch.cuda.synchronize(device)


@dataclass
class RoundOutcome:
    taken: np.ndarray
    log: RoundLog
    ip: object
    logits_rows: list = field(default_factory=list)


class _RoundBuffers:
    """Pinned host staging and device buffers of the device round, kept with the state."""

    def __init__(self, device, gamma: int):
        self.gamma = gamma
        # one device buffer [draft uniforms (γ fp64) | anchor | draft tokens (γ)]: the chunk the
        # verify forward reads is its last γ+1 slots, so one host copy of the first γ+1 slots sends a
        # round's uniforms and anchor, and the drafter writes its tokens straight into the chunk
        self.stage = torch.empty(2 * gamma + 1, dtype=torch.int64, device=device)
        self.stage_h = torch.empty(gamma + 1, dtype=torch.int64, pin_memory=True)
        self.chunk = self.stage[gamma:].view(1, gamma + 1)
        self.u_draft = self.stage[:gamma].view(torch.float64)
        self.u_draft_h = self.stage_h[:gamma].view(torch.float64)
        self.u_ver_h = torch.empty(gamma + 1, dtype=torch.float64, pin_memory=True)
        self.u_ver = torch.empty(gamma + 1, dtype=torch.float64, device=device)
        # the round's results in one device buffer read back by one copy, in 8-byte slots:
        # [accepted (int32) | from_residual, fallback, consumed (int32) | γ+1 tokens | γ confidences (fp32)]
        self.res = torch.empty(4 + gamma + (gamma + 1) // 2, dtype=torch.int64, device=device)
        self.res_h = torch.empty(self.res.numel(), dtype=torch.int64, pin_memory=True)
        self.acc = self.res[0:1].view(torch.int32)[:1]
        self.info = self.res[1:3].view(torch.int32)[:3].view(1, 3)
        self.toks_v = self.res[3:4 + gamma].view(1, gamma + 1)
        self.conf_all = self.res[4 + gamma:].view(torch.float32)[:gamma].view(1, gamma)
        # drafter outputs of the round, and the drafter call captured as a CUDA graph per
        # (state, sampling settings): the same launches, issued by one graph launch
        self.toks = self.q = self.conf = None
        self.draft_graphs: dict = {}


def _spec_round_device(model, draft, ip, y: int, gamma: int, greedy: bool, rng, remaining: int, temperature,
                       top_k) -> RoundOutcome:
    """The round of ``spec_round`` with the device drafter and slice rollback, with one host
    synchronisation: the uniforms go through pinned buffers without waiting, and the rollback takes
    its block index j* = min(k, remaining - 1) straight from the device verification, so the host
    waits only for the small result copy (same RNG order, tokens and state as the general path)."""
    bufs = getattr(ip, "_round_bufs", None)
    if bufs is None or bufs.gamma != gamma:
        bufs = ip._round_bufs = _RoundBuffers(model.device, gamma)
    draft._check_gamma(gamma)
    chunk = bufs.chunk
    # the anchor (and, sampling, the drafter's uniforms before it) in one copy from pinned memory
    bufs.stage_h.numpy()[gamma] = int(y)
    u = None
    if greedy:
        bufs.stage[gamma:gamma + 1].copy_(bufs.stage_h[gamma:], non_blocking=True)
        h2d = chunk.element_size()
    else:
        bufs.u_draft_h.numpy()[:] = rng.random(int(gamma))
        bufs.stage[:gamma + 1].copy_(bufs.stage_h, non_blocking=True)
        h2d = bufs.stage_h.nbytes
        u = bufs.u_draft[None]
    dr = draft.drafter
    if bufs.toks is None:
        V = dr.cfg.vocab_size
        bufs.toks = chunk[:, 1:]  # the drafter's tokens land in the verify chunk
        bufs.q = torch.empty(1, gamma, V, dtype=torch.float64, device=model.device)
        bufs.conf = bufs.conf_all  # the drafter's confidences land in the result buffer
    key = (ip.handle.value, dr._h.value, bool(greedy), float(temperature), None if top_k is None else int(top_k))
    entry = bufs.draft_graphs.get(key)
    call = lambda: dr.propose_into(ip, chunk[:, 0], int(gamma), greedy, bufs.toks, bufs.q, bufs.conf,
                                   temperature=temperature, top_k=top_k, uniforms=u)
    if entry is None:
        call()  # this round's draft; then the same call is captured for the next rounds
        graph = torch.cuda.CUDAGraph()
        n0 = N.launch_count()
        with torch.cuda.graph(graph):
            call()
        n_calls = N.launch_count() - n0
        N.note_replayed(-n_calls)  # capturing issues nothing
        bufs.draft_graphs[key] = (graph, n_calls)
    else:
        graph, n_calls = entry
        graph.replay()
        N.note_replayed(n_calls)
    q_rows = bufs.q
    draft.capture_begin()
    logits = ip.forward(chunk, retain=True)
    x = chunk[:, 1:]
    state = None
    out = (bufs.acc, bufs.toks_v, bufs.info)
    if greedy:
        verify_device(logits.double(), None, x, None, greedy=True, out=out)
    else:
        p = transform_rows(logits[0], temperature, top_k)[None]
        uv, state = draw_uniforms(rng, gamma + 1)
        bufs.u_ver_h.numpy()[:] = uv
        bufs.u_ver.copy_(bufs.u_ver_h, non_blocking=True)
        h2d += bufs.u_ver_h.nbytes
        verify_device(p, q_rows, x, bufs.u_ver[None], greedy=False, out=out)
    # j* = min(k, remaining - 1); k <= γ, so the clamp only matters near the end of a generation
    ip.rollback_launch(bufs.acc if int(remaining) - 1 >= gamma else torch.clamp(bufs.acc, max=int(remaining) - 1))
    bufs.res_h.copy_(bufs.res, non_blocking=True)
    N.note_transfer(h2d=h2d, d2h=bufs.res_h.nbytes)
    torch.cuda.current_stream(model.device).synchronize()
    res = bufs.res_h.numpy()
    k = int(res[:1].view(np.int32)[0])
    info = res[1:3].view(np.int32)
    from_residual, fallback, consumed = bool(info[0]), bool(info[1]), int(info[2])
    tokens = res[3:3 + k + 1].copy()
    if state is not None:
        rewind_uniforms(rng, state, consumed)
    take = min(k + 1, remaining)
    j_star = take - 1
    ip.note_rollback([j_star])
    draft.capture_commit(j_star + 1)
    log = RoundLog(k=k, replay_len=0, t_draft=0.0, t_block=0.0, t_verify=0.0, t_restore_replay=0.0,
                   from_residual=from_residual, fallback=fallback, n_emitted=take,
                   conf=res[4 + gamma:].view(np.float32)[:gamma].tolist())
    return RoundOutcome(taken=tokens[:take].astype(np.int64), log=log, ip=ip)


def spec_round(model, draft, ip, y: int, gamma: int, greedy: bool, rng: np.random.Generator, remaining: int, *,
               seen: np.ndarray | None = None, temperature: float = 1.0, top_k: int | None = 4,
               rollback: str = "slice", timing: bool = True, record_logits: bool = False,
               chunk: torch.Tensor | None = None) -> RoundOutcome:
    """One round of the anchor loop from state ``ip`` with anchor ``y``: draft, retained block
    forward, device verification, rollback to j* = take-1, capture commit (loop.py:381-570)."""
    device = model.device
    has_device_draft = hasattr(draft, "propose_device")
    has_propose = hasattr(draft, "propose_block")
    has_capture = hasattr(draft, "capture_begin")
    if has_device_draft and rollback == "slice" and not timing and not record_logits and hasattr(draft, "drafter"):
        return _spec_round_device(model, draft, ip, y, gamma, greedy, rng, remaining, temperature, top_k)
    if chunk is None:
        chunk = torch.empty(1, gamma + 1, dtype=torch.int64, device=device)
    snap = None
    t_snapshot = 0.0
    if rollback == "snapshot":
        t0 = time.perf_counter()
        snap = ip.clone()
        if timing:
            _sync(device)
        t_snapshot = time.perf_counter() - t0
    # ---- draft ----
    t0 = time.perf_counter()
    conf_rows = None
    conf_d = None
    chunk[0, 0] = y
    if has_device_draft:
        toks_d, q_rows, conf_d = draft.propose_device(chunk[:, 0], gamma, greedy, rng, temperature=temperature,
                                                      top_k=top_k, inference_params_dict=ip)
        chunk[0, 1:] = toks_d[0]
    else:
        if has_propose:
            toks, q_np, conf_rows = draft.propose_block(y, gamma, greedy, rng, temperature=temperature,
                                                        top_k=top_k, inference_params_dict=ip)
        else:
            toks, q_np = _propose_draft(draft, seen, gamma, greedy, rng, temperature=temperature, top_k=top_k)
        chunk[0, 1:] = torch.as_tensor(np.asarray(toks, dtype=np.int64), device=device)
        q_rows = torch.as_tensor(np.ascontiguousarray(q_np), device=device)[None]
    if timing:
        _sync(device)
    t_draft = time.perf_counter() - t0
    # ---- block verify forward ----
    if has_capture:
        draft.capture_begin()
    t0 = time.perf_counter()
    logits, stash = block_forward(model, chunk, ip, retain=True)
    if timing:
        _sync(device)
    t_block = time.perf_counter() - t0
    # ---- verification (device, fp64) ----
    t0 = time.perf_counter()
    x = chunk[:, 1:]
    state = None
    if greedy:
        acc, toks_v, info = verify_device(logits.double(), None, x, None, greedy=True)
    else:
        p = transform_rows(logits[0], temperature, top_k)[None]
        uv, state = draw_uniforms(rng, gamma + 1)
        acc, toks_v, info = verify_device(p, q_rows, x, torch.as_tensor(uv, device=device)[None], greedy=False)
    res = torch.cat([acc.to(torch.int64), info[0].to(torch.int64), toks_v[0]]).cpu().numpy()
    k = int(res[0])
    from_residual, fallback, consumed = bool(res[1]), bool(res[2]), int(res[3])
    tokens = res[4:4 + k + 1]
    if state is not None:
        rewind_uniforms(rng, state, consumed)
    t_verify = time.perf_counter() - t0
    take = min(k + 1, remaining)
    taken = tokens[:take].astype(np.int64)
    j_star = take - 1
    full_accept_kept = (k == gamma) and (take == k + 1)
    replay_len = 0
    t_restore = t_snapshot
    t_slice = 0.0
    if not full_accept_kept:
        if rollback == "snapshot":
            t0 = time.perf_counter()
            ip.close()
            ip = snap
            snap = None
            consume = np.concatenate([[y], taken[:-1]]) if take > 1 else np.array([y])
            replay_len = len(consume)
            block_forward(model, torch.as_tensor(consume, device=device)[None], ip)
            if timing:
                _sync(device)
            t_restore = t_snapshot + (time.perf_counter() - t0)
        else:
            t0 = time.perf_counter()
            slice_states_to_accept(ip, stash, j_star)
            if timing:
                _sync(device)
            t_slice = time.perf_counter() - t0
    if snap is not None:
        snap.close()
    if has_capture:
        draft.capture_commit(j_star + 1)
    rows = []
    if record_logits:
        lg = logits[0].double().cpu().numpy()
        rows = [lg[i] for i in range(take)]
    if conf_d is not None:
        conf_rows = conf_d[0].double().cpu().numpy()
    log = RoundLog(k=k, replay_len=replay_len, t_draft=t_draft, t_block=t_block, t_verify=t_verify,
                   t_restore_replay=t_restore, from_residual=from_residual, fallback=fallback, n_emitted=take,
                   t_snapshot=t_snapshot, t_slice=t_slice,
                   conf=None if conf_rows is None else [float(c) for c in conf_rows])
    return RoundOutcome(taken=taken, log=log, ip=ip, logits_rows=rows)


def spec_round_multi(model, draft, ip, y: int, gamma: int, greedy: bool, rng: np.random.Generator, remaining: int,
                     n_candidates: int, *, seen: np.ndarray | None = None, temperature: float = 1.0,
                     top_k: int | None = 4, record_logits: bool = False) -> RoundOutcome:
    """One SpecInfer round with ``n_candidates`` drafts (loop.py:396-525): B drafts from anchor y, the
    state expanded to B rows, one retained block forward of [B, γ+1], multi-candidate verification
    on the device, rollback of every row to j* and collapse onto the winning row."""
    device = model.device
    B = int(n_candidates)
    V = model.cfg.vocab_size
    t0 = time.perf_counter()
    ip.expand(B)
    if hasattr(draft, "propose_blocks_device"):
        toks_d, q_d, conf_d = draft.propose_blocks_device(y, gamma, greedy, rng, B, temperature=temperature,
                                                          top_k=top_k, inference_params_dict=ip)
    else:
        rows = [_propose_draft(draft, seen, gamma, greedy, rng, temperature=temperature, top_k=top_k)
                for _ in range(B)]
        toks_d = torch.as_tensor(np.stack([t for t, _ in rows]), device=device)
        q_d = torch.as_tensor(np.stack([q for _, q in rows]), device=device)
        conf_d = None
    t_draft = time.perf_counter() - t0
    chunk = torch.cat([torch.full((B, 1), int(y), dtype=torch.int64, device=device), toks_d], dim=1)
    if hasattr(draft, "capture_begin"):
        draft.capture_begin()
    t0 = time.perf_counter()
    logits, stash = block_forward(model, chunk, ip, retain=True)
    t_block = time.perf_counter() - t0
    t0 = time.perf_counter()
    state = None
    if greedy:
        tv, info = verify_device_multicand(logits.double(), None, toks_d, None, greedy=True)
    else:
        p = transform_rows(logits.reshape(B * (gamma + 1), V), temperature, top_k).reshape(B, gamma + 1, V)
        uv, state = draw_uniforms(rng, gamma * B + 1)
        tv, info = verify_device_multicand(p, q_d, toks_d, torch.as_tensor(uv, device=device), greedy=False)
    res = torch.cat([info.to(torch.int64), tv]).cpu().numpy()
    k, from_residual, fallback, consumed, winner = (int(v) for v in res[:5])
    tokens = res[5:5 + k + 1]
    if state is not None:
        rewind_uniforms(rng, state, consumed)
    t_verify = time.perf_counter() - t0
    take = min(k + 1, remaining)
    taken = tokens[:take].astype(np.int64)
    j_star = take - 1
    t0 = time.perf_counter()
    if not (k == gamma and take == k + 1):
        slice_states_to_accept(ip, stash, j_star)
    ip.collapse(winner)
    t_slice = time.perf_counter() - t0
    if hasattr(draft, "capture_commit"):
        draft.capture_commit(j_star + 1, batch_idx=winner)
    rows_out = []
    if record_logits:
        lg = logits[winner].double().cpu().numpy()
        rows_out = [lg[i] for i in range(take)]
    conf = None if conf_d is None else [float(c) for c in conf_d[winner].double().cpu().numpy()]
    log = RoundLog(k=k, replay_len=0, t_draft=t_draft, t_block=t_block, t_verify=t_verify, t_restore_replay=0.0,
                   from_residual=bool(from_residual), fallback=bool(fallback), n_emitted=take, t_slice=t_slice,
                   conf=conf, n_candidates=B, winner=winner)
    return RoundOutcome(taken=taken, log=log, ip=ip, logits_rows=rows_out)


def speculative_generate(model, draft, prompt_ids, n_tokens: int, gamma: int, greedy: bool,
                         rng: np.random.Generator, *, temperature: float = 1.0, top_k: int | None = 4,
                         inference_params_dict=None, record_logits: bool = False, rollback: str = "slice",
                         n_candidates: int = 1, timing: bool = True) -> SpecGenerateResult:
    device = model.device
    pt = torch.as_tensor(prompt_ids)
    if not (pt.ndim == 1 or (pt.ndim == 2 and pt.shape[0] == 1)):
        raise ValueError(f"prompt_ids must be [1, L] (independent streams use the batched API), got {tuple(pt.shape)}")
    n_candidates = int(n_candidates)
    if n_candidates < 1:
        raise ValueError(f"n_candidates must be >= 1, got {n_candidates}")
    if n_candidates > 1 and rollback != "slice":
        raise ValueError("n_candidates > 1 needs rollback='slice' (the winner row is sliced at j*)")
    if n_tokens < 0:
        raise ValueError("n_tokens must be >= 0")
    if gamma < 1:
        raise ValueError("gamma must be >= 1")
    if rollback not in ("slice", "snapshot"):
        raise ValueError(f"rollback must be 'slice' or 'snapshot', got {rollback!r}")
    has_device_draft = hasattr(draft, "propose_device")
    has_propose = hasattr(draft, "propose_block")
    has_capture = hasattr(draft, "capture_begin")
    if has_capture and rollback != "slice":
        raise ValueError("the neural drafter needs rollback='slice' (rejected positions are trimmed at j*)")
    if has_device_draft and int(gamma) > draft.gamma:
        raise ValueError(f"decode γ={gamma} > drafter training γ={draft.gamma}")
    prompt_np = _prompt_host(prompt_ids)
    L = int(prompt_np.shape[0])
    if L < 2:
        raise ValueError(f"prompt length must be >= 2 (the first round needs an anchor), got {L}")
    y = int(prompt_np[-1])
    if n_tokens == 0:
        ip = inference_params_dict or model.initialize_inference_params(max_seqlen=L + gamma + 2)
        return SpecGenerateResult(np.empty(0, dtype=np.int64), [], ip, anchor=y, rollback=rollback)
    seen = prompt_np.copy()
    if inference_params_dict is None:
        ip = model.initialize_inference_params(max_seqlen=L + n_tokens + gamma + 2, max_batch=n_candidates,
                                               max_chunk=_prefill_chunk(model, L))
        if has_capture:
            draft.capture_begin()
        prompt = _as_prompt_ids(prompt_ids, device)
        prefill(model, prompt[:, :-1], ip)
        if has_capture:
            draft.capture_commit(L - 1)
    else:
        ip = inference_params_dict
        if ip.max_batch < n_candidates:
            raise ValueError(f"inference state max_batch={ip.max_batch} < n_candidates={n_candidates}: create the "
                             "state with a larger max_batch")
        if has_capture and int(draft.capture_buffer_len()) != L - 1:
            raise ValueError(f"external state: the drafter's H_ctx buffer is not aligned (对齐): consumed "
                             f"{draft.capture_buffer_len()} != L-1={L - 1}")
    emitted: list[int] = []
    rounds: list[RoundLog] = []
    logit_rows: list[np.ndarray] = []
    chunk = torch.empty(1, gamma + 1, dtype=torch.int64, device=device)
    while len(emitted) < n_tokens:
        if n_candidates > 1:
            out = spec_round_multi(model, draft, ip, y, gamma, greedy, rng, n_tokens - len(emitted), n_candidates,
                                   seen=seen, temperature=temperature, top_k=top_k, record_logits=record_logits)
        else:
            out = spec_round(model, draft, ip, y, gamma, greedy, rng, n_tokens - len(emitted), seen=seen,
                             temperature=temperature, top_k=top_k, rollback=rollback, timing=timing,
                             record_logits=record_logits, chunk=chunk)
        ip = out.ip
        if record_logits:
            logit_rows.extend(out.logits_rows)
        emitted.extend(int(t) for t in out.taken)
        seen = np.concatenate([seen, out.taken])
        y = int(out.taken[-1])
        rounds.append(out.log)
    out_logits = np.stack(logit_rows[:n_tokens]) if record_logits else None
    return SpecGenerateResult(np.asarray(emitted[:n_tokens], dtype=np.int64), rounds, ip, anchor=y,
                              emitted_logits=out_logits, rollback=rollback)


def native_greedy_reference(model, prompt_ids, n_tokens: int, *, record_logits: bool = False):
    """Token-by-token argmax (lowest index on ties) on the same kernels (loop.py:584-624)."""
    device = model.device
    prompt = _as_prompt_ids(prompt_ids, device)
    if n_tokens < 0:
        raise ValueError("n_tokens must be >= 0")
    L = int(prompt.shape[1])
    ip = model.initialize_inference_params(max_seqlen=L + max(n_tokens, 0) + 2, max_chunk=_prefill_chunk(model, L))
    if n_tokens == 0:
        return np.empty(0, dtype=np.int64), ip, None
    last = prefill(model, prompt, ip)[0, -1]
    emitted = np.empty(n_tokens, dtype=np.int64)
    rows = []
    x = torch.empty(1, 1, dtype=torch.int64, device=device)
    for i in range(n_tokens):
        lg = last.double().cpu().numpy()
        if record_logits:
            rows.append(lg)
        tok = int(np.argmax(lg))
        emitted[i] = tok
        if i + 1 < n_tokens:
            x[0, 0] = tok
            last = step_forward_reference(model, x, ip)[0, -1]
    return emitted, ip, (np.stack(rows) if record_logits else None)


def native_sample_reference(model, prompt_ids, n_tokens: int, rng: np.random.Generator, *,
                            temperature: float = 1.0, top_k: int | None = 4) -> np.ndarray:
    """Token-by-token sampling with the shared transform (loop.py:627-658)."""
    device = model.device
    prompt = _as_prompt_ids(prompt_ids, device)
    if n_tokens < 0:
        raise ValueError("n_tokens must be >= 0")
    if n_tokens == 0:
        return np.empty(0, dtype=np.int64)
    L = int(prompt.shape[1])
    ip = model.initialize_inference_params(max_seqlen=L + n_tokens + 2, max_chunk=_prefill_chunk(model, L))
    last = prefill(model, prompt, ip)[0, -1]
    emitted = np.empty(n_tokens, dtype=np.int64)
    x = torch.empty(1, 1, dtype=torch.int64, device=device)

    for i in range(n_tokens):
        probs = transform_rows(last[None], temperature, top_k)
        u = torch.tensor([float(rng.random())], dtype=torch.float64, device=device)
        out = torch.empty(1, dtype=torch.int64, device=device)
        N.check(N.lib().evs_sample(probs.data_ptr(), 1, probs.shape[1], u.data_ptr(), out.data_ptr(),
                                   N.stream_ptr()), "evs_sample")
        tok = int(out.item())
        emitted[i] = tok
        if i + 1 < n_tokens:
            x[0, 0] = tok
            last = step_forward_reference(model, x, ip)[0, -1]
    ip.close()
    return emitted


def teacher_force_to_spec_state(model, prompt_ids, emitted_ids, *, max_seqlen: int | None = None):
    """Prefill the prompt, then step ``emitted[:-1]`` (loop.py:661-685)."""
    prompt = _as_prompt_ids(prompt_ids, model.device)
    emitted = np.asarray(emitted_ids, dtype=np.int64).ravel()
    L, n = int(prompt.shape[1]), int(emitted.size)
    ip = model.initialize_inference_params(max_seqlen=max_seqlen or L + n + 2)
    prefill(model, prompt, ip)
    if n > 1:
        step_forward_reference(model, torch.as_tensor(emitted[:-1], device=model.device)[None], ip)
    return ip


def spec_end_kv_len(prompt_len: int, n_emitted: int) -> int:
    return int(prompt_len) + int(n_emitted) - 1


__all__ = ["RoundLog", "RoundOutcome", "SpecGenerateResult", "spec_round", "spec_round_multi", "native_greedy_reference", "native_sample_reference",
           "spec_end_kv_len", "speculative_generate", "teacher_force_to_spec_state"]
