"""Benchmark: accepted tok/s of single-stream speculative decoding on an Evo2-7B-shaped model.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A *step* is one speculative round of the hot path on one stream: the γ-parallel neural drafter
(γ=12, d=1024, context from block 27), the retained γ+1-token verify forward through the 32
StripedHyena2 blocks (Hyena SE/MR/LI + MHA every 8th block, d=4096, bf16), the device transform
and Leviathan verification (T=1.0, top_k=4), and the replay-free rollback.  The prompt is a
1024-token seeded order-3 Markov ACGT sequence (GC≈0.5); weights are seeded random-init.

``value`` = accepted tokens / device time over K rounds (CUDA events, inputs resident in HBM; the
12.95 GB of weights streamed every round are far larger than L2).  ``e2e`` = the same metric
through the public API (``EvSpark.generate`` on a host prompt string, prefill included, tokens
read back to the host).  ``roofline`` is the dominant kernel group (the tcgen05 projections,
HBM-bound weight streaming) timed with CUDA events inside the library over the timed region.
``cpu_baseline`` times the CPU port of the reference path (``oracle/``) on a bounded sample.

Multi-GPU (torchrun, one process per GPU): every rank decodes its own independent stream
(different prompt seed) with no collectives; the timing is the max over ranks (weak scaling).

``--config evo2_40b`` on N > 1 GPUs (or ``--tp``) shards the target by channels over the N GPUs:
every rank runs the same single stream on its share of the Hyena channels, heads and MLP
features, and the row-parallel partial sums are added across ranks over NVLink inside the
residual RMSNorm; ``value`` = that one stream's accepted tok/s (strong scaling).

``--streams S`` switches to multi-stream decoding: every rank decodes S independent streams
(per-stream prompt and generator seeds) in lockstep batched rounds, one verify forward of
M = 13·S token rows per round; ``value`` = tokens emitted by all streams of all ranks / the
slowest rank's device time.
"""

from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "accepted tok/s single-stream Evo2-7B-shape γ=12; verify-block µs; HBM GB/s"
GAMMA = 12
PROMPT_LEN = 1024
# ncu dram__bytes_read.sum + dram__bytes_write.sum of the tcgen05 projections of one block (in-, out-,
# w1/w2 and w3 projections) of the 4-block 7B-width model, which has the 32-block model's projection
# shapes: 403.8 MB of DRAM traffic for 414.0 MB of algorithmic bytes (weights + activations + fp32
# partials, which stay in L2).  The per-launch traffic below is this measured ratio times the run's
# per-launch algorithmic bytes (the same launch mix per block).
GEMM_TRAFFIC_RATIO = 403.8 / 414.0
GEMM_TRAFFIC_NOTE = ("ncu DRAM bytes of one block's projections on the 4-block 7B-width model (same shapes), "
                     "403.8 MB per 414.0 MB algorithmic; scaled to this run's bytes per launch")
E2E_TOKENS = 1024
VERIFY_REPS = 200


def peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks + throttle reasons sampled every 200 ms during the timed region."""

    def __init__(self, index: int):
        self.path = Path(f"/tmp/evs_clocks_{os.getpid()}.csv")
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.f = open(self.path, "w")
            self.p = subprocess.Popen(["nvidia-smi", f"--id={index}", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                       "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.p = None

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.p.terminate()
        self.p.wait()
        self.f.close()
        rows = [r.split(",") for r in self.path.read_text().strip().splitlines() if r.count(",") >= 8]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip().lower() == "active"})
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": float(rows[0][2]), "reasons": reasons,
                "samples": len(rows), "power_w_max": max(float(r[3]) for r in rows)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def _cpu_target_weights(cfg, seed: int) -> dict:
    """The GPU arm's seeded weights drawn on the host, each GEMM weight rounded to bf16 and held in
    fp32 (the bf16-emulating port computes in fp32), one tensor at a time."""
    import torch

    from evspark_b200.weights import _draw, data_dtype, target_weight_specs

    from concurrent.futures import ThreadPoolExecutor

    def one(item):
        idx, (name, shape, kind, storage) = item
        gen = torch.Generator()
        gen.manual_seed(int(seed) * 1_000_003 + idx)
        t = _draw(kind, shape, gen, "cpu", cfg)
        return name, (t.to(data_dtype(cfg)) if storage == "data" else t).to(torch.float32).contiguous()

    # every tensor has its own generator, so drawing them on several threads gives the same bits
    with ThreadPoolExecutor(max_workers=max(1, (os.cpu_count() or 1))) as ex:
        return dict(ex.map(one, enumerate(target_weight_specs(cfg))))


def cpu_reference_rounds(n_threads: int, steps: int, warmup: int, *, sampled: bool = False,
                         prompt_len: int = PROMPT_LEN, synthetic_context: int = 0) -> dict:
    """The reference path on the host cores (the CPU port in ``oracle/``), timed round by round.

    Workload: the GPU arm's own (1024-token order-3 Markov prompt, Evo2-7B shape, 32 blocks, bf16
    rounding points, fp32 arithmetic; neural drafter d=1024 from block 27; gamma=12, T=1.0,
    top_k=4; fp64 transform + verification; slice rollback).  ``warmup`` untimed rounds, then
    ``steps`` timed rounds; ``ms_per_step`` is their mean and ``value`` = tokens emitted / timed
    seconds, so ``ms_per_step * steps`` is the timed region.  With ``sampled`` (a bounded sample), or
    when the host has too little free memory for the 26 GB of fp32 weights, four 7B-width blocks
    (SE, MR, LI, MHA) run instead and ``value`` is scaled from their measured time to 32 blocks
    (reported as separate fields).  ``synthetic_context`` = L > 0 replaces the prefill (infeasible on
    the host at long context) by a synthetically filled state of L consumed tokens: random KV rows,
    FIR histories and IIR states of the right sizes, and random drafter context rows."""
    import torch

    from evspark_b200.config import DRAFTERS, EVO2_7B, EVO2_7B_SLICE
    from evspark_b200.weights import init_drafter_weights
    from evspark_b200.workload import markov_prompt
    from oracle import specdec as sd
    from oracle.model import OracleTarget

    torch.set_num_threads(n_threads)
    try:
        import psutil

        avail = psutil.virtual_memory().available
    except Exception:  # noqa: BLE001
        avail = 0
    full = avail > 48 * 2**30 and not sampled
    cfg = EVO2_7B if full else EVO2_7B_SLICE
    inject = 27 if full else 2
    t_init = time.perf_counter()
    w = _cpu_target_weights(cfg, 20260820)
    o = OracleTarget(cfg, w, compute=torch.float32, emulate=True)
    dcfg = DRAFTERS["evo2_7b"]
    dw = init_drafter_weights(dcfg, seed=20260830, embed=w["embed"])
    init_s = time.perf_counter() - t_init
    rng = np.random.default_rng(7)
    rounds = warmup + steps
    if synthetic_context:
        L = int(synthetic_context)
        st = o.init_state(1, L + (rounds + 2) * (GAMMA + 1))
        t0 = time.perf_counter()
        g = torch.Generator().manual_seed(5)
        for i in st.kv:
            st.kv[i][:, :L].normal_(generator=g)
        K0, S = cfg.short_filter_length, cfg.state_size
        for i in st.outer:
            st.outer[i] = torch.randn(1, 3 * cfg.d_model, K0 - 1, generator=g)
        for i in st.inner:
            st.inner[i] = torch.randn(1, cfg.d_model, cfg.filter_length(cfg.layer_types[i]) - 1, generator=g)
        for i in st.iir:
            st.iir[i] = torch.randn(1, cfg.d_model, S, generator=g)
        st.lengths[:] = L
        ctx = torch.randn(dcfg.ctx_window, cfg.d_model, generator=g)
        prefill_s = time.perf_counter() - t0
        y = 71
    else:
        prompt = markov_prompt(prompt_len, seed=20260821)
        st = o.init_state(1, prompt_len + (rounds + 2) * (GAMMA + 1))
        t0 = time.perf_counter()
        with torch.no_grad():
            _, _, cap = o.forward(prompt[None, :-1], st, prefill=True, capture_layers=(inject,))
        prefill_s = time.perf_counter() - t0
        ctx = cap[inject][0][-dcfg.ctx_window:].float()
        y = int(prompt[-1])
    times, scaled, emitted = [], [], []
    for r in range(rounds):
        t0 = time.perf_counter()
        with torch.no_grad():
            U, h = sd.drafter_trunk(dw, dcfg, y, ctx, int(ctx.shape[0]))
            toks, q, _ = sd.drafter_serial(dw, U, h, y, False, rng)
            t1 = time.perf_counter()
            lg, stash, capr = o.forward(np.concatenate([[y], toks])[None], st, retain=True, capture_layers=(inject,))
            t2 = time.perf_counter()
        p = np.stack([sd.apply_transform(row, 1.0, 4) for row in lg[0].double().numpy()])
        res = sd.verify_round(toks, q, p, rng)
        k = int(res.accepted_len)
        o.slice(st, stash, k)
        ctx = torch.cat([ctx, capr[inject][0][: k + 1].float()])[-dcfg.ctx_window:]
        y = int(res.tokens[-1])
        t3 = time.perf_counter()
        times.append(t3 - t0)
        scaled.append((t1 - t0) + (t2 - t1) * (32 / cfg.n_layers) + (t3 - t2))
        emitted.append(k + 1)
    t_timed = float(sum(times[warmup:]))
    tokens = float(sum(emitted[warmup:]))
    out = {"cores": n_threads, "init_s": round(init_s, 1), "prefill_s": round(prefill_s, 2),
           "ms_per_step": t_timed / steps * 1e3, "timed_s": t_timed, "tokens": tokens,
           "blocks_run": cfg.n_layers}
    if full:
        out["value"] = tokens / t_timed
        out["sample"] = (f"{steps} timed rounds (after {warmup} untimed) of the full Evo2-7B-shaped round on the "
                         f"host: neural drafter + 13-token verify through 32 blocks + fp64 verify + slice rollback, "
                         f"after a {prompt_len - 1}-token prefill; tau from the random-init drafter")
    else:
        # the 32-block round from the 4 measured blocks: the verify forward x8, drafter and verify once
        t_scaled = float(sum(scaled[warmup:]))
        out["value"] = tokens / t_scaled
        out["ms_per_step_scaled_to_32_blocks"] = round(t_scaled / steps * 1e3, 2)
        out["block_scale"] = 32 / cfg.n_layers
        why = ("a bounded sample" if sampled else
               f"host memory {avail / 2**30:.0f} GiB free is short of the 26 GB of fp32 weights")
        ctx_desc = (f"on a synthetically filled state of {synthetic_context} tokens (random KV rows, FIR "
                    f"histories, IIR states and drafter context)" if synthetic_context else
                    f"after a {prompt_len - 1}-token prefill")
        out["sample"] = (f"{steps} timed rounds (after {warmup} untimed) over 4 of the 32 blocks (SE, MR, LI, MHA; "
                         f"{why}) {ctx_desc}; value scales the measured verify forward x8 to 32 blocks")
    return out


def run_reference(args) -> int:
    world, rank, _ = dist_setup()
    if rank != 0:
        return 0
    n = os.cpu_count() or 1
    t0 = time.perf_counter()
    r = cpu_reference_rounds(n, args.steps, args.warmup)
    wall = time.perf_counter() - t0
    value = r["value"]
    line = {
        "impl": "reference", "metric": METRIC, "value": None if value is None else round(value, 4), "unit": "tok/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(r["ms_per_step"], 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": headline_config(1),
        "cpu_baseline": {"value": None if value is None else round(value, 4), "unit": "tok/s", "cores": r["cores"],
                         "kind": "port", "sample": r["sample"]},
        "e2e": {"value": None if value is None else round(value, 4), "unit": "tok/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "tau": round(r["tokens"] / args.steps, 4), "blocks_run": r["blocks_run"], "init_s": r["init_s"],
        "prefill_s": r["prefill_s"], "wall_s": round(wall, 1),
    }
    for k in ("ms_per_step_scaled_to_32_blocks", "block_scale"):
        if k in r:
            line[k] = r[k]
    print(json.dumps(line), flush=True)
    return 0


def headline_config(world: int) -> dict:
    return {"workload": "evo2_7b-shaped single-stream speculative round: neural drafter + gamma=12 verify "
                        "block + fp64 verify + slice rollback, T=1.0 top_k=4",
            "prompt": f"{PROMPT_LEN}-token order-3 Markov ACGT, GC~0.5, seed per rank",
            "gamma": GAMMA, "d_model": 4096, "n_layers": 32,
            "drafter": "d=1024, 2 layers, ctx 64 from block 27",
            "l2": "inputs larger than L2: 12.95 GB of bf16 weights streamed per step",
            "parallelism": f"independent streams x{world}, no collectives"}


def run_streams(args) -> int:
    """--streams S: S independent streams per rank, batched rounds, no collectives."""
    import torch
    import torch.distributed as dist

    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=device)
    from evspark_b200 import _native as N
    from evspark_b200.config import DRAFTERS, target_config
    from evspark_b200.drafter import DeviceDrafter, layer_index
    from evspark_b200.model import TargetModel
    from evspark_b200.specdec.block.neural_draft import NeuralDraftModel
    from evspark_b200.ranks import combine_timing
    from evspark_b200.specdec.block.streams import StreamBatch
    from evspark_b200.workload import markov_prompt

    S = int(args.streams)
    cfg = target_config(args.config)
    dcfg = DRAFTERS[args.config]
    model = TargetModel.random(cfg, seed=20260820, device=device, init_on="cuda",
                               capture_layers=tuple(layer_index(n) for n in dcfg.inject_layers))
    drafter = DeviceDrafter.random(dcfg, seed=20260830, embed=model.weights["embed"], device=device, init_on="cuda",
                                   max_batch=S)
    nd = NeuralDraftModel(model, drafter, dcfg.inject_layers)
    first = rank * S
    prompts = np.stack([markov_prompt(PROMPT_LEN, seed=20260821 + first + i) for i in range(S)])
    rngs = [np.random.default_rng(7 + first + i) for i in range(S)]
    n_tok = (args.warmup + args.steps + 2) * (GAMMA + 1)
    sb = StreamBatch(model, nd, prompts, n_tok, GAMMA, False, rngs, temperature=1.0, top_k=4)
    for _ in range(args.warmup):
        sb.round()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(local)
    n0 = N.launch_count()
    emitted0 = sum(len(e) for e in sb.emitted)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    ev0.record()
    for _ in range(args.steps):
        torch.cuda.nvtx.range_push("evs_round")  # lets a profiler select the timed rounds
        sb.round()
        torch.cuda.nvtx.range_pop()
    ev1.record()
    torch.cuda.synchronize()
    launches = N.launch_count() - n0
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1)
    tokens = float(sum(len(e) for e in sb.emitted) - emitted0)
    ms, tokens = combine_timing(ms, tokens, device)
    if rank == 0:
        line = {
            "metric": "accepted tok/s multi-stream Evo2-7B-shape γ=12", "value": round(tokens / (ms / 1e3), 3),
            "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"{args.config}-shaped batched speculative rounds: {S} independent streams "
                                   "per GPU, neural drafter + gamma=12 verify forward (M = 13 x streams) + fp64 "
                                   "verify + per-row rollback, T=1.0 top_k=4",
                       "streams_per_gpu": S, "streams_total": S * world,
                       "prompt": f"{PROMPT_LEN}-token order-3 Markov ACGT, GC~0.5, seed per stream",
                       "l2": "inputs larger than L2: the bf16 weights are streamed every round",
                       "parallelism": f"streams partitioned over {world} GPU(s), no collectives"},
            "tau": round(tokens / (args.steps * S * max(world, 1)), 4),
            "clocks": clk, "gpu_launches": int(launches),
        }
        print(json.dumps(line), flush=True)
    sb.ip.close()
    nd.close()
    model.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


def run_tp(args) -> int:
    """One stream on a target channel-sharded over all ranks (config 5: Evo2-40B shape)."""
    import datetime

    import torch
    import torch.distributed as dist

    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=device)
    from evspark_b200 import _native as N
    from evspark_b200.config import DRAFTERS, target_config
    from evspark_b200.drafter import DeviceDrafter, layer_index
    from evspark_b200.model import TargetModel
    from evspark_b200.ranks import combine_timing
    from evspark_b200.specdec.block.driver import prefill
    from evspark_b200.specdec.block.loop import spec_round
    from evspark_b200.specdec.block.neural_draft import NeuralDraftModel
    from evspark_b200.workload import markov_prompt

    cfg = target_config(args.config)
    dcfg = DRAFTERS[args.config]
    L = args.prompt_len or (8192 if args.config == "evo2_40b" else PROMPT_LEN)
    model = TargetModel.random(cfg, seed=20260820, device=device, init_on="cuda", tp=(rank, world),
                               capture_layers=tuple(layer_index(n) for n in dcfg.inject_layers))
    drafter = DeviceDrafter.random(dcfg, seed=20260830, embed=model.weights["embed"], device=device, init_on="cuda")
    nd = NeuralDraftModel(model, drafter, dcfg.inject_layers)
    prompt = markov_prompt(L, seed=20260821)  # the same stream on every rank
    rounds = args.warmup + args.steps
    ip = model.initialize_inference_params(L + (rounds + 4) * (GAMMA + 1) + VERIFY_REPS + 64, max_chunk=args.prefill_chunk or None)
    nd.capture_begin()
    t0 = time.perf_counter()
    prefill(model, torch.as_tensor(prompt[:-1], device=device)[None], ip)
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t0
    nd.capture_commit(L - 1)
    rng = np.random.default_rng(7)
    state = {"ip": ip, "y": int(prompt[-1])}
    chunk = torch.empty(1, GAMMA + 1, dtype=torch.int64, device=device)

    def one_round():
        out = spec_round(model, nd, state["ip"], state["y"], GAMMA, False, rng, 1 << 30, temperature=1.0, top_k=4,
                         timing=False, chunk=chunk)
        state["ip"], state["y"] = out.ip, int(out.taken[-1])
        return len(out.taken)

    for _ in range(args.warmup):
        one_round()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(local)
    n0 = N.launch_count()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    ev0.record()
    tokens = 0
    for _ in range(args.steps):
        torch.cuda.nvtx.range_push("evs_round")  # lets a profiler select the timed rounds
        tokens += one_round()
        torch.cuda.nvtx.range_pop()
    ev1.record()
    torch.cuda.synchronize()
    launches = N.launch_count() - n0
    clk = clocks.stop()
    ms, _ = combine_timing(ev0.elapsed_time(ev1), 0.0, device)
    # the verify forward alone (every rank issues the same calls: the forward is collective over the
    # ranks' shared partial sums), on a clone of the state, each followed by a rollback to k = 0
    vb_chunk = torch.as_tensor(np.concatenate([[state["y"]], markov_prompt(GAMMA, seed=5)]), device=device)[None]
    ipv = state["ip"].clone()
    vb_ms = []
    for i in range(VERIFY_REPS + 2):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        ipv.forward(vb_chunk, retain=True)
        e1.record()
        ipv.rollback(np.zeros(1, dtype=np.int64))
        torch.cuda.synchronize()
        if i >= 2:
            vb_ms.append(e0.elapsed_time(e1))
    ipv.close()
    vb_us, _ = combine_timing(float(np.median(vb_ms)) * 1e3, 0.0, device)
    # per kernel group of the target forward (a profiled pass: events around every group)
    prof_steps = 4
    N.call("evs_profile_start", state["ip"].handle)
    for _ in range(prof_steps):
        one_round()
    torch.cuda.synchronize()
    pl, pms, pb = (C.c_int64 * 4)(), (C.c_double * 4)(), (C.c_double * 4)()
    N.call("evs_profile_stop", state["ip"].handle, pl, pms, pb)
    err = [C.c_int32(), C.c_int32(), C.c_int32()]
    N.check(N.lib().evs_get_device_error(state["ip"].handle, *[C.byref(e) for e in err]), "evs_get_device_error")
    cpu_baseline = None
    if rank == 0 and world == 1 and args.config == "evo2_7b" and args.cpu_steps > 0:
        state["ip"].close()
        state["ip"] = None
        nd.close()
        model.close()
        torch.cuda.empty_cache()
        cpu = cpu_reference_rounds(os.cpu_count() or 1, args.cpu_steps, 1, sampled=True, synthetic_context=L - 1)
        cpu_baseline = {"value": round(cpu["value"], 5), "unit": "tok/s", "cores": cpu["cores"], "kind": "port",
                        "sample": cpu["sample"], "ms_per_step_measured": round(cpu["ms_per_step"], 1),
                        "ms_per_step_scaled_to_32_blocks": cpu.get("ms_per_step_scaled_to_32_blocks")}
    if rank == 0:
        line = {
            "metric": (f"accepted tok/s single-stream {args.config} γ=12, channel-sharded" if world > 1 else
                       f"accepted tok/s single-stream {args.config} γ=12, {L}-token context"), "value":
                round(tokens / (ms / 1e3), 3), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"{args.config}-shaped single-stream speculative round, target sharded by "
                                   f"channels over {world} GPU(s) (row-parallel sums added across ranks over "
                                   "NVLink in the residual RMSNorm), drafter replicated, T=1.0 top_k=4",
                       "prompt": f"{L}-token order-3 Markov ACGT, GC~0.5", "gamma": GAMMA,
                       "d_model": cfg.d_model, "n_layers": cfg.n_layers, "parallelism": f"tp{world}",
                       "l2": "inputs larger than L2: the bf16 weight shards are streamed every round"},
            "tau": round(tokens / args.steps, 4), "prefill_s": round(prefill_s, 3),
            "prefill_tok_s": round((L - 1) / prefill_s, 1), "prefill_chunk": int(ip.max_chunk),
            "verify_block_us": round(vb_us, 1),
            "groups_ms_per_step": {k: round(pms[i] / prof_steps, 4)
                                   for i, k in enumerate(("gemm", "hyena", "attn", "row"))},
            "groups_launches_per_step": {k: int(pl[i] // prof_steps)
                                         for i, k in enumerate(("gemm", "hyena", "attn", "row"))},
            "groups_note": "rank 0, a separate profiled pass with CUDA events around every kernel group of the "
                           "target forward (serialises them); row = embedding, residual + RMSNorm with the "
                           "cross-rank partial sums, SwiGLU, logits",
            "device_error": int(err[0].value), "clocks": clk, "gpu_launches": int(launches),
        }
        if cpu_baseline is not None:
            line["cpu_baseline"] = cpu_baseline
        print(json.dumps(line), flush=True)
    if state["ip"] is not None:
        state["ip"].close()
        nd.close()
        model.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


def run_ours(args) -> int:
    import torch
    import torch.distributed as dist

    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=device)
    from evspark_b200 import _native as N
    from evspark_b200.api import EvSpark
    from evspark_b200.config import DRAFTERS, EVO2_7B
    from evspark_b200.drafter import DeviceDrafter, layer_index
    from evspark_b200.model import TargetModel
    from evspark_b200.specdec.block.driver import prefill
    from evspark_b200.specdec.block.loop import native_greedy_reference, spec_round, speculative_generate
    from evspark_b200.specdec.block.neural_draft import NeuralDraftModel
    from evspark_b200.workload import markov_prompt, to_text

    from evspark_b200.config import target_config

    cfg = target_config(args.config)
    dcfg = DRAFTERS[args.config]
    model = TargetModel.random(cfg, seed=20260820, device=device, init_on="cuda",
                               capture_layers=tuple(layer_index(n) for n in dcfg.inject_layers))
    drafter = DeviceDrafter.random(dcfg, seed=20260830, embed=model.weights["embed"], device=device, init_on="cuda")
    nd = NeuralDraftModel(model, drafter, dcfg.inject_layers)
    prompt = markov_prompt(PROMPT_LEN, seed=20260821 + rank)
    rounds_total = args.warmup + args.steps + min(args.steps, 8)
    ip = model.initialize_inference_params(PROMPT_LEN + (rounds_total + 4) * (GAMMA + 1) + VERIFY_REPS + 64)
    nd.capture_begin()
    prefill(model, torch.as_tensor(prompt[:-1], device=device)[None], ip)
    nd.capture_commit(PROMPT_LEN - 1)
    rng = np.random.default_rng(7 + rank)
    y = int(prompt[-1])
    chunk = torch.empty(1, GAMMA + 1, dtype=torch.int64, device=device)
    seen = prompt.copy()

    def one_round():
        nonlocal ip, y, seen
        out = spec_round(model, nd, ip, y, GAMMA, False, rng, 1 << 30, seen=seen, temperature=1.0, top_k=4,
                         timing=False, chunk=chunk)
        ip = out.ip
        y = int(out.taken[-1])
        return out

    for _ in range(args.warmup):
        one_round()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(local)
    n0 = N.launch_count()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    ev0.record()
    accepted = 0
    ks = []
    for _ in range(args.steps):
        torch.cuda.nvtx.range_push("evs_round")  # lets a profiler select the timed rounds
        out = one_round()
        torch.cuda.nvtx.range_pop()
        accepted += len(out.taken)
        ks.append(out.log.k)
    ev1.record()
    torch.cuda.synchronize()
    launches = N.launch_count() - n0
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1)
    # verify-block latency: CUDA events around the retained verify forward alone (unprofiled, the
    # same kernels and launch overlap as in the rounds), each followed by a rollback to k = 0
    vb_chunk = torch.as_tensor(np.concatenate([[y], markov_prompt(GAMMA, seed=5)]), device=device)[None]
    ipv = ip.clone()
    vb_ms = []
    for i in range(VERIFY_REPS + 2):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        ipv.forward(vb_chunk, retain=True)
        e1.record()
        ipv.rollback(np.zeros(1, dtype=np.int64))
        torch.cuda.synchronize()
        if i >= 2:
            vb_ms.append(e0.elapsed_time(e1))
    ipv.close()
    verify_block_us = float(np.median(vb_ms)) * 1e3
    # a separate profiled pass (events around every kernel group of the verify block) for the
    # per-kernel roofline; its event overhead stays out of the headline number above
    import ctypes as C

    prof_steps = max(1, min(args.steps, 8))
    N.call("evs_profile_start", ip.handle)
    for _ in range(prof_steps):
        one_round()
    torch.cuda.synchronize()
    pl, pms, pb = (C.c_int64 * 4)(), (C.c_double * 4)(), (C.c_double * 4)()
    N.call("evs_profile_stop", ip.handle, pl, pms, pb)
    if world > 1:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        a = torch.tensor([float(accepted)], device=device)
        dist.all_reduce(a, op=dist.ReduceOp.SUM)
        total_accepted = float(a.item())
    else:
        total_accepted = float(accepted)
    value = total_accepted / (ms / 1e3)
    peak, peak_kind = peaks()
    gemm_ms, gemm_bytes, gemm_n = pms[0], pb[0], pl[0]
    achieved = gemm_bytes / (gemm_ms / 1e3) / 1e9 if gemm_ms > 0 else 0.0
    kernel_ms = sum(pms[i] for i in range(4))

    if args.no_extras:
        if rank == 0:
            print(json.dumps({"metric": METRIC, "value": round(value, 3), "unit": "tok/s", "config": args.config,
                              "ms_per_step": round(ms / args.steps, 4), "verify_block_us": round(verify_block_us, 1),
                              "gemm_gbs": round(achieved, 1), "gpu_launches": int(launches)}), flush=True)
        ip.close()
        nd.close()
        model.close()
        return 0

    # ---- e2e through the public API: host prompt string -> EvSpark.generate -> host tokens, the
    # prompt staged from pinned memory, every round's uniforms up and result down (counted) ----
    from evspark_b200.ranks import combine_timing

    es = EvSpark(model, nd, str(device), state_seqlen=PROMPT_LEN + E2E_TOKENS + 64)
    text = to_text(prompt)
    es.generate(text, n_tokens=32, seed=3 + rank)  # first call: drafter graph capture, lazy set-up
    e2e = {}
    for mode, greedy in (("sampled", False), ("greedy", True)):
        x0 = N.transfer_count()
        res = es.generate(text, n_tokens=E2E_TOKENS, seed=11 + rank, greedy=greedy)
        x1 = N.transfer_count()
        wall_ms, toks = combine_timing(res.wall_s * 1e3, float(res.n_tokens), device)
        e2e[mode] = {"value": round(toks / (wall_ms / 1e3), 3), "rounds": int(res.n_rounds),
                     "mean_tau": round(res.mean_tau, 3), "h2d_bytes": int(x1[0] - x0[0]),
                     "d2h_bytes": int(x1[1] - x0[1]), "wall_ms": round(wall_ms, 1)}
    es_s = e2e["sampled"]
    e2e_line = {"value": es_s["value"], "unit": "tok/s",
                "h2d_bytes_per_step": round(es_s["h2d_bytes"] / es_s["rounds"], 1),
                "d2h_bytes_per_step": round(es_s["d2h_bytes"] / es_s["rounds"], 1),
                "n_tokens": E2E_TOKENS, "rounds": es_s["rounds"], "mean_tau": es_s["mean_tau"],
                "prefill_included": True, "aggregate": f"tokens of all {world} rank(s) / slowest rank's wall time",
                "greedy": e2e["greedy"]}

    extra = {}
    if rank == 0 and world == 1:
        # native T=1 decoding (speedup denominator) and an oracle drafter (target's own greedy
        # continuation: every draft accepted, tau = γ+1) on the same model
        pr = torch.as_tensor(prompt, device=device)[None]
        t0 = time.perf_counter()
        nat, ipn, _ = native_greedy_reference(model, pr, 64)
        torch.cuda.synchronize()
        extra["native_greedy_tok_s"] = round(64 / (time.perf_counter() - t0), 2)
        ipn.close()
        cont, ipc, _ = native_greedy_reference(model, pr, 13 * 8)
        ipc.close()

        class OracleDraft:
            def probs(self, prefix):
                out = np.zeros(512)
                i = len(prefix) - PROMPT_LEN
                out[int(cont[i]) if 0 <= i < len(cont) else 65] = 1.0
                return out

        torch.cuda.synchronize()
        t0 = time.perf_counter()
        spec = speculative_generate(model, OracleDraft(), pr, 13 * 8, GAMMA, greedy=True,
                                    rng=np.random.default_rng(0), timing=False)
        torch.cuda.synchronize()
        extra["oracle_drafter_tok_s"] = round(13 * 8 / (time.perf_counter() - t0), 2)
        extra["oracle_drafter_greedy_identical"] = bool(np.array_equal(spec.emitted_ids, cont))
        spec.inference_params_dict.close()
    es._state.close()
    es._state = None
    ip.close()
    nd.close()
    model.close()
    del es, model
    torch.cuda.empty_cache()
    cpu_baseline = None
    if rank == 0 and world == 1:
        cpu = cpu_reference_rounds(os.cpu_count() or 1, args.cpu_steps, 1, sampled=True, prompt_len=256)
        cpu_baseline = {"value": round(cpu["value"], 4), "unit": "tok/s", "cores": cpu["cores"], "kind": "port",
                        "sample": cpu["sample"], "ms_per_step_measured": round(cpu["ms_per_step"], 1),
                        "ms_per_step_scaled_to_32_blocks": cpu.get("ms_per_step_scaled_to_32_blocks"),
                        "blocks_run": cpu["blocks_run"]}

    if rank == 0:
        hy_ms, hy_bytes = pms[1], pb[1]
        hy_gbs = hy_bytes / (hy_ms / 1e3) / 1e9 if hy_ms > 0 else 0.0
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": headline_config(world),
            "tau": round(total_accepted / (args.steps * max(world, 1)), 4),
            "verify_block_us": round(verify_block_us, 1),
            "verify_block_note": f"median of {VERIFY_REPS} CUDA-event timings of the retained 13-token verify "
                                 "forward alone (no profiling events), after the timed rounds",
            "roofline": {"bound": "hbm", "kernel": "gemm_tc (tcgen05 projections)", "achieved": round(achieved, 1),
                         "peak": peak, "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "traffic": round(GEMM_TRAFFIC_RATIO * gemm_bytes / max(gemm_n, 1)),
                         "traffic_note": GEMM_TRAFFIC_NOTE,
                         "launches": int(gemm_n),
                         "bytes_per_launch": round(gemm_bytes / max(gemm_n, 1)),
                         "avg_launch_us": round(gemm_ms / max(gemm_n, 1) * 1e3, 2),
                         "share_of_kernel_time": round(gemm_ms / kernel_ms, 4) if kernel_ms else None,
                         "timing_note": "per-launch CUDA events around every kernel group of a separate "
                                        f"{prof_steps}-round pass (serialises the kernels of a forward)",
                         "groups_ms_per_step": {k: round(pms[i] / prof_steps, 4)
                                                for i, k in enumerate(("gemm", "hyena", "attn", "row"))},
                         "groups_gbs": {k: round(pb[i] / (pms[i] / 1e3) / 1e9, 1) if pms[i] else None
                                        for i, k in enumerate(("gemm", "hyena", "attn", "row"))},
                         "hyena": {"achieved": round(hy_gbs, 1), "frac": round(hy_gbs / peak, 4),
                                   "unit": "GB/s"}},
            "cpu_baseline": cpu_baseline,
            "e2e": e2e_line,
            "clocks": clk,
            "gpu_launches": int(launches),
            **extra,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=("ours", "reference"))
    ap.add_argument("--cpu-steps", type=int, default=3)
    ap.add_argument("--config", default="evo2_7b", help="evo2_7b (headline) or evo2_7b_slice (4 blocks, profiling)")
    ap.add_argument("--no-extras", action="store_true", help="time the rounds only (profiling runs)")
    ap.add_argument("--streams", type=int, default=1, help="independent streams per GPU, decoded in batched rounds")
    ap.add_argument("--tp", action="store_true", help="shard the target by channels over the GPUs (one stream)")
    ap.add_argument("--prompt-len", type=int, default=0, help="prompt length of --tp runs (default 8192 for 40B)")
    ap.add_argument("--prefill-chunk", type=int, default=0, help="tokens per prefill forward of --tp runs (long prompts)")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        return run_reference(args)
    if args.streams > 1:
        return run_streams(args)
    if args.tp or (args.config == "evo2_40b" and int(os.environ.get("WORLD_SIZE", "1")) > 1):
        return run_tp(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
