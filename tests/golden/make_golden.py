"""Generate the golden fixtures that pin the CPU oracle to the reference.

Runs the reference's OWN implementation (an EvSpark checkout, read-only)
unmodified on CPU: its block path (``block_forward``,
``slice_states_to_accept``, ``speculative_generate``, ``native_*_reference``)
drives the oracle StripedHyena2 through ``oracle/vortex_stub``; its verifier,
sampling transform and ``Drafter`` / ``trunk_forward`` / ``serial_sample`` run
directly.  Outputs go to ``tests/golden/*.npz``.  Only this build container has
the reference; the GPU box uses the committed fixtures.

    python tests/golden/make_golden.py --reference <path of the EvSpark checkout>
"""

from __future__ import annotations

import argparse
import hashlib
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]

ACGT = np.array([65, 67, 71, 84], dtype=np.int64)
MODEL_SEED = 20260820
DRAFTER_SEED = 20260830


def weights_digest(w: dict) -> str:
    h = hashlib.sha256()
    for k in sorted(w):
        h.update(k.encode())
        h.update(w[k].detach().float().cpu().numpy().tobytes())
    return h.hexdigest()


def state_arrays(ip, prefix: str, out: dict) -> None:
    for key in ("hcs", "hcm", "hcl"):
        p = ip[key]
        for attr in ("fir_state_dict", "fir_inner_state_dict", "state_dict"):
            for layer, t in getattr(p, attr).items():
                out[f"{prefix}/{attr}/{layer}"] = t.detach().float().numpy()
    out[f"{prefix}/offset"] = np.int64(ip["mha"].seqlen_offset)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of the EvSpark checkout (read-only)")
    args = ap.parse_args()
    sys.path[:0] = [str(REPO), str(REPO / "oracle" / "vortex_stub"), args.reference]
    torch.set_num_threads(8)

    from evspark.specdec.block import (block_forward, clone_inference_params, expand_inference_params,
                                       prefill, slice_states_to_accept, step_forward_reference)
    from evspark.specdec.block.loop import native_greedy_reference, speculative_generate
    from evspark.specdec.block.neural_draft import serial_sample, trunk_forward
    from evspark.specdec.drafts import IdentityDraftModel
    from evspark.specdec.transforms import apply_transform
    from evspark.specdec.verifier import (verify_round, verify_round_greedy, verify_round_greedy_multicand,
                                          verify_round_multicand)
    from evspark.specdec.block.loop import _q_prime_from_raw
    from evspark.train.drafter import Drafter
    from vortex.model.model import StripedHyena

    from evspark_b200.config import DRAFTERS, TINY
    from evspark_b200.weights import init_drafter_weights, init_target_weights
    from oracle.model import OracleTarget

    w = init_target_weights(TINY, seed=MODEL_SEED)
    oracle32 = OracleTarget(TINY, w, compute=torch.float32)
    model = StripedHyena(oracle32, max_batch_size=2)

    # ---- 1. block verify + rollback (config 1: 256-token iid ACGT prompt, γ=12) ----
    out: dict = {"weights_sha256": np.array(weights_digest(w))}
    cases = [("full", 256, 12, (0, 1, 5, 11, 12)), ("short", 64, 4, (0, 2, 4))]
    for name, L, gamma, ks in cases:
        rng = np.random.default_rng(20260821 + L)
        prompt = rng.choice(ACGT, size=L)
        chunk = np.concatenate([[prompt[-1]], rng.choice(ACGT, size=gamma)])
        out[f"{name}/prompt"] = prompt
        out[f"{name}/chunk"] = chunk
        with torch.inference_mode():
            ip = model.initialize_inference_params(max_seqlen=L + 64)
            pre = prefill(model, torch.tensor(prompt[:-1])[None], ip)
            out[f"{name}/prefill_last_logits"] = pre[0, -1].float().numpy()
            state_arrays(ip, f"{name}/after_prefill", out)
            ip_step = clone_inference_params(ip)
            step = step_forward_reference(model, torch.tensor(chunk)[None], ip_step)
            ip_blk = clone_inference_params(ip)
            logits, stash = block_forward(model, torch.tensor(chunk)[None], ip_blk, retain=True)
            out[f"{name}/block_logits"] = logits[0].float().numpy()
            out[f"{name}/step_logits"] = step[0].float().numpy()
            for k in ks:
                ip_k = clone_inference_params(ip_blk)
                slice_states_to_accept(ip_k, stash, k)
                state_arrays(ip_k, f"{name}/slice_k{k}", out)

    # ---- 2. per-row (ragged) slicing, B=2 ----
    rng = np.random.default_rng(20260831)
    L, gamma = 192, 4
    prompt = rng.choice(ACGT, size=L)
    chunks = rng.choice(ACGT, size=(2, gamma + 1))
    chunks[:, 0] = prompt[-1]
    out["ragged/prompt"] = prompt
    out["ragged/chunks"] = chunks
    out["ragged/ks"] = np.array([0, 3])
    with torch.inference_mode():
        ip = model.initialize_inference_params(max_seqlen=L + 64)
        prefill(model, torch.tensor(prompt[:-1])[None], ip)
        expand_inference_params(ip, 2)
        lg, stash = block_forward(model, torch.tensor(chunks), ip, retain=True)
        out["ragged/block_logits"] = lg.float().numpy()
        stash.flash_attn = True  # per-row KV lengths are honoured by the device path
        slice_states_to_accept(ip, stash, np.array([0, 3]))
        state_arrays(ip, "ragged/slice", out)

    # ---- 3. speculative loop: greedy identity and seeded sampling ----
    rng = np.random.default_rng(20260823)
    prompt = rng.choice(ACGT, size=256)
    out["loop/prompt"] = prompt
    n = 48
    nat, _ip, _ = native_greedy_reference(model, torch.tensor(prompt)[None], n)
    out["loop/native_greedy"] = nat
    for gamma in (4, 12):
        spec = speculative_generate(model, IdentityDraftModel(), torch.tensor(prompt)[None], n, gamma,
                                    greedy=True, rng=np.random.default_rng(0))
        out[f"loop/spec_greedy_g{gamma}"] = spec.emitted_ids
        out[f"loop/spec_greedy_g{gamma}_ks"] = np.array([r.k for r in spec.rounds_log])
        spec = speculative_generate(model, IdentityDraftModel(), torch.tensor(prompt)[None], n, gamma,
                                    greedy=False, rng=np.random.default_rng(7), temperature=1.0, top_k=4)
        out[f"loop/spec_sample_g{gamma}"] = spec.emitted_ids
        out[f"loop/spec_sample_g{gamma}_ks"] = np.array([r.k for r in spec.rounds_log])
    np.savez_compressed(HERE / "tiny_model.npz", **out)

    # ---- 4. verifier / transform known-answer vectors ----
    kat: dict = {}
    rng = np.random.default_rng(20260824)
    V, gamma, N = 512, 12, 64
    logits = rng.normal(size=(N, V)) * 3.0
    logits[0, 10] = logits[0, 20] = logits[0].max() + 1.0  # exact tie: lower index wins
    kat["transform/logits"] = logits
    for T, k in ((1.0, 4), (0.7, 4), (1.0, 0), (0.0, 4), (2.0, 1)):
        kat[f"transform/T{T}_k{k}"] = np.stack([apply_transform(r, temperature=T, top_k=k) for r in logits])
    qraw = np.exp(rng.normal(size=(N, V)))
    qraw /= qraw.sum(1, keepdims=True)
    qraw[1, :300] = 0.0
    kat["qprime/raw"] = qraw
    kat["qprime/out"] = np.stack([_q_prime_from_raw(r, 1.0, 4) for r in qraw])
    seeds, toks, ps, qs, res = [], [], [], [], []
    for c in range(200):
        r = np.random.default_rng(1000 + c)
        base = r.dirichlet(np.ones(V) * 0.3, size=gamma + 1)
        q = np.stack([apply_transform(np.log(base[i] + 1e-12) + r.normal(size=V) * (c % 3), 1.0, 4)
                      for i in range(gamma)])
        p = np.stack([apply_transform(np.log(base[i] + 1e-12), 1.0, 4) for i in range(gamma + 1)])
        if c % 17 == 0:
            p[2] = q[2]  # residual underflow -> p fallback path
        x = np.array([int(np.argmax(q[i])) if (c + i) % 4 else int(r.choice(V, p=q[i])) for i in range(gamma)])
        vr = verify_round(x, q, p, np.random.default_rng(50_000 + c))
        seeds.append(50_000 + c)
        toks.append(x)
        ps.append(p)
        qs.append(q)
        res.append([vr.accepted_len, int(vr.from_residual), int(vr.fallback)] + vr.tokens.tolist()
                   + [-1] * (gamma + 1 - len(vr.tokens)))
    kat["verify/seeds"] = np.array(seeds)
    kat["verify/tokens"] = np.array(toks)
    kat["verify/p"] = np.array(ps).astype(np.float32)
    kat["verify/q"] = np.array(qs).astype(np.float32)
    # decisions recomputed on the fp32-rounded rows (the device consumes fp32 probabilities)
    res32 = []
    for c in range(200):
        vr = verify_round(toks[c], kat["verify/q"][c].astype(np.float64), kat["verify/p"][c].astype(np.float64),
                          np.random.default_rng(seeds[c]))
        res32.append([vr.accepted_len, int(vr.from_residual), int(vr.fallback)] + vr.tokens.tolist()
                     + [-1] * (gamma + 1 - len(vr.tokens)))
    kat["verify/result"] = np.array(res32)
    g_p = rng.normal(size=(gamma + 1, V))
    g_p[3, 7] = g_p[3, 9] = g_p[3].max() + 1.0
    g_x = np.array([int(np.argmax(g_p[i])) for i in range(gamma)])
    g_x[5] = (g_x[5] + 1) % V
    vg = verify_round_greedy(g_x, g_p)
    kat["greedy/p"], kat["greedy/x"] = g_p, g_x
    kat["greedy/result"] = np.array([vg.accepted_len] + vg.tokens.tolist())
    mc_x = np.stack([g_x, g_x.copy()])
    mc_x[0, 2] = (mc_x[0, 2] + 1) % V
    vmg = verify_round_greedy_multicand(mc_x, np.stack([g_p, g_p]))
    kat["mc_greedy/x"] = mc_x
    kat["mc_greedy/result"] = np.array([vmg.accepted_len, vmg.winner] + vmg.tokens.tolist())
    mq = np.stack([qs[0], qs[1]])
    mp = np.stack([ps[0], ps[0]])
    mx = np.stack([toks[0], toks[1]])
    vm = verify_round_multicand(mx, mq, mp, np.random.default_rng(4242))
    kat["mc/x"], kat["mc/q"], kat["mc/p"] = mx, mq, mp
    kat["mc/result"] = np.array([vm.accepted_len, vm.winner, int(vm.fallback)] + vm.tokens.tolist())
    # numpy's Generator.choice(V, p) == one uniform + inverse CDF (sampling contract)
    kat["choice/seeds"] = np.arange(500)
    kat["choice/draws"] = np.array([np.random.default_rng(s).choice(V, p=ps[s % 200][s % 13]) for s in range(500)])
    np.savez_compressed(HERE / "verify_kat.npz", **kat)

    # ---- 5. drafter trunk + serial head (tiny drafter, injected from block 2) ----
    dcfg = DRAFTERS["tiny"]
    dw = init_drafter_weights(dcfg, seed=DRAFTER_SEED, embed=w["embed"])
    drafter = Drafter(d_model=dcfg.d_model, n_layers=dcfg.n_layers, gamma=dcfg.gamma, n_inject=dcfg.n_inject,
                      target_hidden=dcfg.target_hidden, ctx_window=dcfg.ctx_window)
    drafter.load_state_dict(dw)
    drafter.eval()
    dr: dict = {"drafter_sha256": np.array(weights_digest(dw))}
    g = torch.Generator().manual_seed(DRAFTER_SEED + 1)
    for T in (0, 9, 64):
        h_raw = torch.randn(T, dcfg.n_inject * dcfg.target_hidden, generator=g)
        anchor = 71
        with torch.no_grad():
            U, h = trunk_forward(drafter, torch.tensor([anchor]), h_raw if T else None, torch.tensor([T]))
            tg, qg, cg = serial_sample(drafter, U, h, anchor, True, np.random.default_rng(0))
            ts, qsx, cs = serial_sample(drafter, U, h, anchor, False, np.random.default_rng(11),
                                        temperature=1.0, top_k=4)
            Ug, hg = trunk_forward(drafter, torch.tensor([anchor]), h_raw if T else None, torch.tensor([T]),
                                   gamma=5)
        dr[f"ctx{T}/h_raw"] = h_raw.numpy()
        dr[f"ctx{T}/U"] = U[0].numpy()
        dr[f"ctx{T}/h"] = h[0].numpy()
        dr[f"ctx{T}/U_g5"] = Ug[0].numpy()
        dr[f"ctx{T}/greedy_tokens"], dr[f"ctx{T}/greedy_q"], dr[f"ctx{T}/greedy_conf"] = tg, qg, cg
        dr[f"ctx{T}/sample_tokens"], dr[f"ctx{T}/sample_q"], dr[f"ctx{T}/sample_conf"] = ts, qsx, cs
    np.savez_compressed(HERE / "drafter_tiny.npz", **dr)

    # ---- 6. drafter at Evo2-7B width (d=1024, 16 heads, context of block-27 outputs, d_target 4096) ----
    from evspark_b200.config import EVO2_7B
    from evspark_b200.weights import init_target_tensor

    dcfg = DRAFTERS["evo2_7b"]
    emb7 = init_target_tensor(EVO2_7B, "embed", seed=MODEL_SEED)
    dw = init_drafter_weights(dcfg, seed=DRAFTER_SEED, embed=emb7)
    drafter = Drafter(d_model=dcfg.d_model, n_layers=dcfg.n_layers, gamma=dcfg.gamma, n_inject=dcfg.n_inject,
                      target_hidden=dcfg.target_hidden, ctx_window=dcfg.ctx_window)
    drafter.load_state_dict(dw)
    drafter.eval()
    dr7: dict = {"drafter_sha256": np.array(weights_digest(dw))}
    g = torch.Generator().manual_seed(DRAFTER_SEED + 7)
    for T in (0, 64):
        h_raw = torch.randn(T, dcfg.n_inject * dcfg.target_hidden, generator=g)
        anchor = 67
        with torch.no_grad():
            U, h = trunk_forward(drafter, torch.tensor([anchor]), h_raw if T else None, torch.tensor([T]))
            tg, qg, cg = serial_sample(drafter, U, h, anchor, True, np.random.default_rng(0))
            ts, qsx, cs = serial_sample(drafter, U, h, anchor, False, np.random.default_rng(11),
                                        temperature=1.0, top_k=4)
        dr7[f"ctx{T}/h_raw"] = h_raw.numpy()
        dr7[f"ctx{T}/U"] = U[0].numpy()
        dr7[f"ctx{T}/h"] = h[0].numpy()
        dr7[f"ctx{T}/greedy_tokens"], dr7[f"ctx{T}/greedy_q"], dr7[f"ctx{T}/greedy_conf"] = tg, qg, cg
        dr7[f"ctx{T}/sample_tokens"], dr7[f"ctx{T}/sample_q"], dr7[f"ctx{T}/sample_conf"] = ts, qsx, cs
    np.savez_compressed(HERE / "drafter_7b.npz", **dr7)
    for f in ("tiny_model.npz", "verify_kat.npz", "drafter_tiny.npz", "drafter_7b.npz"):
        print(f, (HERE / f).stat().st_size, "bytes")


if __name__ == "__main__":
    main()
