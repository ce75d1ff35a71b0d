"""Block-by-block (teacher-forced) parity of a bf16 model against the bf16-emulating oracle.

Two bf16 implementations whose fp32 accumulation orders differ at all drift apart by about one
bf16 rounding of every activation after a few rounding points: a one-ulp flip in an activation
moves the next GEMM's outputs across other rounding boundaries, and so on.  Run end to end, the
oracle computed in fp32 differs from the same oracle computed in fp64 by more than 2e-2 in the
logits of a 4-block Evo2-7B-width model; no kernel can do better than that noise.  So the parity
of a bf16 model is checked where the rounding inputs agree:

* every block runs in the oracle on the device's own input to that block (its residual stream,
  captured in fp32 at every position of the prompt and the verify chunk), and its output is
  compared with the device's output of the same block;
* the oracle's final norm and unembedding run on the device's last residual stream, and the
  logits are compared with the device's logits, within 2e-2 max-abs.

The device's residual streams come from the drafter-context capture ring (four blocks per model
handle; the handles share the weights), so nothing outside the product path is instrumented.
"""

from __future__ import annotations

import numpy as np
import torch

#: bf16 logits (device vs the oracle head on the device's last residual stream), max-abs
TOL_BF16_LOGITS = 2e-2
#: one block's output (device vs the oracle block on the device's input), relative to the block's
#: own contribution to the residual stream: max-abs and RMS.  The oracle computed in fp32 instead
#: of fp64 moves by at most 1.7e-3 (max) and 1.2e-3 (RMS) in these units at Evo2-7B width.
TOL_BLOCK_MAX = 1e-2
TOL_BLOCK_RMS = 5e-3


def capture_rows(ip, slot: int, positions: int, row: int = 0) -> torch.Tensor:
    """Residual stream of capture slot ``slot`` at absolute positions [0, positions), fp32 [P, d]."""
    ptr, ring_len = ip.capture_ring(slot)
    d = ip.model.cfg.d_model
    if positions > ring_len:
        raise ValueError(f"{positions} positions do not fit the {ring_len}-row capture ring")

    class _Ring:  # the ring [max_batch, ring_len, d] as a CUDA array view
        __cuda_array_interface__ = {"shape": (ip.max_batch, ring_len, d), "typestr": "<f4",
                                    "data": (int(ptr), False), "version": 3, "strides": None}

    ring = torch.as_tensor(_Ring(), device=ip.model.device)
    return ring[row, :positions].clone()


def device_block_outputs(cfg, weights: dict, prompt: np.ndarray, chunk: np.ndarray, device, tp=None):
    """Run prefill(prompt) + verify(chunk) on the device, four captured blocks per model handle.

    Returns ``(xs [n_layers, P, d] fp32 on the host, prefill logits [L, V], block logits [T, V])``
    with P = len(prompt) + len(chunk).  The logits of every handle must agree bit for bit.
    """
    from evspark_b200.model import TargetModel
    from evspark_b200.specdec.block import block_forward, prefill

    L, T = len(prompt), len(chunk)
    P = L + T
    xs = [None] * cfg.n_layers
    pre0 = blk0 = None
    for g0 in range(0, cfg.n_layers, 4):
        group = tuple(range(g0, min(g0 + 4, cfg.n_layers)))
        model = TargetModel(cfg, weights, capture_layers=group, device=device, max_chunk=64, tp=tp)
        ip = model.initialize_inference_params(P + 8, max_chunk=64)
        pre = prefill(model, torch.as_tensor(prompt)[None], ip)[0]
        blk = block_forward(model, torch.as_tensor(chunk)[None], ip)[0]
        for j, layer in enumerate(group):
            xs[layer] = capture_rows(ip, j, P).cpu()
        if pre0 is None:
            pre0, blk0 = pre.cpu(), blk.cpu()
        else:
            assert torch.equal(pre.cpu(), pre0) and torch.equal(blk.cpu(), blk0), \
                "capturing other blocks changed the logits"
        ip.close()
        model.close()
    return torch.stack(xs), pre0, blk0


def layer_weights(weights: dict, i: int) -> dict:
    pre = f"blocks.{i}."
    return {k[len(pre):]: v.detach().cpu() for k, v in weights.items() if k.startswith(pre)}


def teacher_forced_report(cfg, weights: dict, ids: np.ndarray, n_prompt: int, xs: torch.Tensor,
                          pre_logits: torch.Tensor, blk_logits: torch.Tensor, free_running: bool = False):
    """Per-block relative errors, the logit error of the teacher-forced head and (optionally) the
    logit error of the oracle run end to end on its own residual stream."""
    from oracle.model import OracleTarget, block_over_segments

    head = OracleTarget(cfg.with_(n_layers=1, layer_types=("mha",)),
                        {"embed": weights["embed"].cpu(), "final_norm": weights["final_norm"].cpu()},
                        compute=torch.float64, emulate=True)
    x_dev = head.embed(ids[None]).to(torch.float32)[0]
    x_free = x_dev.clone()
    blocks = []
    for i in range(cfg.n_layers):
        lw = layer_weights(weights, i)
        segs = [x_dev[None, :n_prompt], x_dev[None, n_prompt:]]
        out = torch.cat(block_over_segments(cfg, i, lw, segs, compute=torch.float64, emulate=True), 1)[0]
        got = xs[i].double()
        contrib = got - x_dev.double()
        delta = got - out
        blocks.append({
            "block": i, "kind": cfg.layer_types[i],
            "rel_max": (delta.abs().max() / contrib.abs().max()).item(),
            "rel_rms": (delta.pow(2).mean().sqrt() / contrib.pow(2).mean().sqrt()).item(),
        })
        if free_running:
            segs = [x_free[None, :n_prompt], x_free[None, n_prompt:]]
            x_free = torch.cat(block_over_segments(cfg, i, lw, segs, compute=torch.float64, emulate=True),
                               1)[0].to(torch.float32)
        x_dev = xs[i]
    ref = head.head(xs[-1].double()[None])[0]
    dev = torch.cat([pre_logits, blk_logits], 0).double()
    rep = {"blocks": blocks, "logits_err": (dev - ref).abs().max().item(), "logit_scale": ref.abs().max().item()}
    if free_running:
        ref_free = head.head(x_free.double()[None])[0]
        rep["free_running_err"] = (dev - ref_free).abs().max().item()
        rep["free_running_rms"] = (dev - ref_free).pow(2).mean().sqrt().item()
    return rep


def assert_teacher_forced(rep: dict) -> None:
    worst_max = max(b["rel_max"] for b in rep["blocks"])
    worst_rms = max(b["rel_rms"] for b in rep["blocks"])
    print(f"[bf16 parity] blocks={len(rep['blocks'])} worst block rel max {worst_max:.2e} rms {worst_rms:.2e}; "
          f"logits err {rep['logits_err']:.3e} (max|logit| {rep['logit_scale']:.2f})"
          + (f"; end to end (not teacher-forced) {rep['free_running_err']:.3e} (rms {rep['free_running_rms']:.3e})"
             if "free_running_err" in rep else ""))
    for b in rep["blocks"]:
        assert b["rel_max"] <= TOL_BLOCK_MAX and b["rel_rms"] <= TOL_BLOCK_RMS, b
    assert rep["logits_err"] <= TOL_BF16_LOGITS, rep["logits_err"]
