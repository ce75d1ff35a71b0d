"""Block-verify driver, native step reference and state snapshots on the device path.

Mirrors evspark/specdec/block/driver.py (names, signatures, offset contract):

* ``prefill`` (driver.py:49-60): offsets must be 0; afterwards every key's offset is L;
  returns logits [B, L, V] whose last row is p(·|prefix).
* ``block_forward`` (driver.py:179-226): chunk [B, T] from the current state; row i of the
  logits is p(·|prefix, x_1..x_{i+1}); offsets advance by T; ``retain=True`` also returns a
  ``ChunkStash`` so that ``slice_states_to_accept`` can roll back without replay.
* ``step_forward_reference`` (driver.py:229-240): the native token-by-token path (T=1 calls of
  the same kernels), row i = logits after consuming x_{i+1}.
* ``clone_inference_params`` / ``expand`` / ``collapse`` / ``snapshot_states`` / ``diff_states``.
"""

from __future__ import annotations

import torch

from evspark_b200.model import PARAM_KEYS, InferenceParams

_HYENA_KEYS = ("hcl", "hcm", "hcs")


def set_seqlen_offsets(inference_params_dict: InferenceParams, offset: int) -> None:
    inference_params_dict.set_offset(int(offset))


def step_seqlen_offsets(inference_params_dict: InferenceParams, n: int = 1) -> None:
    inference_params_dict.set_offset(inference_params_dict.offset + int(n))


def get_seqlen_offset(inference_params_dict: InferenceParams) -> int:
    return int(inference_params_dict.offset)


def clone_inference_params(inference_params_dict: InferenceParams) -> InferenceParams:
    """Full device copy of every state arena (the reference deep-copies, driver.py:40-46)."""
    return inference_params_dict.clone()


def prefill(model, input_ids: torch.Tensor, inference_params_dict: InferenceParams) -> torch.Tensor:
    assert inference_params_dict.offset == 0, "prefill requires seqlen_offset == 0 on every key"
    ids = torch.as_tensor(input_ids).long()
    if ids.dim() == 1:
        ids = ids[None]
    return inference_params_dict.prefill(ids)


def block_forward(model, chunk_ids: torch.Tensor, inference_params_dict: InferenceParams, retain: bool = False):
    from evspark_b200.specdec.block.slice import ChunkStash

    ip = inference_params_dict
    ids = torch.as_tensor(chunk_ids).long()
    if ids.dim() == 1:
        ids = ids[None]
    B = int(ids.shape[0])
    L0 = ip.offset if B <= ip.batch else int(ip.lengths[0])
    lengths_before = torch.as_tensor(ip.lengths[:B].copy(), dtype=torch.int32)
    logits = ip.forward(ids, retain=retain)
    if not retain:
        return logits
    stash = ChunkStash(L0=int(L0), chunk_len=int(ids.shape[1]), flash_attn=True, lengths_before=lengths_before,
                       model=model, uid=ip.retained_uid)
    return logits, stash


def step_forward_reference(model, chunk_ids: torch.Tensor, inference_params_dict: InferenceParams) -> torch.Tensor:
    ids = torch.as_tensor(chunk_ids).long()
    if ids.dim() == 1:
        ids = ids[None]
    outs = [inference_params_dict.forward(ids[:, i:i + 1], retain=False)[:, -1] for i in range(ids.shape[1])]
    return torch.stack(outs, dim=1)


def expand_inference_params(inference_params_dict: InferenceParams, batch: int) -> None:
    B = int(batch)
    if B < 1:
        raise ValueError(f"batch must be >= 1, got {B}")
    if B == 1:
        return
    if inference_params_dict.max_batch < B:
        raise ValueError(f"mha.max_batch_size={inference_params_dict.max_batch} < B={B}: set "
                         "model.config.max_batch_size >= B before initialize_inference_params")
    inference_params_dict.expand(B)


def collapse_inference_params(inference_params_dict: InferenceParams, idx: int) -> None:
    inference_params_dict.collapse(int(idx))


def snapshot_states(inference_params_dict: InferenceParams, kv_len: int | None = None, *,
                    batch_size: int = 1) -> dict:
    """CPU tensor tree in the reference's layout (driver.py:243-278)."""
    ip = inference_params_dict
    bsz = int(batch_size)
    cfg = ip.model.cfg
    snap: dict = {"seqlen_offsets": {k: int(ip.offset) for k in PARAM_KEYS}}
    snap["mha"] = {"key_value_memory_dict": {
        int(i): ip.export(i, 3, rows=bsz, kv_len=kv_len).float().cpu() for i in cfg.layer_idxs("mha")}}
    for key in _HYENA_KEYS:
        entry = {}
        layers = cfg.layer_idxs(key)
        if layers and ip.offset > 0:
            entry["fir_state_dict"] = {int(i): ip.export(i, 0, rows=bsz).cpu() for i in layers}
            if key in ("hcs", "hcm"):
                entry["fir_inner_state_dict"] = {int(i): ip.export(i, 1, rows=bsz).cpu() for i in layers}
            else:
                entry["state_dict"] = {int(i): ip.export(i, 2, rows=bsz).cpu() for i in layers}
        snap[key] = entry
    return snap


def diff_states(a: dict, b: dict) -> dict:
    """Per-tensor max-abs / max-rel differences (driver.py:281-308)."""
    if a["seqlen_offsets"] != b["seqlen_offsets"]:
        raise ValueError(f"seqlen_offsets differ: {a['seqlen_offsets']} vs {b['seqlen_offsets']}")
    out: dict = {}

    def visit(va, vb, path):
        if isinstance(va, dict):
            if set(va) != set(vb):
                raise ValueError(f"state keys differ @{path}: {sorted(va)} vs {sorted(vb)}")
            for k in va:
                visit(va[k], vb[k], f"{path}/{k}")
        else:
            d = (va.float() - vb.float()).abs()
            mx = float(d.max()) if d.numel() else 0.0
            den = float(vb.float().abs().max()) if vb.numel() else 0.0
            out[path] = {"max_abs": mx, "max_rel": mx / max(den, 1e-12)}

    for key in PARAM_KEYS:
        visit(a[key], b[key], key)
    return out
