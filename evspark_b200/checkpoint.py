"""Checkpoint formats of the reference, read on the host (no device needed).

* Drafter ``.pt``: the dict ``torch.save`` writes at evspark/train/train_drafter.py:557-571 --
  ``{scheme, d_model, gamma, ctx_window, state_dict, n_pos, mask_id, offline, dump_dir}`` with the
  ``Drafter`` module's own parameter names (evspark/train/drafter.py:274-336).
  ``read_drafter_checkpoint`` returns the drafter shape, its fp32 parameters, the injection
  layers of its scheme and the remaining metadata.
* Target: the StripedHyena (vortex) state dict that evspark/specdec/block/ar_draft.py:314-338
  hands to vortex ``load_checkpoint``.  The Hyena filter tensors are the ones the reference's
  chunk path reads from each ``HyenaCascade`` (evspark/specdec/block/chunk.py:176-295):
  ``short_filter_weight`` [3d, (1,) K0], ``h`` [G, (1,) K] (SE/MR), ``D`` [d], ``log_poles``
  [G, S, 1] and ``residues`` [G, S] (LI), with ``G = hyena_filter_groups`` groups of d/G channels
  (``repeat_interleave`` over channels).  The dense names follow vortex's module tree
  (``embedding_layer``, ``blocks.N.{pre_norm, post_norm}.scale``, ``blocks.N.projections``,
  ``blocks.N.out_filter_dense``, ``blocks.N.inner_mha_cls.{Wqkv, out_proj}``,
  ``blocks.N.mlp.{l1, l2, l3}``, ``norm.scale``); vortex itself is not available offline, so these
  names are the documented mapping, checked here on synthetic state dicts only.
  ``target_weights_from_vortex`` returns this library's names (``weights.target_weight_specs``).
"""

from __future__ import annotations

import torch

from .config import HCL, HCM, HCS, MHA, DrafterConfig, TargetConfig

#: injection schemes of the reference (evspark/train/drafter.py:25-51), plus the test shapes here
SCHEME_LAYERS: dict[str, tuple[str, ...]] = {
    "S0": (), "S1": ("blocks.31",), "S2": ("blocks.7", "blocks.15", "blocks.23", "blocks.31"),
    "S3": ("blocks.6", "blocks.16", "blocks.27"), "L6": ("blocks.6",), "L16": ("blocks.16",),
    "L27": ("blocks.27",), "L20": ("blocks.20",), "L23": ("blocks.23",), "L30": ("blocks.30",),
    "D16_27": ("blocks.16", "blocks.27"), "D27_30": ("blocks.27", "blocks.30"), "L17": ("blocks.17",),
    "L28": ("blocks.28",), "L29": ("blocks.29",), "D27_31": ("blocks.27", "blocks.31"), "L34": ("blocks.34",),
    "L38": ("blocks.38",), "L41": ("blocks.41",), "L45": ("blocks.45",), "L48": ("blocks.48",),
    "L2": ("blocks.2",),
}


def read_drafter_checkpoint(ckpt, target_hidden: int):
    """A drafter checkpoint (path or loaded dict) -> (DrafterConfig, fp32 state dict, layers, meta)."""
    ck = torch.load(ckpt, map_location="cpu") if not isinstance(ckpt, dict) else ckpt
    for key in ("scheme", "d_model", "gamma", "state_dict"):
        if key not in ck:
            raise ValueError(f"drafter checkpoint has no {key!r} entry")
    scheme = ck["scheme"]
    if scheme not in SCHEME_LAYERS:
        raise ValueError(f"unknown scheme={scheme}; known {tuple(SCHEME_LAYERS)}")
    layers = SCHEME_LAYERS[scheme]
    sd = {k: v.detach().to(torch.float32).contiguous() for k, v in ck["state_dict"].items()}
    n_layers = len({k.split(".")[1] for k in sd if k.startswith("layers.")})
    dcfg = DrafterConfig(d_model=int(ck["d_model"]), gamma=int(ck["gamma"]), inject_layers=layers,
                         target_hidden=int(sd["embed.weight"].shape[1]), n_layers=n_layers,
                         ctx_window=int(ck.get("ctx_window", 64)), mask_id=int(ck.get("mask_id", 256)))
    if dcfg.target_hidden != target_hidden:
        raise ValueError(f"drafter target_hidden {dcfg.target_hidden} != model d_model {target_hidden}")
    meta = {k: v for k, v in ck.items() if k != "state_dict"}
    return dcfg, sd, layers, meta


def _filter_rows(t: torch.Tensor, rows: int, name: str) -> torch.Tensor:
    """[G, (1,) K] or [G, S, 1] per-group filter -> [rows, K]: group g covers rows g*rows/G .. ."""
    if t.dim() == 3:
        t = t.squeeze(1) if t.shape[1] == 1 else t.squeeze(-1)
    if t.dim() != 2 or rows % t.shape[0]:
        raise ValueError(f"{name}: cannot spread {tuple(t.shape)} over {rows} channels")
    if t.shape[0] != rows:
        t = t.repeat_interleave(rows // t.shape[0], 0)
    return t.contiguous()


def _no_bias(sd: dict, name: str) -> None:
    b = sd.get(name)
    if b is not None and bool(torch.any(b != 0)):
        raise ValueError(f"{name}: the target's dense projections and short filters carry no bias")


def target_weights_from_vortex(cfg: TargetConfig, sd: dict) -> dict[str, torch.Tensor]:
    """A vortex StripedHyena state dict -> this library's weight names, shapes and storage dtypes."""
    from .weights import data_dtype, target_weight_specs

    d = cfg.d_model
    out: dict[str, torch.Tensor] = {"embed": sd["embedding_layer.weight"], "final_norm": sd["norm.scale"]}
    if "unembed.weight" in sd and not torch.equal(sd["unembed.weight"], sd["embedding_layer.weight"]):
        raise ValueError("unembed.weight differs from embedding_layer.weight: the unembedding is tied")
    for i, kind in enumerate(cfg.layer_types):
        p, q = f"blocks.{i}.", f"blocks.{i}."
        out[q + "pre_norm"] = sd[p + "pre_norm.scale"]
        out[q + "post_norm"] = sd[p + "post_norm.scale"]
        if kind == MHA:
            out[q + "w_qkv"] = sd[p + "inner_mha_cls.Wqkv.weight"]
            out[q + "w_o"] = sd[p + "inner_mha_cls.out_proj.weight"]
            _no_bias(sd, p + "inner_mha_cls.Wqkv.bias")
            _no_bias(sd, p + "inner_mha_cls.out_proj.bias")
        else:
            out[q + "w_in"] = sd[p + "projections.weight"]
            out[q + "w_out"] = sd[p + "out_filter_dense.weight"]
            out[q + "short_w"] = _filter_rows(sd[p + "filter.short_filter_weight"], 3 * d, "short_filter_weight")
            for b in ("projections.bias", "out_filter_dense.bias", "filter.short_filter_bias"):
                _no_bias(sd, p + b)
            if kind in (HCS, HCM):
                out[q + "inner_w"] = _filter_rows(sd[p + "filter.h"], d, "h")
            if kind in (HCM, HCL):
                out[q + "D"] = sd[p + "filter.D"].reshape(-1)
            if kind == HCL:
                out[q + "log_poles"] = _filter_rows(sd[p + "filter.log_poles"], d, "log_poles")
                out[q + "residues"] = _filter_rows(sd[p + "filter.residues"], d, "residues")
        for src, dst in (("mlp.l1.weight", "w1"), ("mlp.l2.weight", "w2"), ("mlp.l3.weight", "w3")):
            out[q + dst] = sd[p + src]
    res = {}
    for name, shape, _, storage in target_weight_specs(cfg):
        t = out[name]
        if tuple(t.shape) != tuple(shape):
            raise ValueError(f"{name}: shape {tuple(t.shape)} != {tuple(shape)}")
        res[name] = t.detach().to(data_dtype(cfg) if storage == "data" else torch.float32).contiguous()
    return res


def vortex_state_dict(cfg: TargetConfig, weights: dict[str, torch.Tensor], groups: int | None = None) -> dict:
    """The inverse map (this library's names -> vortex names), with per-group filters when
    ``groups`` divides d and every group's channels share one filter (for tests and export)."""
    d = cfg.d_model
    G = groups or d

    def grouped(t: torch.Tensor) -> torch.Tensor:
        return t[:: d // G].contiguous()

    sd = {"embedding_layer.weight": weights["embed"], "norm.scale": weights["final_norm"],
          "unembed.weight": weights["embed"]}
    for i, kind in enumerate(cfg.layer_types):
        p = f"blocks.{i}."
        sd[p + "pre_norm.scale"] = weights[p + "pre_norm"]
        sd[p + "post_norm.scale"] = weights[p + "post_norm"]
        if kind == MHA:
            sd[p + "inner_mha_cls.Wqkv.weight"] = weights[p + "w_qkv"]
            sd[p + "inner_mha_cls.out_proj.weight"] = weights[p + "w_o"]
        else:
            sd[p + "projections.weight"] = weights[p + "w_in"]
            sd[p + "out_filter_dense.weight"] = weights[p + "w_out"]
            sd[p + "filter.short_filter_weight"] = weights[p + "short_w"][:, None, :]
            if kind in (HCS, HCM):
                sd[p + "filter.h"] = grouped(weights[p + "inner_w"])[:, None, :]
            if kind in (HCM, HCL):
                sd[p + "filter.D"] = weights[p + "D"]
            if kind == HCL:
                sd[p + "filter.log_poles"] = grouped(weights[p + "log_poles"])[:, :, None]
                sd[p + "filter.residues"] = grouped(weights[p + "residues"])
        sd[p + "mlp.l1.weight"] = weights[p + "w1"]
        sd[p + "mlp.l2.weight"] = weights[p + "w2"]
        sd[p + "mlp.l3.weight"] = weights[p + "w3"]
    return sd


__all__ = ["SCHEME_LAYERS", "read_drafter_checkpoint", "target_weights_from_vortex", "vortex_state_dict"]
