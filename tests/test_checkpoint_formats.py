"""CPU: the reference's checkpoint formats.

* A drafter ``.pt`` written in the reference schema (evspark/train/train_drafter.py:557-571) from
  the reference ``Drafter`` module's own ``state_dict`` reads back to the same parameters, shape and
  injection layers, and the restated drafter trunk gives the golden outputs from it.
* A StripedHyena (vortex-named) state dict with grouped Hyena filters maps onto this library's
  weight names; the oracle run on the mapped weights equals the oracle on the original weights.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from evspark_b200.checkpoint import read_drafter_checkpoint, target_weights_from_vortex, vortex_state_dict
from evspark_b200.config import DRAFTERS, HCL, HCM, HCS, MHA, TINY, TargetConfig
from evspark_b200.weights import init_drafter_weights, init_target_weights


def test_drafter_checkpoint_round_trip(tmp_path, golden):
    from oracle import specdec as sd

    dcfg = DRAFTERS["tiny"]
    tw = init_target_weights(TINY, seed=20260820)
    dw = init_drafter_weights(dcfg, seed=20260830, embed=tw["embed"])
    path = tmp_path / "L2_g12_tiny.pt"
    torch.save({"scheme": "L2", "d_model": dcfg.d_model, "gamma": dcfg.gamma, "ctx_window": dcfg.ctx_window,
                "state_dict": dw, "n_pos": 1234, "mask_id": 256, "offline": True, "dump_dir": "dumps/L2"}, path)
    cfg2, sd2, layers, meta = read_drafter_checkpoint(str(path), TINY.d_model)
    assert layers == ("blocks.2",) and cfg2.inject_layers == layers
    assert (cfg2.d_model, cfg2.gamma, cfg2.n_layers, cfg2.target_hidden) == (128, 12, 2, 256)
    assert meta["n_pos"] == 1234 and meta["mask_id"] == 256 and "state_dict" not in meta
    assert sorted(sd2) == sorted(dw) and all(torch.equal(sd2[k], dw[k]) for k in dw)
    d = golden("drafter_tiny.npz")
    U, _ = sd.drafter_trunk(sd2, cfg2, 71, torch.from_numpy(d["ctx9/h_raw"]), 9)
    np.testing.assert_allclose(U.numpy(), d["ctx9/U"], atol=2e-5, rtol=1e-4)
    with pytest.raises(ValueError, match="target_hidden"):
        read_drafter_checkpoint(str(path), 4096)
    bad = torch.load(path)
    bad["scheme"] = "L99"
    with pytest.raises(ValueError, match="unknown scheme"):
        read_drafter_checkpoint(bad, TINY.d_model)


def test_drafter_checkpoint_from_reference_module(tmp_path):
    """The state_dict of the reference's own Drafter module (not a hand-built dict) reads back;
    runs where EVSPARK_REFERENCE names an EvSpark checkout."""
    import os
    import sys
    from pathlib import Path

    ref = Path(os.environ.get("EVSPARK_REFERENCE", "/nonexistent"))
    if not (ref / "evspark" / "train" / "drafter.py").exists():
        pytest.skip("EVSPARK_REFERENCE does not name an EvSpark checkout")
    sys.path.insert(0, str(ref))
    try:
        from evspark.train.drafter import Drafter
    finally:
        sys.path.remove(str(ref))
    dcfg = DRAFTERS["tiny"]
    m = Drafter(d_model=dcfg.d_model, n_layers=dcfg.n_layers, gamma=dcfg.gamma, n_inject=dcfg.n_inject,
                target_hidden=dcfg.target_hidden, ctx_window=dcfg.ctx_window)
    path = tmp_path / "d.pt"
    torch.save({"scheme": "L2", "d_model": dcfg.d_model, "gamma": dcfg.gamma, "ctx_window": dcfg.ctx_window,
                "state_dict": m.state_dict(), "n_pos": 0, "mask_id": 256, "offline": True, "dump_dir": ""}, path)
    cfg2, sd2, _, _ = read_drafter_checkpoint(str(path), dcfg.target_hidden)
    from evspark_b200.weights import drafter_weight_specs

    assert sorted(n for n, _, _ in drafter_weight_specs(cfg2)) == sorted(sd2)


CFG = TargetConfig(name="vortex_small", d_model=256, n_layers=4, layer_types=(HCS, HCM, HCL, MHA), n_heads=2,
                   head_dim=128, mlp_inner=512, dtype="bf16")


def _grouped_weights(groups: int):
    """Seeded weights whose Hyena filters are shared by each group of d/groups channels."""
    w = init_target_weights(CFG, seed=3)
    rep = CFG.d_model // groups
    for i, kind in enumerate(CFG.layer_types):
        for slot in ("inner_w", "log_poles", "residues"):
            k = f"blocks.{i}.{slot}"
            if k in w:
                w[k] = w[k][::rep].repeat_interleave(rep, 0).contiguous()
    return w


@pytest.mark.parametrize("groups", [256, 16])
def test_vortex_state_dict_maps_to_the_same_model(groups):
    from oracle.model import OracleTarget

    w = _grouped_weights(groups)
    sd = vortex_state_dict(CFG, w, groups=groups)
    assert sd["blocks.0.filter.h"].shape == (groups, 1, 7)
    assert sd["blocks.2.filter.log_poles"].shape == (groups, 16, 1)
    assert sd["blocks.0.filter.short_filter_weight"].shape == (768, 1, 3)
    w2 = target_weights_from_vortex(CFG, sd)
    assert sorted(w2) == sorted(w)
    for k in w:
        assert w2[k].dtype == w[k].dtype and torch.equal(w2[k], w[k]), k
    ids = np.random.default_rng(0).choice([65, 67, 71, 84], size=20)
    outs = []
    for ww in (w, w2):
        o = OracleTarget(CFG, ww)
        st = o.init_state(1, 32)
        outs.append(o.forward(ids[None], st, prefill=True)[0])
    assert torch.equal(outs[0], outs[1])


def test_vortex_state_dict_rejects_what_the_model_cannot_hold():
    w = init_target_weights(CFG, seed=3)
    sd = vortex_state_dict(CFG, w)
    sd["blocks.0.projections.bias"] = torch.ones(768)
    with pytest.raises(ValueError, match="no bias"):
        target_weights_from_vortex(CFG, sd)
    sd = vortex_state_dict(CFG, w)
    sd["unembed.weight"] = sd["unembed.weight"] + 1
    with pytest.raises(ValueError, match="tied"):
        target_weights_from_vortex(CFG, sd)
    sd = vortex_state_dict(CFG, w)
    sd["blocks.1.mlp.l1.weight"] = sd["blocks.1.mlp.l1.weight"][:-1]
    with pytest.raises(ValueError, match="shape"):
        target_weights_from_vortex(CFG, sd)
