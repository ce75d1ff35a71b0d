"""Channel sharding of the target over GPUs (one process per GPU, ``torch.distributed`` ranks).

Hyena filters are depthwise, so a rank owns a contiguous block of d/world channels h0..h1 and
everything that belongs to them: the in-projection rows 3h..3h+2 (the interleaved x2/x1/v
triplet of channel h), the short filter rows, the inner FIR taps, D, the IIR poles and residues,
and the FIR/IIR state of those channels.  Attention heads split the same way (d/world channels
= n_heads/world heads, their q, k and v rows); the MLP splits its F features.  The projections
back to the residual stream (Hyena out-projection, attention o-projection, w3) are row-parallel:
each rank multiplies its input columns and the library adds the ranks' partial sums inside the
following residual + RMSNorm, reading the peers' buffers over NVLink in rank order.  Norms, the
embedding, the tied unembedding and the drafter are replicated, so every rank holds the same
residual stream, logits and draft, and verification needs no exchange.
"""

from __future__ import annotations

import ctypes as C

import torch

from .config import TargetConfig
from .weights import _draw, data_dtype, target_weight_specs


def _bounds(n: int, rank: int, world: int) -> tuple[int, int]:
    if n % world:
        raise ValueError(f"{n} does not split over {world} ranks")
    k = n // world
    return rank * k, (rank + 1) * k


def shard_tensor(cfg: TargetConfig, name: str, t: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """This rank's part of the full weight ``name`` (layout of ``target_weight_specs``)."""
    if world == 1:
        return t
    d, F = cfg.d_model, cfg.mlp_inner
    h0, h1 = _bounds(d, rank, world)
    f0, f1 = _bounds(F, rank, world)
    slot = name.rsplit(".", 1)[-1]
    if slot in ("embed", "final_norm", "pre_norm", "post_norm"):
        return t
    if slot in ("w_in", "short_w"):  # rows 3h + j of the channels h0..h1
        return t[3 * h0:3 * h1].contiguous()
    if slot in ("inner_w", "D", "log_poles", "residues"):
        return t[h0:h1].contiguous()
    if slot in ("w_out", "w_o"):  # row-parallel: input columns of the local channels
        return t[:, h0:h1].contiguous()
    if slot == "w_qkv":  # q, k and v rows of the local heads
        return torch.cat([t[h0:h1], t[d + h0:d + h1], t[2 * d + h0:2 * d + h1]]).contiguous()
    if slot in ("w1", "w2"):
        return t[f0:f1].contiguous()
    if slot == "w3":
        return t[:, f0:f1].contiguous()
    raise ValueError(f"no sharding rule for {name}")


def shard_target_weights(cfg: TargetConfig, weights: dict[str, torch.Tensor], rank: int,
                         world: int) -> dict[str, torch.Tensor]:
    return {k: shard_tensor(cfg, k, v, rank, world) for k, v in weights.items()}


def unshard_target_weights(cfg: TargetConfig, shards: list[dict[str, torch.Tensor]]) -> dict[str, torch.Tensor]:
    """Inverse of ``shard_target_weights`` over all ranks (shards in rank order)."""
    world = len(shards)
    d = cfg.d_model
    out = {}
    for name in shards[0]:
        parts = [s[name] for s in shards]
        slot = name.rsplit(".", 1)[-1]
        if slot in ("embed", "final_norm", "pre_norm", "post_norm"):
            out[name] = parts[0]
        elif slot in ("w_out", "w_o", "w3"):
            out[name] = torch.cat(parts, dim=1)
        elif slot == "w_qkv":
            dl = d // world
            out[name] = torch.cat([p[j * dl:(j + 1) * dl] for j in range(3) for p in parts])
        else:
            out[name] = torch.cat(parts, dim=0)
    return out


def init_target_weights_sharded(cfg: TargetConfig, rank: int, world: int, seed: int = 20260820,
                                device="cpu") -> dict[str, torch.Tensor]:
    """This rank's part of ``init_target_weights(cfg, seed, device)``: every full tensor is drawn
    with its own seed and cut immediately, so at most one full tensor exists at a time."""
    device = torch.device(device)
    out: dict[str, torch.Tensor] = {}
    for idx, (name, shape, kind, storage) in enumerate(target_weight_specs(cfg)):
        gen = torch.Generator(device=device)
        gen.manual_seed(int(seed) * 1_000_003 + idx)
        t = _draw(kind, shape, gen, device, cfg).to(data_dtype(cfg) if storage == "data" else torch.float32)
        out[name] = shard_tensor(cfg, name, t, rank, world).contiguous()
        del t
    return out


def connect_state(state_handle, lib, world: int, device) -> None:
    """Exchange the states' shared-region handles over the default process group (collective)."""
    import torch.distributed as dist

    from . import _native as N

    h = (C.c_char * 64)()
    N.check(lib.evs_state_tp_handle(state_handle, h), "evs_state_tp_handle")
    mine = bytes(h)
    allh: list = [None] * world
    dist.all_gather_object(allh, mine)
    buf = (C.c_char * (64 * world)).from_buffer_copy(b"".join(allh))
    dev = torch.device(device)
    if dev.type == "cuda":
        with torch.cuda.device(dev):
            N.check(lib.evs_state_tp_connect(state_handle, buf, world), "evs_state_tp_connect")
    else:
        N.check(lib.evs_state_tp_connect(state_handle, buf, world), "evs_state_tp_connect")


def disconnect_state(state_handle, lib, device) -> None:
    """Collective: every rank stops using its peers' regions before any rank frees its own."""
    import torch.distributed as dist

    from . import _native as N

    if torch.device(device).type == "cuda":
        torch.cuda.synchronize(device)
    dist.barrier()
    N.check(lib.evs_state_tp_disconnect(state_handle), "evs_state_tp_disconnect")
    dist.barrier()


__all__ = ["connect_state", "disconnect_state", "init_target_weights_sharded", "shard_target_weights",
           "shard_tensor", "unshard_target_weights"]
