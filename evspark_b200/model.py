"""StripedHyena2 target on one B200, driven through libevspark_sm100.

``TargetModel`` plays the role of vortex's ``StripedHyena`` for the EvSpark block path:
``model(ids, inference_params_dict) -> (logits, None)`` and
``model.initialize_inference_params(max_seqlen)`` (used at evspark/specdec/block/driver.py:55
and evspark/specdec/block/loop.py:341).  Weights live in HBM as torch tensors (plumbing);
every forward is a single ``evs_prefill`` / ``evs_forward`` call into the CUDA library.

``InferenceParams`` is the 4-key state container of the reference (``mha, hcl, hcm, hcs``,
driver.py:22) backed by one device state handle.  Each key exposes ``seqlen_offset`` and
read-only vortex-layout views (``fir_state_dict``, ``fir_inner_state_dict``, ``state_dict``,
``key_value_memory_dict``) exported from the device arenas on access.
"""

from __future__ import annotations

import ctypes as C
import itertools
from collections.abc import Mapping

import numpy as np
import torch

from . import _native as N
from .config import HCL, HCM, HCS, LAYER_CODE, MHA, TargetConfig
from .weights import data_dtype, init_target_weights

PARAM_KEYS = ("mha", "hcl", "hcm", "hcs")
_uid = itertools.count(1)


def require_device(device) -> torch.device:
    device = torch.device(device)
    if device.type != "cuda" or not torch.cuda.is_available():
        raise RuntimeError("evspark_b200 runs on a CUDA B200 (sm_100a); no CUDA device is available")
    with torch.cuda.device(device):
        N.call("evs_device_check")
    return device


class _Config:
    """Attribute + ``get`` access to the model config (the reference reads both styles)."""

    def __init__(self, cfg: TargetConfig):
        self._cfg = cfg
        self.hidden_size = cfg.d_model
        self.vocab_size = cfg.vocab_size
        self.max_batch_size = cfg.max_batch_size
        self.use_flash_attn = True  # per-row KV lengths are always honoured
        self.state_size = cfg.state_size

    def get(self, key, default=None):
        if key in self.__dict__:
            return self.__dict__[key]
        return getattr(self._cfg, key, default)

    def __getattr__(self, key):
        return getattr(self._cfg, key)


class TargetModel:
    def __init__(self, cfg: TargetConfig, weights: dict[str, torch.Tensor], *, capture_layers=(),
                 device="cuda:0", max_chunk: int = 32, tp: tuple[int, int] | None = None):
        """``tp=(rank, world)`` builds rank ``rank`` of a channel-sharded model: ``weights`` are then this
        rank's shards (``evspark_b200.tp.shard_target_weights``) and every rank runs the same calls."""
        self.device = require_device(device)
        self.cfg = cfg
        self.config = _Config(cfg)
        self.max_chunk = int(max_chunk)
        self.capture_layers = tuple(int(x) for x in capture_layers)
        self.tp_rank, self.tp_world = (int(tp[0]), int(tp[1])) if tp else (0, 1)
        if len(self.capture_layers) > 4:
            raise ValueError("at most 4 capture (injection) layers")
        dd = data_dtype(cfg)
        self.weights = {}
        for k, v in weights.items():
            want = torch.float32 if v.dtype == torch.float32 else dd
            self.weights[k] = v.detach().to(device=self.device, dtype=want).contiguous()
        mc = N.ModelConfig()
        mc.vocab_size, mc.d_model, mc.n_layers = cfg.vocab_size, cfg.d_model, cfg.n_layers
        mc.n_heads, mc.head_dim, mc.mlp_inner, mc.state_size = cfg.n_heads, cfg.head_dim, cfg.mlp_inner, cfg.state_size
        mc.short_filter_length, mc.hcs_filter_length = cfg.short_filter_length, cfg.hcs_filter_length
        mc.hcm_filter_length = cfg.hcm_filter_length
        mc.dtype = N.EVS_DTYPE_BF16 if cfg.dtype == "bf16" else N.EVS_DTYPE_FP32
        mc.eps, mc.rope_base = cfg.eps, cfg.rope_base
        for i, k in enumerate(cfg.layer_types):
            mc.layer_kind[i] = LAYER_CODE[k]
        for j in range(4):
            mc.capture_layers[j] = self.capture_layers[j] if j < len(self.capture_layers) else -1
        mc.tp_world, mc.tp_rank = self.tp_world, self.tp_rank
        h = C.c_void_p()
        with torch.cuda.device(self.device):
            N.check(N.lib().evs_model_create(C.byref(mc), C.byref(h)), "evs_model_create")
            self._h = h
            for name, t in self.weights.items():
                if name in ("embed", "final_norm"):
                    layer, slot = -1, N.SLOTS[name]
                else:
                    _, li, nm = name.split(".", 2)
                    layer, slot = int(li), N.SLOTS[nm]
                N.check(N.lib().evs_model_set_tensor(h, layer, slot, t.data_ptr(), t.numel()), name)
            N.check(N.lib().evs_model_finalize(h), "evs_model_finalize")

    @classmethod
    def random(cls, cfg: TargetConfig, seed: int = 20260820, device="cuda:0", *, init_on="cpu", **kw):
        """Seeded random-init weights (drawn on ``init_on``: 'cpu' to share weights with a CPU
        reference run, 'cuda' for speed at 7B scale)."""
        gen_dev = device if init_on == "cuda" else "cpu"
        tp = kw.get("tp")
        if tp and int(tp[1]) > 1:
            from .tp import init_target_weights_sharded

            w = init_target_weights_sharded(cfg, int(tp[0]), int(tp[1]), seed=seed, device=gen_dev)
        else:
            w = init_target_weights(cfg, seed=seed, device=gen_dev)
        return cls(cfg, w, device=device, **kw)

    @property
    def handle(self):
        return self._h

    def initialize_inference_params(self, max_seqlen: int, *, max_batch: int | None = None,
                                    max_chunk: int | None = None) -> "InferenceParams":
        mb = int(max_batch if max_batch is not None else (self.config.max_batch_size or 1))
        return InferenceParams(self, mb, int(max_seqlen), int(max_chunk or self.max_chunk))

    def __call__(self, ids, inference_params_dict=None, padding_mask=None):
        ids = torch.as_tensor(ids, device=self.device).long()
        if ids.dim() == 1:
            ids = ids[None]
        if inference_params_dict is None:
            ip = self.initialize_inference_params(ids.shape[1] + 1, max_batch=ids.shape[0])
            out = ip.prefill(ids)
            ip.close()
            return out, None
        ip = inference_params_dict
        if ip.offset == 0:
            return ip.prefill(ids), None
        return ip.forward(ids, retain=False), None

    def close(self):
        if getattr(self, "_h", None):
            N.lib().evs_model_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class _StateView(Mapping):
    """layer -> vortex-layout state tensor (exported on access, rows [0, batch))."""

    def __init__(self, ip: "InferenceParams", layers: list[int], which: int):
        self._ip, self._layers, self._which = ip, layers, which

    def __getitem__(self, layer):
        if layer not in self._layers:
            raise KeyError(layer)
        return self._ip.export(layer, self._which)

    def __iter__(self):
        return iter(self._layers if self._ip.offset > 0 else [])

    def __len__(self):
        return len(self._layers) if self._ip.offset > 0 else 0


class _KeyParams:
    def __init__(self, ip: "InferenceParams", key: str):
        self._ip, self._key = ip, key
        cfg = ip.model.cfg
        if key == MHA:
            self.key_value_memory_dict = _StateView(ip, cfg.layer_idxs(MHA), 3)
        else:
            layers = cfg.layer_idxs(key)
            self.fir_state_dict = _StateView(ip, layers, 0)
            self.fir_inner_state_dict = _StateView(ip, layers if key in (HCS, HCM) else [], 1)
            self.state_dict = _StateView(ip, layers if key == HCL else [], 2)
            self.fir_filter_length = cfg.filter_length(key) or cfg.short_filter_length
            self.state_dim = cfg.state_size

    @property
    def seqlen_offset(self) -> int:
        return self._ip.offset

    @seqlen_offset.setter
    def seqlen_offset(self, value: int) -> None:
        self._ip.set_offset(int(value))

    @property
    def max_batch_size(self) -> int:
        return self._ip.max_batch

    @property
    def max_seqlen(self) -> int:
        return self._ip.max_seqlen

    @property
    def lengths_per_sample(self):
        return torch.as_tensor(self._ip.lengths[: self._ip.max_batch], dtype=torch.int32, device=self._ip.model.device)


class InferenceParams(dict):
    """Device state of up to ``max_batch`` independent rows, viewed as the reference's 4 keys."""

    def __init__(self, model: TargetModel, max_batch: int, max_seqlen: int, max_chunk: int):
        super().__init__()
        self.model = model
        self.max_batch, self.max_seqlen, self.max_chunk = max_batch, max_seqlen, max_chunk
        self.batch = 1  # rows in use
        self.lengths = np.zeros(max_batch, dtype=np.int64)  # exact host mirror of the device lengths
        self.retained_uid = 0  # id of the last retained forward (ChunkStash validity)
        self.retained_len0 = None
        self.retained_chunk = 0
        h = C.c_void_p()
        with torch.cuda.device(model.device):
            N.check(N.lib().evs_state_create(model.handle, max_batch, max_seqlen, max_chunk, C.byref(h)),
                    "evs_state_create")
        self._h = h
        if model.tp_world > 1:  # collective: every rank creates its state in the same order
            from .tp import connect_state

            connect_state(h, N.lib(), model.tp_world, model.device)
        for k in PARAM_KEYS:
            dict.__setitem__(self, k, _KeyParams(self, k))

    # -- bookkeeping -------------------------------------------------------
    @property
    def handle(self):
        return self._h

    @property
    def offset(self) -> int:
        return int(self.lengths[: self.batch].max())

    def _stream(self):
        return N.stream_ptr()

    def set_offset(self, value: int) -> None:
        if value < 0 or value > self.max_seqlen:
            raise ValueError(f"seqlen_offset {value} outside [0, {self.max_seqlen}]")
        self.set_lengths(np.full(self.batch, value, dtype=np.int64))

    def set_lengths(self, lengths) -> None:
        lengths = np.asarray(lengths, dtype=np.int64).ravel()
        b = lengths.size
        arr = (C.c_int32 * b)(*[int(x) for x in lengths])
        N.check(N.lib().evs_state_set_lengths(self._h, arr, b, self._stream()), "evs_state_set_lengths")
        self.lengths[:b] = lengths
        if np.all(self.lengths[:b] == 0):
            self.retained_uid = 0

    def device_lengths(self, batch: int | None = None) -> np.ndarray:
        b = int(batch or self.batch)
        arr = (C.c_int32 * b)()
        N.check(N.lib().evs_state_get_lengths(self._h, arr, b, self._stream()), "evs_state_get_lengths")
        return np.array(arr[:], dtype=np.int64)

    # -- forward passes ------------------------------------------------------
    def prefill(self, ids: torch.Tensor, last_only: bool = False) -> torch.Tensor:
        ids = ids.to(self.model.device).long().contiguous()
        B, T = ids.shape
        if B > self.max_batch:
            raise ValueError(f"batch {B} > max_batch {self.max_batch}")
        V = self.model.cfg.vocab_size
        logits = torch.empty((B, V) if last_only else (B, T, V), dtype=torch.float32, device=self.model.device)
        N.check(N.lib().evs_prefill(self.model.handle, self._h, ids.data_ptr(), B, T, logits.data_ptr(),
                                    int(last_only), self._stream()), "evs_prefill")
        self.batch = B
        self.lengths[:B] += T
        self.retained_uid = 0
        return logits

    def forward(self, ids: torch.Tensor, retain: bool = False) -> torch.Tensor:
        ids = ids.to(self.model.device).long().contiguous()
        B, T = ids.shape
        if B > self.max_batch:
            raise ValueError(f"batch {B} > max_batch {self.max_batch}")
        V = self.model.cfg.vocab_size
        logits = torch.empty((B, T, V), dtype=torch.float32, device=self.model.device)
        N.check(N.lib().evs_forward(self.model.handle, self._h, ids.data_ptr(), B, T, int(retain), logits.data_ptr(),
                                    self._stream()), "evs_forward")
        self.batch = B
        if retain:
            self.retained_uid = next(_uid)
            self.retained_len0 = self.lengths[:B].copy()
            self.retained_chunk = T
        else:
            self.retained_uid = 0
        self.lengths[:B] += T
        return logits

    def rollback_launch(self, k_dev: torch.Tensor) -> None:
        """Device-side rollback of the last retained forward to the per-row block indices in the int32
        device tensor ``k_dev`` (no host copy).  The host mirror follows with ``note_rollback``."""
        N.check(N.lib().evs_rollback(self._h, k_dev.data_ptr(), int(k_dev.numel()), self._stream()), "evs_rollback")

    def note_rollback(self, ks) -> None:
        """Host mirror of a ``rollback_launch`` whose block indices are now known on the host."""
        ks = np.asarray(ks, dtype=np.int64).ravel()
        self.lengths[: ks.size] = self.retained_len0[: ks.size] + ks + 1
        arr = (C.c_int32 * ks.size)(*[int(x) for x in self.lengths[: ks.size]])
        N.check(N.lib().evs_state_note_lengths(self._h, arr, ks.size), "evs_state_note_lengths")

    def rollback(self, ks: np.ndarray) -> None:
        ks = np.asarray(ks, dtype=np.int64).ravel()
        kd = torch.as_tensor(ks.astype(np.int32), device=self.model.device)
        N.check(N.lib().evs_rollback(self._h, kd.data_ptr(), ks.size, self._stream()), "evs_rollback")
        self.lengths[: ks.size] = self.retained_len0[: ks.size] + ks + 1
        arr = (C.c_int32 * ks.size)(*[int(x) for x in self.lengths[: ks.size]])
        N.check(N.lib().evs_state_note_lengths(self._h, arr, ks.size), "evs_state_note_lengths")

    # -- state management ----------------------------------------------------
    def clone(self) -> "InferenceParams":
        other = InferenceParams(self.model, self.max_batch, self.max_seqlen, self.max_chunk)
        N.check(N.lib().evs_state_copy(other._h, self._h, self._stream()), "evs_state_copy")
        other.batch = self.batch
        other.lengths = self.lengths.copy()
        other.retained_uid = self.retained_uid
        other.retained_len0 = None if self.retained_len0 is None else self.retained_len0.copy()
        other.retained_chunk = self.retained_chunk
        return other

    def expand(self, batch: int) -> None:
        N.check(N.lib().evs_state_expand(self._h, batch, self._stream()), "evs_state_expand")
        self.lengths[1:batch] = self.lengths[0]
        self.batch = batch

    def collapse(self, idx: int) -> None:
        N.check(N.lib().evs_state_collapse(self._h, idx, self._stream()), "evs_state_collapse")
        self.lengths[0] = self.lengths[idx]
        self.batch = 1

    def export(self, layer: int, which: int, rows: int | None = None, kv_len: int | None = None) -> torch.Tensor:
        """Vortex-layout tensor of one state for rows [0, rows): FIR states [B, C, S] (ragged
        widths left-zero-padded), IIR [B, d, S], KV [B, kv_len, 2, H, Dh]."""
        cfg = self.model.cfg
        rows = int(rows or self.batch)
        d = cfg.d_model
        kind = cfg.layer_types[layer]
        outs = []
        if which == 3:
            L = int(kv_len if kv_len is not None else self.offset)
            for b in range(rows):
                n = int(self.lengths[b])
                t = torch.zeros(L, 2, cfg.n_heads, cfg.head_dim, dtype=data_dtype(cfg), device=self.model.device)
                if n > 0 and L > 0:
                    tmp = torch.empty(n, 2, cfg.n_heads, cfg.head_dim, dtype=t.dtype, device=t.device)
                    N.check(N.lib().evs_state_export(self._h, layer, 3, b, n, tmp.data_ptr(), self._stream()),
                            "evs_state_export")
                    m = min(L, n)
                    t[:m] = tmp[:m]
                outs.append(t)
            return torch.stack(outs, 0)
        if which in (0, 1):
            K = cfg.short_filter_length if which == 0 else cfg.filter_length(kind)
            C_ = 3 * d if which == 0 else d
            widths = [min(int(self.lengths[b]), K - 1) for b in range(rows)]
            W = max(widths) if widths else 0
            for b in range(rows):
                t = torch.zeros(C_, W, dtype=torch.float32, device=self.model.device)
                if widths[b] > 0:
                    tmp = torch.empty(C_, widths[b], dtype=torch.float32, device=self.model.device)
                    N.check(N.lib().evs_state_export(self._h, layer, which, b, widths[b], tmp.data_ptr(),
                                                     self._stream()), "evs_state_export")
                    t[:, W - widths[b]:] = tmp
                outs.append(t)
            return torch.stack(outs, 0)
        for b in range(rows):
            t = torch.empty(d, cfg.state_size, dtype=torch.float32, device=self.model.device)
            N.check(N.lib().evs_state_export(self._h, layer, 2, b, 0, t.data_ptr(), self._stream()),
                    "evs_state_export")
            outs.append(t)
        return torch.stack(outs, 0)

    def capture_ring(self, slot: int = 0):
        p = C.c_void_p()
        n = C.c_int()
        N.check(N.lib().evs_state_capture_ring(self._h, slot, C.byref(p), C.byref(n)), "evs_state_capture_ring")
        return p.value, n.value

    def device_error(self):
        code, where, info = C.c_int32(), C.c_int32(), C.c_int32()
        N.check(N.lib().evs_get_device_error(self._h, C.byref(code), C.byref(where), C.byref(info)))
        return code.value, where.value, info.value

    def close(self, collective: bool = True):
        """Free the state.  A channel-sharded state closes collectively (every rank calls close):
        no rank frees its shared region while a peer may still read it."""
        if getattr(self, "_h", None):
            torch.cuda.synchronize(self.model.device)
            if self.model.tp_world > 1 and collective:
                from .tp import disconnect_state

                disconnect_state(self._h, N.lib(), self.model.device)
            N.lib().evs_state_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close(collective=False)
        except Exception:
            pass

    def __deepcopy__(self, memo):
        return self.clone()
