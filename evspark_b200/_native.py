"""ctypes binding of ``libevspark_sm100.so`` (include/evspark_sm100.h).

The library is the only compute path: if it is missing or fails to load, every
device entry point raises immediately — there is no fallback.
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libevspark_sm100.so"

EVS_OK, EVS_EINVAL, EVS_ERANGE, EVS_ETIMEOUT, EVS_ECUDA, EVS_ENODEV, EVS_EDEVICE = range(7)
EVS_MAX_LAYERS = 64
EVS_DTYPE_FP32, EVS_DTYPE_BF16 = 0, 1

# evs_slot
SLOTS = {
    "embed": 0, "final_norm": 1, "pre_norm": 2, "post_norm": 3, "w_in": 4, "short_w": 5, "inner_w": 6, "D": 7,
    "log_poles": 8, "residues": 9, "w_out": 10, "w_qkv": 11, "w_o": 12, "w1": 13, "w2": 14, "w3": 15,
}

# evs_drafter_tensor
D_IDS = {
    "embed.weight": 0, "in_proj.weight": 1, "in_proj.bias": 2, "out_proj.weight": 3, "out_proj.bias": 4,
    "pos.weight": 5, "ctx_proj.weight": 6, "ctx_proj.bias": 7, "ctx_norm.scale": 8, "final_ln.scale": 9,
    "markov": 10, "conf_w.weight": 11, "conf_w.bias": 12,
}
D_LAYER0, D_PER_LAYER = 16, 10
D_LAYER_IDS = {"ln1.scale": 0, "q_proj.weight": 1, "k_proj.weight": 2, "v_proj.weight": 3, "o_proj.weight": 4,
               "ln2.scale": 5, "mlp.0.weight": 6, "mlp.0.bias": 7, "mlp.2.weight": 8, "mlp.2.bias": 9}


def drafter_tensor_id(name: str) -> int:
    if name in D_IDS:
        return D_IDS[name]
    if name.startswith("layers."):
        _, l, rest = name.split(".", 2)
        return D_LAYER0 + int(l) * D_PER_LAYER + D_LAYER_IDS[rest]
    raise KeyError(name)


class ModelConfig(C.Structure):
    _fields_ = [
        ("vocab_size", C.c_int32), ("d_model", C.c_int32), ("n_layers", C.c_int32), ("n_heads", C.c_int32),
        ("head_dim", C.c_int32), ("mlp_inner", C.c_int32), ("state_size", C.c_int32),
        ("short_filter_length", C.c_int32), ("hcs_filter_length", C.c_int32), ("hcm_filter_length", C.c_int32),
        ("dtype", C.c_int32), ("eps", C.c_float), ("rope_base", C.c_float),
        ("layer_kind", C.c_int32 * EVS_MAX_LAYERS), ("capture_layers", C.c_int32 * 4),
        ("tp_world", C.c_int32), ("tp_rank", C.c_int32),
    ]


class DrafterConfig(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("d_model", "n_layers", "n_heads", "gamma", "n_inject", "target_hidden",
                                          "vocab_size", "mask_id", "ctx_window", "mlp_mult")]


_P = C.c_void_p
_I = C.c_int
_PROTOS = {
    "evs_version": (_I, []),
    "evs_last_error": (C.c_char_p, []),
    "evs_device_check": (_I, []),
    "evs_model_create": (_I, [C.POINTER(ModelConfig), C.POINTER(_P)]),
    "evs_model_set_tensor": (_I, [_P, _I, _I, _P, C.c_int64]),
    "evs_model_finalize": (_I, [_P]),
    "evs_model_destroy": (None, [_P]),
    "evs_state_create": (_I, [_P, _I, _I, _I, C.POINTER(_P)]),
    "evs_state_tp_handle": (_I, [_P, _P]),
    "evs_state_tp_connect": (_I, [_P, _P, _I]),
    "evs_state_tp_disconnect": (_I, [_P]),
    "evs_state_destroy": (None, [_P]),
    "evs_state_reset": (_I, [_P, _P]),
    "evs_state_copy": (_I, [_P, _P, _P]),
    "evs_state_get_lengths": (_I, [_P, _P, _I, _P]),
    "evs_state_set_lengths": (_I, [_P, _P, _I, _P]),
    "evs_state_note_lengths": (_I, [_P, _P, _I]),
    "evs_state_expand": (_I, [_P, _I, _P]),
    "evs_state_collapse": (_I, [_P, _I, _P]),
    "evs_state_export": (_I, [_P, _I, _I, _I, _I, _P, _P]),
    "evs_state_capture_ring": (_I, [_P, _I, C.POINTER(_P), C.POINTER(_I)]),
    "evs_prefill": (_I, [_P, _P, _P, _I, _I, _P, _I, _P]),
    "evs_forward": (_I, [_P, _P, _P, _I, _I, _I, _P, _P]),
    "evs_rollback": (_I, [_P, _P, _I, _P]),
    "evs_transform": (_I, [_P, _I, _I, _I, C.c_double, _I, _P, _P]),
    "evs_verify": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _P, _P, _P, _P]),
    "evs_verify_multicand": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _P, _P, _P]),
    "evs_sample": (_I, [_P, _I, _I, _P, _P, _P]),
    "evs_gemm_bf16": (_I, [_P, _P, _P, _I, _I, _I, _I, _P]),
    "evs_gemm_bf16_noalloc": (_I, [_P, _P, _P, _I, _I, _I, _P]),
    "evs_drafter_create": (_I, [C.POINTER(DrafterConfig), _I, C.POINTER(_P)]),
    "evs_drafter_set_tensor": (_I, [_P, _I, _P, C.c_int64]),
    "evs_drafter_finalize": (_I, [_P]),
    "evs_drafter_destroy": (None, [_P]),
    "evs_draft_propose": (_I, [_P, _P, _P, _I, _I, _I, C.c_double, _I, _P, _P, _P, _P, _P, _P, _P]),
    "evs_profile_start": (_I, [_P]),
    "evs_profile_stop": (_I, [_P, _P, _P, _P]),
    "evs_launch_count": (C.c_int64, []),
    "evs_get_device_error": (_I, [_P, C.POINTER(C.c_int32), C.POINTER(C.c_int32), C.POINTER(C.c_int32)]),
    "evs_clear_device_error": (_I, [_P, _P]),
}

_lib = None


def exported_symbols() -> list[str]:
    return list(_PROTOS)


def lib():
    """Load the library (once) and attach prototypes; raises if it is missing."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH.name} is not built: run `python -m evspark_b200.build` (nvcc, sm_100a). "
                "The CUDA extension is the only compute path of evspark_b200.")
        h = C.CDLL(str(LIB_PATH))
        for name, (res, args) in _PROTOS.items():
            f = getattr(h, name)
            f.restype = res
            f.argtypes = args
        _lib = h
    return _lib


class EvsError(RuntimeError):
    pass


def check(status: int, what: str = "") -> None:
    if status == EVS_OK:
        return
    msg = lib().evs_last_error().decode("utf-8", "replace")
    text = f"{what}: {msg}" if what else msg
    if status in (EVS_EINVAL, EVS_ERANGE):
        raise ValueError(text)
    raise EvsError(f"[evs status {status}] {text}")


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)


# kernels of this library launched by CUDA-graph replays (the library's own counter sees only the
# launches its entry points issue): graph replays add the launch count of the captured call
_replayed = 0


def note_replayed(n: int) -> None:
    global _replayed
    _replayed += int(n)


def launch_count() -> int:
    """Kernels of this library launched so far: by its entry points and by graph replays."""
    return int(lib().evs_launch_count()) + _replayed


# host <-> device bytes copied by the decode loop and the facade (the tensors they copy, counted
# where the copy is issued): what one generate call moves across PCIe
_h2d = 0
_d2h = 0


def note_transfer(h2d: int = 0, d2h: int = 0) -> None:
    global _h2d, _d2h
    _h2d += int(h2d)
    _d2h += int(d2h)


def transfer_count() -> tuple[int, int]:
    """(host-to-device, device-to-host) bytes noted so far."""
    return _h2d, _d2h


def ptr(t) -> int | None:
    """Device (or host) address of a torch tensor / None."""
    if t is None:
        return None
    return t.data_ptr()


def stream_ptr(stream=None):
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream
