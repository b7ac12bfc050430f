"""ctypes binding of libb2e.so (include/b2e.h).

The library is built in-tree by hackathon_b200.build. There is no fallback: if it
is missing or does not load, every entry point raises B2ELibraryError.
"""

from __future__ import annotations

import ctypes as C
import os
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libb2e.so"

B2E_OK = 0
DTYPES = {"fp32": 0, "bf16": 1, "fp16": 2}
LAYER_KINDS = {"xlstm": 0, "mamba2": 1, "retnet": 2, "hawk": 3}
FLAG_NO_PDL = 1         # B2E_FLAG_NO_PDL
FLAG_NO_PRIORITIES = 2  # B2E_FLAG_NO_PRIORITIES
FLAG_NO_LATENCY_PATH = 4  # B2E_FLAG_NO_LATENCY_PATH
FLAG_NO_PIPELINE = 8  # B2E_FLAG_NO_PIPELINE


class B2ELibraryError(RuntimeError):
    """libb2e.so is missing or failed to load."""


class B2EError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[b2e status {code}] {msg}")
        self.code = code


class ModelConfigC(C.Structure):
    _fields_ = [("hidden_size", C.c_int32), ("proj_size", C.c_int32), ("tower_depth", C.c_int32),
                ("num_heads", C.c_int32), ("num_features", C.c_int32), ("mamba_head_size", C.c_int32),
                ("mamba_bc_size", C.c_int32)]


class EngineOptionsC(C.Structure):
    _fields_ = [("device", C.c_int32), ("linear_dtype", C.c_int32), ("capacity", C.c_int32),
                ("max_batch", C.c_int32), ("use_graphs", C.c_int32), ("lanes", C.c_int32),
                ("lane_min_rows", C.c_int32), ("flags", C.c_int32), ("lane_towers", C.c_int32)]


class TensorC(C.Structure):
    _fields_ = [("name", C.c_char_p), ("data", C.c_void_p), ("numel", C.c_int64)]


_P = C.c_void_p
_I32 = C.c_int32
_I64 = C.c_int64
_PI64 = C.POINTER(C.c_int64)
_PI32 = C.POINTER(C.c_int32)

# name -> (restype, argtypes)
_SIGS = {
    "b2e_last_error": (C.c_char_p, []),
    "b2e_version": (C.c_char_p, []),
    "b2e_engine_create": (C.c_int, [C.POINTER(ModelConfigC), C.POINTER(EngineOptionsC), C.POINTER(TensorC), _I32,
                                    C.POINTER(_P)]),
    "b2e_engine_destroy": (None, [_P]),
    "b2e_engine_step": (C.c_int, [_P, _P, _P, _I32, _P]),
    "b2e_engine_submit": (C.c_int, [_P, _P, _P, _I32]),
    "b2e_engine_wait": (C.c_int, [_P, _P]),
    "b2e_engine_step_device": (C.c_int, [_P, _P, _P, _I32, _P, _P]),
    "b2e_engine_submit_device": (C.c_int, [_P, _P, _P, _I32, _P, _P]),
    "b2e_set_state_kernel_waves": (C.c_int, [_I32, _P]),
    "b2e_engine_join_device": (C.c_int, [_P, _P]),
    "b2e_engine_device_error": (C.c_int, [_P, _PI32]),
    "b2e_engine_reset_slots": (C.c_int, [_P, _P, _I32]),
    "b2e_engine_slot_bytes": (C.c_int, [_P, _PI64]),
    "b2e_engine_read_slot": (C.c_int, [_P, _I32, _P, _I64]),
    "b2e_engine_write_slot": (C.c_int, [_P, _I32, _P, _I64]),
    "b2e_engine_launches": (C.c_int, [_P, _I32, _PI32]),
    "b2e_engine_latency_rows": (C.c_int, [_P, _PI32, _PI32]),
    "b2e_engine_memory": (C.c_int, [_P, _PI64, _PI64]),
    "b2e_mlstm_step": (C.c_int, [_P, _P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _P, _P]),
    "b2e_retnet_step": (C.c_int, [_P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _P, _P]),
    "b2e_mamba2_step": (C.c_int, [_P, _P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _P, _P]),
    "b2e_linear": (C.c_int, [_P, _I32, _I32, _I32, _P, _I32, _P, _I32, _I32, _P, _P, _P]),
    "b2e_linear_static": (C.c_int, [_P, _I32, _I32, _I32, _P, _I32, _P, _I32, _I32, _P, _P, _P]),
    "b2e_layer_create": (C.c_int, [_I32, C.POINTER(ModelConfigC), C.POINTER(EngineOptionsC), C.POINTER(TensorC),
                                   _I32, C.POINTER(_P)]),
    "b2e_layer_destroy": (None, [_P]),
    "b2e_layer_step_device": (C.c_int, [_P, _P, _P, _I32, _P, _P]),
    "b2e_layer_reset_slots": (C.c_int, [_P, _P, _I32]),
    "b2e_layer_slot_bytes": (C.c_int, [_P, _PI64]),
    "b2e_layer_read_slot": (C.c_int, [_P, _I32, _P, _I64]),
    "b2e_layer_write_slot": (C.c_int, [_P, _I32, _P, _I64]),
    "b2e_ingest_create": (C.c_int, [_I32, _I32, C.POINTER(_P)]),
    "b2e_ingest_destroy": (None, [_P]),
    "b2e_ingest_set_threads": (C.c_int, [_P, _I32]),
    "b2e_ingest_feed": (C.c_int, [_P, _P, _I64, _PI32, _PI32]),
    "b2e_ingest_next_other": (C.c_int, [_P, _P, _I64, _PI64]),
    "b2e_ingest_push": (C.c_int, [_P, _I64, _P, _I64, _P, _PI32]),
    "b2e_ingest_next_drop": (C.c_int, [_P, _PI32]),
    "b2e_ingest_pending": (C.c_int, [_P, _PI64]),
    "b2e_ingest_symbol_count": (C.c_int, [_P, _PI32]),
    "b2e_ingest_symbol_name": (C.c_int, [_P, _I32, _P, _I64, _PI64]),
    "b2e_ingest_take": (C.c_int, [_P, _I64, _P, _P, _P, _P, _PI32, _PI64]),
    "b2e_ingest_take_batch": (C.c_int, [_P, _I32, _P, _P, _P, _PI32]),
    "b2e_encode_response": (C.c_int, [_P, _P, _I64, _I32, C.c_double, _P, _I64, _PI64]),
}

_lib = None
_lock = threading.Lock()


def lib():
    """Load libb2e.so once; raise B2ELibraryError if it is absent or broken."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = Path(os.environ.get("B2E_LIB", LIB_PATH))
            if not path.exists():
                raise B2ELibraryError(
                    f"{path} is missing: build it with `python -m hackathon_b200.build` "
                    "(there is no CPU fallback)")
            try:
                handle = C.CDLL(str(path), mode=C.RTLD_GLOBAL)
            except OSError as exc:
                raise B2ELibraryError(f"cannot load {path}: {exc}") from exc
            for name, (res, args) in _SIGS.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def exported_symbols():
    return sorted(_SIGS)


def check(rc: int) -> None:
    if rc != B2E_OK:
        raise B2EError(rc, lib().b2e_last_error().decode("utf-8", "replace"))


def model_config_c(cfg) -> ModelConfigC:
    return ModelConfigC(cfg.hidden_size, cfg.proj_size, cfg.tower_depth, cfg.num_heads, cfg.num_features,
                        cfg.mamba_head_size, cfg.mamba_bc_size)


def tensor_array(sd):
    """(ctypes TensorC array, keep-alive list) for a name -> float32 array dict."""
    import numpy as np

    keep = []
    arr = (TensorC * len(sd))()
    for i, (name, val) in enumerate(sd.items()):
        a = np.ascontiguousarray(val, dtype=np.float32)
        b = name.encode("utf-8")
        keep += [a, b]
        arr[i] = TensorC(b, a.ctypes.data, a.size)
    return arr, keep
