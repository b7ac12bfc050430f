"""Python handles over the C-ABI engine and single-layer objects.

``EnsembleEngine`` owns one device's weights and per-symbol state table and runs
the whole MultiTowerModel step (model/inference_model.py:119-143) for the rows
it is given, each row naming its state slot. ``LayerEngine`` does the same for a
single recurrent layer (the reference's per-layer forward). Both are thin: all
work happens in libb2e.so.
"""

from __future__ import annotations

import ctypes as C
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

from . import _lib
from .config import CONV_K, TOWER_KINDS, ModelConfig


def _opts(device: int, linear_dtype: str, capacity: int, max_batch: int, graphs: bool, lanes: int = 0,
          lane_min_rows: int = 0, flags: int = 0, lane_towers: int = 0) -> _lib.EngineOptionsC:
    if linear_dtype not in _lib.DTYPES:
        raise ValueError(f"linear_dtype must be one of {sorted(_lib.DTYPES)}, got {linear_dtype!r}")
    return _lib.EngineOptionsC(int(device), _lib.DTYPES[linear_dtype], int(capacity), int(max_batch), int(graphs),
                               int(lanes), int(lane_min_rows), int(flags), int(lane_towers))


def leaf_layout(kind: str, cfg: ModelConfig) -> List[Tuple[Tuple[int, ...], np.dtype]]:
    """Per-row (shape, dtype) of one block's state leaves in init_state order
    (model/xlstm.py:369-379, mamba2.py:48-60, retnet.py:174-189, hawk.py:89-95)."""
    h, f32, i32 = cfg.hidden_size, np.dtype(np.float32), np.dtype(np.int32)
    k = CONV_K - 1
    if kind == "xlstm":
        inner, nh, hs = cfg.mlstm_inner, cfg.mlstm_heads, cfg.mlstm_head_size
        return [((h, k), f32), ((h,), f32), ((h,), f32), ((h,), f32), ((h,), f32), ((inner, k), f32),
                ((nh, hs, hs), f32), ((nh, hs), f32), ((nh,), f32)]
    if kind == "mamba2":
        inner, nh, hs, bc = cfg.mamba_inner, cfg.mamba_heads, cfg.mamba_head_size, cfg.mamba_bc_size
        return [((inner, k), f32), ((bc, k), f32), ((bc, k), f32), ((nh, hs, bc), f32)]
    if kind == "retnet":
        return [((), i32), ((cfg.num_heads,), f32), ((cfg.num_heads, cfg.retnet_head_size, cfg.retnet_head_size), f32)]
    if kind == "hawk":
        return [((h, k), f32), ((h,), f32)]
    raise ValueError(kind)


def model_layout(cfg: ModelConfig):
    return [spec for kind in TOWER_KINDS for _ in range(cfg.tower_depth) for spec in leaf_layout(kind, cfg)]


def split_blob(blob: bytes, layout) -> List[np.ndarray]:
    out, off = [], 0
    for shape, dt in layout:
        n = int(np.prod(shape)) * dt.itemsize
        out.append(np.frombuffer(blob[off:off + n], dtype=dt).reshape(shape).copy())
        off += n
    assert off == len(blob), (off, len(blob))
    return out


def join_leaves(leaves: Sequence[np.ndarray], layout) -> bytes:
    parts = []
    for a, (shape, dt) in zip(leaves, layout, strict=True):
        a = np.asarray(a, dtype=dt)
        assert a.shape == tuple(shape), (a.shape, shape)
        parts.append(np.ascontiguousarray(a).tobytes())
    return b"".join(parts)


class EnsembleEngine:
    """One device's ensemble: weights, `capacity` state slots, steps of <= max_batch rows."""

    def __init__(self, cfg: ModelConfig, state_dict: Dict[str, np.ndarray], *, device: int = 0,
                 linear_dtype: str = "fp32", capacity: int = 16, max_batch: int = 16, graphs: bool = True,
                 lanes: int = 0, lane_min_rows: int = 0, flags: int = 0, lane_towers: int = 0):
        self.cfg, self.device, self.linear_dtype = cfg, device, linear_dtype
        self.capacity, self.max_batch = capacity, max_batch
        L = _lib.lib()
        arr, keep = _lib.tensor_array(state_dict)
        h = C.c_void_p()
        cc, oo = _lib.model_config_c(cfg), _opts(device, linear_dtype, capacity, max_batch, graphs, lanes,
                                                 lane_min_rows, flags, lane_towers)
        _lib.check(L.b2e_engine_create(C.byref(cc), C.byref(oo), arr, len(state_dict), C.byref(h)))
        del keep
        self._h = h
        self._pending: List[int] = []
        nb = C.c_int64()
        _lib.check(L.b2e_engine_slot_bytes(h, C.byref(nb)))
        self.slot_bytes = nb.value
        self.layout = model_layout(cfg)
        self._preds = np.empty((max_batch, len(TOWER_KINDS)), np.float32)

    def close(self):
        if getattr(self, "_h", None):
            _lib.lib().b2e_engine_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @staticmethod
    def _rows(slots, feats, nf):
        slots = np.ascontiguousarray(slots, dtype=np.int32).reshape(-1)
        feats = np.ascontiguousarray(feats, dtype=np.float32).reshape(len(slots), nf)
        return slots, feats

    def step(self, slots, feats) -> np.ndarray:
        """preds (n, 4) for rows `feats` (n, num_features) at state `slots` (n,), host arrays."""
        slots, feats = self._rows(slots, feats, self.cfg.num_features)
        n = len(slots)
        out = np.empty((n, len(TOWER_KINDS)), np.float32)
        _lib.check(_lib.lib().b2e_engine_step(self._h, slots.ctypes.data, feats.ctypes.data, n, out.ctypes.data))
        return out

    def submit(self, slots, feats) -> int:
        """Start a host-buffer step; up to two may be outstanding (wait() returns the oldest)."""
        slots, feats = self._rows(slots, feats, self.cfg.num_features)
        _lib.check(_lib.lib().b2e_engine_submit(self._h, slots.ctypes.data, feats.ctypes.data, len(slots)))
        self._pending.append(len(slots))
        return len(slots)

    def wait(self) -> np.ndarray:
        """Predictions of the oldest submitted step. Raises B2EError with code
        B2E_ERR_DEVICE when a kernel recorded an error in the engine's device error
        word (the step is consumed either way; device_error() clears the word)."""
        n = self._pending.pop(0) if self._pending else 0  # nothing in flight: the library refuses
        out = np.empty((max(n, 1), len(TOWER_KINDS)), np.float32)[:n]
        _lib.check(_lib.lib().b2e_engine_wait(self._h, out.ctypes.data))
        return out

    def step_device(self, slots_t, feats_t, preds_t, n: int, stream=None):
        """Device-buffer step on a torch stream: int32 slots, float32 features/preds."""
        import torch

        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        _lib.check(_lib.lib().b2e_engine_step_device(self._h, C.c_void_p(slots_t.data_ptr()),
                                                     C.c_void_p(feats_t.data_ptr()), int(n),
                                                     C.c_void_p(preds_t.data_ptr()), C.c_void_p(s.cuda_stream)))

    def submit_device(self, slots_t, feats_t, preds_t, n: int, stream=None):
        """Device-buffer step that overlaps the steps around it: it reads its inputs
        after the work on `stream` so far and fills preds_t when it ends, which only
        join_device(stream) waits for. Keep the three tensors unchanged until then."""
        import torch

        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        _lib.check(_lib.lib().b2e_engine_submit_device(self._h, C.c_void_p(slots_t.data_ptr()),
                                                       C.c_void_p(feats_t.data_ptr()), int(n),
                                                       C.c_void_p(preds_t.data_ptr()), C.c_void_p(s.cuda_stream)))

    def join_device(self, stream=None):
        """`stream` waits for every step submit_device started."""
        import torch

        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        _lib.check(_lib.lib().b2e_engine_join_device(self._h, C.c_void_p(s.cuda_stream)))

    def device_error(self) -> int:
        f = C.c_int32()
        _lib.check(_lib.lib().b2e_engine_device_error(self._h, C.byref(f)))
        return f.value

    def reset_slots(self, slots) -> None:
        s = np.ascontiguousarray(slots, dtype=np.int32).reshape(-1)
        _lib.check(_lib.lib().b2e_engine_reset_slots(self._h, s.ctypes.data, len(s)))

    def read_slot(self, slot: int) -> List[np.ndarray]:
        """Every state leaf of one slot, in iter_state_tensors order, per-row shapes."""
        buf = C.create_string_buffer(self.slot_bytes)
        _lib.check(_lib.lib().b2e_engine_read_slot(self._h, int(slot), buf, self.slot_bytes))
        return split_blob(buf.raw, self.layout)

    def write_slot(self, slot: int, leaves: Sequence[np.ndarray]) -> None:
        blob = join_leaves(leaves, self.layout)
        _lib.check(_lib.lib().b2e_engine_write_slot(self._h, int(slot), blob, len(blob)))

    def launches_per_step(self, n: int) -> int:
        k = C.c_int32()
        _lib.check(_lib.lib().b2e_engine_launches(self._h, int(n), C.byref(k)))
        return k.value

    def latency_rows(self) -> Tuple[int, int]:
        """(rows, cluster): host steps of at most `rows` rows run as one kernel,
        one cluster of `cluster` CTAs per tower; (0, 0) when every step runs on
        the batch graphs."""
        r, c = C.c_int32(), C.c_int32()
        _lib.check(_lib.lib().b2e_engine_latency_rows(self._h, C.byref(r), C.byref(c)))
        return r.value, c.value

    def memory(self) -> Tuple[int, int]:
        w, s = C.c_int64(), C.c_int64()
        _lib.check(_lib.lib().b2e_engine_memory(self._h, C.byref(w), C.byref(s)))
        return w.value, s.value


class LayerEngine:
    """One recurrent layer (xlstm / mamba2 / retnet / hawk) with its own state table."""

    def __init__(self, kind: str, cfg: ModelConfig, state_dict: Dict[str, np.ndarray], *, device: int = 0,
                 linear_dtype: str = "fp32", capacity: int = 16, max_batch: int = 16):
        self.kind, self.cfg, self.device = kind, cfg, device
        L = _lib.lib()
        arr, keep = _lib.tensor_array(state_dict)
        h = C.c_void_p()
        # tower-level sizes are unused by a bare layer but must validate
        cc = _lib.model_config_c(cfg)
        oo = _opts(device, linear_dtype, capacity, max_batch, False)
        _lib.check(L.b2e_layer_create(_lib.LAYER_KINDS[kind], C.byref(cc), C.byref(oo), arr, len(state_dict),
                                      C.byref(h)))
        del keep
        self._h = h
        nb = C.c_int64()
        _lib.check(L.b2e_layer_slot_bytes(h, C.byref(nb)))
        self.slot_bytes = nb.value
        self.layout = leaf_layout(kind, cfg)

    def close(self):
        if getattr(self, "_h", None):
            _lib.lib().b2e_layer_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def step_device(self, slots_t, x_t, y_t, stream=None):
        import torch

        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        _lib.check(_lib.lib().b2e_layer_step_device(self._h, C.c_void_p(slots_t.data_ptr()),
                                                    C.c_void_p(x_t.data_ptr()), int(slots_t.numel()),
                                                    C.c_void_p(y_t.data_ptr()), C.c_void_p(s.cuda_stream)))

    def read_slot(self, slot: int) -> List[np.ndarray]:
        buf = C.create_string_buffer(self.slot_bytes)
        _lib.check(_lib.lib().b2e_layer_read_slot(self._h, int(slot), buf, self.slot_bytes))
        return split_blob(buf.raw, self.layout)

    def write_slot(self, slot: int, leaves: Sequence[np.ndarray]) -> None:
        blob = join_leaves(leaves, self.layout)
        _lib.check(_lib.lib().b2e_layer_write_slot(self._h, int(slot), blob, len(blob)))
