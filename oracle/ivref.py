"""ctypes front-end of the CPU oracle (oracle/cpu_ref.cpp) - test infrastructure.

Only tests/, `__graft_entry__.smoke()` and bench.py's CPU-baseline leg import
this module; the product path never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import List, Optional

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libivref.so")
_REF_HALF = os.path.join(_HERE, "_ref", "libref_half.so")
_lib = None


def build(force: bool = False) -> str:
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(
            os.path.join(_HERE, "cpu_ref.cpp")):
        subprocess.run(["make", "-C", _HERE, "libivref.so"], check=True, capture_output=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(_LIB_PATH)
        vp, cp, i64 = ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int64
        L.ivref_create.argtypes = [cp, ctypes.POINTER(vp)]
        L.ivref_destroy.argtypes = [vp]
        L.ivref_set_acc_order.argtypes = [vp, ctypes.c_int]
        L.ivref_set_threads.argtypes = [ctypes.c_int]
        L.ivref_input_numel.argtypes = [vp]
        L.ivref_input_numel.restype = i64
        L.ivref_output_count.argtypes = [vp]
        L.ivref_output_name.argtypes = [vp, ctypes.c_int]
        L.ivref_output_name.restype = cp
        L.ivref_tensor_numel.argtypes = [vp, cp]
        L.ivref_tensor_numel.restype = i64
        L.ivref_tensor_dims.argtypes = [vp, cp, ctypes.POINTER(i64), ctypes.c_int]
        L.ivref_run.argtypes = [vp, vp, ctypes.c_int]
        L.ivref_read_tensor.argtypes = [vp, cp, vp]
        L.ivref_last_error.restype = cp
        for f in ("ivref_f32_to_f16_trunc", "ivref_f32_to_f16_rne"):
            getattr(L, f).argtypes = [vp, vp, ctypes.c_size_t]
        L.ivref_f16_to_f32.argtypes = [vp, vp, ctypes.c_size_t]
        L.ivref_std_sort_desc.argtypes = [vp, ctypes.c_int, vp]
        L.ivref_std_sort_desc.restype = None
        _lib = L
    return _lib


def set_threads(n: int) -> int:
    return lib().ivref_set_threads(n)


def std_sort_desc(scores: np.ndarray) -> np.ndarray:
    """Permutation std::sort applies to a sequence sorted by descending score
    (the reference's final, unstable ordering of the kept detections)."""
    s = np.ascontiguousarray(scores, dtype=np.float32)
    perm = np.empty(s.size, dtype=np.int32)
    if s.size:
        lib().ivref_std_sort_desc(s.ctypes.data, s.size, perm.ctypes.data)
    return perm


def f32_to_f16_trunc(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().ivref_f32_to_f16_trunc(x.ctypes.data, out.ctypes.data, x.size)
    return out


def f32_to_f16_rne(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().ivref_f32_to_f16_rne(x.ctypes.data, out.ctypes.data, x.size)
    return out


def f16_to_f32(h: np.ndarray) -> np.ndarray:
    h = np.ascontiguousarray(h, dtype=np.uint16)
    out = np.empty(h.shape, dtype=np.float32)
    lib().ivref_f16_to_f32(h.ctypes.data, out.ctypes.data, h.size)
    return out


class OraclePlan:
    """CPU restatement of the reference plan executor over one plan file."""

    def __init__(self, plan_path: str, acc_order: int = 0):
        L = lib()
        h = ctypes.c_void_p()
        if L.ivref_create(plan_path.encode(), ctypes.byref(h)) != 0:
            raise RuntimeError(L.ivref_last_error().decode())
        self._h = h
        L.ivref_set_acc_order(h, acc_order)
        self.batch = 0

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and _lib is not None:
            _lib.ivref_destroy(h)
            self._h = None

    @property
    def input_numel(self) -> int:
        return int(lib().ivref_input_numel(self._h))

    def output_names(self) -> List[str]:
        L = lib()
        return [L.ivref_output_name(self._h, i).decode() for i in range(L.ivref_output_count(self._h))]

    def dims(self, name: str) -> List[int]:
        d = (ctypes.c_int64 * 8)()
        r = lib().ivref_tensor_dims(self._h, name.encode(), d, 8)
        if r < 0:
            raise KeyError(name)
        return [int(d[i]) for i in range(r)]

    def run_f16(self, x16: np.ndarray, batch: int) -> None:
        x16 = np.ascontiguousarray(x16, dtype=np.uint16)
        assert x16.size == batch * self.input_numel, (x16.size, batch, self.input_numel)
        if lib().ivref_run(self._h, x16.ctypes.data, batch) != 0:
            raise RuntimeError(lib().ivref_last_error().decode())
        self.batch = batch

    def run(self, x32: np.ndarray, batch: Optional[int] = None) -> List[np.ndarray]:
        """f32 input (truncating host conversion, as the reference backend) -> f32 outputs."""
        b = batch if batch is not None else x32.size // self.input_numel
        self.run_f16(f32_to_f16_trunc(x32), b)
        return [f16_to_f32(self.read_f16(n)).reshape([b] + self.dims(n)[1:]) for n in self.output_names()]

    def read_f16(self, name: str) -> np.ndarray:
        n = int(lib().ivref_tensor_numel(self._h, name.encode()))
        if n < 0:
            raise KeyError(name)
        out = np.empty(n * max(1, self.batch), dtype=np.uint16)
        if lib().ivref_read_tensor(self._h, name.encode(), out.ctypes.data) != 0:
            raise RuntimeError(lib().ivref_last_error().decode())
        return out


def ref_half_lib():
    """The reference's own src/Half.cpp compiled into oracle/_ref (None if absent)."""
    if not os.path.exists(_REF_HALF):
        return None
    L = ctypes.CDLL(_REF_HALF)
    L.ref_f32_to_f16.argtypes = [ctypes.c_float]
    L.ref_f32_to_f16.restype = ctypes.c_uint16
    L.ref_f16_to_f32.argtypes = [ctypes.c_uint16]
    L.ref_f16_to_f32.restype = ctypes.c_float
    L.ref_f32_to_f16_bulk.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t]
    L.ref_f16_to_f32_bulk.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t]
    L.ref_f32_to_f16_scalar_n.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t]
    L.ref_f16_to_f32_scalar_n.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t]
    return L
