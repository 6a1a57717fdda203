"""ctypes binding of the C ABI (include/infvino_b200.h) exported by the in-tree
`libinfvino_b200.so`.  There is no fallback: if the library is missing or does
not load, every entry point raises."""
from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libinfvino_b200.so")

IVC_OK = 0
STATUS_NAMES = {0: "OK", 1: "ARGUMENT", 2: "PLAN", 3: "CUDA", 4: "NUMEL", 5: "KERNEL", 6: "NOT_FOUND"}

FLAG_NO_GRAPH = 0x1
FLAG_NO_FUSION = 0x2
FLAG_DRY_RUN = 0x4
FLAG_NO_TENSOR_CORES = 0x8
FLAG_NO_POOL = 0x10
FLAG_NO_HALO = 0x20
FLAG_NO_PDL = 0x40
FLAG_NO_JIT = 0x80
FLAG_NO_TUNE = 0x100
FLAG_SERIAL = 0x200

# every symbol include/infvino_b200.h declares, with its ctypes signature
_vp, _cp, _i32, _i64, _u32, _sz, _f64 = (ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int, ctypes.c_int64,
                                           ctypes.c_uint, ctypes.c_size_t, ctypes.c_double)
_P = ctypes.POINTER
SIGNATURES = {
    "ivc_create": (_i32, [_cp, _i32, _i32, _u32, _P(_vp)]),
    "ivc_destroy": (None, [_vp]),
    "ivc_last_error": (_cp, [_vp]),
    "ivc_input_name": (_i32, [_vp, _P(_cp)]),
    "ivc_input_dims": (_i32, [_vp, _P(_i64), _i32, _P(_i32)]),
    "ivc_input_numel": (_i64, [_vp]),
    "ivc_output_count": (_i32, [_vp]),
    "ivc_output_name": (_i32, [_vp, _i32, _P(_cp)]),
    "ivc_output_dims": (_i32, [_vp, _i32, _P(_i64), _i32, _P(_i32)]),
    "ivc_output_numel": (_i64, [_vp, _i32]),
    "ivc_tensor_numel": (_i64, [_vp, _cp]),
    "ivc_max_batch": (_i32, [_vp]),
    "ivc_infer_f32": (_i32, [_vp, _vp, _sz, _i32, _P(_vp)]),
    "ivc_set_input_f16": (_i32, [_vp, _vp, _i32]),
    "ivc_run": (_i32, [_vp, _i32]),
    "ivc_run_async": (_i32, [_vp, _i32, _vp]),
    "ivc_read_output_f16": (_i32, [_vp, _i32, _vp, _i32]),
    "ivc_read_tensor_f16": (_i32, [_vp, _cp, _vp, _i32]),
    "ivc_set_input_bgr_u8": (_i32, [_vp, _vp, _i32, _i32, _i32, _sz, _i32, _vp, _vp]),
    "ivc_infer_bgr_u8": (_i32, [_vp, _vp, _i32, _i32, _i32, _sz, _vp, _P(_vp), _vp]),
    "ivc_decode_pose": (_i32, [_vp, _i32, ctypes.c_float, ctypes.c_float, _i32, _i32, _i32, _vp, _vp, _vp]),
    "ivc_read_tensor_f16_noalloc": (_i32, [_vp, _cp, _vp, _i32]),
    "ivc_infer_f16_device": (_i32, [_vp, _vp, _i32, _P(_vp), _vp]),
    "ivc_infer_f32_device": (_i32, [_vp, _vp, _i32, _P(_vp), _vp]),
    "ivc_set_stream": (_i32, [_vp, _vp]),
    "ivc_synchronize": (_i32, [_vp]),
    "ivc_last_infer_ms": (_f64, [_vp]),
    "ivc_step_count": (_i32, [_vp]),
    "ivc_step_info": (_i32, [_vp, _i32, _P(_cp), _P(_cp), _P(_f64), _P(_f64), _P(_f64)]),
    "ivc_profile": (_i32, [_vp, _i32, _P(ctypes.c_float), _i32]),
    "ivc_launch_count": (_i32, [_vp, _i32, _P(_i32)]),
    "ivc_debug_conv_wait": (_i32, [_vp, ctypes.c_longlong, _i32]),
    "ivc_pool_stats": (_i32, [_vp, _P(_i64), _P(_i64), _P(_i64), _P(_i32), _P(_i32), _P(_i32), _P(_i32),
                              _P(_i32)]),
    "ivc_describe": (_i32, [_vp, _cp, _sz]),
    "ivc_device_properties": (_i32, [_i32, _vp]),
    "ivc_f32_to_f16": (None, [_vp, _vp, _sz]),
    "ivc_f16_to_f32": (None, [_vp, _vp, _sz]),
}

class Preprocess(ctypes.Structure):
    """ivc_preprocess (include/infvino_b200.h): infvino::PreprocessConfig."""
    _fields_ = [("letterbox", ctypes.c_int), ("to_rgb", ctypes.c_int), ("normalize", ctypes.c_int),
                ("n_mean", ctypes.c_int), ("n_std", ctypes.c_int), ("mean", ctypes.c_float * 3),
                ("std", ctypes.c_float * 3)]


_lib = None
_lock = threading.Lock()


class NativeError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status
        self.message = message


def lib():
    """Loads the native library (building it first when only sources exist)."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                from . import build as _build
                _build.build()
            L = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def check(status: int, handle=None) -> None:
    if status != IVC_OK:
        msg = lib().ivc_last_error(handle)
        raise NativeError(status, msg.decode() if msg else "")
