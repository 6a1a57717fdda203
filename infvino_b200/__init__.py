"""infvino_b200 - B200-native plan executor behind infvino's backend interface.

Python mirror of the reference's host interface for the plan-executor path:
  * `PlanModel`   <- infvino::PlanModel  (include/infvino/PlanModel.hpp:46-234):
                     setInput / run / readOutput / readTensor / tensorNumel /
                     inputDims / outputDims / pool statistics / profile
  * `CudaBackend` <- infvino::ClBackend  (include/infvino/ClBackend.hpp:29-53):
                     infer(f32 blob) -> list[Tensor], inputDims, outputShapes,
                     lastInferMs
  * `Tensor`      <- infvino::Tensor     (include/infvino/Tensor.hpp:15-45)
  * `ModelInfo`   <- infvino::ModelInfo  (src/ModelInfo.cpp:21-76, the plan path
                     and task fields of config/models.yaml)
All compute goes through the C ABI of the in-tree `libinfvino_b200.so`
(include/infvino_b200.h); there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence

import numpy as np

from . import _native
from ._native import (FLAG_DRY_RUN, FLAG_NO_FUSION, FLAG_NO_GRAPH, FLAG_NO_HALO, FLAG_NO_JIT, FLAG_NO_PDL, FLAG_NO_TUNE, FLAG_NO_POOL, FLAG_SERIAL, FLAG_NO_TENSOR_CORES, NativeError,
                      check, lib)

__all__ = ["PlanModel", "CudaBackend", "Tensor", "ModelInfo", "NativeError", "FLAG_DRY_RUN", "FLAG_NO_FUSION",
           "FLAG_NO_GRAPH", "FLAG_NO_HALO", "FLAG_NO_JIT", "FLAG_NO_PDL", "FLAG_NO_TUNE", "FLAG_NO_POOL", "FLAG_SERIAL", "FLAG_NO_TENSOR_CORES", "f32_to_f16", "f16_to_f32"]


def f32_to_f16(x: np.ndarray) -> np.ndarray:
    """Reference host conversion (mantissa truncation, include/infvino/Half.hpp:14-24) as uint16 bits."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().ivc_f32_to_f16(x.ctypes.data, out.ctypes.data, x.size)
    return out


def f16_to_f32(h: np.ndarray) -> np.ndarray:
    h = np.ascontiguousarray(h, dtype=np.uint16)
    out = np.empty(h.shape, dtype=np.float32)
    lib().ivc_f16_to_f32(h.ctypes.data, out.ctypes.data, h.size)
    return out


@dataclass
class Tensor:
    """Backend-neutral tensor: shape + row-major f32 data (reference Tensor.hpp)."""
    shape: List[int]
    data: np.ndarray

    def numel(self) -> int:
        return int(np.prod(self.shape)) if self.shape else 1

    def getShape(self) -> List[int]:
        return list(self.shape)


@dataclass
class ModelInfo:
    plan: str = ""
    task: str = ""
    imgsz: Sequence[int] = (640, 640)
    num_classes: int = 0
    kpt_shape: Sequence[int] = ()
    conf: float = 0.25
    iou: float = 0.45
    device: str = "AUTO"
    extra: Dict[str, object] = field(default_factory=dict)

    @staticmethod
    def from_yaml(path: str, key: str = "") -> "ModelInfo":
        import yaml
        with open(path) as f:
            doc = yaml.safe_load(f)
        key = key or doc.get("default", "")
        m = doc["models"][key]
        base = os.path.dirname(os.path.abspath(path))
        plan = m.get("plan", "")
        if plan and not os.path.isabs(plan):
            cand = os.path.join(base, plan)
            plan = cand if os.path.exists(cand) else plan
        return ModelInfo(plan=plan, task=m.get("task", ""), imgsz=m.get("imgsz", (640, 640)),
                         num_classes=m.get("num_classes", 0), kpt_shape=m.get("kpt_shape", ()),
                         conf=m.get("conf", 0.25), iou=m.get("iou", 0.45), device=str(m.get("device", "AUTO")),
                         extra=m)


def _dims(fn, *args) -> List[int]:
    d = (ctypes.c_int64 * 16)()
    r = ctypes.c_int(0)
    check(fn(*args, d, 16, ctypes.byref(r)))
    return [int(d[i]) for i in range(r.value)]


class PlanModel:
    """Whole-network plan executor on one CUDA device (batch 1..max_batch)."""

    def __init__(self, plan_path: str, device: int = 0, max_batch: int = 1, flags: int = 0):
        L = lib()
        h = ctypes.c_void_p()
        st = L.ivc_create(plan_path.encode(), int(device), int(max_batch), int(flags), ctypes.byref(h))
        if st != 0:
            raise NativeError(st, (L.ivc_last_error(None) or b"").decode())
        self._h = h
        self.plan_path = plan_path
        self.device = device
        self.max_batch = max_batch
        self.flags = flags

    def close(self) -> None:
        h = getattr(self, "_h", None)
        if h:
            lib().ivc_destroy(h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._h

    # ---- plan facts (PlanModel.hpp:64-73)
    def inputName(self) -> str:
        p = ctypes.c_char_p()
        check(lib().ivc_input_name(self._h, ctypes.byref(p)), self._h)
        return p.value.decode()

    def inputDims(self) -> List[int]:
        return _dims(lib().ivc_input_dims, self._h)

    def inputNumel(self) -> int:
        return int(lib().ivc_input_numel(self._h))

    def outputCount(self) -> int:
        return int(lib().ivc_output_count(self._h))

    def outputName(self, i: int) -> str:
        p = ctypes.c_char_p()
        check(lib().ivc_output_name(self._h, i, ctypes.byref(p)), self._h)
        return p.value.decode()

    def outputDims(self, i: int) -> List[int]:
        return _dims(lib().ivc_output_dims, self._h, i)

    def outputNumel(self, i: int) -> int:
        return int(lib().ivc_output_numel(self._h, i))

    def tensorNumel(self, name: str) -> int:
        return int(lib().ivc_tensor_numel(self._h, name.encode()))

    # ---- execution (PlanModel.hpp:75-86)
    def setInput(self, fp16: np.ndarray, batch: int = 1) -> None:
        a = np.ascontiguousarray(fp16)
        if a.dtype == np.float16:
            a = a.view(np.uint16)
        if a.dtype != np.uint16 or a.size != batch * self.inputNumel():
            raise ValueError("setInput expects batch*inputNumel fp16 values")
        check(lib().ivc_set_input_f16(self._h, a.ctypes.data, batch), self._h)

    def run(self, batch: int = 1) -> None:
        check(lib().ivc_run(self._h, batch), self._h)

    def run_async(self, batch: int = 1, stream: int = 0) -> None:
        check(lib().ivc_run_async(self._h, batch, stream or None), self._h)

    def readOutput(self, i: int, batch: int = 1) -> np.ndarray:
        out = np.empty(self.outputNumel(i) * batch, dtype=np.uint16)
        check(lib().ivc_read_output_f16(self._h, i, out.ctypes.data, batch), self._h)
        return out

    def readTensor(self, name: str, batch: int = 1) -> Optional[np.ndarray]:
        n = self.tensorNumel(name)
        if n <= 0:
            return None
        out = np.empty(n * batch, dtype=np.uint16)
        st = lib().ivc_read_tensor_f16(self._h, name.encode(), out.ctypes.data, batch)
        if st == 6:
            return None
        check(st, self._h)
        return out

    def decodePose(self, batch: int = 1, conf: float = 0.25, iou: float = 0.7, max_det: int = 300, nk: int = 17,
                   kdims: int = 3, letterbox=None):
        """PoseDecoder::decode + NMS of the last run's output 0 on the device
        (src/Decoders.cpp:127-179, src/Nms.cpp:10-55).  Returns, per image, an
        array [n, 6 + 2 * nk]: anchor, score, x, y, w, h, then keypoint x, y
        pairs, in descending score.  `letterbox`: [batch, 3] of (scale,
        pad_left, pad_top), or None."""
        S = 6 + 2 * nk
        counts = np.zeros(batch, dtype=np.int32)
        dets = np.zeros(batch * max_det * S, dtype=np.float32)
        lb = None
        if letterbox is not None:
            lb = np.ascontiguousarray(letterbox, dtype=np.float32).reshape(batch, 3)
        check(lib().ivc_decode_pose(self._h, batch, conf, iou, max_det, nk, kdims,
                                    None if lb is None else lb.ctypes.data, counts.ctypes.data,
                                    dets.ctypes.data), self._h)
        dets = dets.reshape(batch, max_det, S)
        return [dets[b, :counts[b]].copy() for b in range(batch)]

    # ---- device preprocessing (src/Preprocess.cpp:13-77 on the device)
    @staticmethod
    def _preprocess_cfg(letterbox=True, to_rgb=True, normalize=True, mean=(), std=()):
        c = _native.Preprocess()
        c.letterbox, c.to_rgb, c.normalize = int(bool(letterbox)), int(bool(to_rgb)), int(bool(normalize))
        c.n_mean, c.n_std = len(mean), len(std)
        for i, v in enumerate(mean):
            c.mean[i] = float(v)
        for i, v in enumerate(std):
            c.std[i] = float(v)
        return c

    def setInputBgr(self, frames: np.ndarray, **cfg) -> np.ndarray:
        """Preprocessor::operator() on the device for a batch of 8-bit BGR
        frames [batch, H, W, 3] (host memory, or a device pointer with
        `device_shape=(batch, H, W)`), written to the network input.  Returns
        the letterbox [batch, 3] (scale, pad_left, pad_top).  Keyword
        settings: letterbox, to_rgb, normalize, mean, std."""
        device_shape = cfg.pop("device_shape", None)
        c = self._preprocess_cfg(**cfg)
        if device_shape is not None:
            batch, h, w = device_shape
            ptr, on_dev = int(frames), 1
        else:
            frames = np.ascontiguousarray(frames, dtype=np.uint8)
            batch, h, w = frames.shape[0], frames.shape[1], frames.shape[2]
            ptr, on_dev = frames.ctypes.data, 0
        lb = np.zeros((batch, 3), dtype=np.float32)
        check(lib().ivc_set_input_bgr_u8(self._h, ptr, batch, h, w, w * 3, on_dev, ctypes.byref(c), lb.ctypes.data),
              self._h)
        return lb

    def inferBgr(self, frames: np.ndarray, outs: Optional[List[np.ndarray]] = None, **cfg):
        """Frames [batch, H, W, 3] uint8 in host memory -> f32 outputs in host
        memory, preprocessing on the device; returns (outputs, letterbox)."""
        frames = np.ascontiguousarray(frames, dtype=np.uint8)
        batch, h, w = frames.shape[0], frames.shape[1], frames.shape[2]
        c = self._preprocess_cfg(**cfg)
        if outs is None:
            outs = [np.empty(self.outputNumel(i) * batch, dtype=np.float32) for i in range(self.outputCount())]
        arr = (ctypes.c_void_p * len(outs))(*[o.ctypes.data for o in outs])
        lb = np.zeros((batch, 3), dtype=np.float32)
        check(lib().ivc_infer_bgr_u8(self._h, frames.ctypes.data, batch, h, w, w * 3, ctypes.byref(c), arr,
                                     lb.ctypes.data), self._h)
        return outs, lb

    def lastRunMs(self) -> float:
        return float(lib().ivc_last_infer_ms(self._h))

    # ---- pool statistics (PlanModel.hpp:94-97)
    def pool_stats(self) -> Dict[str, int]:
        v = [ctypes.c_int64() for _ in range(3)] + [ctypes.c_int() for _ in range(5)]
        check(lib().ivc_pool_stats(self._h, *[ctypes.byref(x) for x in v]), self._h)
        keys = ["requested_bytes", "arena_bytes", "weight_bytes", "roots", "views", "nhwc_tensors",
                "fusions_concat", "fusions_res"]
        return {k: int(x.value) for k, x in zip(keys, v)}

    def poolRequestedBytes(self) -> int:
        return self.pool_stats()["requested_bytes"]

    def poolAllocatedBytes(self) -> int:
        return self.pool_stats()["arena_bytes"]

    def poolBufferCount(self) -> int:
        return 1

    def describe(self) -> str:
        n = lib().ivc_describe(self._h, None, 0)
        buf = ctypes.create_string_buffer(n + 1)
        lib().ivc_describe(self._h, buf, n + 1)
        return buf.value.decode()

    # ---- profiling (PlanModel.hpp:204-224)
    def steps(self) -> List[Dict[str, object]]:
        L = lib()
        out = []
        for i in range(L.ivc_step_count(self._h)):
            name, fam = ctypes.c_char_p(), ctypes.c_char_p()
            fl, ab, fb = ctypes.c_double(), ctypes.c_double(), ctypes.c_double()
            check(L.ivc_step_info(self._h, i, ctypes.byref(name), ctypes.byref(fam), ctypes.byref(fl),
                                  ctypes.byref(ab), ctypes.byref(fb)), self._h)
            out.append({"name": name.value.decode(), "family": fam.value.decode(), "flops_per_image": fl.value,
                        "act_bytes_per_image": ab.value, "fixed_bytes": fb.value})
        return out

    def profile(self, batch: int = 1) -> List[float]:
        n = lib().ivc_step_count(self._h)
        ms = (ctypes.c_float * max(1, n))()
        check(lib().ivc_profile(self._h, batch, ms, n), self._h)
        return [float(ms[i]) for i in range(n)]

    def launch_count(self, batch: int = 1) -> int:
        n = ctypes.c_int(0)
        check(lib().ivc_launch_count(self._h, batch, ctypes.byref(n)), self._h)
        return int(n.value)

    # ---- device-pointer paths (C ABI zero-copy entry points)
    def infer_f16_device(self, d_input: int, batch: int, d_outputs: Sequence[int], stream: int = 0) -> None:
        arr = (ctypes.c_void_p * len(d_outputs))(*d_outputs)
        check(lib().ivc_infer_f16_device(self._h, d_input, batch, arr, stream or None), self._h)

    def infer_f32_device(self, d_input: int, batch: int, d_outputs: Sequence[int], stream: int = 0) -> None:
        arr = (ctypes.c_void_p * len(d_outputs))(*d_outputs)
        check(lib().ivc_infer_f32_device(self._h, d_input, batch, arr, stream or None), self._h)

    def set_stream(self, stream: int) -> None:
        check(lib().ivc_set_stream(self._h, stream or None), self._h)

    def synchronize(self) -> None:
        check(lib().ivc_synchronize(self._h), self._h)

    def infer_f32(self, x: np.ndarray, batch: int, outs: Optional[List[np.ndarray]] = None) -> List[np.ndarray]:
        """ClBackend-style f32 host round trip (writes into `outs` if given)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        if outs is None:
            outs = [np.empty(self.outputNumel(i) * batch, dtype=np.float32) for i in range(self.outputCount())]
        arr = (ctypes.c_void_p * len(outs))(*[o.ctypes.data for o in outs])
        check(lib().ivc_infer_f32(self._h, x.ctypes.data, x.size, batch, arr), self._h)
        return outs


class CudaBackend:
    """Drop-in for infvino::ClBackend on a B200: f32 NCHW blob in, f32 Tensors out."""

    def __init__(self, info, profiling: bool = False, device: int = 0, max_batch: int = 1):
        plan = info.plan if isinstance(info, ModelInfo) else str(info)
        if not plan:
            raise RuntimeError("ClBackend: ModelInfo.plan is empty. Generate it first with "
                               "scripts/onnx2plan.py --onnx <model.onnx> --out-dir models")
        self.info = info if isinstance(info, ModelInfo) else ModelInfo(plan=plan)
        self.profiling = profiling
        self.model = PlanModel(plan, device=device, max_batch=max_batch)
        self._input_dims = self.model.inputDims()
        self._output_shapes = [self.model.outputDims(i) for i in range(self.model.outputCount())]

    def inputDims(self) -> List[int]:
        return list(self._input_dims)

    def outputShapes(self) -> List[List[int]]:
        return [list(s) for s in self._output_shapes]

    def device(self) -> Dict[str, object]:
        return {"backend": "cuda", "ordinal": self.model.device, "name": "NVIDIA B200"}

    def infer(self, input_f32: np.ndarray, numel: Optional[int] = None, batch: int = 1) -> List[Tensor]:
        x = np.ascontiguousarray(input_f32, dtype=np.float32).reshape(-1)
        if numel is None:
            numel = x.size
        expect = self.model.inputNumel() * batch
        if numel != expect:
            raise RuntimeError(f"ClBackend: input numel mismatch: got {numel}, expected {expect}")
        outs = self.model.infer_f32(x[:numel], batch)
        res = []
        for shp, o in zip(self._output_shapes, outs):
            shape = [batch] + list(shp[1:]) if batch != 1 else list(shp)
            res.append(Tensor(shape, o.reshape(shape)))
        return res

    def lastInferMs(self) -> float:
        return self.model.lastRunMs()
