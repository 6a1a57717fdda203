"""Restatement of the reference's pose decoder and NMS - test infrastructure.

Follows src/Decoders.cpp:127-179 (`PoseDecoder::decode`), :33-65
(`nmsPerClass`) and src/Nms.cpp:10-55 (`iou`, greedy `nms` with a stable sort
by descending score), with the letterbox mapping of
include/infvino/Preprocess.hpp:24-35.  Used by the parity tests to check that
the CUDA path and the CPU oracle produce the same post-NMS detection set.
"""
from __future__ import annotations

from typing import List, Tuple

import numpy as np


def _iou_one_to_many(b, boxes):
    # boxes: [N, 4] as (x, y, w, h) -> Nms.cpp:10-26
    x1 = np.maximum(b[0], boxes[:, 0])
    y1 = np.maximum(b[1], boxes[:, 1])
    x2 = np.minimum(b[0] + b[2], boxes[:, 0] + boxes[:, 2])
    y2 = np.minimum(b[1] + b[3], boxes[:, 1] + boxes[:, 3])
    inter = np.maximum(0.0, x2 - x1) * np.maximum(0.0, y2 - y1)
    area_a = max(0.0, b[2]) * max(0.0, b[3])
    area_b = np.maximum(0.0, boxes[:, 2]) * np.maximum(0.0, boxes[:, 3])
    uni = area_a + area_b - inter
    return np.where(uni > 1e-9, inter / np.where(uni > 1e-9, uni, 1.0), 0.0)


def nms(boxes: np.ndarray, scores: np.ndarray, iou_thr: float) -> List[int]:
    order = np.argsort(-scores, kind="stable")
    removed = np.zeros(len(boxes), dtype=bool)
    keep = []
    for i, idx in enumerate(order):
        if removed[idx]:
            continue
        keep.append(int(idx))
        rest = order[i + 1:]
        rest = rest[~removed[rest]]
        if rest.size:
            ov = _iou_one_to_many(boxes[idx], boxes[rest])
            removed[rest[ov > iou_thr]] = True
    return keep


def pose_decode(out: np.ndarray, conf: float = 0.25, iou: float = 0.7, max_det: int = 300, nk: int = 17,
                kdims: int = 3, scale: float = 1.0, pad: Tuple[int, int] = (0, 0)):
    """out: [56, A] channel-major f32 -> list of (anchor, score, box[4], kpts[nk, 2])."""
    out = np.asarray(out, dtype=np.float32)
    scores = out[4]
    idx = np.nonzero(scores >= conf)[0]
    cx, cy, w, h = out[0, idx], out[1, idx], out[2, idx], out[3, idx]
    x = (cx - pad[0]) / scale
    y = (cy - pad[1]) / scale
    boxes = np.stack([x - w / scale / 2.0, y - h / scale / 2.0, w / scale, h / scale], 1).astype(np.float32)
    keep = nms(boxes, scores[idx], iou) if idx.size else []
    dets = []
    for k in keep:
        a = int(idx[k])
        kp = np.stack([(out[5 + j * kdims, a] - pad[0]) / scale for j in range(nk)]), \
            np.stack([(out[5 + j * kdims + 1, a] - pad[1]) / scale for j in range(nk)])
        dets.append((a, float(scores[a]), boxes[k], np.stack(kp, 1)))
    dets.sort(key=lambda d: -d[1])
    return dets[:max_det]
