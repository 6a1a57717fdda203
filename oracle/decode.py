"""Restatement of the reference's pose decoder and NMS - test infrastructure.

Follows src/Decoders.cpp:127-179 (`PoseDecoder::decode`), :33-65
(`nmsPerClass`: per-class greedy NMS, then the kept list re-sorted by score
with std::sort - unstable, reproduced by calling the same std::sort through the
oracle library - and cut at max_det) and src/Nms.cpp:10-55 (`iou`, greedy
`nms` with a stable sort by descending score), with the letterbox mapping of
include/infvino/Preprocess.hpp:24-35.  Pinned bit for bit to the reference's
own Decoders.cpp / Nms.cpp compiled here (tests/test_decode_pinned.py).  Used by the parity tests to check that
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
                kdims: int = 3, scale: float = 1.0, pad: Tuple[int, int] = (0, 0), tie_order: str = "reference"):
    """out: [56, A] channel-major f32 -> list of (anchor, score, box[4], kpts[nk, 2]).
    tie_order "reference": equal scores in the order of the reference's final
    std::sort; "stable": in keep order (anchor order among equal scores)."""
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
    # src/Decoders.cpp:58-63: the keep list re-sorted by descending score with
    # std::sort (not stable: equal scores take the order std::sort leaves them
    # in, which depends on the whole list), then cut at max_det
    if tie_order == "reference":
        from . import ivref
        dets = [dets[i] for i in ivref.std_sort_desc(np.array([d[1] for d in dets], dtype=np.float32))]
    else:
        dets.sort(key=lambda d: -d[1])
    return dets[:max_det]


def _xywh(out: np.ndarray, idx: np.ndarray) -> np.ndarray:
    cx, cy, w, h = (out[i, idx].astype(np.float64) for i in range(4))
    return np.stack([cx - w / 2.0, cy - h / 2.0, w, h], 1)


def undecided_anchors(out_ref: np.ndarray, out_cmp: np.ndarray, conf: float = 0.25, iou: float = 0.7,
                      max_det: int = 300, chunk: int = 512):
    """Anchors whose post-NMS membership is not decided at the deviation between
    two outputs of the same image (test infrastructure for the NMS-set check).

    delta = max |score_cmp - score_ref|, eps = max |IoU_cmp - IoU_ref| over the
    pairs of potential candidates that come near the IoU threshold.  The greedy
    NMS of `pose_decode` takes three kinds of decisions; an anchor is undecided
    when one of its decisions lies within twice the deviation of the boundary:
      * candidate or not: |score - conf| <= 2 delta;
      * suppressed or not: it has a partner with |IoU - iou| <= 2 eps;
      * who suppresses whom: it overlaps (IoU > iou - 2 eps) a partner whose
        score is within 2 delta of its own (the greedy order may swap);
      * the `max_det` cut, when reached: its score is within 2 delta of the cut.
    A flipped decision can cascade, so the set is closed under overlap (any
    anchor with IoU > iou - 2 eps to an undecided one is undecided as well).
    Outside this set both outputs must give the same detections.
    Returns (undecided anchor set, delta, eps)."""
    s_ref = out_ref[4].astype(np.float64)
    s_cmp = out_cmp[4].astype(np.float64)
    delta = float(np.abs(s_ref - s_cmp).max()) if s_ref.size else 0.0
    pot = np.nonzero((s_ref >= conf - 2 * delta) | (s_cmp >= conf))[0]
    und = set(int(a) for a in pot[np.abs(s_ref[pot] - conf) <= 2 * delta])
    br, bc = _xywh(out_ref, pot), _xywh(out_cmp, pot)
    # pairwise IoU over the potential candidates, in row chunks
    eps = 0.0
    near = []  # (i, j, iou_ref) for pairs that come within 0.3 of the threshold
    for c0 in range(0, pot.size, chunk):
        rows = range(c0, min(c0 + chunk, pot.size))
        ir = np.stack([_iou_one_to_many(br[i], br) for i in rows])
        ic = np.stack([_iou_one_to_many(bc[i], bc) for i in rows])
        mask = np.maximum(ir, ic) > iou - 0.3
        for k in range(mask.shape[0]):
            mask[k, c0 + k] = False
        ii, jj = np.nonzero(mask)
        if ii.size:
            eps = max(eps, float(np.abs(ir[ii, jj] - ic[ii, jj]).max()))
            near.extend(zip((ii + c0).tolist(), jj.tolist(), ir[ii, jj].tolist()))
    adj = {}
    for i, j, v in near:
        a, b = int(pot[i]), int(pot[j])
        if v > iou - 2 * eps:
            adj.setdefault(a, set()).add(b)
            if abs(s_ref[a] - s_ref[b]) <= 2 * delta:
                und.update((a, b))
        if abs(v - iou) <= 2 * eps:
            und.update((a, b))
    dets = pose_decode(out_ref, conf=conf, iou=iou, max_det=10 ** 9)
    if len(dets) >= max_det:
        cut = dets[max_det - 1][1]
        und.update(int(a) for a in pot[np.abs(s_ref[pot] - cut) <= 2 * delta])
    todo = list(und)
    while todo:
        a = todo.pop()
        for b in adj.get(a, ()):
            if b not in und:
                und.add(b)
                todo.append(b)
    if und and len(dets) >= max_det:
        # a flip ahead of the cut moves the cut by one detection per flip
        kept = [d[1] for d in dets]
        lo = kept[min(len(kept) - 1, max_det - 1 + len(und))]
        hi = kept[max(0, max_det - 1 - len(und))]
        und.update(int(a) for a in pot[(s_ref[pot] >= lo - 2 * delta) & (s_ref[pot] <= hi + 2 * delta)])
    return und, delta, eps
