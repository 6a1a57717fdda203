"""Generates tests/golden/decode_vectors.npz by running the reference's own
pose decoder and NMS (src/Decoders.cpp `PoseDecoder::decode` with
`nmsPerClass`, src/Nms.cpp), compiled from the reference sources into
oracle/_ref/libref_decode.so by `make -C oracle ref` (oracle/ref_decode_shim.cpp).

Cases: seeded synthetic pose outputs (spread scores, several letterboxes),
adversarial ones (score ties, scores at the confidence bound, duplicate,
empty and negative boxes, an IoU at the threshold, the max_det cut inside a
tie) and one real network output (the CPU oracle's run of a YOLOv8n-pose plan
at 320x320 with a trained-like class head).  tests/test_decode_pinned.py
replays every case through oracle/decode.py.

Run from the repository root:  python tests/golden/make_decode_golden.py
"""
import ctypes
import os
import sys
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
LIB = os.path.join(ROOT, "oracle", "_ref", "libref_decode.so")
OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "decode_vectors.npz")
NK, KD = 17, 3
C = 5 + NK * KD


def synthetic(rng, A, lo_score=-3.0):
    out = np.zeros((C, A), np.float32)
    out[0] = rng.uniform(0, 640, A)
    out[1] = rng.uniform(0, 640, A)
    out[2] = rng.uniform(4, 160, A)
    out[3] = rng.uniform(4, 160, A)
    out[4] = 1.0 / (1.0 + np.exp(-rng.normal(lo_score, 1.5, A)))
    for j in range(NK):
        out[5 + KD * j] = out[0] + rng.normal(0, 20, A)
        out[6 + KD * j] = out[1] + rng.normal(0, 20, A)
        out[7 + KD * j] = rng.uniform(0, 1, A)
    return out


def main():
    if not os.path.exists(LIB):
        raise SystemExit("oracle/_ref/libref_decode.so missing: run `make -C oracle ref` first")
    L = ctypes.CDLL(LIB)
    L.ref_pose_decode.restype = ctypes.c_int
    L.ref_pose_decode.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_float,
                                  ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_int, ctypes.c_int,
                                  ctypes.c_void_p, ctypes.c_int]
    rng = np.random.default_rng(2024)
    cases = {}

    def add(name, out, conf=0.25, iou=0.7, max_det=300, scale=1.0, pad=(0, 0)):
        # the executor's outputs are fp16 values widened to f32: the cases use
        # such values too, and store them as fp16 (exact)
        out = np.ascontiguousarray(np.asarray(out, dtype=np.float16).astype(np.float32))
        A = out.shape[1]
        cap = A
        dets = np.zeros((cap, 5 + 2 * NK), np.float32)
        n = L.ref_pose_decode(out.ctypes.data, C, A, conf, iou, max_det, NK, KD, scale, pad[0], pad[1],
                              dets.ctypes.data, cap)
        assert 0 <= n <= cap, n
        cases[name] = dict(out=out.astype(np.float16), dets=dets[:n].copy(),
                           params=np.array([conf, iou, max_det, scale, pad[0], pad[1]], np.float64))

    # spread scores, identity letterbox and two real letterboxes
    add("synthetic", synthetic(rng, 1200))
    add("synthetic_lb_half", synthetic(rng, 1200), scale=0.5, pad=(0, 140))
    add("synthetic_lb_odd", synthetic(rng, 1200), scale=0.3125, pad=(37, 0), iou=0.45)
    # many candidates: the max_det cut
    add("dense_maxdet", synthetic(rng, 1200, lo_score=0.5), max_det=100)
    # score ties (stable order by anchor), scores at the bound, duplicates,
    # empty / negative boxes, an IoU at the threshold
    out = synthetic(rng, 600, lo_score=-1.0)
    out[4, 0:80] = 0.5                       # a tie block
    out[4, 80:90] = np.float32(0.25)         # exactly at conf (candidates)
    out[4, 90:95] = np.float32(np.nextafter(np.float16(0.25), np.float16(0)))  # just below (fp16)
    out[:, 100:110] = out[:, 0:1]            # duplicates of anchor 0 (same score: tie)
    out[2, 110:115] = 0.0                    # zero width
    out[3, 115:120] = -5.0                   # negative height
    # two boxes whose IoU is exactly 0.5: [0,0,4,4] and [0,0,4,2] -> inter 8, union 16
    out[0:4, 120] = [2, 2, 4, 4]
    out[0:4, 121] = [2, 1, 4, 2]
    out[4, 120], out[4, 121] = 0.9, 0.8
    add("adversarial_iou07", out)
    add("adversarial_iou05", out, iou=0.5)
    add("adversarial_tie_cut", out, max_det=45)
    # no candidate at all
    add("empty", synthetic(rng, 256, lo_score=-12.0))
    # one real network output: the oracle's run of a 320x320 YOLOv8n-pose plan
    # whose final class conv is scaled like a trained head
    from infvino_b200 import plangen
    from oracle import ivref
    p = plangen.yolov8n_pose(tempfile.mkdtemp(prefix="ivb_dec_"), imgsz=320, cls_gain=100.0, cls_shift=-3.0)
    o = ivref.OraclePlan(p)
    x = np.random.default_rng(11).random(o.input_numel, dtype=np.float32)
    o.run(x, 1)
    net = ivref.f16_to_f32(o.read_f16("output0")).reshape(C, -1)
    add("network_y8_320", net)
    add("network_y8_320_lb", net, scale=0.5, pad=(0, 40), iou=0.5)

    flat = {}
    for name, c in cases.items():
        for k, v in c.items():
            flat[f"{name}/{k}"] = v
    np.savez_compressed(OUT, **flat)
    print("wrote", OUT, len(cases), "cases", {n: len(c["dets"]) for n, c in cases.items()}, os.path.getsize(OUT),
          "bytes")


if __name__ == "__main__":
    sys.exit(main())
