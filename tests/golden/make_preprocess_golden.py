"""Generates tests/golden/preprocess_vectors.npz: the reference's image
preprocessing (src/Preprocess.cpp:13-77, `Preprocessor::operator()`) run with
the OpenCV calls it makes (cv2 4.13 here: cv::resize INTER_LINEAR,
cv::copyMakeBorder, cv::dnn::blobFromImage), on seeded 8-bit BGR images.
tests/test_preprocess_pinned.py replays every case through
oracle/preprocess.py; the device kernel is checked against that restatement.

Run from the repository root:  python tests/golden/make_preprocess_golden.py
"""
import os
import sys

import cv2
import numpy as np

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "preprocess_vectors.npz")


def reference_preprocess(bgr, in_h, in_w, letterbox, to_rgb, normalize, mean, std):
    """Preprocess.cpp:13-77 step by step, with float32 arithmetic where the
    C++ uses float (std::round is half away from zero)."""
    if letterbox:
        scale = np.float32(min(np.float32(in_w) / np.float32(bgr.shape[1]), np.float32(in_h) / np.float32(bgr.shape[0])))
        rw = int(np.floor(np.float32(bgr.shape[1]) * scale + np.float32(0.5)))
        rh = int(np.floor(np.float32(bgr.shape[0]) * scale + np.float32(0.5)))
        pw, ph = in_w - rw, in_h - rh
        pl, pt = pw // 2, ph // 2
        resized = cv2.resize(bgr, (rw, rh), interpolation=cv2.INTER_LINEAR)
        canvas = cv2.copyMakeBorder(resized, pt, ph - pt, pl, pw - pl, cv2.BORDER_CONSTANT, value=(114, 114, 114))
        info = (float(scale), pl, pt)
    else:
        canvas = cv2.resize(bgr, (in_w, in_h), interpolation=cv2.INTER_LINEAR)
        info = (1.0, 0, 0)
    blob = cv2.dnn.blobFromImage(canvas, (1.0 / 255.0) if normalize else 1.0, (in_w, in_h), (0, 0, 0),
                                 swapRB=to_rgb, crop=False, ddepth=cv2.CV_32F)[0]
    for c in range(blob.shape[0]):
        if len(mean) or len(std):
            m = np.float32(mean[c]) if c < len(mean) else np.float32(0)
            s = np.float32(std[c]) if c < len(std) else np.float32(1)
            if s == 0:
                s = np.float32(1)
            blob[c] = (blob[c] - m) / s
    return blob.astype(np.float32), info


def main():
    rng = np.random.default_rng(77)
    cases = {
        "up2_exact": (48, 64, 96, 128, 1, 1, 1, (), ()),
        "down_pad_top": (90, 160, 96, 128, 1, 1, 1, (), ()),
        "down_pad_left": (200, 150, 96, 96, 1, 1, 1, (), ()),
        "odd_up": (37, 53, 64, 64, 1, 1, 1, (), ()),
        "direct_resize": (50, 70, 64, 96, 0, 1, 1, (), ()),
        "mean_std": (60, 80, 64, 64, 1, 1, 1, (0.485, 0.456, 0.406), (0.229, 0.224, 0.225)),
        "bgr_raw": (45, 61, 64, 64, 1, 0, 0, (), ()),
        "identity": (64, 64, 64, 64, 1, 1, 1, (), ()),
    }
    flat = {}
    for name, (H, W, ih, iw, lb, rgb, norm, mean, std) in cases.items():
        img = rng.integers(0, 256, (H, W, 3), dtype=np.uint8)
        blob, info = reference_preprocess(img, ih, iw, lb, rgb, norm, mean, std)
        flat[f"{name}/image"] = img
        flat[f"{name}/params"] = np.array([ih, iw, lb, rgb, norm], np.int64)
        flat[f"{name}/mean"] = np.array(mean, np.float32)
        flat[f"{name}/std"] = np.array(std, np.float32)
        flat[f"{name}/blob"] = blob
        flat[f"{name}/letterbox"] = np.array(info, np.float32)
    np.savez_compressed(OUT, **flat)
    print("wrote", OUT, len(cases), "cases", os.path.getsize(OUT), "bytes")


if __name__ == "__main__":
    sys.exit(main())
