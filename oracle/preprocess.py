"""Restatement of the reference's image preprocessing - TEST INFRASTRUCTURE.

Follows src/Preprocess.cpp:13-77 (`Preprocessor::operator()`): letterbox
(scale = min(in_w / cols, in_h / rows) in float, resized size rounded half
away from zero, padding split with the odd pixel at the right / bottom),
cv::resize INTER_LINEAR, cv::copyMakeBorder with 114, cv::dnn::blobFromImage
(BGR -> RGB swap, x 1/255 in float), then (v - mean) / std per channel; and
the f32 -> f16 truncating cast ClBackend::infer applies to that blob
(include/infvino/Half.hpp:14-24).

The image operations are OpenCV's (a dependency absent from the reference
tree; OpenCV 4.13 is the version this restatement is pinned to, through the
golden vectors of tests/golden/make_preprocess_golden.py generated with cv2).
Their published algorithm for 8-bit images, restated here:
  * cv::resize INTER_LINEAR: per destination column, the source coordinate
    fx = float((dx + 0.5) * scale - 0.5) with scale = 1 / (dw / sw) (computed
    in double, rounded to float), sx = floor(fx), weight fx - sx; columns left of the image or past
    its last column are clamped with weight 0; weights are 11-bit fixed point
    (round(w * 2048)); the horizontal pass sums two taps in int32.  Rows use
    the same coordinate rule but keep their weights when the row index is
    clamped (both taps then read the same edge row).  The vertical pass is the
    vectorised one: ((b0 * (r0 >> 4)) >> 16) + ((b1 * (r1 >> 4)) >> 16) + 2) >> 2;
  * blobFromImage with scalefactor 1/255: float(u8) * float(1/255).
"""
from __future__ import annotations

import numpy as np


def _round_half_away(x: np.float32) -> int:
    x = float(x)
    return int(np.floor(x + 0.5)) if x >= 0 else -int(np.floor(-x + 0.5))


def letterbox_geometry(src_h: int, src_w: int, in_h: int, in_w: int):
    """(scale, resized_w, resized_h, pad_left, pad_top) as Preprocess.cpp:20-27 computes them."""
    scale = min(np.float32(in_w) / np.float32(src_w), np.float32(in_h) / np.float32(src_h))
    scale = np.float32(scale)
    rw = _round_half_away(np.float32(np.float32(src_w) * scale))
    rh = _round_half_away(np.float32(np.float32(src_h) * scale))
    return scale, rw, rh, (in_w - rw) // 2, (in_h - rh) // 2


def _coords(src: int, dst: int, clamp_weight: bool):
    scale = 1.0 / (dst / src)  # OpenCV's scale: the inverse of dsize / ssize, in double
    d = np.arange(dst, dtype=np.float64)
    f = ((d + 0.5) * scale - 0.5).astype(np.float32)
    s = np.floor(f).astype(np.int64)
    f = (f - s.astype(np.float32)).astype(np.float32)
    if clamp_weight:
        lo = s < 0
        f[lo] = 0
        s[lo] = 0
        hi = s >= src - 1
        f[hi] = 0
        s[hi] = src - 1
    w1 = np.round(f * np.float32(2048)).astype(np.int64)
    w0 = np.round((np.float32(1) - f) * np.float32(2048)).astype(np.int64)
    return np.clip(s, 0, src - 1), np.clip(s + 1, 0, src - 1), w0, w1


def resize_linear_u8(img: np.ndarray, dw: int, dh: int) -> np.ndarray:
    """cv::resize(img, (dw, dh), INTER_LINEAR) for an HxWxC uint8 image."""
    H, W, _ = img.shape
    sx, sx1, a0, a1 = _coords(W, dw, True)
    sy, sy1, b0, b1 = _coords(H, dh, False)
    I = img.astype(np.int64)
    hor = I[:, sx, :] * a0[None, :, None] + I[:, sx1, :] * a1[None, :, None]
    r0, r1 = hor[sy], hor[sy1]
    b0, b1 = b0[:, None, None], b1[:, None, None]
    v = (((b0 * (r0 >> 4)) >> 16) + ((b1 * (r1 >> 4)) >> 16) + 2) >> 2
    return np.clip(v, 0, 255).astype(np.uint8)


def preprocess(bgr: np.ndarray, in_h: int, in_w: int, letterbox: bool = True, to_rgb: bool = True,
               normalize: bool = True, mean=(), std=()):
    """Preprocessor::operator() -> (f32 NCHW blob [3, in_h, in_w], (scale, pad_left, pad_top))."""
    H, W, _ = bgr.shape
    if letterbox:
        scale, rw, rh, pl, pt = letterbox_geometry(H, W, in_h, in_w)
        canvas = np.full((in_h, in_w, 3), 114, dtype=np.uint8)
        canvas[pt:pt + rh, pl:pl + rw] = resize_linear_u8(bgr, rw, rh)
        info = (float(scale), pl, pt)
    else:
        canvas = resize_linear_u8(bgr, in_w, in_h)
        info = (1.0, 0, 0)
    chw = canvas[:, :, ::-1] if to_rgb else canvas
    blob = chw.transpose(2, 0, 1).astype(np.float32)
    if normalize:
        blob = blob * np.float32(1.0 / 255.0)
    if len(mean) or len(std):
        for c in range(3):
            m = np.float32(mean[c]) if c < len(mean) else np.float32(0)
            s = np.float32(std[c]) if c < len(std) else np.float32(1)
            if s == 0:
                s = np.float32(1)
            blob[c] = (blob[c] - m) / s
    return np.ascontiguousarray(blob, dtype=np.float32), info
