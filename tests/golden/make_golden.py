"""Generates tests/golden/half_vectors.npz from the reference's own fp16
conversion code (src/Half.cpp + include/infvino/Half.hpp), compiled into
oracle/_ref/libref_half.so by `make -C oracle ref`.

Run from the repository root:  python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from oracle import ivref  # noqa: E402


def f32_inputs() -> np.ndarray:
    special = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1.0, -1.0, 65504.0, 65519.99, 65520.0, 65536.0,
                        70000.0, 6.1035156e-05, 6.1e-05, 5.96e-08, 2.98e-08, 1e-10, 1e30, -1e30, 0.5, 0.1,
                        1.0009765625, 1.00048828125, 2049.0, 3.4028235e38], dtype=np.float32)
    rng = np.random.default_rng(2024)
    bits = rng.integers(0, 2 ** 32, size=8192, dtype=np.uint64).astype(np.uint32).view(np.float32)
    uni = rng.random(4096, dtype=np.float32)                        # the image input distribution
    wide = (rng.standard_normal(4096) * 3000).astype(np.float32)
    tiny = (rng.standard_normal(2048) * 1e-5).astype(np.float32)    # around the half subnormal range
    return np.concatenate([special, bits, uni, wide, tiny]).astype(np.float32)


def main():
    L = ivref.ref_half_lib()
    if L is None:
        raise SystemExit("oracle/_ref/libref_half.so missing: run `make -C oracle ref` first")
    x = f32_inputs()
    scalar = np.empty(x.size, dtype=np.uint16)
    L.ref_f32_to_f16_scalar_n(x.ctypes.data, scalar.ctypes.data, x.size)
    bulk = np.empty(x.size, dtype=np.uint16)
    L.ref_f32_to_f16_bulk(x.ctypes.data, bulk.ctypes.data, x.size)
    h = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    widen = np.empty(h.size, dtype=np.float32)
    L.ref_f16_to_f32_bulk(h.ctypes.data, widen.ctypes.data, h.size)
    widen_scalar = np.empty(h.size, dtype=np.float32)
    L.ref_f16_to_f32_scalar_n(h.ctypes.data, widen_scalar.ctypes.data, h.size)
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "half_vectors.npz")
    np.savez_compressed(out, f32_in=x.view(np.uint32), f16_trunc_scalar=scalar, f16_trunc_bulk=bulk,
                        f16_all=h, f32_widen_bulk=widen.view(np.uint32), f32_widen_scalar=widen_scalar.view(np.uint32))
    print("wrote", out, os.path.getsize(out), "bytes")


if __name__ == "__main__":
    main()
