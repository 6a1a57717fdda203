"""fp16 conversions pinned to the reference's own code.

The golden vectors in tests/golden/half_vectors.npz were produced by the
reference's src/Half.cpp (built from its sources into oracle/_ref by
`make -C oracle ref`; generator: tests/golden/make_golden.py).  Both the oracle
and the product's host/device conversions must reproduce them bit for bit:
truncating f32->f16 (include/infvino/Half.hpp:14-24) and exact f16->f32
(Half.hpp:26-47)."""
import os

import numpy as np
import pytest

from oracle import ivref

GOLD = os.path.join(os.path.dirname(__file__), "golden", "half_vectors.npz")


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD)


def test_golden_scalar_vs_bulk(gold):
    # The reference's AVX2 bulk paths agree with its scalar functions except for
    # fp16 NaN inputs, which the bulk widening (src/Half.cpp:58-84) turns into
    # +-inf while the scalar one (Half.hpp:26-47) keeps the NaN.  This build
    # follows the scalar semantics (NaN stays NaN).
    assert np.array_equal(gold["f16_trunc_scalar"], gold["f16_trunc_bulk"])
    h = gold["f16_all"]
    nan = (((h >> 10) & 31) == 31) & ((h & 0x3FF) != 0)
    ws, wb = gold["f32_widen_scalar"], gold["f32_widen_bulk"]
    assert np.array_equal(ws[~nan], wb[~nan])
    assert np.all((wb[nan] & 0x7FFFFFFF) == 0x7F800000)


def test_oracle_truncating_cast_matches_reference(gold):
    x = gold["f32_in"].view(np.float32)
    assert np.array_equal(ivref.f32_to_f16_trunc(x), gold["f16_trunc_scalar"])


def test_oracle_widening_matches_reference(gold):
    got = ivref.f16_to_f32(gold["f16_all"]).view(np.uint32)
    assert np.array_equal(got, gold["f32_widen_scalar"])


def test_product_host_cast_matches_reference(gold):
    import infvino_b200 as ivb
    x = gold["f32_in"].view(np.float32)
    assert np.array_equal(ivb.f32_to_f16(x), gold["f16_trunc_scalar"])
    assert np.array_equal(ivb.f16_to_f32(gold["f16_all"]).view(np.uint32), gold["f32_widen_scalar"])


def test_oracle_rne_cast_matches_ieee():
    # node outputs are rounded to nearest-even; numpy's float16 cast is IEEE RNE
    rng = np.random.default_rng(3)
    x = np.concatenate([rng.integers(0, 2 ** 32, 200000, dtype=np.uint64).astype(np.uint32).view(np.float32),
                        (rng.standard_normal(100000) * 1e-5).astype(np.float32),
                        (rng.standard_normal(100000) * 3e4).astype(np.float32)])
    x = x[np.isfinite(x)]
    ref = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(ivref.f32_to_f16_rne(x), ref)


@pytest.mark.skipif(ivref.ref_half_lib() is None, reason="reference Half.cpp not built here (oracle/_ref)")
def test_live_reference_half_random():
    L = ivref.ref_half_lib()
    rng = np.random.default_rng(11)
    x = rng.integers(0, 2 ** 32, 1 << 20, dtype=np.uint64).astype(np.uint32).view(np.float32)
    ref = np.empty(x.size, dtype=np.uint16)
    L.ref_f32_to_f16_bulk(x.ctypes.data, ref.ctypes.data, x.size)
    assert np.array_equal(ivref.f32_to_f16_trunc(x), ref)


def test_product_host_cast_large_and_concurrent():
    """The product's host cast is vectorised and spread over a shared worker
    pool: arrays far above the pool's split threshold, lengths that leave a
    scalar tail after the 16-wide vector loop, and several calls at once from
    different threads (ctypes releases the GIL) each give the reference's
    truncation (oracle/ivref.py) bit for bit."""
    import threading
    import infvino_b200 as ivb
    rng = np.random.default_rng(41)
    bits = rng.integers(0, 1 << 32, size=(1 << 21) + 13, dtype=np.uint64).astype(np.uint32)
    specials = np.array([0, 0x80000000, 0x7f800000, 0xff800000, 0x7fc00000, 0x38800000, 0x387fffff, 0x477fe000,
                         0x477ff000, 0x47800000, 0x33800000, 0xb8800000], dtype=np.uint32)
    bits[:specials.size] = specials
    x = bits.view(np.float32)
    want = ivref.f32_to_f16_trunc(x)
    assert np.array_equal(ivb.f32_to_f16(x), want)
    for n in (1, 15, 16, 17, 31, 1000003):
        assert np.array_equal(ivb.f32_to_f16(x[:n]), want[:n]), n
    results, errors = {}, []

    def work(k):
        try:
            sl = slice(k * 1000, k * 1000 + (1 << 20) + k)
            results[k] = np.array_equal(ivb.f32_to_f16(x[sl]), want[sl])
        except Exception as e:  # reported below
            errors.append(e)

    threads = [threading.Thread(target=work, args=(k,)) for k in range(6)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errors and all(results.get(k) for k in range(6)), (errors, results)


def test_product_host_cast_any_destination_alignment():
    """The host cast streams its stores from the first 32-byte boundary of the
    destination on (scalar head before it): every start offset inside a line,
    short and long spans, give the reference's truncation bit for bit."""
    from infvino_b200 import _native
    L = _native.lib()
    rng = np.random.default_rng(43)
    x = rng.integers(0, 1 << 32, size=300000, dtype=np.uint64).astype(np.uint32).view(np.float32)
    want = ivref.f32_to_f16_trunc(x)
    buf = np.zeros(x.size + 64, dtype=np.uint16)
    for off in range(0, 17):
        for n in (1, 7, 16, 33, 100, 299000):
            dst = buf[off:off + n]
            dst[:] = 0xFFFF
            L.ivc_f32_to_f16(x.ctypes.data, dst.ctypes.data, n)
            assert np.array_equal(dst, want[:n]), (off, n)
