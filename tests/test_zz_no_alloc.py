"""ivc_read_tensor_f16_noalloc, the allocation-free variant of
ivc_read_tensor_f16 (static 4 MiB device scratch per device).  This file is
collected last on purpose: the variant's scratch is process-wide state, and the
tests must hold both alone and after every other test in the process."""
import numpy as np
import pytest

import infvino_b200 as ivb
from infvino_b200 import _native, plangen

SCRATCH_BYTES = 4 << 20


def _first_nhwc_tensor(m):
    for line in m.describe().splitlines():
        parts = line.split()
        if parts and parts[0] == "tensor" and "nhwc" in parts and "init" not in parts:
            return parts[1]
    raise AssertionError("no NHWC tensor in the plan")


def _free_bytes(dev):
    """Free device memory (cudaMemGetInfo) as the process's context sees it."""
    import torch
    free, _ = torch.cuda.mem_get_info(dev)
    return free


@pytest.mark.gpu
def test_noalloc_read_matches_read_tensor(tmp_path):
    # the 1x1 producer's 64-channel NHWC output: 3.28 MB per 160x160 image
    p = plangen.op_conv(str(tmp_path / "p"), 64, 16, 160, 160, 3, 1, producer=True)
    m = ivb.PlanModel(p, device=0, max_batch=2)
    x = np.random.default_rng(3).random(2 * m.inputNumel(), dtype=np.float32)
    m.setInput(ivb.f32_to_f16(x), 2)
    m.run(2)
    L = _native.lib()
    nhwc = _first_nhwc_tensor(m)
    cases = [(nhwc, 1), (m.outputName(0), 2)]  # relayout through the scratch; dense copy
    for name, batch in cases:
        ref = m.readTensor(name, batch)
        assert ref is not None and ref.any()
        for _ in range(2):  # two calls in a row reuse the same static buffer
            got = np.full_like(ref, 0xFFFF)
            assert L.ivc_read_tensor_f16_noalloc(m._h, name.encode(), got.ctypes.data, batch) == 0
            assert np.array_equal(got, ref), name
    # a request above the static scratch is refused, with the sizes in the message
    need = m.tensorNumel(nhwc) * 2 * 2
    assert need > SCRATCH_BYTES
    buf = np.zeros(m.tensorNumel(nhwc) * 2, dtype=np.uint16)
    assert L.ivc_read_tensor_f16_noalloc(m._h, nhwc.encode(), buf.ctypes.data, 2) == 1  # IVC_ERR_ARGUMENT
    msg = L.ivc_last_error(m._h).decode()
    assert str(need) in msg and str(SCRATCH_BYTES) in msg, msg
    # and the handle keeps working afterwards
    got = np.zeros(m.tensorNumel(nhwc), dtype=np.uint16)
    assert L.ivc_read_tensor_f16_noalloc(m._h, nhwc.encode(), got.ctypes.data, 1) == 0
    assert np.array_equal(got, m.readTensor(nhwc, 1))
    m.close()


@pytest.mark.gpu
def test_noalloc_read_allocates_no_device_memory(tmp_path):
    """On a fresh handle that never grew its relayout scratch, a relayout read
    leaves the device's free memory unchanged, while the allocating read of the
    same tensor takes memory (the control that the measurement sees an
    allocation)."""
    p = plangen.op_conv(str(tmp_path / "p"), 64, 16, 160, 160, 3, 1, producer=True)
    m = ivb.PlanModel(p, device=0, max_batch=1)
    x = np.random.default_rng(4).random(m.inputNumel(), dtype=np.float32)
    m.setInput(ivb.f32_to_f16(x), 1)
    m.run(1)
    L = _native.lib()
    nhwc = _first_nhwc_tensor(m)
    small = np.zeros(m.tensorNumel(m.outputName(0)), dtype=np.uint16)
    # a first call resolves the static buffer's address (the module is loaded by then)
    assert L.ivc_read_tensor_f16_noalloc(m._h, m.outputName(0).encode(), small.ctypes.data, 1) == 0
    m.synchronize()
    got = np.zeros(m.tensorNumel(nhwc), dtype=np.uint16)
    assert got.nbytes > 2 << 20  # larger than the allocation granularity
    before = _free_bytes(0)
    for _ in range(3):
        assert L.ivc_read_tensor_f16_noalloc(m._h, nhwc.encode(), got.ctypes.data, 1) == 0
    after = _free_bytes(0)
    assert after == before, (before, after)
    ref = m.readTensor(nhwc, 1)  # grows the handle's scratch with cudaMalloc
    assert _free_bytes(0) < after
    assert np.array_equal(got, ref)
    m.close()


@pytest.mark.gpu
def test_noalloc_alternating_devices(tmp_path):
    """One thread alternates allocation-free reads between handles on two
    devices: each call makes its handle's device current before it launches."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two devices")
    p = plangen.op_conv(str(tmp_path / "p"), 64, 16, 80, 80, 3, 1, producer=True)
    ms = [ivb.PlanModel(p, device=d, max_batch=1) for d in (0, 1)]
    x = np.random.default_rng(5).random(ms[0].inputNumel(), dtype=np.float32)
    for m in ms:
        m.setInput(ivb.f32_to_f16(x), 1)
        m.run(1)
    L = _native.lib()
    nhwc = _first_nhwc_tensor(ms[0])
    ref = ms[0].readTensor(nhwc, 1)
    for _ in range(3):
        for m in ms:
            got = np.zeros_like(ref)
            assert L.ivc_read_tensor_f16_noalloc(m._h, nhwc.encode(), got.ctypes.data, 1) == 0, \
                L.ivc_last_error(m._h)
            assert np.array_equal(got, ref)
    for m in ms:
        m.close()
