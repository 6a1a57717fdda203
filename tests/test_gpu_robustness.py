"""Failure handling on the GPU without any fault: the convolution kernel's
bounded waits.  A probe makes each conv CTA first wait on a barrier that
nothing arrives on; with a short limit that wait runs out, the kernel drains
its copies and MMAs, releases TMEM and reports its status word, and the call
returns IVC_ERR_KERNEL.  The handle must then run correctly again."""
import re

import numpy as np
import pytest

import infvino_b200 as ivb
from infvino_b200 import _native, plangen

IVC_ERR_KERNEL = 5
# kernel status words of a bounded wait that ran out: the probe's own (7), or
# that of another role whose wait, as short, ran out first (1-4: full, empty,
# accumulator full, accumulator empty); first one wins
TIMEOUT_STATUS = {1, 2, 3, 4, 7}
SHORT_LIMIT = 2_000_000  # SM clocks, about 1 ms
DEFAULT_LIMIT = 4_000_000_000


@pytest.mark.gpu
@pytest.mark.parametrize("flags", [0, ivb.FLAG_NO_GRAPH], ids=["graph", "eager"])
def test_conv_wait_timeout_reported_and_handle_recovers(tmp_path, flags):
    # a 3x3 conv between two 1x1 convs: three conv_tc launches per run
    p = plangen.op_conv(str(tmp_path / "p"), 32, 32, 40, 40, 3, 1, producer=True, consumer=True)
    m = ivb.PlanModel(p, device=0, max_batch=2, flags=flags)
    x = np.random.default_rng(11).random(2 * m.inputNumel(), dtype=np.float32)
    m.setInput(ivb.f32_to_f16(x), 2)
    m.run(2)
    ref = m.readOutput(0, 2)
    L = _native.lib()
    assert L.ivc_debug_conv_wait(m.handle, SHORT_LIMIT, 1) == 0
    for _ in range(2):  # the status word is reset after each report
        with pytest.raises(ivb.NativeError) as e:
            m.run(2)
        assert e.value.status == IVC_ERR_KERNEL, str(e.value)
        code = re.search(r"status (\d+)", e.value.message)
        assert code and int(code.group(1)) in TIMEOUT_STATUS, e.value.message
    # a short limit without the probe: the waits complete well inside it
    assert L.ivc_debug_conv_wait(m.handle, 200_000_000, 0) == 0
    m.run(2)
    assert np.array_equal(m.readOutput(0, 2), ref)
    assert L.ivc_debug_conv_wait(m.handle, DEFAULT_LIMIT, 0) == 0
    m.setInput(ivb.f32_to_f16(x), 2)
    m.run(2)
    assert np.array_equal(m.readOutput(0, 2), ref)
    m.close()


@pytest.mark.gpu
def test_conv_wait_probe_on_network(tmp_path):
    """The probe on a whole network (every conv launch aborts), then the same
    handle reproduces its earlier output bit for bit."""
    p = plangen.yolov8n_pose(str(tmp_path / "y8"), imgsz=320)
    m = ivb.PlanModel(p, device=0, max_batch=2)
    x = np.random.default_rng(12).random(2 * m.inputNumel(), dtype=np.float32)
    m.setInput(ivb.f32_to_f16(x), 2)
    m.run(2)
    ref = m.readOutput(0, 2)
    L = _native.lib()
    assert L.ivc_debug_conv_wait(m.handle, SHORT_LIMIT, 1) == 0
    with pytest.raises(ivb.NativeError) as e:
        m.run(2)
    assert e.value.status == IVC_ERR_KERNEL
    assert L.ivc_debug_conv_wait(m.handle, DEFAULT_LIMIT, 0) == 0
    m.setInput(ivb.f32_to_f16(x), 2)
    m.run(2)
    assert np.array_equal(m.readOutput(0, 2), ref)
    m.close()
