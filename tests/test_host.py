"""Host-side logic, no GPU: C-ABI exports, plan parsing and its errors, the
load-time rewrites, layout planning and the liveness arena allocator
(IVC_FLAG_DRY_RUN builds everything except device state)."""
import os
import re

import numpy as np
import pytest

import infvino_b200 as ivb
from infvino_b200 import _native, plangen

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_library_exports_every_declared_symbol():
    hdr = open(os.path.join(ROOT, "include", "infvino_b200.h")).read()
    declared = set(re.findall(r"\b(ivc_[a-z0-9_]+)\s*\(", hdr))
    assert declared == set(_native.SIGNATURES), declared ^ set(_native.SIGNATURES)
    L = _native.lib()
    for name in declared:
        assert hasattr(L, name), name


def dry(plan, max_batch=64, flags=0):
    return ivb.PlanModel(plan, max_batch=max_batch, flags=ivb.FLAG_DRY_RUN | flags)


def test_yolov8n_pose_plan_facts(model_plans):
    m = dry(model_plans["yolov8n-pose"])
    assert m.inputName() == "images" and m.inputDims() == [1, 3, 640, 640]
    assert m.outputCount() == 1 and m.outputDims(0) == [1, 56, 8400]
    steps = m.steps()
    gflop = sum(s["flops_per_image"] for s in steps) / 1e9
    # the reference publishes 9.178 GFLOP for yolov8n-pose conv+gemm work
    # (docs/budget-analysis-3models.md:73)
    assert abs(gflop - 9.178) < 0.002, gflop
    st = m.pool_stats()
    assert st["fusions_concat"] == 13 and st["fusions_res"] == 6
    # liveness packing (the graph input keeps its own bytes for the whole run,
    # as the reference's input buffer does)
    assert 0 < st["arena_bytes"] < st["requested_bytes"] / 3
    fam = {s["family"] for s in steps}
    assert {"conv3x3_tc", "conv1x1_tc", "stem3x3"} <= fam


def test_mobilenet_and_yolo11_plan_facts(model_plans):
    m = dry(model_plans["mobilenetv3-small"], 8)
    assert m.outputDims(0) == [1, 1000]
    gflop = sum(s["flops_per_image"] for s in m.steps()) / 1e9
    assert 0.10 < gflop < 0.13
    m11 = dry(model_plans["yolo11n-pose"], 8)
    fam = [s["family"] for s in m11.steps()]
    assert "bmm" in fam and "depthwise" in fam


def test_allocator_reuses_memory_and_views(model_plans):
    m = dry(model_plans["yolov8n-pose"], 1, ivb.FLAG_SERIAL)
    st = m.pool_stats()
    assert st["views"] > 0            # reshape + zero-copy channel splits
    text = m.describe()
    # every arena placement line has a lifetime; with one stream, roots whose
    # node lifetimes intersect never share bytes (values that stay inside a
    # fused step are not materialized and may)
    roots = []
    placed = 0
    for line in text.splitlines():
        mm = re.search(r"arena=(\d+) life=\[(-?\d+),(-?\d+)\] bytes/img=(\d+)", line)
        if mm:
            placed += 1
            if "unmaterialized" in line:
                continue
            off, b, d, sz = map(int, mm.groups())
            roots.append((off, off + ((sz + 255) // 256) * 256, b, d))
    assert placed == st["roots"] and len(roots) < placed
    for i in range(len(roots)):
        for j in range(i + 1, len(roots)):
            a, c = roots[i], roots[j]
            if a[2] <= c[3] and c[2] <= a[3]:
                assert a[1] <= c[0] or c[1] <= a[0], (a, c)


def test_no_fusion_flag(model_plans):
    m = dry(model_plans["yolov8n-pose"], 1, ivb.FLAG_NO_FUSION)
    st = m.pool_stats()
    assert st["fusions_concat"] == 0 and st["fusions_res"] == 0


def _write(tmp_path, text, inits=()):
    d = tmp_path
    for name, n in inits:
        np.zeros(n, dtype=np.float16).tofile(os.path.join(d, f"init_{name}.bin"))
    p = os.path.join(d, "model.plan")
    open(p, "w").write(text)
    return p


@pytest.mark.parametrize("text,msg", [
    ("tensor y 1 4\noutput y\n", "plan has no 'input' line"),
    ("input x 1 4\ntensor y 1 4\nnode ew_unary x y op=0 n=4\n", "plan has no 'output' line"),
    ("input x 1 4\noutput y\n", "output tensor not declared"),
    ("input x 1 4\ninit w init_w.bin 4\noutput x\n", "cannot open init"),
    ("input x 1 4\ntensor y 1 4\nnode frobnicate x y\noutput y\n", "unknown op"),
    ("input x 1 4\ntensor y 1 4\nnode ew_unary x,zz y op=0\noutput y\n", "missing tensor"),
])
def test_plan_errors(tmp_path, text, msg):
    p = _write(str(tmp_path), text)
    with pytest.raises(ivb.NativeError) as e:
        dry(p, 1)
    assert msg in str(e.value)


def test_short_init_file(tmp_path):
    p = _write(str(tmp_path), "input x 1 4\ninit w init_w.bin 8\ntensor y 1 4\n"
               "node ew_binary x,w y op=0 n=4 b_scalar=0\noutput y\n", inits=[("w", 4)])
    with pytest.raises(ivb.NativeError) as e:
        dry(p, 1)
    assert "too short" in str(e.value)


def test_empty_plan_path():
    with pytest.raises(RuntimeError):
        ivb.CudaBackend(ivb.ModelInfo(plan=""))


def test_plangen_matches_onnx2plan_conventions(tmp_path):
    p = plangen.yolov8n_pose(str(tmp_path / "y8"))
    lines = open(p).read().splitlines()
    assert lines[0] == "input images 1 3 640 640"
    conv0 = next(l for l in lines if l.startswith("node conv3x3"))
    assert conv0 == ("node conv3x3 images,model.0.weight,model.0.bias,- model.0.out "
                     "stride=2 pad=1 Hout=320 Wout=320 act=1 cfg=64,8,1,32,8,2")
    # dbox * strides: ONNX-style right-aligned broadcast strides (onnx2plan.py:244-277)
    mul = [l for l in lines if l.startswith("node ew_binary") and "bdims=1,4,8400" in l]
    assert mul and mul[0].endswith("op=2 n=33600 b_scalar=0 bdims=1,4,8400,33600,8400,1,8400,0,1")
    assert lines[-1] == "output output0"


def test_fastdiv_formula_exact():
    """The conv kernel's multiply-high division (conv_tc.cuh FastDiv):
    s = ceil(log2 d), m = floor(2^(31+s)/d) + 1, q = (n*m) >> (31+s) equals n // d
    for 0 <= n < 2^31.  Checked at the ends of the range and on random n for
    divisors of every size, including powers of two and their neighbours."""
    rng = np.random.default_rng(5)
    divs = set(range(1, 300)) | {(1 << k) + e for k in range(1, 31) for e in (-1, 0, 1)}
    divs |= set(int(v) for v in rng.integers(1, 1 << 31, 2000))
    for d in sorted(divs):
        if not 1 <= d < (1 << 31):
            continue
        s = 0
        while (1 << s) < d:
            s += 1
        m = (1 << (31 + s)) // d + 1
        assert m < (1 << 32)
        n = np.concatenate([np.arange(0, 64), (1 << 31) - 1 - np.arange(64), rng.integers(0, 1 << 31, 200),
                            d * rng.integers(0, (1 << 31) // d, 50), d * rng.integers(1, (1 << 31) // d + 1, 50) - 1])
        n = n[(n >= 0) & (n < (1 << 31))].astype(object)
        q = [(int(x) * m) >> (31 + s) for x in n]
        assert q == [int(x) // d for x in n], d


def test_head_branches_on_side_streams(model_plans):
    """The pose head's independent branches are spread over several streams;
    IVC_FLAG_SERIAL keeps every step on one stream, and then the arena equals
    the serial liveness packing.  Placement is self-checked (construction
    throws on an overlap of roots whose accesses are not ordered)."""
    p = model_plans["yolov8n-pose"]
    con = ivb.PlanModel(p, device=0, max_batch=8, flags=ivb.FLAG_DRY_RUN)
    ser = ivb.PlanModel(p, device=0, max_batch=8, flags=ivb.FLAG_DRY_RUN | ivb.FLAG_SERIAL)
    side = [ln for ln in con.describe().splitlines() if ln.startswith("step") and "[stream " in ln and "[stream 0]" not in ln]
    assert len(side) >= 9 and all("model.22." in ln or "tail:" in ln for ln in side), side
    assert not any("[stream " in ln for ln in ser.describe().splitlines())
    assert ser.pool_stats()["arena_bytes"] <= con.pool_stats()["arena_bytes"]


def test_tail_program_compiles(model_plans):
    """The fused decode tail's generated CUDA source compiles with NVRTC for
    sm_100a (a dry run compiles without loading); NO_JIT keeps the
    interpreting kernel."""
    for name in ("yolov8n-pose", "yolo11n-pose"):
        p = model_plans[name]
        d = ivb.PlanModel(p, device=0, max_batch=1, flags=ivb.FLAG_DRY_RUN).describe()
        tail = [ln for ln in d.splitlines() if ln.startswith("step decode_tail")]
        assert len(tail) == 1 and "jit=V4" in tail[0], tail
        d = ivb.PlanModel(p, device=0, max_batch=1, flags=ivb.FLAG_DRY_RUN | ivb.FLAG_NO_JIT).describe()
        tail = [ln for ln in d.splitlines() if ln.startswith("step decode_tail")]
        assert len(tail) == 1 and "jit=" not in tail[0], tail


def test_sppf_pool_chain_one_step(model_plans):
    """The SPPF block's three chained 5x5 pools lower to one step (the plane of
    each 8-channel group pooled three times in shared memory); NO_FUSION keeps
    one step per pool."""
    for name in ("yolov8n-pose", "yolo11n-pose"):
        p = model_plans[name]
        fused = [s["family"] for s in ivb.PlanModel(p, device=0, max_batch=2, flags=ivb.FLAG_DRY_RUN).steps()]
        plain = [s["family"] for s in ivb.PlanModel(p, device=0, max_batch=2,
                                                    flags=ivb.FLAG_DRY_RUN | ivb.FLAG_NO_FUSION).steps()]
        assert fused.count("maxpool_chain") == 1 and "maxpool" not in fused, name
        assert plain.count("maxpool") == 3 and "maxpool_chain" not in plain, name


def test_head_concats_in_place_and_tail_fused(model_plans):
    """The head's anchor-axis concats are written in place by their convolutions,
    and everything after them (DFL softmax + projection, box / keypoint decode,
    sigmoids, the final concats) is one fused tail step; NO_FUSION keeps the
    plan's node-per-step form."""
    p = model_plans["yolov8n-pose"]
    fused = ivb.PlanModel(p, device=0, max_batch=2, flags=ivb.FLAG_DRY_RUN)
    plain = ivb.PlanModel(p, device=0, max_batch=2, flags=ivb.FLAG_DRY_RUN | ivb.FLAG_NO_FUSION)
    fam = [s["family"] for s in fused.steps()]
    names = [s["name"] for s in fused.steps()]
    assert fam.count("decode_tail") == 1 and names[-1] == "tail:output0"
    for f in ("softmax_axis", "permute_0213", "slice_axis", "ew_unary", "dfl_fused"):
        assert f not in fam, f
    assert len(plain.steps()) - len(fused.steps()) >= 20
    for cat in ("box_cat", "kpt_cat", "cls_cat"):
        assert not any(n.endswith(cat) for n in names), cat
    assert sum(n.endswith(c) for n in (s["name"] for s in plain.steps()) for c in ("box_cat", "kpt_cat", "cls_cat")) == 3
    d = fused.describe()
    assert "tensor model.22.cv2.0.2.out planar root=model.22.box_cat off=0" in d
    assert "tensor model.22.cv2.1.2.out planar root=model.22.box_cat off=6400" in d


def test_sibling_convs_merged(model_plans):
    """The pose head's first three convolutions at each scale read one input
    with one geometry: they become one convolution over their output channels
    side by side (each member padded to a multiple of 8), the member outputs
    channel views of it at 16-byte aligned offsets; the merged step counts the
    members' FLOPs, not the padding.  NO_FUSION keeps them separate."""
    p = model_plans["yolov8n-pose"]
    m = dry(p, 2)
    plain = {s["name"]: s for s in dry(p, 2, ivb.FLAG_NO_FUSION).steps()}
    d = m.describe()
    merged = {s["name"]: s for s in m.steps() if ":siblings:" in s["name"]}
    assert len(merged) == 3
    assert not any(":siblings:" in n for n in plain)
    for scale in range(3):
        root = f"siblings:model.22.cv4.{scale}.0.out"
        for br, off in (("cv4", 0), ("cv2", 56), ("cv3", 120)):
            assert f"tensor model.22.{br}.{scale}.0.out nhwc root={root} off={off}" in d, (br, scale)
            assert f"conv3x3:model.22.{br}.{scale}.0.out" not in {s["name"] for s in m.steps()}
        want = sum(plain[f"conv3x3:model.22.{br}.{scale}.0.out"]["flops_per_image"] for br in ("cv2", "cv3", "cv4"))
        assert merged["conv3x3:" + root]["flops_per_image"] == want


def test_dry_run_handle_refuses_device_calls(model_plans):
    """A dry run builds everything but device state: calls that would run,
    read or decode refuse with a clear error instead of touching the GPU."""
    m = dry(model_plans["yolov8n-pose"], 2)
    x = np.zeros(m.inputNumel(), dtype=np.uint16)
    for call in (lambda: m.setInput(x, 1), lambda: m.run(1), lambda: m.readOutput(0, 1),
                 lambda: m.decodePose(1)):
        with pytest.raises(ivb.NativeError) as e:
            call()
        assert "dry run handle" in str(e.value), str(e.value)
    # the allocation-free read refuses the same way, before it resolves any
    # device address (no CUDA call on a dry run handle)
    L = _native.lib()
    buf = np.zeros(m.tensorNumel(m.outputName(0)), dtype=np.uint16)
    st = L.ivc_read_tensor_f16_noalloc(m.handle, m.outputName(0).encode(), buf.ctypes.data, 1)
    assert st != 0
    assert "dry run handle" in L.ivc_last_error(m.handle).decode()
    # so does the conv wait diagnostic
    assert L.ivc_debug_conv_wait(m.handle, 1000, 1) != 0
    assert "dry run handle" in L.ivc_last_error(m.handle).decode()
