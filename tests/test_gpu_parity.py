"""Parity of the CUDA path (through the C ABI) against the CPU oracle.

Op level: every kernel family on seeded inputs, batch 1 and batch > 1.  Both
sides accumulate in fp32 and apply the reference's rounding points, so almost
every element is bit-identical; a different fp32 summation order may flip a
rounding, and a producer node's flip is amplified by the next node, so the
bound is two fp16 ulps at the tensor's scale (|d| <= 2 * 2^-10 * max|ref|) on
at most 1% of the elements.
Network level (BASELINE tolerances): raw head tensors max-abs <= 2e-2 and
relative L2 <= 1e-3; decoded box / keypoint coordinates within 0.5 px; identical
post-NMS detection sets; two different inputs in one process (reuse check).
"""
import os

import numpy as np
import pytest

import infvino_b200 as ivb
from infvino_b200 import plangen
from oracle import decode, ivref

pytestmark = pytest.mark.gpu


def ulp_diff(a16: np.ndarray, b16: np.ndarray) -> np.ndarray:
    """Distance in fp16 ulps between two arrays of fp16 bit patterns."""
    def ordinal(h):
        h = h.astype(np.int32)
        return np.where(h & 0x8000, -(h & 0x7FFF), h & 0x7FFF)
    return np.abs(ordinal(a16) - ordinal(b16))


def run_both(plan, batch, seed=0, flags=ivb.FLAG_NO_POOL, return_input=False):
    # NO_POOL keeps every intermediate tensor readable after the run (the
    # reference's INFVINO_NO_POOL diagnostic), numerics are unchanged
    o = ivref.OraclePlan(plan)
    x = np.random.default_rng(seed).random(batch * o.input_numel, dtype=np.float32)
    x16 = ivref.f32_to_f16_trunc(x)
    o.run_f16(x16, batch)
    m = ivb.PlanModel(plan, device=0, max_batch=batch, flags=flags)
    m.setInput(x16, batch)
    m.run(batch)
    return (o, m, x16) if return_input else (o, m)


def check_op(plan, batch, ulps=2.0, max_frac=0.01):
    o, m = run_both(plan, batch)
    for i in range(m.outputCount()):
        got = m.readOutput(i, batch)
        ref = o.read_f16(m.outputName(i))
        assert got.shape == ref.shape
        g, r = ivref.f16_to_f32(got), ivref.f16_to_f32(ref)
        assert np.isfinite(g).all()
        scale = float(np.abs(r).max())
        d = np.abs(g.astype(np.float64) - r)
        assert d.max() <= ulps * 2.0 ** -10 * scale, (plan, float(d.max()), scale)
        frac = float(np.mean(ulp_diff(got, ref) > 0))
        assert frac <= max_frac, (plan, frac)
    m.close()


CONV1 = [(16, 16, 80), (32, 64, 40), (64, 32, 40), (128, 128, 20), (256, 64, 20), (48, 256, 20), (24, 88, 14)]


@pytest.mark.parametrize("cin,cout,hw", CONV1)
@pytest.mark.parametrize("batch", [1, 5])
def test_conv1x1(plan_dir, cin, cout, hw, batch):
    p = plangen.op_conv(os.path.join(plan_dir, f"c1_{cin}_{cout}_{hw}"), cin, cout, hw, hw, 1, act=1, producer=True)
    check_op(p, batch)


CONV3 = [(16, 16, 40, 1), (32, 32, 20, 1), (64, 64, 40, 2), (16, 32, 80, 2), (64, 51, 20, 1), (51, 51, 40, 1),
         (128, 128, 10, 1), (128, 256, 20, 2), (64, 64, 7, 1), (256, 64, 20, 1),
         # weights too large to stay resident: halo tiles with each chunk's nine tap blocks in the stage
         (128, 64, 40, 1), (128, 51, 40, 1), (192, 64, 20, 1), (128, 64, 13, 1)]


@pytest.mark.parametrize("cin,cout,hw,s", CONV3)
@pytest.mark.parametrize("batch", [1, 3])
def test_conv3x3(plan_dir, cin, cout, hw, s, batch):
    p = plangen.op_conv(os.path.join(plan_dir, f"c3_{cin}_{cout}_{hw}_{s}"), cin, cout, hw, hw, 3, s, act=1,
                        producer=True)
    check_op(p, batch)


# 3x3 convs whose weights fit neither resident nor travelling with each halo
# stage: N split in two or four tiles, each CTA keeping one N tile's weights
# (the YOLOv8 head's merged P3 conv, the 20x20 128-channel bottlenecks, a
# stride-2 conv, Cout not a multiple of the N tile)
SPLIT3 = [(128, 128, 20, 1, 64), (64, 179, 40, 1, 16), (64, 128, 40, 2, 8), (128, 179, 20, 1, 2), (128, 128, 10, 1, 3)]


@pytest.mark.parametrize("cin,cout,hw,s,batch", SPLIT3)
def test_conv3x3_split_resident(plan_dir, cin, cout, hw, s, batch):
    p = plangen.op_conv(os.path.join(plan_dir, f"sp_{cin}_{cout}_{hw}_{s}"), cin, cout, hw, hw, 3, s, act=1,
                        producer=True, consumer=True)
    o, m = run_both(p, batch, flags=ivb.FLAG_NO_POOL | ivb.FLAG_NO_TUNE)
    geo = [ln for ln in m.describe().splitlines() if ln.startswith("step conv3x3_tc conv3x3:op.out")]
    assert geo and f"halo={s}" in geo[0], geo
    # the op's own output against the oracle (the usual bar), and the consumer's
    # (which amplifies the op's rounding flips: the max-abs bound only)
    for name, frac_bound in (("op.out", 0.01), (m.outputName(0), None)):
        got = m.readTensor(name, batch)
        ref = o.read_f16(name)
        g, r = ivref.f16_to_f32(got), ivref.f16_to_f32(ref)
        scale = float(np.abs(r).max())
        assert np.abs(g.astype(np.float64) - r).max() <= 2.0 * 2.0 ** -10 * scale, name
        if frac_bound is not None:
            assert float(np.mean(ulp_diff(got, ref) > 0)) <= frac_bound, name
    m.close()


@pytest.mark.parametrize("act", [0, 3])
def test_conv3x3_activations(plan_dir, act):
    p = plangen.op_conv(os.path.join(plan_dir, f"c3act{act}"), 32, 32, 20, 20, 3, 1, act=act)
    check_op(p, 2)


@pytest.mark.parametrize("act", [0, 1, 2, 3, 4])
def test_conv1x1_activations(plan_dir, act):
    p = plangen.op_conv(os.path.join(plan_dir, f"c1act{act}"), 32, 48, 20, 20, 1, 1, act=act)
    check_op(p, 2)


def test_conv3x3_residual(plan_dir):
    p = plangen.op_conv(os.path.join(plan_dir, "c3res"), 32, 32, 20, 20, 3, 1, residual=True, producer=True)
    check_op(p, 3)


# Larger launches whose tiles span several 128-pixel M blocks (the tile size is
# picked per batch from the tile count): partial tiles at the right edge and at
# the end of the pixel range, stride-2 phases, a residual, Cout not a multiple
# of 16, and many tiles per CTA with four accumulator buffers.
MULTIBLOCK = [  # cin, cout, input hw, ksize, stride, batch, residual
    (16, 16, 160, 3, 1, 64, True),
    (16, 16, 100, 3, 1, 8, False),
    (16, 32, 100, 3, 2, 16, False),
    (32, 32, 60, 3, 1, 16, True),
    (64, 51, 52, 3, 1, 16, False),
    (48, 32, 90, 1, 1, 8, False),
    (16, 16, 100, 1, 1, 8, False),
    (32, 64, 80, 1, 1, 32, False),
]


# 3x3 convs with one TMA box per tap (IVC_FLAG_NO_HALO, and the path of
# convolutions whose weights fit no halo stage): 16-pixel-wide tiles of 8 * mb
# rows, M block j being rows 8j .. 8j+7; partial tiles at the bottom edge.
MULTIBLOCK_BOXES = [
    (32, 32, 64, 3, 1, 16, True),
    (16, 32, 128, 3, 2, 16, False),
    (64, 51, 80, 3, 1, 16, False),
]


@pytest.mark.parametrize("cin,cout,hw,k,s,batch,res,boxes",
                         [c + (False,) for c in MULTIBLOCK] + [c + (True,) for c in MULTIBLOCK_BOXES])
def test_conv_multiblock_tiles(plan_dir, cin, cout, hw, k, s, batch, res, boxes):
    p = plangen.op_conv(os.path.join(plan_dir, f"mb_{cin}_{cout}_{hw}_{k}_{s}_{int(res)}"), cin, cout, hw, hw, k, s,
                        act=1, residual=res, producer=True)
    # the cost model's geometry (load-time tuning could pick one M block)
    o, m = run_both(p, batch, flags=ivb.FLAG_NO_POOL | ivb.FLAG_NO_TUNE | (ivb.FLAG_NO_HALO if boxes else 0))
    geo = [ln for ln in m.describe().splitlines() if ln.startswith("step conv") and "_tc " in ln]
    assert geo and all(f"[B={batch} mb=" in ln for ln in geo), geo
    assert any(f"[B={batch} mb=1 " not in ln for ln in geo), geo  # several M blocks per tile
    for i in range(m.outputCount()):
        got = m.readOutput(i, batch)
        ref = o.read_f16(m.outputName(i))
        g, r = ivref.f16_to_f32(got), ivref.f16_to_f32(ref)
        scale = float(np.abs(r).max())
        assert np.abs(g.astype(np.float64) - r).max() <= 2.0 * 2.0 ** -10 * scale
        assert float(np.mean(ulp_diff(got, ref) > 0)) <= 0.01
    m.close()


# (a thread per pixel up to 1024 pixels; the 36x36 plane takes two per thread)
@pytest.mark.parametrize("c,hw,levels,batch", [(128, 20, 3, 1), (128, 20, 3, 9), (64, 13, 2, 5), (32, 7, 3, 3),
                                               (16, 32, 3, 2), (16, 36, 3, 2)])
def test_sppf_pool_chain(plan_dir, c, hw, levels, batch):
    p = plangen.op_sppf(os.path.join(plan_dir, f"sppf_{c}_{hw}_{levels}"), c, hw, hw, levels)
    m = ivb.PlanModel(p, max_batch=1, flags=ivb.FLAG_DRY_RUN)
    assert [s["family"] for s in m.steps()].count("maxpool_chain") == 1
    m.close()
    check_op(p, batch)
    # max is exact: each level equals 5x5 max pools (out-of-image taps skipped)
    # of this handle's own pool input, restated in numpy, value for value
    o, m = run_both(p, batch)
    cur = m.readTensor("pre.out", batch).view(np.float16).reshape(batch, c, hw, hw)
    for lv in range(levels):
        pad = np.pad(cur, ((0, 0), (0, 0), (2, 2), (2, 2)), constant_values=-np.inf)
        cur = np.lib.stride_tricks.sliding_window_view(pad, (5, 5), axis=(2, 3)).max(axis=(4, 5))
        got = m.readTensor(f"mp_{lv + 1}", batch).view(np.float16).reshape(batch, c, hw, hw)
        assert np.array_equal(got, cur), lv
    m.close()


@pytest.mark.parametrize("c,hw,s,batch", [(128, 20, 2, 1), (256, 20, 2, 6), (64, 9, 3, 4)])
def test_upsample_nearest(plan_dir, c, hw, s, batch):
    p = plangen.op_upsample(os.path.join(plan_dir, f"up_{c}_{hw}_{s}"), c, hw, hw, s)
    check_op(p, batch)


# the SE-block and classifier shapes of MobileNetV3-small (56^2 .. 7^2), plus
# fewer pixels than the 128 summation lanes and a ragged last round
@pytest.mark.parametrize("c,hw,batch", [(16, 56, 3), (96, 14, 2), (576, 7, 4), (40, 11, 5), (24, 13, 1)])
def test_gap_reference_order(plan_dir, c, hw, batch):
    """The channels-last global average pool sums in the reference's lane
    order (128 lane-strided sums, then the tree): bit-identical to the oracle."""
    p = plangen.op_gap(os.path.join(plan_dir, f"gap_{c}_{hw}"), c, hw, hw)
    m = ivb.PlanModel(p, max_batch=1, flags=ivb.FLAG_DRY_RUN)
    assert any(" nhwc " in ln for ln in m.describe().splitlines() if ln.startswith("tensor pre.out"))
    o, m = run_both(p, batch)
    assert np.array_equal(m.readOutput(0, batch), o.read_f16(m.outputName(0)))
    m.close()


# MobileNetV3-small's squeeze-excitation blocks (channels, squeeze width, plane)
@pytest.mark.parametrize("c,hw,batch", [(16, 56, 3), (96, 14, 2), (576, 7, 4), (240, 14, 1)])
def test_se_block(plan_dir, c, hw, batch):
    """Pool, the one-pixel fc1 / fc2 convs on the tensor cores (M = the batch)
    and the broadcast multiply match the oracle."""
    p = plangen.op_se(os.path.join(plan_dir, f"se_{c}_{hw}"), c, hw, hw)
    m = ivb.PlanModel(p, max_batch=1, flags=ivb.FLAG_DRY_RUN)
    fams = [st["family"] for st in m.steps()]
    assert fams == ["conv_direct", "gap", "conv1x1_tc", "conv1x1_tc", "ew_binary"], fams
    check_op(p, batch)


# YOLO11's C2PSA attention at its P5 size (20x20, 2 heads), one head, and
# sizes that leave partial 64 x 64 product tiles and K slices
@pytest.mark.parametrize("c,hw,heads,batch", [(128, 20, 2, 2), (64, 12, 1, 3), (128, 7, 2, 1), (64, 9, 2, 4)])
def test_attention_block(plan_dir, c, hw, heads, batch):
    """Both transposing permutes fold into their bmm (no permute launch), the
    tiled bmm and the row softmax match the oracle, and the folded network
    equals the unfolded one bit for bit."""
    p = plangen.op_attention(os.path.join(plan_dir, f"att_{c}_{hw}_{heads}"), c, hw, hw, heads)
    m = ivb.PlanModel(p, max_batch=1, flags=ivb.FLAG_DRY_RUN)
    fams = [st["family"] for st in m.steps()]
    assert "permute_0213" not in fams and fams.count("bmm") == 2, fams
    # eight rounding points in a row, and a flipped score changes its whole
    # softmax row: at most 2 ulps anywhere, and at most 5% of the elements off
    check_op(p, batch, max_frac=0.05)
    x = np.random.default_rng(9).random(batch * m.inputNumel(), dtype=np.float32)
    outs = []
    for flags in (0, ivb.FLAG_NO_FUSION):
        mm = ivb.PlanModel(p, device=0, max_batch=batch, flags=flags)
        mm.setInput(ivb.f32_to_f16(x), batch)
        mm.run(batch)
        outs.append(mm.readOutput(0, batch))
        mm.close()
    assert np.array_equal(outs[0], outs[1])


@pytest.mark.parametrize("batch", [4, 48])
def test_concat_conv1x1_cat4(plan_dir, batch):
    p = plangen.op_cat_conv1x1(os.path.join(plan_dir, "cat"), [16, 16, 32, 64], 64, 40, 40)
    m = ivb.PlanModel(p, max_batch=1, flags=ivb.FLAG_DRY_RUN)
    assert m.pool_stats()["fusions_concat"] == 1
    check_op(p, batch)


@pytest.mark.parametrize("c,k,s,act", [(16, 3, 2, 2), (72, 3, 2, 2), (88, 3, 1, 2), (96, 5, 2, 3), (240, 5, 1, 3),
                                       (576, 5, 1, 3), (64, 3, 1, 1), (20, 3, 1, 4)])
def test_depthwise(plan_dir, c, k, s, act):
    p = plangen.op_conv(os.path.join(plan_dir, f"dw_{c}_{k}_{s}_{act}"), c, c, 14, 14, k, s, act=act, groups=c,
                        producer=True)
    check_op(p, 3)


# BASELINE config 2's depthwise resolutions (112..7) with MobileNet's channel
# counts; `producer` puts a 1x1 conv in front and one behind (channels-last
# input and output, the 8-channel kernel), without them the depthwise reads
# the planar plan input and writes the planar output (four-output strips for
# all four K / S pairs, a partial last strip, and the one-output kernel)
@pytest.mark.parametrize("c,k,s,hw,act,producer", [
    (16, 3, 2, 112, 2, True), (72, 3, 2, 56, 2, True), (96, 5, 2, 28, 3, True), (240, 5, 1, 14, 3, True),
    (576, 5, 1, 7, 3, True), (88, 3, 1, 56, 2, True), (16, 3, 1, 112, 1, False), (72, 5, 2, 28, 4, False),
    (24, 3, 2, 7, 3, False), (32, 3, 2, 112, 2, False), (40, 5, 1, 56, 3, False), (24, 5, 2, 112, 0, False),
    (32, 3, 1, 50, 1, False)])
def test_depthwise_resolutions(plan_dir, c, k, s, hw, act, producer):
    p = plangen.op_conv(os.path.join(plan_dir, f"dwr_{c}_{k}_{s}_{hw}_{int(producer)}"), c, c, hw, hw, k, s, act=act,
                        groups=c, producer=producer, consumer=producer)
    m = ivb.PlanModel(p, max_batch=1, flags=ivb.FLAG_DRY_RUN)
    lay = {ln.split()[1]: " nhwc " in ln for ln in m.describe().splitlines() if ln.startswith("tensor")}
    assert lay["op.out"] == producer
    check_op(p, 3)


# planar depthwise over planes of at most 512 pixels with enough planes to fill
# the GPU: whole planes staged in shared memory, 16 per block (the last block
# partial in the 120-channel cases)
@pytest.mark.parametrize("c,k,s,hw,act,batch", [(128, 3, 1, 20, 0, 20), (120, 5, 2, 14, 3, 21), (96, 3, 2, 20, 2, 25),
                                                (120, 5, 1, 7, 1, 21)])
def test_depthwise_planar_small_planes(plan_dir, c, k, s, hw, act, batch):
    p = plangen.op_conv(os.path.join(plan_dir, f"dwp_{c}_{k}_{s}_{hw}"), c, c, hw, hw, k, s, act=act, groups=c)
    check_op(p, batch)


def test_generic_grouped_conv(plan_dir):
    # conv_general with groups != Cin: the reference's generic kernel (act code 2 = HardSwish there)
    p = plangen.op_conv(os.path.join(plan_dir, "grp"), 32, 32, 12, 12, 3, 1, act=2, groups=4)
    check_op(p, 2)


def test_stem(plan_dir):
    p = plangen.op_conv(os.path.join(plan_dir, "stem"), 3, 16, 96, 96, 3, 2, act=1)
    check_op(p, 3)


def test_no_tensor_core_route_matches(plan_dir):
    p = plangen.op_conv(os.path.join(plan_dir, "c3ntc"), 32, 64, 20, 20, 3, 1, act=1)
    o, m = run_both(p, 2, flags=ivb.FLAG_NO_TENSOR_CORES)
    assert ulp_diff(m.readOutput(0, 2), o.read_f16(m.outputName(0))).max() <= 1


# ------------------------------------------------------------------ networks
HEADS_V8 = [f"model.22.cv{b}.{i}.2.out" for b in (2, 3, 4) for i in range(3)]


def head_check(m, o, names, batch, plan, x16):
    """max-abs <= 2e-2 and rel-L2 <= 1e-3, where the oracle's own noise floor
    allows it: two fp32-accumulating runs that differ only in summation order
    (oracle natural vs reversed K order) already disagree by rel-L2 ~2e-3 on
    the small random-init class-head tensors, so the rel-L2 bound is
    max(1e-3, 2 x that floor)."""
    o_rev = ivref.OraclePlan(plan, acc_order=1)
    o_rev.run_f16(x16, batch)
    for n in names:
        g = ivref.f16_to_f32(m.readTensor(n, batch)).astype(np.float64)
        r = ivref.f16_to_f32(o.read_f16(n)).astype(np.float64)
        r2 = ivref.f16_to_f32(o_rev.read_f16(n)).astype(np.float64)
        maxabs = np.abs(g - r).max()
        rel = np.linalg.norm(g - r) / max(1e-30, np.linalg.norm(r))
        floor = np.linalg.norm(r2 - r) / max(1e-30, np.linalg.norm(r))
        assert maxabs <= 2e-2 and rel <= max(1e-3, 2.0 * floor), (n, maxabs, rel, floor)


def decode_check(out_gpu, out_ref):
    """Decoded coordinates within 0.5 px, and the post-NMS detection set (the
    reference's pose decoder + greedy NMS at IoU 0.7, restated in
    oracle/decode.py) identical to the oracle's for every detection whose
    decisions are clear of the measured GPU-oracle deviation: the sets may differ
    only in anchors that `decode.undecided_anchors` reports (a score within 2x
    the deviation of conf 0.25, an IoU within 2x of 0.7, a near-tie in the greedy
    order, and what overlaps them).  Returns the number of undecided anchors;
    with none, the sets are identical."""
    coord = [0, 1, 2, 3] + [5 + 3 * k for k in range(17)] + [6 + 3 * k for k in range(17)]
    d = np.abs(out_gpu[coord].astype(np.float64) - out_ref[coord])
    assert d.max() <= 0.5, float(d.max())
    und, delta, eps = decode.undecided_anchors(out_ref, out_gpu)
    got = {a for a, *_ in decode.pose_decode(out_gpu)}
    ref = {a for a, *_ in decode.pose_decode(out_ref)}
    assert (got ^ ref) <= und, (sorted((got ^ ref) - und)[:8], delta, eps)
    if not und:
        assert got == ref
    return len(und)


@pytest.mark.parametrize("batch", [1, 2])
def test_yolov8n_pose(model_plans, batch):
    p = model_plans["yolov8n-pose"]
    o, m, x16 = run_both(p, batch, seed=10 + batch, return_input=True)
    head_check(m, o, HEADS_V8, batch, p, x16)
    got = ivref.f16_to_f32(m.readOutput(0, batch)).reshape(batch, 56, 8400)
    ref = ivref.f16_to_f32(o.read_f16("output0")).reshape(batch, 56, 8400)
    for b in range(batch):
        decode_check(got[b], ref[b])
    m.close()


@pytest.mark.parametrize("seed", [11, 13, 17, 19, 23, 29, 31, 37])
def test_yolov8n_pose_nms_identical(plan_dir, seed):
    """Random-init class scores are all ~sigmoid(0.01) ~ 0.5 (ties everywhere,
    300 detections cut by max_det), so the NMS set is checked on a variant whose
    final class conv is scaled (gain 100, bias -3): 24-29 anchors pass conf 0.25
    with spread scores, as with trained weights.  The GPU's set equals the
    oracle's except for at most a few anchors whose score or IoU lies within
    twice the measured deviation of a threshold."""
    p = plangen.yolov8n_pose(os.path.join(plan_dir, "y8_peaked"), cls_gain=100.0, cls_shift=-3.0)
    o, m = run_both(p, 1, seed=seed)
    got = ivref.f16_to_f32(m.readOutput(0, 1)).reshape(56, 8400)
    ref = ivref.f16_to_f32(o.read_f16("output0")).reshape(56, 8400)
    n_und = decode_check(got, ref)
    assert n_und <= 4, n_und
    sets = [{a for a, *_ in decode.pose_decode(v)} for v in (got, ref)]
    path = os.environ.get("IVB_PARITY_REPORT")
    if path:  # the achieved agreement, for the record
        import json
        with open(path, "a") as f:
            f.write(json.dumps({"test": "nms_identical", "seed": seed, "identical": sets[0] == sets[1],
                                "detections": len(sets[1]), "undecided": n_und}) + "\n")
    m.close()


def test_yolo11n_pose(model_plans):
    p = model_plans["yolo11n-pose"]
    o, m, x16 = run_both(p, 1, seed=21, return_input=True)
    head_check(m, o, [f"model.23.cv{b}.{i}.2.out" for b in (2, 3, 4) for i in range(3)], 1, p, x16)
    got = ivref.f16_to_f32(m.readOutput(0, 1)).reshape(56, 8400)
    ref = ivref.f16_to_f32(o.read_f16("output0")).reshape(56, 8400)
    decode_check(got, ref)
    m.close()


@pytest.mark.parametrize("batch", [1, 4])
def test_mobilenetv3_small(model_plans, batch):
    p = model_plans["mobilenetv3-small"]
    o, m = run_both(p, batch, seed=30 + batch)
    g = ivref.f16_to_f32(m.readOutput(0, batch)).astype(np.float64)
    r = ivref.f16_to_f32(o.read_f16(m.outputName(0))).astype(np.float64)
    assert np.abs(g - r).max() <= 2e-2
    assert np.linalg.norm(g - r) / np.linalg.norm(r) <= 2e-3
    assert np.array_equal(g.reshape(batch, -1).argmax(1), r.reshape(batch, -1).argmax(1))
    m.close()


def test_backend_reuse_two_inputs(model_plans):
    """ClBackend-style f32 API; frame B after frame A equals a fresh B-only run
    (the reference's reuse check, scripts/reuse_check.py:6-11)."""
    p = model_plans["yolov8n-pose"]
    be = ivb.CudaBackend(ivb.ModelInfo(plan=p))
    n = int(np.prod(be.inputDims()))
    xa = np.random.default_rng(1).random(n, dtype=np.float32)
    xb = np.random.default_rng(2).random(n, dtype=np.float32)
    be.infer(xa)
    yb = be.infer(xb)[0].data.copy()
    fresh = ivb.CudaBackend(ivb.ModelInfo(plan=p)).infer(xb)[0].data
    assert np.array_equal(yb, fresh)
    assert be.lastInferMs() > 0
    with pytest.raises(ivb.NativeError) as e:
        be.model.infer_f32(xa[:-1], 1)
    assert "numel mismatch" in str(e.value)


def test_run_repeats_without_set_input(model_plans):
    """PlanModel::run() called again after one setInput() reads the same input
    (the graph input keeps its own memory, as the reference's input buffer
    does): the output is the same every time."""
    p = model_plans["yolov8n-pose"]
    m = ivb.PlanModel(p, max_batch=2)
    x = np.random.default_rng(6).random(2 * m.inputNumel(), dtype=np.float32)
    m.setInput(ivb.f32_to_f16(x), 2)
    m.run(2)
    y0 = m.readOutput(0, 2)
    for _ in range(3):
        m.run(2)
        assert np.array_equal(m.readOutput(0, 2), y0)
    m.close()


def test_batched_equals_single(model_plans):
    """Image b of a batch-3 run equals the same image run alone (batch sharding is exact)."""
    p = model_plans["yolov8n-pose"]
    m = ivb.PlanModel(p, max_batch=3)
    n = m.inputNumel()
    x = np.random.default_rng(5).random(3 * n, dtype=np.float32)
    yb = m.infer_f32(x, 3)[0].reshape(3, -1)
    for b in range(3):
        y1 = m.infer_f32(x[b * n:(b + 1) * n], 1)[0]
        assert np.array_equal(y1, yb[b])
    m.close()


def test_head_fusions_bit_identical(plan_dir):
    """Concat-in-place, the merged sibling convolutions and the fused DFL step
    change no output bit: the default handle equals a NO_FUSION handle (the plan
    run node by node, plus no CAT4/RES rewrites) on the decoded output, and the
    in-place and merged head tensors read back the same.  Both handles use one
    TMA box per tap for 3x3 convs: a merged head conv's weights fit no halo
    stage, and the halo tiles sum a multi-chunk conv's k-blocks chunk by chunk
    where the per-tap boxes go tap by tap."""
    p = plangen.yolov8n_pose(os.path.join(plan_dir, "y8_320"), imgsz=320)
    n = 3 * 320 * 320
    x = np.random.default_rng(17).random(2 * n, dtype=np.float32)
    a = ivb.PlanModel(p, max_batch=2, flags=ivb.FLAG_NO_POOL | ivb.FLAG_NO_HALO)
    b = ivb.PlanModel(p, max_batch=2, flags=ivb.FLAG_NO_POOL | ivb.FLAG_NO_HALO | ivb.FLAG_NO_FUSION)
    assert any(ln.startswith("step conv3x3_tc conv3x3:siblings:") for ln in a.describe().splitlines())
    ya, yb = a.infer_f32(x, 2)[0], b.infer_f32(x, 2)[0]
    assert np.array_equal(ya, yb)
    for name in ("model.22.cv2.1.2.out", "model.22.cv4.2.2.out", "model.22.cv3.0.2.out", "model.22.cv4.0.0.out",
                 "model.22.cv2.1.0.out", "model.22.cv3.2.0.out"):
        assert np.array_equal(a.readTensor(name, 2), b.readTensor(name, 2)), name
    a.close()
    b.close()


@pytest.mark.parametrize("model,imgsz,batch", [("y8", 320, 2), ("y8", 640, 3), ("y11", 320, 1)])
def test_tail_compiled_equals_interpreted(plan_dir, model, imgsz, batch):
    """The load-time compiled decode tail (NVRTC) is active on the device and
    gives bit-identical outputs to the interpreting tail kernel (NO_JIT)."""
    gen = plangen.yolov8n_pose if model == "y8" else plangen.yolo11n_pose
    p = gen(os.path.join(plan_dir, f"{model}_{imgsz}"), imgsz=imgsz)
    x = np.random.default_rng(23).random(batch * 3 * imgsz * imgsz, dtype=np.float32)
    a = ivb.PlanModel(p, max_batch=batch)
    b = ivb.PlanModel(p, max_batch=batch, flags=ivb.FLAG_NO_JIT)
    tail_a = [ln for ln in a.describe().splitlines() if ln.startswith("step decode_tail")]
    tail_b = [ln for ln in b.describe().splitlines() if ln.startswith("step decode_tail")]
    assert tail_a and "jit=V" in tail_a[0], tail_a
    assert tail_b and "jit=" not in tail_b[0], tail_b
    ya, yb = a.infer_f32(x, batch)[0], b.infer_f32(x, batch)[0]
    assert np.array_equal(ya, yb)
    a.close()
    b.close()


def test_tuned_geometry_changes_no_bit(plan_dir):
    """Load-time tuning times several tile geometries per conv and keeps the
    fastest; every geometry accumulates each output in the same order, so the
    tuned handle equals the cost-model handle bit for bit."""
    p = plangen.yolov8n_pose(os.path.join(plan_dir, "y8_320"), imgsz=320)
    x = np.random.default_rng(29).random(6 * 3 * 320 * 320, dtype=np.float32)
    a = ivb.PlanModel(p, max_batch=6)
    b = ivb.PlanModel(p, max_batch=6, flags=ivb.FLAG_NO_TUNE)
    ya, yb = a.infer_f32(x, 6)[0], b.infer_f32(x, 6)[0]
    assert np.array_equal(ya, yb)
    da, db = a.describe(), b.describe()
    assert " tuned" in da and " tuned" not in db and " model" in db
    a.close()
    b.close()


@pytest.mark.parametrize("model,batch", [("yolov8n-pose", 3), ("yolo11n-pose", 2), ("mobilenetv3-small", 4)])
def test_concurrent_branches_equal_serial(model_plans, model, batch):
    """The graph with the head's branches on side streams gives the same bits
    as the one-stream graph, and keeps doing so on a second run (no stale or
    overwritten buffer between concurrent branches)."""
    p = model_plans[model]
    a = ivb.PlanModel(p, max_batch=batch)
    b = ivb.PlanModel(p, max_batch=batch, flags=ivb.FLAG_SERIAL)
    n = a.inputNumel()
    for seed in (31, 37):
        x = np.random.default_rng(seed).random(batch * n, dtype=np.float32)
        ya, yb = a.infer_f32(x, batch), b.infer_f32(x, batch)
        for u, v in zip(ya, yb):
            assert np.array_equal(u, v)
    a.close()
    b.close()


def test_graph_and_eager_agree(model_plans):
    p = model_plans["mobilenetv3-small"]
    x = np.random.default_rng(9).random(2 * 3 * 224 * 224, dtype=np.float32)
    a = ivb.PlanModel(p, max_batch=2).infer_f32(x, 2)[0]
    b = ivb.PlanModel(p, max_batch=2, flags=ivb.FLAG_NO_GRAPH).infer_f32(x, 2)[0]
    c = ivb.PlanModel(p, max_batch=2, flags=ivb.FLAG_NO_FUSION).infer_f32(x, 2)[0]
    assert np.array_equal(a, b) and np.array_equal(a, c)


def test_infer_f32_chunked_equals_device_path(model_plans):
    """ClBackend::infer on host buffers pipelines chunks of 16 images (copies
    overlapping the network); the outputs equal one device-resident pass over
    the whole batch, image for image."""
    p = model_plans["yolov8n-pose"]
    m = ivb.PlanModel(p, max_batch=40)
    n = m.inputNumel()
    x = np.random.default_rng(23).random(40 * n, dtype=np.float32)
    y_host = m.infer_f32(x, 40)[0]
    import torch
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty(40 * m.outputNumel(0), dtype=torch.float32, device="cuda")
    m.infer_f32_device(xd.data_ptr(), 40, [yd.data_ptr()])
    m.synchronize()
    assert np.array_equal(y_host, yd.cpu().numpy())
    m.close()


def test_infer_f32_split_tuning_changes_no_bit(model_plans):
    """The first calls of ivc_infer_f32 at a batch of 32 or more try five
    host / device cast splits; every call returns the same bits."""
    import torch
    p = model_plans["yolov8n-pose"]
    m = ivb.PlanModel(p, device=0, max_batch=32)
    n = m.inputNumel()
    x = torch.empty(32 * n, dtype=torch.float32, pin_memory=True)
    x.numpy()[:] = np.random.default_rng(41).random(32 * n, dtype=np.float32)
    y = torch.empty(32 * m.outputNumel(0), dtype=torch.float32, pin_memory=True)
    ref = None
    for _ in range(13):
        m.infer_f32(x.numpy(), 32, [y.numpy()])
        if ref is None:
            ref = y.numpy().copy()
        else:
            assert np.array_equal(y.numpy(), ref)
    m.close()


@pytest.mark.parametrize("batch", [1, 3, 40])
def test_infer_f32_pinned_and_pageable_agree(model_plans, batch):
    """ClBackend::infer from page-locked buffers (copied directly, half the
    batch cast on the host) and from pageable ones (every image cast on the
    host into pinned chunks, results staged back through pinned chunks) give
    the same bits, and so does a pinned input with a pageable output."""
    import torch
    p = model_plans["yolov8n-pose"]
    m = ivb.PlanModel(p, max_batch=batch)
    n, no = m.inputNumel(), m.outputNumel(0)
    x = np.random.default_rng(41).random(batch * n, dtype=np.float32)
    xp = torch.from_numpy(x).pin_memory()
    yp = torch.empty(batch * no, dtype=torch.float32).pin_memory()
    m.infer_f32(xp.numpy(), batch, [yp.numpy()])
    y_page = m.infer_f32(x, batch)[0]
    assert np.array_equal(y_page, yp.numpy())
    y_mixed = np.empty(batch * no, dtype=np.float32)
    m.infer_f32(xp.numpy(), batch, [y_mixed])
    assert np.array_equal(y_mixed, y_page)
    m.close()
