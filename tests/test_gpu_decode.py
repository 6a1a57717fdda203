"""Device pose decode + NMS (ivc_decode_pose) against the oracle's restatement
of the reference's PoseDecoder::decode, nmsPerClass and nms (oracle/decode.py)
on the same network outputs: the same detections in the same order, with the
same anchor, score, box and keypoint values bit for bit."""
import os

import numpy as np
import pytest

import infvino_b200 as ivb
from infvino_b200 import plangen
from oracle import decode


def check_against_oracle(m, y, batch, conf, iou, max_det, letterbox):
    got = m.decodePose(batch, conf=conf, iou=iou, max_det=max_det, letterbox=letterbox)
    total = 0
    for b in range(batch):
        scale, pl, pt = (1.0, 0.0, 0.0) if letterbox is None else (float(v) for v in letterbox[b])
        ref = decode.pose_decode(y[b], conf=conf, iou=iou, max_det=max_det, scale=scale, pad=(pl, pt))
        assert got[b].shape == (len(ref), 6 + 2 * 17), (b, got[b].shape, len(ref))
        for k, (a, s, box, kp) in enumerate(ref):
            row = got[b][k]
            assert int(row[0]) == a and row[1] == np.float32(s), (b, k, row[:2], a, s)
            assert np.array_equal(row[2:6], np.asarray(box, dtype=np.float32)), (b, k)
            assert np.array_equal(row[6:].reshape(17, 2), np.asarray(kp, dtype=np.float32)), (b, k)
        total += len(ref)
    return total


@pytest.mark.gpu
def test_device_pose_decode_peaked(plan_dir):
    """A class head scaled to give a few dozen detections per image (as with
    trained weights), three images, per-image letterboxes."""
    p = plangen.yolov8n_pose(os.path.join(plan_dir, "y8_peaked_dec"), cls_gain=100.0, cls_shift=-3.0)
    m = ivb.PlanModel(p, max_batch=3)
    x = np.random.default_rng(61).random(3 * m.inputNumel(), dtype=np.float32)
    y = m.infer_f32(x, 3)[0].reshape(3, 56, -1)
    lb = np.array([[1.0, 0.0, 0.0], [0.5, 3.0, 7.0], [0.8125, 0.0, 80.0]], dtype=np.float32)
    n = check_against_oracle(m, y, 3, 0.25, 0.7, 300, lb)
    assert n >= 30, n
    assert check_against_oracle(m, y, 3, 0.25, 0.7, 300, None) == n
    m.close()


@pytest.mark.gpu
def test_device_pose_decode_every_anchor_a_candidate(plan_dir):
    """Random-init class scores are all ~0.5: every anchor is a candidate, many
    scores tie in fp16 (equal scores in the order of the reference's final
    std::sort, which decides the max_det cut among them), and the cut is
    reached; twice in a row, and with a smaller cut."""
    p = plangen.yolov8n_pose(os.path.join(plan_dir, "y8_320_dec"), imgsz=320)
    m = ivb.PlanModel(p, max_batch=2)
    x = np.random.default_rng(62).random(2 * m.inputNumel(), dtype=np.float32)
    y = m.infer_f32(x, 2)[0].reshape(2, 56, -1)
    assert (y[:, 4] >= 0.25).all()
    for _ in range(2):
        assert check_against_oracle(m, y, 2, 0.25, 0.7, 300, None) == 600
    assert check_against_oracle(m, y, 2, 0.25, 0.5, 40, None) == 80
    m.close()


def identity_plan(out_dir, A):
    """A plan whose output is its input ([1, 56, A] plus a zero initializer,
    exact in fp16): the decoder's input can be set value by value."""
    pw = plangen.PlanWriter(5)
    x = pw.input("x", [1, 56, A])
    z = pw.init("zero", np.zeros((1, 56, A), dtype=np.float16))
    pw.output(pw.add(x, z, name="y"))
    return pw.save(out_dir)


def adversarial_outputs(rng, batch, A):
    """Pose outputs built to stress the decoder: scores from a handful of fp16
    values (exact ties everywhere, one of them exactly `conf` and one just
    below it), clusters of identical boxes, boxes of zero and negative size,
    small random shifts that put many IoUs near the threshold, and random
    keypoints."""
    y = np.zeros((batch, 56, A), dtype=np.float32)
    levels = np.array([0.25, 0.2499, 0.5, 0.75, 0.875, 1.0, 0.0], dtype=np.float16).astype(np.float32)
    for b in range(batch):
        y[b, 4] = rng.choice(levels, A)
        centers = rng.uniform(0, 640, (A // 16, 2))
        k = rng.integers(0, len(centers), A)
        y[b, 0] = centers[k, 0] + rng.choice([0.0, 0.0, 1.5, -3.0, 8.0], A)
        y[b, 1] = centers[k, 1] + rng.choice([0.0, 2.0, -4.0], A)
        y[b, 2] = rng.choice([40.0, 48.0, 0.0, -5.0, 64.0, 20.0], A)
        y[b, 3] = rng.choice([40.0, 32.0, 56.0, 0.0], A)
        y[b, 5:] = rng.uniform(-50, 700, (51, A))
    return y.astype(np.float16)


@pytest.mark.gpu
@pytest.mark.parametrize("conf,iou,max_det", [(0.25, 0.7, 300), (0.5, 0.45, 50), (0.0, 0.0, 2048)])
def test_device_pose_decode_adversarial(plan_dir, conf, iou, max_det):
    A, B = 2048, 3
    p = identity_plan(os.path.join(plan_dir, "pose_identity"), A)
    m = ivb.PlanModel(p, max_batch=B)
    y16 = adversarial_outputs(np.random.default_rng(63), B, A)
    m.setInput(y16.view(np.uint16).ravel(), B)
    m.run(B)
    y = y16.astype(np.float32)
    assert np.array_equal(ivb.f16_to_f32(m.readOutput(0, B)).reshape(B, 56, A), y)
    lb = np.array([[0.75, 16.0, 0.0], [1.0, 0.0, 0.0], [0.5, 0.0, 140.0]], dtype=np.float32)
    n = check_against_oracle(m, y, B, conf, iou, max_det, lb)
    assert n > 0
    m.close()


@pytest.mark.gpu
@pytest.mark.parametrize("pinned", [False, True])
def test_device_pose_decode_after_chunked_infer(plan_dir, pinned):
    """ClBackend::infer on a large batch runs the network chunk by chunk; the
    device decode afterwards still sees every image of the batch (the same
    detections as after one device-resident run of the whole batch)."""
    import torch
    B = 40
    p = plangen.yolov8n_pose(os.path.join(plan_dir, "y8_320_chunk"), imgsz=320, cls_gain=100.0, cls_shift=-3.0)
    m = ivb.PlanModel(p, max_batch=B)
    x = np.random.default_rng(64).random(B * m.inputNumel(), dtype=np.float32)
    m.setInput(ivb.f32_to_f16(x), B)
    m.run(B)
    ref = m.decodePose(B)
    xs = torch.from_numpy(x).pin_memory().numpy() if pinned else x
    y = m.infer_f32(xs, B)[0].reshape(B, 56, -1)
    got = m.decodePose(B)
    assert sum(len(d) for d in ref) > 0
    for b in range(B):
        assert np.array_equal(got[b], ref[b]), b
    assert check_against_oracle(m, y, B, 0.25, 0.7, 300, None) == sum(len(d) for d in ref)
    m.close()
