"""Device preprocessing (ivc_set_input_bgr_u8 / ivc_infer_bgr_u8) against the
restatement of the reference's Preprocessor (oracle/preprocess.py, itself
pinned to OpenCV's output by tests/test_preprocess_pinned.py) followed by the
reference's truncating f32 -> f16 cast: the network input must be identical
bit for bit, and so must everything computed from it."""
import os

import numpy as np
import pytest

import infvino_b200 as ivb
from infvino_b200 import plangen
from oracle import ivref, preprocess

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(__file__), "golden", "preprocess_vectors.npz")


def identity_plan(out_dir, h, w):
    """A plan whose input is [1, 3, h, w] and whose output is that input plus
    zero (exact), so the input can be read back."""
    pw = plangen.PlanWriter(5)
    x = pw.input("x", [1, 3, h, w])
    z = pw.init("zero", np.zeros((1, 3, h, w), dtype=np.float16))
    pw.output(pw.add(x, z, name="y"))
    return pw.save(out_dir)


def expected_input(frames, in_h, in_w, **cfg):
    blobs, lbs = [], []
    for f in frames:
        blob, info = preprocess.preprocess(f, in_h, in_w, **cfg)
        blobs.append(ivref.f32_to_f16_trunc(blob).ravel())
        lbs.append(info)
    return np.concatenate(blobs), np.array(lbs, dtype=np.float32)


def test_preprocess_golden_cases(plan_dir):
    g = np.load(GOLD)
    names = sorted({k.split("/")[0] for k in g.files})
    for name in names:
        ih, iw, lb, rgb, norm = (int(v) for v in g[f"{name}/params"])
        cfg = dict(letterbox=bool(lb), to_rgb=bool(rgb), normalize=bool(norm), mean=tuple(g[f"{name}/mean"]),
                   std=tuple(g[f"{name}/std"]))
        m = ivb.PlanModel(identity_plan(os.path.join(plan_dir, f"pp_{ih}x{iw}"), ih, iw), max_batch=2)
        img = g[f"{name}/image"]
        frames = np.stack([img, img[::-1].copy()])  # two different frames of one size
        got_lb = m.setInputBgr(frames, **cfg)
        want, want_lb = expected_input(frames, ih, iw, **cfg)
        assert np.array_equal(m.readTensor("x", 2), want), name
        # the first frame against the reference's own blob from the fixture
        assert np.array_equal(m.readTensor("x", 1), ivref.f32_to_f16_trunc(g[f"{name}/blob"]).ravel()), name
        assert np.array_equal(got_lb, want_lb), (name, got_lb, want_lb)
        m.close()


@pytest.mark.parametrize("h,w", [(720, 1280), (480, 640), (1080, 1920), (640, 640), (333, 517)])
def test_preprocess_network_input(plan_dir, model_plans, h, w):
    """Camera-sized frames into YOLOv8n-pose's 640x640 input."""
    m = ivb.PlanModel(model_plans["yolov8n-pose"], max_batch=3)
    frames = np.random.default_rng(h * 7 + w).integers(0, 256, (3, h, w, 3), dtype=np.uint8)
    lb = m.setInputBgr(frames)
    want, want_lb = expected_input(frames, 640, 640)
    assert np.array_equal(m.readTensor("images", 3), want)
    assert np.array_equal(lb, want_lb)
    m.close()


def test_preprocess_mobilenet_mean_std(model_plans):
    """Plain resize with ImageNet mean / std (a classifier's preprocessing)."""
    m = ivb.PlanModel(model_plans["mobilenetv3-small"], max_batch=2)
    frames = np.random.default_rng(3).integers(0, 256, (2, 375, 500, 3), dtype=np.uint8)
    cfg = dict(letterbox=False, mean=(0.485, 0.456, 0.406), std=(0.229, 0.224, 0.225))
    m.setInputBgr(frames, **cfg)
    want, _ = expected_input(frames, 224, 224, **cfg)
    assert np.array_equal(m.readTensor(m.inputName(), 2), want)
    m.close()


@pytest.mark.parametrize("batch,pinned", [(3, False), (40, False), (40, True)])
def test_infer_bgr_equals_device_path(plan_dir, batch, pinned):
    """End to end from frames (chunked for large batches, pinned or pageable
    frames) equals preprocessing on the device then one run of the batch, and
    the device decode afterwards sees every image."""
    import torch
    p = plangen.yolov8n_pose(os.path.join(plan_dir, "y8_320_pp"), imgsz=320, cls_gain=100.0, cls_shift=-3.0)
    m = ivb.PlanModel(p, max_batch=batch)
    frames = np.random.default_rng(batch).integers(0, 256, (batch, 240, 320, 3), dtype=np.uint8)
    lb = m.setInputBgr(frames)
    m.run(batch)
    ref = ivb.f16_to_f32(m.readOutput(0, batch))
    ref_dets = m.decodePose(batch, letterbox=lb)
    fr = torch.from_numpy(frames).pin_memory().numpy() if pinned else frames
    outs, lb2 = m.inferBgr(fr)
    assert np.array_equal(outs[0], ref)
    assert np.array_equal(lb2, lb)
    dets = m.decodePose(batch, letterbox=lb2)
    for b in range(batch):
        assert np.array_equal(dets[b], ref_dets[b]), b
    m.close()


def test_preprocess_frames_on_device(model_plans):
    import torch
    m = ivb.PlanModel(model_plans["yolov8n-pose"], max_batch=2)
    frames = np.random.default_rng(9).integers(0, 256, (2, 360, 640, 3), dtype=np.uint8)
    m.setInputBgr(frames)
    host = m.readTensor("images", 2)
    dev = torch.from_numpy(frames).cuda()
    m.setInputBgr(dev.data_ptr(), device_shape=(2, 360, 640))
    assert np.array_equal(m.readTensor("images", 2), host)
    m.close()
