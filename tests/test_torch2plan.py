"""The plan producer (infvino_b200/torch2plan.py): PyTorch models converted to
the reference's plan format run through the CPU oracle within fp16 storage
precision of PyTorch's own fp32 forward, and (on a GPU) through the executor
within the usual parity bar of the oracle.

Models: torchvision's MobileNetV3-small (random init, BN statistics
randomised) and a YOLOv8-style network written here with the blocks the pose
models use (Conv-BN-SiLU, C2f with chunk + concat + residual bottlenecks,
SPPF with chained max pools, nearest upsampling, a neck concat)."""
import os

import numpy as np
import pytest
import torch
import torch.nn as nn

import infvino_b200 as ivb
from infvino_b200 import torch2plan
from oracle import ivref


class ConvBnSiLU(nn.Module):
    def __init__(self, c1, c2, k=1, s=1):
        super().__init__()
        self.conv = nn.Conv2d(c1, c2, k, s, k // 2, bias=False)
        self.bn = nn.BatchNorm2d(c2)
        self.act = nn.SiLU()

    def forward(self, x):
        return self.act(self.bn(self.conv(x)))


class Bottleneck(nn.Module):
    def __init__(self, c, shortcut=True):
        super().__init__()
        self.cv1, self.cv2 = ConvBnSiLU(c, c, 3), ConvBnSiLU(c, c, 3)
        self.add = shortcut

    def forward(self, x):
        y = self.cv2(self.cv1(x))
        return x + y if self.add else y


class C2f(nn.Module):
    def __init__(self, c1, c2, n=1, shortcut=True):
        super().__init__()
        self.c = c2 // 2
        self.cv1 = ConvBnSiLU(c1, 2 * self.c, 1)
        self.cv2 = ConvBnSiLU((2 + n) * self.c, c2, 1)
        self.m = nn.ModuleList(Bottleneck(self.c, shortcut) for _ in range(n))

    def forward(self, x):
        a, b = self.cv1(x).chunk(2, 1)  # (tuple unpacking: torch.fx traces it)
        y = [a, b]
        for m in self.m:
            y.append(m(y[-1]))
        return self.cv2(torch.cat(y, 1))


class SPPF(nn.Module):
    def __init__(self, c1, c2):
        super().__init__()
        self.cv1 = ConvBnSiLU(c1, c1 // 2, 1)
        self.cv2 = ConvBnSiLU(c1 // 2 * 4, c2, 1)
        self.m = nn.MaxPool2d(5, 1, 2)

    def forward(self, x):
        x = self.cv1(x)
        y1 = self.m(x)
        y2 = self.m(y1)
        return self.cv2(torch.cat((x, y1, y2, self.m(y2)), 1))


class TinyYolo(nn.Module):
    """Backbone to stride 16, SPPF, an upsampling neck and a 1x1 head."""

    def __init__(self):
        super().__init__()
        self.b0 = ConvBnSiLU(3, 16, 3, 2)
        self.b1 = ConvBnSiLU(16, 32, 3, 2)
        self.c2 = C2f(32, 32, 1)
        self.b3 = ConvBnSiLU(32, 64, 3, 2)
        self.c4 = C2f(64, 64, 2)
        self.b5 = ConvBnSiLU(64, 64, 3, 2)
        self.sppf = SPPF(64, 64)
        self.up = nn.Upsample(scale_factor=2, mode="nearest")
        self.c6 = C2f(128, 32, 1, shortcut=False)
        self.head = nn.Conv2d(32, 21, 1)

    def forward(self, x):
        p3 = self.c4(self.b3(self.c2(self.b1(self.b0(x)))))
        p4 = self.sppf(self.b5(p3))
        y = self.c6(torch.cat((self.up(p4), p3), 1))
        return torch.sigmoid(self.head(y))


def _randomise_bn(m, seed):
    g = torch.Generator().manual_seed(seed)
    for mod in m.modules():
        if isinstance(mod, nn.BatchNorm2d):
            c = mod.num_features
            mod.running_mean.copy_(torch.rand(c, generator=g) * 0.2 - 0.1)
            mod.running_var.copy_(torch.rand(c, generator=g) + 0.5)
            mod.weight.data.copy_(torch.rand(c, generator=g) + 0.5)
            mod.bias.data.copy_(torch.rand(c, generator=g) * 0.2 - 0.1)
    return m.eval()


def _models():
    import torchvision
    torch.manual_seed(0)
    mb = _randomise_bn(torchvision.models.mobilenet_v3_small(weights=None), 1)
    torch.manual_seed(1)
    yo = _randomise_bn(TinyYolo(), 2)
    return {"mobilenet_v3_small": (mb, (1, 3, 224, 224)), "tiny_yolo": (yo, (1, 3, 128, 160))}


def _torch_out(model, x, shape):
    with torch.no_grad():
        return model(torch.from_numpy(x.reshape(shape))).double().numpy().ravel()


@pytest.mark.parametrize("name", ["mobilenet_v3_small", "tiny_yolo"])
def test_converted_plan_matches_torch_on_the_oracle(tmp_path, name):
    model, shape = _models()[name]
    plan = torch2plan.convert(model, shape, str(tmp_path / name))
    text = open(plan).read()
    # the routing of scripts/onnx2plan.py: Conv+BN+SiLU folded into the convs
    assert "BatchNorm" not in text and "ew_unary" not in text.split("conv")[0]
    o = ivref.OraclePlan(plan)
    x = np.random.default_rng(5).random(int(np.prod(shape)), dtype=np.float32)
    o.run(x, 1)
    got = ivref.f16_to_f32(o.read_f16(o.output_names()[0])).astype(np.float64)
    ref = _torch_out(model, x, shape)
    rel = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    # fp16 storage of every activation against PyTorch's fp32 (the reference
    # checks its own plans against ONNX Runtime FP32 at mean_rel < 2e-2,
    # scripts/numerical_check.py:62-78)
    assert rel < 5e-3, rel
    if name == "mobilenet_v3_small":
        assert got.argmax() == ref.argmax()


def test_converter_routes_ops_like_onnx2plan(tmp_path):
    model, shape = _models()["tiny_yolo"]
    text = open(torch2plan.convert(model, shape, str(tmp_path / "ty"))).read().splitlines()
    ops = [ln.split()[1] for ln in text if ln.startswith("node ")]
    assert ops.count("conv3x3") >= 9 and "conv1x1" in ops and "copy_c" in ops and "concat4" in ops
    assert "maxpool" in ops and "resize_nn" in ops and "ew_binary" in ops
    s2 = [ln for ln in text if ln.startswith("node conv3x3") and "stride=2" in ln]
    assert s2 and all(ln.endswith("cfg=64,8,1,32,8,2") or "cfg=64,8,1,32,8,2" in ln for ln in s2)
    assert any("act=1" in ln for ln in text if ln.startswith("node conv3x3"))
    # the final sigmoid follows a 1x1 conv with a bias: folded as act=5
    assert any(ln.startswith("node conv1x1") and "act=5" in ln for ln in text)


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["mobilenet_v3_small", "tiny_yolo"])
def test_converted_plan_on_the_executor(tmp_path, name):
    model, shape = _models()[name]
    plan = torch2plan.convert(model, shape, str(tmp_path / name))
    o = ivref.OraclePlan(plan)
    x = np.random.default_rng(6).random(2 * int(np.prod(shape)), dtype=np.float32)
    x16 = ivref.f32_to_f16_trunc(x)
    o.run_f16(x16, 2)
    m = ivb.PlanModel(plan, max_batch=2)
    m.setInput(x16, 2)
    m.run(2)
    g = ivref.f16_to_f32(m.readOutput(0, 2)).astype(np.float64)
    r = ivref.f16_to_f32(o.read_f16(m.outputName(0))).astype(np.float64)
    assert np.abs(g - r).max() <= 2e-2 and np.linalg.norm(g - r) <= 2e-3 * np.linalg.norm(r)
    m.close()
