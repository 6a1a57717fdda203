"""Synthetic execution-plan emitter (the `model.plan` + fp16 `init_*.bin` format).

The reference turns an ONNX graph into a text plan with `scripts/onnx2plan.py`
(grammar: `include/infvino/PlanModel.hpp:6-12`; op mapping:
`scripts/onnx2plan.py:169-424`).  No ONNX models, `onnx` or `ultralytics` exist
on this machine, so this module writes the same plan text directly from an
architecture description, with seeded random-init weights:

* conv weights He-normal (std = sqrt(2 / fan_in)) stored as fp16, biases
  N(0, 0.01) - batch-norm is assumed folded into the conv, as the exporter does;
* op lines follow onnx2plan exactly: `conv3x3 x,w,b,- out stride= pad= Hout=
  Wout= act= [cfg=]`, `conv1x1 w,x,b,- out act=`, `conv_general x,w,b out K= S=
  P= G= Hout= Wout= act=`, and the small ops with the attribute names and
  values onnx2plan computes (`bdims` broadcast strides included,
  `scripts/onnx2plan.py:244-277`);
* activation codes are canonical: 1=SiLU 2=ReLU 3=HardSwish 4=HardSigmoid
  5=Sigmoid on convs, and `ew_unary` uses 0=sigmoid (`onnx2plan.py:130-138,
  231-243`).

Models: YOLOv8n-pose, MobileNetV3-small, YOLO11n-pose (architecture from
their public descriptions), plus single-op plans for the kernel sweeps.
"""
from __future__ import annotations

import math
import os
from typing import Dict, List, Optional, Sequence

import numpy as np

FP16 = np.float16


class PlanWriter:
    """Accumulates plan lines in emission order and the fp16 initializers."""

    def __init__(self, seed: int = 1234):
        self.lines: List[str] = []
        self.inits: Dict[str, np.ndarray] = {}
        self.shapes: Dict[str, List[int]] = {}
        self.declared = set()
        self.rng = np.random.default_rng(seed)
        self._uid = 0

    # ---- naming ----
    def fresh(self, stem: str) -> str:
        self._uid += 1
        return f"{stem}_{self._uid}"

    # ---- declarations (same line syntax as onnx2plan) ----
    def input(self, name: str, dims: Sequence[int]) -> str:
        self.declared.add(name)
        self.shapes[name] = list(dims)
        self.lines.append("input {} {}".format(name, " ".join(str(d) for d in dims)))
        return name

    def init(self, name: str, arr: np.ndarray) -> str:
        arr = np.asarray(arr).astype(FP16)
        self.inits[name] = arr
        self.shapes[name] = list(arr.shape)
        self.declared.add(name)
        base = "init_{}.bin".format(name.replace("/", "_"))
        self.lines.append("init {} {} {}".format(name, base, " ".join(str(d) for d in arr.shape)).rstrip())
        return name

    def tensor(self, name: str, dims: Sequence[int]) -> str:
        if name not in self.declared:
            self.declared.add(name)
            self.shapes[name] = list(dims)
            self.lines.append("tensor {} {}".format(name, " ".join(str(d) for d in dims)))
        return name

    def node(self, kind: str, ins: Sequence[str], outs: Sequence[str], **attrs) -> None:
        a = " ".join(f"{k}={v}" for k, v in attrs.items() if v is not None)
        self.lines.append("node {} {} {} {}".format(kind, ",".join(ins) or "-", ",".join(outs), a))

    def output(self, name: str) -> None:
        self.lines.append(f"output {name}")

    def save(self, out_dir: str, plan_name: str = "model.plan") -> str:
        os.makedirs(out_dir, exist_ok=True)
        for name, arr in self.inits.items():
            arr.astype("<f2").tofile(os.path.join(out_dir, "init_{}.bin".format(name.replace("/", "_"))))
        path = os.path.join(out_dir, plan_name)
        with open(path, "w") as f:
            f.write("\n".join(self.lines) + "\n")
        return path

    # ---- random init ----
    def he_weight(self, name: str, shape: Sequence[int], fan_in: int, gain: float = 1.0) -> str:
        std = gain * math.sqrt(2.0 / max(1, fan_in))
        return self.init(name, self.rng.normal(0.0, std, size=tuple(shape)))

    def bias(self, name: str, n: int) -> str:
        return self.init(name, self.rng.normal(0.0, 0.01, size=(n,)))

    # ---- layer helpers (emit exactly what onnx2plan would) ----
    def conv(self, x: str, cout: int, k: int, s: int = 1, act: int = 0, groups: int = 1,
             bias: bool = True, name: Optional[str] = None, gain: float = 1.0) -> str:
        """Conv2d (+ folded BN) + optional fused activation; pad = k // 2."""
        cin, h, w = self.shapes[x][1], self.shapes[x][2], self.shapes[x][3]
        p = k // 2
        ho = (h + 2 * p - k) // s + 1
        wo = (w + 2 * p - k) // s + 1
        stem = name or self.fresh("conv")
        wn = self.he_weight(stem + ".weight", (cout, cin // groups, k, k), (cin // groups) * k * k, gain)
        bn = self.bias(stem + ".bias", cout) if bias else None
        out = self.tensor(stem + ".out", [1, cout, ho, wo])
        if k == 3 and groups == 1 and s in (1, 2):
            # onnx2plan only fuses SiLU / HardSwish into conv3x3 (ACT_CODE_CONV + conv_act)
            assert act in (0, 1, 3), act
            cfg = None if s == 1 else "64,8,1,32,8,2"
            self.node("conv3x3", [x, wn, bn or "-", "-"], [out], stride=s, pad=p, Hout=ho, Wout=wo,
                      act=(act or None), cfg=cfg)
        elif k == 1 and groups == 1:
            self.node("conv1x1", [wn, x, bn or "-", "-"], [out], act=(act or None))
        else:
            self.node("conv_general", [x, wn, bn or "-"], [out], K=k, S=s, P=p, G=groups, Hout=ho,
                      Wout=wo, act=(act or None))
        return out

    def gemm(self, x: str, n: int, act: int = 0, name: Optional[str] = None) -> str:
        """ONNX Gemm(transB=1) -> conv1x1 with a 2-D weight (onnx2plan.py:406-422)."""
        k = self.shapes[x][-1]
        stem = name or self.fresh("fc")
        wn = self.he_weight(stem + ".weight", (n, k), k)
        bn = self.bias(stem + ".bias", n)
        out = self.tensor(stem + ".out", [self.shapes[x][0], n])
        self.node("conv1x1", [wn, x, bn, "-"], [out], act=(act or None))
        return out

    def add(self, a: str, b: str, op: int = 0, name: Optional[str] = None) -> str:
        """Same-shape or broadcast ew_binary with onnx2plan's bdims / b_scalar rules."""
        oshape = self._bcast_shape(self.shapes[a], self.shapes[b])
        out = self.tensor(name or self.fresh("ew"), oshape)
        asha, bsha = self.shapes[a], self.shapes[b]
        bdims = None
        b_scalar = 0
        if list(asha) != list(oshape) or (b in self.inits and list(self.inits[b].shape) != list(oshape)):
            rank = len(oshape)

            def align(s):
                return [1] * (rank - len(s)) + list(s)

            def strides(aligned):
                st = [0] * rank
                acc = 1
                for i in range(rank - 1, -1, -1):
                    st[i] = 0 if (aligned[i] == 1 and oshape[i] != 1) else acc
                    acc *= aligned[i]
                return st

            bdims = (oshape, strides(align(asha)), strides(align(bsha)))
        if b in self.inits and self.inits[b].size == 1 and list(asha) == list(oshape):
            b_scalar = 1
        n = int(np.prod(oshape))
        self.node("ew_binary", [a, b], [out], op=op, n=n, b_scalar=b_scalar,
                  bdims=(",".join(",".join(str(v) for v in g) for g in bdims) if bdims else None))
        return out

    @staticmethod
    def _bcast_shape(a: Sequence[int], b: Sequence[int]) -> List[int]:
        r = max(len(a), len(b))
        a2 = [1] * (r - len(a)) + list(a)
        b2 = [1] * (r - len(b)) + list(b)
        return [max(x, y) for x, y in zip(a2, b2)]

    def unary(self, x: str, op: int, name: Optional[str] = None) -> str:
        out = self.tensor(name or self.fresh("un"), self.shapes[x])
        self.node("ew_unary", [x], [out], op=op, n=int(np.prod(self.shapes[x])))
        return out

    def split_c(self, x: str, counts: Sequence[int]) -> List[str]:
        """ONNX Split on axis 1 -> copy_c per output (onnx2plan.py:298-312)."""
        _, c, h, w = self.shapes[x]
        outs, c0 = [], 0
        for cnt in counts:
            o = self.tensor(self.fresh("split"), [1, cnt, h, w])
            self.node("copy_c", [x], [o], HW=h * w, c0=c0, cnt=cnt, dst_off=0)
            outs.append(o)
            c0 += cnt
        return outs

    def concat(self, xs: Sequence[str], axis: int, name: Optional[str] = None) -> str:
        shapes = [self.shapes[x] for x in xs]
        rank = len(shapes[0])
        if axis < 0:
            axis += rank
        oshape = list(shapes[0])
        oshape[axis] = sum(s[axis] for s in shapes)
        outer = int(np.prod(oshape[:axis]))
        inner = int(np.prod(oshape[axis + 1:]))
        dims = [s[axis] for s in shapes]
        ins = list(xs)
        assert len(ins) <= 4
        while len(ins) < 4:
            ins.append("-")
            dims.append(0)
        out = self.tensor(name or self.fresh("cat"), oshape)
        self.node("concat4", ins, [out], ca=dims[0], cb=dims[1], cc=dims[2], cd=dims[3],
                  outer=outer, inner=inner)
        return out

    def maxpool(self, x: str, k: int = 5, s: int = 1, p: int = 2) -> str:
        _, c, h, w = self.shapes[x]
        ho, wo = (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1
        out = self.tensor(self.fresh("mp"), [1, c, ho, wo])
        self.node("maxpool", [x], [out], C=c, H=h, W=w, Hout=ho, Wout=wo, K=k, S=s, P=p)
        return out

    def upsample(self, x: str, s: int = 2) -> str:
        _, c, h, w = self.shapes[x]
        out = self.tensor(self.fresh("up"), [1, c, h * s, w * s])
        self.node("resize_nn", [x], [out], C=c, H=h, W=w, S=s)
        return out

    def reshape(self, x: str, dims: Sequence[int]) -> str:
        assert int(np.prod(dims)) == int(np.prod(self.shapes[x]))
        out = self.tensor(self.fresh("rs"), dims)
        self.node("reshape", [x], [out])
        return out

    def slice_axis(self, x: str, axis: int, start: int, length: int) -> str:
        xs = self.shapes[x]
        outer = int(np.prod(xs[:axis]))
        inner = int(np.prod(xs[axis + 1:]))
        os_ = list(xs)
        os_[axis] = length
        out = self.tensor(self.fresh("sl"), os_)
        self.node("slice_axis", [x], [out], outer=outer, axdim=xs[axis], inner=inner, start=start,
                  len=length)
        return out

    def permute(self, x: str, perm: Sequence[int]) -> str:
        xs = self.shapes[x]
        assert perm[0] == 0 and list(perm) in ([0, 2, 1, 3], [0, 1, 3, 2])
        mode = 0 if list(perm) == [0, 2, 1, 3] else 1
        os_ = [xs[i] for i in perm]
        out = self.tensor(self.fresh("perm"), os_)
        self.node("permute_0213", [x], [out], D1=xs[1], D2=xs[2], I=int(np.prod(xs[3:])), mode=mode)
        return out

    def softmax(self, x: str, axis: int) -> str:
        xs = self.shapes[x]
        outer = int(np.prod(xs[:axis])) if axis > 0 else 1
        inner = int(np.prod(xs[axis + 1:])) if axis + 1 < len(xs) else 1
        out = self.tensor(self.fresh("sm"), xs)
        self.node("softmax_axis", [x], [out], outer=outer, axdim=xs[axis], inner=inner)
        return out

    def gap(self, x: str) -> str:
        _, c, h, w = self.shapes[x]
        out = self.tensor(self.fresh("gap"), [1, c, 1, 1])
        self.node("gap", [x], [out], C=c, HW=h * w)
        return out

    def bmm(self, a: str, b: str) -> str:
        asha, bsha = self.shapes[a], self.shapes[b]
        out = self.tensor(self.fresh("bmm"), [asha[0], asha[1], asha[2], bsha[3]])
        self.node("bmm", [a, b], [out], B0=asha[0], B1=asha[1], M=asha[2], K=asha[3], N=bsha[3])
        return out


# ---------------------------------------------------------------------------
# YOLOv8n-pose (width 0.25, depth 0.33): backbone / PAN-FPN neck / pose head
# ---------------------------------------------------------------------------

def _c2f(pw: PlanWriter, x: str, c2: int, n: int, shortcut: bool, tag: str) -> str:
    c = c2 // 2
    y = pw.conv(x, 2 * c, 1, act=1, name=f"{tag}.cv1")
    a, b = pw.split_c(y, [c, c])
    ys = [a, b]
    for i in range(n):
        t = pw.conv(ys[-1], c, 3, act=1, name=f"{tag}.m{i}.cv1")
        t = pw.conv(t, c, 3, act=1, name=f"{tag}.m{i}.cv2")
        if shortcut:
            t = pw.add(ys[-1], t, 0, name=f"{tag}.m{i}.add")
        ys.append(t)
    cat = pw.concat(ys, 1, name=f"{tag}.cat")
    return pw.conv(cat, c2, 1, act=1, name=f"{tag}.cv2")


def _sppf(pw: PlanWriter, x: str, c2: int, tag: str) -> str:
    c1 = pw.shapes[x][1]
    y0 = pw.conv(x, c1 // 2, 1, act=1, name=f"{tag}.cv1")
    y1 = pw.maxpool(y0)
    y2 = pw.maxpool(y1)
    y3 = pw.maxpool(y2)
    cat = pw.concat([y0, y1, y2, y3], 1, name=f"{tag}.cat")
    return pw.conv(cat, c2, 1, act=1, name=f"{tag}.cv2")


def _anchors(levels: Sequence[int], strides: Sequence[int], offset: float = 0.5):
    pts, sts = [], []
    for hw, s in zip(levels, strides):
        sy, sx = np.meshgrid(np.arange(hw) + offset, np.arange(hw) + offset, indexing="ij")
        pts.append(np.stack([sx.ravel(), sy.ravel()], 0))
        sts.append(np.full((hw * hw,), s, dtype=np.float32))
    return np.concatenate(pts, 1).astype(np.float32), np.concatenate(sts, 0)


def _pose_head(pw: PlanWriter, feats: Sequence[str], c2: int, c3: int, c4: int, tag: str,
               dw_cls: bool = False, cls_gain: float = 1.0, cls_shift: float = 0.0) -> str:
    """Pose head + in-graph decode (DFL, dist2bbox, keypoint decode) -> [1, 56, A]."""
    nk, reg = 51, 16
    hws = [pw.shapes[f][2] for f in feats]
    A = sum(h * h for h in hws)
    # keypoint branch first (Pose.forward evaluates cv4 before Detect.forward)
    kv = []
    for i, f in enumerate(feats):
        t = pw.conv(f, c4, 3, act=1, name=f"{tag}.cv4.{i}.0")
        t = pw.conv(t, c4, 3, act=1, name=f"{tag}.cv4.{i}.1")
        t = pw.conv(t, nk, 1, act=0, name=f"{tag}.cv4.{i}.2")
        kv.append(pw.reshape(t, [1, nk, hws[i] * hws[i]]))
    kpt = pw.concat(kv, 2, name=f"{tag}.kpt_cat")
    bv, cv = [], []
    for i, f in enumerate(feats):
        t = pw.conv(f, c2, 3, act=1, name=f"{tag}.cv2.{i}.0")
        t = pw.conv(t, c2, 3, act=1, name=f"{tag}.cv2.{i}.1")
        t = pw.conv(t, 4 * reg, 1, act=0, name=f"{tag}.cv2.{i}.2")
        bv.append(pw.reshape(t, [1, 4 * reg, hws[i] * hws[i]]))
        if dw_cls:
            # YOLO11 class branch: (DW 3x3 + 1x1) x2, then 1x1 -> nc
            cin = pw.shapes[f][1]
            u = pw.conv(f, cin, 3, act=1, groups=cin, name=f"{tag}.cv3.{i}.0.0")
            u = pw.conv(u, c3, 1, act=1, name=f"{tag}.cv3.{i}.0.1")
            u = pw.conv(u, c3, 3, act=1, groups=c3, name=f"{tag}.cv3.{i}.1.0")
            u = pw.conv(u, c3, 1, act=1, name=f"{tag}.cv3.{i}.1.1")
        else:
            u = pw.conv(f, c3, 3, act=1, name=f"{tag}.cv3.{i}.0")
            u = pw.conv(u, c3, 3, act=1, name=f"{tag}.cv3.{i}.1")
        u = pw.conv(u, 1, 1, act=0, name=f"{tag}.cv3.{i}.2", gain=cls_gain)
        if cls_shift:
            bname = f"{tag}.cv3.{i}.2.bias"
            pw.inits[bname] = (pw.inits[bname].astype(np.float32) + cls_shift).astype(FP16)
        cv.append(pw.reshape(u, [1, 1, hws[i] * hws[i]]))
    box = pw.concat(bv, 2, name=f"{tag}.box_cat")
    cls = pw.concat(cv, 2, name=f"{tag}.cls_cat")
    # DFL: view [1,4,16,A] -> transpose(2,1) -> softmax(1) -> 1x1 conv 16->1 (weights 0..15)
    d = pw.reshape(box, [1, 4, reg, A])
    d = pw.permute(d, [0, 2, 1, 3])
    d = pw.softmax(d, 1)
    dflw = pw.init(f"{tag}.dfl.conv.weight", np.arange(reg, dtype=np.float32).reshape(1, reg, 1, 1))
    dout = pw.tensor(pw.fresh("dfl"), [1, 1, 4, A])
    pw.node("conv1x1", [dflw, d, "-", "-"], [dout])
    dist = pw.reshape(dout, [1, 4, A])
    strides = [640 // h for h in hws]
    anc, st = _anchors(hws, strides)
    anchors = pw.init(f"{tag}.anchors", anc.reshape(1, 2, A))
    strides_t = pw.init(f"{tag}.strides", st.reshape(1, A))
    lt = pw.slice_axis(dist, 1, 0, 2)
    rb = pw.slice_axis(dist, 1, 2, 2)
    x1y1 = pw.add(anchors, lt, 1)
    x2y2 = pw.add(anchors, rb, 0)
    cxy = pw.add(x1y1, x2y2, 0)
    two = pw.init(f"{tag}.const_two", np.array(2.0, dtype=np.float32))
    cxy = pw.add(cxy, two, 3)
    wh = pw.add(x2y2, x1y1, 1)
    dbox = pw.concat([cxy, wh], 1)
    dbox = pw.add(dbox, strides_t, 2)
    cls_s = pw.unary(cls, 0)
    # keypoints: view [1,17,3,A]; xy*2 + (anchor-0.5), * stride; vis sigmoid
    kr = pw.reshape(kpt, [1, 17, 3, A])
    kxy = pw.slice_axis(kr, 2, 0, 2)
    kxy = pw.add(kxy, pw.init(f"{tag}.const_two_k", np.array(2.0, dtype=np.float32)), 2)
    kxy = pw.add(kxy, pw.init(f"{tag}.anchors_m05", (anc - 0.5).reshape(2, A)), 0)
    kxy = pw.add(kxy, strides_t, 2)
    kvis = pw.slice_axis(kr, 2, 2, 1)
    kvis = pw.unary(kvis, 0)
    kc = pw.concat([kxy, kvis], 2)
    kf = pw.reshape(kc, [1, nk, A])
    out = pw.concat([dbox, cls_s, kf], 1, name="output0")
    return out


def yolov8n_pose(out_dir: str, seed: int = 1234, imgsz: int = 640, cls_gain: float = 1.0,
                 cls_shift: float = 0.0) -> str:
    """`cls_gain` scales the final class-conv weights and `cls_shift` offsets its
    bias (defaults: plain He-normal / N(0, 0.01)).  The NMS parity test uses a
    large gain and a negative shift so that a few anchors score high, as with
    trained weights, and the post-NMS detection set is well defined."""
    pw = PlanWriter(seed)
    x = pw.input("images", [1, 3, imgsz, imgsz])
    x = pw.conv(x, 16, 3, 2, act=1, name="model.0")
    x = pw.conv(x, 32, 3, 2, act=1, name="model.1")
    x = _c2f(pw, x, 32, 1, True, "model.2")
    x = pw.conv(x, 64, 3, 2, act=1, name="model.3")
    p3 = _c2f(pw, x, 64, 2, True, "model.4")
    x = pw.conv(p3, 128, 3, 2, act=1, name="model.5")
    p4 = _c2f(pw, x, 128, 2, True, "model.6")
    x = pw.conv(p4, 256, 3, 2, act=1, name="model.7")
    x = _c2f(pw, x, 256, 1, True, "model.8")
    p5 = _sppf(pw, x, 256, "model.9")
    x = pw.upsample(p5)
    x = pw.concat([x, p4], 1, name="model.11")
    n12 = _c2f(pw, x, 128, 1, False, "model.12")
    x = pw.upsample(n12)
    x = pw.concat([x, p3], 1, name="model.14")
    o3 = _c2f(pw, x, 64, 1, False, "model.15")
    x = pw.conv(o3, 64, 3, 2, act=1, name="model.16")
    x = pw.concat([x, n12], 1, name="model.17")
    o4 = _c2f(pw, x, 128, 1, False, "model.18")
    x = pw.conv(o4, 128, 3, 2, act=1, name="model.19")
    x = pw.concat([x, p5], 1, name="model.20")
    o5 = _c2f(pw, x, 256, 1, False, "model.21")
    out = _pose_head(pw, [o3, o4, o5], c2=64, c3=64, c4=51, tag="model.22", cls_gain=cls_gain,
                     cls_shift=cls_shift)
    pw.output(out)
    return pw.save(out_dir)


# ---------------------------------------------------------------------------
# YOLO11n-pose: C3k2 blocks, C2PSA attention at P5, depthwise-separable cls head
# ---------------------------------------------------------------------------

def _bottleneck(pw, x, c, shortcut, tag, e=1.0):
    c_ = int(c * e)
    t = pw.conv(x, c_, 3, act=1, name=f"{tag}.cv1")
    t = pw.conv(t, c, 3, act=1, name=f"{tag}.cv2")
    return pw.add(x, t, 0, name=f"{tag}.add") if shortcut else t


def _c3k(pw, x, c2, n, shortcut, tag):
    c_ = c2 // 2
    a = pw.conv(x, c_, 1, act=1, name=f"{tag}.cv1")
    b = pw.conv(x, c_, 1, act=1, name=f"{tag}.cv2")
    for i in range(n):
        a = _bottleneck(pw, a, c_, shortcut, f"{tag}.m{i}")
    cat = pw.concat([a, b], 1, name=f"{tag}.cat")
    return pw.conv(cat, c2, 1, act=1, name=f"{tag}.cv3")


def _c3k2(pw, x, c2, n, c3k, e, shortcut, tag):
    c = int(c2 * e)
    y = pw.conv(x, 2 * c, 1, act=1, name=f"{tag}.cv1")
    a, b = pw.split_c(y, [c, c])
    ys = [a, b]
    for i in range(n):
        if c3k:
            t = _c3k(pw, ys[-1], c, 2, shortcut, f"{tag}.m{i}")
        else:
            t = _bottleneck(pw, ys[-1], c, shortcut, f"{tag}.m{i}", e=0.5)
        ys.append(t)
    cat = pw.concat(ys, 1, name=f"{tag}.cat")
    return pw.conv(cat, c2, 1, act=1, name=f"{tag}.cv2")


def _attention(pw, x, dim, num_heads, tag):
    """Position-sensitive attention (key_dim = head_dim/2) as plan ops."""
    _, C, H, W = pw.shapes[x]
    N = H * W
    head_dim = dim // num_heads
    key_dim = head_dim // 2
    h = dim + key_dim * num_heads * 2
    qkv = pw.conv(x, h, 1, act=0, name=f"{tag}.qkv")
    qkv = pw.reshape(qkv, [1, num_heads, key_dim * 2 + head_dim, N])
    q = pw.slice_axis(qkv, 2, 0, key_dim)
    k = pw.slice_axis(qkv, 2, key_dim, key_dim)
    v = pw.slice_axis(qkv, 2, 2 * key_dim, head_dim)
    qt = pw.permute(q, [0, 1, 3, 2])
    attn = pw.bmm(qt, k)
    scale = pw.init(f"{tag}.scale", np.array(key_dim ** -0.5, dtype=np.float32))
    attn = pw.add(attn, scale, 2)
    attn = pw.softmax(attn, 3)
    at = pw.permute(attn, [0, 1, 3, 2])
    o = pw.bmm(v, at)
    o = pw.reshape(o, [1, C, H, W])
    vv = pw.reshape(v, [1, C, H, W])
    pe = pw.conv(vv, C, 3, act=0, groups=C, name=f"{tag}.pe")
    o = pw.add(o, pe, 0)
    return pw.conv(o, C, 1, act=0, name=f"{tag}.proj")


def _c2psa(pw, x, c2, n, tag):
    c = c2 // 2
    y = pw.conv(x, 2 * c, 1, act=1, name=f"{tag}.cv1")
    a, b = pw.split_c(y, [c, c])
    for i in range(n):
        t = _attention(pw, b, c, c // 64, f"{tag}.m{i}.attn")
        b = pw.add(b, t, 0)
        f1 = pw.conv(b, 2 * c, 1, act=1, name=f"{tag}.m{i}.ffn0")
        f2 = pw.conv(f1, c, 1, act=0, name=f"{tag}.m{i}.ffn1")
        b = pw.add(b, f2, 0)
    cat = pw.concat([a, b], 1, name=f"{tag}.cat")
    return pw.conv(cat, c2, 1, act=1, name=f"{tag}.cv2")


def yolo11n_pose(out_dir: str, seed: int = 1234, imgsz: int = 640) -> str:
    pw = PlanWriter(seed)
    x = pw.input("images", [1, 3, imgsz, imgsz])
    x = pw.conv(x, 16, 3, 2, act=1, name="model.0")
    x = pw.conv(x, 32, 3, 2, act=1, name="model.1")
    x = _c3k2(pw, x, 64, 1, False, 0.25, True, "model.2")
    x = pw.conv(x, 64, 3, 2, act=1, name="model.3")
    p3 = _c3k2(pw, x, 128, 1, False, 0.25, True, "model.4")
    x = pw.conv(p3, 128, 3, 2, act=1, name="model.5")
    p4 = _c3k2(pw, x, 128, 1, True, 0.5, True, "model.6")
    x = pw.conv(p4, 256, 3, 2, act=1, name="model.7")
    x = _c3k2(pw, x, 256, 1, True, 0.5, True, "model.8")
    x = _sppf(pw, x, 256, "model.9")
    p5 = _c2psa(pw, x, 256, 1, "model.10")
    x = pw.upsample(p5)
    x = pw.concat([x, p4], 1, name="model.12")
    n13 = _c3k2(pw, x, 128, 1, False, 0.5, True, "model.13")
    x = pw.upsample(n13)
    x = pw.concat([x, p3], 1, name="model.15")
    o3 = _c3k2(pw, x, 64, 1, False, 0.5, True, "model.16")
    x = pw.conv(o3, 64, 3, 2, act=1, name="model.17")
    x = pw.concat([x, n13], 1, name="model.18")
    o4 = _c3k2(pw, x, 128, 1, False, 0.5, True, "model.19")
    x = pw.conv(o4, 128, 3, 2, act=1, name="model.20")
    x = pw.concat([x, p5], 1, name="model.21")
    o5 = _c3k2(pw, x, 256, 1, True, 0.5, True, "model.22")
    out = _pose_head(pw, [o3, o4, o5], c2=64, c3=64, c4=51, tag="model.23", dw_cls=True)
    pw.output(out)
    return pw.save(out_dir)


# ---------------------------------------------------------------------------
# MobileNetV3-small classifier
# ---------------------------------------------------------------------------

def _make_divisible(v: float, divisor: int = 8) -> int:
    new_v = max(divisor, int(v + divisor / 2) // divisor * divisor)
    if new_v < 0.9 * v:
        new_v += divisor
    return new_v


MBV3_SMALL = [
    # in, kernel, expanded, out, SE, activation (2=ReLU 3=HardSwish), stride
    (16, 3, 16, 16, True, 2, 2),
    (16, 3, 72, 24, False, 2, 2),
    (24, 3, 88, 24, False, 2, 1),
    (24, 5, 96, 40, True, 3, 2),
    (40, 5, 240, 40, True, 3, 1),
    (40, 5, 240, 40, True, 3, 1),
    (40, 5, 120, 48, True, 3, 1),
    (48, 5, 144, 48, True, 3, 1),
    (48, 5, 288, 96, True, 3, 2),
    (96, 5, 576, 96, True, 3, 1),
    (96, 5, 576, 96, True, 3, 1),
]


def mobilenetv3_small(out_dir: str, seed: int = 1234, imgsz: int = 224) -> str:
    pw = PlanWriter(seed)
    x = pw.input("input", [1, 3, imgsz, imgsz])
    x = pw.conv(x, 16, 3, 2, act=3, name="features.0")
    for i, (cin, k, exp, cout, se, act, s) in enumerate(MBV3_SMALL):
        tag = f"features.{i + 1}"
        inp = x
        if exp != cin:
            x = pw.conv(x, exp, 1, act=act, name=f"{tag}.expand")
        x = pw.conv(x, exp, k, s, act=act, groups=exp, name=f"{tag}.dw")
        if se:
            sq = _make_divisible(exp // 4, 8)
            g = pw.gap(x)
            g = pw.conv(g, sq, 1, act=2, name=f"{tag}.se.fc1")
            g = pw.conv(g, exp, 1, act=4, name=f"{tag}.se.fc2")
            x = pw.add(g, x, 2, name=f"{tag}.se.mul")
        x = pw.conv(x, cout, 1, act=0, name=f"{tag}.project")
        if s == 1 and cin == cout:
            x = pw.add(x, inp, 0, name=f"{tag}.add")
    x = pw.conv(x, 576, 1, act=3, name="features.12")
    x = pw.gap(x)
    x = pw.reshape(x, [1, 576])
    x = pw.gemm(x, 1024, act=3, name="classifier.0")
    out = pw.gemm(x, 1000, act=0, name="classifier.3")
    pw.output(out)
    return pw.save(out_dir)


# ---------------------------------------------------------------------------
# single-op plans (kernel sweeps)
# ---------------------------------------------------------------------------

def op_conv(out_dir: str, cin: int, cout: int, h: int, w: int, k: int, s: int = 1, act: int = 1,
            groups: int = 1, residual: bool = False, seed: int = 7, producer: bool = False,
            consumer: bool = False) -> str:
    """One convolution node; `producer` puts a 1x1 conv in front so that the
    measured conv reads a channels-last activation, `consumer` one behind it
    so that it writes one (as inside a network)."""
    pw = PlanWriter(seed)
    x = pw.input("x", [1, cin, h, w])
    if producer:
        x = pw.conv(x, cin, 1, act=1, name="pre")
    y = pw.conv(x, cout, k, s, act=act, groups=groups, name="op")
    if residual:
        y = pw.add(y, x, 0, name="res")
    if consumer:
        y = pw.conv(y, cout, 1, act=1, name="post")
    pw.output(y)
    return pw.save(out_dir)


def op_sppf(out_dir: str, c: int, h: int, w: int, levels: int = 3, seed: int = 7) -> str:
    """conv1x1 -> `levels` chained 5x5 max pools -> concat of all -> conv1x1
    (the SPPF block with channels-last tensors on both sides)."""
    pw = PlanWriter(seed)
    x = pw.input("x", [1, c, h, w])
    x = pw.conv(x, c, 1, act=1, name="pre")
    ys = [x]
    for _ in range(levels):
        ys.append(pw.maxpool(ys[-1], 5, 1, 2))
    y = pw.conv(pw.concat(ys, 1), c, 1, act=1, name="post")
    pw.output(y)
    return pw.save(out_dir)


def op_gap(out_dir: str, c: int, h: int, w: int, seed: int = 7) -> str:
    """conv1x1 -> global average pool (a channels-last input, as in the SE
    blocks and the classifier of MobileNetV3)."""
    pw = PlanWriter(seed)
    x = pw.input("x", [1, c, h, w])
    x = pw.conv(x, c, 1, act=1, name="pre")
    pw.output(pw.gap(x))
    return pw.save(out_dir)


def op_se(out_dir: str, c: int, h: int, w: int, seed: int = 7) -> str:
    """conv1x1 -> MobileNetV3's squeeze-excitation: global pool, fc1 (ReLU) and
    fc2 (HardSigmoid) as one-pixel 1x1 convs, channel-wise multiply."""
    pw = PlanWriter(seed)
    x = pw.input("x", [1, c, h, w])
    x = pw.conv(x, c, 1, act=1, name="pre")
    g = pw.gap(x)
    g = pw.conv(g, _make_divisible(c // 4, 8), 1, act=2, name="op.fc1")
    g = pw.conv(g, c, 1, act=4, name="op.fc2")
    pw.output(pw.add(g, x, 2, name="op.mul"))
    return pw.save(out_dir)


def op_attention(out_dir: str, c: int, h: int, w: int, heads: int = 0, seed: int = 7) -> str:
    """conv1x1 -> the position-sensitive attention block of YOLO11's C2PSA
    (qkv conv, slices, transposing permutes, two bmm, scale, softmax, pe
    depthwise conv, proj conv)."""
    pw = PlanWriter(seed)
    x = pw.input("x", [1, c, h, w])
    x = pw.conv(x, c, 1, act=1, name="pre")
    pw.output(_attention(pw, x, c, heads or max(1, c // 64), "op"))
    return pw.save(out_dir)


def op_upsample(out_dir: str, c: int, h: int, w: int, s: int = 2, seed: int = 7) -> str:
    """conv1x1 -> nearest upsample by s -> conv1x1 (channels-last both sides)."""
    pw = PlanWriter(seed)
    x = pw.input("x", [1, c, h, w])
    x = pw.conv(x, c, 1, act=1, name="pre")
    y = pw.conv(pw.upsample(x, s), c, 1, act=1, name="post")
    pw.output(y)
    return pw.save(out_dir)


def op_cat_conv1x1(out_dir: str, chans: Sequence[int], cout: int, h: int, w: int, act: int = 1,
                   seed: int = 7) -> str:
    """concat4 -> conv1x1 (exercises the CAT4 load-time rewrite)."""
    pw = PlanWriter(seed)
    x = pw.input("x", [1, chans[0], h, w])
    srcs = [pw.conv(x, chans[0], 1, act=1, name="pre")]
    for i, c in enumerate(chans[1:]):
        srcs.append(pw.conv(srcs[-1], c, 1, act=1, name=f"pre{i}"))
    cat = pw.concat(srcs, 1)
    y = pw.conv(cat, cout, 1, act=act, name="op")
    pw.output(y)
    return pw.save(out_dir)


def write_input(path: str, dims: Sequence[int], seed: int) -> np.ndarray:
    x = np.random.default_rng(seed).random(tuple(dims), dtype=np.float32)
    x.tofile(path)
    return x


MODELS = {
    "yolov8n-pose": yolov8n_pose,
    "yolo11n-pose": yolo11n_pose,
    "mobilenetv3-small": mobilenetv3_small,
}
