"""The CPU oracle pinned to the reference's own kernel code.

tests/golden/ref_kernels.npz holds outputs of the reference's OpenCL kernels
(kernels/ops.cl, kernels/conv_general.cl, kernels/gemm.cl, kernels/conv_ov.cl)
executed on the CPU (generator:
tests/golden/make_kernel_golden.py; build recipe: `make -C oracle ref`).  Each
case is replayed here through the oracle as a one-node plan.

* elementwise / layout / pooling / softmax / gap / bmm / generic conv: bit-exact;
* depthwise_f16, gemm_f16 (conv1x1 and its CAT4 form) and conv3x3_ov
  accumulate in fp16: bit-exact against the oracle's fp16 accumulation mode,
  which pins the oracle's indexing (taps, strides, padding, concat channel
  order, weight layout) and its epilogue (half(acc) + bias, activation,
  residual after activation); the oracle's fp32 mode (the build's contract)
  shares all of that and stays within the fp16 accumulator's drift of it.
"""
import os

import numpy as np
import pytest

from oracle import ivref

GOLD = os.path.join(os.path.dirname(__file__), "golden", "ref_kernels.npz")
_g = np.load(GOLD)
CASES = sorted({k.split("/")[0] for k in _g.files})


def ulp(a, b):
    def o(h):
        h = h.astype(np.int32)
        return np.where(h & 0x8000, -(h & 0x7FFF), h & 0x7FFF)
    return np.abs(o(a) - o(b))


def build_plan(tmp, name):
    if f"{name}/plan_text" in _g.files:  # a whole plan (contractions, CAT4)
        first = str(_g[f"{name}/plan_input"])
        for n in str(_g[f"{name}/inputs"]).split(","):
            if n != first:
                _g[f"{name}/in/{n}"].astype("<u2").tofile(os.path.join(tmp, f"init_{n}.bin"))
        path = os.path.join(tmp, "model.plan")
        with open(path, "w") as f:
            f.write(str(_g[f"{name}/plan_text"]))
        return path, _g[f"{name}/in/{first}"]
    op = str(_g[f"{name}/op"])
    attrs = str(_g[f"{name}/attrs"])
    names = str(_g[f"{name}/inputs"]).split(",")
    lines = []
    first = names[0]
    lines.append("input {} {}".format(first, " ".join(str(int(d)) for d in _g[f"{name}/dims/{first}"])))
    for n in names[1:]:
        arr = _g[f"{name}/in/{n}"]
        arr.astype("<u2").tofile(os.path.join(tmp, f"init_{n}.bin"))
        lines.append("init {} init_{}.bin {}".format(n, n, " ".join(str(int(d)) for d in _g[f"{name}/dims/{n}"])))
    lines.append("tensor y {}".format(" ".join(str(int(d)) for d in _g[f"{name}/out_dims"])))
    if op == "concat4":
        kv = dict(t.split("=") for t in attrs.split())
        cnt = [int(kv[k]) for k in ("ca", "cb", "cc", "cd")]
        it = iter(names)
        ins = [next(it) if c > 0 else "-" for c in cnt]
    else:
        ins = names
    lines.append(f"node {op} {','.join(ins)} y {attrs}")
    lines.append("output y")
    path = os.path.join(tmp, "model.plan")
    with open(path, "w") as f:
        f.write("\n".join(lines) + "\n")
    return path, _g[f"{name}/in/{first}"]


FP16_ACC = ("depthwise_", "gemm_", "gemmcat_", "conv3x3ov_")


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference_kernel(tmp_path, name):
    plan, x = build_plan(str(tmp_path), name)
    ref = _g[f"{name}/out"]
    half_acc = name.startswith(FP16_ACC)
    o = ivref.OraclePlan(plan, acc_order=2 if half_acc else 0)
    o.run_f16(x, 1)
    got = o.read_f16("y")
    assert got.shape == ref.shape
    d = ulp(got, ref)
    assert d.max() == 0, (name, int(d.max()), int((d > 0).sum()))
    if half_acc:
        # The contract's fp32 accumulation (the oracle's default mode, which
        # shares every index and epilogue step checked bit-exactly above) stays
        # close to the reference's fp16 accumulation: depthwise (9 or 25 terms)
        # within 2 fp16 ulps of the output scale; the convolutions (16 to 144
        # terms) within the fp16 accumulator's own drift (measured on these
        # cases: rel-L2 up to 2.0e-3, 4.6 ulps of the output scale), bounded at
        # rel-L2 3e-3 and 6 ulps.
        o32 = ivref.OraclePlan(plan, acc_order=0)
        o32.run_f16(x, 1)
        g, r = ivref.f16_to_f32(o32.read_f16("y")).astype(np.float64), ivref.f16_to_f32(ref).astype(np.float64)
        if name.startswith("depthwise_"):
            assert np.abs(g - r).max() <= 2 * 2.0 ** -10 * np.abs(r).max()
        else:
            assert np.linalg.norm(g - r) <= 3e-3 * np.linalg.norm(r), (name, np.linalg.norm(g - r) / np.linalg.norm(r))
            assert np.abs(g - r).max() <= 6 * 2.0 ** -10 * np.abs(r).max(), (name, np.abs(g - r).max())
