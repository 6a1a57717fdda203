"""Generates tests/golden/ref_kernels.npz by running the reference's OpenCL
kernels themselves (kernels/ops.cl, kernels/conv_general.cl, kernels/gemm.cl,
kernels/conv_ov.cl), compiled on the CPU into oracle/_ref/libclref.so by
`make -C oracle ref` (see oracle/clref/).

Every case stores its seeded fp16 inputs, the node attributes the plan would
carry, and the reference kernel's fp16 output.  tests/test_oracle_pinned.py
replays each case through the CPU oracle as a one-node plan.

Run from the repository root:  python tests/golden/make_kernel_golden.py
"""
import ctypes
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
LIB = os.path.join(ROOT, "oracle", "_ref", "libclref.so")
OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "ref_kernels.npz")


def h(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.float16)).view(np.uint16)


def main():
    if not os.path.exists(LIB):
        raise SystemExit("oracle/_ref/libclref.so missing: run `make -C oracle ref` first")
    L = ctypes.CDLL(LIB)
    VPT = ctypes.c_void_p
    L.clref_gemm.argtypes = [VPT, VPT, VPT] + [ctypes.c_int] * 3 + [VPT, VPT] + [ctypes.c_int] * 2 + [VPT] * 3 + \
        [ctypes.c_int] * 7
    L.clref_conv3x3_ov.argtypes = [VPT] * 5 + [ctypes.c_int] * 8
    rng = np.random.default_rng(99)
    cases = {}

    def P(a):
        return a.ctypes.data_as(ctypes.c_void_p)

    def add(name, op, inputs, attrs, out, dims):
        """inputs: list of (tensor name, uint16 array, dims); attrs: node attrs; out: uint16 output."""
        cases[name] = dict(op=op, inputs=inputs, attrs=attrs, out=out, dims=dims)

    def normal(shape, scale=1.0):
        return h(rng.standard_normal(shape) * scale)

    # ---- elementwise
    for op in range(4):
        for bs in (0, 1):
            a = normal(240)
            b = normal(1 if bs else 240) if op != 3 else h(rng.uniform(0.5, 2.0, 1 if bs else 240))
            y = np.zeros(240, np.uint16)
            L.clref_ew_binary(P(a), P(b), P(y), 240, op, bs)
            add(f"ew_binary_op{op}_bs{bs}", "ew_binary", [("a", a, [1, 240]), ("b", b, [1] if bs else [1, 240])],
                dict(op=op, n=240, b_scalar=bs), y, [1, 240])
    # broadcast (pose decode: [1,17,2,A] + [2,A]; [1,4,A] * [1,A])
    A = 40
    for op, ashape, bshape in [(0, [1, 17, 2, A], [2, A]), (2, [1, 17, 2, A], [1, A]), (2, [1, 4, A], [1, A]),
                               (1, [1, 2, A], [1, 2, A])]:
        oshape = ashape
        rank = len(oshape)

        def strides(s):
            al = [1] * (rank - len(s)) + list(s)
            st, acc = [0] * rank, 1
            for i in range(rank - 1, -1, -1):
                st[i] = 0 if (al[i] == 1 and oshape[i] != 1) else acc
                acc *= al[i]
            return st

        dims = np.array(list(oshape) + strides(ashape) + strides(bshape), dtype=np.int32)
        a, b = normal(int(np.prod(ashape))), normal(int(np.prod(bshape)))
        n = int(np.prod(oshape))
        y = np.zeros(n, np.uint16)
        L.clref_ew_binary_bcast(P(a), P(b), P(y), n, op, rank, P(dims))
        add(f"ew_binary_bcast_{op}_{'x'.join(map(str, bshape))}", "ew_binary", [("a", a, ashape), ("b", b, bshape)],
            dict(op=op, n=n, b_scalar=0, bdims=",".join(str(int(v)) for v in dims)), y, oshape)
    # SE scale: [1,C,1,1] * [1,C,H,W] through ew_binary_ch (the reference's pick for this pattern)
    C, HW = 8, 49
    a, b = normal(C), normal(C * HW)
    y = np.zeros(C * HW, np.uint16)
    L.clref_ew_binary_ch(P(a), P(b), P(y), HW, C, 2, 1)
    dims = [1, C, 7, 7, C, 1, 0, 0, C * HW, HW, 7, 1]
    add("ew_binary_ch_se", "ew_binary", [("a", a, [1, C, 1, 1]), ("b", b, [1, C, 7, 7])],
        dict(op=2, n=C * HW, b_scalar=0, bdims=",".join(map(str, dims))), y, [1, C, 7, 7])
    for op in range(5):
        x = h(rng.uniform(-8, 8, 300))
        y = np.zeros(300, np.uint16)
        L.clref_ew_unary(P(x), P(y), 300, op)
        add(f"ew_unary_op{op}", "ew_unary", [("x", x, [1, 300])], dict(op=op, n=300), y, [1, 300])
    # ---- layout
    x = normal(6 * 25)
    y = np.zeros(3 * 25, np.uint16)
    L.clref_copy_c(P(x), P(y), 25, 2, 3, 0)
    add("copy_c", "copy_c", [("x", x, [1, 6, 5, 5])], dict(HW=25, c0=2, cnt=3, dst_off=0), y, [1, 3, 5, 5])
    x = normal(3 * 5 * 7)
    y = np.zeros(3 * 3 * 7, np.uint16)
    L.clref_slice_axis(P(x), P(y), 3, 5, 7, 1, 3)
    add("slice_axis", "slice_axis", [("x", x, [1, 3, 5, 7])], dict(outer=3, axdim=5, inner=7, start=1, len=3), y,
        [1, 3, 3, 7])
    for outer, inner, cs in [(2, 5, (1, 2, 3, 0)), (1, 40, (4, 1, 3, 2)), (3, 1, (6, 4, 2, 0))]:
        srcs = [normal(outer * c * inner) if c else np.zeros(1, np.uint16) for c in cs]
        tot = sum(cs)
        y = np.zeros(outer * tot * inner, np.uint16)
        L.clref_concat4(P(srcs[0]), cs[0], P(srcs[1]), cs[1], P(srcs[2]), cs[2], P(srcs[3]), cs[3], P(y), outer, inner)
        ins = [(f"s{i}", srcs[i], [1, outer, cs[i], inner]) for i in range(4) if cs[i]]
        add(f"concat4_{outer}_{inner}", "concat4", ins,
            dict(ca=cs[0], cb=cs[1], cc=cs[2], cd=cs[3], outer=outer, inner=inner), y, [1, outer, tot, inner])
    for (Cc, H, W, K, S, P_) in [(3, 9, 9, 5, 1, 2), (2, 9, 8, 3, 2, 1)]:
        Ho, Wo = (H + 2 * P_ - K) // S + 1, (W + 2 * P_ - K) // S + 1
        x = normal(Cc * H * W)
        y = np.zeros(Cc * Ho * Wo, np.uint16)
        L.clref_maxpool(P(x), P(y), Cc, H, W, Ho, Wo, K, S, P_)
        add(f"maxpool_k{K}s{S}", "maxpool", [("x", x, [1, Cc, H, W])], dict(C=Cc, H=H, W=W, Hout=Ho, Wout=Wo, K=K, S=S, P=P_),
            y, [1, Cc, Ho, Wo])
    x = normal(3 * 4 * 5)
    y = np.zeros(3 * 8 * 10, np.uint16)
    L.clref_resize_nn(P(x), P(y), 3, 4, 5, 2)
    add("resize_nn", "resize_nn", [("x", x, [1, 3, 4, 5])], dict(C=3, H=4, W=5, S=2), y, [1, 3, 8, 10])
    x = normal(2 * 16 * 30, 3.0)
    y = np.zeros(x.size, np.uint16)
    L.clref_softmax_axis(P(x), P(y), 2, 16, 30)
    add("softmax_axis_dfl", "softmax_axis", [("x", x, [1, 2, 16, 30])], dict(outer=2, axdim=16, inner=30), y,
        [1, 2, 16, 30])
    for D1, D2, I, mode in [(4, 6, 10, 0), (2, 5, 7, 1)]:
        x = normal(D1 * D2 * I)
        y = np.zeros(x.size, np.uint16)
        L.clref_permute_0213(P(x), P(y), D1, D2, I, mode)
        oshape = [1, D2, D1, I] if mode == 0 else [1, D1, I, D2]
        add(f"permute_mode{mode}", "permute_0213", [("x", x, [1, D1, D2, I])], dict(D1=D1, D2=D2, I=I, mode=mode), y,
            oshape)
    for Cc, H, W in [(5, 15, 20), (4, 7, 7), (3, 56, 56)]:
        x = normal(Cc * H * W)
        y = np.zeros(Cc, np.uint16)
        L.clref_gap_r(P(x), P(y), Cc, H * W)
        add(f"gap_{Cc}_{H}x{W}", "gap", [("x", x, [1, Cc, H, W])], dict(C=Cc, HW=H * W), y, [1, Cc, 1, 1])
    a, b = normal(2 * 5 * 7), normal(2 * 7 * 6)
    y = np.zeros(2 * 5 * 6, np.uint16)
    L.clref_bmm(P(a), P(b), P(y), 1, 2, 5, 7, 6)
    add("bmm", "bmm", [("a", a, [1, 2, 5, 7]), ("b", b, [1, 2, 7, 6])], dict(B0=1, B1=2, M=5, K=7, N=6), y,
        [1, 2, 5, 6])
    x, bb = normal(4 * 6), normal(4)
    y = np.zeros(24, np.uint16)
    L.clref_bias_add(P(x), P(bb), P(y), 24, 6)
    add("bias_add", "bias_add", [("x", x, [1, 4, 6]), ("b", bb, [4])], dict(HW=6), y, [1, 4, 6])
    # ---- convolutions
    for (Cin, Cout, H, W, K, S, G, act) in [(4, 6, 9, 9, 3, 1, 1, 0), (4, 6, 9, 9, 3, 2, 1, 1), (6, 4, 8, 8, 1, 1, 1, 2),
                                            (8, 8, 7, 7, 3, 1, 2, 3), (6, 6, 9, 9, 5, 2, 3, 4)]:
        P_ = K // 2
        Ho, Wo = (H + 2 * P_ - K) // S + 1, (W + 2 * P_ - K) // S + 1
        x = h(rng.uniform(0, 1, Cin * H * W))
        w = normal(Cout * (Cin // G) * K * K, np.sqrt(2.0 / (Cin // G * K * K)))
        bias = normal(Cout, 0.05)
        y = np.zeros(Cout * Ho * Wo, np.uint16)
        L.clref_conv_general(P(x), P(w), P(bias), P(y), Cin, H, W, Cout, Ho, Wo, K, S, P_, G, act)
        add(f"conv_general_{Cin}_{Cout}_k{K}s{S}g{G}a{act}", "conv_general",
            [("x", x, [1, Cin, H, W]), ("w", w, [Cout, Cin // G, K, K]), ("bias", bias, [Cout])],
            dict(K=K, S=S, P=P_, G=G, Hout=Ho, Wout=Wo, act=act), y, [1, Cout, Ho, Wo])
    for (Cc, H, W, K, S, act) in [(5, 9, 9, 3, 1, 0), (6, 10, 10, 3, 2, 2), (4, 9, 9, 5, 1, 3), (3, 11, 11, 5, 2, 3),
                                  (4, 8, 8, 3, 1, 1), (5, 7, 7, 5, 1, 4), (7, 8, 9, 3, 2, 3), (6, 9, 9, 3, 1, 2)]:
        P_ = K // 2
        Ho, Wo = (H + 2 * P_ - K) // S + 1, (W + 2 * P_ - K) // S + 1
        x = normal(Cc * H * W)
        w = normal(Cc * K * K, np.sqrt(2.0 / (K * K)))
        bias = normal(Cc, 0.05)
        y = np.zeros(Cc * Ho * Wo, np.uint16)
        r = L.clref_depthwise(P(x), P(w), P(bias), P(y), Cc, H, W, Ho, Wo, K, S, act)
        assert r == 0, (K, S, act)
        add(f"depthwise_{Cc}_k{K}s{S}a{act}", "conv_general",
            [("x", x, [1, Cc, H, W]), ("w", w, [Cc, 1, K, K]), ("bias", bias, [Cc])],
            dict(K=K, S=S, P=P_, G=Cc, Hout=Ho, Wout=Wo, act=act), y, [1, Cc, Ho, Wo])

    # ---- the contractions, fp16 accumulation as in the reference: gemm_f16
    # (conv1x1 with N > 1, plain and CAT4) and conv3x3_ov.  These cases carry
    # their whole plan: the CAT4 one is concat4 + conv1x1 (the executor's
    # load-time rewrite turns it into conv1x1_cat4, which the reference runs as
    # gemm_f16 with CAT4 staging); residuals and extra sources are inits.

    def plan_case(name, plan_input, tensors, lines, y, ydims):
        cases[name] = dict(op="plan", inputs=tensors, attrs={}, out=y, dims=ydims, plan_input=plan_input,
                           plan_text="\n".join(lines) + "\n")

    def decl(kind, n, d):
        return f"{kind} {n} " + ("" if kind == "input" else f"init_{n}.bin ") + " ".join(map(str, d))

    for (Cin, Cout, Hh, Ww, act, res) in [(40, 32, 10, 10, 1, 0), (16, 16, 8, 9, 0, 0), (32, 70, 5, 13, 3, 0),
                                          (64, 40, 6, 6, 1, 1), (24, 20, 7, 7, 2, 0), (36, 24, 5, 5, 4, 0),
                                          (20, 12, 4, 4, 5, 0), (72, 130, 9, 9, 1, 0), (33, 16, 6, 6, 3, 1)]:
        N = Hh * Ww
        x = h(rng.uniform(-1, 1, Cin * N))
        w = normal(Cout * Cin, np.sqrt(2.0 / Cin))
        bias = normal(Cout, 0.05)
        rr = normal(Cout * N) if res else None
        y = np.zeros(Cout * N, np.uint16)
        r = L.clref_gemm(P(w), P(x), P(y), Cout, N, Cin, P(bias), P(rr) if res else None, act, 0, None, None, None,
                         0, 0, 0, 0, 0, 0, 0)
        assert r == 0, (act, res)
        t = [("x", x, [1, Cin, Hh, Ww]), ("w", w, [Cout, Cin]), ("bias", bias, [Cout])]
        if res:
            t.append(("res", rr, [1, Cout, Hh, Ww]))
        lines = [decl("input", "x", [1, Cin, Hh, Ww])] + [decl("init", n, d) for n, _, d in t[1:]]
        lines += [f"tensor y 1 {Cout} {Hh} {Ww}",
                  f"node conv1x1 w,x,bias,{'res' if res else '-'} y act={act}", "output y"]
        plan_case(f"gemm_{Cin}_{Cout}_{N}_a{act}_r{res}", "x", t, lines, y, [1, Cout, Hh, Ww])
    for (cs, Cout, Hh, Ww, act, res) in [((16, 16, 16, 0), 32, 10, 10, 1, 0), ((8, 24, 16, 8), 40, 9, 7, 0, 0),
                                         ((16, 8, 0, 0), 24, 6, 8, 1, 1)]:
        N = Hh * Ww
        Cin = sum(cs)
        srcs = [h(rng.uniform(-1, 1, c * N)) if c else np.zeros(1, np.uint16) for c in cs]
        w = normal(Cout * Cin, np.sqrt(2.0 / Cin))
        bias = normal(Cout, 0.05)
        rr = normal(Cout * N) if res else None
        y = np.zeros(Cout * N, np.uint16)
        r = L.clref_gemm(P(w), P(srcs[0]), P(y), Cout, N, Cin, P(bias), P(rr) if res else None, act, 1,
                         P(srcs[1]), P(srcs[2]), P(srcs[3]), cs[0], cs[1], cs[2], 0, 0, 0, 0)
        assert r == 0, (act, res)
        names = [f"s{i}" for i in range(4)]
        t = [("s0", srcs[0], [1, cs[0], Hh, Ww])] + [(names[i], srcs[i], [1, cs[i], Hh, Ww]) for i in (1, 2, 3) if cs[i]]
        t += [("w", w, [Cout, Cin]), ("bias", bias, [Cout])]
        if res:
            t.append(("res", rr, [1, Cout, Hh, Ww]))
        lines = [decl("input", "s0", [1, cs[0], Hh, Ww])] + [decl("init", n, d) for n, _, d in t[1:]]
        cat_ins = ",".join(names[i] if cs[i] else "-" for i in range(4))
        lines += [f"tensor cat 1 {Cin} {Hh} {Ww}", f"tensor y 1 {Cout} {Hh} {Ww}",
                  f"node concat4 {cat_ins} cat ca={cs[0]} cb={cs[1]} cc={cs[2]} cd={cs[3]} outer=1 inner={N}",
                  f"node conv1x1 w,cat,bias,{'res' if res else '-'} y act={act}", "output y"]
        plan_case(f"gemmcat_{'_'.join(map(str, cs))}_{Cout}_a{act}_r{res}", "s0", t, lines, y, [1, Cout, Hh, Ww])
    for (Cin, Cout, Hh, Ww, S, act, res) in [(8, 32, 12, 12, 1, 1, 0), (8, 16, 12, 12, 2, 1, 0), (16, 51, 10, 10, 1, 1, 0),
                                             (3, 16, 20, 20, 2, 1, 0), (8, 8, 9, 9, 1, 1, 1), (12, 24, 16, 16, 2, 0, 0),
                                             (16, 40, 8, 8, 1, 3, 0), (6, 33, 11, 13, 2, 3, 0), (10, 20, 10, 10, 2, 1, 1),
                                             (7, 9, 8, 11, 1, 0, 0)]:
        Ho, Wo = (Hh - 1) // S + 1, (Ww - 1) // S + 1
        x = h(rng.uniform(-1, 1, Cin * Hh * Ww))
        w = normal(Cout * Cin * 9, np.sqrt(2.0 / (Cin * 9)))
        bias = normal(Cout, 0.05)
        rr = normal(Cout * Ho * Wo) if res else None
        y = np.zeros(Cout * Ho * Wo, np.uint16)
        r = L.clref_conv3x3_ov(P(x), P(w), P(bias), P(rr) if res else None, P(y), Cin, Hh, Ww, Cout, Ho, Wo, S, act)
        assert r == 0, (S, act, res)
        t = [("x", x, [1, Cin, Hh, Ww]), ("w", w, [Cout, Cin, 3, 3]), ("bias", bias, [Cout])]
        if res:
            t.append(("res", rr, [1, Cout, Ho, Wo]))
        lines = [decl("input", "x", [1, Cin, Hh, Ww])] + [decl("init", n, d) for n, _, d in t[1:]]
        lines += [f"tensor y 1 {Cout} {Ho} {Wo}",
                  f"node conv3x3 x,w,bias,{'res' if res else '-'} y stride={S} pad=1 Hout={Ho} Wout={Wo} act={act}",
                  "output y"]
        plan_case(f"conv3x3ov_{Cin}_{Cout}_{Hh}x{Ww}_s{S}_a{act}_r{res}", "x", t, lines, y, [1, Cout, Ho, Wo])

    flat = {}
    for name, c in cases.items():
        flat[f"{name}/op"] = np.array(c["op"])
        flat[f"{name}/attrs"] = np.array(" ".join(f"{k}={v}" for k, v in c["attrs"].items()))
        flat[f"{name}/out"] = c["out"]
        flat[f"{name}/out_dims"] = np.array(c["dims"], dtype=np.int64)
        flat[f"{name}/inputs"] = np.array(",".join(n for n, _, _ in c["inputs"]))
        if "plan_text" in c:
            flat[f"{name}/plan_text"] = np.array(c["plan_text"])
            flat[f"{name}/plan_input"] = np.array(c["plan_input"])
        for n, arr, d in c["inputs"]:
            flat[f"{name}/in/{n}"] = arr
            flat[f"{name}/dims/{n}"] = np.array(d, dtype=np.int64)
    np.savez_compressed(OUT, **flat)
    print("wrote", OUT, len(cases), "cases", os.path.getsize(OUT), "bytes")


if __name__ == "__main__":
    sys.exit(main())
