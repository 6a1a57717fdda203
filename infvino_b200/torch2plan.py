"""PyTorch module -> plan converter (the reference's scripts/onnx2plan.py
converts ONNX graphs; onnx is not a dependency here, so this traces the model
with torch.fx instead and writes the same plan format).

    from infvino_b200 import torch2plan
    plan_path = torch2plan.convert(model.eval(), (1, 3, 640, 640), "models/net")

Writes <out_dir>/model.plan and one fp16 init_<name>.bin per initializer
(paths relative to the plan, as scripts/onnx2plan.py:53-70 writes them).  The
plan grammar, op names, attributes, node routing and activation-fusion rules
follow scripts/onnx2plan.py so that the executor sees what it would see for
the same network exported to ONNX:
  * Conv2d (+ BatchNorm2d folded in eval mode): 3x3 with groups 1 and stride 1
    or 2 -> conv3x3 (stride 2 carries the cfg attribute); 1x1 with groups 1 ->
    conv1x1; anything else (depthwise, 5x5, grouped) -> conv_general;
    (onnx2plan.py:172-226)
  * a conv's sole activation consumer is folded into the conv when its kernel
    family implements it (SiLU everywhere; 1x1: Sigmoid, ReLU, HardSwish,
    HardSigmoid; 3x3: HardSwish; generic: HardSwish, ReLU, HardSigmoid),
    canonical codes 1=SiLU 2=ReLU 3=HardSwish 4=HardSigmoid 5=Sigmoid
    (onnx2plan.py:126-148); other activations -> ew_unary
    (0=sigmoid 1=silu 2=relu 3=hswish 4=hsigmoid);
  * Linear -> conv1x1 on the flattened vector (onnx2plan.py:416-430);
  * add / sub / mul / div, with ONNX-style broadcast strides `bdims` when the
    shapes differ and b_scalar for a one-element constant (:245-279);
  * cat -> concat4 (chained beyond four sources, :280-297); chunk / split
    along channels -> copy_c, along other axes -> slice_axis (:298-326);
  * MaxPool2d -> maxpool; nearest Upsample / interpolate by an integer factor
    -> resize_nn; global average pooling -> gap; flatten / reshape / view ->
    reshape; softmax -> softmax_axis; Dropout / Identity -> the tensor itself.
Batch 1 (dim 0 of every tensor), as the reference's plans declare.  The
model must trace with torch.fx: no data-dependent control flow, and chunk /
split results unpacked into names (`a, b = x.chunk(2, 1)`) rather than
iterated (`list(x.chunk(2, 1))`).
"""
from __future__ import annotations

import operator
import os
import re
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

ACT_1X1 = {"sigmoid": 5, "relu": 2, "hardswish": 3, "hardsigmoid": 4, "silu": 1}
ACT_3X3 = {"hardswish": 3, "silu": 1}
ACT_GENERAL = {"hardswish": 3, "relu": 2, "hardsigmoid": 4, "silu": 1}
UNARY_CODE = {"sigmoid": 0, "silu": 1, "relu": 2, "hardswish": 3, "hardsigmoid": 4}
BINARY_CODE = {"add": 0, "sub": 1, "mul": 2, "div": 3}


def _sanitize(name: str) -> str:
    return re.sub(r"[^A-Za-z0-9_.]", "_", name)


class _Writer:
    def __init__(self, out_dir: str):
        self.out_dir = out_dir
        self.lines: List[str] = []
        self.declared = set()
        self.n_inits = 0

    def init(self, name: str, arr: np.ndarray) -> str:
        name = _sanitize(name)
        if name in self.declared:
            return name
        a = np.ascontiguousarray(arr, dtype=np.float16)
        base = f"init_{name}.bin"
        a.tofile(os.path.join(self.out_dir, base))
        self.lines.append("init {} {} {}".format(name, base, " ".join(str(int(d)) for d in (a.shape or (1,)))))
        self.declared.add(name)
        self.n_inits += 1
        return name

    def tensor(self, name: str, dims: Sequence[int]) -> str:
        if name not in self.declared:
            self.declared.add(name)
            self.lines.append("tensor {} {}".format(name, " ".join(str(int(d)) for d in dims)))
        return name

    def node(self, kind: str, ins: Sequence[str], outs: Sequence[str], **attrs):
        a = " ".join(f"{k}={v}" for k, v in attrs.items() if v is not None)
        self.lines.append("node {} {} {} {}".format(kind, ",".join(ins) or "-", ",".join(outs), a).rstrip())


def _act_kind(gm, n) -> Optional[str]:
    """The activation a graph node applies, if it is one."""
    import torch
    import torch.nn as nn
    import torch.nn.functional as F
    if n.op == "call_module":
        m = gm.get_submodule(n.target)
        for cls, k in ((nn.SiLU, "silu"), (nn.ReLU, "relu"), (nn.Hardswish, "hardswish"),
                       (nn.Hardsigmoid, "hardsigmoid"), (nn.Sigmoid, "sigmoid")):
            if isinstance(m, cls):
                return k
        return None
    if n.op in ("call_function", "call_method"):
        t = n.target
        table = {F.silu: "silu", F.relu: "relu", torch.relu: "relu", F.hardswish: "hardswish",
                 F.hardsigmoid: "hardsigmoid", torch.sigmoid: "sigmoid", F.sigmoid: "sigmoid",
                 "sigmoid": "sigmoid", "relu": "relu"}
        return table.get(t)
    return None


def convert(model, input_shape: Sequence[int], out_dir: str, input_name: str = "images",
            plan_name: str = "model.plan") -> str:
    """Traces `model` (in eval mode) on a seeded input of `input_shape` and
    writes the plan and its inits into `out_dir`; returns the plan path."""
    import torch
    import torch.fx
    import torch.nn as nn
    import torch.nn.functional as F
    from torch.fx.passes.shape_prop import ShapeProp

    os.makedirs(out_dir, exist_ok=True)
    model = model.eval()
    gm = torch.fx.symbolic_trace(model)
    example = torch.rand(*input_shape, generator=torch.Generator().manual_seed(0))
    with torch.no_grad():
        ShapeProp(gm).propagate(example)
    nodes = list(gm.graph.nodes)
    users = {n: list(n.users) for n in nodes}

    def shape(n) -> List[int]:
        tm = n.meta.get("tensor_meta")
        if tm is None:
            raise NotImplementedError(f"no shape for {n.format_node()}")
        return list(tm.shape)

    w = _Writer(out_dir)
    name_of: Dict[object, str] = {}   # fx node -> plan tensor name
    done = set()                      # nodes folded into an earlier one

    def tname(n) -> str:
        return _sanitize(n.name)

    def declare(n, name: Optional[str] = None) -> str:
        nm = name or tname(n)
        w.tensor(nm, shape(n))
        name_of[n] = nm
        return nm

    def sole_user(n):
        us = users.get(n, [])
        return us[0] if len(us) == 1 else None

    def is_module(n, cls) -> bool:
        return n.op == "call_module" and isinstance(gm.get_submodule(n.target), cls)

    def fold_act(n, table) -> Tuple[object, int]:
        u = sole_user(n)
        if u is not None and u.op != "output":
            k = _act_kind(gm, u)
            if k in table:
                done.add(u)
                return u, table[k]
        return n, 0

    def emit_conv(n):
        conv = gm.get_submodule(n.target)
        if conv.padding_mode != "zeros" or conv.kernel_size[0] != conv.kernel_size[1] or \
                conv.stride[0] != conv.stride[1] or conv.dilation != (1, 1):
            raise NotImplementedError(f"conv {n.target}: only square kernels, equal strides, zero padding")
        W = conv.weight.detach().double().numpy()
        B = conv.bias.detach().double().numpy() if conv.bias is not None else None
        last = n
        bn_user = sole_user(n)
        if bn_user is not None and is_module(bn_user, nn.BatchNorm2d):  # fold BN (eval statistics)
            bn = gm.get_submodule(bn_user.target)
            g = bn.weight.detach().double().numpy() if bn.weight is not None else np.ones(W.shape[0])
            beta = bn.bias.detach().double().numpy() if bn.bias is not None else np.zeros(W.shape[0])
            s = g / np.sqrt(bn.running_var.detach().double().numpy() + bn.eps)
            W = W * s[:, None, None, None]
            B = (B if B is not None else 0.0) - bn.running_mean.detach().double().numpy()
            B = B * s + beta
            done.add(bn_user)
            last = bn_user
        k, st, pad, groups = conv.kernel_size[0], conv.stride[0], conv.padding[0], conv.groups
        if isinstance(pad, str):
            raise NotImplementedError(f"conv {n.target}: string padding")
        cout, cin_g = W.shape[0], W.shape[1]
        x = name_of[n.args[0]]
        wname = w.init(f"{n.target}.weight", W.reshape(cout, cin_g, k, k) if k != 1 or groups != 1
                       else W.reshape(cout, cin_g))
        bname = w.init(f"{n.target}.bias", B) if B is not None else "-"
        oshape = shape(last)
        if k == 3 and groups == 1 and st in (1, 2):
            final, act = fold_act(last, ACT_3X3)
            out = declare(final)
            name_of[last] = out
            w.node("conv3x3", [x, wname, bname, "-"], [out], stride=st, pad=pad, Hout=oshape[2], Wout=oshape[3],
                   act=(act or None), cfg=(None if st == 1 else "64,8,1,32,8,2"))
        elif k == 1 and groups == 1 and st == 1 and pad == 0:
            final, act = fold_act(last, ACT_1X1)
            out = declare(final)
            name_of[last] = out
            w.node("conv1x1", [wname, x, bname, "-"], [out], act=(act or None))
        else:
            final, act = fold_act(last, ACT_GENERAL)
            out = declare(final)
            name_of[last] = out
            w.node("conv_general", [x, wname, bname], [out], K=k, S=st, P=pad, G=groups, Hout=oshape[2],
                   Wout=oshape[3], act=(act or None))

    def emit_linear(n):
        lin = gm.get_submodule(n.target)
        x = name_of[n.args[0]]
        wname = w.init(f"{n.target}.weight", lin.weight.detach().numpy())
        bname = w.init(f"{n.target}.bias", lin.bias.detach().numpy()) if lin.bias is not None else "-"
        final, act = fold_act(n, ACT_1X1)
        out = declare(final)
        name_of[n] = out
        w.node("conv1x1", [wname, x, bname, "-"], [out], act=(act or None))

    def operand(a, n, ref_shape) -> Tuple[str, List[int]]:
        if hasattr(a, "op"):
            return name_of[a], shape(a)
        arr = np.array(a, dtype=np.float32).reshape(-1) if np.ndim(a) else np.array([a], dtype=np.float32)
        return w.init(f"{n.name}_const", arr), list(arr.shape)

    def emit_binary(n, kind):
        a, b = n.args[0], n.args[1]
        if not hasattr(a, "op"):  # constant first: a + x == x + a (only for commutative ops)
            if kind not in ("add", "mul"):
                raise NotImplementedError(f"{n.format_node()}: constant left operand")
            a, b = b, a
        an, ash = operand(a, n, None)
        bn_, bsh = operand(b, n, None)
        osh = shape(n)
        out = declare(n)
        b_scalar, bdims = 0, None
        b_const = not hasattr(b, "op")
        if list(ash) != list(osh) or (b_const and list(bsh) != list(osh)):
            rank = len(osh)

            def strides(s):
                al = [1] * (rank - len(s)) + list(s)
                st, acc = [0] * rank, 1
                for i in range(rank - 1, -1, -1):
                    st[i] = 0 if (al[i] == 1 and osh[i] != 1) else acc
                    acc *= al[i]
                return st

            bdims = ",".join(str(int(v)) for v in list(osh) + strides(ash) + strides(bsh))
        if b_const and int(np.prod(bsh)) == 1 and list(ash) == list(osh):
            b_scalar, bdims = 1, None
        elif b_const and list(bsh) != list(osh):
            raise NotImplementedError(f"{n.format_node()}: a constant operand that is neither scalar nor full-size")
        w.node("ew_binary", [an, bn_], [out], op=BINARY_CODE[kind], n=int(np.prod(osh)), b_scalar=b_scalar,
               bdims=bdims)

    def emit_concat(n, srcs, dim):
        osh = shape(n)
        rank = len(osh)
        dim = dim + rank if dim < 0 else dim
        outer, inner = int(np.prod(osh[:dim])), int(np.prod(osh[dim + 1:]))
        names = [name_of[s] for s in srcs]
        counts = [shape(s)[dim] for s in srcs]
        while len(names) > 4:  # concat4 chains: the first four into a partial tensor
            part = f"{tname(n)}_part{len(names)}"
            psh = list(osh)
            psh[dim] = sum(counts[:4])
            w.tensor(part, psh)
            w.node("concat4", names[:4], [part], ca=counts[0], cb=counts[1], cc=counts[2], cd=counts[3],
                   outer=outer, inner=inner)
            names, counts = [part] + names[4:], [psh[dim]] + counts[4:]
        while len(names) < 4:
            names.append("-")
            counts.append(0)
        out = declare(n)
        w.node("concat4", names, [out], ca=counts[0], cb=counts[1], cc=counts[2], cd=counts[3], outer=outer,
               inner=inner)

    def emit_split(n, parts, dim):
        """chunk / split: the getitem users of `n` become copy_c / slice_axis nodes."""
        x = name_of[n.args[0]]
        xsh = shape(n.args[0])
        rank = len(xsh)
        dim = dim + rank if dim < 0 else dim
        starts = np.concatenate([[0], np.cumsum(parts)[:-1]]).astype(int)
        for u in users[n]:
            if not (u.op == "call_function" and u.target == operator.getitem):
                raise NotImplementedError(f"split result used as a whole: {u.format_node()}")
            i = u.args[1]
            out = declare(u)
            if dim == 1:
                w.node("copy_c", [x], [out], HW=int(np.prod(xsh[2:])), c0=int(starts[i]), cnt=int(parts[i]), dst_off=0)
            else:
                w.node("slice_axis", [x], [out], outer=int(np.prod(xsh[:dim])), axdim=xsh[dim],
                       inner=int(np.prod(xsh[dim + 1:])), start=int(starts[i]), len=int(parts[i]))
            done.add(u)

    for n in nodes:
        if n in done:
            continue
        if n.op == "placeholder":
            name_of[n] = input_name
            w.declared.add(input_name)
            w.lines.append("input {} {}".format(input_name, " ".join(str(d) for d in shape(n))))
            continue
        if n.op == "output":
            outs = n.args[0] if isinstance(n.args[0], (tuple, list)) else [n.args[0]]
            for o in outs:
                w.lines.append(f"output {name_of[o]}")
            continue
        if n.op == "get_attr":
            raise NotImplementedError(f"parameter used directly: {n.target}")
        if n.op == "call_module":
            m = gm.get_submodule(n.target)
            if isinstance(m, nn.Conv2d):
                emit_conv(n)
            elif isinstance(m, nn.Linear):
                emit_linear(n)
            elif isinstance(m, (nn.Dropout, nn.Identity)):
                name_of[n] = name_of[n.args[0]]
            elif isinstance(m, nn.MaxPool2d):
                k = m.kernel_size if isinstance(m.kernel_size, int) else m.kernel_size[0]
                s = m.stride if isinstance(m.stride, int) else m.stride[0]
                p = m.padding if isinstance(m.padding, int) else m.padding[0]
                xsh, osh = shape(n.args[0]), shape(n)
                out = declare(n)
                w.node("maxpool", [name_of[n.args[0]]], [out], C=xsh[1], H=xsh[2], W=xsh[3], Hout=osh[2],
                       Wout=osh[3], K=k, S=s, P=p)
            elif isinstance(m, nn.Upsample):
                if m.mode != "nearest":
                    raise NotImplementedError(f"upsample mode {m.mode}")
                xsh, osh = shape(n.args[0]), shape(n)
                out = declare(n)
                w.node("resize_nn", [name_of[n.args[0]]], [out], C=xsh[1], H=xsh[2], W=xsh[3], S=osh[2] // xsh[2])
            elif isinstance(m, nn.AdaptiveAvgPool2d):
                if tuple(shape(n)[2:]) != (1, 1):
                    raise NotImplementedError("adaptive average pooling to a size other than 1x1")
                xsh = shape(n.args[0])
                out = declare(n)
                w.node("gap", [name_of[n.args[0]]], [out], C=xsh[1], HW=xsh[2] * xsh[3])
            elif isinstance(m, nn.Flatten):
                out = declare(n)
                w.node("reshape", [name_of[n.args[0]]], [out])
            elif isinstance(m, nn.Softmax):
                xsh = shape(n.args[0])
                ax = m.dim + len(xsh) if m.dim < 0 else m.dim
                out = declare(n)
                w.node("softmax_axis", [name_of[n.args[0]]], [out], outer=int(np.prod(xsh[:ax])), axdim=xsh[ax],
                       inner=int(np.prod(xsh[ax + 1:])))
            elif _act_kind(gm, n):
                out = declare(n)
                w.node("ew_unary", [name_of[n.args[0]]], [out], op=UNARY_CODE[_act_kind(gm, n)],
                       n=int(np.prod(shape(n))))
            else:
                raise NotImplementedError(f"module {type(m).__name__} ({n.target})")
            continue
        t = n.target
        if _act_kind(gm, n):
            out = declare(n)
            w.node("ew_unary", [name_of[n.args[0]]], [out], op=UNARY_CODE[_act_kind(gm, n)], n=int(np.prod(shape(n))))
        elif t in (operator.add, operator.iadd, torch.add, "add", "add_"):
            emit_binary(n, "add")
        elif t in (operator.sub, torch.sub, "sub"):
            emit_binary(n, "sub")
        elif t in (operator.mul, operator.imul, torch.mul, "mul", "mul_"):
            emit_binary(n, "mul")
        elif t in (operator.truediv, torch.div, "div"):
            emit_binary(n, "div")
        elif t in (torch.cat, torch.concat):
            dim = n.kwargs.get("dim", n.args[1] if len(n.args) > 1 else 0)
            emit_concat(n, list(n.args[0]), dim)
        elif t in (torch.chunk, "chunk"):
            xsh = shape(n.args[0])
            chunks = n.args[1] if len(n.args) > 1 else n.kwargs["chunks"]
            dim = n.kwargs.get("dim", n.args[2] if len(n.args) > 2 else 0)
            size = -(-xsh[dim] // chunks)
            parts = [min(size, xsh[dim] - i * size) for i in range(chunks) if i * size < xsh[dim]]
            emit_split(n, parts, dim)
        elif t in (torch.split, "split"):
            xsh = shape(n.args[0])
            sz = n.args[1] if len(n.args) > 1 else n.kwargs["split_size_or_sections"]
            dim = n.kwargs.get("dim", n.args[2] if len(n.args) > 2 else 0)
            parts = list(sz) if isinstance(sz, (list, tuple)) else [min(sz, xsh[dim] - s) for s in range(0, xsh[dim], sz)]
            emit_split(n, parts, dim)
        elif t in (torch.flatten, "flatten", "view", "reshape", torch.reshape):
            out = declare(n)
            w.node("reshape", [name_of[n.args[0]]], [out])
        elif t in (F.adaptive_avg_pool2d,):
            xsh = shape(n.args[0])
            out = declare(n)
            w.node("gap", [name_of[n.args[0]]], [out], C=xsh[1], HW=xsh[2] * xsh[3])
        elif t in (F.max_pool2d,):
            xsh, osh = shape(n.args[0]), shape(n)
            k = n.kwargs.get("kernel_size", n.args[1] if len(n.args) > 1 else None)
            s = n.kwargs.get("stride", n.args[2] if len(n.args) > 2 else k) or k
            p = n.kwargs.get("padding", n.args[3] if len(n.args) > 3 else 0)
            out = declare(n)
            w.node("maxpool", [name_of[n.args[0]]], [out], C=xsh[1], H=xsh[2], W=xsh[3], Hout=osh[2], Wout=osh[3],
                   K=k, S=s, P=p)
        elif t in (F.interpolate,):
            if n.kwargs.get("mode", "nearest") != "nearest":
                raise NotImplementedError("interpolate: nearest only")
            xsh, osh = shape(n.args[0]), shape(n)
            out = declare(n)
            w.node("resize_nn", [name_of[n.args[0]]], [out], C=xsh[1], H=xsh[2], W=xsh[3], S=osh[2] // xsh[2])
        elif t in (torch.softmax, F.softmax, "softmax"):
            xsh = shape(n.args[0])
            dim = n.kwargs.get("dim", n.args[1] if len(n.args) > 1 else -1)
            ax = dim + len(xsh) if dim < 0 else dim
            out = declare(n)
            w.node("softmax_axis", [name_of[n.args[0]]], [out], outer=int(np.prod(xsh[:ax])), axdim=xsh[ax],
                   inner=int(np.prod(xsh[ax + 1:])))
        elif t in ("contiguous",) or t is torch.Tensor.contiguous:
            name_of[n] = name_of[n.args[0]]
        else:
            raise NotImplementedError(f"unsupported node {n.format_node()}")

    path = os.path.join(out_dir, plan_name)
    with open(path, "w") as f:
        f.write("\n".join(w.lines) + "\n")
    return path
