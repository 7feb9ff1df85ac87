"""ONNX emission of the five benchmark graphs, in the shape the reference emits them.

The reference front end (C#) turns `[Module]` classes into a concrete ONNX graph
(FastOnnxModelBuilder.BuildInternalOnnxModel, src/Shorokoo/Core/Factory/FastOnnxModelBuilder.cs:165-300)
and hands the serialized bytes to the backend plugin (src/Shorokoo/Core/ComputeContext.cs:199-207).
No .NET runtime exists on this machine, so these builders re-create those graphs from the module
sources, keeping the emission quirks the backend has to accept:

* node names ``N<k>``, value names ``N<k>_T<j>``, graph inputs with rank-only symbolic dims
  (FastOnnxProtoFactory.cs:65-96) and name-only graph outputs (:107-113);
* weights as ``raw_data`` initializers (FastOnnxProtoFactory.cs:120-159);
* runtime shape chains on graph inputs (``Shape -> Gather -> Unsqueeze -> Concat -> Reshape``,
  ``ReduceProd``) because model inputs are never folded upstream (FastProcessors.cs:4691);
* inference-mode FrozenBatchNorm as primitive ``Div/Sqrt/Mul/Sub/Add`` over initializers
  (samples/RetinaNet/ResNet.cs:177-201), ``Identity`` after scalar shape ops;
* ``[Hyper]`` scalars either specialised (folded) or, with ``live_hypers``, emitted as leading graph
  inputs feeding ``If``/``Loop`` nodes (Documentation/inference.md:128-155).

Inputs come from ``numpy.random.Generator(PCG64(seed))``; weights from an independent
``Generator(PCG64(seed + WEIGHT_SEED_OFFSET))`` so that a model's weights do not depend on the
batch size it is built for.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

from . import onnx_writer as W

WEIGHT_SEED_OFFSET = 1000
INT64_MAX = (1 << 63) - 1


@dataclass
class ModelCase:
    """A synthesized model plus its seeded inputs."""
    name: str
    model: bytes
    inputs: List[Tuple[str, np.ndarray]]
    output_names: List[str]
    macs: int                                 # multiply-accumulates of Conv/MatMul nodes
    params: Dict[str, np.ndarray] = field(default_factory=dict)   # torch-style path -> array

    @property
    def flops(self) -> int:
        return 2 * self.macs


class Builder:
    """Emits nodes in the reference's naming style and tracks static shapes for FLOP counting."""

    def __init__(self, weight_seed: int, dead_code: bool = False):
        self.k = 0
        self.nodes: List[W.Node] = []
        self.inits: List[W.Tensor] = []
        self.inputs: List[W.ValueInfo] = []
        self.outputs: List[W.ValueInfo] = []
        self.rng = np.random.Generator(np.random.PCG64(weight_seed))
        self.shape: Dict[str, Tuple[int, ...]] = {}
        self.params: Dict[str, np.ndarray] = {}
        self.macs = 0
        self.dead_code = dead_code
        self.stack: List[List[W.Node]] = [self.nodes]
        # Optional BatchNorm calibration: value name -> activation (torch, NCHW) of a small seeded
        # calibration batch, propagated alongside emission (used by retinanet(calibrate_bn=True)).
        self.calib: Dict[str, object] = {}
        self.params_by_name: Dict[str, np.ndarray] = {}

    # -- raw emission -------------------------------------------------------------------------
    def _next(self) -> int:
        self.k += 1
        return self.k

    def op(self, op_type: str, inputs: Sequence[str], n_out: int = 1, **attrs):
        k = self._next()
        outs = [f"N{k}_T{j}" for j in range(n_out)]
        alist = []
        for a, v in attrs.items():
            if v is None:
                continue
            alist.append(W.Attr(a, v) if not isinstance(v, W.Attr) else v)
        self.stack[-1].append(W.Node(op_type, list(inputs), outs, name=f"N{k}", attrs=alist))
        return outs[0] if n_out == 1 else outs

    def const(self, arr, encoding: str = "typed") -> str:
        arr = np.asarray(arr)
        return self.op("Constant", [], value=W.Tensor("", arr, encoding=encoding))

    def init(self, arr: np.ndarray, path: str = "") -> str:
        k = self._next()
        name = f"N{k}_T0"
        self.inits.append(W.Tensor(name, np.ascontiguousarray(arr), encoding="raw"))
        self.shape[name] = tuple(arr.shape)
        self.params_by_name[name] = arr
        if path:
            self.params[path] = arr
        return name

    def graph_input(self, elem: int, rank: int, shape=None) -> str:
        k = self._next()
        name = f"N{k}_T0"
        self.inputs.append(W.ValueInfo(name, elem, rank=rank, metadata={"InputType": "ReadyInput"}))
        if shape is not None:
            self.shape[name] = tuple(shape)
        return name

    def ident(self, x: str) -> str:
        y = self.op("Identity", [x])
        if x in self.shape:
            self.shape[y] = self.shape[x]
        return y

    # -- shape-chain helpers (Tensor.ShapeTensor()[axis], Vector literals) --------------------
    def dim(self, x: str, axis: int) -> str:
        s = self.op("Shape", [x])
        g = self.op("Gather", [s, self.const(np.array(axis, np.int64))], axis=0)
        return self.ident(g)

    def unsq(self, s: str) -> str:
        return self.ident(self.op("Unsqueeze", [s, self.const(np.array([0], np.int64))]))

    def vec(self, parts: Sequence) -> str:
        """Concat of [1]-vectors; ints become Constant([v])."""
        items = []
        for p in parts:
            if isinstance(p, (int, np.integer)):
                items.append(self.const(np.array([p], np.int64)))
            else:
                items.append(p)
        return self.op("Concat", items, axis=0)

    # -- layers -------------------------------------------------------------------------------
    def conv(self, x: str, w: str, b: Optional[str], kernel: int, stride: int, pads=None,
             auto_pad: str = "NOTSET") -> str:
        n, c, h, wd = self.shape[x]
        cout = self.shape[w][0]
        if auto_pad == "SAME_UPPER":
            ho, wo = -(-h // stride), -(-wd // stride)
        else:
            p = pads or [0, 0, 0, 0]
            ho = (h + p[0] + p[2] - kernel) // stride + 1
            wo = (wd + p[1] + p[3] - kernel) // stride + 1
        inputs = [x, w] + ([b] if b is not None else [])
        y = self.op("Conv", inputs, auto_pad=auto_pad, dilations=[1, 1], group=1,
                    kernel_shape=[kernel, kernel],
                    pads=(pads if auto_pad == "NOTSET" else None), strides=[stride, stride])
        self.shape[y] = (n, cout, ho, wo)
        self.macs += n * ho * wo * cout * c * kernel * kernel
        if x in self.calib:
            import torch
            import torch.nn.functional as F
            xt = self.calib[x]
            if auto_pad == "SAME_UPPER":
                ch, cw = xt.shape[2], xt.shape[3]
                th = max((-(-ch // stride) - 1) * stride + kernel - ch, 0)
                tw = max((-(-cw // stride) - 1) * stride + kernel - cw, 0)
                xt = F.pad(xt, (tw // 2, tw - tw // 2, th // 2, th - th // 2))
            elif pads:
                xt = F.pad(xt, (pads[1], pads[3], pads[0], pads[2]))
            wt = torch.from_numpy(self.params_by_name[w])
            bt = torch.from_numpy(self.params_by_name[b]) if b in self.params_by_name else None
            self.calib[y] = F.conv2d(xt, wt, bt, stride=stride)
        return y

    def unary(self, op: str, x: str) -> str:
        y = self.op(op, [x])
        self.shape[y] = self.shape[x]
        if x in self.calib and op == "Relu":
            self.calib[y] = self.calib[x].clamp_min(0)
        return y

    def binary(self, op: str, a: str, b: str) -> str:
        y = self.op(op, [a, b])
        if a in self.shape and b in self.shape:
            self.shape[y] = tuple(np.broadcast_shapes(self.shape[a], self.shape[b]))
        if a in self.calib and b in self.calib and op == "Add":
            self.calib[y] = self.calib[a] + self.calib[b]
        return y

    def model(self, name: str, functions=()) -> bytes:
        g = W.Graph(name, self.nodes, self.inits, self.inputs, self.outputs)
        return W.Model(g, functions=list(functions)).encode()

    def subgraph(self, name: str, body) -> W.Graph:
        """Builds a nested graph; ``body()`` emits nodes and returns (inputs, outputs)."""
        nodes: List[W.Node] = []
        self.stack.append(nodes)
        try:
            ins, outs = body()
        finally:
            self.stack.pop()
        return W.Graph(name, nodes, [], ins, outs)

    def branch_identity(self, x: str) -> W.Graph:
        """If branch of an eager IfElse: both values are built outside, the branch forwards one
        (src/Shorokoo/Core/Nodes/IfOps.cs:19-23)."""
        def body():
            y = self.op("Identity", [x])
            return [], [W.ValueInfo(y)]
        return self.subgraph(f"br{self.k}", body)

    def if_else(self, cond: str, then_v: str, else_v: str) -> str:
        y = self.op("If", [cond], then_branch=self.branch_identity(then_v),
                    else_branch=self.branch_identity(else_v))
        if then_v in self.shape:
            self.shape[y] = self.shape[then_v]
        return y


# ================================================================================================
# Initialisers (src/Shorokoo.Modules/Initializers/Initializers.cs:113-164)
# ================================================================================================

def _fan_in(shape):
    return int(np.prod(shape[1:]))


def xavier_uniform(rng, shape):
    bound = math.sqrt(6.0 / (_fan_in(shape) + shape[0] * int(np.prod(shape[2:]))))
    return rng.uniform(-bound, bound, size=shape).astype(np.float32)


def kaiming_uniform(rng, shape):
    bound = math.sqrt(6.0 / _fan_in(shape))
    return rng.uniform(-bound, bound, size=shape).astype(np.float32)


def kaiming_normal(rng, shape):
    std = math.sqrt(2.0 / _fan_in(shape))
    return (rng.standard_normal(size=shape, dtype=np.float32) * np.float32(std)).astype(np.float32)


# ================================================================================================
# Config 1: StackedLinear (tests/ReadmeValidation/Modules.cs:6-28)
# ================================================================================================

def stacked_linear(batch: int = 4096, n: int = 1024, depth: int = 8, seed: int = 42,
                   live_depth: bool = False, bias_scale: float = 0.0) -> ModelCase:
    rng_in = np.random.Generator(np.random.PCG64(seed))
    x_val = rng_in.random(size=(batch, n), dtype=np.float32)
    B = Builder(seed + WEIGHT_SEED_OFFSET)
    inputs = []
    if live_depth:
        d_in = B.graph_input(W.INT64, 0)
        inputs.append((d_in, np.array(depth, np.int64)))
    x = B.graph_input(W.FLOAT, 2, (batch, n))
    inputs.append((x, x_val))
    w = B.init(xavier_uniform(B.rng, (n, n)), "w")
    bias = np.zeros(n, np.float32) if bias_scale == 0 else \
        (B.rng.standard_normal(n, dtype=np.float32) * np.float32(bias_scale))
    b = B.init(bias, "b")
    if not live_depth:
        h = x
        for i in range(depth):
            wt = B.op("Transpose", [w], perm=[1, 0])
            B.shape[wt] = (n, n)
            mm = B.op("MatMul", [h, wt])
            B.shape[mm] = (batch, n)
            B.macs += batch * n * n
            z = B.binary("Add", mm, b)
            h = z if i == depth - 1 else B.unary("Relu", z)
        out = h
    else:
        # Loop(M = depth) with the isLast IfElse inside the body (LoopAPI.Iterate, OnnxOp.HZ.cs:20-30).
        def body():
            it = f"L{B.k}_iter"
            cin = f"L{B.k}_cond"
            hin = f"L{B.k}_h"
            wt = B.op("Transpose", [w], perm=[1, 0])
            z = B.op("Add", [B.op("MatMul", [hin, wt]), b])
            nxt = B.op("Add", [it, B.const(np.array(1, np.int64))])
            is_last = B.op("Equal", [nxt, d_in])
            relu = B.op("Relu", [z])
            hout = B.op("If", [is_last], then_branch=B.branch_identity(z),
                        else_branch=B.branch_identity(relu))
            cout = B.op("Identity", [cin])
            return ([W.ValueInfo(it, W.INT64, dims=[]), W.ValueInfo(cin, W.BOOL, dims=[]),
                     W.ValueInfo(hin, W.FLOAT, rank=2)],
                    [W.ValueInfo(cout), W.ValueInfo(hout)])
        g = B.subgraph("loop_body", body)
        out = B.op("Loop", [d_in, "", x], body=g)
        B.macs += depth * batch * n * n
    B.outputs.append(W.ValueInfo(out))
    return ModelCase("stacked_linear", B.model("StackedLinear"), inputs, [out], B.macs, B.params)


# ================================================================================================
# Config 2: untied MLP of Linear layers (src/Shorokoo.Modules/Layers/Linear.cs:25-39)
# ================================================================================================

def linear(B: Builder, x: str, out_features: int, relu: bool, path: str, bias_scale: float = 0.0) -> str:
    """Linear: flatten trailing dims via the runtime shape chain, MatMul(x, W^T) + b."""
    batch = B.dim(x, 0)
    shp = B.op("Shape", [x])
    tail = B.op("Slice", [shp, B.const(np.array([1], np.int64)), B.const(np.array([INT64_MAX], np.int64))])
    in_f = B.ident(B.op("ReduceProd", [tail], keepdims=0))
    flat = B.op("Reshape", [x, B.op("Concat", [B.unsq(batch), B.unsq(in_f)], axis=0)])
    xs = B.shape[x]
    kin = int(np.prod(xs[1:]))
    B.shape[flat] = (xs[0], kin)
    w = B.init(kaiming_uniform(B.rng, (out_features, kin)), path + ".weight")
    wt = B.op("Transpose", [w], perm=[1, 0])
    mm = B.op("MatMul", [flat, wt])
    B.shape[mm] = (xs[0], out_features)
    B.macs += xs[0] * kin * out_features
    bias = np.zeros(out_features, np.float32) if bias_scale == 0 else \
        B.rng.standard_normal(out_features, dtype=np.float32) * np.float32(bias_scale)
    b = B.init(bias, path + ".bias")
    y = B.binary("Add", mm, b)
    return B.unary("Relu", y) if relu else y


def mlp(batch: int = 8192, widths: Sequence[int] = (1024, 4096, 4096, 4096, 4096, 4096, 1000),
        seed: int = 1, bias_scale: float = 0.0) -> ModelCase:
    rng_in = np.random.Generator(np.random.PCG64(seed))
    x_val = rng_in.standard_normal(size=(batch, widths[0]), dtype=np.float32)
    B = Builder(seed + WEIGHT_SEED_OFFSET)
    x = B.graph_input(W.FLOAT, 2, (batch, widths[0]))
    h = x
    for i, wdt in enumerate(widths[1:]):
        h = linear(B, h, wdt, relu=(i < len(widths) - 2), path=f"layers.{i}", bias_scale=bias_scale)
    B.outputs.append(W.ValueInfo(h))
    return ModelCase("mlp", B.model("MLP"), [(x, x_val)], [h], B.macs, B.params)


# ================================================================================================
# Configs 3-5: ResNet-18 / ResNet-50 / RetinaNet (samples/RetinaNet/ResNet.cs, RetinaNetDetector.cs)
# ================================================================================================

@dataclass
class ResNetOpts:
    eps_input: Optional[str] = None         # live bnEps graph input, else folded constant
    eps: float = 1e-5
    calibrate_bn: bool = False              # running stats from the calibration batch (tests only)
    bn_affine_scale: float = 0.0            # >0 draws gamma/beta around 1/0 (tests only)


def frozen_bn(B: Builder, x: str, path: str, o: ResNetOpts) -> str:
    """FrozenBatchNorm (ResNet.cs:177-201): scale = w / sqrt(var + eps); shift = b - mean*scale;
    y = x*scale + shift, params reshaped to [1, C, 1, 1] through a runtime Shape chain."""
    c_dim = B.dim(x, 1)
    C = B.shape[x][1]
    rng = B.rng
    mean = (rng.standard_normal(C, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
    var = rng.uniform(0.5, 1.5, size=C).astype(np.float32)
    if x in B.calib and o.calibrate_bn:   # frozen statistics of the calibration batch
        xt = B.calib[x]
        mean = xt.mean(dim=(0, 2, 3)).numpy().astype(np.float32)
        var = (xt.var(dim=(0, 2, 3), unbiased=False) + 1e-3).numpy().astype(np.float32)
    if o.bn_affine_scale > 0:
        gamma = (1.0 + o.bn_affine_scale * rng.standard_normal(C)).astype(np.float32)
        beta = (o.bn_affine_scale * rng.standard_normal(C)).astype(np.float32)
    else:
        gamma = np.ones(C, np.float32)
        beta = np.zeros(C, np.float32)
    rm = B.init(mean, path + ".running_mean")
    rv = B.init(var, path + ".running_var")
    wt = B.init(gamma, path + ".weight")
    bs = B.init(beta, path + ".bias")
    shp = B.vec([1, B.unsq(c_dim), 1, 1])
    r_mean = B.op("Reshape", [rm, shp])
    r_var = B.op("Reshape", [rv, shp])
    r_w = B.op("Reshape", [wt, shp])
    r_b = B.op("Reshape", [bs, shp])
    eps = o.eps_input if o.eps_input is not None else B.const(np.array(o.eps, np.float32))
    scale = B.op("Div", [r_w, B.op("Sqrt", [B.op("Add", [r_var, eps])])])
    shift = B.op("Sub", [r_b, B.op("Mul", [r_mean, scale])])
    y = B.op("Add", [B.op("Mul", [x, scale]), shift])
    B.shape[y] = B.shape[x]
    if x in B.calib:
        import torch
        sc = gamma / np.sqrt(var + np.float32(o.eps))
        sh = beta - mean * sc
        B.calib[y] = B.calib[x] * torch.from_numpy(sc).view(1, -1, 1, 1) + torch.from_numpy(sh).view(1, -1, 1, 1)
    return y


def resnet_conv(B: Builder, x: str, filters: int, k: int, s: int, path: str) -> str:
    """Conv2Dk{k}{k}s{s}{s} (ResNet.cs:204-277): Kaiming-normal W, VectorFill(filters, 0) bias."""
    cin = B.shape[x][1]
    w = B.init(kaiming_normal(B.rng, (filters, cin, k, k)), path + ".weight")
    bias = B.op("ConstantOfShape", [B.const(np.array([filters], np.int64))],
                value=W.Tensor("", np.array([0.0], np.float32), encoding="raw"))
    pad = 0 if k == 1 else (1 if k == 3 else 0)
    return B.conv(x, w, bias, k, s, pads=[pad, pad, pad, pad])


def bottleneck(B: Builder, x: str, filters: int, stride: int, downsample: bool, path: str,
               o: ResNetOpts) -> str:
    """BottleneckS11/S22 (ResNet.cs:280-357): stride on the 3x3, projection shortcut when downsample."""
    c1 = B.unary("Relu", frozen_bn(B, resnet_conv(B, x, filters, 1, 1, path + ".conv1"), path + ".bn1", o))
    c2 = B.unary("Relu", frozen_bn(B, resnet_conv(B, c1, filters, 3, stride, path + ".conv2"), path + ".bn2", o))
    c3 = frozen_bn(B, resnet_conv(B, c2, 4 * filters, 1, 1, path + ".conv3"), path + ".bn3", o)
    if downsample:
        sc = resnet_conv(B, x, 4 * filters, 1, stride, path + ".downsample.0")
        sc = frozen_bn(B, sc, path + ".downsample.1", o)
    else:
        if B.dead_code:   # the unused shortcut branch the eager IfElse built (ResNet.cs:297-299)
            dead = resnet_conv(B, x, 4 * filters, 1, stride, path + ".dead_shortcut")
            frozen_bn(B, dead, path + ".dead_shortcut_bn", o)
        sc = x
    return B.unary("Relu", B.binary("Add", c3, sc))


def basic_block(B: Builder, x: str, filters: int, stride: int, downsample: bool, path: str,
                o: ResNetOpts) -> str:
    """BasicBlockS11/S22 (ResNet.cs:442-481)."""
    c1 = B.unary("Relu", frozen_bn(B, resnet_conv(B, x, filters, 3, stride, path + ".conv1"), path + ".bn1", o))
    c2 = frozen_bn(B, resnet_conv(B, c1, filters, 3, 1, path + ".conv2"), path + ".bn2", o)
    if downsample:
        sc = frozen_bn(B, resnet_conv(B, x, filters, 1, stride, path + ".downsample.0"), path + ".downsample.1", o)
    else:
        if B.dead_code:
            dead = resnet_conv(B, x, filters, 1, stride, path + ".dead_shortcut")
            frozen_bn(B, dead, path + ".dead_shortcut_bn", o)
        sc = x
    return B.unary("Relu", B.binary("Add", c2, sc))


def stem(B: Builder, x: str, o: ResNetOpts) -> str:
    """ResNetStem (ResNet.cs:360-372): explicit Pad(3) -> Conv7x7/2 (pads 0) -> BN -> Relu -> MaxPool 3x3/2 p1."""
    pads = B.const(np.array([0, 0, 3, 3, 0, 0, 3, 3], np.int64))
    xp = B.op("Pad", [x, pads, B.const(np.array(0.0, np.float32))], mode="constant")
    n, c, h, w = B.shape[x]
    B.shape[xp] = (n, c, h + 6, w + 6)
    if x in B.calib:
        import torch.nn.functional as F
        B.calib[xp] = F.pad(B.calib[x], (3, 3, 3, 3))
    y = B.unary("Relu", frozen_bn(B, resnet_conv(B, xp, 64, 7, 2, "conv1"), "bn1", o))
    mp = B.op("MaxPool", [y], ceil_mode=0, dilations=[1, 1], kernel_shape=[3, 3], pads=[1, 1, 1, 1],
              storage_order=0, strides=[2, 2])
    n, c, h, w = B.shape[y]
    B.shape[mp] = (n, c, (h + 2 - 3) // 2 + 1, (w + 2 - 3) // 2 + 1)
    if y in B.calib:
        import torch.nn.functional as F
        B.calib[mp] = F.max_pool2d(B.calib[y], 3, 2, 1)
    return mp


def classification_head(B: Builder, x: str, num_classes: int, o: ResNetOpts,
                        include_top, apply_softmax) -> str:
    """ClassificationHead (ResNet.cs:374-388) + DenseBasic (:102-125): GAP, flatten, MatMul(W^T)+b."""
    g = B.op("GlobalAveragePool", [x])
    n, c, _, _ = B.shape[x]
    B.shape[g] = (n, c, 1, 1)
    batch = B.dim(g, 0)
    shp = B.op("Shape", [g])
    tail = B.op("Slice", [shp, B.const(np.array([1], np.int64)), B.const(np.array([INT64_MAX], np.int64))])
    in_f = B.ident(B.op("ReduceProd", [tail], keepdims=0))
    flat = B.op("Reshape", [g, B.op("Concat", [B.unsq(batch), B.unsq(in_f)], axis=0)])
    w = B.init((B.rng.standard_normal((num_classes, c), dtype=np.float32) * np.float32(0.02)).astype(np.float32),
               "fc.weight")
    wt = B.op("Transpose", [w], perm=[1, 0])
    mm = B.op("MatMul", [flat, wt])
    B.macs += n * c * num_classes
    fc_bias = np.zeros(num_classes, np.float32) if o.bn_affine_scale == 0 else \
        (o.bn_affine_scale * B.rng.standard_normal(num_classes)).astype(np.float32)
    b = B.init(fc_bias, "fc.bias")
    top = B.op("Add", [mm, b])
    B.shape[top] = (n, num_classes)
    if isinstance(apply_softmax, str):
        sm = B.op("Softmax", [top], axis=-1)
        top = B.if_else(apply_softmax, sm, top)
    elif apply_softmax:
        top = B.op("Softmax", [top], axis=-1)
    B.shape[top] = (n, num_classes)
    if isinstance(include_top, str):
        return B.if_else(include_top, top, g)
    return top if include_top else g


def _resnet_inputs(B: Builder, live: bool, num_classes: int, x_shape, x_elem: int = W.FLOAT):
    """Hyper inputs come first when not specialised (RealCheckpointPredictionTests.cs:29-37)."""
    o = ResNetOpts()
    hyper_vals = []
    include_top, apply_softmax = True, False
    if live:
        nc = B.graph_input(W.INT64, 0)
        mom = B.graph_input(W.FLOAT, 0)
        eps = B.graph_input(W.FLOAT, 0)
        it = B.graph_input(W.BOOL, 0)
        sm = B.graph_input(W.BOOL, 0)
        hyper_vals = [(nc, np.array(num_classes, np.int64)), (mom, np.array(0.9, np.float32)),
                      (eps, np.array(1e-5, np.float32)), (it, np.array(True)), (sm, np.array(False))]
        o.eps_input = eps
        include_top, apply_softmax = it, sm
    x = B.graph_input(x_elem, 4, x_shape)
    return x, o, hyper_vals, include_top, apply_softmax


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """float32 values rounded to bfloat16 / float16 (nearest even), still as float32."""
    if dtype == "float16":
        return x.astype(np.float16).astype(np.float32)
    if dtype == "bfloat16":
        u = np.ascontiguousarray(x, np.float32).view(np.uint32)
        r = ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000))
        return r.view(np.float32)
    return x


def resnet(depth: int = 50, batch: int = 512, hw: Tuple[int, int] = (224, 224), seed: int = 11,
           num_classes: int = 1000, live_hypers: bool = False, dead_code: bool = False,
           affine_scale: float = 0.0, apply_softmax: Optional[bool] = None,
           include_top: Optional[bool] = None, input_dtype: str = "float32") -> ModelCase:
    """``input_dtype`` "bfloat16" / "float16": the image arrives as a 16-bit float tensor (a caller's
    CreateTensor<BFloat16 / Float16>) and a Cast to float32 feeds the stem; the case's input array
    holds the 16-bit values widened to float32."""
    rng_in = np.random.Generator(np.random.PCG64(seed))
    x_val = rng_in.standard_normal(size=(batch, 3, hw[0], hw[1]), dtype=np.float32)
    B = Builder(seed + WEIGHT_SEED_OFFSET, dead_code=dead_code)
    x, o, hyper_vals, inc_top, app_sm = _resnet_inputs(B, live_hypers, num_classes, x_val.shape,
                                                       {"float32": W.FLOAT, "bfloat16": W.BFLOAT16,
                                                        "float16": W.FLOAT16}[input_dtype])
    x_in = x
    if input_dtype != "float32":
        x_val = round_to(x_val, input_dtype)
        x = B.op("Cast", [x_in], to=W.FLOAT)
        B.shape[x] = x_val.shape
    o.bn_affine_scale = affine_scale
    if apply_softmax is not None:
        if live_hypers:
            hyper_vals[4] = (hyper_vals[4][0], np.array(bool(apply_softmax)))
        else:
            app_sm = apply_softmax
    if include_top is not None:
        if live_hypers:
            hyper_vals[3] = (hyper_vals[3][0], np.array(bool(include_top)))
        else:
            inc_top = include_top
    h = stem(B, x, o)
    if depth == 50:
        for li, (f, nb) in enumerate([(64, 3), (128, 4), (256, 6), (512, 3)]):
            for bi in range(nb):
                s = 2 if (li > 0 and bi == 0) else 1
                h = bottleneck(B, h, f, s, bi == 0, f"layer{li + 1}.{bi}", o)
    elif depth == 18:
        for li, f in enumerate([64, 128, 256, 512]):
            for bi in range(2):
                s = 2 if (li > 0 and bi == 0) else 1
                h = basic_block(B, h, f, s, li > 0 and bi == 0, f"layer{li + 1}.{bi}", o)
    else:
        raise ValueError(depth)
    out = classification_head(B, h, num_classes, o, inc_top, app_sm)
    B.outputs.append(W.ValueInfo(out))
    inputs = hyper_vals + [(x_in, x_val)]
    return ModelCase(f"resnet{depth}", B.model(f"ResNet{depth}"), inputs, [out], B.macs, B.params)


def kaiming_uniform_a1(rng, shape):
    """Kaiming-uniform with negative slope a=1: U(-b, b), b = sqrt(3 / fan_in) (torchvision's FPN init)."""
    bound = math.sqrt(3.0 / _fan_in(shape))
    return rng.uniform(-bound, bound, size=shape).astype(np.float32)


def head_normal(rng, shape):
    """N(0, 0.01^2): torchvision's RetinaNet head-conv init."""
    return (rng.standard_normal(size=shape, dtype=np.float32) * np.float32(0.01)).astype(np.float32)


def ret_conv(B: Builder, x: str, filters: int, k: int, stride: int, path: str,
             bias_value: float = 0.0, bias_scale: float = 0.0, normalize_input: bool = False) -> str:
    """RetConv1x1 / RetConv3x3 / RetConv3x3Stride2 (RetinaNetDetector.cs:282-334): trainable bias,
    3x3 convs use auto_pad SAME_UPPER (asymmetric pads on even inputs)."""
    cin = B.shape[x][1]
    wv = kaiming_uniform_a1(B.rng, (filters, cin, k, k))
    if normalize_input and x in B.calib:   # data-dependent scale: unit-variance lateral outputs
        wv = (wv / np.float32(float(B.calib[x].std()))).astype(np.float32)
    w = B.init(wv, path + ".weight")
    bias = np.full(filters, bias_value, np.float32)
    if bias_scale:
        bias = bias + (bias_scale * B.rng.standard_normal(filters)).astype(np.float32)
    b = B.init(bias, path + ".bias")
    if k == 1:
        return B.conv(x, w, b, 1, stride, pads=[0, 0, 0, 0])
    return B.conv(x, w, b, k, stride, auto_pad="SAME_UPPER")


class _SharedConv:
    """A conv whose initializers are created once and reused at every pyramid level."""

    def __init__(self, B: Builder, cin: int, filters: int, path: str, bias_value=0.0, bias_scale=0.0, init=None):
        self.w = B.init((init or head_normal)(B.rng, (filters, cin, 3, 3)), path + ".weight")
        bias = np.full(filters, bias_value, np.float32)
        if bias_scale:
            bias = bias + (bias_scale * B.rng.standard_normal(filters)).astype(np.float32)
        self.b = B.init(bias, path + ".bias")

    def __call__(self, B: Builder, x: str) -> str:
        return B.conv(x, self.w, self.b, 3, 1, auto_pad="SAME_UPPER")


class _GroupNormParams:
    """gamma / beta of one RetGroupNorm: ones / zeros (RetInitSimple :41-50, RetInitZeros :67-76),
    perturbed by ``affine_scale`` for the parity tests; created once per head position and shared
    by every pyramid level, like the head's convs (one head instance is called on each level)."""

    def __init__(self, B: Builder, c: int, path: str, affine_scale: float = 0.0):
        gv = np.ones(c, np.float32)
        bv = np.zeros(c, np.float32)
        if affine_scale:
            gv = gv + (affine_scale * B.rng.standard_normal(c)).astype(np.float32)
            bv = bv + (affine_scale * B.rng.standard_normal(c)).astype(np.float32)
        self.c = c
        self.gamma = B.init(gv, path + ".weight")
        self.beta = B.init(bv, path + ".bias")


def group_norm(B: Builder, x: str, num_groups: int, params: _GroupNormParams) -> str:
    """RetGroupNorm (RetinaNetDetector.cs:337-372) as the exporter writes it: x [B, C, H, W] reshaped
    to [B, G, C/G, H, W] through a runtime shape chain, ReduceMean over axes 2-4 (keepdims), the
    biased variance as the mean of (x - mean) * (x - mean) (two Sub nodes, as the module writes
    the difference twice), (x - mean) / Sqrt(var + 1e-5), reshaped back, times gamma reshaped to
    [1, C, 1, 1] plus beta reshaped to [1, C, 1, 1]."""
    n, c, hh, ww = B.shape[x]
    bsz, hd, wd = B.dim(x, 0), B.dim(x, 2), B.dim(x, 3)
    xr = B.op("Reshape", [x, B.vec([B.unsq(bsz), num_groups, c // num_groups, B.unsq(hd), B.unsq(wd)])])
    B.shape[xr] = (n, num_groups, c // num_groups, hh, ww)
    axes = B.const(np.array([2, 3, 4], np.int64))
    mean = B.op("ReduceMean", [xr, axes], keepdims=1)
    B.shape[mean] = (n, num_groups, 1, 1, 1)
    d1, d2 = B.binary("Sub", xr, mean), B.binary("Sub", xr, mean)
    var = B.op("ReduceMean", [B.binary("Mul", d1, d2), axes], keepdims=1)
    B.shape[var] = (n, num_groups, 1, 1, 1)
    eps = B.const(np.array(1e-5, np.float32))
    B.shape[eps] = ()
    den = B.unary("Sqrt", B.binary("Add", var, eps))
    norm = B.binary("Div", B.binary("Sub", xr, mean), den)
    y = B.op("Reshape", [norm, B.vec([B.unsq(bsz), c, B.unsq(hd), B.unsq(wd)])])
    B.shape[y] = (n, c, hh, ww)
    four = B.const(np.array([1, c, 1, 1], np.int64))
    gamma = B.op("Reshape", [params.gamma, four])
    beta = B.op("Reshape", [params.beta, four])
    B.shape[gamma] = B.shape[beta] = (1, c, 1, 1)
    return B.binary("Add", B.binary("Mul", y, gamma), beta)


def retinanet(batch: int = 16, hw: Tuple[int, int] = (800, 1024), seed: int = 13, num_classes: int = 80,
              num_anchors: int = 9, fpn: int = 256, sigmoid: bool = True, affine_scale: float = 0.0,
              backbone_widths: Sequence[int] = (64, 128, 256, 512),
              backbone_blocks: Sequence[int] = (3, 4, 6, 3), calibrate_bn: bool = False,
              norm_heads: bool = False, num_groups: int = 32) -> ModelCase:
    """RetinaNetResNet50NoNorm (RetinaNetDetector.cs:828-886) + Sigmoid on the class output; with
    ``norm_heads`` RetinaNetResNet50 (:957-971): the same backbone and FPN with the GroupNorm heads
    RetClassificationHeadWithNorm / RetRegressionHeadWithNorm (:492-536, :578-642), each of the four
    tower convs followed by RetGroupNorm (``num_groups`` groups of the 256 channels) and ReLU.

    The class-head bias starts at -ln(99) (focal-loss prior 0.01, RetInitClsBias :79-99). FPN convs are
    Kaiming-uniform(a=1) and head convs N(0, 0.01^2), the initialisation of the torchvision RetinaNet
    the sample mirrors; the sample's own constant 0.02 fill (RetInitXavier :53-61) would make every
    output channel identical. With ``calibrate_bn`` the backbone's frozen BatchNorm statistics are the
    per-channel mean/variance of a seeded 2x3x128x128 calibration batch (the state a trained detector's
    frozen BN carries); uncalibrated statistics let the un-normalised residual stream grow by orders
    of magnitude, which turns the sigmoid outputs into a sign test on logits near zero."""
    rng_in = np.random.Generator(np.random.PCG64(seed))
    x_val = rng_in.standard_normal(size=(batch, 3, hw[0], hw[1]), dtype=np.float32)
    B = Builder(seed + WEIGHT_SEED_OFFSET)
    o = ResNetOpts(bn_affine_scale=affine_scale, calibrate_bn=calibrate_bn)
    x = B.graph_input(W.FLOAT, 4, x_val.shape)
    if True:   # seeded calibration batch: FPN input scales (and BN statistics with calibrate_bn)
        import torch
        cal = np.random.Generator(np.random.PCG64(seed + 2 * WEIGHT_SEED_OFFSET))
        B.calib[x] = torch.from_numpy(cal.standard_normal((2, 3, 128, 128), dtype=np.float32))
    h = stem(B, x, o)
    feats = []
    for li, (f, nb) in enumerate(zip(backbone_widths, backbone_blocks)):
        for bi in range(nb):
            s = 2 if (li > 0 and bi == 0) else 1
            h = bottleneck(B, h, f, s, bi == 0, f"backbone.layer{li + 1}.{bi}", o)
        feats.append(h)
    c3, c4, c5 = feats[1], feats[2], feats[3]
    # FPN (RetFeaturePyramidNetworkFull, :401-450)
    p5_1 = ret_conv(B, c5, fpn, 1, 1, "fpn.inner5", bias_scale=affine_scale, normalize_input=True)
    p4_1 = ret_conv(B, c4, fpn, 1, 1, "fpn.inner4", bias_scale=affine_scale, normalize_input=True)
    p3_1 = ret_conv(B, c3, fpn, 1, 1, "fpn.inner3", bias_scale=affine_scale, normalize_input=True)

    def up2(v):   # RetUpsampleNearest (:375-384): Resize nearest, scales [1,1,2,2], default attrs
        y = B.op("Resize", [v, "", B.const(np.array([1.0, 1.0, 2.0, 2.0], np.float32))], mode="nearest")
        n, c, hh, ww = B.shape[v]
        B.shape[y] = (n, c, 2 * hh, 2 * ww)
        return y

    p4 = B.binary("Add", p4_1, up2(p5_1))
    p3s = B.binary("Add", p3_1, up2(p4))
    p5 = ret_conv(B, p5_1, fpn, 3, 1, "fpn.layer5", bias_scale=affine_scale)
    p4 = ret_conv(B, p4, fpn, 3, 1, "fpn.layer4", bias_scale=affine_scale)
    p3 = ret_conv(B, p3s, fpn, 3, 1, "fpn.layer3", bias_scale=affine_scale)
    p6 = ret_conv(B, p5, fpn, 3, 2, "fpn.p6", bias_scale=affine_scale)
    p7 = ret_conv(B, B.unary("Relu", p6), fpn, 3, 2, "fpn.p7", bias_scale=affine_scale)
    levels = [p3, p4, p5, p6, p7]
    # Shared heads (RetClassificationHead :539-571, RetRegressionHead :644-680)
    cls_convs = [_SharedConv(B, fpn, fpn, f"cls.conv{i}", bias_scale=affine_scale, init=kaiming_normal)
                 for i in range(4)]
    cls_out = _SharedConv(B, fpn, num_anchors * num_classes, "cls.logits",
                          bias_value=-math.log(99.0), bias_scale=affine_scale)
    reg_convs = [_SharedConv(B, fpn, fpn, f"reg.conv{i}", bias_scale=affine_scale, init=kaiming_normal)
                 for i in range(4)]
    reg_out = _SharedConv(B, fpn, num_anchors * 4, "reg.deltas", bias_scale=affine_scale)

    cls_norms = [_GroupNormParams(B, fpn, f"cls.norm{i}", affine_scale) for i in range(4)] if norm_heads else None
    reg_norms = [_GroupNormParams(B, fpn, f"reg.norm{i}", affine_scale) for i in range(4)] if norm_heads else None

    def head(feat, convs, final, k, norms):
        v = feat
        for i, c in enumerate(convs):
            v = c(B, v)
            if norms:
                v = group_norm(B, v, num_groups, norms[i])
            v = B.unary("Relu", v)
        v = final(B, v)
        n, _, hh, ww = B.shape[v]
        bsz, hd, wd = B.dim(v, 0), B.dim(v, 2), B.dim(v, 3)
        r = B.op("Reshape", [v, B.vec([B.unsq(bsz), num_anchors, k, B.unsq(hd), B.unsq(wd)])])
        t = B.op("Transpose", [r], perm=[0, 3, 4, 1, 2])
        B.shape[t] = (n, hh, ww, num_anchors, k)
        return t

    cls = [head(p, cls_convs, cls_out, num_classes, cls_norms) for p in levels]
    reg = [head(p, reg_convs, reg_out, 4, reg_norms) for p in levels]
    bsz = B.dim(cls[0], 0)
    cls = [B.op("Reshape", [c, B.vec([B.unsq(bsz), -1, num_classes])]) for c in cls]
    reg = [B.op("Reshape", [r, B.vec([B.unsq(bsz), -1, 4])]) for r in reg]
    classifications = B.op("Concat", cls, axis=1)
    regressions = B.op("Concat", reg, axis=1)
    if sigmoid:
        classifications = B.op("Sigmoid", [classifications])
    B.outputs += [W.ValueInfo(classifications), W.ValueInfo(regressions)]
    name = "RetinaNetResNet50" if norm_heads else "RetinaNetResNet50NoNorm"
    return ModelCase("retinanet_gn" if norm_heads else "retinanet", B.model(name), [(x, x_val)],
                     [classifications, regressions], B.macs, B.params)


# ================================================================================================
# Adjacent model: Vision Transformer (samples/RetinaNet/ViTNet.cs)
# ================================================================================================

VIT_VARIANTS = {   # embed_dim, heads, layers, mlp_dim (ViTTiny :310-353, ViTSmall :361-392, ViTBase :403-434)
    "tiny": (192, 3, 12, 768),
    "small": (384, 6, 12, 1536),
    "base": (768, 12, 12, 3072),
}


def _vit_linear(B: Builder, x: str, w: str, b: str, rows: int, k: int, n: int) -> str:
    """ViTLinear / the attention and MLP projections: MatMul(x, W [in, out]) + b."""
    y = B.op("MatMul", [x, w])
    shp = B.shape[x]
    B.shape[y] = tuple(shp[:-1]) + (n,)
    B.macs += rows * k * n
    return B.binary("Add", y, b)


class _ViTLayerNormParams:
    def __init__(self, B: Builder, d: int, path: str, affine_scale: float):
        gv = np.ones(d, np.float32)
        bv = np.zeros(d, np.float32)
        if affine_scale:
            gv = gv + (affine_scale * B.rng.standard_normal(d)).astype(np.float32)
            bv = bv + (affine_scale * B.rng.standard_normal(d)).astype(np.float32)
        self.gamma = B.init(gv, path + ".weight")
        self.beta = B.init(bv, path + ".bias")


def vit_layer_norm(B: Builder, x: str, p: _ViTLayerNormParams, eps: float) -> str:
    """ViTLayerNorm (ViTNet.cs:51-72): mean over the last axis (keepdims), the biased variance as the
    mean of Pow(x - mean, 2), (x - mean) / Sqrt(var + eps) (the difference written twice), times
    gamma plus beta."""
    axes = B.const(np.array([-1], np.int64))
    shp = B.shape[x]
    mean = B.op("ReduceMean", [x, axes], keepdims=1)
    B.shape[mean] = tuple(shp[:-1]) + (1,)
    two = B.const(np.array(2.0, np.float32))
    B.shape[two] = ()
    var = B.op("ReduceMean", [B.binary("Pow", B.binary("Sub", x, mean), two), axes], keepdims=1)
    B.shape[var] = B.shape[mean]
    eps_c = B.const(np.array(eps, np.float32))
    B.shape[eps_c] = ()
    den = B.unary("Sqrt", B.binary("Add", var, eps_c))
    y = B.binary("Div", B.binary("Sub", x, mean), den)
    B.shape[p.gamma] = B.shape[p.beta] = (shp[-1],)
    return B.binary("Add", B.binary("Mul", y, p.gamma), p.beta)


def vit(variant: str = "base", batch: int = 1, hw: Tuple[int, int] = (224, 224), seed: int = 17,
        num_classes: int = 1000, apply_softmax: bool = False, affine_scale: float = 0.0, layers: Optional[int] = None,
        patch: int = 16) -> ModelCase:
    """ViTTiny / ViTSmall / ViTBase (ViTNet.cs:310-434), batch 1 as the module's graph allows (the
    [1, 1, D] class token is concatenated to the patch sequence without a batch broadcast).

    Patch embedding (ViTPatchEmbed :80-118): Conv 16x16 / 16 -> Reshape [B, D, P] -> Transpose
    [0, 2, 1]; class token and positional embedding (initializers); the transformer block
    (ViTTransformerBlock :247-268) applied ``layers`` times with tied weights (the block model is
    called inside LoopAPI.Iterate, like StackedLinear; the Loop is unrolled at export): pre-norm
    LayerNorm -> ViTAttention (:155-207: QKV MatMul + bias, Reshape [B, S, 3, H, hd], Transpose
    [2, 0, 3, 1, 4], Slice + Squeeze per Q / K / V, Q MatMul Transpose(K) times 1 / sqrt(hd),
    Softmax(-1), MatMul V, Transpose [0, 2, 1, 3], Reshape [B, S, D], projection MatMul + bias) ->
    residual Add -> LayerNorm -> ViTMlp (:217-239: MatMul + bias, Gelu(approximate="tanh"), MatMul +
    bias) -> residual Add; final LayerNorm; ViTClassHead (:275-297: Slice of the class token, Reshape
    [B, D], MatMul + bias, Softmax when apply_softmax).

    Weights: the sample's ViTInitSimple fills every parameter with 1.0, which makes all channels
    identical; these are random instead (projections Xavier-uniform, patch conv N(0, 0.02^2), class
    token and positions N(0, 0.02^2), LayerNorm gamma 1 / beta 0, biases zero unless
    ``affine_scale`` perturbs them)."""
    D, H, L, M = VIT_VARIANTS[variant]
    if layers is not None:
        L = layers
    hd = D // H
    rng_in = np.random.Generator(np.random.PCG64(seed))
    x_val = rng_in.standard_normal(size=(batch, 3, hw[0], hw[1]), dtype=np.float32)
    B = Builder(seed + WEIGHT_SEED_OFFSET)
    x = B.graph_input(W.FLOAT, 4, x_val.shape)
    eps = 1e-6

    def bias(n, path):
        v = np.zeros(n, np.float32) if not affine_scale else \
            (affine_scale * B.rng.standard_normal(n)).astype(np.float32)
        return B.init(v, path)

    # patch embedding
    pw = B.init((0.02 * B.rng.standard_normal((D, 3, patch, patch))).astype(np.float32), "patch_embed.weight")
    pb = bias(D, "patch_embed.bias")
    pe = B.op("Conv", [x, pw, pb], auto_pad="NOTSET", dilations=[1, 1], group=1, kernel_shape=[patch, patch],
              pads=[0, 0, 0, 0], strides=[patch, patch])
    gh, gw = hw[0] // patch, hw[1] // patch
    B.shape[pe] = (batch, D, gh, gw)
    B.macs += batch * D * gh * gw * 3 * patch * patch
    bsz, h_, w_ = B.dim(x, 0), B.dim(x, 2), B.dim(x, 3)
    ps = B.const(np.array(patch, np.int64))
    npatch = B.ident(B.op("Mul", [B.op("Div", [h_, ps]), B.op("Div", [w_, ps])]))
    fl = B.op("Reshape", [pe, B.vec([B.unsq(bsz), D, B.unsq(npatch)])])
    B.shape[fl] = (batch, D, gh * gw)
    tok = B.op("Transpose", [fl], perm=[0, 2, 1])
    S = gh * gw + 1
    B.shape[tok] = (batch, gh * gw, D)
    cls = B.init((0.02 * B.rng.standard_normal((1, 1, D))).astype(np.float32), "cls_token")
    if variant != "tiny":   # ViTSmall / ViTBase tile the token by [1, 1, 1]
        cls = B.op("Tile", [cls, B.const(np.array([1, 1, 1], np.int64))])
    B.shape[cls] = (1, 1, D)
    h = B.op("Concat", [cls, tok], axis=1)
    B.shape[h] = (batch, S, D)
    pos = B.init((0.02 * B.rng.standard_normal((1, S, D))).astype(np.float32), "pos_embed")
    B.shape[pos] = (1, S, D)
    h = B.binary("Add", h, pos)
    # one set of block weights (tied across the iterations)
    ln1 = _ViTLayerNormParams(B, D, "block.norm1", affine_scale)
    ln2 = _ViTLayerNormParams(B, D, "block.norm2", affine_scale)
    wqkv = B.init(xavier_uniform(B.rng, (D, 3 * D)), "block.attn.qkv.weight")
    bqkv = bias(3 * D, "block.attn.qkv.bias")
    wproj = B.init(xavier_uniform(B.rng, (D, D)), "block.attn.proj.weight")
    bproj = bias(D, "block.attn.proj.bias")
    w1 = B.init(xavier_uniform(B.rng, (D, M)), "block.mlp.fc1.weight")
    b1 = bias(M, "block.mlp.fc1.bias")
    w2 = B.init(xavier_uniform(B.rng, (M, D)), "block.mlp.fc2.weight")
    b2 = bias(D, "block.mlp.fc2.bias")
    scale = B.ident(B.op("Div", [B.const(np.array(1.0, np.float32)),
                                 B.op("Sqrt", [B.op("Cast", [B.const(np.array(hd, np.int64))], to=W.FLOAT)])]))
    B.shape[scale] = ()
    big = np.iinfo(np.int32).max
    rows = batch * S
    for _ in range(L):
        n1 = vit_layer_norm(B, h, ln1, eps)
        qkv = _vit_linear(B, n1, wqkv, bqkv, rows, D, 3 * D)
        sb, ss = B.dim(n1, 0), B.dim(n1, 1)
        r5 = B.op("Reshape", [qkv, B.vec([B.unsq(sb), B.unsq(ss), 3, H, hd])])
        B.shape[r5] = (batch, S, 3, H, hd)
        t5 = B.op("Transpose", [r5], perm=[2, 0, 3, 1, 4])
        B.shape[t5] = (3, batch, H, S, hd)
        parts = []
        for i in range(3):
            sl = B.op("Slice", [t5, B.const(np.array([i, 0, 0, 0, 0], np.int64)),
                                B.const(np.array([i + 1, big, big, big, big], np.int64))])
            sq = B.op("Squeeze", [sl, B.const(np.array([0], np.int64))])
            B.shape[sq] = (batch, H, S, hd)
            parts.append(sq)
        q, k, v = parts
        kt = B.op("Transpose", [k], perm=[0, 1, 3, 2])
        B.shape[kt] = (batch, H, hd, S)
        sc = B.op("MatMul", [q, kt])
        B.shape[sc] = (batch, H, S, S)
        B.macs += batch * H * S * S * hd
        sc = B.binary("Mul", sc, scale)
        att = B.op("Softmax", [sc], axis=-1)
        B.shape[att] = (batch, H, S, S)
        ctx = B.op("MatMul", [att, v])
        B.shape[ctx] = (batch, H, S, hd)
        B.macs += batch * H * S * S * hd
        ctx = B.op("Transpose", [ctx], perm=[0, 2, 1, 3])
        B.shape[ctx] = (batch, S, H, hd)
        ctx = B.op("Reshape", [ctx, B.vec([B.unsq(sb), B.unsq(ss), D])])
        B.shape[ctx] = (batch, S, D)
        h = B.binary("Add", h, _vit_linear(B, ctx, wproj, bproj, rows, D, D))
        n2 = vit_layer_norm(B, h, ln2, eps)
        f1 = _vit_linear(B, n2, w1, b1, rows, D, M)
        g = B.op("Gelu", [f1], approximate="tanh")
        B.shape[g] = B.shape[f1]
        h = B.binary("Add", h, _vit_linear(B, g, w2, b2, rows, M, D))
    h = vit_layer_norm(B, h, _ViTLayerNormParams(B, D, "norm", affine_scale), eps)
    clsv = B.op("Slice", [h, B.const(np.array([0, 0, 0], np.int64)), B.const(np.array([big, 1, big], np.int64))])
    B.shape[clsv] = (batch, 1, D)
    clsv = B.op("Reshape", [clsv, B.vec([B.unsq(B.dim(h, 0)), D])])
    B.shape[clsv] = (batch, D)
    wh = B.init(xavier_uniform(B.rng, (D, num_classes)), "head.weight")
    logits = _vit_linear(B, clsv, wh, bias(num_classes, "head.bias"), batch, D, num_classes)
    if apply_softmax:
        logits = B.op("Softmax", [logits], axis=-1)
    B.outputs.append(W.ValueInfo(logits))
    name = {"tiny": "ViTTiny", "small": "ViTSmall", "base": "ViTBase"}[variant]
    return ModelCase(f"vit_{variant}", B.model(name), [(x, x_val)], [logits], B.macs, B.params)


# Headline configurations (sizes, seeds) of the five workloads.
CONFIGS = {
    "stacked_linear": dict(fn=stacked_linear, kwargs=dict(batch=4096, n=1024, depth=8, seed=42)),
    "mlp": dict(fn=mlp, kwargs=dict(batch=8192, seed=1)),
    "resnet18": dict(fn=resnet, kwargs=dict(depth=18, batch=256, seed=7)),
    "resnet50": dict(fn=resnet, kwargs=dict(depth=50, batch=512, seed=11)),
    "retinanet": dict(fn=retinanet, kwargs=dict(batch=16, seed=13)),
    # adjacent model: the GroupNorm-head detector (RetinaNetResNet50, 32 groups)
    "retinanet_gn": dict(fn=retinanet, kwargs=dict(batch=16, seed=13, norm_heads=True)),
    # adjacent model: ViT-B/16 (ViTBase), batch 1 as its graph allows
    "vit_base": dict(fn=vit, kwargs=dict(variant="base", batch=1, seed=17)),
}


def build(name: str, **overrides) -> ModelCase:
    cfg = CONFIGS[name]
    kw = dict(cfg["kwargs"])
    kw.update(overrides)
    return cfg["fn"](**kw)
