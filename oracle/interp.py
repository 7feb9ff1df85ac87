"""ORACLE (test infrastructure only): CPU restatement of the reference's ONNX Runtime CPU path.

The reference executes every concrete graph through ONNX Runtime 1.26 (the CPU EP in
src/Backend/OnnxRuntime/Shorokoo.LinuxCPU/LinuxCpuInferenceFactory.cs:5-9, glue in
src/Backend/OnnxRuntime/Shorokoo.OnnxRuntime/OrtSessionFactory.cs:23-42 and
OrtInferenceSession.cs:15-36).  ORT is a NuGet binary absent from this machine, so this module
re-states the ONNX opset-21 semantics of exactly the operators the reference emits for the
inference hot path, interpreting the same ONNX bytes the B200 library receives.

* ``precision="fp32"`` computes float tensors in float32 (the stand-in for ORT-CPU's fp32 kernels,
  and the timed CPU baseline);
* ``precision="fp64"`` promotes every float tensor to float64 (ground truth for error analysis);
* ``precision="bf16-operands"`` computes in float32 but rounds both operands of every Conv / MatMul
  to bfloat16 (round-to-nearest-even), the arithmetic of a bf16 tensor-core path with fp32
  accumulation. It separates a kernel bug from the precision floor of bf16 operands;
* ``precision="tf32-operands"`` does the same with TF32 operands (fp32 rounded to 10 explicit
  mantissa bits, nearest even): the arithmetic of the TF32 accuracy mode.

Conv / MatMul use torch CPU kernels (torch.nn.functional.conv2d, torch.matmul) for speed; everything
else is numpy.  ``oracle/ref_small.c`` re-derives Conv / MaxPool / GEMM with plain loops so the
torch-backed pieces are themselves cross-checked on small shapes.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use this module.
"""
from __future__ import annotations

import math
import os
from typing import Dict, List, Optional, Sequence

import numpy as np

from .onnx_decode import GraphP, ModelP, NodeP, decode_model

try:
    import torch
    import torch.nn.functional as F
except ImportError:  # pragma: no cover
    torch = None


class OracleError(RuntimeError):
    pass


def _i(a) -> List[int]:
    return [int(v) for v in np.asarray(a).reshape(-1)]


class Interpreter:
    def __init__(self, model_bytes: bytes, precision: str = "fp32", threads: Optional[int] = None):
        if precision not in ("fp32", "fp64", "bf16-operands", "tf32-operands"):
            raise ValueError(precision)
        self.model: ModelP = decode_model(model_bytes)
        self.precision = precision
        self.fdt = np.float64 if precision == "fp64" else np.float32
        self.functions = {(f.domain, f.name): f for f in self.model.functions}
        self.inits = {t.name: self._cast_float(t.to_numpy()) for t in self.model.graph.initializers}
        if torch is not None:
            torch.set_num_threads(threads or len(os.sched_getaffinity(0)))

    @property
    def input_names(self) -> List[str]:
        inits = set(self.inits)
        return [v.name for v in self.model.graph.inputs if v.name not in inits]

    @property
    def output_names(self) -> List[str]:
        return [v.name for v in self.model.graph.outputs]

    def _cast_float(self, a: np.ndarray) -> np.ndarray:
        if a.dtype in (np.float32, np.float64, np.float16):
            return a.astype(self.fdt)
        return a

    # ------------------------------------------------------------------------------------------
    def run(self, inputs: Dict[str, np.ndarray], output_names: Optional[Sequence[str]] = None):
        env: Dict[str, np.ndarray] = dict(self.inits)
        for name in self.input_names:
            if name not in inputs:
                raise OracleError(f"missing input {name}")
            env[name] = self._cast_float(np.asarray(inputs[name]))
        outs = self._run_graph(self.model.graph, env)
        names = list(output_names) if output_names is not None else self.output_names
        return [outs[n] for n in names]

    def _run_graph(self, g: GraphP, env: Dict[str, np.ndarray]) -> Dict[str, np.ndarray]:
        for node in g.nodes:
            ins = [env[i] if i else None for i in node.inputs]
            res = self._exec(node, ins, env)
            for name, val in zip(node.outputs, res):
                if name:
                    env[name] = val
        return {o.name: env[o.name] for o in g.outputs}

    def _sub(self, g: GraphP, env, bound: Dict[str, np.ndarray]):
        scope = dict(env)
        scope.update(bound)
        for t in g.initializers:
            scope[t.name] = self._cast_float(t.to_numpy())
        return self._run_graph(g, scope)

    # ------------------------------------------------------------------------------------------
    def _exec(self, n: NodeP, x: List[Optional[np.ndarray]], env) -> List[np.ndarray]:
        op = n.op_type
        if n.domain not in ("", "ai.onnx"):
            fn = self.functions.get((n.domain, op))
            if fn is None:
                raise OracleError(f"unknown function {n.domain}.{op}")
            scope = dict(env)
            scope.update({k: v for k, v in zip(fn.inputs, x)})
            for node in fn.nodes:
                res = self._exec(node, [scope[i] if i else None for i in node.inputs], scope)
                for name, val in zip(node.outputs, res):
                    scope[name] = val
            return [scope[o] for o in fn.outputs]
        h = getattr(self, "op_" + op, None)
        if h is None:
            raise OracleError(f"unsupported op {op}")
        r = h(n, x, env)
        return r if isinstance(r, list) else [r]

    # --- control flow (ONNX If / Loop) -----------------------------------------------------------
    def op_If(self, n, x, env):
        g = n.attr("then_branch") if bool(np.asarray(x[0]).reshape(-1)[0]) else n.attr("else_branch")
        outs = self._sub(g, env, {})
        return [outs[o.name] for o in g.outputs]

    def op_Loop(self, n, x, env):
        body: GraphP = n.attr("body")
        m = x[0]
        cond = x[1]
        carried = list(x[2:])
        trip = int(np.asarray(m).reshape(-1)[0]) if m is not None else (1 << 62)
        keep = bool(np.asarray(cond).reshape(-1)[0]) if cond is not None else True
        nc = len(carried)
        scans: List[List[np.ndarray]] = [[] for _ in range(len(body.outputs) - 1 - nc)]
        i = 0
        while i < trip and keep:
            bound = {body.inputs[0].name: np.array(i, np.int64), body.inputs[1].name: np.array(keep)}
            for vi, v in zip(body.inputs[2:], carried):
                bound[vi.name] = v
            outs = self._sub(body, env, bound)
            vals = [outs[o.name] for o in body.outputs]
            keep = bool(np.asarray(vals[0]).reshape(-1)[0])
            carried = vals[1:1 + nc]
            for s, v in zip(scans, vals[1 + nc:]):
                s.append(v)
            i += 1
        return carried + [np.stack(s) if s else np.zeros((0,), self.fdt) for s in scans]

    # --- constants / shape ops --------------------------------------------------------------------
    def op_Constant(self, n, x, env):
        t = n.attr("value")
        if t is not None:
            return self._cast_float(t.to_numpy())
        if "value_float" in n.attrs:
            return np.array(n.attr("value_float"), self.fdt)
        if "value_int" in n.attrs:
            return np.array(n.attr("value_int"), np.int64)
        if "value_ints" in n.attrs:
            return np.array(n.attr("value_ints"), np.int64)
        if "value_floats" in n.attrs:
            return np.array(n.attr("value_floats"), self.fdt)
        raise OracleError("Constant without value")

    def op_ConstantOfShape(self, n, x, env):
        t = n.attr("value")
        v = self._cast_float(t.to_numpy()).reshape(-1)[0] if t is not None else self.fdt(0)
        dt = v.dtype if t is not None else self.fdt
        return np.full(_i(x[0]), v, dtype=dt)

    def op_Identity(self, n, x, env):
        return x[0]

    def op_Shape(self, n, x, env):
        s = np.array(x[0].shape, np.int64)
        start = n.attr("start", 0)
        end = n.attr("end", None)
        return s[start:end] if end is not None else s[start:]

    def op_Size(self, n, x, env):
        return np.array(x[0].size, np.int64)

    def op_Gather(self, n, x, env):
        axis = n.attr("axis", 0)
        idx = np.asarray(x[1]).astype(np.int64)
        dim = x[0].shape[axis]
        idx = np.where(idx < 0, idx + dim, idx)
        return np.take(x[0], idx, axis=axis)

    def op_Slice(self, n, x, env):
        data = x[0]
        starts, ends = _i(x[1]), _i(x[2])
        axes = _i(x[3]) if len(x) > 3 and x[3] is not None else list(range(len(starts)))
        steps = _i(x[4]) if len(x) > 4 and x[4] is not None else [1] * len(starts)
        sl = [slice(None)] * data.ndim
        for s, e, a, st in zip(starts, ends, axes, steps):
            a = a + data.ndim if a < 0 else a
            d = data.shape[a]
            if st > 0:
                s = min(max(s + d if s < 0 else s, 0), d)
                e = min(max(e + d if e < 0 else e, 0), d)
            else:
                s = min(max(s + d if s < 0 else s, -1), d - 1)
                e = min(max(e + d if e < 0 else e, -1), d - 1)
                if e < 0:
                    e = None
            sl[a] = slice(s, e, st)
        return data[tuple(sl)]

    def op_Unsqueeze(self, n, x, env):
        axes = _i(x[1]) if len(x) > 1 and x[1] is not None else _i(n.attr("axes"))
        r = x[0].ndim + len(axes)
        out = x[0]
        for a in sorted(a + r if a < 0 else a for a in axes):
            out = np.expand_dims(out, a)
        return out

    def op_Squeeze(self, n, x, env):
        if len(x) > 1 and x[1] is not None:
            axes = tuple(a + x[0].ndim if a < 0 else a for a in _i(x[1]))
            return np.squeeze(x[0], axis=axes)
        return np.squeeze(x[0])

    def op_Concat(self, n, x, env):
        return np.concatenate([v for v in x if v is not None], axis=n.attr("axis"))

    def op_Reshape(self, n, x, env):
        shape = _i(x[1])
        allowzero = n.attr("allowzero", 0)
        out = []
        for i, s in enumerate(shape):
            out.append(x[0].shape[i] if (s == 0 and not allowzero) else s)
        return x[0].reshape(out)

    def op_Flatten(self, n, x, env):
        a = n.attr("axis", 1)
        a = a + x[0].ndim if a < 0 else a
        return x[0].reshape(int(np.prod(x[0].shape[:a])), -1)

    def op_Transpose(self, n, x, env):
        perm = n.attr("perm")
        return np.ascontiguousarray(np.transpose(x[0], perm if perm else None))

    def op_Expand(self, n, x, env):
        shape = np.broadcast_shapes(x[0].shape, tuple(_i(x[1])))
        return np.broadcast_to(x[0], shape).copy()

    def op_Cast(self, n, x, env):
        from .onnx_decode import ONNX_TO_NP
        to = n.attr("to")
        dt = ONNX_TO_NP[to]
        if dt in (np.float32, np.float64):
            dt = self.fdt
        return x[0].astype(dt)

    def op_Range(self, n, x, env):
        return np.arange(x[0].item(), x[1].item(), x[2].item()).astype(x[0].dtype)

    def _reduce(self, n, x, fn):
        if len(x) > 1 and x[1] is not None:
            axes = _i(x[1])
        else:
            axes = n.attr("axes", None)
        keep = bool(n.attr("keepdims", 1))
        if not axes:
            if n.attr("noop_with_empty_axes", 0):
                return x[0]
            axes = None
        else:
            axes = tuple(a + x[0].ndim if a < 0 else a for a in axes)
        return np.asarray(fn(x[0], axis=axes, keepdims=keep))

    def op_ReduceProd(self, n, x, env):
        return self._reduce(n, x, np.prod).astype(x[0].dtype)

    def op_ReduceSum(self, n, x, env):
        return self._reduce(n, x, np.sum).astype(x[0].dtype)

    def op_ReduceMean(self, n, x, env):
        return self._reduce(n, x, np.mean).astype(x[0].dtype)

    def op_ReduceMax(self, n, x, env):
        return self._reduce(n, x, np.max).astype(x[0].dtype)

    # --- elementwise ----------------------------------------------------------------------------
    @staticmethod
    def _bin(a, b, f):
        r = f(a, b)
        return np.asarray(r).astype(np.result_type(a.dtype, b.dtype)) if r.dtype != np.bool_ else r

    def op_Add(self, n, x, env):
        return self._bin(x[0], x[1], np.add)

    def op_Sub(self, n, x, env):
        return self._bin(x[0], x[1], np.subtract)

    def op_Mul(self, n, x, env):
        return self._bin(x[0], x[1], np.multiply)

    def op_Div(self, n, x, env):
        if np.issubdtype(x[0].dtype, np.integer):
            return np.trunc(x[0] / x[1]).astype(x[0].dtype)
        return self._bin(x[0], x[1], np.divide)

    def op_Pow(self, n, x, env):
        return np.power(x[0], x[1]).astype(x[0].dtype)

    def op_Max(self, n, x, env):
        out = x[0]
        for v in x[1:]:
            out = np.maximum(out, v)
        return out

    def op_Min(self, n, x, env):
        out = x[0]
        for v in x[1:]:
            out = np.minimum(out, v)
        return out

    def op_Equal(self, n, x, env):
        return np.equal(x[0], x[1])

    def op_Less(self, n, x, env):
        return np.less(x[0], x[1])

    def op_Greater(self, n, x, env):
        return np.greater(x[0], x[1])

    def op_Not(self, n, x, env):
        return np.logical_not(x[0])

    def op_And(self, n, x, env):
        return np.logical_and(x[0], x[1])

    def op_Or(self, n, x, env):
        return np.logical_or(x[0], x[1])

    def op_Where(self, n, x, env):
        return np.where(x[0], x[1], x[2])

    def op_Sqrt(self, n, x, env):
        return np.sqrt(x[0])

    def op_Neg(self, n, x, env):
        return -x[0]

    def op_Abs(self, n, x, env):
        return np.abs(x[0])

    def op_Exp(self, n, x, env):
        return np.exp(x[0])

    def op_Log(self, n, x, env):
        return np.log(x[0])

    def op_Reciprocal(self, n, x, env):
        return (1.0 / x[0]).astype(x[0].dtype)

    def op_Tanh(self, n, x, env):
        return np.tanh(x[0])

    def op_Relu(self, n, x, env):
        return np.maximum(x[0], 0).astype(x[0].dtype)

    def op_Sigmoid(self, n, x, env):
        v = x[0]
        one = v.dtype.type(1)
        return (one / (one + np.exp(-v))).astype(v.dtype)

    def op_Gelu(self, n, x, env):
        """ONNX Gelu (opset 20): approximate="none" x * Phi(x) with the error function, "tanh"
        0.5 x (1 + tanh(sqrt(2 / pi) (x + 0.044715 x^3))) (ViTMlp, ViTNet.cs:217-239)."""
        v = x[0]
        approx = n.attr("approximate", b"none")
        if isinstance(approx, bytes):
            approx = approx.decode()
        w = v.astype(np.float64)
        if approx == "tanh":
            y = 0.5 * w * (1.0 + np.tanh(math.sqrt(2.0 / math.pi) * (w + 0.044715 * w ** 3)))
        else:
            y = 0.5 * w * (1.0 + np.vectorize(math.erf)(w / math.sqrt(2.0)))
        return y.astype(v.dtype)

    def op_Tile(self, n, x, env):
        return np.tile(x[0], [int(r) for r in x[1]])

    def op_Softmax(self, n, x, env):
        axis = n.attr("axis", -1)
        v = x[0]
        m = np.max(v, axis=axis, keepdims=True)
        e = np.exp(v - m)
        return (e / np.sum(e, axis=axis, keepdims=True)).astype(v.dtype)

    # --- dense / conv / pool ----------------------------------------------------------------------
    def _t(self, a):
        return torch.from_numpy(np.ascontiguousarray(a))

    def _op_round(self, a):
        """Operand rounding of the bf16 / TF32 tensor-core paths (identity in fp32 / fp64 modes)."""
        if self.precision == "bf16-operands":
            return torch.from_numpy(np.ascontiguousarray(a, np.float32)).bfloat16().float().numpy()
        if self.precision == "tf32-operands":
            u = np.ascontiguousarray(a, np.float32).view(np.uint32)
            finite = (u & np.uint32(0x7F800000)) != np.uint32(0x7F800000)
            r = (u + np.uint32(0xFFF) + ((u >> np.uint32(13)) & np.uint32(1))) & np.uint32(0xFFFFE000)
            return np.where(finite, r, u).view(np.float32)
        return a

    def op_MatMul(self, n, x, env):
        a, b = self._op_round(x[0]), self._op_round(x[1])
        if torch is not None and a.dtype == b.dtype and a.dtype in (np.float32, np.float64):
            return torch.matmul(self._t(a), self._t(b)).numpy()
        return np.matmul(a, b)

    def op_Gemm(self, n, x, env):
        a, b = x[0], x[1]
        if n.attr("transA", 0):
            a = a.T
        if n.attr("transB", 0):
            b = b.T
        y = n.attr("alpha", 1.0) * self.op_MatMul(n, [a, b], env)
        if len(x) > 2 and x[2] is not None:
            y = y + n.attr("beta", 1.0) * x[2]
        return y.astype(a.dtype)

    @staticmethod
    def conv_pads(in_sp, k, s, d, auto_pad, pads):
        """Explicit pads vs SAME_UPPER/SAME_LOWER/VALID (src/Shorokoo/Core/Inference/Ops/Conv.cs:34-61)."""
        nd = len(in_sp)
        if isinstance(auto_pad, bytes):
            auto_pad = auto_pad.decode()
        if auto_pad in ("SAME_UPPER", "SAME_LOWER"):
            begin, end = [], []
            for i in range(nd):
                out = -(-in_sp[i] // s[i])
                total = max((out - 1) * s[i] + (k[i] - 1) * d[i] + 1 - in_sp[i], 0)
                small = total // 2
                big = total - small
                if auto_pad == "SAME_UPPER":
                    begin.append(small)
                    end.append(big)
                else:
                    begin.append(big)
                    end.append(small)
            return begin + end
        if auto_pad == "VALID":
            return [0] * (2 * nd)
        return list(pads) if pads else [0] * (2 * nd)

    def op_Conv(self, n, x, env):
        X, Wt = self._op_round(x[0]), self._op_round(x[1])
        B = x[2] if len(x) > 2 else None
        k = n.attr("kernel_shape") or list(Wt.shape[2:])
        nd = len(k)
        s = n.attr("strides") or [1] * nd
        d = n.attr("dilations") or [1] * nd
        g = n.attr("group", 1)
        pads = self.conv_pads(X.shape[2:], k, s, d, n.attr("auto_pad", b"NOTSET"), n.attr("pads"))
        if nd != 2:
            raise OracleError("only 2-D Conv")
        xt = self._t(X)
        if any(pads):
            xt = F.pad(xt, (pads[1], pads[3], pads[0], pads[2]))
        y = F.conv2d(xt, self._t(Wt), None if B is None else self._t(B), stride=s, dilation=d, groups=g)
        return y.numpy()

    def op_MaxPool(self, n, x, env):
        X = x[0]
        k = n.attr("kernel_shape")
        s = n.attr("strides") or [1, 1]
        d = n.attr("dilations") or [1, 1]
        pads = self.conv_pads(X.shape[2:], k, s, d, n.attr("auto_pad", b"NOTSET"), n.attr("pads"))
        ceil = bool(n.attr("ceil_mode", 0))
        xt = self._t(X)
        # Pad with -inf explicitly (asymmetric pads), then pool without padding.
        ph = (pads[0], pads[2])
        pw = (pads[1], pads[3])
        out_h = self._pool_out(X.shape[2], k[0], s[0], d[0], ph, ceil)
        out_w = self._pool_out(X.shape[3], k[1], s[1], d[1], pw, ceil)
        need_h = (out_h - 1) * s[0] + (k[0] - 1) * d[0] + 1
        need_w = (out_w - 1) * s[1] + (k[1] - 1) * d[1] + 1
        extra_h = max(need_h - (X.shape[2] + ph[0] + ph[1]), 0)
        extra_w = max(need_w - (X.shape[3] + pw[0] + pw[1]), 0)
        xt = F.pad(xt, (pw[0], pw[1] + extra_w, ph[0], ph[1] + extra_h), value=-math.inf)
        y = F.max_pool2d(xt, kernel_size=k, stride=s, dilation=d)
        return y[:, :, :out_h, :out_w].contiguous().numpy()

    @staticmethod
    def _pool_out(size, k, s, d, pads, ceil):
        eff = (k - 1) * d + 1
        num = size + pads[0] + pads[1] - eff
        out = (-(-num // s) if ceil else num // s) + 1
        if ceil and (out - 1) * s >= size + pads[0]:
            out -= 1        # last window must start inside the input or the begin padding
        return out

    def op_GlobalAveragePool(self, n, x, env):
        X = x[0]
        axes = tuple(range(2, X.ndim))
        return np.mean(X, axis=axes, keepdims=True, dtype=np.float64).astype(X.dtype)

    def op_GlobalMaxPool(self, n, x, env):
        X = x[0]
        return np.max(X, axis=tuple(range(2, X.ndim)), keepdims=True)

    def op_SequenceConstruct(self, n, x, env):
        return [list(x)]

    def op_SequenceAt(self, n, x, env):
        k = int(np.asarray(x[1]).reshape(-1)[0])
        return x[0][k]

    def op_SequenceLength(self, n, x, env):
        return np.array(len(x[0]), np.int64)

    def op_Pad(self, n, x, env):
        X = x[0]
        mode = n.attr("mode", b"constant")
        mode = mode.decode() if isinstance(mode, bytes) else mode
        pads = _i(x[1])
        val = x[2].reshape(-1)[0] if len(x) > 2 and x[2] is not None and x[2].size else 0
        nd = X.ndim
        axes = _i(x[3]) if len(x) > 3 and x[3] is not None else list(range(nd))
        width = [(0, 0)] * nd
        for j, a in enumerate(axes):
            a = a + nd if a < 0 else a
            width[a] = (pads[j], pads[j + len(axes)])
        if any(p < 0 for w in width for p in w):
            raise OracleError("negative pads")
        if mode == "constant":
            return np.pad(X, width, mode="constant", constant_values=val)
        return np.pad(X, width, mode={"reflect": "reflect", "edge": "edge", "wrap": "wrap"}[mode])

    def op_Resize(self, n, x, env):
        X = x[0]
        mode = n.attr("mode", b"nearest")
        mode = mode.decode() if isinstance(mode, bytes) else mode
        if mode != "nearest":
            raise OracleError("only nearest Resize")
        ctm = n.attr("coordinate_transformation_mode", b"half_pixel")
        ctm = ctm.decode() if isinstance(ctm, bytes) else ctm
        nmode = n.attr("nearest_mode", b"round_prefer_floor")
        nmode = nmode.decode() if isinstance(nmode, bytes) else nmode
        scales = x[2] if len(x) > 2 and x[2] is not None and x[2].size else None
        sizes = x[3] if len(x) > 3 and x[3] is not None and x[3].size else None
        if sizes is not None:
            out_shape = _i(sizes)
            sc = [o / i for o, i in zip(out_shape, X.shape)]
        else:
            sc = [float(v) for v in np.asarray(scales, np.float32).reshape(-1)]
            out_shape = [int(math.floor(i * s)) for i, s in zip(X.shape, sc)]
        out = X
        for ax in range(X.ndim):
            if out_shape[ax] == X.shape[ax] and sc[ax] == 1.0:
                continue
            idx = self._nearest_index(out_shape[ax], X.shape[ax], sc[ax], ctm, nmode)
            out = np.take(out, idx, axis=ax)
        return out

    @staticmethod
    def _nearest_index(out_len, in_len, scale, ctm, nmode):
        o = np.arange(out_len, dtype=np.float64)
        if ctm == "half_pixel":
            xo = (o + 0.5) / scale - 0.5
        elif ctm == "asymmetric":
            xo = o / scale
        elif ctm == "align_corners":
            xo = o * (in_len - 1) / (out_len - 1) if out_len > 1 else np.zeros_like(o)
        elif ctm == "pytorch_half_pixel":
            xo = (o + 0.5) / scale - 0.5 if out_len > 1 else np.zeros_like(o)
        else:
            raise OracleError(f"coordinate_transformation_mode {ctm}")
        if nmode == "round_prefer_floor":
            idx = np.where(xo - np.floor(xo) == 0.5, np.floor(xo), np.round(xo))
        elif nmode == "round_prefer_ceil":
            idx = np.where(xo - np.floor(xo) == 0.5, np.ceil(xo), np.round(xo))
        elif nmode == "floor":
            idx = np.floor(xo)
        else:
            idx = np.ceil(xo)
        return np.clip(idx, 0, in_len - 1).astype(np.int64)


def run_model(model_bytes: bytes, inputs, precision: str = "fp32", output_names=None):
    """Convenience: decode, run once, return outputs as a list of arrays."""
    it = Interpreter(model_bytes, precision)
    feed = dict(inputs) if not isinstance(inputs, dict) else inputs
    return it.run(feed, output_names)
