"""Shared test helpers: run a synthesized model through the backend's plugin interface and through
the oracle, and compare them the way the parity gate states it."""
from __future__ import annotations

import numpy as np

from oracle.interp import Interpreter
from shorokoo_b200 import B200InferenceSessionFactory
from shorokoo_b200.emit import onnx_writer as W
from shorokoo_b200.emit.graphs import Builder, ModelCase, kaiming_normal

# bf16 tensor-core path: max|gpu - ref| / max|ref| per output tensor (normwise relative error).
BF16_TOL = 1e-2


def run_backend(case: ModelCase, num_devices: int = 1, factory=None):
    f = factory or B200InferenceSessionFactory(num_devices=num_devices)
    sess = f.CreateSession(case.model)
    feeds = {name: f.CreateTensor(arr) for name, arr in case.inputs}
    outs = sess.Run(feeds, case.output_names)
    res = [o.numpy() for o in outs]
    for o in outs:
        o.Dispose()
    sess.Dispose()
    return res


def run_oracle(case: ModelCase, precision: str = "fp32"):
    return Interpreter(case.model, precision).run(dict(case.inputs), case.output_names)


def normwise_err(got: np.ndarray, ref: np.ndarray) -> float:
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    denom = max(float(np.abs(ref).max()) if ref.size else 0.0, 1e-30)
    return float(np.abs(got - ref).max()) / denom if ref.size else 0.0


def assert_close(got, ref, tol=BF16_TOL, what=""):
    e = normwise_err(got, ref)
    assert np.all(np.isfinite(got)), f"{what}: non-finite output"
    assert e <= tol, f"{what}: normwise error {e:.3e} > {tol:.1e}"
    return e


def conv_case(n=2, c=16, h=9, w=9, cout=24, k=3, stride=1, pads=None, auto_pad="NOTSET", dil=1,
              bias=True, bn=False, residual=False, relu=False, sigmoid=False, upsample_residual=False,
              seed=0) -> ModelCase:
    """A single Conv (+ per-channel affine, residual add, activation) graph in the reference's style."""
    rng = np.random.Generator(np.random.PCG64(seed))
    x = rng.standard_normal((n, c, h, w), dtype=np.float32)
    B = Builder(seed + 1)
    xi = B.graph_input(W.FLOAT, 4, x.shape)
    inputs = [(xi, x)]
    wt = B.init(kaiming_normal(B.rng, (cout, c, k, k)), "w")
    b = B.init((0.3 * B.rng.standard_normal(cout)).astype(np.float32), "b") if bias else None
    inputs_list = [xi, wt] + ([b] if b else [])
    if auto_pad == "NOTSET":
        p = pads if pads is not None else [k // 2] * 4
        y = B.op("Conv", inputs_list, auto_pad="NOTSET", dilations=[dil, dil], group=1, kernel_shape=[k, k],
                 pads=p, strides=[stride, stride])
        ho = (h + p[0] + p[2] - ((k - 1) * dil + 1)) // stride + 1
        wo = (w + p[1] + p[3] - ((k - 1) * dil + 1)) // stride + 1
    else:
        y = B.op("Conv", inputs_list, auto_pad=auto_pad, dilations=[dil, dil], group=1, kernel_shape=[k, k],
                 strides=[stride, stride])
        ho, wo = -(-h // stride), -(-w // stride)
    B.shape[y] = (n, cout, ho, wo)
    if bn:
        s = B.init((1 + 0.2 * B.rng.standard_normal((1, cout, 1, 1))).astype(np.float32), "s")
        t = B.init((0.2 * B.rng.standard_normal((1, cout, 1, 1))).astype(np.float32), "t")
        y = B.op("Add", [B.op("Mul", [y, s]), t])
    if residual:
        r = rng.standard_normal((n, cout, ho, wo), dtype=np.float32)
        ri = B.graph_input(W.FLOAT, 4, r.shape)
        inputs.append((ri, r))
        y = B.op("Add", [y, ri])
    if upsample_residual:
        r = rng.standard_normal((n, cout, ho // 2, wo // 2), dtype=np.float32)
        ri = B.graph_input(W.FLOAT, 4, r.shape)
        inputs.append((ri, r))
        up = B.op("Resize", [ri, "", B.const(np.array([1, 1, 2, 2], np.float32))], mode="nearest")
        y = B.op("Add", [y, up])
    if relu:
        y = B.op("Relu", [y])
    if sigmoid:
        y = B.op("Sigmoid", [y])
    B.outputs.append(W.ValueInfo(y))
    return ModelCase("conv", B.model("conv"), inputs, [y], n * ho * wo * cout * c * k * k)
