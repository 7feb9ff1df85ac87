"""Pins the oracle (CPU restatement of the reference's ONNX Runtime CPU path) before it is trusted:

* against the reference's own PyTorch references, run here and frozen as fixtures (tests/golden):
  the ResNet-18 twin of make-reference-logits.py and the Linear script tests/pytorch-reference/linear.py;
* against known answers from the reference's tests: GpuExecutionTests (2 + 3 = 5) and the Conv /
  MaxPool shape audits of tests/Shorokoo.Tests/Modules/QeePoolConvAuditModules.cs, with all-ones
  weights so the values are countable by hand;
* against plain-C loops (oracle/ref_small.c) for the torch-backed Conv / MaxPool / GEMM pieces.
"""
import ctypes as C
import os
import subprocess

import numpy as np
import pytest

from oracle.interp import Interpreter
from shorokoo_b200.emit import graphs
from shorokoo_b200.emit import onnx_writer as W
from shorokoo_b200.emit.graphs import Builder

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_resnet18_golden_pytorch_twin():
    d = np.load(os.path.join(GOLDEN, "resnet18_torchref.npz"))
    case = graphs.resnet(**eval(str(d["kwargs"])))
    np.testing.assert_array_equal(case.inputs[-1][1], d["x"])
    from tests.golden.gen_golden import param_checksum
    np.testing.assert_allclose(param_checksum(case.params), d["param_checksum"], rtol=0, atol=0)
    for prec, tol in (("fp32", 5e-6), ("fp64", 5e-6)):
        y = Interpreter(case.model, prec).run(dict(case.inputs))[0]
        err = np.abs(y - d["logits"]).max() / np.abs(d["logits"]).max()
        assert err < tol, (prec, err)


def test_linear_golden_pytorch_script():
    d = np.load(os.path.join(GOLDEN, "linear_pytorchref.npz"))
    case = graphs.mlp(**eval(str(d["kwargs"])))
    np.testing.assert_array_equal(case.params["layers.0.weight"], d["w"])
    y = Interpreter(case.model).run(dict(case.inputs))[0]
    np.testing.assert_allclose(y, d["y"], rtol=1e-6, atol=1e-6)


def _scalar_add_model():
    B = Builder(0)
    a = B.graph_input(W.FLOAT, 0)
    b = B.graph_input(W.FLOAT, 0)
    c = B.op("Add", [a, b])
    B.outputs.append(W.ValueInfo(c))
    return B.model("add"), a, b, c


def test_gpu_execution_known_answer_on_oracle():
    """GpuExecutionTests.CudaProvider_AddTwoFloat32Scalars_ReturnsCorrectSum: 2 + 3 == 5."""
    m, a, b, c = _scalar_add_model()
    y = Interpreter(m).run({a: np.array(2.0, np.float32), b: np.array(3.0, np.float32)})[0]
    assert float(y) == 5.0


def _ones_conv(x_shape, w_shape, **attrs):
    B = Builder(0)
    x = B.graph_input(W.FLOAT, 4, x_shape)
    w = B.init(np.ones(w_shape, np.float32))
    bb = B.init(np.ones(w_shape[0], np.float32))
    y = B.op("Conv", [x, w, bb], **attrs)
    B.outputs.append(W.ValueInfo(y))
    return B.model("c"), x


def _count_taps(H, W_, k, s, d, pads):
    """Number of in-bounds taps per output position (all-ones input and weights)."""
    oh = (H + pads[0] + pads[2] - ((k - 1) * d + 1)) // s + 1
    ow = (W_ + pads[1] + pads[3] - ((k - 1) * d + 1)) // s + 1
    out = np.zeros((oh, ow))
    for i in range(oh):
        for j in range(ow):
            cnt = 0
            for a in range(k):
                for b in range(k):
                    hi, wi = i * s - pads[0] + a * d, j * s - pads[1] + b * d
                    cnt += (0 <= hi < H) and (0 <= wi < W_)
            out[i, j] = cnt
    return out


@pytest.mark.parametrize("attrs,expect,pads,k,s,d,cin_per_group", [
    # QeeConvShapeAuditCheck: x [1,4,9,9]; expected dims from the audit
    (dict(auto_pad="NOTSET", dilations=[1, 1], group=2, kernel_shape=[3, 3], pads=[1, 1, 1, 1], strides=[2, 2]),
     (1, 6, 5, 5), [1, 1, 1, 1], 3, 2, 1, 2),
    (dict(auto_pad="NOTSET", dilations=[2, 2], group=1, kernel_shape=[3, 3], pads=[0, 0, 0, 0], strides=[1, 1]),
     (1, 2, 5, 5), [0, 0, 0, 0], 3, 1, 2, 4),
    (dict(auto_pad="SAME_UPPER", dilations=[1, 1], group=1, kernel_shape=[3, 3], strides=[2, 2]),
     (1, 2, 5, 5), [1, 1, 1, 1], 3, 2, 1, 4),
    (dict(auto_pad="VALID", dilations=[1, 1], group=1, kernel_shape=[3, 3], strides=[1, 1]),
     (1, 2, 7, 7), [0, 0, 0, 0], 3, 1, 1, 4),
])
def test_conv_shape_audit_known_answers(attrs, expect, pads, k, s, d, cin_per_group):
    w_shape = (expect[1], cin_per_group, 3, 3)
    m, x = _ones_conv((1, 4, 9, 9), w_shape, **attrs)
    y = Interpreter(m).run({x: np.ones((1, 4, 9, 9), np.float32)})[0]
    assert y.shape == expect
    taps = _count_taps(9, 9, k, s, d, pads)
    np.testing.assert_array_equal(y[0, 0], taps * cin_per_group + 1.0)


@pytest.mark.parametrize("attrs,expect", [
    # QeeMaxPoolShapeAuditCheck on x [1,1,10,10]
    (dict(ceil_mode=0, dilations=[2, 2], kernel_shape=[3, 3], pads=[0, 0, 0, 0], strides=[1, 1]), (1, 1, 6, 6)),
    (dict(ceil_mode=1, dilations=[1, 1], kernel_shape=[2, 2], pads=[0, 0, 0, 0], strides=[3, 3]), (1, 1, 4, 4)),
    (dict(ceil_mode=1, dilations=[1, 1], kernel_shape=[2, 2], pads=[1, 1, 1, 1], strides=[4, 4]), (1, 1, 3, 3)),
    (dict(ceil_mode=0, dilations=[1, 1], kernel_shape=[3, 3], pads=[1, 0, 2, 0], strides=[2, 2]), (1, 1, 6, 4)),
    (dict(auto_pad="SAME_LOWER", ceil_mode=0, dilations=[1, 1], kernel_shape=[3, 3], strides=[2, 2]), (1, 1, 5, 5)),
])
def test_maxpool_shape_audit_known_answers(attrs, expect):
    B = Builder(0)
    x = B.graph_input(W.FLOAT, 4, (1, 1, 10, 10))
    y = B.op("MaxPool", [x], **attrs)
    B.outputs.append(W.ValueInfo(y))
    xv = np.arange(100, dtype=np.float32).reshape(1, 1, 10, 10)
    out = Interpreter(B.model("p")).run({x: xv})[0]
    assert out.shape == expect
    # increasing input: every window's max is its bottom-right in-bounds element
    assert np.all(np.diff(out[0, 0], axis=1) >= 0) and np.all(np.diff(out[0, 0], axis=0) >= 0)


@pytest.fixture(scope="module")
def ref_small():
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle")], check=True)
    lib = C.CDLL(os.path.join(ROOT, "oracle", "_build", "libref_small.so"))
    return lib


def _dp(a):
    return a.ctypes.data_as(C.POINTER(C.c_double))


@pytest.mark.parametrize("n,c,h,w,m,k,s,d,pads,g", [
    (2, 3, 11, 9, 5, 7, 2, 1, [3, 3, 3, 3], 1), (1, 8, 7, 7, 6, 3, 1, 2, [2, 1, 2, 1], 1),
    (1, 4, 9, 9, 6, 3, 2, 1, [1, 1, 1, 1], 2), (2, 16, 5, 6, 8, 1, 2, 1, [0, 0, 0, 0], 1),
    (1, 4, 6, 5, 4, 3, 2, 1, [0, 0, 1, 1], 1),   # SAME_UPPER-style asymmetric pads
])
def test_oracle_conv_matches_plain_c(ref_small, n, c, h, w, m, k, s, d, pads, g):
    rng = np.random.default_rng(0)
    x = rng.standard_normal((n, c, h, w))
    wt = rng.standard_normal((m, c // g, k, k))
    b = rng.standard_normal(m)
    B = Builder(0)
    xi = B.graph_input(W.FLOAT, 4, x.shape)
    wi = B.init(wt.astype(np.float32))
    bi = B.init(b.astype(np.float32))
    y = B.op("Conv", [xi, wi, bi], dilations=[d, d], group=g, kernel_shape=[k, k], pads=pads, strides=[s, s])
    B.outputs.append(W.ValueInfo(y))
    got = Interpreter(B.model("c"), "fp64").run({xi: x.astype(np.float32)})[0]
    x32 = x.astype(np.float32).astype(np.float64)
    w32 = wt.astype(np.float32).astype(np.float64)
    b32 = b.astype(np.float32).astype(np.float64)
    out = np.zeros(got.shape)
    ref_small.ref_conv2d(_dp(x32), _dp(w32), _dp(b32), _dp(out), *[C.c_int64(v) for v in (
        n, c, h, w, m, k, k, s, s, d, d, pads[0], pads[1], pads[2], pads[3], g)])
    np.testing.assert_allclose(got, out, rtol=1e-12, atol=1e-10)


def test_oracle_maxpool_and_gemm_match_plain_c(ref_small):
    rng = np.random.default_rng(1)
    x = rng.standard_normal((2, 3, 13, 11)).astype(np.float32)
    B = Builder(0)
    xi = B.graph_input(W.FLOAT, 4, x.shape)
    y = B.op("MaxPool", [xi], kernel_shape=[3, 3], pads=[1, 1, 1, 1], strides=[2, 2])
    B.outputs.append(W.ValueInfo(y))
    got = Interpreter(B.model("p"), "fp64").run({xi: x})[0]
    out = np.zeros(got.shape)
    xd = x.astype(np.float64)
    ref_small.ref_maxpool2d(_dp(xd), _dp(out), *[C.c_int64(v) for v in (2, 3, 13, 11, got.shape[2], got.shape[3],
                                                                           3, 3, 2, 2, 1, 1, 1, 1)])
    np.testing.assert_array_equal(got, out)
    a = rng.standard_normal((7, 5))
    bm = rng.standard_normal((5, 3))
    case = graphs.mlp(batch=7, widths=(5, 3), seed=9, bias_scale=0.3)
    wgt = case.params["layers.0.weight"].astype(np.float64)
    bias = case.params["layers.0.bias"].astype(np.float64)
    xin = case.inputs[0][1].astype(np.float64)
    got = Interpreter(case.model, "fp64").run(dict(case.inputs))[0]
    out = np.zeros((7, 3))
    wt = np.ascontiguousarray(wgt.T)
    ref_small.ref_gemm(_dp(xin), _dp(wt), _dp(bias), _dp(out), C.c_int64(7), C.c_int64(3), C.c_int64(5))
    np.testing.assert_allclose(got, out, rtol=1e-12)
    del a, bm


def test_oracle_resize_nearest_is_floor_half():
    """Default Resize attrs (half_pixel + round_prefer_floor) at scale 2 pick floor(i/2) (Tensor.cs:367-379)."""
    B = Builder(0)
    x = B.graph_input(W.FLOAT, 4, (1, 1, 3, 5))
    y = B.op("Resize", [x, "", B.const(np.array([1, 1, 2, 2], np.float32))], mode="nearest")
    B.outputs.append(W.ValueInfo(y))
    xv = np.arange(15, dtype=np.float32).reshape(1, 1, 3, 5)
    out = Interpreter(B.model("r")).run({x: xv})[0]
    ii, jj = np.meshgrid(np.arange(6) // 2, np.arange(10) // 2, indexing="ij")
    np.testing.assert_array_equal(out[0, 0], xv[0, 0][ii, jj])


def test_oracle_live_hyper_control_flow():
    """Live-[Hyper] If/Loop graphs evaluate like their specialised twins."""
    a = graphs.stacked_linear(batch=4, n=16, depth=3, seed=2, live_depth=True, bias_scale=0.2)
    b = graphs.stacked_linear(batch=4, n=16, depth=3, seed=2, live_depth=False, bias_scale=0.2)
    ya = Interpreter(a.model).run(dict(a.inputs))[0]
    yb = Interpreter(b.model).run(dict(b.inputs))[0]
    np.testing.assert_allclose(ya, yb, rtol=1e-6)
    c = graphs.resnet(depth=18, batch=1, hw=(32, 32), seed=3, live_hypers=True, apply_softmax=True)
    y = Interpreter(c.model).run(dict(c.inputs))[0]
    np.testing.assert_allclose(y.sum(-1), 1.0, rtol=1e-5)
