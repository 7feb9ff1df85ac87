"""GPU parity of the two graph rewrites the reference's exporter applies before a model reaches the
backend (src/Shorokoo/Core/Factory/FastOnnxModelBuilder.cs):

* Upsample -> Resize(X, roi="", scales, sizes="", mode, coordinate_transformation_mode="asymmetric")
  (LowerUpsampleToResize, :626-660), both as the residual of a conv (the FPN top-down path, fused
  into the conv) and as a standalone op whose result is a graph output (the gather kernel);
* training-mode BatchNormalization -> ReduceMean / Sub / Mul / ReduceMean / Add(eps) / Sqrt / Div /
  Reshape(scale, bias to [1,-1,1,1]) / Mul / Add, plus the running-statistics update
  Reshape(batch mean, [-1]) * (1 - momentum) + running mean * momentum
  (LowerTrainingBatchNormalizationInGraph, :768-925, static-rank branch).

Both run through the plugin interface against the fp32 oracle at the bf16 gate. The training-BN
chain reduces over the batch axis, so the session cannot shard it; its batch statistics are
computed by the generic kernels in fp32."""
import numpy as np
import pytest

from helpers import BF16_TOL, assert_close, run_backend, run_oracle
from shorokoo_b200.emit import onnx_writer as W
from shorokoo_b200.emit.graphs import Builder, ModelCase, kaiming_normal

pytestmark = pytest.mark.gpu


def _resize_asym(B, x, scale):
    """Upsample(X, scales) after the exporter's rewrite."""
    n, c, h, w = B.shape[x]
    sc = B.const(np.array([1.0, 1.0, scale, scale], np.float32))
    y = B.op("Resize", [x, "", sc, ""], mode="nearest", coordinate_transformation_mode="asymmetric")
    B.shape[y] = (n, c, int(h * scale), int(w * scale))
    return y


def upsample_case(seed=21):
    rng = np.random.Generator(np.random.PCG64(seed))
    fine = rng.standard_normal((2, 96, 20, 26), dtype=np.float32)
    coarse = rng.standard_normal((2, 128, 10, 13), dtype=np.float32)
    B = Builder(seed + 1000)
    xf = B.graph_input(W.FLOAT, 4, fine.shape)
    xc = B.graph_input(W.FLOAT, 4, coarse.shape)
    wl = B.init(kaiming_normal(B.rng, (64, 96, 1, 1)), "lateral.weight")
    bl = B.init((0.1 * B.rng.standard_normal(64)).astype(np.float32), "lateral.bias")
    wc = B.init(kaiming_normal(B.rng, (64, 128, 1, 1)), "top.weight")
    lat = B.conv(xf, wl, bl, 1, 1, pads=[0, 0, 0, 0])
    top = B.conv(xc, wc, None, 1, 1, pads=[0, 0, 0, 0])
    p = B.binary("Add", lat, _resize_asym(B, top, 2.0))   # fused: the conv's upsampled residual
    ws = B.init(kaiming_normal(B.rng, (64, 64, 3, 3)), "smooth.weight")
    out = B.unary("Relu", B.conv(p, ws, None, 3, 1, pads=[1, 1, 1, 1]))
    up = _resize_asym(B, B.ident(xc), 2.0)   # standalone: gather kernel, graph output
    B.outputs += [W.ValueInfo(out), W.ValueInfo(up)]
    return ModelCase("upsample_asym", B.model("upsample_asym"), [(xf, fine), (xc, coarse)], [out, up], B.macs)


def training_bn_case(seed=31, momentum=0.9, eps=1e-5):
    rng = np.random.Generator(np.random.PCG64(seed))
    x = rng.standard_normal((4, 32, 12, 14), dtype=np.float32)
    B = Builder(seed + 1000)
    xi = B.graph_input(W.FLOAT, 4, x.shape)
    w = B.init(kaiming_normal(B.rng, (48, 32, 3, 3)), "conv.weight")
    h = B.conv(xi, w, None, 3, 1, pads=[1, 1, 1, 1])
    scale = B.init((1 + 0.2 * B.rng.standard_normal(48)).astype(np.float32), "bn.weight")
    bias = B.init((0.2 * B.rng.standard_normal(48)).astype(np.float32), "bn.bias")
    rmean = B.init((0.1 * B.rng.standard_normal(48)).astype(np.float32), "bn.running_mean")
    axes = B.const(np.array([0, 2, 3], np.int64))
    bm = B.op("ReduceMean", [h, axes], keepdims=1)
    centered = B.op("Sub", [h, bm])
    sq = B.op("Mul", [centered, centered])
    bv = B.op("ReduceMean", [sq, axes], keepdims=1)
    std = B.op("Sqrt", [B.op("Add", [bv, B.const(np.array(eps, np.float32))])])
    norm = B.op("Div", [centered, std])
    chan = B.const(np.array([1, -1, 1, 1], np.int64))
    y = B.op("Add", [B.op("Mul", [norm, B.op("Reshape", [scale, chan])]), B.op("Reshape", [bias, chan])])
    y = B.op("Relu", [y])
    flat = B.const(np.array([-1], np.int64))
    new_mean = B.op("Add", [B.op("Mul", [rmean, B.const(np.array(momentum, np.float32))]),
                            B.op("Mul", [B.op("Reshape", [bm, flat]), B.const(np.array(1 - momentum, np.float32))])])
    B.outputs += [W.ValueInfo(y), W.ValueInfo(new_mean)]
    return ModelCase("training_bn", B.model("training_bn"), [(xi, x)], [y, new_mean], B.macs)


def test_upsample_lowered_to_asymmetric_resize():
    case = upsample_case()
    got = run_backend(case)
    ref = run_oracle(case)
    assert_close(got[0], ref[0], what="conv + asymmetric-resize residual")
    # the standalone resize only moves values: exact
    assert got[1].shape == (2, 128, 20, 26)
    np.testing.assert_array_equal(got[1], ref[1])


def test_training_batchnorm_decomposition():
    case = training_bn_case()
    got = run_backend(case)
    ref = run_oracle(case)
    assert_close(got[0], ref[0], tol=BF16_TOL, what="training-BN chain output")
    assert_close(got[1], ref[1], tol=BF16_TOL, what="running-mean update")
