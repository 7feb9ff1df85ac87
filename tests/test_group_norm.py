"""GroupNorm (RetGroupNorm, samples/RetinaNet/RetinaNetDetector.cs:337-372; the GroupNorm layer,
src/Shorokoo.Modules/Layers/Normalization.cs:278-310) as the exporter writes it: Reshape to
[N, G, C/G, H, W] (or [N, G, -1]), ReduceMean, two Sub nodes for (x - mean) * (x - mean), the
biased variance, Add(eps), Sqrt, Div, Reshape back, per-channel gamma / beta, ReLU.

Host side (no GPU): the primitives fuse into one GroupNorm op (the GroupNorm RetinaNet heads: 40
of them, each with its ReLU), and chains the fusion must not take (an intermediate that is also a
graph output, a reduction over other axes) stay primitive. The oracle's GroupNorm matches numpy.
GPU side: the three-pass kernel (statistics with a per-channel shift, a double-precision merge,
the affine + ReLU pass) against numpy in float64 over bf16 (conv-produced) and fp32 inputs,
several channel / group counts, tiny and large maps; the GroupNorm RetinaNet against the oracle at
the bf16 and TF32 gates."""
import numpy as np
import pytest

from helpers import BF16_TOL, assert_close, run_backend, run_oracle
from shorokoo_b200.emit import graphs
from shorokoo_b200.emit import onnx_writer as W
from shorokoo_b200.emit.graphs import Builder, ModelCase, _GroupNormParams, group_norm, kaiming_normal
from test_native_host import kinds, lower


def _gn_ref(x, G, gamma, beta, eps=1e-5, relu=False):
    n, c, h, w = x.shape
    xr = x.astype(np.float64).reshape(n, G, -1)
    mu = xr.mean(axis=2, keepdims=True)
    var = ((xr - mu) ** 2).mean(axis=2, keepdims=True)
    y = ((xr - mu) / np.sqrt(var + eps)).reshape(n, c, h, w) * gamma.reshape(1, c, 1, 1) + beta.reshape(1, c, 1, 1)
    return np.maximum(y, 0) if relu else y


def _case(n, c, h, w, G, relu, conv_before=False, conv_after=False, mean_shift=0.0, seed=3, output_mid=False):
    """x -> [3x3 conv] -> GroupNorm(G) -> [ReLU] -> [1x1 conv]."""
    rng = np.random.Generator(np.random.PCG64(seed))
    x = (rng.standard_normal((n, c, h, w), dtype=np.float32) + np.float32(mean_shift)).astype(np.float32)
    B = Builder(seed + 1)
    xi = B.graph_input(W.FLOAT, 4, x.shape)
    v = xi
    if conv_before:
        wt = B.init(kaiming_normal(B.rng, (c, c, 3, 3)), "w0")
        bias = B.init((mean_shift + 0.3 * B.rng.standard_normal(c)).astype(np.float32), "b0")
        v = B.conv(v, wt, bias, 3, 1, pads=[1, 1, 1, 1])
    p = _GroupNormParams(B, c, "gn", affine_scale=0.3)
    y = group_norm(B, v, G, p)
    if relu:
        y = B.unary("Relu", y)
    outs = [y]
    if conv_after:
        w2 = B.init(kaiming_normal(B.rng, (16, c, 1, 1)), "w2")
        outs = [B.conv(y, w2, None, 1, 1, pads=[0, 0, 0, 0])]
    if output_mid:
        outs.append(v)
    for o in outs:
        B.outputs.append(W.ValueInfo(o))
    gamma = B.params["gn.weight"] if "gn.weight" in B.params else None
    return ModelCase("gn", B.model("gn"), [(xi, x)], outs, B.macs, B.params), x


def test_group_norm_heads_fuse():
    case = graphs.retinanet(batch=1, hw=(64, 96), seed=5, norm_heads=True, affine_scale=0.1,
                            backbone_widths=(8, 16, 32, 64), backbone_blocks=(1, 1, 1, 1), fpn=64, num_groups=8,
                            num_classes=5, num_anchors=3)
    lines = lower(case)
    k = kinds(lines)
    assert k["GroupNorm"] == 40 and "ReduceMean" not in k and "Sqrt" not in k and "Sub" not in k, k
    assert all(l.endswith("act=1") for l in lines if l.startswith("GroupNorm")), lines


def test_group_norm_not_fused_when_an_intermediate_is_read():
    case, _ = _case(1, 32, 6, 6, 4, relu=True, conv_before=True, output_mid=False)
    assert kinds(lower(case))["GroupNorm"] == 1
    # the normalised map before the affine is also a graph output: the affine stays outside, or the
    # whole chain stays primitive; either way the oracle and backend agree (GPU tests)
    B = Builder(9)
    x = np.random.Generator(np.random.PCG64(9)).standard_normal((2, 16, 4, 4), dtype=np.float32)
    xi = B.graph_input(W.FLOAT, 4, x.shape)
    xr = B.op("Reshape", [xi, B.const(np.array([2, 4, -1], np.int64))])
    B.shape[xr] = (2, 4, 64)
    mu = B.op("ReduceMean", [xr, B.const(np.array([2], np.int64))], keepdims=1)
    B.outputs.append(W.ValueInfo(mu))   # the mean is read by the caller
    d = B.op("Sub", [xr, mu])
    var = B.op("ReduceMean", [B.op("Mul", [d, d]), B.const(np.array([2], np.int64))], keepdims=1)
    y = B.op("Div", [d, B.op("Sqrt", [B.op("Add", [var, B.const(np.array(1e-5, np.float32))])])])
    y = B.op("Reshape", [y, B.const(np.array([2, 16, 4, 4], np.int64))])
    B.outputs.append(W.ValueInfo(y))
    k = kinds(lower(ModelCase("gn2", B.model("gn2"), [(xi, x)], [mu, y], 0)))
    assert "GroupNorm" not in k and k["ReduceMean"] == 2, k


def test_oracle_group_norm_matches_numpy():
    case, x = _case(2, 32, 5, 7, 8, relu=True)
    got = run_oracle(case)[0]
    ref = _gn_ref(x, 8, case.params["gn.weight"], case.params["gn.bias"], relu=True)
    np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-5)


@pytest.mark.gpu
@pytest.mark.parametrize("n,c,h,w,G,relu,conv_before,conv_after,shift", [
    (2, 256, 20, 24, 32, True, False, False, 0.0),     # fp32 input converted to NHWC, fp32 output
    (2, 256, 20, 24, 32, True, True, True, 0.0),       # conv output (bf16) -> GN -> conv (bf16)
    (3, 64, 9, 7, 8, False, True, False, 3.0),         # large mean against the spread (shifted sums)
    (1, 128, 1, 3, 4, True, True, True, 0.0),          # tiny map: fewer pixels than threads
    (2, 32, 50, 64, 32, True, False, True, 0.0),       # one channel per group (InstanceNorm)
    (2, 512, 7, 8, 16, True, True, True, 0.0),         # 32 channels per group
])
def test_group_norm_kernel(n, c, h, w, G, relu, conv_before, conv_after, shift):
    case, x = _case(n, c, h, w, G, relu, conv_before=conv_before, conv_after=conv_after, mean_shift=shift)
    got = run_backend(case)[0]
    ref = run_oracle(case)[0]
    tol = BF16_TOL if (conv_before or conv_after) else 1e-5
    assert_close(got, ref, tol=tol, what=f"group norm {n}x{c}x{h}x{w} G={G}")
    if not (conv_before or conv_after):   # the kernel alone, fp32 in and out, against float64
        e = _gn_ref(x, G, case.params["gn.weight"], case.params["gn.bias"], relu=relu)
        np.testing.assert_allclose(got, e, rtol=2e-5, atol=2e-5)


@pytest.mark.gpu
def test_group_norm_retinanet_bf16_and_tf32():
    case = graphs.retinanet(batch=2, hw=(128, 160), seed=5, norm_heads=True, affine_scale=0.1)
    ref = run_oracle(case)
    from shorokoo_b200 import B200InferenceSessionFactory
    for prec, tol in (("bf16", BF16_TOL), ("tf32", 2e-3)):
        got = run_backend(case, factory=B200InferenceSessionFactory(num_devices=1, precision=prec))
        for g, r, nm in zip(got, ref, ("class", "box")):
            assert g.shape == r.shape
            assert_close(g, r, tol=tol, what=f"GroupNorm RetinaNet {nm} ({prec})")
