"""GPU parity of the TF32 accuracy modes (precision="tf32": fp32 operands read as TF32 by
tcgen05.mma kind::tf32, fp32 accumulation, fp32 activations rounded to the TF32 grid) against the
fp32 oracle at the TF32 gate, normwise max|gpu - ref| / max|ref| <= 2e-3 per output, and against
the oracle with TF32-rounded operands (the mode's own arithmetic) more tightly."""
import numpy as np
import pytest

from helpers import assert_close, conv_case, run_oracle
from shorokoo_b200 import B200InferenceSessionFactory
from shorokoo_b200.emit import graphs
from helpers import run_backend

pytestmark = pytest.mark.gpu

TF32_TOL = 2e-3


def _tf32(case):
    return run_backend(case, factory=B200InferenceSessionFactory(num_devices=1, precision="tf32"))


@pytest.mark.parametrize("m,k,n,relu", [
    (300, 200, 100, True), (1000, 96, 1000, False), (513, 1024, 4096, True), (2, 2048, 1000, False),
])
def test_tf32_gemm(m, k, n, relu):
    widths = (k, n) if not relu else (k, n, n)
    case = graphs.mlp(batch=m, widths=widths, seed=3, bias_scale=0.5)
    got = _tf32(case)[0]
    assert_close(got, run_oracle(case)[0], tol=TF32_TOL, what=f"tf32 gemm {m}x{k}x{n}")


@pytest.mark.parametrize("kw", [
    dict(c=64, cout=64, k=1, pads=[0, 0, 0, 0]),                                   # row-matrix 1x1
    dict(c=64, cout=256, k=1, pads=[0, 0, 0, 0], bn=True, residual=True, relu=True),
    dict(c=24, cout=40, k=3, h=11, w=7),                                           # gather, 16-byte units
    dict(c=3, cout=64, k=7, stride=2, pads=[3, 3, 3, 3], h=32, w=32, bn=True, relu=True),  # stem
    dict(c=32, cout=48, k=3, stride=2, auto_pad="SAME_UPPER", h=25, w=32),
    dict(c=64, cout=720, k=3, auto_pad="SAME_UPPER", h=7, w=8, sigmoid=True),
    dict(n=2, c=64, cout=64, k=3, h=32, w=32, bn=True, relu=True),                 # im2col (128-byte pixels)
    dict(n=2, c=128, cout=256, k=1, stride=2, pads=[0, 0, 0, 0], h=28, w=28),
    dict(n=2, c=64, cout=32, k=5, pads=[1, 2, 3, 0], h=20, w=30),
    dict(c=128, cout=64, k=1, pads=[0, 0, 0, 0], h=10, w=16, upsample_residual=True),
])
def test_tf32_conv(kw):
    case = conv_case(**kw)
    got = _tf32(case)[0]
    assert_close(got, run_oracle(case)[0], tol=TF32_TOL, what=f"tf32 conv {kw}")
    assert_close(got, run_oracle(case, "tf32-operands")[0], tol=5e-4, what=f"tf32 conv {kw} vs tf32 oracle")


@pytest.mark.parametrize("name,kw", [
    ("resnet50", dict(batch=2, hw=(64, 64), affine_scale=0.1)),
    ("resnet18", dict(batch=3, hw=(96, 96))),
    ("stacked_linear", dict(batch=64)),
])
def test_tf32_model_parity(name, kw):
    case = graphs.build(name, **kw)
    got = _tf32(case)
    ref = run_oracle(case)
    for g, r, o in zip(got, ref, case.output_names):
        assert_close(g, r, tol=TF32_TOL, what=f"tf32 {name} {kw} output {o}")


def test_tf32_retinanet_meets_the_tf32_gate():
    """The detection graph whose 57-conv dense chains put single-pass TF32 operands at 2.4e-3 (class)
    / 1.8e-3 (box) from the fp32 oracle (the oracle with TF32-rounded operands, 2.8e-3 / 2.5e-3 at
    800x1024): the TF32 session's precision policy runs the contractions past the first 16 of such a
    chain as TF32x3, which meets the 2e-3 TF32 gate."""
    case = graphs.retinanet(batch=1, hw=(128, 160))
    got = _tf32(case)
    ref = run_oracle(case)
    for g, r, o in zip(got, ref, case.output_names):
        assert_close(g, r, tol=TF32_TOL, what=f"tf32 retinanet {o} vs fp32 oracle")


def test_precision_is_validated():
    with pytest.raises(ValueError):
        B200InferenceSessionFactory(precision="fp8")


# ---- TF32x3: error-compensated TF32 (x = hi + lo, hi*hi + hi*lo + lo*hi per K slice) ----------
X3_TOL = 5e-5   # single convs / GEMMs land at 1e-6 - 3e-5 (fp32-accumulation bound)


def _x3(case):
    return run_backend(case, factory=B200InferenceSessionFactory(num_devices=1, precision="tf32x3"))


@pytest.mark.parametrize("kw", [
    dict(c=64, cout=256, k=1, pads=[0, 0, 0, 0], bn=True, residual=True, relu=True),  # rows + residual
    dict(c=24, cout=40, k=3, h=11, w=7),                                           # gather
    dict(n=2, c=64, cout=64, k=3, h=32, w=32, bn=True, relu=True),                 # im2col
    dict(c=3, cout=64, k=7, stride=2, pads=[3, 3, 3, 3], h=32, w=32),              # stem
    dict(c=128, cout=64, k=1, pads=[0, 0, 0, 0], h=10, w=16, upsample_residual=True),
])
def test_tf32x3_conv(kw):
    case = conv_case(**kw)
    got = _x3(case)[0]
    assert_close(got, run_oracle(case)[0], tol=X3_TOL, what=f"tf32x3 conv {kw}")


def test_tf32x3_gemm():
    case = graphs.mlp(batch=513, widths=(1024, 4096, 100), seed=3, bias_scale=0.5)
    assert_close(_x3(case)[0], run_oracle(case)[0], tol=X3_TOL, what="tf32x3 mlp")


def test_tf32x3_retinanet_meets_the_tf32_gate():
    """The graph at the single-pass TF32 floor: with error-compensated TF32 both detection outputs
    meet the 2e-3 TF32 gate with margin (measured 4.5e-4 / 2.2e-4). Single convs land at 1e-6 -
    5e-6; what remains on deep graphs is the tensor core's fp32 accumulation, whose error grows
    with the reduction length (3e-5 on one K=4096 GEMM with exact hi / lo operands)."""
    case = graphs.retinanet(batch=1, hw=(128, 160))
    got = _x3(case)
    ref = run_oracle(case)
    for g, r, o in zip(got, ref, case.output_names):
        assert_close(g, r, tol=1e-3, what=f"tf32x3 retinanet {o} (2e-3 gate with margin)")
