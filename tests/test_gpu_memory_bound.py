"""GPU tests of the memory-bound kernels on their vectorised and per-element paths, against numpy.

* elementwise / strided copy: the host collapses the dimensions every operand walks contiguously
  and, when the innermost run is a multiple of 4 elements and aligned, each thread moves four
  elements with one 16-byte (fp32) access; broadcast operands (stride 0) are one load. Shapes below
  take both paths (innermost runs of 8, 12, 7, 1) and broadcasts along inner and outer axes.
* global average / max pool: 128-bit loads of 8 bf16 or 4 fp32 channels per pixel, warp-shuffle
  and shared-memory reduction; channel counts that are not a multiple of the vector width take the
  scalar kernel.

fp32 arithmetic of single ops: results are exact (copies, max) or within a few ulp (sums, sigmoid).
"""
import numpy as np
import pytest

from helpers import run_backend
from shorokoo_b200.emit import onnx_writer as W
from shorokoo_b200.emit.graphs import Builder, ModelCase

pytestmark = pytest.mark.gpu


def _binary_case(op, sa, sb, seed):
    rng = np.random.Generator(np.random.PCG64(seed))
    a = rng.standard_normal(sa, dtype=np.float32)
    b = rng.standard_normal(sb, dtype=np.float32) + (3.0 if op == "Div" else 0.0)
    B = Builder(seed)
    ai = B.graph_input(W.FLOAT, len(sa), sa)
    bi = B.graph_input(W.FLOAT, len(sb), sb)
    y = B.op(op, [ai, bi])
    B.outputs.append(W.ValueInfo(y))
    return ModelCase(op, B.model(op), [(ai, a), (bi, b)], [y], 0), a, b


@pytest.mark.parametrize("op,sa,sb", [
    ("Add", (2, 3, 4, 8), (1, 3, 1, 1)),        # per-channel broadcast, inner run 32
    ("Mul", (5, 12), (12,)),                     # row broadcast (stride 1 inner, 0 outer)
    ("Sub", (4, 6, 8), (4, 6, 1)),               # inner broadcast (stride 0 inner)
    ("Div", (3, 7), (3, 7)),                     # inner run 21: per-element path
    ("Max", (64, 1, 9), (1, 40, 1)),             # outer-product broadcast, inner run 9
    ("Add", (1000, 4), (1000, 4)),               # large, contiguous
])
def test_binary_elementwise(op, sa, sb):
    case, a, b = _binary_case(op, sa, sb, 11)
    got = run_backend(case)[0]
    ref = {"Add": np.add, "Mul": np.multiply, "Sub": np.subtract, "Div": np.divide, "Max": np.maximum}[op](a, b)
    np.testing.assert_allclose(got, ref, rtol=2e-7, atol=0)


@pytest.mark.parametrize("shape,perm", [((2, 3, 8, 16), [0, 2, 3, 1]), ((4, 5, 6), [2, 0, 1]), ((8, 12), [1, 0])])
def test_transpose_then_sigmoid(shape, perm):
    # Transpose is a view; Sigmoid reads it strided (innermost stride != 1) and writes contiguously.
    rng = np.random.Generator(np.random.PCG64(3))
    x = rng.standard_normal(shape, dtype=np.float32)
    B = Builder(3)
    xi = B.graph_input(W.FLOAT, len(shape), shape)
    y = B.op("Sigmoid", [B.op("Transpose", [xi], perm=perm)])
    B.outputs.append(W.ValueInfo(y))
    got = run_backend(ModelCase("t", B.model("t"), [(xi, x)], [y], 0))[0]
    ref = 1.0 / (1.0 + np.exp(-np.transpose(x, perm).astype(np.float64)))
    np.testing.assert_allclose(got, ref, rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("shapes,axis", [([(2, 5, 8), (2, 3, 8)], 1), ([(3, 4), (3, 6), (3, 2)], 1),
                                         ([(2, 3, 7), (2, 3, 5)], 2)])
def test_concat_copies(shapes, axis):
    rng = np.random.Generator(np.random.PCG64(4))
    xs = [rng.standard_normal(s, dtype=np.float32) for s in shapes]
    B = Builder(4)
    ins = [B.graph_input(W.FLOAT, len(s), s) for s in shapes]
    y = B.op("Concat", ins, axis=axis)
    B.outputs.append(W.ValueInfo(y))
    got = run_backend(ModelCase("c", B.model("c"), list(zip(ins, xs)), [y], 0))[0]
    np.testing.assert_array_equal(got, np.concatenate(xs, axis=axis))


@pytest.mark.parametrize("op", ["GlobalAveragePool", "GlobalMaxPool"])
@pytest.mark.parametrize("n,c,h,w", [(3, 64, 7, 7), (2, 2048, 7, 7), (2, 96, 5, 3), (2, 36, 4, 4), (1, 6, 3, 3)])
def test_global_pool(op, n, c, h, w):
    rng = np.random.Generator(np.random.PCG64(5))
    x = rng.standard_normal((n, c, h, w), dtype=np.float32)
    B = Builder(5)
    xi = B.graph_input(W.FLOAT, 4, x.shape)
    y = B.op(op, [xi])
    B.outputs.append(W.ValueInfo(y))
    got = run_backend(ModelCase("p", B.model("p"), [(xi, x)], [y], 0))[0]
    ref = x.astype(np.float64).mean((2, 3), keepdims=True) if op == "GlobalAveragePool" else x.max((2, 3), keepdims=True)
    assert got.shape == (n, c, 1, 1)
    np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-6)
