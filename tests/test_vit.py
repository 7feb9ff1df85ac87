"""Vision Transformer (samples/RetinaNet/ViTNet.cs: ViTTiny / ViTSmall / ViTBase) through the
backend: the exporter's primitives fuse into LayerNorm (ReduceMean / Sub / Pow / ReduceMean /
Add(eps) / Sqrt / Div / Mul / Add), Attention (MatMul(q, Transpose(k)) * scale -> Softmax ->
MatMul(., v), run by one tcgen05 kernel per 128-query tile and head) and FusedGemm epilogues with
the tanh-approximated GELU; the class token's Tile folds on the host.

Host side (no GPU): the fusion counts on ViT-Ti / ViT-S graphs, the oracle's Gelu and Tile.
GPU side: the attention kernel against float64 numpy over sequence lengths 1 to 256 (one and two
query tiles, ragged key counts), heads, batch, rank-3 operands; LayerNorm and GELU against numpy;
ViT-Ti (two blocks) against the oracle at the bf16 and TF32 gates; ViT-B/16 at its configured size
(batch 1, 224x224, 12 blocks) at the bf16 gate."""
import math

import numpy as np
import pytest

from helpers import BF16_TOL, assert_close, run_backend, run_oracle
from shorokoo_b200.emit import graphs
from shorokoo_b200.emit import onnx_writer as W
from shorokoo_b200.emit.graphs import Builder, ModelCase, _ViTLayerNormParams, vit_layer_norm
from test_native_host import kinds, lower


@pytest.mark.parametrize("variant,layers", [("tiny", 2), ("small", 1)])
def test_vit_fuses(variant, layers):
    lines = lower(graphs.vit(variant, layers=layers))
    k = kinds(lines)
    assert k["LayerNorm"] == 2 * layers + 1 and k["Attention"] == layers, k
    assert k["FusedGemm"] == 4 * layers + 1 and k["FusedConv"] == 1, k
    for op in ("Softmax", "ReduceMean", "Gelu", "MatMul", "Sqrt", "Pow", "Tile"):
        assert op not in k, (op, k)
    assert sum(1 for l in lines if l.startswith("FusedGemm") and "act=3" in l) == layers


def test_oracle_gelu_and_tile():
    B = Builder(3)
    x = np.linspace(-6, 6, 97, dtype=np.float32).reshape(1, 97)
    xi = B.graph_input(W.FLOAT, 2, x.shape)
    t = B.op("Gelu", [xi], approximate="tanh")
    e = B.op("Gelu", [xi])
    r = B.op("Tile", [xi, B.const(np.array([2, 1], np.int64))])
    B.outputs += [W.ValueInfo(t), W.ValueInfo(e), W.ValueInfo(r)]
    got = run_oracle(ModelCase("g", B.model("g"), [(xi, x)], [t, e, r], 0))
    w = x.astype(np.float64)
    np.testing.assert_allclose(got[0], 0.5 * w * (1 + np.tanh(math.sqrt(2 / math.pi) * (w + 0.044715 * w ** 3))),
                               rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(got[1], 0.5 * w * (1 + np.vectorize(math.erf)(w / math.sqrt(2))), rtol=1e-6, atol=1e-6)
    np.testing.assert_array_equal(got[2], np.tile(x, (2, 1)))


def _attention_case(b, h, s, hd=64, seed=7, rank=4, scale=None):
    rng = np.random.Generator(np.random.PCG64(seed))
    shape = (b, h, s, hd) if rank == 4 else (b, s, hd)
    q, k, v = (rng.standard_normal(shape, dtype=np.float32) for _ in range(3))
    B = Builder(seed)
    qi, ki, vi = (B.graph_input(W.FLOAT, rank, shape) for _ in range(3))
    perm = [0, 1, 3, 2] if rank == 4 else [0, 2, 1]
    kt = B.op("Transpose", [ki], perm=perm)
    sc = B.op("MatMul", [qi, kt])
    scale = 1.0 / math.sqrt(hd) if scale is None else scale
    sc = B.op("Mul", [sc, B.const(np.array(scale, np.float32))])
    p = B.op("Softmax", [sc], axis=-1)
    y = B.op("MatMul", [p, vi])
    B.outputs.append(W.ValueInfo(y))
    case = ModelCase("attn", B.model("attn"), [(qi, q), (ki, k), (vi, v)], [y], 0)
    s64 = np.einsum("...qd,...kd->...qk", q.astype(np.float64), k.astype(np.float64)) * scale
    s64 -= s64.max(-1, keepdims=True)
    p64 = np.exp(s64)
    p64 /= p64.sum(-1, keepdims=True)
    return case, np.einsum("...qk,...kd->...qd", p64, v.astype(np.float64))


def test_attention_fuses_standalone():
    case, _ = _attention_case(1, 2, 10)
    k = kinds(lower(case))
    assert k["Attention"] == 1 and "MatMul" not in k and "Softmax" not in k, k


@pytest.mark.gpu
@pytest.mark.parametrize("b,h,s,rank", [(1, 3, 197, 4), (2, 2, 1, 4), (1, 1, 7, 4), (1, 2, 128, 4),
                                        (1, 2, 129, 4), (2, 12, 256, 4), (3, 1, 50, 3)])
def test_attention_kernel(b, h, s, rank):
    case, ref = _attention_case(b, h, s, rank=rank)
    got = run_backend(case)[0]
    assert got.shape == ref.shape
    assert_close(got, ref, tol=BF16_TOL, what=f"attention b{b} h{h} s{s}")


@pytest.mark.gpu
def test_layer_norm_and_gelu_kernels():
    rng = np.random.Generator(np.random.PCG64(5))
    x = (rng.standard_normal((2, 37, 192), dtype=np.float32) * 3 + 1.5).astype(np.float32)
    B = Builder(5)
    xi = B.graph_input(W.FLOAT, 3, x.shape)
    p = _ViTLayerNormParams(B, 192, "ln", 0.2)
    y = vit_layer_norm(B, xi, p, 1e-6)
    g1 = B.op("Gelu", [xi], approximate="tanh")
    g2 = B.op("Gelu", [xi])
    B.outputs += [W.ValueInfo(y), W.ValueInfo(g1), W.ValueInfo(g2)]
    case = ModelCase("ln", B.model("ln"), [(xi, x)], [y, g1, g2], 0, B.params)
    got = run_backend(case)
    w = x.astype(np.float64)
    mu = w.mean(-1, keepdims=True)
    ln = (w - mu) / np.sqrt(((w - mu) ** 2).mean(-1, keepdims=True) + 1e-6) * B.params["ln.weight"] + B.params["ln.bias"]
    np.testing.assert_allclose(got[0], ln, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(got[1], 0.5 * w * (1 + np.tanh(math.sqrt(2 / math.pi) * (w + 0.044715 * w ** 3))),
                               rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(got[2], 0.5 * w * (1 + np.vectorize(math.erf)(w / math.sqrt(2))), rtol=1e-5, atol=1e-6)


@pytest.mark.gpu
@pytest.mark.parametrize("variant,layers,prec,tol", [("tiny", 2, "bf16", BF16_TOL), ("tiny", 2, "tf32", 2e-3),
                                                     ("small", 1, "bf16", BF16_TOL)])
def test_vit_blocks(variant, layers, prec, tol):
    from shorokoo_b200 import B200InferenceSessionFactory
    case = graphs.vit(variant, layers=layers, affine_scale=0.1)
    got = run_backend(case, factory=B200InferenceSessionFactory(num_devices=1, precision=prec))[0]
    assert_close(got, run_oracle(case)[0], tol=tol, what=f"ViT-{variant} {layers} blocks ({prec})")


@pytest.mark.gpu
def test_vit_base_full_size():
    case = graphs.build("vit_base")
    got = run_backend(case)[0]
    e = assert_close(got, run_oracle(case)[0], tol=BF16_TOL, what="ViT-B/16 batch 1 224x224")
    print(f"ViT-B/16: normwise error {e:.2e} (gate 1e-2)")
