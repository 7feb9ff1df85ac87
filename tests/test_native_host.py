"""Host-side tests of the native library (no GPU needed): the C ABI loads and exports exactly what
include/shorokoo_b200.h declares, host tensor values behave like IShorokooTensorValue, the plan-time
lowering resolves the reference's emission quirks (shape chains, live-[Hyper] If / Loop, dead
initializers, FrozenBatchNorm folding, Pad folding, head Reshape/Transpose views), and failures are
reported as the plugin contract requires (unsupported op = hard error at CreateSession)."""
import ctypes as C
import re
import subprocess

import numpy as np
import pytest

from shorokoo_b200 import (B200ArgumentError, B200InferenceSessionFactory, B200InvalidOperationError,
                           B200NotSupportedError, ShorokooOnnxValueType, ShorokooTensorElementType, _native)
from shorokoo_b200.emit import graphs
from shorokoo_b200.emit import onnx_writer as W
from shorokoo_b200.emit.graphs import Builder

F = B200InferenceSessionFactory()


def test_library_exports_exactly_the_header():
    out = subprocess.run(["nm", "-D", "--defined-only", _native.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = sorted(set(re.findall(r" T (sb_\w+)", out)))
    assert exported == _native.header_symbols()
    lib = _native.lib()
    for name in _native.header_symbols():
        assert hasattr(lib, name)
    assert lib.sb_version() >= 100


def test_tensor_values_roundtrip():
    a = np.arange(24, dtype=np.float32).reshape(2, 3, 4)
    v = F.CreateTensor(a)
    assert v.ValueType == ShorokooOnnxValueType.Tensor
    assert v.ElementType == ShorokooTensorElementType.Float
    assert v.Shape == [2, 3, 4]
    np.testing.assert_array_equal(v.GetTensorDataAsSpan(), a)
    v.GetTensorMutableDataAsSpan()[0, 0, 0] = 7
    assert v.GetTensorDataAsSpan()[0, 0, 0] == 7
    s = F.CreateTensor(np.array(3, np.int64))
    assert s.Shape == [] and s.GetTensorDataAsSpan() == 3
    r = F.CreateTensorFromRawBytes(ShorokooTensorElementType.BFloat16, b"\x80\x3f\x00\x40", [2])
    assert r.ElementType == ShorokooTensorElementType.BFloat16 and r.Shape == [2]
    st = F.CreateStringTensor(["a", "bc", ""], [3])
    assert st.GetStringTensorData() == ["a", "bc", ""]
    seq = F.CreateSequence([F.CreateTensor(np.zeros(2, np.int64)), F.CreateTensor(np.ones(3, np.int64))])
    assert seq.ValueType == ShorokooOnnxValueType.Sequence and seq.GetValueCount() == 2
    assert seq.GetSequenceElementType() == ShorokooTensorElementType.Int64
    assert seq.GetValue(1).Shape == [3]
    with pytest.raises(B200ArgumentError):
        F.CreateTensor(np.zeros(6, np.float32), [4])
    with pytest.raises(B200NotSupportedError):
        F.CreateTensorFromRawBytes(ShorokooTensorElementType.String, b"", [0])


def lower(case, inputs=None):
    vals = [F.CreateTensor(a) for _, a in (inputs or case.inputs)]
    arr = (C.c_void_p * max(len(vals), 1))(*[v._h.value for v in vals])
    buf = C.create_string_buffer(1 << 22)
    need = C.c_size_t()
    st = _native.lib().sb_debug_lower(case.model, len(case.model), len(vals), arr, buf, len(buf), C.byref(need))
    if st:
        raise RuntimeError(_native.lib().sb_last_error().decode())
    lines = buf.value.decode().strip().split("\n")
    return lines


def kinds(lines):
    from collections import Counter
    return Counter(l.split()[0] for l in lines if not l.startswith(("output", "separable")))


def test_lowering_resnet50_fuses_everything():
    lines = lower(graphs.resnet(depth=50, batch=2, hw=(64, 64)))
    k = kinds(lines)
    # 53 convs, less the four projection shortcuts (1x1, stride 1 in stage 1 and 2 after it), each
    # merged into the conv that adds it
    assert k == {"FusedConv": 49, "MaxPool": 1, "GlobalAveragePool": 1, "Reshape": 1, "FusedGemm": 1}, k
    stem = [l for l in lines if l.startswith("FusedConv")][0]
    assert "k=7x7 s=2 pads=[3,3,3,3]" in stem and "act=1" in stem   # Pad folded, BN folded, ReLU fused
    assert sum("residual=0" in l for l in lines) == 12                # one residual add per other bottleneck
    merged = [l for l in lines if "concat" in l]
    assert len(merged) == 4 and all("k=1x1 s=1" in l and "act=1" in l for l in merged), merged
    assert sum("concat/1" in l for l in merged) == 1 and sum("concat/2" in l for l in merged) == 3
    assert lines[-1] == "separable=1"


def test_lowering_live_hypers_and_dead_code():
    case = graphs.resnet(depth=50, batch=2, hw=(64, 64), live_hypers=True, dead_code=True)
    k = kinds(lower(case))
    assert k["FusedConv"] == 49 and k["FusedGemm"] == 1      # dead shortcut convs pruned
    case = graphs.resnet(depth=18, batch=2, hw=(64, 64), live_hypers=True, apply_softmax=True)
    assert kinds(lower(case))["Softmax"] == 1
    # includeTop=false drops the head entirely
    case = graphs.resnet(depth=18, batch=2, hw=(64, 64), live_hypers=True, include_top=False)
    k = kinds(lower(case))
    assert "FusedGemm" not in k and k["GlobalAveragePool"] == 1


def test_lowering_unrolls_live_loop():
    case = graphs.stacked_linear(batch=8, n=64, depth=5, live_depth=True)
    k = kinds(lower(case))
    assert k["FusedGemm"] == 5
    # a different trip count gives a different plan
    inputs = [(case.inputs[0][0], np.array(2, np.int64)), case.inputs[1]]
    assert kinds(lower(case, inputs))["FusedGemm"] == 2


def test_lowering_retinanet_heads_are_views():
    lines = lower(graphs.retinanet(batch=1, hw=(128, 160)))
    k = kinds(lines)
    assert k["FusedConv"] == 107                             # (the backbone's four shortcuts merged)
    assert sum("residual=1" in l for l in lines) == 2        # FPN top-down adds with nearest-2x upsample
    assert k["Concat"] == 2 and k["Sigmoid"] == 0
    # the class Sigmoid after the concat is applied by the five class-logit convs' epilogues
    assert sum(",720," in l.split("->")[1] and "act=2" in l for l in lines if l.startswith("FusedConv")) == 5
    assert [l for l in lines if l.startswith("output")] == ["output [1,3852,80] device", "output [1,3852,4] device"]


def test_unsupported_operator_is_a_hard_error_at_create_session():
    B = Builder(0)
    x = B.graph_input(W.FLOAT, 2, (2, 2))
    y = B.op("NonMaxSuppression", [x])
    B.outputs.append(W.ValueInfo(y))
    with pytest.raises(B200NotSupportedError, match="NonMaxSuppression"):
        F.CreateSession(B.model("bad"))


@pytest.mark.parametrize("blob", [b"", b"\x0a\xff\xff\xff\xff\x0f", b"\x3a\x05abc", bytes(range(7, 40))])
def test_malformed_model_bytes(blob):
    with pytest.raises((B200ArgumentError, B200NotSupportedError)):
        F.CreateSession(blob)


def test_truncated_model():
    case = graphs.stacked_linear(batch=2, n=8, depth=2)
    with pytest.raises(B200ArgumentError):
        F.CreateSession(case.model[: len(case.model) // 2])


def test_precision_argument_is_validated_before_any_device_work():
    import ctypes as C
    from shorokoo_b200 import _native
    case = graphs.stacked_linear(batch=2, n=8, depth=2)
    out = C.c_void_p()
    st = _native.lib().sb_session_create_ex(case.model, len(case.model), 0, 0, 0, 0, 7, C.byref(out))
    assert st == 1 and out.value is None
    assert "precision" in _native.lib().sb_last_error().decode()
    with pytest.raises(ValueError):
        B200InferenceSessionFactory(precision="fp16")


def test_no_gpu_reports_cuda_error():
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    case = graphs.stacked_linear(batch=2, n=8, depth=2)
    with pytest.raises(B200InvalidOperationError, match="CUDA"):
        F.CreateSession(case.model)


def test_shape_errors_at_lowering():
    case = graphs.mlp(batch=4, widths=(16, 8))
    bad = [(case.inputs[0][0], np.zeros((4, 15), np.float32))]
    with pytest.raises(RuntimeError, match="inner dimensions|MatMul"):
        lower(case, bad)


def _bottleneck(c=128, cmid=64, cout=256, stride=2, h=15, w=13, shortcut_relu=False, shortcut_output=False):
    from shorokoo_b200.emit import onnx_writer as W
    from shorokoo_b200.emit.graphs import Builder, ModelCase, kaiming_normal

    def conv(B, x, cin, co, k, s=1, relu=False, res=None):
        wt = B.init(kaiming_normal(B.rng, (co, cin, k, k)), "w")
        b = B.init(np.zeros(co, np.float32), "b")
        y = B.op("Conv", [x, wt, b], auto_pad="NOTSET", dilations=[1, 1], group=1, kernel_shape=[k, k],
                 pads=[k // 2] * 4, strides=[s, s])
        if res is not None:
            y = B.op("Add", [y, res])
        return B.op("Relu", [y]) if relu else y

    x = np.zeros((2, c, h, w), np.float32)
    B = Builder(5)
    xi = B.graph_input(W.FLOAT, 4, x.shape)
    ho, wo = (h - 1) // stride + 1, (w - 1) // stride + 1
    a = conv(B, xi, c, cmid, 1, relu=True)
    bb = conv(B, a, cmid, cmid, 3, s=stride, relu=True)
    sc = conv(B, xi, c, cout, 1, s=stride, relu=shortcut_relu)
    y = conv(B, bb, cmid, cout, 1, relu=True, res=sc)
    for t, ch, hh, ww in ((a, cmid, h, w), (bb, cmid, ho, wo), (sc, cout, ho, wo), (y, cout, ho, wo)):
        B.shape[t] = (2, ch, hh, ww)
    B.outputs.append(W.ValueInfo(y))
    outs = [y]
    if shortcut_output:
        B.outputs.append(W.ValueInfo(sc))
        outs.append(sc)
    return ModelCase("bottleneck", B.model("bottleneck"), [(xi, x)], outs, 0)


# The projection shortcut is merged into the conv that adds it only when that is exact and the
# kernel can read both operands in whole k-tiles.
@pytest.mark.parametrize("kw,merged", [
    (dict(), True),                              # stride-2 shortcut over an odd-sized map
    (dict(stride=1, h=12, w=10), True),
    (dict(shortcut_output=True), False),         # the shortcut's output is also a graph output
    (dict(c=96), False),                         # 96 input channels: not whole 64-channel k-tiles
    (dict(cmid=48), False),
    (dict(shortcut_relu=True), False),           # an activation of its own: not a linear term
])
def test_projection_shortcut_merge_conditions(kw, merged):
    lines = lower(_bottleneck(**kw))
    k = kinds(lines)
    got = [l for l in lines if "concat" in l]
    assert bool(got) == merged, lines
    assert k["FusedConv"] == (3 if merged else 4), k
