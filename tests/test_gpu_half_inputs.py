"""GPU tests of 16-bit float graph inputs (the reference's CreateTensor<BFloat16 / Float16>,
src/Backend/OnnxRuntime/Shorokoo.OnnxRuntime/OrtSessionFactory.cs:46-55): the image crosses PCIe in
its 16-bit type (half the bytes of float32) and a Cast to float32 feeds the stem. bfloat16 inputs
are read directly by the stem's space-to-depth conversion, float16 ones are widened to float32 on the
device first.

The model with a 16-bit input must give exactly what the float32-input model gives on the same
values widened to float32 (the stem rounds its operand to bfloat16 either way), and match the
fp32 oracle at the bf16 gate; the batched case runs through Run's micro-batch pipeline decision."""
import numpy as np
import pytest

from helpers import BF16_TOL, assert_close, run_backend, run_oracle
from shorokoo_b200 import B200InferenceSessionFactory, ShorokooTensorElementType
from shorokoo_b200.emit import graphs

pytestmark = pytest.mark.gpu


def _run_16bit(case, dtype):
    name, x = case.inputs[-1]
    f = B200InferenceSessionFactory(num_devices=1)
    sess = f.CreateSession(case.model)
    if dtype == "bfloat16":
        bits = (np.ascontiguousarray(x, np.float32).view(np.uint32) >> 16).astype(np.uint16)
        v = f.CreateTensorFromRawBytes(ShorokooTensorElementType.BFloat16, bits.tobytes(), list(x.shape))
    else:
        v = f.CreateTensor(x.astype(np.float16))
    assert v.ElementType == {"bfloat16": ShorokooTensorElementType.BFloat16,
                             "float16": ShorokooTensorElementType.Float16}[dtype]
    outs = sess.Run({name: v}, case.output_names)
    got = outs[0].numpy()
    for o in outs:
        o.Dispose()
    sess.Dispose()
    return got


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
@pytest.mark.parametrize("batch,hw", [(3, (64, 64)), (256, (160, 160))])
def test_resnet18_with_16bit_image_input(dtype, batch, hw):
    case16 = graphs.resnet(depth=18, batch=batch, hw=hw, seed=5, input_dtype=dtype)
    got = _run_16bit(case16, dtype)
    # the float32-input model on the same (widened) values
    case32 = graphs.resnet(depth=18, batch=batch, hw=hw, seed=5)
    x16 = case16.inputs[-1][1]
    ref32 = run_backend(graphs.ModelCase(case32.name, case32.model, [(case32.inputs[-1][0], x16)],
                                         case32.output_names, case32.macs))[0]
    if batch < 8:   # one plan on both sides: bit for bit
        np.testing.assert_array_equal(got, ref32)
    else:           # Run may cut either batch into other chunk plans (other summation orders)
        assert_close(got, ref32, tol=BF16_TOL, what=f"{dtype} input vs float32 input")
    rows = np.r_[0:2, batch - 2:batch]
    sub = graphs.ModelCase(case16.name, case16.model, [(case16.inputs[-1][0], x16[rows])], case16.output_names, 0)
    assert_close(got[rows], run_oracle(sub)[0], tol=BF16_TOL, what=f"resnet18 {dtype} input vs oracle")
