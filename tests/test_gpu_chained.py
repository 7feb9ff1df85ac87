"""GPU tests of device-resident outputs for chained runs (sb_session_run_device): a model's outputs
stay in device memory and feed the next model's Run device to device, with no host round trip. The
chained result must equal the same chain through host tensors, bit for bit (the same plans run on
the same values), and reading a device-resident value copies it to the host on demand."""
import numpy as np
import pytest

from helpers import assert_close, run_oracle
from shorokoo_b200 import B200InferenceSessionFactory
from shorokoo_b200.emit import graphs

pytestmark = pytest.mark.gpu


def test_chained_mlps_stay_on_the_device():
    a = graphs.mlp(batch=512, widths=(256, 512, 384), seed=11, bias_scale=0.5)
    b = graphs.mlp(batch=512, widths=(384, 256, 100), seed=12, bias_scale=0.5)
    f = B200InferenceSessionFactory(num_devices=1)
    sa, sb = f.CreateSession(a.model), f.CreateSession(b.model)
    xa = f.CreateTensor(a.inputs[0][1])
    # host path
    ha = sa.Run({a.inputs[0][0]: xa}, a.output_names)[0]
    hb = sb.Run({b.inputs[0][0]: ha}, b.output_names)[0].numpy()
    # device path: the intermediate never leaves the device
    da = sa.RunOnDevice({a.inputs[0][0]: xa}, a.output_names)[0]
    ptr, dev = da.DevicePointer
    assert ptr is not None and dev == 0
    db = sb.RunOnDevice({b.inputs[0][0]: da}, b.output_names)[0]
    assert db.DevicePointer[0] is not None
    np.testing.assert_array_equal(db.numpy(), hb)            # copied to the host on first read
    np.testing.assert_array_equal(da.numpy(), ha.numpy())
    # a device-resident input to the host-output Run as well
    hb2 = sb.Run({b.inputs[0][0]: da}, b.output_names)[0].numpy()
    np.testing.assert_array_equal(hb2, hb)
    # and the chain matches the oracle
    ref_a = run_oracle(a)[0]
    ref = run_oracle(graphs.ModelCase(b.name, b.model, [(b.inputs[0][0], ref_a)], b.output_names, 0))[0]
    assert_close(hb, ref, what="chained mlp vs oracle")
    for v in (xa, ha, da, db):
        v.Dispose()
