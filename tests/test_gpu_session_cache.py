"""GPU test of the process-wide session cache: ComputeContext.Execute creates a new session per call
(ComputeContext.cs:318-359), so a second session on the same model bytes (and options) must share
the first one's plans, give the same results, and count once in the cache; a different model or
precision is a separate entry."""
import numpy as np
import pytest

from helpers import run_backend
from shorokoo_b200 import B200InferenceSessionFactory
from shorokoo_b200.emit import graphs

pytestmark = pytest.mark.gpu


def test_same_model_bytes_share_one_cached_session():
    F = B200InferenceSessionFactory(num_devices=1)
    F.ClearSessionCache()
    a = graphs.mlp(batch=64, widths=(128, 256, 64), seed=21, bias_scale=0.5)
    b = graphs.mlp(batch=64, widths=(128, 256, 32), seed=22, bias_scale=0.5)
    r1 = run_backend(a, factory=F)[0]          # creates, runs, disposes its handle
    r2 = run_backend(a, factory=F)[0]          # same bytes: the cached session
    r3 = run_backend(b, factory=F)[0]
    assert np.array_equal(r1, r2)
    assert r3.shape == (64, 32)
    assert F.ClearSessionCache() == 2          # a and b, a counted once
    assert F.ClearSessionCache() == 0


def test_precision_is_part_of_the_cache_key():
    F16 = B200InferenceSessionFactory(num_devices=1, precision="bf16")
    F32 = B200InferenceSessionFactory(num_devices=1, precision="tf32")
    F16.ClearSessionCache()
    a = graphs.mlp(batch=64, widths=(128, 256, 64), seed=23, bias_scale=0.5)
    g16 = run_backend(a, factory=F16)[0]
    g32 = run_backend(a, factory=F32)[0]
    assert not np.array_equal(g16, g32)        # different operand precision, different plans
    assert F16.ClearSessionCache() == 2
