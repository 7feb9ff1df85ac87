"""Multi-GPU parity: a session over two devices shards the batch (contiguous dim-0 slices, weights
replicated, no collective) and must return the single-device result up to summation order (a
shard may pick another tile width and split of K across MMA lanes), which matches the oracle. Skipped when fewer than two GPUs are visible."""
import numpy as np
import pytest

from helpers import assert_close, run_backend, run_oracle
from shorokoo_b200.emit import graphs

pytestmark = pytest.mark.gpu


def _gpus():
    import torch
    return torch.cuda.device_count()


@pytest.mark.parametrize("case_fn", [
    lambda: graphs.resnet(depth=18, batch=6, hw=(64, 64), seed=5),
    lambda: graphs.mlp(batch=301, widths=(256, 512, 128), seed=4, bias_scale=0.5),
])
def test_two_device_shards_match_one_device(case_fn):
    if _gpus() < 2:
        pytest.skip("needs two GPUs")
    case = case_fn()
    one = run_backend(case, num_devices=1)
    two = run_backend(case, num_devices=2)
    ref = run_oracle(case)
    for a, b, r in zip(one, two, ref):
        assert a.shape == b.shape == r.shape
        assert_close(b, a, what="two-device shards vs one device")
        assert_close(b, r, what="two-device shards vs oracle")
