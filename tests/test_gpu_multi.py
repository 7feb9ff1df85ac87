"""Multi-GPU parity of one session over two devices (SHOROKOO_B200_DEVICES / num_devices=2): the
batch is sharded (contiguous dim-0 slices, weights replicated, no collective), each shard's plan
runs on its own device from its own host thread, and the result must be the single-device one up to
summation order (a shard may pick another tile width and split of K across MMA lanes), which
matches the oracle.

Inputs wrapped from pageable memory (WrapTensor, as CreateTensor<T> aliases a managed array) are
staged per device through that device's own page-locked slots, narrowed to bf16 when the plan only
reads them as bf16: bit-identical to the pinned-input run. A batch whose shards carry 32 MiB of
copies or more is cut per shard into micro-batch chunks when the measured schedule model says so.
Skipped when fewer than two GPUs are visible."""
import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest

from helpers import BF16_TOL, assert_close, run_backend, run_oracle
from shorokoo_b200.emit import graphs

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _gpus():
    import torch
    return torch.cuda.device_count()


def _need_two():
    if _gpus() < 2:
        pytest.skip("needs two GPUs")


@pytest.mark.parametrize("case_fn", [
    lambda: graphs.resnet(depth=18, batch=6, hw=(64, 64), seed=5),
    lambda: graphs.mlp(batch=301, widths=(256, 512, 128), seed=4, bias_scale=0.5),
])
def test_two_device_shards_match_one_device(case_fn):
    _need_two()
    case = case_fn()
    one = run_backend(case, num_devices=1)
    two = run_backend(case, num_devices=2)
    ref = run_oracle(case)
    for a, b, r in zip(one, two, ref):
        assert a.shape == b.shape == r.shape
        assert_close(b, a, what="two-device shards vs one device")
        assert_close(b, r, what="two-device shards vs oracle")


def test_all_visible_devices_shard_and_match_one_device():
    """Every visible GPU (up to 8): ResNet-18 batch 13 (ragged shards) and the MLP, against one
    device and the oracle."""
    n = min(_gpus(), 8)
    if n < 3:
        pytest.skip("needs three or more GPUs")
    for case in (graphs.resnet(depth=18, batch=13, hw=(64, 64), seed=6),
                 graphs.mlp(batch=1001, widths=(256, 512, 128), seed=4, bias_scale=0.5)):
        one = run_backend(case, num_devices=1)
        many = run_backend(case, num_devices=n)
        ref = run_oracle(case)
        for a, b, r in zip(one, many, ref):
            assert a.shape == b.shape == r.shape
            assert_close(b, a, what=f"{n}-device shards vs one device")
            assert_close(b, r, what=f"{n}-device shards vs oracle")


def _run(case, num_devices, wrap):
    from shorokoo_b200 import B200InferenceSessionFactory
    f = B200InferenceSessionFactory(num_devices=num_devices)
    sess = f.CreateSession(case.model)
    feeds = {n: (f.WrapTensor(a) if wrap else f.CreateTensor(a)) for n, a in case.inputs}
    assert sess.stats(feeds)["devices"] == num_devices
    outs = sess.Run(feeds, case.output_names)
    got = [o.numpy() for o in outs]
    h2d, _ = sess.transfer_bytes(feeds)
    for o in outs:
        o.Dispose()
    for v in feeds.values():
        v.Dispose()
    sess.Dispose()
    return got, h2d


def test_two_device_wrapped_pageable_input_is_staged_per_device():
    _need_two()
    case = graphs.resnet(depth=18, batch=10, hw=(96, 96), seed=8)
    pinned, h_pinned = _run(case, 2, wrap=False)
    wrapped, h_wrapped = _run(case, 2, wrap=True)
    x = case.inputs[-1][1]
    assert h_pinned == x.nbytes and h_wrapped == x.nbytes // 2   # narrowed to bf16 while staged
    for a, b in zip(pinned, wrapped):
        np.testing.assert_array_equal(b, a)
    rows = np.r_[0:2, 8:10]
    sub = graphs.ModelCase(case.name, case.model, [(case.inputs[-1][0], x[rows])], case.output_names, 0)
    assert_close(wrapped[0][rows], run_oracle(sub)[0], what="two-device wrapped input vs oracle")


CHILD = textwrap.dedent("""
    import os, sys
    import numpy as np
    sys.path.insert(0, {root!r})
    from shorokoo_b200 import B200InferenceSessionFactory
    from shorokoo_b200.emit import graphs
    case = {case}
    res = []
    for nd in (1, 2):
        f = B200InferenceSessionFactory(num_devices=nd)
        sess = f.CreateSession(case.model)
        feeds = {{n: f.WrapTensor(a) for n, a in case.inputs}}
        outs = sess.Run(feeds, case.output_names)
        res.append(outs[0].numpy())
        for o in outs:
            o.Dispose()
        sess.Dispose()
    np.save(os.path.join({out!r}, "one.npy"), res[0])
    np.save(os.path.join({out!r}, "two.npy"), res[1])
""")


def test_two_device_shards_cut_into_chunks(tmp_path):
    """MLP bs16384 (64 MB of input, 16 MB of output): each 8192-row shard carries 40 MB of copies
    and is cut into 1024 + 1024 + 3072 + 3072-row chunks on its own device, when the schedule model
    (measured on that device) says that beats one piece."""
    _need_two()
    expr = "graphs.mlp(batch=16384, widths=(1024, 512, 256), seed=7, bias_scale=0.5)"
    code = CHILD.format(root=ROOT, case=expr, out=str(tmp_path))
    env = dict(os.environ, SHOROKOO_B200_DEBUG="1")
    env.pop("SHOROKOO_B200_PIPELINE", None)
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    log = r.stderr
    for d in (0, 1):
        assert f"(device {d})" in log, log[-2000:]
    one, two = np.load(tmp_path / "one.npy"), np.load(tmp_path / "two.npy")
    print([l for l in log.splitlines() if "pipeline" in l or "staging" in l])
    assert one.shape == two.shape
    assert_close(two, one, tol=BF16_TOL, what="two-device chunked shards vs one device")
    case = graphs.mlp(batch=16384, widths=(1024, 512, 256), seed=7, bias_scale=0.5)
    rows = np.r_[0:3, 8190:8194, 16381:16384]   # both ends and the shard seam
    sub = graphs.ModelCase(case.name, case.model, [(case.inputs[-1][0], case.inputs[-1][1][rows])],
                           case.output_names, 0)
    assert_close(two[rows], run_oracle(sub)[0], tol=BF16_TOL, what="two-device chunked shards vs oracle")
