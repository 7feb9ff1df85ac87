"""GPU test of sb_linear_noalloc, the Linear entry point for callers that cannot allocate device
memory (pre-budgeted device memory, a host runtime that owns the allocator, allocation-free hot
loops). It must give the same result as the session path (sb_session_run on the equivalent ONNX
Linear) for two calls in a row, since every call reuses the same fixed scratch array.

This file is collected last on purpose, so a run that stops at the first failure has already run
every other test."""
import ctypes as C

import numpy as np
import pytest

from helpers import BF16_TOL, assert_close, run_backend
from shorokoo_b200 import _native
from shorokoo_b200.emit import graphs

pytestmark = pytest.mark.gpu


def _noalloc(x, w, b, relu):
    import torch
    dev = torch.device("cuda:0")
    xt = torch.from_numpy(x).to(dev)
    wt = torch.from_numpy(w).to(dev)
    bt = torch.from_numpy(b).to(dev)
    yt = torch.full((x.shape[0], w.shape[0]), float("nan"), device=dev)
    torch.cuda.synchronize()
    st = _native.lib().sb_linear_noalloc(C.c_void_p(xt.data_ptr()), C.c_void_p(wt.data_ptr()),
                                         C.c_void_p(bt.data_ptr()), C.c_void_p(yt.data_ptr()),
                                         x.shape[0], x.shape[1], w.shape[0], int(relu), None)
    assert st == 0, _native.lib().sb_last_error().decode()
    return yt.cpu().numpy()


def test_noalloc_linear_matches_session_path_twice():
    for m, k, n, relu, seed in ((300, 200, 100, False, 3), (64, 512, 1000, True, 4)):
        case = graphs.mlp(batch=m, widths=(k, n), seed=seed, bias_scale=0.5)
        ref = run_backend(case)[0]
        if relu:
            ref = np.maximum(ref, 0)
        x = case.inputs[0][1]
        got = _noalloc(x, case.params["layers.0.weight"], case.params["layers.0.bias"], relu)
        assert got.shape == ref.shape
        assert_close(got, ref, tol=BF16_TOL, what=f"noalloc linear {m}x{k}->{n}")


def test_noalloc_linear_rejects_sizes_beyond_scratch():
    st = _native.lib().sb_linear_noalloc(C.c_void_p(16), C.c_void_p(16), None, C.c_void_p(16),
                                         1 << 20, 4096, 4096, 0, None)
    assert st == 1
    assert "scratch" in _native.lib().sb_last_error().decode()
