"""GPU test of sb_linear_noalloc, the Linear entry point for callers that cannot allocate device
memory (pre-budgeted device memory, a host runtime that owns the allocator, allocation-free hot
loops). Its result is checked against a numpy GEMM over the same bf16-rounded operands with fp32
accumulation (the arithmetic of the bf16 tensor-core path), independent of the library's own
session path. Every call reuses the same fixed scratch array, so the calls run back to back: a
large layer, then a ragged one (K and N not multiples of 8 or 4, no bias, so the row-store epilogue
and the zero padding of the reduction are exercised) whose scratch still holds the first call's
operands, then the large layer again. It is also checked against the library's session entry point
(a one-layer MLP model run through a session) on two calls in a row.

This file is collected last on purpose, so a run that stops at the first failure has already run
every other test."""
import ctypes as C

import numpy as np
import pytest

from helpers import BF16_TOL, assert_close
from shorokoo_b200 import _native

pytestmark = pytest.mark.gpu


def _bf16(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).bfloat16().float().numpy()


def _expected(x, w, b, relu):
    y = _bf16(x).astype(np.float64) @ _bf16(w).astype(np.float64).T
    if b is not None:
        y = y + b
    return np.maximum(y, 0) if relu else y


def _noalloc(x, w, b, relu):
    import torch
    dev = torch.device("cuda:0")
    xt = torch.from_numpy(x).to(dev)
    wt = torch.from_numpy(w).to(dev)
    bt = torch.from_numpy(b).to(dev) if b is not None else None
    yt = torch.full((x.shape[0], w.shape[0]), float("nan"), device=dev)
    torch.cuda.synchronize()
    st = _native.lib().sb_linear_noalloc(C.c_void_p(xt.data_ptr()), C.c_void_p(wt.data_ptr()),
                                         C.c_void_p(bt.data_ptr()) if bt is not None else None,
                                         C.c_void_p(yt.data_ptr()), x.shape[0], x.shape[1], w.shape[0],
                                         int(relu), None)
    assert st == 0, _native.lib().sb_last_error().decode()
    return yt.cpu().numpy()


def _layer(m, k, n, bias, seed):
    rng = np.random.Generator(np.random.PCG64(seed))
    x = rng.standard_normal((m, k), dtype=np.float32)
    w = (rng.standard_normal((n, k), dtype=np.float32) / np.sqrt(k)).astype(np.float32)
    b = (0.5 * rng.standard_normal(n)).astype(np.float32) if bias else None
    return x, w, b


def test_noalloc_linear_matches_bf16_gemm_on_consecutive_calls():
    calls = [((300, 200, 100), True, False, 3), ((37, 13, 7), False, True, 4), ((64, 512, 1000), True, True, 5),
             ((300, 200, 100), True, False, 3)]
    for (m, k, n), bias, relu, seed in calls:
        x, w, b = _layer(m, k, n, bias, seed)
        got = _noalloc(x, w, b, relu)
        ref = _expected(x, w, b, relu)
        assert got.shape == ref.shape
        assert np.all(np.isfinite(got)), f"{m}x{k}->{n}: rows or columns left unwritten"
        assert_close(got, ref, tol=BF16_TOL, what=f"noalloc linear {m}x{k}->{n} bias={bias} relu={relu}")
        # fp32 accumulation of exact bf16 products: far tighter than the bf16 gate
        assert np.abs(got - ref).max() <= 1e-4 * max(1.0, float(np.abs(ref).max())), f"{m}x{k}->{n}"


@pytest.mark.parametrize("m,k,n", [(300, 200, 100), (513, 1024, 1000)])
def test_noalloc_linear_matches_the_session_entry_point(m, k, n):
    """The same layer through a session (sb_session_run over a one-layer MLP model whose weights are
    known) and through sb_linear_noalloc, twice in a row, within the bf16 gate of the other GPU tests."""
    from helpers import run_backend
    from shorokoo_b200.emit import graphs
    case = graphs.mlp(batch=m, widths=(k, n), seed=11, bias_scale=0.5)
    x = case.inputs[0][1]
    w, b = case.params["layers.0.weight"], case.params["layers.0.bias"]
    ref = run_backend(case)[0]
    for _ in range(2):
        got = _noalloc(x, w, b, False)
        assert_close(got, ref, tol=BF16_TOL, what=f"noalloc vs session linear {m}x{k}->{n}")


def test_noalloc_linear_rejects_sizes_beyond_scratch():
    st = _native.lib().sb_linear_noalloc(C.c_void_p(16), C.c_void_p(16), None, C.c_void_p(16),
                                         1 << 20, 4096, 4096, 0, None)
    assert st == 1
    assert "scratch" in _native.lib().sb_last_error().decode()
