"""The host-side float32 -> bfloat16 narrowing a Run applies while staging a pageable float32 input
that the plan only reads as bfloat16 (sb_debug_narrow_bf16 runs the same code: AVX2 with
non-temporal stores where the CPU has it, scalar heads and tails). It must equal the device's own
rounding of a float32 operand, round to nearest even, bit for bit, so that a narrowed batch gives
the same results as the float32 one: checked against numpy integer arithmetic on ties, carries into
the exponent, overflow to infinity, denormals, signed zeros, infinities and NaNs (quieted, sign and
upper payload kept), for lengths and offsets that leave unaligned heads and ragged tails, over one
and several threads."""
import ctypes as C

import numpy as np
import pytest

from shorokoo_b200 import _native


def _expected(x: np.ndarray) -> np.ndarray:
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF
    nan = ((u & 0x7F800000) == 0x7F800000) & ((u & 0x007FFFFF) != 0)
    return np.where(nan, (u >> 16) | 0x40, r).astype(np.uint16)


def _narrow(x: np.ndarray, threads: int, dst_offset: int = 0) -> np.ndarray:
    buf = np.zeros(x.size + dst_offset + 8, np.uint16)
    out = buf[dst_offset:dst_offset + x.size]
    st = _native.lib().sb_debug_narrow_bf16(x.ctypes.data_as(C.c_void_p), out.ctypes.data_as(C.c_void_p),
                                            x.size, threads)
    assert st == 0
    assert not buf[dst_offset + x.size:].any()   # nothing written past the end
    return out.copy()


def _special():
    bits = np.array([
        0x00000000, 0x80000000,                 # signed zeros
        0x3F808000, 0x3F818000,                 # ties: even stays, odd rounds up
        0x3F807FFF, 0x3F808001,                 # just below / above a tie
        0x3FFFFFFF, 0x7F7FFFFF,                 # carry into the exponent; largest finite -> inf
        0x7F800000, 0xFF800000,                 # infinities
        0x7FC00000, 0xFFC00001, 0x7F800001,     # NaNs (the signalling one is quieted)
        0x7FBF0000, 0x00000001, 0x00008000,     # denormals (a tie at the smallest)
        0x00018000, 0x807FFFFF, 0x00400000,
    ], np.uint32)
    return bits.view(np.float32)


@pytest.mark.parametrize("threads", [1, 4])
def test_special_values(threads):
    x = np.tile(_special(), 7)   # 133 values: vector body plus a scalar tail
    np.testing.assert_array_equal(_narrow(x, threads), _expected(x))


@pytest.mark.parametrize("n,dst_offset", [(1, 0), (15, 0), (16, 0), (17, 3), (1000, 5), (4096 + 13, 1)])
def test_unaligned_heads_and_ragged_tails(n, dst_offset):
    rng = np.random.Generator(np.random.PCG64(n))
    x = rng.integers(0, 2**32, n, dtype=np.uint64).astype(np.uint32).view(np.float32)
    np.testing.assert_array_equal(_narrow(x, 1, dst_offset), _expected(x))


def test_large_batch_over_threads():
    # 3 Mi values: pieces of 1 Mi per thread
    rng = np.random.Generator(np.random.PCG64(3))
    x = rng.standard_normal(3 * 2**20 + 77, dtype=np.float32)
    x[::1001] = _special()[np.arange(x[::1001].size) % _special().size]
    np.testing.assert_array_equal(_narrow(x, 16), _expected(x))
