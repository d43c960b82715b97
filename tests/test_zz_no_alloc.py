"""fc_matmul_noalloc - the matmul entry point for callers that cannot
allocate device memory (a process whose caching allocator already owns the
free memory, or a path that must not fail on out-of-memory).  It works in a
fixed device array instead of cudaMalloc; its results must equal fc_matmul's.

Collected last on purpose: it runs after every other test and also alone."""
import ctypes

import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu

FP = ctypes.POINTER(ctypes.c_float)


def weights(rng, fmt, O, K):
    if fmt == 1:
        values = rng.integers(-127, 128, size=(O, K), dtype=np.int8).view(np.uint8)
        bits = (np.uint16(3 << 10) | rng.integers(0, 1024, size=(O, K // 32)).astype(np.uint16))
        return values, bits
    nib = rng.integers(0, 16, size=(O, K), dtype=np.uint8)
    values = (nib[:, 0::2] | (nib[:, 1::2] << 4)).astype(np.uint8)
    if fmt == 2:
        bits = (np.uint16(7 << 10) | rng.integers(0, 1024, size=(O, K // 32)).astype(np.uint16))
    else:
        bits = rng.integers(118, 122, size=(O, K // 32)).astype(np.uint8)
    return values, bits


def call(fn, fmt, values, bits, x, O, K):
    S = x.shape[0]
    y = np.zeros((S, O), dtype=np.float32)
    err = ctypes.create_string_buffer(256)
    ok = fn(fmt, y.ctypes.data_as(FP), np.ascontiguousarray(x).ctypes.data_as(FP),
            values.ctypes.data_as(ctypes.c_void_p), bits.ctypes.data_as(ctypes.c_void_p),
            O, K, S, err, len(err))
    return ok, y, err.value


@pytest.mark.parametrize("fmt,O,K,S", [(1, 576, 2048, 4), (2, 100, 1408, 3), (3, 1024, 4096, 1)])
def test_noalloc_matches_fc_matmul_on_two_calls(fc, fmt, O, K, S):
    lib = fc.lib()
    for call_no in range(2):
        rng = np.random.default_rng(100 * fmt + call_no)
        values, bits = weights(rng, fmt, O, K)
        x = rng.standard_normal((S, K)).astype(np.float32)
        ok_ref, ref, e_ref = call(lib.fc_matmul, fmt, values, bits, x, O, K)
        ok, y, e = call(lib.fc_matmul_noalloc, fmt, values, bits, x, O, K)
        assert ok_ref, e_ref
        assert ok, e
        assert rel_l2(y, ref) < 1e-5, f"call {call_no}"


def test_noalloc_rejects_shapes_beyond_its_workspace(fc):
    lib = fc.lib()
    O, K = 4096, 4096  # a q8 image of ~17 MiB does not fit the fixed workspace
    values = np.zeros((O, K), dtype=np.uint8)
    bits = np.zeros((O, K // 32), dtype=np.uint16)
    x = np.zeros((1, K), dtype=np.float32)
    ok, _, e = call(lib.fc_matmul_noalloc, 1, values, bits, x, O, K)
    assert not ok and b"exceeds" in e


def test_noalloc_rejects_more_than_eight_rows(fc):
    lib = fc.lib()
    O, K, S = 64, 64, 9
    values = np.zeros((O, K), dtype=np.uint8)
    bits = np.zeros((O, K // 32), dtype=np.uint16)
    x = np.zeros((S, K), dtype=np.float32)
    ok, _, e = call(lib.fc_matmul_noalloc, 1, values, bits, x, O, K)
    assert not ok and b"8-row limit" in e
