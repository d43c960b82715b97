"""Dequant-GEMV kernel parity: fc_matmul (CUDA, through the C ABI) against the
oracle's fp32 restatement on the same logical weights (the test shape of
tests/test_backend_metal.c:39-79: random weights, random x, several rows),
including K that is not a multiple of the 64/128-column chunk and row
counts that leave a partial 32-row tile."""
import ctypes

import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu


def make_weights(rng, fmt, O, K):
    if fmt == 1:  # Q8
        values = rng.integers(-127, 128, size=(O, K), dtype=np.int8)
        packed = values.view(np.uint8)
        bits = (np.uint16(3 << 10) | rng.integers(0, 1024, size=(O, K // 32)).astype(np.uint16))
        scales = bits.view(np.float16).astype(np.float32)
        return values, packed, bits, scales
    nib = rng.integers(0, 16, size=(O, K), dtype=np.uint8)
    packed = (nib[:, 0::2] | (nib[:, 1::2] << 4)).astype(np.uint8)
    if fmt == 2:  # Q4
        values = (nib.astype(np.int16) - 8).astype(np.int8)
        bits = (np.uint16(7 << 10) | rng.integers(0, 1024, size=(O, K // 32)).astype(np.uint16))
        scales = bits.view(np.float16).astype(np.float32)
        return values, packed, bits, scales
    values = nib.astype(np.int8)  # e2m1 codes
    bits = rng.integers(118, 122, size=(O, K // 32)).astype(np.uint8)
    scales = np.ldexp(1.0, bits.astype(np.int32) - 127).astype(np.float32)
    return values, packed, bits, scales


@pytest.mark.parametrize("fmt", [1, 2, 3])
@pytest.mark.parametrize("O,K,S", [(48, 96, 1), (64, 1408, 4), (100, 256, 8), (576, 2048, 3),
                                   (16, 32, 2), (1024, 4096, 1)])
def test_matmul_matches_oracle(fc, oracle_lib, fmt, O, K, S):
    rng = np.random.default_rng(O * 7 + K + S + fmt)
    values, packed, bits, scales = make_weights(rng, fmt, O, K)
    x = rng.standard_normal((S, K)).astype(np.float32)
    ref = oracle_lib.gemv(fmt, values, scales, x)
    y = np.zeros((S, O), dtype=np.float32)
    err = ctypes.create_string_buffer(256)
    ok = fc.lib().fc_matmul(fmt, y.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                            x.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                            packed.ctypes.data_as(ctypes.c_void_p), bits.ctypes.data_as(ctypes.c_void_p),
                            O, K, S, err, len(err))
    assert ok, err.value
    # fp32-accumulated dequant GEMV: the reference's own bar is rel < 1e-3
    # against f64 (tests/test_backend_metal.c:57); the north-star bar is 2e-2.
    assert rel_l2(y, ref) < 1e-5
    denom = np.abs(ref) + 1e-3 * np.abs(ref).max()
    assert np.max(np.abs(y - ref) / denom) < 1e-3


def test_matmul_rows_are_independent(fc):
    """Row s of a multi-row GEMV equals the same row computed alone, bit for bit."""
    rng = np.random.default_rng(3)
    O, K = 256, 1024
    values, packed, bits, scales = make_weights(rng, 1, O, K)
    x = rng.standard_normal((8, K)).astype(np.float32)
    err = ctypes.create_string_buffer(256)

    def run(xs):
        y = np.zeros((xs.shape[0], O), dtype=np.float32)
        assert fc.lib().fc_matmul(1, y.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                                  np.ascontiguousarray(xs).ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                                  packed.ctypes.data_as(ctypes.c_void_p), bits.ctypes.data_as(ctypes.c_void_p),
                                  O, K, xs.shape[0], err, len(err)), err.value
        return y

    full = run(x)
    for s in range(8):
        assert np.array_equal(run(x[s:s + 1])[0], full[s])


def test_matmul_rejects_bad_shapes(fc):
    err = ctypes.create_string_buffer(256)
    y = np.zeros(8, dtype=np.float32)
    x = np.zeros(40, dtype=np.float32)
    w = np.zeros(40, dtype=np.int8)
    assert not fc.lib().fc_matmul(1, y.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                                  x.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                                  w.ctypes.data_as(ctypes.c_void_p), w.ctypes.data_as(ctypes.c_void_p),
                                  1, 40, 1, err, len(err))
    assert b"invalid" in err.value
