"""The oracle against floyd's own C reference headers, compiled from the
reference checkout into oracle/_ref/ (moe_route.h, moe_exec.h,
deepseek_v4_quant.h), on identical random inputs; and the reference's own
unit-test binaries.  Skipped where oracle/_ref was not built (no reference
checkout)."""
import ctypes
import os
import subprocess

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(os.path.dirname(HERE), "oracle", "_ref")
HARNESS = os.path.join(REF, "libref_harness.so")

pytestmark = pytest.mark.skipif(not os.path.exists(HARNESS), reason="oracle/_ref not built")

FP = ctypes.POINTER(ctypes.c_float)
IP = ctypes.POINTER(ctypes.c_int)


@pytest.fixture(scope="module")
def ref():
    L = ctypes.CDLL(HARNESS)
    L.ref_route_select.argtypes = [FP, FP, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                   ctypes.c_float, IP, FP]
    L.ref_route_fixed.argtypes = [FP, ctypes.c_int, IP, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                  ctypes.c_float, FP]
    L.ref_moe_forward.argtypes = [ctypes.c_int] * 6 + [ctypes.c_float, ctypes.c_float, FP, FP,
                                  ctypes.c_void_p, ctypes.c_int, FP, ctypes.c_int, FP, FP, IP,
                                  ctypes.c_int, FP]
    L.ref_fp4_matmul.argtypes = [FP, FP, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                 ctypes.c_int, ctypes.c_int]
    return L


@pytest.mark.parametrize("binary", ["test_moe_route", "test_moe_exec", "test_deepseek_v4_quant"])
def test_reference_unit_tests_pass(binary):
    path = os.path.join(REF, binary)
    if not os.path.exists(path):
        pytest.skip("binary not built")
    out = subprocess.run([path], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0, out.stderr
    assert "ok" in out.stdout


@pytest.mark.parametrize("score_fn", [0, 1, 2])
@pytest.mark.parametrize("E,K", [(16, 4), (64, 6), (256, 8)])
def test_route_select_matches_reference(oracle_lib, ref, score_fn, E, K):
    rng = np.random.default_rng(E * 10 + score_fn)
    for trial in range(20):
        logits = (rng.standard_normal(E) * 2).astype(np.float32)
        if trial % 5 == 0:  # ties
            logits[: E // 2] = logits[0]
        bias = (rng.standard_normal(E) * 0.1).astype(np.float32) if trial % 2 else None
        n, idx, w = oracle_lib.route(logits, bias, K, score_fn, 1, 2.446)
        ridx = np.zeros(K, dtype=np.int32)
        rw = np.zeros(K, dtype=np.float32)
        rn = ref.ref_route_select(logits.ctypes.data_as(FP),
                                  bias.ctypes.data_as(FP) if bias is not None else None,
                                  E, K, score_fn, 1, 2.446, ridx.ctypes.data_as(IP), rw.ctypes.data_as(FP))
        assert n == rn
        assert np.array_equal(idx, ridx)
        assert np.array_equal(w, rw)


def test_route_fixed_matches_reference(oracle_lib, ref):
    rng = np.random.default_rng(1)
    for _ in range(20):
        logits = rng.standard_normal(32).astype(np.float32)
        fixed = rng.choice(32, size=6, replace=False).astype(np.int32)
        n, idx, w = oracle_lib.route(logits, None, 6, 2, 1, 1.5, fixed=fixed)
        rw = np.zeros(6, dtype=np.float32)
        ref.ref_route_fixed(logits.ctypes.data_as(FP), 32, fixed.ctypes.data_as(IP), 6, 2, 1, 1.5,
                            rw.ctypes.data_as(FP))
        assert np.array_equal(w, rw)


def test_fp4_matmul_matches_reference(oracle_lib, ref):
    """The oracle's e2m1 / ue8m0 GEMV against deepseek_v4_fp4_matmul_f32
    (deepseek_v4_quant.h:103-139) on the same packed codes and scales."""
    rng = np.random.default_rng(2)
    O, K, S = 48, 256, 3
    codes = rng.integers(0, 16, size=(O, K), dtype=np.uint8)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)
    e8 = rng.integers(118, 124, size=(O, K // 32)).astype(np.uint8)
    x = rng.standard_normal((S, K)).astype(np.float32)
    y_ref = np.zeros((S, O), dtype=np.float32)
    assert ref.ref_fp4_matmul(y_ref.ctypes.data_as(FP), x.ctypes.data_as(FP), S,
                              packed.ctypes.data_as(ctypes.c_void_p), e8.ctypes.data_as(ctypes.c_void_p), O, K)
    scales = np.ldexp(1.0, e8.astype(np.int32) - 127).astype(np.float32)
    y = oracle_lib.gemv(3, codes.astype(np.int8), scales, x)
    # the reference multiplies each value by its scale before summing; the
    # oracle sums a group and then scales: equal to fp32 rounding
    assert np.allclose(y, y_ref, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("score_fn,limit", [(0, 0.0), (1, 0.0), (2, 0.5)])
def test_moe_forward_matches_reference(oracle_lib, ref, score_fn, limit):
    """moe_f32_forward (moe_exec.h:65-114) against the oracle's MoE row
    (the code path its session forward runs) on the same fp32 experts:
    routing, clamped SwiGLU, ascending-expert accumulation, shared expert."""
    D, I, E, K, T = 64, 32, 16, 4, 5
    rng = np.random.default_rng(3 + score_fn)
    router = (rng.standard_normal((E, D)) * 0.3).astype(np.float32)
    block = (rng.standard_normal((E, 3, D * I)) * 0.2).astype(np.float32)
    shared = (rng.standard_normal((3, D * I)) * 0.2).astype(np.float32)
    x = rng.standard_normal((T, D)).astype(np.float32)
    tok = np.arange(T, dtype=np.int32)
    y_ref = np.zeros((T, D), dtype=np.float32)
    assert ref.ref_moe_forward(D, I, E, K, score_fn, 1, 1.5, limit, router.ctypes.data_as(FP), None,
                               None, 64, block.ctypes.data_as(FP), 1, shared.ctypes.data_as(FP),
                               x.ctypes.data_as(FP), tok.ctypes.data_as(IP), T, y_ref.ctypes.data_as(FP))
    L = oracle_lib.lib()
    L.orc_moe_forward_f32.argtypes = [ctypes.c_int] * 6 + [ctypes.c_float, ctypes.c_float, FP, FP, FP,
                                      ctypes.c_int, FP, FP, ctypes.c_int, FP]
    y = np.zeros((T, D), dtype=np.float32)
    assert L.orc_moe_forward_f32(D, I, E, K, score_fn, 1, 1.5, limit, router.ctypes.data_as(FP), None,
                                 block.ctypes.data_as(FP), 1, shared.ctypes.data_as(FP),
                                 x.ctypes.data_as(FP), T, y.ctypes.data_as(FP))
    # same operations in the same order: equal up to the reference's float
    # expression grouping of w[k] * projected[d]
    assert np.allclose(y, y_ref, rtol=1e-6, atol=1e-6)
