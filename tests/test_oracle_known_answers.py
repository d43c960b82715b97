"""The oracle restatement pinned against the reference's own known answers
(tests/test_moe_route.c, tests/test_moe_exec.c, tests/test_deepseek_v4_quant.c,
tests/test_deepseek_v4_mxfp4.c) and against published Philox4x32-10 vectors."""
import math

import numpy as np
import pytest

from floyd_b200 import SCORE_SIGMOID, SCORE_SOFTMAX, SCORE_SQRT_SOFTPLUS


def silu(x):
    return x / (1.0 + math.exp(-x))


def test_philox_known_answers(oracle_lib):
    # Random123 kat_vectors, philox4x32 with 10 rounds
    assert oracle_lib.philox([0, 0, 0, 0], [0, 0]) == [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]
    assert oracle_lib.philox([0xFFFFFFFF] * 4, [0xFFFFFFFF] * 2) == [0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]
    assert oracle_lib.philox([0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344],
                             [0xA4093822, 0x299F31D0]) == [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]


def test_sigmoid_bias_affects_selection_only(oracle_lib):
    # tests/test_moe_route.c:16-34
    n, idx, w = oracle_lib.route([0.0, 2.0, -2.0], [0.0, -1.5, 2.0], 2, SCORE_SIGMOID, 0, 1.0)
    assert n == 2 and list(idx) == [2, 0]
    assert abs(w[0] - 1.0 / (1.0 + math.exp(2.0))) <= 1e-6
    assert abs(w[1] - 0.5) <= 1e-6


def test_softmax_is_stable_and_selects_top_k(oracle_lib):
    # tests/test_moe_route.c:41-57
    n, idx, w = oracle_lib.route([1000.0, 1001.0, 999.0], None, 2, SCORE_SOFTMAX, 0, 1.0)
    denom = math.exp(-1.0) + 1.0 + math.exp(-2.0)
    assert list(idx) == [1, 0]
    assert abs(w[0] - 1.0 / denom) <= 1e-6 and abs(w[1] - math.exp(-1.0) / denom) <= 1e-6


def test_sqrt_softplus_scores(oracle_lib):
    # tests/test_moe_route.c:59-72
    n, idx, w = oracle_lib.route([-2.0, 0.0, 2.0], None, 2, SCORE_SQRT_SOFTPLUS, 0, 1.0)
    assert list(idx) == [2, 1]
    assert abs(w[0] - math.sqrt(math.log1p(math.exp(2.0)))) <= 1e-6
    assert abs(w[1] - math.sqrt(math.log(2.0))) <= 1e-6


def test_ties_keep_lower_expert_index(oracle_lib):
    # tests/test_moe_route.c:74-85
    n, idx, w = oracle_lib.route([0.0, 0.0, 0.0], None, 2, SCORE_SIGMOID, 0, 1.0)
    assert list(idx) == [0, 1]


def test_finalize_normalizes_and_scales(oracle_lib):
    # tests/test_moe_route.c:87-96 restated through a full route: fixed
    # experts {0, 1} with weights 0.2 / 0.3 -> 0.8 / 1.2 at scale 2.
    logits = [math.log(0.2 / 0.8), math.log(0.3 / 0.7), 0.0]  # sigmoid -> 0.2, 0.3
    n, idx, w = oracle_lib.route(logits, None, 2, SCORE_SIGMOID, 1, 2.0, fixed=[0, 1])
    assert abs(w[0] - 0.8) <= 1e-5 and abs(w[1] - 1.2) <= 1e-5


def test_fixed_route_uses_supplied_experts(oracle_lib):
    # tests/test_moe_route.c:98-113
    n, idx, w = oracle_lib.route([-1.0, 0.0, 2.0], None, 2, SCORE_SQRT_SOFTPLUS, 1, 1.5, fixed=[2, 0])
    first = math.sqrt(math.log1p(math.exp(2.0)))
    second = math.sqrt(math.log1p(math.exp(-1.0)))
    assert n == 2
    assert abs(w[0] - first / (first + second) * 1.5) <= 1e-6
    assert abs(w[1] - second / (first + second) * 1.5) <= 1e-6


def test_fp4_codes_nibble_order_and_e8m0(oracle_lib):
    # tests/test_deepseek_v4_quant.c:17-44
    expected = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, 0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0]
    L = oracle_lib.lib()
    for i in range(16):
        assert L.orc_e2m1_to_f32(i) == expected[i]
    assert L.orc_e8m0_to_f32(0) == math.ldexp(1.0, -127)
    assert L.orc_e8m0_to_f32(125) == 0.25 and L.orc_e8m0_to_f32(127) == 1.0
    assert L.orc_e8m0_to_f32(128) == 2.0 and L.orc_e8m0_to_f32(254) == math.ldexp(1.0, 127)
    assert math.isnan(L.orc_e8m0_to_f32(255))


def test_fp4_dequant_changes_scale_at_32(oracle_lib):
    # tests/test_deepseek_v4_quant.c:46-58: packed 0x22 (code 2 = 1.0) with
    # scales 126 / 128 -> 0.5 for the first 32 values, 2.0 for the next 32.
    values = np.full((1, 64), 2, dtype=np.int8)
    scales = np.array([[0.5, 2.0]], dtype=np.float32)
    x = np.eye(64, dtype=np.float32)
    y = oracle_lib.gemv(3, values, scales, x)[:, 0]
    assert np.all(y[:32] == 0.5) and np.all(y[32:] == 2.0)


def test_fp16_conversion_round_trip(oracle_lib):
    L = oracle_lib.lib()
    for bits in [0x0000, 0x0001, 0x03FF, 0x0400, 0x3C00, 0x7BFF, 0x8001, 0xC000]:
        assert L.orc_f32_to_fp16(L.orc_fp16_to_f32(bits)) == bits
    assert L.orc_f32_to_fp16(1.0 + 2.0 ** -11) == 0x3C00   # tie -> even
    assert L.orc_f32_to_fp16(1.0 + 3 * 2.0 ** -11) == 0x3C02
    assert L.orc_f32_to_fp16(70000.0) == 0x7C00


def test_greedy_commit_rule(oracle_lib):
    # dspark-metal.patch:1793-1797: commit = 1 + leading matches of
    # row_tops[i-1] == proposal[i]
    import ctypes
    L = oracle_lib.lib()

    def commit(tops, ids):
        t = np.array(tops, dtype=np.int32)
        i = np.array(ids, dtype=np.int32)
        return L.orc_accept_greedy(t.ctypes.data_as(ctypes.POINTER(ctypes.c_int)),
                                   i.ctypes.data_as(ctypes.POINTER(ctypes.c_int)), len(ids) - 1)

    assert commit([5, 6, 7, 8], [9, 5, 6, 7]) == 4
    assert commit([5, 6, 7, 8], [9, 5, 0, 7]) == 2
    assert commit([5, 6, 7, 8], [9, 1, 6, 7]) == 1
    assert commit([5], [9]) == 1


def test_argmax_rule(oracle_lib):
    import ctypes
    L = oracle_lib.lib()
    a = np.array([1.0, 3.0, 3.0, np.nan, 2.0], dtype=np.float32)
    assert L.orc_argmax(a.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), 5) == 1
    b = np.array([np.nan, -1.0, -1.0], dtype=np.float32)
    assert L.orc_argmax(b.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), 3) == 1
