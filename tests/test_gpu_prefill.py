"""The prefill path on the tcgen05 tensor cores (sessions whose max_batch is
wider than a verify, moonlight_session_prefill, moonlight_metal.m:1988-2005):

  - the dequant GEMM alone (fc_matmul with more than 8 rows) against the
    oracle's fp32 restatement, every weight format, partial m- and n-tiles;
  - whole prefills against the oracle's forward of the same tokens: the
    last row's logits, the latent KV cache the prefill wrote, and a decode
    after it, for every model family of the configs (dense first layer,
    softmax / sigmoid / sqrt-softplus + hash routing, q8 / q4 / mxfp4,
    q-lora, shared experts, SwiGLU clamp);
  - appends after a seeded context in chunks of up to max_batch, and an
    append below the verify width (which takes the GEMV path).

The GEMM rounds activations and dequantized weights to fp16 once and
accumulates in fp32, so the bar is the north-star tolerance (2e-2 relative
L2 on logits), not the GEMV's exactness."""
import ctypes

import numpy as np
import pytest

from conftest import rel_l2
from test_gpu_matmul import make_weights
from test_gpu_verify import C1, C2_SMALL, C3_SMALL, C4_SMALL, KV_SEED, LOGIT_TOL, SIGMOID_SMALL, check_rows, pair

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("fmt", [1, 2, 3])
@pytest.mark.parametrize("O,K,S", [(576, 2048, 200), (256, 1408, 9), (1024, 512, 300), (64, 256, 129)])
def test_gemm_matches_oracle(fc, oracle_lib, fmt, O, K, S):
    rng = np.random.default_rng(O * 3 + K + S + fmt)
    values, packed, bits, scales = make_weights(rng, fmt, O, K)
    x = rng.standard_normal((S, K)).astype(np.float32)
    ref = oracle_lib.gemv(fmt, values, scales, x)
    y = np.full((S, O), np.nan, dtype=np.float32)
    err = ctypes.create_string_buffer(256)
    ok = fc.lib().fc_matmul(fmt, y.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                            x.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                            packed.ctypes.data_as(ctypes.c_void_p), bits.ctypes.data_as(ctypes.c_void_p),
                            O, K, S, err, len(err))
    assert ok, err.value
    assert np.isfinite(y).all()
    # two fp16 roundings per product: relative error ~ 2^-11 per term
    assert rel_l2(y, ref) < 2e-3


def test_gemm_rejects_unaligned_outputs(fc):
    err = ctypes.create_string_buffer(256)
    y = np.zeros(16 * 40, dtype=np.float32)
    x = np.zeros(16 * 64, dtype=np.float32)
    w = np.zeros(40 * 64, dtype=np.int8)
    assert not fc.lib().fc_matmul(1, y.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                                  x.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                                  w.ctypes.data_as(ctypes.c_void_p), w.ctypes.data_as(ctypes.c_void_p),
                                  40, 64, 16, err, len(err))
    assert b"invalid" in err.value


CASES = [("c1", C1), ("c2s", C2_SMALL), ("c3s", C3_SMALL), ("sig", SIGMOID_SMALL), ("c4s", C4_SMALL)]


def _prefill_pair(cfg, name, T, max_batch, context=None):
    import floyd_b200
    from oracle import oracle
    gm, om = pair(cfg, name)
    ctx = context or T + 16
    rng = np.random.default_rng(T + 11)
    ids = rng.integers(0, cfg["vocab_size"], size=T).tolist()
    gs = floyd_b200.Session(gm, ctx, max_batch)
    os_ = oracle.OracleSession(om, ctx, kv_fp16=True)
    return gs, os_, ids


@pytest.mark.parametrize("name,cfg", CASES)
def test_prefill_matches_oracle(name, cfg):
    T = 200
    gs, os_, ids = _prefill_pair(cfg, name, T, T)
    last = gs.prefill(ids)
    ol, _, _ = os_.forward(ids)
    check_rows(last[None], ol[-1:])
    assert gs.position() == T
    # the latent cache the prefill appended (fp16 in both).  Layer 0 sees
    # only the embeddings: every row within 5e-3.  Deeper layers follow the
    # routing of the layers below; a token whose top-k has a near tie may
    # pick another expert under the GEMM's fp16 rounding (as it may under
    # any change of summation order), so a few rows may differ more.
    for layer in (0, cfg["layer_count"] - 1):
        glat, grope = gs.copy_kv(layer)
        olat, orope = os_.copy_kv(layer)
        g = np.concatenate([glat, grope], axis=1)
        o = np.concatenate([olat, orope], axis=1)
        row = np.linalg.norm(g - o, axis=1) / np.linalg.norm(o, axis=1)
        bad = int((row > 5e-3).sum())
        assert bad <= (0 if layer == 0 else T // 50), f"layer {layer}: {bad} rows, worst {row.max()}"
        assert np.median(row) < 2e-3, f"layer {layer} median {np.median(row)}"
        assert rel_l2(g, o) < LOGIT_TOL, f"layer {layer}"
    # a decode on top of the prefilled cache
    g = gs.decode(ids[-1])
    o, _, _ = os_.forward([ids[-1]])
    check_rows(g[None], o)


def test_prefill_over_seeded_context_and_chunks():
    """Appends after a seeded prefix at max_batch 128: chunks of 128, 128
    and 44 tokens (GEMM path), then 5 tokens (GEMV path)."""
    cfg, name = C3_SMALL, "c3s"
    import floyd_b200
    from oracle import oracle
    gm, om = pair(cfg, name)
    ctx = 700
    gs = floyd_b200.Session(gm, ctx, 128)
    os_ = oracle.OracleSession(om, ctx, kv_fp16=True)
    gs.seed_context(150, KV_SEED)
    os_.seed_context(150, KV_SEED)
    rng = np.random.default_rng(5)
    ids = rng.integers(0, cfg["vocab_size"], size=300).tolist()
    for a, b in ((0, 128), (128, 256), (256, 300)):
        last = gs.append(ids[a:b])
        ol, _, _ = os_.forward(ids[a:b])
        check_rows(last[None], ol[-1:])
    tail = [1, 2, 3, 4, 5]
    last = gs.append(tail)
    ol, _, _ = os_.forward(tail)
    check_rows(last[None], ol[-1:])
    assert gs.position() == 455
    glat, _ = gs.copy_kv(1)
    olat, _ = os_.copy_kv(1)
    assert rel_l2(glat, olat) < LOGIT_TOL / 4


def test_prefill_then_verify_rows():
    """A verify after a GEMM prefill sees the cache the prefill wrote."""
    cfg, name = C2_SMALL, "c2s"
    gs, os_, ids = _prefill_pair(cfg, name, 160, 160, context=200)
    gs.prefill(ids)
    os_.forward(ids)
    v = [7, 8, 9, 10]
    gs.verify(v)
    g = gs.row_logits(4)
    _, _, o, _ = os_.verify(v)
    check_rows(g, o)
