"""Verify-step parity of the CUDA backend (through the C ABI) against the CPU
oracle on identical seeded models, plus the batch-row == decode,
rollback and acceptance contracts of the reference
(tests/test_deepseek_v4_ds4_batch_parity.sh:65,80; dspark-metal.patch
:1793-1906; tests/test_moonlight_metal_runtime.c:106-115)."""
import ctypes

import numpy as np
import pytest

from conftest import rel_l2, top_margin
from floyd_b200 import ACCEPT_SAMPLE, CONFIGS, FMT_MXFP4, FMT_Q4, FMT_Q8, SCORE_SIGMOID, SCORE_SQRT_SOFTPLUS, scaled

pytestmark = pytest.mark.gpu

SEED = 0
KV_SEED = 7
MARGIN = 1e-3       # north-star: tokens bit-exact unless the top-1 margin < 1e-3
LOGIT_TOL = 2e-2    # north-star: logits / hidden within 2e-2 relative L2

C1 = CONFIGS["c1_tiny"]
C4_SMALL = scaled(CONFIGS["c4_ds4_flash"], hidden_size=1024, layer_count=4, head_count=8,
                  q_lora_rank=256, expert_count=32, experts_per_token=8,
                  moe_intermediate_size=256, vocab_size=4096, hash_layer_count=1,
                  context=300, rows=4)
C2_SMALL = scaled(CONFIGS["c2_moonlight_q8"], layer_count=3, vocab_size=4096, expert_count=16,
                  dense_intermediate_size=1024, moe_intermediate_size=160,
                  context=200, rows=4)
C3_SMALL = scaled(C2_SMALL, dense_format=FMT_Q4, expert_format=FMT_Q4)
SIGMOID_SMALL = scaled(C2_SMALL, score_fn=SCORE_SIGMOID, has_selection_bias=1,
                       expert_format=FMT_MXFP4)

_models = {}


def pair(cfg, name):
    """(GPU model, oracle model) for a config, built once per test session."""
    if name not in _models:
        import floyd_b200
        from oracle import oracle
        _models[name] = (floyd_b200.Model(cfg, seed=SEED), oracle.OracleModel(cfg, SEED))
    return _models[name]


def sessions(cfg, name, context=None, prefix=None, max_batch=None):
    import floyd_b200
    from oracle import oracle
    gm, om = pair(cfg, name)
    ctx = context or cfg["context"] + 16
    prefix = cfg["context"] if prefix is None else prefix
    gs = floyd_b200.Session(gm, ctx, max_batch or 8)
    gs.set_layer_trace(True)
    os_ = oracle.OracleSession(om, ctx, kv_fp16=True)
    if prefix:
        gs.seed_context(prefix, KV_SEED)
        os_.seed_context(prefix, KV_SEED)
    return gs, os_


def check_rows(gpu_logits, ora_logits):
    assert rel_l2(gpu_logits, ora_logits) < LOGIT_TOL
    for r in range(gpu_logits.shape[0]):
        g, o = int(np.argmax(gpu_logits[r])), int(np.argmax(ora_logits[r]))
        if g != o:
            assert top_margin(ora_logits[r]) < MARGIN, f"row {r}: {g} != {o}"


@pytest.mark.parametrize("name,cfg", [("c1", C1), ("c4s", C4_SMALL), ("c2s", C2_SMALL),
                                      ("c3s", C3_SMALL), ("sig", SIGMOID_SMALL)])
def test_synthetic_weights_identical(name, cfg):
    gm, om = pair(cfg, name)
    D = cfg["hidden_size"]
    names = ["model.embed_tokens.weight", "model.layers.0.self_attn.kv_b_proj.weight",
             "lm_head.weight"]
    last = cfg["layer_count"] - 1
    if cfg["first_dense_layer_count"] < cfg["layer_count"]:
        names += [f"model.layers.{last}.mlp.experts.3.gate_proj.weight",
                  f"model.layers.{last}.mlp.experts.{cfg['expert_count'] - 1}.down_proj.weight"]
    for n in names:
        fmt = cfg["expert_format"] if ".experts." in n else cfg["dense_format"]
        rows_cols = {"model.embed_tokens.weight": (cfg["vocab_size"], D), "lm_head.weight": (cfg["vocab_size"], D)}
        if "kv_b" in n:
            O, K = cfg["head_count"] * (cfg["qk_nope_dim"] + cfg["value_dim"]), cfg["kv_lora_rank"]
        elif "down_proj" in n:
            O, K = D, cfg["moe_intermediate_size"]
        elif "gate_proj" in n:
            O, K = cfg["moe_intermediate_size"], D
        else:
            O, K = rows_cols[n]
        nbytes = O * K if fmt == FMT_Q8 else O * K // 2
        sbytes = O * (K // 32) * (1 if fmt == FMT_MXFP4 else 2)
        assert np.array_equal(gm.get_tensor(n, nbytes), om.get_tensor(n, nbytes)), n
        assert np.array_equal(gm.get_tensor(n + ".gs", sbytes), om.get_tensor(n, sbytes, scales=True)), n
    router = f"model.layers.{last}.mlp.gate.weight"
    if cfg["first_dense_layer_count"] < cfg["layer_count"]:
        nb = cfg["expert_count"] * D * 4
        assert np.array_equal(gm.get_tensor(router, nb), om.get_tensor(router, nb))
    nb = D * 4
    assert np.array_equal(gm.get_tensor("model.norm.weight", nb), om.get_tensor("model.norm.weight", nb))


@pytest.mark.parametrize("name,cfg", [("c1", C1), ("c4s", C4_SMALL), ("c2s", C2_SMALL),
                                      ("c3s", C3_SMALL), ("sig", SIGMOID_SMALL)])
def test_verify_matches_oracle(name, cfg):
    gs, os_ = sessions(cfg, name)
    rng = np.random.default_rng(11)
    ids = rng.integers(0, cfg["vocab_size"], size=4).tolist()
    em, nxt, _ = gs.verify(ids)
    g_logits = gs.row_logits(4)
    oem, onxt, o_logits, o_tops = os_.verify(ids)
    check_rows(g_logits, o_logits)
    margins = [top_margin(o_logits[r]) for r in range(4)]
    if min(margins) >= MARGIN:
        assert em == oem and nxt == onxt
    assert gs.position() == os_.position()
    # latent KV written by this verify (fp16 cache on both sides)
    P = gs.position()
    for layer in range(cfg["layer_count"]):
        gl, gr = gs.copy_kv(layer)
        ol, orr = os_.copy_kv(layer)
        assert np.array_equal(gl[:cfg["context"]], ol[:cfg["context"]])  # seeded prefix
        assert rel_l2(gl[cfg["context"]:P], ol[cfg["context"]:P]) < 1e-3
        assert rel_l2(gr[cfg["context"]:P], orr[cfg["context"]:P]) < 1e-3


@pytest.mark.parametrize("name,cfg", [("c1", C1), ("c4s", C4_SMALL)])
def test_layer_outputs_and_routes_match_oracle(name, cfg):
    gs, os_ = sessions(cfg, name)
    ids = [5, 17, 301, 4000 % cfg["vocab_size"]]
    gs.verify(ids)
    g_layers = gs.layer_outputs(4)
    o_logits, o_layers, o_routes = os_.forward(ids, want_layers=True, want_routes=True)
    for layer in range(cfg["layer_count"]):
        assert rel_l2(g_layers[layer], o_layers[layer]) < LOGIT_TOL, layer
        if layer >= cfg["first_dense_layer_count"]:
            g_r = gs.routes(layer, 4)
            assert np.array_equal(np.sort(g_r, axis=1), np.sort(o_routes[layer], axis=1)), layer


@pytest.mark.parametrize("name,cfg", [("c1", C1), ("c4s", C4_SMALL), ("c3s", C3_SMALL)])
def test_verify_rows_equal_sequential_decode(name, cfg):
    """A verify row is bit-identical to the same token decoded alone at the
    same position (tests/test_deepseek_v4_ds4_batch_parity.sh:65,80)."""
    a, _ = sessions(cfg, name)
    b, _ = sessions(cfg, name)
    ids = [3, 1000, 77, 2024]
    a.verify(ids)
    batch = a.row_logits(4)
    batch_layers = a.layer_outputs(4)
    for r, t in enumerate(ids):
        single = b.decode(t)
        assert np.array_equal(single, batch[r]), f"row {r}"
        assert np.array_equal(b.layer_outputs(1)[:, 0], batch_layers[:, r]), f"row {r}"


def greedy_stream(cfg, name, first, n):
    """Target's own greedy continuation via plain decode."""
    s, _ = sessions(cfg, name)
    toks = [first]
    logits = s.decode(first)
    for _ in range(n):
        t = int(np.argmax(logits))
        toks.append(t)
        logits = s.decode(t)
    return toks


def test_planted_drafts_commit_and_rollback():
    cfg, name = C1, "c1"
    stream = greedy_stream(cfg, name, 42, 8)        # stream[i+1] = argmax after stream[..i]
    s, _ = sessions(cfg, name)
    p0 = s.position()
    # all three drafts correct -> commit 4, next = stream[4]
    em, nxt, _ = s.verify(stream[0:4])
    assert em == stream[0:4] and nxt == stream[4] and s.position() == p0 + 4
    # second draft wrong -> commit 2 (ids[0], ids[1]), next = stream[6]
    bad = [stream[4], stream[5], (stream[6] + 1) % cfg["vocab_size"], stream[7]]
    em, nxt, _ = s.verify(bad)
    assert em == stream[4:6] and nxt == stream[6] and s.position() == p0 + 6
    # the rolled-back session continues exactly like plain decode
    em, nxt, _ = s.verify([stream[6], stream[7], stream[8]])
    assert em == stream[6:9]
    st = s.stats()
    assert st["cpu_fallbacks"] == 0 and st["verify_calls"] == 3


def test_rollback_then_decode_is_bit_exact():
    cfg, name = C1, "c1"
    a, _ = sessions(cfg, name)
    b, _ = sessions(cfg, name)
    a.verify([9, 8, 7, 6])
    a.rollback(cfg["context"] + 1)      # keep only the first row
    la = a.decode(123)
    b.decode(9)
    lb = b.decode(123)
    assert np.array_equal(la, lb)


def test_sampling_decisions_match_oracle(oracle_lib):
    """Rejection-sampling acceptance (no reference implementation: parity
    unpinned) against the oracle's Philox restatement on the same logits."""
    import floyd_b200
    cfg, name = C1, "c1"
    s, _ = sessions(cfg, name, context=cfg["context"] + 200)
    V = cfg["vocab_size"]
    rng = np.random.default_rng(5)
    agree = 0
    for counter in range(24):
        ids = rng.integers(0, V, size=4).tolist()
        base = s.position()
        em, nxt, _ = s.verify(ids, mode=ACCEPT_SAMPLE, temperature=0.7, seed=1, counter=counter)
        logits = s.row_logits(4)
        nxt_o = ctypes.c_int()
        idp = np.array(ids, dtype=np.int32)
        commit_o = oracle_lib.lib().orc_accept_sample(
            logits.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), V,
            idp.ctypes.data_as(ctypes.POINTER(ctypes.c_int)), 3, 0.7, 1, counter, ctypes.byref(nxt_o))
        if len(em) == commit_o and nxt == nxt_o.value:
            agree += 1
        assert s.position() == base + len(em)
    assert agree == 24


@pytest.mark.parametrize("temperature", [1e-3, 0.02])
def test_low_temperature_sampling_matches_oracle(oracle_lib, temperature):
    """At low temperature drafts equal to the greedy stream are mostly
    accepted: the accept branch, the residual resample and the bonus sample
    all run, and every decision equals the oracle's on the same logits."""
    cfg, name = C1, "c1"
    V = cfg["vocab_size"]
    stream = greedy_stream(cfg, name, 42, 4)
    accepted = 0
    for counter in range(12):
        s, _ = sessions(cfg, name)
        em, nxt, _ = s.verify(stream[0:4], mode=ACCEPT_SAMPLE, temperature=temperature, seed=1,
                              counter=counter)
        logits = s.row_logits(4)
        nxt_o = ctypes.c_int()
        idp = np.array(stream[0:4], dtype=np.int32)
        commit_o = oracle_lib.lib().orc_accept_sample(
            logits.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), V,
            idp.ctypes.data_as(ctypes.POINTER(ctypes.c_int)), 3, temperature, 1, counter,
            ctypes.byref(nxt_o))
        assert len(em) == commit_o and nxt == nxt_o.value
        accepted += len(em) - 1
    assert accepted >= 12


def test_zero_draft_verify_equals_decode():
    cfg, name = C1, "c1"
    a, _ = sessions(cfg, name)
    b, _ = sessions(cfg, name)
    em, nxt, logits = a.verify([55], want_logits=True)
    ref = b.decode(55)
    assert em == [55] and nxt == int(np.argmax(ref))
    assert np.array_equal(logits, ref)


def test_request_validation_and_stats():
    import floyd_b200
    cfg, name = C1, "c1"
    gm, _ = pair(cfg, name)
    s = floyd_b200.Session(gm, 16, 4)
    with pytest.raises(floyd_b200.FloydError):
        s.append([1])                       # append needs position > 0
    s.prefill([1, 2, 3])
    before = s.stats()
    with pytest.raises(floyd_b200.FloydError):
        s.verify([1, 2, 3, 4, 5])           # 5 rows > max_batch 4
    with pytest.raises(floyd_b200.FloydError):
        s.verify([cfg["vocab_size"], 1])    # id out of range
    with pytest.raises(floyd_b200.FloydError):
        s.prefill([1])                      # prefill needs an empty session
    for _ in range(3):
        s.verify([4, 5, 6, 7])
    after = s.stats()
    assert after["buffer_allocations"] == before["buffer_allocations"]
    assert after["cpu_fallbacks"] == 0
    assert s.position() <= 16
    s.rollback(2)
    assert s.position() == 2
    s.rollback(10)                          # clamped: never moves forward
    assert s.position() == 2
    s.reset()
    assert s.position() == 0
    with pytest.raises(floyd_b200.FloydError):
        floyd_b200.Session(gm, 4, 8)        # max_batch > context


def test_context_full_is_rejected():
    import floyd_b200
    cfg, name = C1, "c1"
    gm, _ = pair(cfg, name)
    s = floyd_b200.Session(gm, 8, 4)
    s.prefill([1, 2, 3, 4])
    s.append([1, 2, 3, 4])
    with pytest.raises(floyd_b200.FloydError):
        s.decode(1)
    with pytest.raises(floyd_b200.FloydError):
        s.verify([1, 2])


def test_chunked_prefill_matches_oracle():
    """Prefill longer than one 8-row pass (moonlight_metal.m:1988-2005)."""
    import floyd_b200
    from oracle import oracle
    cfg, name = C1, "c1"
    gm, om = pair(cfg, name)
    s = floyd_b200.Session(gm, 64, 20)
    ids = list(range(100, 120))
    last = s.prefill(ids)
    o = oracle.OracleSession(om, 64, kv_fp16=True)
    ol, _, _ = o.forward(ids)
    check_rows(last[None], ol[-1:])


def test_spec_runtime_shim(fc):
    """deepseek_v4_runtime_{init,forward,argmax,verify_token,reset,free}
    (tests/test_deepseek_v4_spec_runtime.c:24-49)."""
    lib = fc.lib()
    cfg, name = C1, "c1"
    gm, _ = pair(cfg, name)
    rt = fc._lib.FcRuntime()
    assert lib.fc_runtime_init(ctypes.byref(rt), gm.handle, 64, 8)
    ids = np.array([3, 1, 4, 1, 5], dtype=np.int32)
    lp = ctypes.POINTER(ctypes.c_float)()
    assert lib.fc_runtime_forward(ctypes.byref(rt), ids.ctypes.data_as(ctypes.POINTER(ctypes.c_int)), 5,
                                  ctypes.byref(lp))
    logits = np.ctypeslib.as_array(lp, shape=(cfg["vocab_size"],)).copy()
    top = lib.fc_runtime_argmax(lp, cfg["vocab_size"])
    assert top == int(np.argmax(logits))
    acc = ctypes.c_int()
    assert lib.fc_runtime_verify_token(lp, cfg["vocab_size"], top, ctypes.byref(acc)) == top and acc.value == 1
    lib.fc_runtime_verify_token(lp, cfg["vocab_size"], top + 1, ctypes.byref(acc))
    assert acc.value == 0
    assert rt.last_count == 5 and rt.last_start_position == 0
    lib.fc_runtime_reset(ctypes.byref(rt))
    lib.fc_runtime_free(ctypes.byref(rt))


@pytest.mark.parametrize("seed", [11, 12])
def test_mtp_drafts_match_oracle(seed):
    """The on-device MTP drafter (run in the verify graph after acceptance)
    proposes the same k tokens as the oracle's restatement."""
    cfg, name = C4_SMALL, "c4s"
    assert cfg["mtp_layers"] == 1
    gs, os_ = sessions(cfg, name)
    rng = np.random.default_rng(seed)
    ids = rng.integers(0, cfg["vocab_size"], size=4).tolist()
    em, nxt, _ = gs.verify(ids)
    oem, onxt, _, _ = os_.verify(ids)
    assert em == oem and nxt == onxt
    assert gs.drafts() == os_.drafts()
    assert len(gs.drafts()) == 3
    # the drafter leaves the target's state alone: a decode afterwards still
    # matches the oracle
    g = gs.decode(nxt)
    o, _, _ = os_.forward([nxt])
    check_rows(g[None, :], o)
