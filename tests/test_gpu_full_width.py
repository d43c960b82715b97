"""Parity at the widths BASELINE.json names, on 2-layer slices.

The other verify tests run the oracle on narrowed configs; here the CUDA path
and the oracle run the exact C4 (DS4-Flash stand-in) and C2 / C3
(Moonlight-shaped q8 / q4) widths - hidden size, heads, latent and rope
widths, q-lora, expert count and top-k, expert width, vocabulary, context -
with only the layer count cut to 2, so that the CPU oracle finishes in
seconds.  The C4 slice keeps one hash-routed layer, one score-routed layer
and the 1-layer MTP drafter; at 64 heads x 4 rows it runs the tcgen05
attention kernel, the C2 / C3 slices (16 heads) the mma.sync one.

Bars (the north-star's): logits within 2e-2 relative L2, greedy tokens
bit-exact unless the oracle's top-1 margin is below 1e-3, route sets equal
per layer, committed counts and MTP proposals equal.  The reference's own
contract for the same checks: tests/test_moonlight_metal_runtime.c and
tests/test_deepseek_v4_ds4_batch_parity.sh:65,80."""
import ctypes

import numpy as np
import pytest

from conftest import rel_l2, top_margin
from floyd_b200 import ACCEPT_SAMPLE, CONFIGS, FMT_Q4, scaled

pytestmark = pytest.mark.gpu

SEED = 0
KV_SEED = 7
MARGIN = 1e-3       # tokens bit-exact unless the top-1 margin < 1e-3
LOGIT_TOL = 2e-2    # logits / hidden states within 2e-2 relative L2

C4_SLICE = scaled(CONFIGS["c4_ds4_flash"], layer_count=2, hash_layer_count=1)
C2_SLICE = scaled(CONFIGS["c2_moonlight_q8"], layer_count=2)
C3_SLICE = scaled(CONFIGS["c2_moonlight_q8"], layer_count=2, dense_format=FMT_Q4,
                  expert_format=FMT_Q4)

_cache = {}


def pair(name):
    """(GPU model, oracle model) of one slice; only one slice is resident at a
    time, so the host and device memory of the three stay bounded."""
    import floyd_b200
    from oracle import oracle
    if name not in _cache:
        for old in list(_cache):
            gm, om = _cache.pop(old)
            gm.close()
            om.close()
        cfg = {"c4": C4_SLICE, "c2": C2_SLICE, "c3": C3_SLICE}[name]
        _cache[name] = (floyd_b200.Model(cfg, seed=SEED), oracle.OracleModel(cfg, SEED))
    return _cache[name]


def gpu_session(name, cfg):
    import floyd_b200
    gm, _ = pair(name)
    gs = floyd_b200.Session(gm, cfg["context"] + 16, 8)
    gs.set_layer_trace(True)
    gs.seed_context(cfg["context"], KV_SEED)
    return gs


def oracle_session(name, cfg):
    from oracle import oracle
    _, om = pair(name)
    os_ = oracle.OracleSession(om, cfg["context"] + 16, kv_fp16=True)
    os_.seed_context(cfg["context"], KV_SEED)
    return os_


def sessions(name, cfg):
    return gpu_session(name, cfg), oracle_session(name, cfg)


def check_rows(g, o):
    assert rel_l2(g, o) < LOGIT_TOL, rel_l2(g, o)
    for r in range(g.shape[0]):
        a, b = int(np.argmax(g[r])), int(np.argmax(o[r]))
        if a != b:
            assert top_margin(o[r]) < MARGIN, f"row {r}: {a} != {b}"


SLICES = [("c4", C4_SLICE), ("c2", C2_SLICE), ("c3", C3_SLICE)]


@pytest.mark.parametrize("name,cfg", SLICES)
def test_full_width_verify_matches_oracle(name, cfg):
    gs, os_ = sessions(name, cfg)
    rng = np.random.default_rng(21)
    ids = rng.integers(0, cfg["vocab_size"], size=4).tolist()
    em, nxt, _ = gs.verify(ids)
    g_logits = gs.row_logits(4)
    g_layers = gs.layer_outputs(4)
    g_routes = {l: gs.routes(l, 4) for l in range(cfg["first_dense_layer_count"], cfg["layer_count"])}
    oem, onxt, o_logits, _ = os_.verify(ids)
    check_rows(g_logits, o_logits)
    if min(top_margin(o_logits[r]) for r in range(4)) >= MARGIN:
        assert em == oem and nxt == onxt
    assert gs.position() == os_.position()
    # per-layer hidden states and route sets of the same rows
    _, o_layers, o_routes = oracle_session(name, cfg).forward(ids, want_layers=True,
                                                              want_routes=True)
    for layer in range(cfg["layer_count"]):
        assert rel_l2(g_layers[layer], o_layers[layer]) < LOGIT_TOL, layer
        if layer >= cfg["first_dense_layer_count"]:
            assert np.array_equal(np.sort(g_routes[layer], axis=1),
                                  np.sort(o_routes[layer], axis=1)), layer
    # the latent rows this verify appended (fp16 cache on both sides)
    P = gs.position()
    for layer in range(cfg["layer_count"]):
        gl, gr = gs.copy_kv(layer)
        ol, orr = os_.copy_kv(layer)
        assert rel_l2(gl[cfg["context"]:P], ol[cfg["context"]:P]) < 1e-3
        assert rel_l2(gr[cfg["context"]:P], orr[cfg["context"]:P]) < 1e-3
    if cfg.get("mtp_layers"):
        assert gs.drafts() == os_.drafts() and len(gs.drafts()) == 3


@pytest.mark.parametrize("name,cfg", SLICES)
def test_full_width_decode_matches_oracle(name, cfg):
    """One plain decode row (configs[1] is a draft-0 decode)."""
    gs, os_ = sessions(name, cfg)
    g = gs.decode(1234)
    o, _, _ = os_.forward([1234])
    check_rows(g[None, :], o)


def greedy_stream(name, cfg, first, n):
    gs = gpu_session(name, cfg)
    toks = [first]
    logits = gs.decode(first)
    for _ in range(n):
        t = int(np.argmax(logits))
        toks.append(t)
        logits = gs.decode(t)
    return toks


def test_full_width_rejection_sampling_branches(oracle_lib):
    """Rejection sampling at the C4 widths with drafts that can be accepted:
    drafts are the target's greedy continuation, at temperatures low enough
    that p(draft) is large (synthetic full-width logits are nearly flat at
    T = 0.7, where every draft is rejected).  Across the rounds the accept
    branch, the residual resample of a rejected draft and the bonus sample
    after a fully accepted round all run, and every decision equals the
    oracle's Philox restatement on the same logits."""
    name, cfg = "c4", C4_SLICE
    V = cfg["vocab_size"]
    stream = greedy_stream(name, cfg, 42, 4)
    gs = gpu_session(name, cfg)
    p0 = gs.position()
    commits = []
    for temperature in (1e-3, 0.02, 0.05):
        for counter in range(8):
            ids = list(stream[0:4])
            if counter % 4 == 3:   # one planted wrong draft: forces a rejection
                ids[2] = (ids[2] + 1) % V
            gs.rollback(p0)
            em, nxt, _ = gs.verify(ids, mode=ACCEPT_SAMPLE, temperature=temperature, seed=1,
                                   counter=counter)
            logits = gs.row_logits(4)
            nxt_o = ctypes.c_int()
            idp = np.array(ids, dtype=np.int32)
            commit_o = oracle_lib.lib().orc_accept_sample(
                logits.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), V,
                idp.ctypes.data_as(ctypes.POINTER(ctypes.c_int)), 3, temperature, 1, counter,
                ctypes.byref(nxt_o))
            assert len(em) == commit_o and nxt == nxt_o.value, (temperature, counter)
            assert em == ids[:len(em)]
            commits.append(len(em))
    assert 4 in commits                          # full accept + bonus sample
    assert any(1 <= c < 4 for c in commits)      # a rejection + residual resample
    assert sum(c - 1 for c in commits) >= len(commits)   # the accept branch ran often
