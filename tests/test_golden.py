"""The oracle against a transformers DeepseekV3 golden fixture
(tests/golden/make_golden.py): compressed-latent MLA with interleaved RoPE,
dense first layer, sigmoid + bias routing with shared experts, final norm and
lm-head, in fp32 (the oracle's reference-exact fp32 cache mode)."""
import os

import numpy as np
import pytest

from conftest import rel_l2

FIX = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "deepseek_v3_tiny.npz")


def oracle_config():
    from floyd_b200 import FMT_Q8, SCORE_SIGMOID
    return dict(hidden_size=64, layer_count=2, vocab_size=128, head_count=2, q_lora_rank=0,
                kv_lora_rank=32, qk_nope_dim=16, qk_rope_dim=8, value_dim=16, expert_count=8,
                experts_per_token=2, moe_intermediate_size=32, shared_expert_count=1,
                first_dense_layer_count=1, dense_intermediate_size=96, hash_layer_count=0,
                score_fn=SCORE_SIGMOID, normalize_topk=1, has_selection_bias=1,
                routed_scale=2.446, swiglu_limit=0.0, rms_norm_epsilon=1e-5, rope_theta=50000.0,
                dense_format=FMT_Q8, expert_format=FMT_Q8)


@pytest.fixture(scope="module")
def golden_run(oracle_lib):
    from oracle import oracle
    d = np.load(FIX)
    m = oracle.OracleModel(oracle_config(), 0)
    for name in d.files:
        if name in ("ids", "logits", "layer0") or "rotary" in name:
            continue
        m.set_f32(name, d[name])
    s = oracle.OracleSession(m, 64, kv_fp16=False)
    logits, layers, routes = s.forward(d["ids"], want_layers=True, want_routes=True)
    return d, logits, layers, routes, m, s


def test_golden_layer0_hidden(golden_run):
    d, logits, layers, routes, _, _ = golden_run
    assert rel_l2(layers[0], d["layer0"]) < 1e-5


def test_golden_logits_and_argmax(golden_run):
    d, logits, *_ = golden_run
    assert rel_l2(logits, d["logits"]) < 1e-5
    assert np.array_equal(np.argmax(logits, axis=1), np.argmax(d["logits"], axis=1))


def test_golden_split_prefill_equals_full(golden_run, oracle_lib):
    """Prefill of a prefix then row-by-row decode reproduces the full forward
    (tests/test_moonlight_metal_mla.c: prefill vs split prefix + decode)."""
    from oracle import oracle
    d, logits, _, _, m, _ = golden_run
    s = oracle.OracleSession(m, 64, kv_fp16=False)
    ids = d["ids"]
    first, _, _ = s.forward(ids[:6])
    rows = [first]
    for t in ids[6:]:
        lg, _, _ = s.forward([t])
        rows.append(lg)
    split = np.concatenate(rows)
    assert rel_l2(split, logits) < 1e-6
