"""The spec-runtime drafter calls (deepseek_v4_runtime.h:180-223) over the
on-device MTP drafter: fc_runtime_dspark_prefill fills the drafter's latent
cache over the prompt and later forwards extend it; fc_runtime_dspark_propose
makes five greedy proposals.  Checked against the oracle's restatement
(orc_dspark_rows / orc_dspark_propose) on the same seeded model."""
import ctypes

import numpy as np
import pytest

from conftest import top_margin
from floyd_b200 import CONFIGS, scaled

pytestmark = pytest.mark.gpu

C4_SMALL = scaled(CONFIGS["c4_ds4_flash"], hidden_size=1024, layer_count=4, head_count=8,
                  q_lora_rank=256, expert_count=32, experts_per_token=8,
                  moe_intermediate_size=256, vocab_size=4096, hash_layer_count=1,
                  context=300, rows=4)


def test_dspark_prefill_and_propose_match_oracle(fc):
    from oracle import oracle
    lib = fc.lib()
    cfg = C4_SMALL
    gm = fc.Model(cfg, seed=0)
    om = oracle.OracleModel(cfg, 0)
    rt = fc._lib.FcRuntime()
    assert lib.fc_runtime_init(ctypes.byref(rt), gm.handle, 64, 8)
    os_ = oracle.OracleSession(om, 64, kv_fp16=True)
    prompt = np.array([11, 503, 77, 9, 1200, 64, 3000, 5, 42, 999, 17, 2048], dtype=np.int32)
    lp = ctypes.POINTER(ctypes.c_float)()
    IP = ctypes.POINTER(ctypes.c_int)
    assert lib.fc_runtime_forward(ctypes.byref(rt), prompt.ctypes.data_as(IP), len(prompt), ctypes.byref(lp))
    o_logits, _, _ = os_.forward(prompt.tolist())
    assert not lib.fc_runtime_dspark_propose(ctypes.byref(rt), 1, None, None)  # not prefilled yet
    assert lib.fc_runtime_dspark_prefill(ctypes.byref(rt))
    os_.dspark_rows(0, len(prompt) - 1)
    assert rt.dspark_ready == 1
    assert not lib.fc_runtime_dspark_prefill(ctypes.byref(rt))  # once per runtime

    def propose(token):
        ids = (ctypes.c_int64 * 6)()
        conf = (ctypes.c_float * 5)()
        assert lib.fc_runtime_dspark_propose(ctypes.byref(rt), token, ids, conf)
        return list(ids), np.array(conf[:])

    nxt = int(np.argmax(np.ctypeslib.as_array(lp, shape=(cfg["vocab_size"],))))
    ids, conf = propose(nxt)
    p = len(prompt) - 1
    o_ids, o_conf = os_.dspark_propose(p, nxt)
    assert ids[0] == nxt and ids[1:] == o_ids, (ids, o_ids)
    assert np.allclose(conf, o_conf, rtol=2e-2, atol=2e-2)

    # one more token: the forward extends the drafter's cache (dspark_ready)
    one = np.array([ids[1]], dtype=np.int32)
    assert lib.fc_runtime_forward(ctypes.byref(rt), one.ctypes.data_as(IP), 1, ctypes.byref(lp))
    o_logits, _, _ = os_.forward([ids[1]])
    os_.dspark_rows(p, 1)
    g = np.ctypeslib.as_array(lp, shape=(cfg["vocab_size"],)).copy()
    nxt = int(np.argmax(g))
    if top_margin(o_logits[0]) >= 1e-3:
        assert nxt == int(np.argmax(o_logits[0]))
    ids, conf = propose(nxt)
    o_ids, o_conf = os_.dspark_propose(p + 1, nxt)
    assert ids[1:] == o_ids, (ids, o_ids)
    lib.fc_runtime_reset(ctypes.byref(rt))
    assert rt.dspark_ready == 0
    lib.fc_runtime_free(ctypes.byref(rt))
