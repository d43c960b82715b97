"""The tcgen05 latent-attention kernel (taken when a verify batch fills a
128-query tile: rows x heads >= 128) against the CPU oracle, against the
mma.sync kernel, and for verify-row == decode bit-exactness
(tests/test_deepseek_v4_ds4_batch_parity.sh:65,80 for the contract)."""
import os

import numpy as np
import pytest

from floyd_b200 import CONFIGS, scaled
from test_gpu_verify import LOGIT_TOL, check_rows, rel_l2, sessions

pytestmark = pytest.mark.gpu

# 32 heads x 4 rows = one full 128-query tile; long enough for several
# 32-key blocks per split and a partial last block
C4_TC = scaled(CONFIGS["c4_ds4_flash"], hidden_size=1024, layer_count=3, head_count=32,
               q_lora_rank=256, expert_count=32, experts_per_token=8,
               moe_intermediate_size=256, vocab_size=4096, hash_layer_count=1,
               context=2000, rows=4)
C1_TC = scaled(CONFIGS["c1_tiny"], head_count=32, context=1500, rows=4)   # L = 256 variant


@pytest.mark.parametrize("name,cfg", [("c4tc", C4_TC), ("c1tc", C1_TC)])
def test_tc_attention_verify_matches_oracle(name, cfg):
    gs, os_ = sessions(cfg, name)
    ids = [11, 222, 3333 % cfg["vocab_size"], 44]
    gs.verify(ids)
    g = gs.row_logits(4)
    _, _, o, _ = os_.verify(ids)
    check_rows(g, o)


@pytest.mark.parametrize("name,cfg", [("c4tc", C4_TC), ("c1tc", C1_TC)])
def test_tc_attention_rows_equal_decode(name, cfg):
    a, _ = sessions(cfg, name)
    b, _ = sessions(cfg, name)
    ids = [3, 1000, 77, 2024]
    a.verify(ids)
    batch = a.row_logits(4)
    for r, t in enumerate(ids):
        assert np.array_equal(b.decode(t), batch[r]), f"row {r}"


def test_tc_attention_agrees_with_mma_kernel():
    cfg, name = C4_TC, "c4tc"
    out = {}
    for mode in ("mma", "tc"):
        os.environ["FLOYD_ATTENTION"] = mode
        try:
            s, _ = sessions(cfg, name)
        finally:
            del os.environ["FLOYD_ATTENTION"]
        s.verify([7, 8, 9, 10])
        out[mode] = s.row_logits(4)
    assert rel_l2(out["tc"], out["mma"]) < LOGIT_TOL / 10


def test_tc_attention_short_and_empty_splits():
    """A context shorter than one split: most splits see no key (zero
    partials, m = -inf) and the combine must skip them."""
    cfg, name = C4_TC, "c4tc"
    gs, os_ = sessions(cfg, name, context=cfg["context"] + 16, prefix=40)
    ids = [5, 6, 7, 8]
    gs.verify(ids)
    _, _, o, _ = os_.verify(ids)
    check_rows(gs.row_logits(4), o)
