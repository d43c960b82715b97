"""The byte and FLOP models behind the bench's roofline figures, checked
against the hot-path scope's own estimates (no GPU): one C4 verify moves
about 23.05 GB of algorithmic bytes (4 rows, ctx 16384, 30.5 unique experts
per layer), one C2 decode about 3.01 GB with an fp32 latent cache (2.88 GB
with this backend's fp16 cache), and a 2048-token C3 prefill is about
9.2 TFLOP of linear work."""
import pytest

from floyd_b200.configs import CONFIGS, prefill_flops, step_bytes


def test_c4_verify_bytes():
    assert step_bytes(CONFIGS["c4_ds4_flash"], 4, 16384, 30.5) == pytest.approx(23.05e9, rel=5e-3)


def test_c2_decode_bytes():
    cfg = CONFIGS["c2_moonlight_q8"]
    fp16_kv = 4096 * (cfg["kv_lora_rank"] + cfg["qk_rope_dim"]) * 2 * cfg["layer_count"]
    assert step_bytes(cfg, 1, 4096, 6) + fp16_kv == pytest.approx(3.01e9, rel=1e-2)


def test_c3_prefill_flops():
    f = prefill_flops(CONFIGS["c3_moonlight_q4"], 2048)
    assert f["linear"] == pytest.approx(9.2e12, rel=1e-2)
    # decompressed attention: 2 x heads x (nope + rope + v) per visible pair
    c = CONFIGS["c3_moonlight_q4"]
    pairs = 2048 * 2049 / 2
    per_pair = 2 * c["head_count"] * (c["qk_nope_dim"] + c["qk_rope_dim"] + c["value_dim"])
    assert f["attention"] == pytest.approx(c["layer_count"] * per_pair * pairs)


def test_prefill_flops_grow_with_a_prefix():
    c = CONFIGS["c3_moonlight_q4"]
    a, b = prefill_flops(c, 512), prefill_flops(c, 512, start=1024)
    assert b["attention"] > a["attention"] and b["linear"] > a["linear"]
