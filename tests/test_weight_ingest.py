"""Weight ingest from checkpoint block formats.

CPU: fc_blocks_to_logical against a numpy restatement of the GGUF Q8_0 block
({fp16 d; int8 q[32]}) and the DS4 MXFP4 block ({ue8m0 e; uint8 q[16]},
element j low nibble, j + 16 high nibble of q[j];
patches/ds4/deepseek-v4-mxfp4-runtime.patch, deepseek-v4-dspark-metal.patch:4430-4460).
GPU: set_tensor_blocks / set_tensor_rowscale round trips through the model."""
import numpy as np
import pytest

import floyd_b200
from floyd_b200 import BLOCKS_MXFP4, BLOCKS_Q8_0, CONFIGS, scaled


def _q8_blocks(rng, rows, cols):
    nb = rows * cols // 32
    d = rng.normal(0, 0.01, size=nb).astype(np.float16)
    q = rng.integers(-128, 128, size=(nb, 32)).astype(np.int8)
    raw = np.zeros((nb, 34), dtype=np.uint8)
    raw[:, :2] = d.view(np.uint8).reshape(nb, 2)
    raw[:, 2:] = q.view(np.uint8)
    return raw, d, q


def _mx_blocks(rng, rows, cols):
    nb = rows * cols // 32
    e = rng.integers(100, 135, size=nb).astype(np.uint8)
    codes = rng.integers(0, 16, size=(nb, 32)).astype(np.uint8)
    raw = np.zeros((nb, 17), dtype=np.uint8)
    raw[:, 0] = e
    raw[:, 1:] = codes[:, :16] | (codes[:, 16:] << 4)
    return raw, e, codes


def test_q8_0_blocks_to_logical():
    rng = np.random.default_rng(0)
    rows, cols = 3, 96
    raw, d, q = _q8_blocks(rng, rows, cols)
    values, scales = floyd_b200.blocks_to_logical(BLOCKS_Q8_0, raw, rows, cols)
    assert np.array_equal(values.reshape(-1), q.reshape(-1))
    assert np.array_equal(scales.reshape(-1), d.view(np.uint16))


def test_mxfp4_blocks_to_logical():
    rng = np.random.default_rng(1)
    rows, cols = 2, 128
    raw, e, codes = _mx_blocks(rng, rows, cols)
    values, scales = floyd_b200.blocks_to_logical(BLOCKS_MXFP4, raw, rows, cols)
    logical = codes.reshape(rows, cols)        # element order within the row
    packed = logical[:, 0::2] | (logical[:, 1::2] << 4)
    assert np.array_equal(values, packed)
    assert np.array_equal(scales.reshape(-1), e)


def test_blocks_size_checked():
    with pytest.raises(floyd_b200.FloydError):
        floyd_b200.blocks_to_logical(BLOCKS_Q8_0, np.zeros(33, np.uint8), 1, 32)


@pytest.mark.gpu
def test_ingest_round_trips_on_device():
    cfg = scaled(CONFIGS["c4_ds4_flash"], hidden_size=256, layer_count=1, head_count=4, q_lora_rank=64,
                 expert_count=8, experts_per_token=2, moe_intermediate_size=64, vocab_size=512,
                 hash_layer_count=0, mtp_layers=0, context=64, rows=4)
    m = floyd_b200.Model(cfg, seed=0)
    rng = np.random.default_rng(2)
    # q8 attention matrix from Q8_0 blocks
    D, O = cfg["hidden_size"], cfg["q_lora_rank"]
    raw, d, q = _q8_blocks(rng, O, D)
    name = "model.layers.0.self_attn.q_a_proj.weight"
    m.set_tensor_blocks(name, BLOCKS_Q8_0, raw)
    assert np.array_equal(m.get_tensor(name, O * D).view(np.int8), q.reshape(-1))
    assert np.array_equal(m.get_tensor(name + ".gs", O * D // 32 * 2).view(np.uint16), d.view(np.uint16))
    # MXFP4 expert from MXFP4 blocks
    I = cfg["moe_intermediate_size"]
    raw, e, codes = _mx_blocks(rng, I, D)
    name = "model.layers.0.mlp.experts.5.gate_proj.weight"
    m.set_tensor_blocks(name, BLOCKS_MXFP4, raw)
    logical = codes.reshape(I, D)
    assert np.array_equal(m.get_tensor(name, I * D // 2), (logical[:, 0::2] | (logical[:, 1::2] << 4)).reshape(-1))
    assert np.array_equal(m.get_tensor(name + ".gs", I * D // 32), e)
    # Moonlight container: int8 values + one fp32 scale per row
    vals = rng.integers(-128, 128, size=(O, D)).astype(np.int8)
    rs = rng.uniform(1e-3, 1e-1, size=O).astype(np.float32)
    name = "model.layers.0.self_attn.q_a_proj.weight"
    m.set_tensor_rowscale(name, vals.view(np.uint8), rs)
    got = m.get_tensor(name + ".gs", O * D // 32 * 2).view(np.uint16).reshape(O, D // 32)
    assert np.array_equal(got, np.repeat(rs.astype(np.float16).view(np.uint16)[:, None], D // 32, axis=1))
    # a block of the wrong kind is refused
    with pytest.raises(floyd_b200.FloydError):
        m.set_tensor_blocks(name, BLOCKS_MXFP4, np.zeros(O * D // 32 * 17, np.uint8))
