"""Model configurations of the benchmark (BASELINE.json `configs`).

Each entry is a dict of FcModelConfig fields plus the workload keys used by
the tests and bench.py (`context`, `rows`, ...).  Architecture numbers follow
the configs verbatim; the values the configs leave open are stated here:
  - RMSNorm epsilon 1e-5 and rope theta 50000 for the Moonlight-shaped models
    (the reference's tiny fixture, tools/make_oracle.py:16-33);
  - C1 / C2 softmax gates normalize the top-k weights
    (norm_topk_prob=True in tools/make_oracle.py:29); C2 scales by 2.446;
  - the DS4-Flash stand-in (C4) uses q_lora 1024, nope / v 128, sqrt-softplus
    scores with a selection bias, hash routing on the first 3 layers,
    routed_scale 1.5 and swiglu_limit 10, like deepseek_v4_forward.h
    (:18-27, :1208-1278).
"""
from ._lib import FMT_MXFP4, FMT_Q4, FMT_Q8, SCORE_SOFTMAX, SCORE_SQRT_SOFTPLUS

_MOONLIGHT = dict(
    hidden_size=2048, layer_count=27, vocab_size=163840, head_count=16,
    q_lora_rank=0, kv_lora_rank=512, qk_nope_dim=128, qk_rope_dim=64, value_dim=128,
    expert_count=64, experts_per_token=6, moe_intermediate_size=1408,
    shared_expert_count=2, first_dense_layer_count=1, dense_intermediate_size=11264,
    hash_layer_count=0, score_fn=SCORE_SOFTMAX, normalize_topk=1, has_selection_bias=0,
    routed_scale=2.446, swiglu_limit=0.0, rms_norm_epsilon=1e-5, rope_theta=50000.0,
    dense_format=FMT_Q8, expert_format=FMT_Q8,
)

CONFIGS = {
    # tiny synthetic verify step (CPU-runnable)
    "c1_tiny": dict(
        hidden_size=1024, layer_count=2, vocab_size=8192, head_count=16,
        q_lora_rank=0, kv_lora_rank=256, qk_nope_dim=64, qk_rope_dim=64, value_dim=64,
        expert_count=16, experts_per_token=4, moe_intermediate_size=512,
        shared_expert_count=1, first_dense_layer_count=0, dense_intermediate_size=0,
        hash_layer_count=0, score_fn=SCORE_SOFTMAX, normalize_topk=1, has_selection_bias=0,
        routed_scale=1.0, swiglu_limit=0.0, rms_norm_epsilon=1e-5, rope_theta=50000.0,
        dense_format=FMT_Q8, expert_format=FMT_Q8,
        context=512, rows=4),
    # Moonlight-16B-A3B-shaped q8 decode, ctx 4096
    "c2_moonlight_q8": dict(_MOONLIGHT, context=4096, rows=1),
    # same model, q4
    "c3_moonlight_q4": dict(_MOONLIGHT, dense_format=FMT_Q4, expert_format=FMT_Q4,
                            context=4096, rows=1),
    # DS4-Flash-style stand-in, draft 3 at ctx 16384
    "c4_ds4_flash": dict(
        hidden_size=4096, layer_count=43, vocab_size=129280, head_count=64,
        q_lora_rank=1024, kv_lora_rank=512, qk_nope_dim=128, qk_rope_dim=64, value_dim=128,
        expert_count=256, experts_per_token=8, moe_intermediate_size=2048,
        shared_expert_count=1, first_dense_layer_count=0, dense_intermediate_size=0,
        hash_layer_count=3, score_fn=SCORE_SQRT_SOFTPLUS, normalize_topk=1,
        has_selection_bias=1, routed_scale=1.5, swiglu_limit=10.0,
        rms_norm_epsilon=1e-6, rope_theta=10000.0,
        dense_format=FMT_Q8, expert_format=FMT_MXFP4, mtp_layers=1,
        context=16384, rows=4),
}


def model_fields(cfg):
    """The FcModelConfig part of a config dict."""
    from ._lib import FcModelConfig
    names = {n for n, _ in FcModelConfig._fields_}
    return {k: v for k, v in cfg.items() if k in names}


def scaled(cfg, **over):
    """A copy of `cfg` with fields overridden (smaller test variants)."""
    out = dict(cfg)
    out.update(over)
    return out


_BPP = {FMT_Q8: 34 / 32, FMT_Q4: 18 / 32, FMT_MXFP4: 17 / 32}


def step_bytes(cfg, rows, context, active_experts_per_layer):
    """Algorithmic HBM bytes of one forward of `rows` rows at `context` keys:
    every weight the step needs read once at its stored bytes per parameter,
    the latent KV (fp16) read once, the router in fp32."""
    c = cfg
    D, H, L, R = c["hidden_size"], c["head_count"], c["kv_lora_rank"], c["qk_rope_dim"]
    NP, VD = c["qk_nope_dim"], c["value_dim"]
    df, ef = _BPP[c["dense_format"]], _BPP[c["expert_format"]]
    attn = (c["q_lora_rank"] * D + H * (NP + R) * c["q_lora_rank"] if c["q_lora_rank"]
            else H * (NP + R) * D)
    attn += (L + R) * D + H * (NP + VD) * L + D * H * VD
    per_layer_dense = attn * df
    total = 0.0
    for layer in range(c["layer_count"]):
        total += per_layer_dense
        if layer < c["first_dense_layer_count"]:
            total += 3 * D * c["dense_intermediate_size"] * df
        else:
            I = c["moe_intermediate_size"]
            total += active_experts_per_layer * 3 * D * I * ef
            total += 3 * D * I * c["shared_expert_count"] * df
            total += c["expert_count"] * D * 4
        total += context * (L + R) * 2
    total += c["vocab_size"] * D * df  # lm-head
    return total


def prefill_flops(cfg, tokens, start=0):
    """Algorithmic FLOPs of one prefill chunk of `tokens` rows at positions
    start .. start + tokens - 1, in the form the prefill path computes:
    every linear layer 2 x params per row (q, kv_a, o; routed experts at
    experts_per_token per row, shared / dense MLPs, the router), keys and
    values decompressed from the latent cache for all start + tokens
    positions (kv_b: H x (nope + v) x L per position), and attention
    2 x H x (nope + rope + v) per visible (query, key) pair.
    Returns {"linear": F, "attention": F}."""
    c = cfg
    D, H, L, R = c["hidden_size"], c["head_count"], c["kv_lora_rank"], c["qk_rope_dim"]
    NP, VD = c["qk_nope_dim"], c["value_dim"]
    q = (D * c["q_lora_rank"] + c["q_lora_rank"] * H * (NP + R)) if c["q_lora_rank"] else D * H * (NP + R)
    per_row = q + D * (L + R) + H * VD * D
    linear = 0.0
    for layer in range(c["layer_count"]):
        linear += per_row * tokens + H * (NP + VD) * L * (start + tokens)
        if layer < c["first_dense_layer_count"]:
            linear += 3 * D * c["dense_intermediate_size"] * tokens
        else:
            I = c["moe_intermediate_size"]
            linear += (c["experts_per_token"] * 3 * D * I + 3 * D * I * c["shared_expert_count"]
                       + D * c["expert_count"]) * tokens
    pairs = tokens * start + tokens * (tokens + 1) / 2
    attention = 2.0 * c["layer_count"] * H * (NP + R + VD) * pairs
    return {"linear": 2.0 * linear, "attention": attention}
