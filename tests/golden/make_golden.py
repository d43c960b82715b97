"""Generates tests/golden/deepseek_v3_tiny.npz: a tiny random DeepseekV3 (the
architecture floyd's Moonlight runtime executes; the reference builds its own
fixtures the same way, tools/make_oracle.py:12-44) with compressed-latent MLA
(q_lora none), interleaved RoPE, a dense first layer, sigmoid + bias routing
with shared experts, and its fp32 logits / hidden states from transformers.

    python tests/golden/make_golden.py        (needs torch + transformers)

The fixture pins the oracle's MLA / RoPE / MoE / norm semantics
(tests/test_golden.py).  Weights are stored under the checkpoint names the
oracle and the CUDA backend use.
"""
import os

import numpy as np
import torch

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "deepseek_v3_tiny.npz")

CFG = dict(vocab_size=128, hidden_size=64, intermediate_size=96, moe_intermediate_size=32,
           num_hidden_layers=2, first_k_dense_replace=1, num_attention_heads=2,
           num_key_value_heads=2, n_routed_experts=8, num_experts_per_tok=2, n_shared_experts=1,
           q_lora_rank=None, kv_lora_rank=32, qk_nope_head_dim=16, qk_rope_head_dim=8,
           v_head_dim=16, n_group=1, topk_group=1, norm_topk_prob=True,
           routed_scaling_factor=2.446, rope_theta=50000.0, rope_scaling=None,
           tie_word_embeddings=False, rms_norm_eps=1e-5, max_position_embeddings=256,
           attention_bias=False)
IDS = [3, 14, 15, 92, 65, 35, 89, 79, 32, 38]


def main():
    from transformers import DeepseekV3Config, DeepseekV3ForCausalLM
    torch.manual_seed(1234)
    cfg = DeepseekV3Config(**CFG)
    cfg._attn_implementation = "eager"
    model = DeepseekV3ForCausalLM(cfg).eval()
    with torch.no_grad():
        for _, p in model.named_parameters():
            if p.dim() >= 2:
                p.normal_(0, 0.1)
            else:
                p.copy_(1.0 + 0.1 * torch.randn_like(p))
        for layer in model.model.layers:
            if hasattr(layer.mlp, "gate"):
                layer.mlp.gate.e_score_correction_bias.copy_(
                    torch.linspace(-0.1, 0.1, cfg.n_routed_experts))
        out = model(torch.tensor([IDS]), output_hidden_states=True, use_cache=False)
    arrays = {"ids": np.array(IDS, dtype=np.int32),
              "logits": out.logits[0].float().numpy(),
              "layer0": out.hidden_states[1][0].float().numpy()}
    inter = cfg.moe_intermediate_size
    for name, t in model.state_dict().items():
        t = t.float().numpy()
        if name.endswith(".mlp.experts.gate_up_proj"):
            base = name[: -len(".gate_up_proj")]
            for e in range(t.shape[0]):
                arrays[f"{base}.{e}.gate_proj.weight"] = t[e, :inter]
                arrays[f"{base}.{e}.up_proj.weight"] = t[e, inter:]
        elif name.endswith(".mlp.experts.down_proj"):
            base = name[: -len(".down_proj")]
            for e in range(t.shape[0]):
                arrays[f"{base}.{e}.down_proj.weight"] = t[e]
        else:
            arrays[name] = t
    np.savez_compressed(OUT, **arrays)
    print(OUT, os.path.getsize(OUT))


if __name__ == "__main__":
    main()
