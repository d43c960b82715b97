"""Writes a tiny floyd Moonlight container plus its expected outputs.

    python tests/golden/make_container.py OUT_DIR        (needs torch + transformers)

OUT_DIR/model/    config.json + model.safetensors in the layout of floyd's
                  converter (tools/convert_moonlight.py): every 2-D weight
                  except the embedding, the lm-head and the MoE router as U8
                  int8 values plus `name`.qs fp32 per-row scales; the rest F32.
OUT_DIR/oracle.safetensors
                  the expected intermediates of the C boundary tests (the
                  names floyd's Metal tests read: embed, layer.0.input_norm,
                  layer.0.q, layer.0.kv_a, layer.0.kv_norm, layer.0.attn,
                  layer.L.post_norm, layer.1.router_* / routed_mlp /
                  shared_mlp / mlp, layer.0.mlp, layer.L.output, final_input,
                  final_norm, logits, greedy).

The model is a small random transformers DeepseekV3 - the architecture of
Moonlight (MLA without q-lora, a dense first layer, sigmoid + bias routing,
two shared experts), as floyd builds its own tiny fixture
(tools/make_oracle.py:12-44) - with widths this backend's kernels take
(latent 256, rope 64).  Its weights are quantized with the converter's int8
rule (per-row absmax / 127, round to nearest) and the dequantized values are
written back into the model before the expected outputs are computed, so the
expectations describe exactly the container's weights.
"""
import json
import os
import sys

import numpy as np
import torch

CFG = dict(vocab_size=512, hidden_size=256, intermediate_size=512, moe_intermediate_size=64,
           num_hidden_layers=3, first_k_dense_replace=1, num_attention_heads=4,
           num_key_value_heads=4, n_routed_experts=16, num_experts_per_tok=4, n_shared_experts=2,
           q_lora_rank=None, kv_lora_rank=256, qk_nope_head_dim=64, qk_rope_head_dim=64,
           v_head_dim=64, n_group=1, topk_group=1, norm_topk_prob=True,
           routed_scaling_factor=2.446, scoring_func="sigmoid", topk_method="noaux_tc",
           rope_theta=50000.0, rope_scaling=None, tie_word_embeddings=False, rms_norm_eps=1e-5,
           max_position_embeddings=512, attention_bias=False, num_nextn_predict_layers=0)
IDS = [7, 301, 45, 222, 9, 128, 77, 400, 3, 64, 250, 19]


def quant_int8(w):
    """The converter's int8 rule: one scale per row = absmax / 127."""
    amax = np.abs(w).max(axis=1, keepdims=True)
    s = np.maximum(amax / 127.0, 1e-8).astype(np.float32)
    q = np.clip(np.rint(w / s), -128, 127).astype(np.int8)
    return q, s[:, 0]


def quantizable(name, t):
    if not (name.endswith(".weight") and t.ndim == 2):
        return False
    if "embed_tokens" in name or name == "lm_head.weight" or name.endswith("mlp.gate.weight"):
        return False
    return True


def split_experts(sd, inter):
    out = {}
    for name, t in sd.items():
        t = t.detach().float().numpy()
        if name.endswith(".mlp.experts.gate_up_proj"):
            base = name[: -len(".gate_up_proj")]
            for e in range(t.shape[0]):
                out[f"{base}.{e}.gate_proj.weight"] = np.ascontiguousarray(t[e, :inter])
                out[f"{base}.{e}.up_proj.weight"] = np.ascontiguousarray(t[e, inter:])
        elif name.endswith(".mlp.experts.down_proj"):
            base = name[: -len(".down_proj")]
            for e in range(t.shape[0]):
                out[f"{base}.{e}.down_proj.weight"] = np.ascontiguousarray(t[e])
        else:
            out[name] = np.ascontiguousarray(t)
    return out


def build(out_dir):
    from safetensors.numpy import save_file
    from transformers import DeepseekV3Config, DeepseekV3ForCausalLM

    torch.manual_seed(1234)
    cfg = DeepseekV3Config(**CFG)
    cfg._attn_implementation = "eager"
    model = DeepseekV3ForCausalLM(cfg).eval()
    inter = cfg.moe_intermediate_size
    with torch.no_grad():
        for _, p in model.named_parameters():
            if p.dim() >= 2:
                p.normal_(0, 0.05)
            else:
                p.copy_(1.0 + 0.05 * torch.randn_like(p))
        for layer in model.model.layers:
            if hasattr(layer.mlp, "gate"):
                layer.mlp.gate.e_score_correction_bias.copy_(torch.linspace(-0.1, 0.1, cfg.n_routed_experts))

    # quantize, write the container, put the dequantized weights back
    tensors = split_experts(model.state_dict(), inter)
    container, deq = {}, {}
    for name, t in tensors.items():
        if quantizable(name, t):
            q, s = quant_int8(t)
            container[name] = q.reshape(-1).view(np.uint8).copy()
            container[name + ".qs"] = s
            deq[name] = q.astype(np.float32) * s[:, None]
        else:
            container[name] = t.astype(np.float32)
    sd = model.state_dict()
    with torch.no_grad():
        for name in list(sd):
            if name.endswith(".mlp.experts.gate_up_proj"):
                base = name[: -len(".gate_up_proj")]
                for e in range(sd[name].shape[0]):
                    sd[name][e, :inter] = torch.from_numpy(deq[f"{base}.{e}.gate_proj.weight"])
                    sd[name][e, inter:] = torch.from_numpy(deq[f"{base}.{e}.up_proj.weight"])
            elif name.endswith(".mlp.experts.down_proj"):
                base = name[: -len(".down_proj")]
                for e in range(sd[name].shape[0]):
                    sd[name][e] = torch.from_numpy(deq[f"{base}.{e}.down_proj.weight"])
            elif name in deq:
                sd[name].copy_(torch.from_numpy(deq[name]))

    mdir = os.path.join(out_dir, "model")
    os.makedirs(mdir, exist_ok=True)
    save_file(container, os.path.join(mdir, "model.safetensors"))
    conf = {k: v for k, v in CFG.items()}
    conf["architectures"] = ["DeepseekV3ForCausalLM"]
    json.dump(conf, open(os.path.join(mdir, "config.json"), "w"), indent=1)

    # expected intermediates through forward hooks
    got = {}

    def keep(name, fn=lambda out: out):
        def hook(_mod, _inp, out):
            got[name] = fn(out).detach().float()[0] if fn(out).dim() == 3 else fn(out).detach().float()
        return hook

    mm = model.model
    hooks = [mm.embed_tokens.register_forward_hook(keep("embed")),
             mm.layers[0].input_layernorm.register_forward_hook(keep("layer.0.input_norm")),
             mm.layers[0].self_attn.q_proj.register_forward_hook(keep("layer.0.q")),
             mm.layers[0].self_attn.kv_a_proj_with_mqa.register_forward_hook(keep("layer.0.kv_a")),
             mm.layers[0].self_attn.kv_a_layernorm.register_forward_hook(keep("layer.0.kv_norm")),
             mm.layers[0].self_attn.register_forward_hook(keep("layer.0.attn", lambda o: o[0])),
             mm.layers[0].mlp.register_forward_hook(keep("layer.0.mlp")),
             mm.layers[1].mlp.gate.register_forward_hook(keep("layer.1.router_scores")),
             mm.layers[1].mlp.shared_experts.register_forward_hook(keep("layer.1.shared_mlp")),
             mm.layers[1].mlp.register_forward_hook(keep("layer.1.mlp")),
             mm.norm.register_forward_hook(keep("final_norm"))]
    for l, layer in enumerate(mm.layers):
        hooks.append(layer.post_attention_layernorm.register_forward_hook(keep(f"layer.{l}.post_norm")))
        hooks.append(layer.register_forward_hook(
            keep(f"layer.{l}.output", lambda o: o[0] if isinstance(o, tuple) else o)))

    def experts_hook(layer):
        def hook(_mod, inp, out):
            got[f"layer.{layer}.router_ids"] = inp[1].detach().clone()
            if layer == 1:
                got["layer.1.router_weights"] = inp[2].detach().float().clone()
                got["layer.1.routed_mlp"] = out.detach().float().reshape(len(IDS), -1)
        return hook

    for l in range(cfg.first_k_dense_replace, cfg.num_hidden_layers):
        hooks.append(mm.layers[l].mlp.experts.register_forward_hook(experts_hook(l)))
    with torch.no_grad():
        out = model(torch.tensor([IDS]), use_cache=False)
    for h in hooks:
        h.remove()
    logits = out.logits[0].float()
    greedy0 = int(torch.argmax(logits[-1]))
    with torch.no_grad():
        out2 = model(torch.tensor([IDS + [greedy0]]), use_cache=False)
    greedy1 = int(torch.argmax(out2.logits[0, -1]))

    oracle = {"input_ids": np.array(IDS, dtype=np.int64),
              "greedy": np.array([greedy0, greedy1], dtype=np.int64),
              "logits": logits.numpy(),
              "final_input": got[f"layer.{len(mm.layers) - 1}.output"].numpy()}
    for k, v in got.items():
        arr = v.numpy()
        if k.endswith(".router_ids"):
            arr = arr.astype(np.int64)
        oracle[k] = np.ascontiguousarray(arr.reshape(len(IDS), -1) if arr.ndim >= 2 or arr.size > 1 else arr)
    oracle = {k: np.ascontiguousarray(v) for k, v in oracle.items()}
    save_file(oracle, os.path.join(out_dir, "oracle.safetensors"))
    return mdir


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_container.py OUT_DIR")
    print(build(sys.argv[1]))
