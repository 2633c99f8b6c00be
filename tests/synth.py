"""Seeded synthetic Qwen3-MoE checkpoints held in memory (test helper).

Builds the config.json dict and the safetensors-style tensor map of a
Qwen3MoeForCausalLM model with random N(0, 0.02) weights and unit norm
weights, in the naming of the reference's TensorNaming (src/model/arch.rs),
so the oracle (oracle/model.py) and the GPU decoder read the same model.
Routed experts are produced already encoded (q8_0 / q4_0) by
formats.SyntheticLayer, one layer's set shared by every MoE layer, so
Qwen3-30B-sized expert shapes need no float copy of every expert.
"""
import importlib
from concurrent.futures import ThreadPoolExecutor

import numpy as np

fmt = importlib.import_module("hale-token_b200.formats")


def _bf16_bits(a):
    u = a.view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def _normal(rng, rows, cols, dtype, std=0.02):
    """(safetensors dtype, shape, raw uint8) of a [rows, cols] N(0, std)
    matrix, drawn in chunks so large vocabularies stay cheap."""
    out = np.empty((rows, cols), np.uint16 if dtype == "BF16" else np.float32)
    step = max(1, (1 << 24) // cols)
    for r0 in range(0, rows, step):
        r1 = min(rows, r0 + step)
        v = rng.standard_normal((r1 - r0, cols), dtype=np.float32) * np.float32(std)
        out[r0:r1] = _bf16_bits(v) if dtype == "BF16" else v
    return (dtype, (rows, cols), out.reshape(-1).view(np.uint8))


def _vec(n):
    return ("F32", (n,), np.ones(n, np.float32).view(np.uint8))


def qwen3_moe(seed, layers, hidden, heads, kv_heads, head_dim, experts, top_k, inter, vocab,
              expert_dtype, dense_dtype="F32", theta=1e6, eps=1e-6, tie=False):
    """-> (hf_config, tensors, expert_encoded(layer, expert, proj))."""
    hf = {"architectures": ["Qwen3MoeForCausalLM"], "hidden_size": hidden, "num_hidden_layers": layers,
          "num_attention_heads": heads, "num_key_value_heads": kv_heads, "head_dim": head_dim,
          "vocab_size": vocab, "rms_norm_eps": eps, "rope_theta": theta, "num_experts": experts,
          "num_experts_per_tok": top_k, "moe_intermediate_size": inter, "intermediate_size": inter,
          "norm_topk_prob": True, "decoder_sparse_step": 1, "mlp_only_layers": [],
          "tie_word_embeddings": tie, "max_position_embeddings": 4096}
    rng = np.random.default_rng([seed, 0x5EED])
    t = {"model.embed_tokens.weight": _normal(rng, vocab, hidden, dense_dtype),
         "model.norm.weight": _vec(hidden)}
    if not tie:
        t["lm_head.weight"] = _normal(rng, vocab, hidden, dense_dtype)
    for l in range(layers):
        p = f"model.layers.{l}."
        t[p + "input_layernorm.weight"] = _vec(hidden)
        t[p + "post_attention_layernorm.weight"] = _vec(hidden)
        t[p + "self_attn.q_proj.weight"] = _normal(rng, heads * head_dim, hidden, dense_dtype)
        t[p + "self_attn.k_proj.weight"] = _normal(rng, kv_heads * head_dim, hidden, dense_dtype)
        t[p + "self_attn.v_proj.weight"] = _normal(rng, kv_heads * head_dim, hidden, dense_dtype)
        t[p + "self_attn.o_proj.weight"] = _normal(rng, hidden, heads * head_dim, dense_dtype)
        t[p + "self_attn.q_norm.weight"] = _vec(head_dim)
        t[p + "self_attn.k_norm.weight"] = _vec(head_dim)
        t[p + "mlp.gate.weight"] = _normal(rng, experts, hidden, "F32")
    ld = fmt.SyntheticLayer(seed, experts, hidden, inter, expert_dtype)
    with ThreadPoolExecutor(8) as ex:
        enc = list(ex.map(ld.expert_encoded, range(experts)))
    proj = {"gate": 0, "up": 1, "down": 2}
    return hf, t, (lambda l, e, pj: enc[e][proj[pj]])
