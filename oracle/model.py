"""Loads a tiny Hugging Face-style MoE checkpoint into the oracle's decoder.

TEST INFRASTRUCTURE ONLY. Mirrors the reference's config normalisation
(src/config.rs:254-314), tensor naming (src/model/arch.rs:30-118) and model
assembly (src/model/transformer.rs:58-150) closely enough to run the golden
fixtures through ho_model_forward (transformer.rs:168-239).
"""
import ctypes as C
import json
import os
import struct

import numpy as np

from . import oracle as O

_ST_DTYPES = {"F32": (np.float32, O.F32), "BF16": (np.uint16, O.BF16), "F16": (np.uint16, O.F16)}


def read_safetensors(path):
    """Minimal safetensors reader -> {name: (dtype_str, shape, raw uint8 array)}."""
    with open(path, "rb") as f:
        blob = f.read()
    (hlen,) = struct.unpack("<Q", blob[:8])
    header = json.loads(blob[8:8 + hlen])
    base = 8 + hlen
    out = {}
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        a, b = meta["data_offsets"]
        out[name] = (meta["dtype"], tuple(meta["shape"]),
                     np.frombuffer(blob, dtype=np.uint8, count=b - a, offset=base + a))
    return out


def normalize_config(hf):
    """ModelConfig::from_hf (config.rs:254-314)."""
    arch = hf["architectures"][0]
    if arch not in ("Qwen3MoeForCausalLM", "MixtralForCausalLM"):
        raise ValueError(f"unsupported model architecture `{arch}`")
    qwen = arch == "Qwen3MoeForCausalLM"
    n_exp = hf.get("num_experts", hf.get("num_local_experts"))
    dense_inter = hf.get("intermediate_size") or 0
    layers = hf["num_hidden_layers"]
    if qwen:
        step = max(hf.get("decoder_sparse_step") or 1, 1)
        mlp_only = hf.get("mlp_only_layers") or []
        dense = [i for i in range(layers) if i in mlp_only or (i + 1) % step != 0]
        normalize = bool(hf.get("norm_topk_prob") or False)
    else:
        dense = []
        normalize = True
    return {
        "qwen": qwen,
        "hidden": hf["hidden_size"],
        "expert_inter": hf.get("moe_intermediate_size") or dense_inter,
        "dense_inter": dense_inter,
        "layers": layers,
        "heads": hf["num_attention_heads"],
        "kv_heads": hf.get("num_key_value_heads") or hf["num_attention_heads"],
        "head_dim": hf.get("head_dim") or hf["hidden_size"] // hf["num_attention_heads"],
        "vocab": hf["vocab_size"],
        "eps": float(hf.get("rms_norm_eps", 1e-6)),
        "theta": float(hf.get("rope_theta", 10000.0)),
        "max_pos": hf.get("max_position_embeddings", 4096),
        "experts": n_exp,
        "top_k": hf["num_experts_per_tok"],
        "normalize": normalize,
        "tie": bool(hf.get("tie_word_embeddings", False)),
        "dense_layers": dense,
    }


def _names(qwen):
    """TensorNaming (arch.rs:30-118)."""
    if qwen:
        proj = {"gate": "gate_proj", "up": "up_proj", "down": "down_proj"}
        return (lambda l, e, p: f"model.layers.{l}.mlp.experts.{e}.{proj[p]}.weight",
                lambda l: f"model.layers.{l}.mlp.gate.weight",
                lambda l, p: f"model.layers.{l}.mlp.{proj[p]}.weight")
    w = {"gate": "w1", "down": "w2", "up": "w3"}
    proj = {"gate": "gate_proj", "up": "up_proj", "down": "down_proj"}
    return (lambda l, e, p: f"model.layers.{l}.block_sparse_moe.experts.{e}.{w[p]}.weight",
            lambda l: f"model.layers.{l}.block_sparse_moe.gate.weight",
            lambda l, p: f"model.layers.{l}.mlp.{proj[p]}.weight")


class OracleModel:
    """A fixture model held in numpy buffers and exposed as an ho_model.

    `expert_dtype` re-encodes every routed expert (the pack converter's job,
    src/convert.rs:56-127 via WeightMatrix::convert, matrix.rs:103-109).
    """

    def __init__(self, directory=None, expert_dtype=None, hf_config=None, tensors=None, expert_encoded=None):
        """From a checkpoint directory (config.json + model.safetensors), or
        from memory: `hf_config` (the config.json dict) and `tensors`
        ({name: (safetensors dtype, shape, raw uint8)}). `expert_encoded`
        (optional): (layer, expert, "gate"|"up"|"down") -> that routed
        expert matrix already encoded in expert_dtype, for models whose
        experts are not held as float tensors."""
        if directory is not None:
            with open(os.path.join(directory, "config.json")) as f:
                hf_config = json.load(f)
            tensors = read_safetensors(os.path.join(directory, "model.safetensors"))
        self.cfg = normalize_config(hf_config)
        self.t = tensors
        self.expert_encoded = expert_encoded
        self._keep = []
        c = self.cfg
        expert_name, router_name, dense_name = _names(c["qwen"])
        h, hd = c["hidden"], c["head_dim"]
        self.expert_dtype = expert_dtype

        emb = self.matrix("model.embed_tokens.weight")
        head = emb if (c["tie"] or "lm_head.weight" not in self.t) else self.matrix("lm_head.weight")
        layers = []
        self.layer_experts = []
        for l in range(c["layers"]):
            p = f"model.layers.{l}."
            L = O.Layer()
            L.input_norm = self.vector(p + "input_layernorm.weight")
            L.post_norm = self.vector(p + "post_attention_layernorm.weight")
            L.q = self.matrix(p + "self_attn.q_proj.weight")
            L.k = self.matrix(p + "self_attn.k_proj.weight")
            L.v = self.matrix(p + "self_attn.v_proj.weight")
            L.o = self.matrix(p + "self_attn.o_proj.weight")
            if c["qwen"]:
                L.q_norm = self.vector(p + "self_attn.q_norm.weight")
                L.k_norm = self.vector(p + "self_attn.k_norm.weight")
            else:
                L.q_norm = None
                L.k_norm = None
            if l in c["dense_layers"]:
                L.is_moe = 0
                L.dense = O.Expert(self.matrix(dense_name(l, "gate")), self.matrix(dense_name(l, "up")),
                                   self.matrix(dense_name(l, "down")))
                self.layer_experts.append(None)
            else:
                L.is_moe = 1
                L.router = self.matrix(router_name(l))
                exps = []
                for e in range(c["experts"]):
                    if expert_encoded is not None:
                        exps.append(O.Expert(*(self.encoded_matrix(expert_dtype, expert_encoded(l, e, pj),
                                                                   *self.expert_shape(pj))
                                               for pj in ("gate", "up", "down"))))
                    else:
                        exps.append(O.Expert(*(self.matrix(expert_name(l, e, pj), expert_dtype)
                                               for pj in ("gate", "up", "down"))))
                arr = (O.Expert * len(exps))(*exps)
                self._keep.append(arr)
                L.experts = C.cast(arr, C.c_void_p)
                self.layer_experts.append(exps)
            layers.append(L)
        self.layers = (O.Layer * len(layers))(*layers)
        m = O.Model()
        m.hidden, m.n_layers, m.n_heads, m.n_kv_heads = h, c["layers"], c["heads"], c["kv_heads"]
        m.head_dim, m.vocab, m.n_experts, m.top_k = hd, c["vocab"], c["experts"] or 0, c["top_k"]
        m.normalize_topk = int(c["normalize"])
        m.eps, m.rope_theta = c["eps"], c["theta"]
        m.embed, m.lm_head = emb, head
        m.final_norm = self.vector("model.norm.weight")
        m.layers = C.cast(self.layers, C.c_void_p)
        self.model = m

    def raw(self, name):
        dt, shape, raw = self.t[name]
        return dt, shape, raw

    def f32(self, name):
        dt, shape, raw = self.t[name]
        if dt == "F32":
            return raw.view(np.float32).reshape(shape)
        if dt == "BF16":
            return (raw.view(np.uint16).astype(np.uint32) << 16).view(np.float32).reshape(shape)
        return O.decode(O.F16, raw.reshape(shape[0], -1), shape[-1])

    def matrix(self, name, dtype=None):
        """TensorSource::matrix (loader/safetensors.rs:141-160); optional re-encode."""
        dt, shape, raw = self.t[name]
        native = _ST_DTYPES[dt][1]
        rows, cols = shape
        if dtype is None or dtype == native:
            data = np.ascontiguousarray(raw)
            d = native
        else:
            data = O.encode(dtype, self.f32(name))
            d = dtype
        self._keep.append(data)
        return O.Matrix(d, rows, cols, data.ctypes.data)

    def expert_shape(self, proj):
        h, i = self.cfg["hidden"], self.cfg["expert_inter"]
        return (h, i) if proj == "down" else (i, h)

    def encoded_matrix(self, dtype, data, rows, cols):
        data = np.ascontiguousarray(data)
        assert data.nbytes == rows * O.row_bytes(dtype, cols)
        self._keep.append(data)
        return O.Matrix(dtype, rows, cols, data.ctypes.data)

    def vector(self, name):
        """TensorSource::vector (loader/safetensors.rs:162-170): decoded to f32."""
        v = np.ascontiguousarray(self.f32(name), dtype=np.float32)
        self._keep.append(v)
        return v.ctypes.data

    def new_cache(self, max_len):
        c = self.cfg
        shape = (c["layers"], max_len, c["kv_heads"] * c["head_dim"])
        return np.zeros(shape, dtype=np.float32), np.zeros(shape, dtype=np.float32), max_len

    def forward(self, token, position, cache, want_logits=True, parallel=True):
        kc, vc, max_len = cache
        hidden = np.zeros(self.cfg["hidden"], dtype=np.float32)
        logits = np.zeros(self.cfg["vocab"], dtype=np.float32) if want_logits else None
        rc = O.lib().ho_model_forward(C.byref(self.model), token, position, kc.ctypes.data,
                                      vc.ctypes.data, max_len, hidden.ctypes.data,
                                      logits.ctypes.data if logits is not None else None,
                                      int(parallel))
        if rc != 0:
            raise ValueError("bad token or position")
        return logits if want_logits else hidden

    def teacher_forced_logits(self, tokens):
        """tests/common/mod.rs:55-63."""
        cache = self.new_cache(len(tokens))
        return np.stack([self.forward(t, i, cache) for i, t in enumerate(tokens)])

    def greedy(self, prompt, n):
        """generate() with SamplingParams::greedy() (generator.rs:55-94)."""
        cache = self.new_cache(len(prompt) + n)
        for i, t in enumerate(prompt):
            logits = self.forward(t, i, cache, want_logits=(i == len(prompt) - 1))
        out = []
        pos = len(prompt)
        for step in range(n):
            tok = O.argmax(logits)
            out.append(tok)
            if step + 1 == n:
                break
            logits = self.forward(tok, pos, cache)
            pos += 1
        return out
