"""Checkpoint loading on the host: config normalisation, tensor naming and
the safetensors reader.

Follows the reference's unit tests in src/config.rs:289-356 (Qwen3-30B-A3B
and Mixtral-8x7B parameter counts, sparse step, unknown architecture) and
src/loader/safetensors.rs:277-362 (write/read round trip, index-selected
shards, overflowing offsets, truncated file), and checks that the loader
hands the decoder exactly the tensors the oracle's fixture loader reads.
"""
import importlib
import json
import os
import struct

import numpy as np
import pytest

from oracle import model as OM
from oracle import oracle as O

L = importlib.import_module("hale-token_b200.loader")
fmt = importlib.import_module("hale-token_b200.formats")

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")

QWEN3_30B = {
    "architectures": ["Qwen3MoeForCausalLM"],
    "hidden_size": 2048, "intermediate_size": 6144, "moe_intermediate_size": 768,
    "num_hidden_layers": 48, "num_attention_heads": 32, "num_key_value_heads": 4,
    "head_dim": 128, "vocab_size": 151936, "rms_norm_eps": 1e-6,
    "rope_theta": 1000000.0, "max_position_embeddings": 40960,
    "num_experts": 128, "num_experts_per_tok": 8, "norm_topk_prob": True,
    "decoder_sparse_step": 1, "mlp_only_layers": [], "tie_word_embeddings": False,
    "bos_token_id": 151643, "eos_token_id": 151645,
}
MIXTRAL_8X7B = {
    "architectures": ["MixtralForCausalLM"], "hidden_size": 4096,
    "intermediate_size": 14336, "num_hidden_layers": 32,
    "num_attention_heads": 32, "num_key_value_heads": 8, "vocab_size": 32000,
    "num_local_experts": 8, "num_experts_per_tok": 2, "eos_token_id": [2],
}


def test_parses_qwen3_30b_and_counts_parameters():
    c = L.ModelConfig.from_json_str(json.dumps(QWEN3_30B))
    assert c.architecture == L.QWEN3_MOE
    assert c.num_experts == 128 and c.num_moe_layers() == 48 and c.normalize_topk
    assert 30.0 <= c.total_params() / 1e9 < 31.0
    assert 3.0 <= c.active_params() / 1e9 < 3.6
    assert c.eos_token_ids == [151645] and c.bos_token_id == 151643
    assert c.rope_theta == 1e6 and c.max_position_embeddings == 40960


def test_mixtral_uses_num_local_experts_and_always_normalizes():
    c = L.ModelConfig.from_hf(dict(MIXTRAL_8X7B))
    assert c.num_experts == 8 and c.head_dim == 128
    assert c.expert_intermediate_size == 14336 and c.normalize_topk
    assert c.eos_token_ids == [2]
    assert 46.0 <= c.total_params() / 1e9 < 47.5
    assert c.rms_norm_eps == 1e-6 and c.rope_theta == 10000.0 and c.max_position_embeddings == 4096


def test_mixtral_ignores_norm_topk_prob_and_sparse_step():
    c = L.ModelConfig.from_hf(dict(MIXTRAL_8X7B, norm_topk_prob=False, decoder_sparse_step=2))
    assert c.normalize_topk and c.dense_layers == []


def test_sparse_step_marks_dense_layers():
    c = L.ModelConfig.from_hf(dict(QWEN3_30B, decoder_sparse_step=2))
    assert not c.is_moe_layer(0) and c.is_moe_layer(1)
    assert c.num_moe_layers() == 24


def test_mlp_only_layers_and_zero_step():
    c = L.ModelConfig.from_hf(dict(QWEN3_30B, mlp_only_layers=[0, 5], decoder_sparse_step=0))
    assert c.dense_layers == [0, 5]
    assert c.num_moe_layers() == 46


def test_qwen3_norm_topk_prob_defaults_to_false():
    hf = dict(QWEN3_30B)
    del hf["norm_topk_prob"]
    assert not L.ModelConfig.from_hf(hf).normalize_topk


def test_defaults_for_kv_heads_and_head_dim():
    hf = dict(MIXTRAL_8X7B)
    del hf["num_key_value_heads"]
    c = L.ModelConfig.from_hf(hf)
    assert c.num_kv_heads == 32 and c.head_dim == 128


def test_rejects_unknown_architecture():
    with pytest.raises(L.LoadError, match="unsupported model architecture"):
        L.ModelConfig.from_hf(dict(QWEN3_30B, architectures=["LlamaForCausalLM"]))
    with pytest.raises(L.LoadError):
        L.ModelConfig.from_hf(dict(QWEN3_30B, architectures=[]))


@pytest.mark.parametrize("patch", [
    {"num_key_value_heads": 5},          # 32 % 5 != 0
    {"head_dim": 127},                   # RoPE rotates pairs
    {"num_experts_per_tok": 0},
    {"num_experts_per_tok": 129},
])
def test_validate_rejects_inconsistent_shapes(patch):
    with pytest.raises(L.LoadError):
        L.ModelConfig.from_hf(dict(QWEN3_30B, **patch))


def test_missing_expert_count_and_bad_json():
    hf = dict(QWEN3_30B)
    del hf["num_experts"]
    with pytest.raises(L.LoadError, match="expert count"):
        L.ModelConfig.from_hf(hf)
    with pytest.raises(L.LoadError):
        L.ModelConfig.from_json_str("{not json")


def test_naming_of_both_architectures():
    q, m = L.Naming(L.QWEN3_MOE), L.Naming(L.MIXTRAL)
    assert q.expert(3, 7, "up") == "model.layers.3.mlp.experts.7.up_proj.weight"
    assert q.router(3) == "model.layers.3.mlp.gate.weight"
    assert m.expert(3, 7, "gate") == "model.layers.3.block_sparse_moe.experts.7.w1.weight"
    assert m.expert(3, 7, "down") == "model.layers.3.block_sparse_moe.experts.7.w2.weight"
    assert m.expert(3, 7, "up") == "model.layers.3.block_sparse_moe.experts.7.w3.weight"
    assert m.router(0) == "model.layers.0.block_sparse_moe.gate.weight"
    assert q.dense_mlp(1, "down") == "model.layers.1.mlp.down_proj.weight"
    assert L.Naming.attention(2, "q_norm") == "model.layers.2.self_attn.q_norm.weight"


def test_write_then_read_round_trip(tmp_path):
    w = fmt.encode(fmt.BF16, np.array([[1, 2, 3], [4, 5, 6]], np.float32))
    norm = np.array([0.5, -0.5], np.float32)
    L.write_safetensors(tmp_path / "model.safetensors",
                        [("w", [2, 3], "BF16", w), ("norm", [2], "F32", norm)])
    ck = L.Checkpoint.open_dir(str(tmp_path))
    assert ck.names() == ["norm", "w"]
    dt, rows, cols, data = ck.matrix("w")
    assert (dt, rows, cols) == (fmt.BF16, 2, 3)
    assert ck.f32("w").tolist() == [[1, 2, 3], [4, 5, 6]]
    assert ck.vector("norm").tolist() == [0.5, -0.5]
    with pytest.raises(L.MissingTensor):
        ck.matrix("absent")
    with pytest.raises(L.LoadError, match="expected 2-D"):
        ck.matrix("norm")
    with pytest.raises(L.LoadError, match="expected 1-D"):
        ck.vector("w")
    with open(tmp_path / "model.safetensors", "rb") as f:
        (hlen,) = struct.unpack("<Q", f.read(8))
    assert hlen % 8 == 0


def test_f16_tensors_decode_exactly(tmp_path):
    v = np.array([1.5, -2.25, 65504.0, 6.1035156e-05], np.float32)
    L.write_safetensors(tmp_path / "a.safetensors", [("v", [4], "F16", v.astype(np.float16))])
    assert L.Checkpoint.open_dir(str(tmp_path)).vector("v").tolist() == v.tolist()


def test_index_json_selects_the_listed_shards_only(tmp_path):
    one = np.array([[1.0, 2.0]], np.float32)
    L.write_safetensors(tmp_path / "model-00001-of-00001.safetensors", [("a", [1, 2], "F32", one)])
    L.write_safetensors(tmp_path / "consolidated.safetensors", [("other", [1, 2], "F32", one)])
    (tmp_path / "model.safetensors.index.json").write_text(
        '{"metadata": {}, "weight_map": {"a": "model-00001-of-00001.safetensors"}}')
    ck = L.Checkpoint.open_dir(str(tmp_path))
    assert ck.contains("a") and not ck.contains("other")


def test_shards_without_index_are_all_read(tmp_path):
    for i, n in enumerate(["b", "a"]):
        L.write_safetensors(tmp_path / f"part{i}.safetensors", [(n, [1], "F32", np.array([i], np.float32))])
    ck = L.Checkpoint.open_dir(str(tmp_path))
    assert ck.names() == ["a", "b"] and ck.vector("a").tolist() == [1.0]


def test_rejects_offsets_that_would_overflow(tmp_path):
    header = json.dumps({"t": {"dtype": "F32", "shape": [1], "data_offsets": [0, 2 ** 64 - 5]}}).encode()
    (tmp_path / "x.safetensors").write_bytes(struct.pack("<Q", len(header)) + header)
    with pytest.raises(L.LoadError, match="outside the file"):
        L.Checkpoint.open_dir(str(tmp_path))


def test_rejects_truncated_file_and_empty_dir(tmp_path):
    (tmp_path / "bad.safetensors").write_bytes(struct.pack("<Q", 1000))
    with pytest.raises(L.LoadError):
        L.Checkpoint.open_dir(str(tmp_path))
    empty = tmp_path / "empty"
    empty.mkdir()
    with pytest.raises(L.LoadError, match="no .safetensors"):
        L.Checkpoint.open_dir(str(empty))


def test_rejects_reversed_offsets_and_unsupported_dtype(tmp_path):
    header = json.dumps({"t": {"dtype": "F32", "shape": [1], "data_offsets": [4, 0]}}).encode()
    (tmp_path / "x.safetensors").write_bytes(struct.pack("<Q", len(header)) + header + bytes(4))
    with pytest.raises(L.LoadError):
        L.Checkpoint.open_dir(str(tmp_path))
    good = tmp_path / "g"
    good.mkdir()
    header = json.dumps({"t": {"dtype": "I32", "shape": [1, 1], "data_offsets": [0, 4]}}).encode()
    (good / "x.safetensors").write_bytes(struct.pack("<Q", len(header)) + header + bytes(4))
    with pytest.raises(L.LoadError, match="unsupported dtype"):
        L.Checkpoint.open_dir(str(good)).matrix("t")


@pytest.mark.parametrize("name", ["tiny-qwen3-moe", "tiny-mixtral"])
def test_fixture_config_matches_the_oracle_loader(name):
    d = os.path.join(GOLDEN, name)
    c = L.ModelConfig.from_dir(d)
    with open(os.path.join(d, "config.json")) as f:
        o = OM.normalize_config(json.load(f))
    assert (c.architecture == L.QWEN3_MOE) == o["qwen"]
    got = (c.hidden_size, c.expert_intermediate_size, c.dense_intermediate_size, c.num_layers, c.num_heads,
           c.num_kv_heads, c.head_dim, c.vocab_size, c.rms_norm_eps, c.rope_theta, c.max_position_embeddings,
           c.num_experts, c.experts_per_token, c.normalize_topk, c.tie_word_embeddings, c.dense_layers)
    want = tuple(o[k] for k in ("hidden", "expert_inter", "dense_inter", "layers", "heads", "kv_heads", "head_dim",
                                "vocab", "eps", "theta", "max_pos", "experts", "top_k", "normalize", "tie",
                                "dense_layers"))
    assert got == want


@pytest.mark.parametrize("name", ["tiny-qwen3-moe", "tiny-mixtral"])
@pytest.mark.parametrize("expert_dtype", [fmt.Q8_0, fmt.Q4_0])
def test_fixture_tensors_match_the_oracle_loader(name, expert_dtype):
    """Every tensor the decoder receives equals the oracle fixture loader's
    bytes, and each expert record equals the oracle encoder's rows."""
    d = os.path.join(GOLDEN, name)
    w = L.ModelWeights(d, expert_dtype)
    om = OM.OracleModel(d)
    expert_name, router_name, dense_name = OM._names(om.cfg["qwen"])

    def same(m, name):
        dt, shape, raw = om.raw(name)
        assert m[0] == {"F32": fmt.F32, "F16": fmt.F16, "BF16": fmt.BF16}[dt]
        assert (m[1], m[2]) == shape and bytes(m[3]) == bytes(raw)

    for l, Ld in enumerate(w.layers):
        p = f"model.layers.{l}."
        for k, n in (("q", "q_proj"), ("k", "k_proj"), ("v", "v_proj"), ("o", "o_proj")):
            same(Ld[k], p + f"self_attn.{n}.weight")
        np.testing.assert_array_equal(Ld["input_norm"], om.f32(p + "input_layernorm.weight"))
        np.testing.assert_array_equal(Ld["post_norm"], om.f32(p + "post_attention_layernorm.weight"))
        if om.cfg["qwen"]:
            np.testing.assert_array_equal(Ld["q_norm"], om.f32(p + "self_attn.q_norm.weight"))
        if l in om.cfg["dense_layers"]:
            for pj in ("gate", "up", "down"):
                same(Ld[f"dense_{pj}"], dense_name(l, pj))
        else:
            same(Ld["router"], router_name(l))
    for j, l in enumerate(w.moe_layers):
        for e in range(om.cfg["experts"]):
            want = fmt.pack_record(*[O.encode(expert_dtype, om.f32(expert_name(l, e, pj)))
                                     for pj in ("gate", "up", "down")])
            assert bytes(w.expert_record(j, e)) == bytes(want)
    same(w.embed, "model.embed_tokens.weight")
    np.testing.assert_array_equal(w.final_norm, om.f32("model.norm.weight"))


def test_missing_expert_tensor_is_reported(tmp_path):
    src = os.path.join(GOLDEN, "tiny-mixtral")
    ck = L.Checkpoint.open_dir(src)
    keep = [n for n in ck.names() if ".experts.3.w2." not in n]
    tensors = []
    for n in keep:
        dt, shape, raw = ck.raw(n)
        tensors.append((n, shape, dt, np.asarray(raw)))
    L.write_safetensors(tmp_path / "model.safetensors", tensors)
    with open(os.path.join(src, "config.json")) as f:
        (tmp_path / "config.json").write_text(f.read())
    with pytest.raises(L.MissingTensor, match="experts.3.w2"):
        L.ModelWeights(str(tmp_path))
