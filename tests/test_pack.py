"""Expert pack (experts.hpk), the converter and the tier planning, on the host.

Follows the reference's unit tests in src/expert/pack.rs:301-366 (records
written in any order read back, quantized packs smaller, garbage rejected),
src/expert/planner.rs:394-412 (budget split), src/expert/stats.rs:134-155
(hottest experts) and the converter's output (src/convert.rs:56-127).
"""
import importlib
import json
import os
import struct

import numpy as np
import pytest

from oracle import oracle as O

L = importlib.import_module("hale-token_b200.loader")
pk = importlib.import_module("hale-token_b200.pack")
fmt = importlib.import_module("hale-token_b200.formats")
hale = importlib.import_module("hale-token_b200")

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
TINY = {"architectures": ["MixtralForCausalLM"], "hidden_size": 64, "intermediate_size": 32,
        "num_hidden_layers": 2, "num_attention_heads": 4, "vocab_size": 10,
        "num_local_experts": 3, "num_experts_per_tok": 2}


def _expert(seed, dtype):
    m = lambda r, c, s: np.sin((np.arange(r * c, dtype=np.float32) + np.float32(s)) * np.float32(0.37)).reshape(r, c)
    return fmt.pack_record(fmt.encode(dtype, m(32, 64, seed)), fmt.encode(dtype, m(32, 64, seed + 1)),
                           fmt.encode(dtype, m(64, 32, seed + 2)))


def test_header_alignment_and_sizes():
    c = L.ModelConfig.from_hf(dict(TINY))
    f32 = pk.PackHeader.for_model(c, fmt.F32)
    q4 = pk.PackHeader.for_model(c, fmt.Q4_0)
    assert f32.record_stride % pk.ALIGN == 0 and f32.data_offset % pk.ALIGN == 0
    assert f32.record_bytes == 3 * 32 * 64 * 4
    assert q4.record_bytes * 7 < f32.record_bytes
    assert q4.moe_layers == [0, 1] and q4.num_experts == 3
    assert q4.file_size() == q4.data_offset + 2 * 3 * q4.record_stride
    js = json.loads(q4.to_json())
    assert list(js) == ["version", "dtype", "hidden_size", "intermediate_size", "num_experts", "moe_layers",
                        "record_bytes", "record_stride", "data_offset"]
    assert js["dtype"] == "q4_0"


@pytest.mark.parametrize("dtype", [fmt.F32, fmt.Q8_0, fmt.Q4_0])
def test_write_then_read_every_expert_in_any_order(tmp_path, dtype):
    c = L.ModelConfig.from_hf(dict(TINY))
    hd = pk.PackHeader.for_model(c, dtype)
    path = str(tmp_path / pk.PACK_FILE_NAME)
    w = pk.PackWriter(path, hd)
    keys = [(1, 2), (0, 0), (1, 0), (0, 1), (0, 2), (1, 1)]
    for l, e in keys:
        w.write_record(l, e, _expert(l * 10.0 + e, dtype))
    w.finish()
    src = pk.PackSource(path)
    assert src.header == hd
    for l, e in keys:
        assert bytes(src.record(l, e)) == bytes(_expert(l * 10.0 + e, dtype))
    assert src.expert_bytes == hd.record_bytes
    gate, up, down = src.split(src.record(1, 2))
    assert down.shape == (64, fmt.row_bytes(dtype, 32))
    with pytest.raises(L.LoadError, match="out of range"):
        src.record(0, 3)
    with pytest.raises(L.LoadError, match="no experts"):
        src.record(2, 0)
    with pytest.raises(L.LoadError, match="expected"):
        w2 = pk.PackWriter(str(tmp_path / "b.hpk"), hd)
        w2.write_record(0, 0, np.zeros(5, np.uint8))


def test_rejects_garbage_truncated_and_future_packs(tmp_path):
    junk = tmp_path / "junk.hpk"
    junk.write_bytes(b"definitely not a pack")
    with pytest.raises(L.LoadError, match="not a Hale expert pack"):
        pk.PackSource(str(junk))
    c = L.ModelConfig.from_hf(dict(TINY))
    hd = pk.PackHeader.for_model(c, fmt.Q8_0)
    path = tmp_path / "t.hpk"
    w = pk.PackWriter(str(path), hd)
    w.finish()
    with open(path, "r+b") as f:
        f.truncate(hd.file_size() - 1)
    with pytest.raises(L.LoadError, match="truncated pack"):
        pk.PackSource(str(path))
    hd2 = pk.PackHeader.for_model(c, fmt.Q8_0)
    hd2.version = 2
    pk.PackWriter(str(tmp_path / "v.hpk"), hd2).finish()
    with pytest.raises(L.LoadError, match="version 2"):
        pk.PackSource(str(tmp_path / "v.hpk"))
    big = tmp_path / "big.hpk"
    big.write_bytes(pk.MAGIC + struct.pack("<Q", pk.ALIGN * 64 + 1))
    with pytest.raises(L.LoadError, match="header too large"):
        pk.PackSource(str(big))


def test_decode_matches_the_oracle():
    rng = np.random.default_rng(3)
    v = rng.standard_normal((7, 128)).astype(np.float32)
    for dt in (fmt.F32, fmt.F16, fmt.BF16, fmt.Q8_0, fmt.Q4_0):
        enc = fmt.encode(dt, v)
        got = fmt.decode(dt, enc, 128)
        want = np.asarray(O.decode(dt, enc, 128), np.float32).reshape(7, 128)
        assert (got.view(np.uint32) == want.view(np.uint32)).all()


@pytest.mark.parametrize("name", ["tiny-qwen3-moe", "tiny-mixtral"])
def test_convert_checkpoint_layout(tmp_path, name):
    src = os.path.join(GOLDEN, name)
    dst = str(tmp_path / "out")
    rep = pk.convert_checkpoint(src, dst, fmt.Q4_0)
    assert sorted(os.listdir(dst)) == ["config.json", "dense.safetensors", "experts.hpk"]
    ck_src, ck_dst = L.Checkpoint.open_dir(src), L.Checkpoint.open_dir(dst)
    assert not any(".experts." in n for n in ck_dst.names())
    assert ck_dst.names() == [n for n in ck_src.names() if ".experts." not in n]
    for n in ck_dst.names():
        assert ck_dst.raw(n)[:2] == ck_src.raw(n)[:2] and bytes(ck_dst.raw(n)[2]) == bytes(ck_src.raw(n)[2])
    orig = L.ModelWeights(src, fmt.Q4_0)
    conv = L.ModelWeights(dst)
    assert conv.pack is not None and conv.expert_dtype == fmt.Q4_0
    assert rep["experts"] == len(orig.moe_layers) * orig.config.num_experts
    for j in range(len(orig.moe_layers)):
        for e in range(orig.config.num_experts):
            assert bytes(conv.expert_record(j, e)) == bytes(orig.expert_record(j, e))
    with pytest.raises(L.LoadError, match="must differ"):
        pk.convert_checkpoint(src, src)


def test_pack_in_another_dtype_is_reencoded(tmp_path):
    src = os.path.join(GOLDEN, "tiny-mixtral")
    dst = str(tmp_path / "q8")
    pk.convert_checkpoint(src, dst, fmt.Q8_0)
    w = L.ModelWeights(dst, fmt.Q4_0)
    hd = w.pack.header
    rec = w.pack.record(hd.moe_layers[0], 1)
    g, u, d = fmt.split_record(rec, fmt.Q8_0, hd.hidden_size, hd.intermediate_size)
    want = fmt.pack_record(fmt.encode(fmt.Q4_0, fmt.decode(fmt.Q8_0, g, hd.hidden_size)),
                           fmt.encode(fmt.Q4_0, fmt.decode(fmt.Q8_0, u, hd.hidden_size)),
                           fmt.encode(fmt.Q4_0, fmt.decode(fmt.Q8_0, d, hd.intermediate_size)))
    assert bytes(w.expert_record(0, 1)) == bytes(want)


def test_pack_must_match_the_config(tmp_path):
    src = os.path.join(GOLDEN, "tiny-mixtral")
    dst = tmp_path / "x"
    pk.convert_checkpoint(src, str(dst), fmt.Q8_0)
    cfg = json.loads((dst / "config.json").read_text())
    cfg["num_local_experts"] += 1
    (dst / "config.json").write_text(json.dumps(cfg))
    with pytest.raises(L.LoadError, match="does not match config.json"):
        L.ModelWeights(str(dst))


def test_small_budgets_pin_instead_of_thrashing_an_lru():
    assert L.split_budget(12, 48, 24) == (12, 0)
    assert L.split_budget(47, 48, 24) == (47, 0)
    assert L.split_budget(100, 1000, 24) == (50, 50)
    assert L.split_budget(2000, 1000, 24) == (1000, 0)


def test_hottest_orders_by_count_and_skips_unused():
    counts = np.zeros((2, 4), np.uint64)
    counts[1, 2], counts[0, 1], counts[0, 3] = 5, 3, 1
    assert L.hottest(counts, 10) == [(1, 2), (0, 1), (0, 3)]
    assert L.hottest(counts, 1) == [(1, 2)]
    counts[0, 0] = 5  # tie: lower index first
    assert L.hottest(counts, 2) == [(0, 0), (1, 2)]


def test_choose_pinned_spreads_over_layers_after_the_hottest():
    counts = np.zeros((3, 4), np.uint64)
    counts[2, 3] = 9
    assert L.choose_pinned(counts, 3, 4, 5) == [(2, 3), (0, 0), (1, 0), (2, 0), (0, 1)]
    assert L.choose_pinned(None, 3, 4, 4) == [(0, 0), (1, 0), (2, 0), (0, 1)]
    assert len(L.choose_pinned(None, 3, 4, 99)) == 12


def test_cache_policy_from_a_budget():
    c = L.ModelConfig.from_hf(dict(TINY))   # 2 MoE layers x 3 experts, top-2: 4 per token
    rb = 1000
    p = L.cache_policy(c, rb, 3 * rb)        # 3 < 2 * 4: all pinned
    assert isinstance(p, hale.CachePolicy) and len(p.pinned) == 3 and p.lru_bytes == 0
    p = L.cache_policy(c, rb, 6 * rb + 999)  # everything fits
    assert len(p.pinned) == 6 and p.lru_bytes == 0
    big = L.ModelConfig.from_hf(dict(TINY, num_hidden_layers=8, num_local_experts=8))  # 64 experts, 16 per token
    p = L.cache_policy(big, rb, 40 * rb)
    assert len(p.pinned) == 20 and p.lru_bytes == 20 * rb


def test_routing_stats_save_load_and_merge(tmp_path):
    s = L.RoutingStats(1, 3)
    s.record(0, 2)
    path = tmp_path / "stats.json"
    s.save(path)
    loaded = L.RoutingStats.load(path)
    assert loaded == s
    loaded.merge(s)
    assert loaded.count(0, 2) == 2
    loaded.merge(L.RoutingStats(2, 3))          # other shapes are ignored
    assert loaded.total() == 2
    d = json.loads(path.read_text())
    assert d == {"num_layers": 1, "num_experts": 3, "counts": [0, 0, 1]}
    path.write_text('{"num_layers": 2, "num_experts": 3, "counts": [1]}')
    with pytest.raises(L.LoadError, match="does not match"):
        L.RoutingStats.load(path)


def test_routing_stats_hottest_coverage_and_pool_layers():
    s = L.RoutingStats(2, 4)
    for _ in range(5):
        s.record(1, 2)
    for _ in range(3):
        s.record(0, 1)
    s.record(0, 3)
    assert s.hottest(10) == [(1, 2), (0, 1), (0, 3)]
    assert abs(s.coverage(2) - 8 / 9) < 1e-12
    c = L.ModelConfig.from_hf({"architectures": ["Qwen3MoeForCausalLM"], "hidden_size": 64,
                               "num_hidden_layers": 3, "num_attention_heads": 4, "vocab_size": 10,
                               "num_experts": 4, "num_experts_per_tok": 2, "mlp_only_layers": [1]})
    st = L.RoutingStats(3, 4)
    st.record(2, 3)                              # model layer 2 = MoE ordinal 1
    pc = st.pool_counts(c)
    assert pc.shape == (2, 4) and pc[1, 3] == 1 and pc.sum() == 1
    p = L.cache_policy(c, 100, 300, pc)         # 3 of 8 experts, below 2 x 4 per token: all pinned
    assert p.pinned == [(1, 3), (0, 0), (1, 0)] and p.lru_bytes == 0
