"""Tiered expert pools on the GPU (pinned + LRU in HBM, the rest in
page-locked host memory) against the resident pool and the reference's
cache semantics.

Restates the reference's tests/tiered_cache.rs:26-61 ("where an expert lives
must never change the answer": streaming with room for one expert gives the
same logits as fully resident), :104-126 (a routing-stats warm start pins
the hottest experts) and src/expert/cache.rs:244-272 (tiers consulted in
order, LRU eviction, counters). Expected counters come from a host
restatement of ExpertCache::fetch + LruCache (cache.rs:124-194,
lru.rs:97-125) driven by the same routes.
"""
import importlib
import json
import os
from collections import OrderedDict

import numpy as np
import pytest

from oracle import model as OM

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

hale = importlib.import_module("hale-token_b200")
fmt = importlib.import_module("hale-token_b200.formats")
loader = importlib.import_module("hale-token_b200.loader")
pk = importlib.import_module("hale-token_b200.pack")

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    c = hale.Context(0)
    yield c
    c.check()
    c.close()


class _DevBytes:
    def __init__(self, ptr, n):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "|u1", "data": (int(ptr), False), "version": 3}


def read_device(ptr, n):
    return torch.as_tensor(_DevBytes(ptr, n), device="cuda").cpu().numpy().copy()


class RefCache:
    """ExpertCache::fetch over LruCache (byte budget, equal weights)."""

    def __init__(self, pinned, lru_bytes, record_bytes):
        self.pinned, self.cap, self.w = set(pinned), lru_bytes, record_bytes
        self.lru = OrderedDict()
        self.pinned_hits = self.lru_hits = self.misses = 0

    def fetch(self, keys):
        missing = []
        for k in keys:
            if k in self.pinned:
                self.pinned_hits += 1
            elif k in self.lru:
                self.lru.move_to_end(k)
                self.lru_hits += 1
            else:
                missing.append(k)
        for k in missing:
            self.lru.pop(k, None)
            if self.w > self.cap:
                continue
            while (len(self.lru) + 1) * self.w > self.cap:
                self.lru.popitem(last=False)
            self.lru[k] = True
        self.misses += len(missing)

    def counters(self):
        return self.pinned_hits, self.lru_hits, self.misses, len(self.lru), len(self.lru) * self.w


def upload_all(pool, layers):
    for j, ld in enumerate(layers):
        for e in range(ld.E):
            pool.upload(j, e, ld.record(e))


def test_tiers_are_consulted_in_order(ctx):
    layers = [fmt.SyntheticLayer(70 + j, 8, 128, 64, fmt.Q8_0) for j in range(2)]
    res = hale.Pool(ctx, fmt.Q8_0, 128, 64, 2, 8)
    upload_all(res, layers)
    rb = res.expert_bytes
    pool = hale.Pool(ctx, fmt.Q8_0, 128, 64, 2, 8, policy=hale.CachePolicy([(0, 0)], 2 * rb))
    upload_all(pool, layers)
    assert pool.hbm_slots == 1 + 2 + 8
    s = pool.stats()
    assert (s.pinned_experts, s.pinned_bytes, s.lru_capacity_bytes, s.misses) == (1, rb, 2 * rb, 0)

    keys = [(0, 0), (0, 1), (0, 2)]
    got, want = pool.fetch(keys), res.fetch(keys)
    for g, w in zip(got, want):
        n = 3 * (w[1] - w[0])      # gate | up | down, equal tiled sizes
        assert (read_device(g[0], n) == read_device(w[0], n)).all()
    pool.fetch([(0, 1), (0, 2)])   # both LRU hits
    pool.fetch([(0, 3)])           # evicts (0, 1), the least recently used
    g = pool.fetch([(0, 1)])       # a miss again
    w = res.fetch([(0, 1)])
    n = 3 * (w[0][1] - w[0][0])
    assert (read_device(g[0][0], n) == read_device(w[0][0], n)).all()
    s = pool.stats()
    assert (s.pinned_hits, s.lru_hits, s.misses) == (1, 2, 4)
    assert (s.lru_experts, s.lru_bytes, s.bytes_loaded) == (2, 2 * rb, 4 * rb)
    assert s.load_seconds > 0 and not s.passthrough
    assert pool.routing_counts()[0, 1] == 3
    with pytest.raises(hale.HaleError):
        pool.fetch([(2, 0)])


def _forward(ctx, pool, ld, layer_idx, x, k, norm):
    r_dev = torch.from_numpy(fmt.encode(fmt.F32, ld.router)).cuda()
    layer = hale.moe_layer(layer_idx, r_dev, fmt.F32, ld.E, k, norm)
    out = torch.full((x.shape[0], ld.H), float("nan"), dtype=torch.float32, device="cuda")
    idx = torch.zeros((x.shape[0], k), dtype=torch.int32, device="cuda")
    w = torch.zeros((x.shape[0], k), dtype=torch.float32, device="cuda")
    hale.moe_forward(ctx, pool, layer, torch.from_numpy(x).cuda(), out, idx, w)
    torch.cuda.synchronize()
    return out.cpu().numpy(), idx.cpu().numpy()


@pytest.mark.parametrize("dtype", [fmt.Q8_0, fmt.Q4_0])
@pytest.mark.parametrize("policy", ["one-expert", "pinned+lru", "nothing"])
def test_tiered_forward_is_bit_identical_to_resident(ctx, dtype, policy):
    E, H, I, k = 16, 256, 128, 4
    layers = [fmt.SyntheticLayer(90 + j, E, H, I, dtype) for j in range(2)]
    res = hale.Pool(ctx, dtype, H, I, 2, E)
    upload_all(res, layers)
    rb = res.expert_bytes
    pinned, lru = {"one-expert": ([], rb), "pinned+lru": ([(0, 3), (1, 5), (1, 0)], 6 * rb),
                   "nothing": ([], 0)}[policy]
    pool = hale.Pool(ctx, dtype, H, I, 2, E, policy=hale.CachePolicy(pinned, lru))
    upload_all(pool, layers)
    ref = RefCache(pinned, lru, rb)
    for step, (j, m) in enumerate([(0, 1), (1, 1), (0, 5), (1, 64), (0, 1), (0, 33), (1, 2)]):
        x = layers[j].tokens(m, seed=step)
        want, want_idx = _forward(ctx, res, layers[j], j, x, k, True)
        got, got_idx = _forward(ctx, pool, layers[j], j, x, k, True)
        assert (got_idx == want_idx).all()
        assert (got.view(np.uint32) == want.view(np.uint32)).all(), f"step {step}: tiers changed the result"
        for t in range(m):
            ref.fetch([(j, int(e)) for e in want_idx[t]])
    s = pool.stats()
    assert (s.pinned_hits, s.lru_hits, s.misses, s.lru_experts, s.lru_bytes) == ref.counters()
    assert s.bytes_loaded == ref.misses * rb
    routed = res.routing_counts()
    assert (pool.routing_counts() == routed).all()


def test_routing_stats_warm_start_pins_the_hottest_experts(ctx, tmp_path):
    E, H, I, k = 16, 128, 64, 2
    layers = [fmt.SyntheticLayer(110 + j, E, H, I, fmt.Q8_0) for j in range(2)]
    rb = layers[0].expert_bytes()
    first = hale.Pool(ctx, fmt.Q8_0, H, I, 2, E, policy=hale.CachePolicy([], 1))
    upload_all(first, layers)
    for j in range(2):
        _forward(ctx, first, layers[j], j, layers[j].tokens(8, seed=j), k, False)
    cfg = loader.ModelConfig.from_hf({"architectures": ["MixtralForCausalLM"], "hidden_size": H,
                                      "intermediate_size": I, "num_hidden_layers": 2, "num_attention_heads": 4,
                                      "vocab_size": 10, "num_local_experts": E, "num_experts_per_tok": k})
    # saved after the first run and loaded at the next start (stats.rs save / load)
    loader.RoutingStats.from_pool(first, cfg).save(tmp_path / "routing.json")
    counts = loader.RoutingStats.load(tmp_path / "routing.json").pool_counts(cfg)
    assert (counts == first.routing_counts()).all()
    policy = loader.cache_policy(cfg, rb, 4 * rb, counts)   # 4 < 2 x (2 layers x top-2): all pinned
    assert len(policy.pinned) == 4 and policy.lru_bytes == 0
    assert policy.pinned == loader.hottest(counts, 4)
    second = hale.Pool(ctx, fmt.Q8_0, H, I, 2, E, policy=policy)
    upload_all(second, layers)
    for j in range(2):
        _forward(ctx, second, layers[j], j, layers[j].tokens(8, seed=j), k, False)
    s = second.stats()
    assert (s.pinned_experts, s.lru_capacity_bytes) == (4, 0)
    assert s.pinned_hits > 0


@pytest.mark.parametrize("name", ["tiny-qwen3-moe", "tiny-mixtral"])
def test_streaming_decoder_is_bit_identical_to_resident(ctx, tmp_path, name):
    """tiered_cache.rs:26-61 on a converted model directory (dense
    safetensors + experts.hpk): room for a single expert in HBM."""
    src = os.path.join(GOLDEN, name)
    with open(os.path.join(src, "expected.json")) as f:
        tokens = json.load(f)["tokens"]
    dst = str(tmp_path / "converted")
    pk.convert_checkpoint(src, dst, fmt.Q8_0)
    want = OM.OracleModel(src, expert_dtype=fmt.Q8_0).teacher_forced_logits(tokens)

    def run(**kw):
        dec, pool, cfg = loader.load_decoder(ctx, dst, max_len=len(tokens), **kw)
        logits = torch.empty(cfg.vocab_size, dtype=torch.float32, device="cuda")
        out = []
        for i, t in enumerate(tokens):
            dec.forward(t, i, logits)
            out.append(logits.cpu().numpy().copy())
        ctx.check()
        s = pool.stats()
        dec.close()
        return np.stack(out), s

    resident, r = run()
    assert r.misses == 0 and r.pinned_experts > 0
    one = loader.ModelWeights(dst).record_bytes
    streaming, s = run(policy=hale.CachePolicy([], one))
    assert s.misses > s.lru_hits and s.bytes_loaded > 0
    assert (resident.view(np.uint32) == streaming.view(np.uint32)).all(), "tiers changed the result"
    assert (resident.view(np.uint32) == want.view(np.uint32)).all()
    budget, b = run(expert_hbm_bytes=3 * one)
    assert b.pinned_experts == 3 and b.lru_capacity_bytes == 0
    assert (budget.view(np.uint32) == want.view(np.uint32)).all()


def test_expert_source_fills_the_cold_tier_and_reports_io_errors(ctx):
    """ExpertSource::load (src/expert/mod.rs:110-124) as a host callback:
    a tiered pool with nothing uploaded asks the source for each expert the
    first time a request names it -- the results equal the resident pool's.
    A source that fails (like CountingSource's injected I/O error,
    src/expert/cache.rs:211-244) makes the forward return E_IO before any
    counter or slot changes; the pool then serves normally again."""
    E, H, I, k = 16, 256, 128, 4
    dtype = fmt.Q8_0
    ld = fmt.SyntheticLayer(77, E, H, I, dtype)
    res = hale.Pool(ctx, dtype, H, I, 1, E)
    upload_all(res, [ld])
    rb = res.expert_bytes
    pool = hale.Pool(ctx, dtype, H, I, 1, E, policy=hale.CachePolicy([(0, 2)], 3 * rb))
    records = {e: fmt.pack_record(*ld.expert_encoded(e)) for e in range(E)}
    asked = []

    def good(layer, expert):
        asked.append((layer, expert))
        return records[expert]

    pool.set_source(good)
    x = ld.tokens(6, seed=1)
    want, want_idx = _forward(ctx, res, ld, 0, x, k, True)
    got, got_idx = _forward(ctx, pool, ld, 0, x, k, True)
    assert (got_idx == want_idx).all()
    assert (got.view(np.uint32) == want.view(np.uint32)).all()
    first = sorted(set(asked))
    assert first == sorted({(0, int(e)) for e in want_idx.reshape(-1)})     # each expert asked once
    before = pool.stats()
    # a failing source: an expert no request has named yet
    unseen = [e for e in range(E) if (0, e) not in set(asked)]
    bad_expert = unseen[0]
    pool.set_source(lambda layer, expert: None if expert == bad_expert else records[expert])
    x2 = None
    for seed in range(2, 400):             # tokens whose routes name the failing expert
        cand = ld.tokens(4, seed=seed)
        _, idx_c = _forward(ctx, res, ld, 0, cand, k, True)
        if bad_expert in idx_c:
            x2 = cand
            break
    assert x2 is not None
    with pytest.raises(hale.HaleError) as ei:
        _forward(ctx, pool, ld, 0, x2, k, True)
    assert ei.value.status == hale.E_IO
    after = pool.stats()
    assert (after.pinned_hits, after.lru_hits, after.misses, after.lru_experts) == \
        (before.pinned_hits, before.lru_hits, before.misses, before.lru_experts)
    pool.set_source(good)
    want2, _ = _forward(ctx, res, ld, 0, x2, k, True)
    got2, _ = _forward(ctx, pool, ld, 0, x2, k, True)
    assert (got2.view(np.uint32) == want2.view(np.uint32)).all()
    ctx.check()
