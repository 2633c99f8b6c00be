"""GPU parity: the CUDA path through the C ABI against the CPU oracle.

Bar: router top-k indices and per-block int32 dot
sums bit-exact; layer outputs and logits within 1e-4 relative. This build
holds every comparison below to bit-exactness (the kernels keep the
reference's f32 operation order and glibc's expf), except where a test
states a tolerance.
"""
import importlib

import numpy as np
import pytest

from oracle import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

hale = importlib.import_module("hale-token_b200")
fmt = importlib.import_module("hale-token_b200.formats")

REL_TOL = 1e-4  # the north star's layer-output / logit tolerance


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    c = hale.Context(0)
    yield c
    c.check()
    c.close()


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def bits(a):
    a = np.ascontiguousarray(a)
    return a.view(np.uint32) if a.dtype == np.float32 else a


def assert_bit_equal(got, want, what=""):
    got, want = np.asarray(got), np.asarray(want)
    assert got.shape == want.shape, (what, got.shape, want.shape)
    eq = bits(got) == bits(want)
    if not eq.all():
        i = np.argwhere(~eq)[0]
        raise AssertionError(f"{what}: {(~eq).sum()} of {eq.size} differ; first at {tuple(i)}: "
                             f"got {got[tuple(i)]!r} want {want[tuple(i)]!r}")


# ---------------------------------------------------------------------------
# Q8Activations::quantize (quant.rs:77-93)
# ---------------------------------------------------------------------------
def test_quantize_q8_is_bit_exact(ctx):
    rng = np.random.default_rng(0)
    x = rng.standard_normal((7, 256)).astype(np.float32)
    x[1, :32] = 0.0                      # zero block -> scale 0, inv 0
    x[2, 40] = 1e30                      # huge value
    x[3, 64:96] = np.float32(0.5) * np.arange(32, dtype=np.float32)  # exact halves
    x[4, 100] = np.nan                   # NaN is ignored by the max and casts to 0
    scales = torch.zeros((7, 8), dtype=torch.float32, device="cuda")
    quants = torch.zeros((7, 256), dtype=torch.int8, device="cuda")
    hale.quantize_q8(ctx, dev(x), scales, quants)
    ws, wq = O.quantize_q8(x)
    torch.cuda.synchronize()
    assert_bit_equal(scales.cpu().numpy(), ws, "scales")
    assert_bit_equal(quants.cpu().numpy(), wq, "quants")


# ---------------------------------------------------------------------------
# WeightMatrix::matvec, quantized (matrix.rs:115-126, quant.rs:115-144)
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("dtype", [fmt.Q4_0, fmt.Q8_0])
@pytest.mark.parametrize("rows,cols,m", [(70, 64, 1), (64, 256, 3), (96, 2048, 8), (33, 768, 33),
                                         (768, 2048, 2)])
def test_quantized_matvec_and_block_sums_are_bit_exact(ctx, dtype, rows, cols, m):
    rng = np.random.default_rng(rows * 7 + cols + m)
    w = rng.standard_normal((rows, cols)).astype(np.float32) * 0.02
    enc = fmt.encode(dtype, w)
    x = rng.standard_normal((m, cols)).astype(np.float32)
    mat = hale.Matrix(ctx, dtype, rows, cols, enc)
    out = torch.zeros((m, rows), dtype=torch.float32, device="cuda")
    sums = torch.zeros((m, rows, cols // 32), dtype=torch.int32, device="cuda")
    mat.matvec(dev(x), out, sums)
    torch.cuda.synchronize()
    got, got_sums = out.cpu().numpy(), sums.cpu().numpy()
    want = np.stack([O.matvec(dtype, enc, rows, cols, x[t]) for t in range(m)])
    assert_bit_equal(got, want, "matvec")
    for t in range(m):
        xs, xq = O.quantize_q8(x[t])
        for r in range(0, rows, max(1, rows // 9)):
            _, s = O.dot_quantized(dtype, enc[r], xs, xq, want_block_sums=True)
            assert_bit_equal(got_sums[t, r], s, f"block sums t={t} r={r}")


@pytest.mark.parametrize("dtype", [fmt.Q4_0, fmt.Q8_0])
@pytest.mark.parametrize("rows,cols,m", [(70, 64, 3), (96, 2048, 8), (33, 768, 13), (768, 2048, 5)])
def test_quantized_matvec_without_block_sums_is_bit_exact(ctx, dtype, rows, cols, m):
    """Without the block-sum output, passes of 3+ rows take the warp-level
    tensor-core MMA path; results must not change."""
    rng = np.random.default_rng(rows * 11 + cols + m)
    enc = fmt.encode(dtype, rng.standard_normal((rows, cols)).astype(np.float32) * 0.02)
    x = rng.standard_normal((m, cols)).astype(np.float32)
    mat = hale.Matrix(ctx, dtype, rows, cols, enc)
    out = torch.zeros((m, rows), dtype=torch.float32, device="cuda")
    mat.matvec(dev(x), out)
    torch.cuda.synchronize()
    want = np.stack([O.matvec(dtype, enc, rows, cols, x[t]) for t in range(m)])
    assert_bit_equal(out.cpu().numpy(), want, "matvec")


@pytest.mark.parametrize("dtype", [fmt.Q4_0, fmt.Q8_0])
def test_block_sums_are_bit_exact_on_identical_quantized_inputs(ctx, dtype):
    """dot_quantized with caller-supplied Q8Activations (quant.rs:107-113)."""
    rng = np.random.default_rng(11)
    rows, cols, m = 64, 768, 5
    enc = fmt.encode(dtype, rng.standard_normal((rows, cols)).astype(np.float32) * 0.02)
    xs, xq = O.quantize_q8(rng.standard_normal((m, cols)).astype(np.float32))
    xq[0, :32] = -128                    # the i8 extremes the activations can hold
    xq[1, 32:64] = 127
    mat = hale.Matrix(ctx, dtype, rows, cols, enc)
    out = torch.zeros((m, rows), dtype=torch.float32, device="cuda")
    sums = torch.zeros((m, rows, cols // 32), dtype=torch.int32, device="cuda")
    mat.matvec_q8(dev(xs), dev(xq), out, sums)
    torch.cuda.synchronize()
    for t in range(m):
        for r in range(rows):
            v, s = O.dot_quantized(dtype, enc[r], xs[t], xq[t], want_block_sums=True)
            assert_bit_equal(sums[t, r].cpu().numpy(), s, "sums")
            assert_bit_equal(np.float32(out[t, r].item()), np.float32(v), "dot")


# ---------------------------------------------------------------------------
# float matvec / lm_head (quant.rs:146-202, transformer.rs:217-221)
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("dtype", [fmt.F32, fmt.BF16, fmt.F16])
@pytest.mark.parametrize("rows,cols,m", [(70, 64, 1), (37, 13, 2), (300, 100, 5), (1024, 256, 9)])
def test_float_matvec_is_bit_exact(ctx, dtype, rows, cols, m):
    rng = np.random.default_rng(rows + cols * 3 + m)
    w = rng.standard_normal((rows, cols)).astype(np.float32) * 0.05
    enc = fmt.encode(dtype, w)
    x = rng.standard_normal((m, cols)).astype(np.float32)
    mat = hale.Matrix(ctx, dtype, rows, cols, enc)
    out = torch.zeros((m, rows), dtype=torch.float32, device="cuda")
    mat.lm_head(dev(x), out)
    torch.cuda.synchronize()
    want = np.stack([O.matvec(dtype, enc, rows, cols, x[t]) for t in range(m)])
    assert_bit_equal(out.cpu().numpy(), want, "float matvec")


def test_lm_head_at_vocab_scale(ctx):
    """Transformer::logits on a [V=32000, H=4096] bf16 head (Mixtral shape)."""
    rng = np.random.default_rng(5)
    V, H = 32000, 4096
    w = (rng.standard_normal((V, H), dtype=np.float32) * 0.02)
    enc = fmt.encode(fmt.BF16, w)
    h = rng.standard_normal((2, H)).astype(np.float32)
    mat = hale.Matrix(ctx, fmt.BF16, V, H, enc)
    out = torch.zeros((2, V), dtype=torch.float32, device="cuda")
    mat.lm_head(dev(h), out)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    rows = rng.choice(V, 512, replace=False)
    for t in range(2):
        want = O.matvec(fmt.BF16, enc[rows], len(rows), H, h[t])
        assert_bit_equal(got[t, rows], want, "lm_head rows")


# ---------------------------------------------------------------------------
# MoeLayer::route (moe.rs:36-53)
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("E,k,H,m,norm,rdt", [(16, 4, 256, 5, True, fmt.F32), (128, 8, 2048, 64, True, fmt.F32),
                                              (8, 2, 64, 3, False, fmt.BF16), (128, 8, 2048, 1, True, fmt.BF16),
                                              (12, 3, 40, 7, True, fmt.F32), (5, 2, 13, 3, True, fmt.F32)])
def test_route_matches_the_oracle_bit_for_bit(ctx, E, k, H, m, norm, rdt):
    rng = np.random.default_rng(E + k + H + m)
    router = rng.standard_normal((E, H)).astype(np.float32) * 0.02
    renc = fmt.encode(rdt, router)
    x = rng.standard_normal((m, H)).astype(np.float32)
    r_dev = dev(renc)
    layer = hale.moe_layer(0, r_dev, rdt, E, k, norm)
    idx = torch.zeros((m, k), dtype=torch.int32, device="cuda")
    w = torch.zeros((m, k), dtype=torch.float32, device="cuda")
    probs = torch.zeros((m, E), dtype=torch.float32, device="cuda")
    hale.moe_route(ctx, layer, H, dev(x), idx, w, probs)
    torch.cuda.synchronize()
    for t in range(m):
        wi, ww = O.moe_route(rdt, renc, E, k, norm, x[t])
        assert list(idx[t].cpu().numpy()) == list(wi), t
        assert_bit_equal(w[t].cpu().numpy(), ww, f"weights t={t}")
        lg = O.matvec(rdt, renc, E, H, x[t])
        assert_bit_equal(probs[t].cpu().numpy(), O.softmax(lg), f"probs t={t}")


def test_route_ties_prefer_the_lower_expert_index(ctx):
    """topk.rs:130-139: equal router rows give equal probabilities."""
    E, k, H = 8, 3, 64
    rng = np.random.default_rng(1)
    router = rng.standard_normal((E, H)).astype(np.float32) * 0.02
    router[5] = router[2]
    router[6] = router[2]
    router[7] = router[1]
    x = rng.standard_normal((4, H)).astype(np.float32)
    renc = fmt.encode(fmt.F32, router)
    layer = hale.moe_layer(0, dev(renc), fmt.F32, E, k, True)
    idx = torch.zeros((4, k), dtype=torch.int32, device="cuda")
    w = torch.zeros((4, k), dtype=torch.float32, device="cuda")
    hale.moe_route(ctx, layer, H, dev(x), idx, w)
    torch.cuda.synchronize()
    for t in range(4):
        wi, ww = O.moe_route(fmt.F32, renc, E, k, True, x[t])
        assert list(idx[t].cpu().numpy()) == list(wi)
        assert_bit_equal(w[t].cpu().numpy(), ww)


# ---------------------------------------------------------------------------
# MoeLayer::forward (moe.rs:56-70) through the expert pool
# ---------------------------------------------------------------------------
def build_pool(ctx, layer_def, n_layers=1, layer_index=0):
    pool = hale.Pool(ctx, layer_def.dtype, layer_def.H, layer_def.I, n_layers, layer_def.E)
    experts = []
    for e in range(layer_def.E):
        g, u, d = layer_def.expert_encoded(e)
        pool.upload(layer_index, e, fmt.pack_record(g, u, d))
        experts.append(O.ExpertWeights(layer_def.dtype, layer_def.H, layer_def.I, g, u, d))
    return pool, experts


def run_forward(ctx, pool, ld, x, k, norm, layer_index=0, rdt=fmt.F32):
    renc = fmt.encode(rdt, ld.router)
    r_dev = dev(renc)
    layer = hale.moe_layer(layer_index, r_dev, rdt, ld.E, k, norm)
    m = x.shape[0]
    out = torch.full((m, ld.H), float("nan"), dtype=torch.float32, device="cuda")
    idx = torch.zeros((m, k), dtype=torch.int32, device="cuda")
    w = torch.zeros((m, k), dtype=torch.float32, device="cuda")
    hale.moe_forward(ctx, pool, layer, dev(x), out, idx, w)
    ctx.check()
    return out.cpu().numpy(), idx.cpu().numpy(), w.cpu().numpy(), renc


@pytest.mark.parametrize("dtype", [fmt.Q8_0, fmt.Q4_0])
@pytest.mark.parametrize("m", [1, 2, 7, 32, 40])
def test_moe_forward_tiny_config_is_bit_exact(ctx, dtype, m):
    """BASELINE config 0 layer shape: H=256, 16 experts top-4, I=128."""
    ld = fmt.SyntheticLayer(100 + m, 16, 256, 128, dtype)
    pool, experts = build_pool(ctx, ld)
    x = ld.tokens(m)
    out, idx, w, renc = run_forward(ctx, pool, ld, x, 4, True)
    want, widx, ww = O.moe_forward(fmt.F32, renc, experts, 4, True, x)
    assert np.array_equal(idx, widx.astype(np.int32))
    assert_bit_equal(w, ww, "weights")
    assert_bit_equal(out, want, "layer output")


@pytest.mark.parametrize("m", [1, 8, 64, 512])
def test_moe_forward_qwen3_30b_shape_is_bit_exact(ctx, m):
    """BASELINE config 1 shape: H=2048, 128 experts top-8, I=768, q4_0, at
    every batch size the config names. Every token of the batch is checked
    against the oracle (the -march=native OpenMP build keeps M=512 to about
    a second of CPU time)."""
    ld = fmt.SyntheticLayer(7, 128, 2048, 768, fmt.Q4_0)
    pool, experts = build_pool(ctx, ld)
    x = ld.tokens(m)
    out, idx, w, renc = run_forward(ctx, pool, ld, x, 8, True)
    want, widx, ww = O.moe_forward(fmt.F32, renc, experts, 8, True, x, native=True)
    assert np.array_equal(idx, widx.astype(np.int32))
    assert_bit_equal(w, ww, "weights")
    assert_bit_equal(out, want, "layer output")


def test_moe_forward_full_batch_properties(ctx):
    """M=512 (the largest config-1 batch) on other seeds: deterministic run
    to run, routing stats count every route, and every token matches the
    oracle."""
    ld = fmt.SyntheticLayer(9, 128, 2048, 768, fmt.Q4_0)
    pool, experts = build_pool(ctx, ld)
    x = ld.tokens(512)
    a = run_forward(ctx, pool, ld, x, 8, True)
    b = run_forward(ctx, pool, ld, x, 8, True)
    assert_bit_equal(a[0], b[0], "determinism")
    want, widx, ww = O.moe_forward(fmt.F32, a[3], experts, 8, True, x, native=True)
    assert np.array_equal(a[1], widx.astype(np.int32))
    assert_bit_equal(a[0], want, "every token")
    counts = pool.routing_counts()
    assert counts.sum() == 2 * 512 * 8
    per_expert = np.bincount(a[1].reshape(-1), minlength=128)
    assert np.array_equal(counts[0], 2 * per_expert)


def test_moe_forward_mixtral_q8_shape_sample(ctx):
    """q8_0 experts, 8 experts top-2, H=4096 (Mixtral layout, I reduced)."""
    ld = fmt.SyntheticLayer(21, 8, 4096, 1024, fmt.Q8_0)
    pool, experts = build_pool(ctx, ld)
    x = ld.tokens(6)
    out, idx, w, renc = run_forward(ctx, pool, ld, x, 2, True)
    want, widx, ww = O.moe_forward(fmt.F32, renc, experts, 2, True, x)
    assert np.array_equal(idx, widx.astype(np.int32))
    assert_bit_equal(out, want, "layer output")


def test_moe_forward_host_buffers_and_second_layer(ctx):
    """hale_moe_forward_host with a 2-layer pool, routing layer 1."""
    ld = fmt.SyntheticLayer(31, 16, 256, 128, fmt.Q4_0)
    pool = hale.Pool(ctx, fmt.Q4_0, 256, 128, 2, 16)
    experts = []
    for e in range(16):
        g, u, d = ld.expert_encoded(e)
        pool.upload(1, e, fmt.pack_record(g, u, d))
        experts.append(O.ExpertWeights(fmt.Q4_0, 256, 128, g, u, d))
    x = ld.tokens(5)
    renc = fmt.encode(fmt.F32, ld.router)
    layer = hale.moe_layer(1, dev(renc), fmt.F32, 16, 4, True)
    out = np.zeros((5, 256), np.float32)
    idx = np.zeros((5, 4), np.int32)
    w = np.zeros((5, 4), np.float32)
    hale.moe_forward_host(ctx, pool, layer, x, out, idx, w)
    want, widx, ww = O.moe_forward(fmt.F32, renc, experts, 4, True, x)
    assert_bit_equal(out, want, "host forward")
    # layer 0 has no experts uploaded: forward must refuse, not guess
    layer0 = hale.moe_layer(0, dev(renc), fmt.F32, 16, 4, True)
    with pytest.raises(hale.HaleError) as ei:
        hale.moe_forward_host(ctx, pool, layer0, x, out)
    assert ei.value.status == hale.E_INVALID_ARGUMENT


def test_moe_forward_host_replays_with_new_inputs(ctx):
    """Repeated host-buffer calls on the same page-locked buffers replay one
    captured graph: every call must still read the buffers' current contents
    and match the oracle, also after the workspace grew in between."""
    ld = fmt.SyntheticLayer(33, 16, 256, 128, fmt.Q8_0)
    pool, experts = build_pool(ctx, ld)
    renc = fmt.encode(fmt.F32, ld.router)
    layer = hale.moe_layer(0, dev(renc), fmt.F32, 16, 4, True)
    xh = torch.empty((6, 256), dtype=torch.float32).pin_memory()
    oh = torch.empty((6, 256), dtype=torch.float32).pin_memory()
    ih = torch.empty((6, 4), dtype=torch.int32).pin_memory()
    for step in range(5):
        if step == 3:   # a bigger call grows the workspace: cached graphs must be dropped
            big = torch.from_numpy(ld.tokens(1500, seed=77)).cuda()
            hale.moe_forward(ctx, pool, layer, big, torch.empty_like(big))
            ctx.check()
        x = ld.tokens(6, seed=step)
        xh.copy_(torch.from_numpy(x))
        hale.moe_forward_host(ctx, pool, layer, xh, oh, ih)
        want, widx, _ = O.moe_forward(fmt.F32, renc, experts, 4, True, x)
        assert np.array_equal(ih.numpy(), widx.astype(np.int32)), f"step {step}"
        assert_bit_equal(oh.numpy(), want, f"host forward step {step}")


def test_pool_fetch_keeps_request_order_and_counts(ctx):
    """ExpertProvider::fetch (cache.rs:246-272 analogue)."""
    ld = fmt.SyntheticLayer(41, 4, 64, 32, fmt.Q8_0)
    pool, _ = build_pool(ctx, ld)
    views = pool.fetch([(0, 2), (0, 0), (0, 2)])
    assert views[0] == views[2] and views[0] != views[1]
    s = pool.stats()
    assert (s.pinned_hits, s.misses, s.pinned_experts) == (3, 0, 4)
    with pytest.raises(hale.HaleError):
        pool.fetch([(0, 9)])
    assert pool.stats().misses == 1
    counts = pool.routing_counts()
    assert counts[0, 2] == 2 and counts[0, 0] == 1


def test_bad_arguments_are_errors_not_crashes(ctx):
    ld = fmt.SyntheticLayer(51, 4, 64, 32, fmt.Q4_0)
    pool, _ = build_pool(ctx, ld)
    renc = dev(fmt.encode(fmt.F32, ld.router))
    x = dev(ld.tokens(2))
    out = torch.zeros((2, 64), device="cuda")
    for k in (0, 5):
        with pytest.raises(hale.HaleError):
            hale.moe_forward(ctx, pool, hale.moe_layer(0, renc, fmt.F32, 4, k, True), x, out)
    with pytest.raises(hale.HaleError):
        hale.moe_forward(ctx, pool, hale.moe_layer(0, renc, fmt.Q8_0, 4, 2, True), x, out)
    with pytest.raises(hale.HaleError):  # wrong record size
        pool.upload(0, 1, np.zeros(10, np.uint8))
    with pytest.raises(hale.HaleError):  # ragged quantized rows
        hale.Matrix(ctx, fmt.Q4_0, 2, 33, np.zeros(40, np.uint8))


# ---------------------------------------------------------------------------
# Sampler (sampler.rs)
# ---------------------------------------------------------------------------
def gpu_sample(ctx, logits, params, seeds, seen=None, steps=1):
    B = logits.shape[0]
    lg = dev(logits)
    rng = torch.tensor([max(int(s), 1) for s in seeds], dtype=torch.uint64, device="cuda")
    out = torch.zeros(B, dtype=torch.int32, device="cuda")
    seen_t = dev(seen) if seen is not None else None
    res = []
    for _ in range(steps):
        hale.sample(ctx, lg, params, rng, out, seen_t)
        res.append(out.cpu().numpy().copy())
    return np.stack(res, 1)


def test_greedy_sampling_matches_argmax(ctx):
    """sampler.rs:152-156 plus ties (first max wins) and a NaN at index 0."""
    V = 151936
    rng = np.random.default_rng(2)
    lg = rng.standard_normal((4, V)).astype(np.float32)
    lg[1, 100] = lg[1, 99000] = 50.0      # tie -> lower index
    lg[2, 0] = np.nan                     # the reference's scan keeps index 0
    lg[3, :] = -np.inf
    p = hale.SamplingParams(0.0, 1.0, 0, 1.0)
    got = gpu_sample(ctx, lg, p, [1, 1, 1, 1])[:, 0]
    want = [O.argmax(r) for r in lg]
    assert list(got) == want


@pytest.mark.parametrize("T,top_p,top_k,V", [(0.7, 0.9, 40, 151936), (0.7, 0.8, 20, 151936),
                                             (1.0, 0.9, 0, 5), (1.3, 0.95, 1000, 32000),
                                             (0.5, 1.0, 64, 1024)])
def test_top_k_top_p_stream_matches_the_oracle(ctx, T, top_p, top_k, V):
    """TopPSampler::sample (sampler.rs:80-123): same seed, same tokens."""
    rng = np.random.default_rng(int(T * 100) + V + top_k)
    B, steps = 3, 40
    lg = (rng.standard_normal((B, V)) * 3).astype(np.float32)
    if V == 5:
        lg = np.tile(np.float32([10.0, 9.5, 0.0, -5.0, -5.0]), (B, 1))
    p = hale.SamplingParams(T, top_p, top_k, 1.0)
    seeds = [7, 123456789, 42]
    got = gpu_sample(ctx, lg, p, seeds, steps=steps)
    for b in range(B):
        s = O.Sampler(temperature=T, top_p=top_p, top_k=top_k, seed=seeds[b])
        want = [s.sample(lg[b]) for _ in range(steps)]
        assert list(got[b]) == want, b


def test_top_k_one_is_greedy_on_gpu(ctx):
    """sampler.rs:186-198"""
    lg = np.tile(np.float32([0.0, 0.1, 0.05]), (2, 1))
    got = gpu_sample(ctx, lg, hale.SamplingParams(2.0, 1.0, 1, 1.0), [3, 4], steps=20)
    assert (got == 1).all()


def test_repetition_penalty_matches_the_oracle(ctx):
    """Extension (config 5: T=0.7, top-k 20, top-p 0.8, penalty 1.1)."""
    V, B, steps = 151936, 2, 30
    rng = np.random.default_rng(9)
    lg = (rng.standard_normal((B, V)) * 2).astype(np.float32)
    top = np.argsort(-lg, axis=1)[:, :30].astype(np.int32)
    seen = np.concatenate([top[:, ::2], np.full((B, 3), -1, np.int32)], axis=1)
    p = hale.SamplingParams(0.7, 0.8, 20, 1.1)
    got = gpu_sample(ctx, lg, p, [11, 12], seen=seen, steps=steps)
    for b in range(B):
        s = O.Sampler(temperature=0.7, top_p=0.8, top_k=20, seed=[11, 12][b])
        want = [s.sample(lg[b], seen=seen[b], repetition_penalty=1.1) for _ in range(steps)]
        assert list(got[b]) == want


@pytest.mark.parametrize("T,top_p,top_k,scale,steps", [(0.7, 0.9, 0, 3.0, 6), (1.0, 0.95, 0, 1.0, 3),
                                                         (0.7, 0.8, 5000, 3.0, 6), (0.9, 1.0, 0, 8.0, 4)])
def test_full_vocabulary_stream_matches_the_oracle(ctx, T, top_p, top_k, scale, steps):
    """top_k = 0 keeps every candidate (sampler.rs:84-93: the whole
    vocabulary sorted), and top_k above 1024 keeps thousands: the seeded
    streams equal the oracle's at V = 151936, for a peaked (scale 8) and a
    flat (scale 1) logit row and with no nucleus cut (top_p 1)."""
    V, B = 151936, 2
    rng = np.random.default_rng(int(T * 10) + top_k + int(scale))
    lg = (rng.standard_normal((B, V)) * scale).astype(np.float32)
    lg[0, 100] = lg[0, 90000] = float(lg[0].max())   # a tie at the top: lower index first
    p = hale.SamplingParams(T, top_p, top_k, 1.0)
    seeds = [5, 987654321]
    got = gpu_sample(ctx, lg, p, seeds, steps=steps)
    for b in range(B):
        s = O.Sampler(temperature=T, top_p=top_p, top_k=top_k, seed=seeds[b])
        want = [s.sample(lg[b]) for _ in range(steps)]
        assert list(got[b]) == want, b


def test_full_vocabulary_with_repetition_penalty(ctx):
    V, B, steps = 32000, 3, 5
    rng = np.random.default_rng(17)
    lg = (rng.standard_normal((B, V)) * 2).astype(np.float32)
    seen = np.argsort(-lg, axis=1)[:, :50].astype(np.int32)
    p = hale.SamplingParams(0.8, 0.9, 0, 1.1)
    got = gpu_sample(ctx, lg, p, [1, 2, 3], seen=seen, steps=steps)
    for b in range(B):
        s = O.Sampler(temperature=0.8, top_p=0.9, top_k=0, seed=[1, 2, 3][b])
        want = [s.sample(lg[b], seen=seen[b], repetition_penalty=1.1) for _ in range(steps)]
        assert list(got[b]) == want


def test_kernels_were_launched_from_this_library(ctx):
    assert ctx.launches > 0
