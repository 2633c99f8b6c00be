"""GPU parity of the one-launch MoE layer for a single token.

At one token an "auto" context runs the whole layer (router logits, softmax
and top-k, the chosen experts' gate/up and down, the best-first combine) as
one launch (moe_token_kernel). Its output, top-k indices and weights must
equal the oracle (MoeLayer::forward, src/moe.rs:56-70) bit for bit, and the
three-launch path of a "dp4a" context, over router dtypes, top-k
normalisation, expert formats and shapes that take the kernel's different
work splits (several router rows per CTA, several gate/up or down units per
CTA, whole-record prefetch).
"""
import importlib

import numpy as np
import pytest

from oracle import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

hale = importlib.import_module("hale-token_b200")
fmt = importlib.import_module("hale-token_b200.formats")


@pytest.fixture(scope="module")
def ctxs():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    cs = {"auto": hale.Context(0), "dp4a": hale.Context(0, expert_kernel="dp4a")}
    yield cs
    for c in cs.values():
        c.check()
        c.close()


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def assert_bit_equal(got, want, what=""):
    got, want = np.ascontiguousarray(got), np.ascontiguousarray(want)
    assert got.shape == want.shape, (what, got.shape, want.shape)
    eq = got.view(np.uint32) == want.view(np.uint32)
    if not eq.all():
        i = tuple(np.argwhere(~eq)[0])
        raise AssertionError(f"{what}: {(~eq).sum()} of {eq.size} differ; first at {i}: got {got[i]!r} want {want[i]!r}")


def make_pool(ctx, ld):
    pool = hale.Pool(ctx, ld.dtype, ld.H, ld.I, 1, ld.E)
    for e in range(ld.E):
        pool.upload(0, e, fmt.pack_record(*ld.expert_encoded(e)))
    return pool


def forward(ctx, pool, ld, renc, rdt, x, k, normalize):
    layer = hale.moe_layer(0, dev(renc), rdt, ld.E, k, normalize)
    m = x.shape[0]
    out = torch.full((m, ld.H), float("nan"), dtype=torch.float32, device="cuda")
    idx = torch.full((m, k), -1, dtype=torch.int32, device="cuda")
    w = torch.full((m, k), float("nan"), dtype=torch.float32, device="cuda")
    hale.moe_forward(ctx, pool, layer, dev(x), out, idx, w)
    ctx.check()
    return out.cpu().numpy(), idx.cpu().numpy(), w.cpu().numpy()


def oracle(ld, renc, rdt, x, k, normalize, chosen):
    """The oracle layer with real weights for the experts the routes name
    (routes are checked against MoeLayer::route separately); the others are
    never read."""
    ph = O.ExpertWeights(ld.dtype, ld.H, ld.I, *ld.expert_encoded(int(chosen[0])))
    ex = [O.ExpertWeights(ld.dtype, ld.H, ld.I, *ld.expert_encoded(e)) if e in set(chosen.tolist()) else ph
          for e in range(ld.E)]
    return O.moe_forward(rdt, renc, ex, k, normalize, x, native=True)


def check(ctxs, ld, rdt, k, normalize, seed=0):
    renc = fmt.encode(rdt, ld.router)
    x = ld.tokens(1, seed=seed)
    pa = make_pool(ctxs["auto"], ld)
    launches0 = ctxs["auto"].launches
    out, idx, w = forward(ctxs["auto"], pa, ld, renc, rdt, x, k, normalize)
    assert ctxs["auto"].launches - launches0 == 1, "one launch for the single-token layer"
    ridx, rw = O.moe_route(rdt, renc, ld.E, k, normalize, x[0])
    assert np.array_equal(idx[0], ridx.astype(np.int32)), (idx, ridx)
    assert_bit_equal(w[0], rw, "top-k weights")
    want, widx, ww = oracle(ld, renc, rdt, x, k, normalize, ridx)
    assert np.array_equal(idx, widx.astype(np.int32))
    assert_bit_equal(out, want, "layer output vs oracle")
    out_dp, idx_dp, w_dp = forward(ctxs["dp4a"], make_pool(ctxs["dp4a"], ld), ld, renc, rdt, x, k, normalize)
    assert np.array_equal(idx, idx_dp)
    assert_bit_equal(w, w_dp, "weights vs three-launch path")
    assert_bit_equal(out, out_dp, "output vs three-launch path")
    # routing counts of the resident pool: one route per chosen expert
    counts = pa.routing_counts()
    want_counts = np.zeros(ld.E, np.uint64)
    want_counts[idx[0]] = 1
    assert np.array_equal(counts[0], want_counts)
    return out


@pytest.mark.parametrize("dtype", [fmt.Q4_0, fmt.Q8_0])
@pytest.mark.parametrize("rdt", [fmt.F32, fmt.BF16, fmt.F16])
@pytest.mark.parametrize("normalize", [True, False])
def test_tiny_layer(ctxs, dtype, rdt, normalize):
    """16 experts top-4, H=256, I=128: a 32-CTA grid."""
    ld = fmt.SyntheticLayer(71, 16, 256, 128, dtype)
    check(ctxs, ld, rdt, 4, normalize)


@pytest.mark.parametrize("dtype", [fmt.Q4_0, fmt.Q8_0])
@pytest.mark.parametrize("seed", [0, 1, 2])
def test_qwen3_shape(ctxs, dtype, seed):
    """BASELINE config-1 layer (H=2048, 128 experts top-8, I=768): the
    decode-time case, one gate/up and one down unit per CTA."""
    ld = fmt.SyntheticLayer(11, 128, 2048, 768, dtype)
    check(ctxs, ld, fmt.F32, 8, True, seed=seed)


def test_top1_and_top_k_32(ctxs):
    """k = 1 (no combine beyond one slot) and k = 32 (the largest the
    router supports: 256 chain threads in the down phase)."""
    ld = fmt.SyntheticLayer(13, 64, 512, 256, fmt.Q4_0)
    check(ctxs, ld, fmt.F32, 1, True)
    check(ctxs, ld, fmt.F32, 32, False)


def test_more_experts_than_ctas(ctxs):
    """256 experts, q8_0 at H=4096: shared memory allows one CTA per SM, so
    each CTA chains the logits of two router rows."""
    ld = fmt.SyntheticLayer(17, 256, 4096, 256, fmt.Q8_0)
    check(ctxs, ld, fmt.BF16, 8, True)


def test_mixtral_shape_several_down_units(ctxs):
    """8 experts top-2, H=4096 (Mixtral hidden size), I=1024: 512 down units
    over fewer CTAs."""
    ld = fmt.SyntheticLayer(19, 8, 4096, 1024, fmt.Q4_0)
    check(ctxs, ld, fmt.F32, 2, True)


def test_wide_intermediate_prefetches_whole_records(ctxs):
    """I=8192 with 2 of 8 experts: more gate/up units than CTAs, so every
    CTA takes several and the L2 prefetch covers whole expert records."""
    ld = fmt.SyntheticLayer(23, 8, 1024, 8192, fmt.Q4_0)
    check(ctxs, ld, fmt.F32, 2, True)


def test_repeated_calls_reset_the_grid_barrier(ctxs):
    """The last CTA resets the barrier counters: many calls in a row, and
    calls alternating with batched calls, give identical bits."""
    ctx = ctxs["auto"]
    ld = fmt.SyntheticLayer(5, 32, 512, 256, fmt.Q4_0)
    renc = fmt.encode(fmt.F32, ld.router)
    pool = make_pool(ctx, ld)
    x = ld.tokens(1)
    first = forward(ctx, pool, ld, renc, fmt.F32, x, 4, True)[0]
    for i in range(20):
        if i % 5 == 4:
            forward(ctx, pool, ld, renc, fmt.F32, ld.tokens(9), 4, True)
        assert_bit_equal(forward(ctx, pool, ld, renc, fmt.F32, x, 4, True)[0], first, f"call {i}")
