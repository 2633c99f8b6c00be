"""GPU parity of the expert-kernel families.

Contexts here force a family at every batch size the shapes allow: "ws" the
warp-specialised streaming kernels (TMA tensor loads, warp MMA), "tc" the
tcgen05 kind::i8 kernels, "ps" the persistent streaming warp-MMA kernels,
"dp4a" the per-CTA kernels. Each must equal the oracle (MoeLayer::forward,
src/moe.rs:56-70, with dot_q4_0 / dot_q8_0 of src/tensor/quant.rs:115-144)
bit for bit, and the per-CTA kernels on whole batches too large for the
oracle to check every token.
"""
import importlib

import numpy as np
import pytest

from oracle import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

hale = importlib.import_module("hale-token_b200")
fmt = importlib.import_module("hale-token_b200.formats")


FAMILIES = ["ws", "tc", "ps"]


@pytest.fixture(scope="module")
def ctxs():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    cs = {name: hale.Context(0, expert_kernel=name) for name in FAMILIES + ["dp4a"]}
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


def oracle_experts(ld):
    return [O.ExpertWeights(ld.dtype, ld.H, ld.I, *ld.expert_encoded(e)) for e in range(ld.E)]


def forward(ctx, pool, ld, x, k):
    renc = fmt.encode(fmt.F32, ld.router)
    layer = hale.moe_layer(0, dev(renc), fmt.F32, ld.E, k, True)
    m = x.shape[0]
    out = torch.full((m, ld.H), float("nan"), dtype=torch.float32, device="cuda")
    idx = torch.zeros((m, k), dtype=torch.int32, device="cuda")
    w = torch.zeros((m, k), dtype=torch.float32, device="cuda")
    hale.moe_forward(ctx, pool, layer, dev(x), out, idx, w)
    ctx.check()
    return out.cpu().numpy(), idx.cpu().numpy(), renc


@pytest.mark.parametrize("family", FAMILIES)
@pytest.mark.parametrize("dtype", [fmt.Q4_0, fmt.Q8_0])
@pytest.mark.parametrize("m", [1, 3, 16, 40, 64, 100])
def test_tiny_layer_matches_oracle(ctxs, family, dtype, m):
    """16 experts top-4, H=256, I=128: one to several passes per expert (for
    tc both pass widths: 8 tokens below M*k = 16*E, 16 from there)."""
    tc = ctxs[family]
    ld = fmt.SyntheticLayer(300 + m, 16, 256, 128, dtype)
    pool = make_pool(tc, ld)
    x = ld.tokens(m)
    out, idx, renc = forward(tc, pool, ld, x, 4)
    want, widx, _ = O.moe_forward(fmt.F32, renc, oracle_experts(ld), 4, True, x)
    assert np.array_equal(idx, widx.astype(np.int32))
    assert_bit_equal(out, want, "layer output")


@pytest.mark.parametrize("family", FAMILIES)
@pytest.mark.parametrize("m", [8, 64, 512])
def test_qwen3_shape_matches_oracle_and_dp4a(ctxs, family, m):
    """H=2048, 128 experts top-8, I=768, q4_0: every token against the
    oracle and against the per-CTA kernels."""
    tc, dp = ctxs[family], ctxs["dp4a"]
    ld = fmt.SyntheticLayer(11, 128, 2048, 768, fmt.Q4_0)
    x = ld.tokens(m)
    out_tc, idx, renc = forward(tc, make_pool(tc, ld), ld, x, 8)
    out_dp, idx_dp, _ = forward(dp, make_pool(dp, ld), ld, x, 8)
    assert np.array_equal(idx, idx_dp)
    assert_bit_equal(out_tc, out_dp, "tc vs dp4a")
    want, _, _ = O.moe_forward(fmt.F32, renc, oracle_experts(ld), 8, True, x, native=True)
    assert_bit_equal(out_tc, want, "every token")


@pytest.mark.parametrize("family", FAMILIES)
def test_q8_wide_hidden_with_shallow_ring(ctxs, family):
    """q8_0, H=4096 (Mixtral hidden size): the activation stage takes much of
    shared memory, leaving the weight ring a shallow depth."""
    tc, dp = ctxs[family], ctxs["dp4a"]
    ld = fmt.SyntheticLayer(23, 8, 4096, 1024, fmt.Q8_0)
    x = ld.tokens(24)
    out_tc, idx, renc = forward(tc, make_pool(tc, ld), ld, x, 2)
    out_dp, _, _ = forward(dp, make_pool(dp, ld), ld, x, 2)
    assert_bit_equal(out_tc, out_dp, "tc vs dp4a")
    want, _, _ = O.moe_forward(fmt.F32, renc, oracle_experts(ld), 2, True, x[:4])
    assert_bit_equal(out_tc[:4], want, "first tokens")


@pytest.mark.parametrize("family", FAMILIES)
def test_repeated_calls_are_deterministic(ctxs, family):
    """The persistent kernels reset their combine counters: two calls in a row
    give identical bits."""
    tc = ctxs[family]
    ld = fmt.SyntheticLayer(5, 32, 512, 256, fmt.Q4_0)
    pool = make_pool(tc, ld)
    x = ld.tokens(200)
    a = forward(tc, pool, ld, x, 4)[0]
    b = forward(tc, pool, ld, x, 4)[0]
    assert_bit_equal(a, b, "second call")


@pytest.mark.parametrize("family", FAMILIES)
def test_q4_wide_hidden_takes_short_stages(ctxs, family):
    """q4_0, H=4096 (Qwen3-235B hidden size): the streaming kernels fall back
    to 4-block stages to fit two CTAs per SM; every token against the
    oracle."""
    tc, dp = ctxs[family], ctxs["dp4a"]
    ld = fmt.SyntheticLayer(29, 16, 4096, 512, fmt.Q4_0)
    x = ld.tokens(40)
    out_tc, idx, renc = forward(tc, make_pool(tc, ld), ld, x, 8)
    out_dp, _, _ = forward(dp, make_pool(dp, ld), ld, x, 8)
    assert_bit_equal(out_tc, out_dp, "family vs dp4a")
    want, _, _ = O.moe_forward(fmt.F32, renc, oracle_experts(ld), 8, True, x, native=True)
    assert_bit_equal(out_tc, want, "every token")
