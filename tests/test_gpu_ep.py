"""Expert parallelism through the C ABI on one GPU, ranks emulated in-process.

For R ranks, every "home" rank's tokens go through hale_ep_dispatch; the
records are moved between the emulated ranks exactly as the all-to-all-v of
hale-token_b200/ep.py moves them (segments by the dispatch counts, source
rank ascending); each owner runs hale_ep_experts with a pool holding only its
E/R experts; the y rows go back along the reverse splits and
hale_ep_combine sums them. Every rank's output must equal hale_moe_forward
over the full pool (itself pinned to the oracle, moe.rs:56-70) bit for bit.
"""
import importlib

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

hale = importlib.import_module("hale-token_b200")
fmt = importlib.import_module("hale-token_b200.formats")


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    c = hale.Context(0)
    yield c
    c.check()
    c.close()


def pool_of(ctx, ld, experts):
    p = hale.Pool(ctx, ld.dtype, ld.H, ld.I, 1, len(experts))
    for local, e in enumerate(experts):
        p.upload(0, local, fmt.pack_record(*ld.expert_encoded(e)))
    return p


def split(t, counts):
    out, o = [], 0
    for c in counts:
        out.append(t[o:o + c])
        o += c
    return out


def run_emulated(ctx, ld, k, R, m_tokens, seed):
    ep = importlib.import_module("hale-token_b200.ep")
    router = torch.from_numpy(fmt.encode(fmt.F32, ld.router)).cuda()
    layer = hale.moe_layer(0, router, fmt.F32, ld.E, k, True)
    epr = ld.E // R
    pools = [pool_of(ctx, ld, range(o * epr, (o + 1) * epr)) for o in range(R)]
    backends = [ep.CudaEpBackend(ctx, pools[o], layer, ld.H, o, R) for o in range(R)]
    xs = [torch.from_numpy(ld.tokens(m_tokens, seed=seed + r)).cuda() for r in range(R)]
    sent = [backends[r].dispatch(xs[r]) for r in range(R)]            # (counts, (q, aux, meta))
    ys = []
    for o in range(R):
        parts = [[split(buf, sent[r][0])[o] for buf in sent[r][1]] for r in range(R)]
        rq, ra, rm = (torch.cat([p[i] for p in parts]) for i in range(3))
        ys.append((backends[o].experts(rq, ra, rm), [sent[r][0][o] for r in range(R)]))
    outs = []
    for r in range(R):
        y_back = torch.cat([split(ys[o][0], ys[o][1])[r] for o in range(R)])
        outs.append(backends[r].combine(sent[r][1][2], y_back, m_tokens))
    ctx.check()
    full = pool_of(ctx, ld, range(ld.E))
    for r in range(R):
        want = torch.full((m_tokens, ld.H), float("nan"), device="cuda")
        hale.moe_forward(ctx, full, layer, xs[r], want)
        ctx.check()
        got, exp = outs[r].cpu().numpy(), want.cpu().numpy()
        diff = (got.view(np.uint32) != exp.view(np.uint32)).sum()
        assert diff == 0, f"rank {r}: {diff} of {got.size} values differ from the 1-GPU layer"
    return sent


@pytest.mark.parametrize("R", [1, 2, 4])
@pytest.mark.parametrize("dtype", [fmt.Q4_0, fmt.Q8_0])
def test_ep_tiny_layer_matches_single_gpu(ctx, R, dtype):
    run_emulated(ctx, fmt.SyntheticLayer(61, 16, 256, 128, dtype), 4, R, 9, 900)


@pytest.mark.parametrize("R,m", [(2, 64), (8, 64), (8, 1)])
def test_ep_qwen3_shape_matches_single_gpu(ctx, R, m):
    """H=2048, 128 experts top-8, I=768, q4_0; at M=1 most owners get nothing."""
    sent = run_emulated(ctx, fmt.SyntheticLayer(62, 128, 2048, 768, fmt.Q4_0), 8, R, m, 1000)
    assert all(sum(s[0]) == m * 8 for s in sent)


def test_ep_dispatch_rejects_uneven_split(ctx):
    ld = fmt.SyntheticLayer(63, 12, 64, 64, fmt.Q8_0)
    router = torch.from_numpy(fmt.encode(fmt.F32, ld.router)).cuda()
    layer = hale.moe_layer(0, router, fmt.F32, 12, 2, True)
    x = torch.from_numpy(ld.tokens(2)).cuda()
    q = torch.empty((4, 64), dtype=torch.int8, device="cuda")
    aux = torch.empty((4, 2 * hale.q8_aux_pairs(64)), dtype=torch.int32, device="cuda")
    meta = torch.empty((4, 4), dtype=torch.int32, device="cuda")
    with pytest.raises(hale.HaleError) as ei:
        hale.ep_dispatch(ctx, layer, 64, x, 5, q, aux, meta)
    assert ei.value.status == hale.E_INVALID_ARGUMENT


# ---------------------------------------------------------------------------
# hale_moe_forward_ep on one rank: the whole one-call path (records stored
# into the exchange block, gathered, expert kernels writing y rows into the
# y_back half, flags, combine) with this GPU as its own peer.
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("dtype,H,I,E,k", [(fmt.Q4_0, 2048, 768, 128, 8), (fmt.Q8_0, 256, 128, 16, 4),
                                           (fmt.Q4_0, 4096, 512, 16, 8)])
def test_one_call_ep_on_one_rank_matches_the_layer(ctx, dtype, H, I, E, k):
    ld = fmt.SyntheticLayer(91, E, H, I, dtype)
    router = torch.from_numpy(fmt.encode(fmt.F32, ld.router)).cuda()
    layer = hale.moe_layer(0, router, fmt.F32, E, k, True)
    pool = pool_of(ctx, ld, range(E))
    comm = hale.Comm(ctx, 1, 0, None, H, E, k, 64)
    try:
        # calls alternate between the block's halves; 0 tokens is a legal call
        for m in (64, 1, 37, 0, 64, 5):
            x = torch.from_numpy(ld.tokens(max(m, 1), seed=500 + m)).cuda()[:m]
            out = torch.full((m, H), float("nan"), device="cuda")
            idx = torch.zeros((m, k), dtype=torch.int32, device="cuda")
            if m:
                hale.moe_forward_ep(ctx, comm, pool, layer, x, out, idx)
            else:
                hale.moe_forward_ep(ctx, comm, pool, layer, torch.empty((0, H), device="cuda"), out)
            want = torch.full((m, H), float("nan"), device="cuda")
            widx = torch.zeros((m, k), dtype=torch.int32, device="cuda")
            if m:
                hale.moe_forward(ctx, pool, layer, x, want, widx)
            ctx.check()
            assert torch.equal(idx, widx)
            assert np.array_equal(out.cpu().numpy().view(np.uint32), want.cpu().numpy().view(np.uint32)), m
    finally:
        comm.close()


def test_one_call_ep_rejects_mismatched_shapes(ctx):
    ld = fmt.SyntheticLayer(92, 16, 256, 128, fmt.Q8_0)
    router = torch.from_numpy(fmt.encode(fmt.F32, ld.router)).cuda()
    layer = hale.moe_layer(0, router, fmt.F32, 16, 4, True)
    pool = pool_of(ctx, ld, range(16))
    with pytest.raises(hale.HaleError) as ei:
        hale.Comm(ctx, 3, 0, None, 256, 16, 4, 8)          # 16 experts over 3 ranks
    assert ei.value.status == hale.E_INVALID_ARGUMENT
    comm = hale.Comm(ctx, 1, 0, None, 256, 16, 4, 8)
    try:
        x = torch.zeros((9, 256), device="cuda")
        out = torch.empty((9, 256), device="cuda")
        with pytest.raises(hale.HaleError) as ei:
            hale.moe_forward_ep(ctx, comm, pool, layer, x, out)   # more than max_tokens
        assert ei.value.status == hale.E_INVALID_ARGUMENT
        other = hale.moe_layer(0, router, fmt.F32, 16, 2, True)
        with pytest.raises(hale.HaleError) as ei:
            hale.moe_forward_ep(ctx, comm, pool, other, x[:2], out[:2])   # top-2 vs the comm's top-4
        assert ei.value.status == hale.E_INVALID_ARGUMENT
    finally:
        comm.close()
