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
