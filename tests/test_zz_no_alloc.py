"""The allocation-free routing entry point (hale_moe_route_noalloc).

It serves hosts that cannot call cudaMalloc while routing -- a serving loop
replaying captured CUDA graphs, or an embedding whose device memory is one
fixed arena reserved up front. This file is collected last on purpose: a
failure here leaves every other test already run.

Checks, through the C ABI: the result equals hale_moe_route's (bit for bit,
the tolerance every routing test here uses) on two calls in a row; device
free memory does not change across those calls; oversized requests are
rejected.
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
    torch.cuda.set_device(0)
    c = hale.Context(0)
    yield c
    c.close()


@pytest.mark.parametrize("E,k,H,M,rdt", [(128, 8, 2048, 64, fmt.F32), (16, 4, 256, 5, fmt.BF16),
                                         (128, 8, 2048, 1, fmt.F32), (12, 3, 40, 7, fmt.F32)])
def test_noalloc_route_matches_the_allocating_route_twice(ctx, E, k, H, M, rdt):
    rng = np.random.default_rng(E * 7 + M)
    router = torch.from_numpy(fmt.encode(rdt, rng.standard_normal((E, H)).astype(np.float32) * 0.02)).cuda()
    x = torch.from_numpy(rng.standard_normal((M, H)).astype(np.float32)).cuda()
    layer = hale.moe_layer(0, router, rdt, E, k, True)
    want_idx = torch.zeros((M, k), dtype=torch.int32, device="cuda")
    want_w = torch.zeros((M, k), dtype=torch.float32, device="cuda")
    want_p = torch.zeros((M, E), dtype=torch.float32, device="cuda")
    hale.moe_route(ctx, layer, H, x, want_idx, want_w, want_p)
    outs = [(torch.full((M, k), -1, dtype=torch.int32, device="cuda"),
             torch.full((M, k), float("nan"), dtype=torch.float32, device="cuda"),
             torch.full((M, E), float("nan"), dtype=torch.float32, device="cuda")) for _ in range(2)]
    torch.cuda.synchronize()
    # first call sets up the scratch address on this device (outside any capture)
    hale.moe_route_noalloc(router, rdt, E, k, True, H, x, *outs[0])
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    hale.moe_route_noalloc(router, rdt, E, k, True, H, x, *outs[1])
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0, "the no-allocation call changed free device memory"
    for idx, w, p in outs:
        assert torch.equal(idx, want_idx)
        assert torch.equal(w.view(torch.int32), want_w.view(torch.int32))
        assert torch.equal(p.view(torch.int32), want_p.view(torch.int32))


def test_noalloc_route_rejects_requests_beyond_its_scratch(ctx):
    E, k, H, M = 256, 8, 64, 1100
    router = torch.zeros((E, H), dtype=torch.float32, device="cuda")
    x = torch.zeros((M, H), dtype=torch.float32, device="cuda")
    idx = torch.zeros((M, k), dtype=torch.int32, device="cuda")
    w = torch.zeros((M, k), dtype=torch.float32, device="cuda")
    with pytest.raises(hale.HaleError) as ei:
        hale.moe_route_noalloc(router, fmt.F32, E, k, True, H, x, idx, w)
    assert ei.value.status == hale.E_INVALID_ARGUMENT
    assert "scratch" in str(ei.value)
