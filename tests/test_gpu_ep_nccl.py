"""Expert parallelism on several GPUs (skipped below 2 GPUs).

One process per GPU; rank r holds only experts [r*E/R, (r+1)*E/R) of the
layer and its own tokens. Two paths move the records and y rows:
hale_moe_forward_ep (one C call per layer: stores into peer memory over
NVLink, flags, no host synchronisation) and hale-token_b200/ep.py's NCCL
all-to-all-v around the hale_ep_* device halves. Each rank's output must
equal hale_moe_forward with the full expert pool on its own GPU bit for bit
(moe.rs:56-70).
"""
import datetime
import importlib
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _rank_main(rank, world, port, uid, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch
    import torch.distributed as dist
    hale = importlib.import_module("hale-token_b200")
    fmt = importlib.import_module("hale-token_b200.formats")
    ep = importlib.import_module("hale-token_b200.ep")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        ctx = hale.Context(rank)
        ld = fmt.SyntheticLayer(71, 128, 2048, 768, fmt.Q4_0)
        epr = 128 // world
        router = torch.from_numpy(fmt.encode(fmt.F32, ld.router)).cuda()
        layer = hale.moe_layer(0, router, fmt.F32, 128, 8, True)
        local = hale.Pool(ctx, fmt.Q4_0, 2048, 768, 1, epr)
        for le in range(epr):
            local.upload(0, le, fmt.pack_record(*ld.expert_encoded(rank * epr + le)))
        full = hale.Pool(ctx, fmt.Q4_0, 2048, 768, 1, 128)
        for e in range(128):
            full.upload(0, e, fmt.pack_record(*ld.expert_encoded(e)))
        backend = ep.CudaEpBackend(ctx, local, layer, 2048, rank, world)
        exch = ep.Exchange(device=f"cuda:{rank}")
        for m in (64, 1, 37):
            x = torch.from_numpy(ld.tokens(m, seed=2000 + 10 * rank + m)).cuda()
            out = ep.moe_forward_ep(backend, exch, x)
            torch.cuda.synchronize()
            want = torch.full((m, 2048), float("nan"), device="cuda")
            hale.moe_forward(ctx, full, layer, x, want)
            ctx.check()
            diff = int((out.cpu().numpy().view(np.uint32) != want.cpu().numpy().view(np.uint32)).sum())
            results.put((rank, m, diff))
        dist.barrier()
        # the one-call path: ranks bring different token counts, 0 included
        comm = hale.Comm(ctx, world, rank, uid, 2048, 128, 8, 64)
        try:
            for step in range(4):
                m = (64, 1, 0, 37)[(step + rank) % 4]
                x = torch.from_numpy(ld.tokens(max(m, 1), seed=3000 + 10 * rank + step)).cuda()[:m]
                out = torch.full((m, 2048), float("nan"), device="cuda")
                hale.moe_forward_ep(ctx, comm, local, layer, x, out)
                want = torch.full((m, 2048), float("nan"), device="cuda")
                if m:
                    hale.moe_forward(ctx, full, layer, x, want)
                ctx.check()
                diff = int((out.cpu().numpy().view(np.uint32) != want.cpu().numpy().view(np.uint32)).sum())
                results.put((rank, 100 + step, diff))
        finally:
            comm.close()
    except Exception as exc:
        results.put((rank, -1, repr(exc)))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_ep_over_nccl_matches_single_gpu():
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    if n < 2:
        pytest.skip("needs 2 or more GPUs")
    world = 2 if n < 4 else (4 if n < 8 else 8)
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    uid = importlib.import_module("hale-token_b200").comm_unique_id()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, uid, results)) for r in range(world)]
    for p in procs:
        p.start()
    got = []
    try:
        for _ in range(world * 7):
            got.append(results.get(timeout=240))
            if got[-1][1] == -1:
                break
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for rank, m, info in got:
        assert m != -1, f"rank {rank} failed: {info}"
        assert info == 0, f"rank {rank}, {m} tokens: {info} values differ from the 1-GPU layer"
    assert len(got) == world * 7
