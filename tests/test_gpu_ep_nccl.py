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


def _rank_main(rank, world, port, uid, uid2, uid3, results):
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
        # whole-model decode with expert-parallel MoE layers: this rank's own
        # sequence; its logits equal the one-GPU decoder's at every position
        import sys
        sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
        import synth
        from oracle import model as OM
        from test_gpu_decoder import build_decoder
        cases = ((fmt.Q8_0, uid2, (0, 3, 256, 8, 2, 32, 16, 4, 128, 512)),   # config-0 form: 16 experts top-4
                 (fmt.Q4_0, uid3, (3, 2, 512, 8, 2, 64, 8, 2, 256, 320)))    # Mixtral form: 8 experts top-2
        for qt, duid, shape in cases:
            seed, L, Hh, nh, nkv, hd, E2, k2, I2, V2 = shape
            hf, tt, enc = synth.qwen3_moe(seed, L, Hh, nh, nkv, hd, E2, k2, I2, V2, qt, "F32")
            om = OM.OracleModel(expert_dtype=qt, hf_config=hf, tensors=tt, expert_encoded=enc)
            e_r = E2 // world
            toks = np.random.default_rng(40 + rank).integers(0, V2, 9).tolist()
            full_dec = build_decoder(ctx, om, qt, len(toks) + 1, max_batch=4)
            ep_dec = build_decoder(ctx, om, qt, len(toks) + 1, max_batch=4,
                                   experts=range(rank * e_r, (rank + 1) * e_r))
            dcomm = hale.Comm(ctx, world, rank, duid, Hh, E2, k2, 4)
            try:
                ep_dec.set_comm(dcomm)
                got, want = [], []
                lg = torch.empty((4, V2), dtype=torch.float32, device="cuda")
                lw = torch.empty((4, V2), dtype=torch.float32, device="cuda")
                ep_dec.step(toks[:4], list(range(4)), logits=lg)
                full_dec.step(toks[:4], list(range(4)), logits=lw)
                got.append(lg.cpu().numpy().copy())
                want.append(lw.cpu().numpy().copy())
                for i in range(4, len(toks)):
                    ep_dec.step([toks[i]], [i], logits=lg[:1])
                    full_dec.step([toks[i]], [i], logits=lw[:1])
                    got.append(lg[:1].cpu().numpy().copy())
                    want.append(lw[:1].cpu().numpy().copy())
                # a step in which rank 0 has no rows: it still joins every
                # MoE layer's exchange, so the others' tokens reach its experts
                if rank == 0:
                    ep_dec.step([], [])
                else:
                    ep_dec.step([toks[0]], [len(toks)], logits=lg[:1])
                    full_dec.step([toks[0]], [len(toks)], logits=lw[:1])
                    got.append(lg[:1].cpu().numpy().copy())
                    want.append(lw[:1].cpu().numpy().copy())
                ctx.check()
                diff = int((np.concatenate(got).view(np.uint32) != np.concatenate(want).view(np.uint32)).sum())
                results.put((rank, 200 + qt, diff))
            finally:
                ep_dec.set_comm(None)
                dcomm.close()
                ep_dec.close()
                full_dec.close()
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
    hl = importlib.import_module("hale-token_b200")
    uid, uid2, uid3 = hl.comm_unique_id(), hl.comm_unique_id(), hl.comm_unique_id()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, uid, uid2, uid3, results)) for r in range(world)]
    for p in procs:
        p.start()
    got = []
    try:
        for _ in range(world * 9):
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
    assert len(got) == world * 9
