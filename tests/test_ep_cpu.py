"""Expert-parallel layer protocol on CPU ranks (gloo).

The orchestration of hale-token_b200/ep.py (count exchange, three
all-to-all-v of the route records, the y rows back, best-first combine) runs
on world_size 2 and 4 gloo ranks with a CPU backend built on the oracle:
dispatch packs exactly what hale_ep_dispatch packs, and every owner computes
its experts from the q8 bytes it received (dot_quantized on the wire data,
quant.rs:107-144; silu(g) * u and the q8 of h as Expert::forward,
expert/mod.rs:91-103). The result must equal the single-process oracle
MoeLayer::forward (moe.rs:56-70) bit for bit on every rank.
"""
import datetime
import importlib
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

from oracle import oracle as O

fmt = importlib.import_module("hale-token_b200.formats")

E, H, I, K = 16, 256, 128, 4


def aux_pairs(cols):
    nb = cols // 32
    return (nb + 1) & ~1


class OracleEpBackend:
    """dispatch / experts / combine of one rank, on the CPU oracle."""

    def __init__(self, ld, rank, world):
        import torch
        self.torch = torch
        self.ld, self.rank, self.world = ld, rank, world
        self.epr = E // world
        self.renc = fmt.encode(fmt.F32, ld.router)
        self.enc = {e: ld.expert_encoded(e) for e in range(rank * self.epr, (rank + 1) * self.epr)}

    def dispatch(self, x):
        x = x.numpy()
        m = x.shape[0]
        nb, pairs = H // 32, aux_pairs(H)
        xs, xq = O.quantize_q8(x)
        routes = []
        for t in range(m):
            idx, w = O.moe_route(fmt.F32, self.renc, E, K, True, x[t])
            for s in range(K):
                routes.append((int(idx[s]), t * K + s, t, s, np.float32(w[s])))
        routes.sort(key=lambda r: (r[0], r[1]))  # experts ascending, then route id: owner ranks grouped
        n = len(routes)
        q = np.zeros((n, H), np.int8)
        aux = np.zeros((n, 2 * pairs), np.int32)
        meta = np.zeros((n, 4), np.int32)
        for j, (e, _, t, s, w) in enumerate(routes):
            q[j] = xq[t]
            aux[j, 0:2 * nb:2] = xs[t].view(np.int32)
            aux[j, 1:2 * nb:2] = -8 * xq[t].astype(np.int32).reshape(nb, 32).sum(1)
            meta[j] = (t, s, e, np.array([w], np.float32).view(np.int32)[0])
        counts = [sum(1 for r in routes if r[0] // self.epr == o) for o in range(self.world)]
        t_ = self.torch.from_numpy
        return counts, (t_(q), t_(aux), t_(meta))

    def experts(self, q, aux, meta):
        q, aux, meta = q.numpy(), aux.numpy(), meta.numpy()
        nb_h, nb_i = H // 32, I // 32
        y = np.zeros((q.shape[0], H), np.float32)
        for j in range(q.shape[0]):
            e = int(meta[j, 2])
            assert e // self.epr == self.rank, "record routed to the wrong owner"
            g_enc, u_enc, d_enc = self.enc[e]
            xs = np.ascontiguousarray(aux[j, 0:2 * nb_h:2]).view(np.float32)
            g = np.array([O.dot_quantized(self.ld.dtype, g_enc[r], xs, q[j]) for r in range(I)], np.float32)
            u = np.array([O.dot_quantized(self.ld.dtype, u_enc[r], xs, q[j]) for r in range(I)], np.float32)
            h = np.array([np.float32(O.silu(g[r])) * u[r] for r in range(I)], np.float32)
            hs, hq = O.quantize_q8(h)
            assert hs.shape[0] == nb_i
            y[j] = [O.dot_quantized(self.ld.dtype, d_enc[c], hs, hq) for c in range(H)]
        return self.torch.from_numpy(y)

    def combine(self, meta, y_back, m_tokens):
        meta, y_back = meta.numpy(), y_back.numpy()
        pos = {(int(meta[j, 0]), int(meta[j, 1])): j for j in range(meta.shape[0])}
        out = np.zeros((m_tokens, H), np.float32)
        for t in range(m_tokens):
            for s in range(K):
                j = pos[(t, s)]
                w = np.array([meta[j, 3]], np.int32).view(np.float32)[0]
                out[t] = out[t] + w * y_back[j]
        return self.torch.from_numpy(out)


def _rank_main(rank, world, port, m_tokens, results):
    import torch.distributed as dist
    ep = importlib.import_module("hale-token_b200.ep")
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        ld = fmt.SyntheticLayer(77, E, H, I, fmt.Q4_0)
        x = ld.tokens(m_tokens, seed=500 + rank)
        import torch
        out = ep.moe_forward_ep(OracleEpBackend(ld, rank, world), ep.Exchange(device="cpu"), torch.from_numpy(x))
        experts = [O.ExpertWeights(ld.dtype, H, I, *ld.expert_encoded(e)) for e in range(E)]
        want = O.moe_forward(fmt.F32, fmt.encode(fmt.F32, ld.router), experts, K, True, x)[0]
        got = out.numpy()
        results.put((rank, bool(np.array_equal(got.view(np.uint32), want.view(np.uint32))),
                     int((got.view(np.uint32) != want.view(np.uint32)).sum())))
    except Exception as exc:  # reported to the parent, which fails the test
        results.put((rank, False, repr(exc)))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world,m_tokens", [(2, 5), (4, 3)])
def test_ep_protocol_on_gloo_ranks_is_bit_exact(world, m_tokens):
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, m_tokens, results)) for r in range(world)]
    for p in procs:
        p.start()
    got = [results.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, info in sorted(got, key=lambda t: t[0]):
        assert ok, f"rank {rank}: {info}"
