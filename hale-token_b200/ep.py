"""Expert-parallel MoE layer: one process per GPU, experts partitioned over ranks.

MoeLayer::forward (src/model/moe.rs:56-70) with the experts of a layer split
into R contiguous blocks of E / R; rank r owns experts [r*E/R, (r+1)*E/R)
(weights in a local hale_pool with local ids 0 .. E/R - 1). Each rank brings
its own tokens (data-parallel attention upstream). One call:

  1. dispatch (home): route the rank's tokens over all E experts, quantize
     each token once, pack one record per route grouped by owner rank;
  2. exchange the per-rank record counts, then the records (all-to-all-v);
  3. experts (owner): run the local experts on the received records;
  4. send the y rows back along the reverse splits (all-to-all-v);
  5. combine (home): best-first weighted sum per token.

Bit-identical to the 1-GPU layer: q8 activations are a pure function of x,
each expert computes each record independently, and the combine keeps the
reference's route order.

The exchange uses torch.distributed (NCCL with CUDA tensors, gloo with CPU
tensors); the device work goes through a backend object with dispatch /
experts / combine methods -- CudaEpBackend here (the C ABI's hale_ep_*).
"""
import importlib

import torch
import torch.distributed as dist

hale = importlib.import_module("hale-token_b200")


class Exchange:
    """All-to-all-v of row blocks within a process group."""

    def __init__(self, group=None, device="cpu"):
        self.group = group
        self.device = torch.device(device)
        self.world = dist.get_world_size(group)

    def counts(self, send_counts):
        """Each rank's send counts to every rank -> what this rank receives from each."""
        s = torch.tensor(send_counts, dtype=torch.int64, device=self.device)
        r = torch.empty_like(s)
        dist.all_to_all_single(r, s, group=self.group)
        return [int(v) for v in r.tolist()]

    def rows(self, send, send_counts, recv_counts):
        """Rows of `send` (split by send_counts along dim 0) to their ranks;
        returns the rows received, source rank ascending."""
        out = torch.empty((sum(recv_counts),) + tuple(send.shape[1:]), dtype=send.dtype, device=send.device)
        # gloo exchanges bytes most portably; NCCL takes any dtype
        if send.device.type == "cpu":
            s8 = send.contiguous().view(torch.uint8).reshape(send.shape[0], -1)
            o8 = out.view(torch.uint8).reshape(out.shape[0], -1)
            dist.all_to_all_single(o8, s8, recv_counts, send_counts, group=self.group)
        else:
            dist.all_to_all_single(out, send.contiguous(), recv_counts, send_counts, group=self.group)
        return out


def moe_forward_ep(backend, exchange, x):
    """One expert-parallel layer call for this rank's tokens x [M, H]. Returns
    out [M, H] (on the backend's device)."""
    counts, (q, aux, meta) = backend.dispatch(x)
    recv_counts = exchange.counts(counts)
    rq = exchange.rows(q, counts, recv_counts)
    ra = exchange.rows(aux, counts, recv_counts)
    rm = exchange.rows(meta, counts, recv_counts)
    y = backend.experts(rq, ra, rm)
    y_back = exchange.rows(y, recv_counts, counts)
    return backend.combine(meta, y_back, x.shape[0])


class CudaEpBackend:
    """The C ABI's hale_ep_* calls for one rank.

    ctx: this rank's hale Context; pool: its local experts (E/R per layer);
    layer: the hale_moe_layer (router replicated on every rank) with
    `layer.layer` the pool layer; rank, n_ranks: this rank's place.
    """

    def __init__(self, ctx, pool, layer, hidden, rank, n_ranks, stream=None):
        self.ctx, self.pool, self.layer = ctx, pool, layer
        self.hidden, self.rank, self.n_ranks = hidden, rank, n_ranks
        self.k = layer.top_k
        self.epr = layer.n_experts // n_ranks
        self.pairs = hale.q8_aux_pairs(hidden)
        self.stream = stream

    def dispatch(self, x):
        m = x.shape[0]
        n = m * self.k
        dev = x.device
        q = torch.empty((n, self.hidden), dtype=torch.int8, device=dev)
        aux = torch.empty((n, 2 * self.pairs), dtype=torch.int32, device=dev)
        meta = torch.empty((n, 4), dtype=torch.int32, device=dev)
        counts = hale.ep_dispatch(self.ctx, self.layer, self.hidden, x, self.n_ranks, q, aux, meta,
                                  stream=self.stream)
        return counts, (q, aux, meta)

    def experts(self, q, aux, meta):
        y = torch.empty((q.shape[0], self.hidden), dtype=torch.float32, device=q.device)
        if q.shape[0]:
            hale.ep_experts(self.ctx, self.pool, self.layer.layer, self.rank * self.epr, q, aux, meta, y,
                            stream=self.stream)
        return y

    def combine(self, meta, y_back, m_tokens):
        out = torch.empty((m_tokens, self.hidden), dtype=torch.float32, device=y_back.device)
        hale.ep_combine(self.ctx, meta, y_back, m_tokens, self.k, self.hidden, out, stream=self.stream)
        return out
