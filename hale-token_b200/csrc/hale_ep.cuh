// hale_ep.cuh -- device side of expert parallelism for the MoE layer.
//
// Experts of a layer are partitioned over R ranks in contiguous blocks of
// E / R. MoeLayer::forward (src/model/moe.rs:56-70) splits into:
//   home rank : route its tokens (all E experts), quantize each token once --
//               Q8Activations are a pure function of x, so shipping the q8
//               blocks equals the reference re-quantizing x inside each
//               expert -- and pack one record per route, grouped by owner
//               rank (ep_pack_kernel);
//   owner rank: run its experts on the records it receives, grouped here by
//               expert (ep_count_kernel / ep_scatter_kernel), with the
//               ordinary expert kernels at k = 1;
//   home rank : out[t] = sum over the token's routes, best first, of
//               w * y (ep_combine_kernel) -- the 1-GPU combine order, so the
//               result is bit-identical to 1 GPU.
// The host moves the records and the y rows between ranks (all-to-all-v).
#pragma once

#include "hale_kernels.cuh"

namespace hale {

// Record metadata: home token, route slot (best-first rank), global expert,
// routing weight bits.
struct EpMeta {
    int token, slot, expert, wbits;
};

// One warp per record j of the send order (= the expert lists' slot order,
// experts ascending, so records come grouped by owner rank).
__global__ void ep_pack_kernel(const int* __restrict__ elist, const int* __restrict__ topk_idx,
                               const float* __restrict__ topk_w, const int8_t* __restrict__ xq,
                               const int2* __restrict__ xaux, int n, int k, int H, int nbp, int8_t* __restrict__ send_q,
                               int2* __restrict__ send_a, EpMeta* __restrict__ send_meta) {
    const int j = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (j >= n) return;
    const int route = elist[j], tok = route / k;
    const uint4* src = reinterpret_cast<const uint4*>(xq + (size_t)tok * H);
    uint4* dst = reinterpret_cast<uint4*>(send_q + (size_t)j * H);
    for (int i = lane; i < H / 16; i += 32) dst[i] = __ldg(src + i);
    const int2* asrc = xaux + (size_t)tok * nbp;
    int2* adst = send_a + (size_t)j * nbp;
    for (int i = lane; i < nbp; i += 32) adst[i] = __ldg(asrc + i);
    if (lane == 0) {
        EpMeta m;
        m.token = tok;
        m.slot = route - tok * k;
        m.expert = topk_idx[route];
        m.wbits = __float_as_int(topk_w[route]);
        send_meta[j] = m;
    }
}

// counts[r] = routes whose expert lies in [r * epr, (r + 1) * epr).
__global__ void ep_rank_counts_kernel(const int* __restrict__ elist_off, int R, int epr,
                                      unsigned long long* __restrict__ counts) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r < R) counts[r] = (unsigned long long)(elist_off[(r + 1) * epr] - elist_off[r * epr]);
}

// Owner, one CTA: per-expert counts of the n received records, their
// exclusive scan into elist_off [El + 1], the active list, zeroed cursors.
// A record naming an expert outside [expert0, expert0 + El) raises
// kErrBounds and is left out.
__global__ void __launch_bounds__(1024) ep_count_kernel(const EpMeta* __restrict__ meta, int n, int expert0, int El,
                                                        int* __restrict__ elist_off, int* __restrict__ cursor,
                                                        int* __restrict__ active, int* __restrict__ n_active,
                                                        uint32_t* err) {
    extern __shared__ int s_cnt[];  // [El]
    for (int e = threadIdx.x; e < El; e += blockDim.x) s_cnt[e] = 0;
    __syncthreads();
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
        const int le = meta[j].expert - expert0;
        if (le < 0 || le >= El) {
            raise_error(err, kErrBounds);
            continue;
        }
        atomicAdd(&s_cnt[le], 1);
    }
    __syncthreads();
    // the active list with the most records first (ties: lower id), the
    // order in which the persistent expert kernels claim work
    for (int e = threadIdx.x; e < El; e += blockDim.x) {
        const int c = s_cnt[e];
        if (!c) continue;
        int rank = 0;
        for (int e2 = 0; e2 < El; e2++) rank += (s_cnt[e2] > c) || (s_cnt[e2] == c && e2 < e);
        active[rank] = e;
    }
    if (threadIdx.x == 0) {
        int off = 0, na = 0;
        for (int e = 0; e < El; e++) {
            elist_off[e] = off;
            cursor[e] = 0;
            na += s_cnt[e] > 0;
            off += s_cnt[e];
        }
        elist_off[El] = off;
        *n_active = na;
    }
}

// Owner: elist[elist_off[le] + c] = record index, c a per-expert cursor. The
// order inside an expert's list does not change any result: every record is
// its own token, computed independently.
__global__ void ep_scatter_kernel(const EpMeta* __restrict__ meta, int n, int expert0, int El,
                                  const int* __restrict__ elist_off, int* __restrict__ cursor, int* __restrict__ elist,
                                  float* __restrict__ ones) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= n) return;
    ones[j] = 1.0f;
    const int le = meta[j].expert - expert0;
    if (le < 0 || le >= El) return;
    elist[elist_off[le] + atomicAdd(&cursor[le], 1)] = j;
}

// Home: pos[token * k + slot] = record index of that route.
__global__ void ep_pos_kernel(const EpMeta* __restrict__ meta, int n, int M, int k, int* __restrict__ pos,
                              uint32_t* err) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= n) return;
    const EpMeta m = meta[j];
    if (m.token < 0 || m.token >= M || m.slot < 0 || m.slot >= k) {
        raise_error(err, kErrBounds);
        return;
    }
    pos[m.token * k + m.slot] = j;
}

// Home: out[t][c] = sum_s w_s * y[pos[t*k + s]][c], s best first, starting
// from 0 (moe.rs:63-68).
// A route no record covered (pos left at -1) raises kErrBounds.
__global__ void ep_combine_kernel(const EpMeta* __restrict__ meta, const int* __restrict__ pos,
                                  const float* __restrict__ y, int n, int M, int k, int H, float* __restrict__ out,
                                  uint32_t* err) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x, t = blockIdx.y;
    if (c >= H || t >= M) return;
    float o = 0.0f;
    for (int s = 0; s < k; s++) {
        const int j = pos[t * k + s];
        if (j < 0 || j >= n) {
            raise_error(err, kErrBounds);
            return;
        }
        const float w = __int_as_float(meta[j].wbits);
        o = fadd(o, fmul(w, __ldg(y + (size_t)j * H + c)));
    }
    out[(size_t)t * H + c] = o;
}

}  // namespace hale
