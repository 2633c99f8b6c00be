// hale_p2p.cuh -- expert parallelism over NVLink peer memory.
//
// MoeLayer::forward (src/model/moe.rs:56-70) with the experts of a layer
// split over R ranks (rank r owns [r * E/R, (r+1) * E/R)), one process per
// GPU. Every rank holds one exchange block of the same layout; peers map it
// through CUDA IPC, so the exchange is plain stores over NVLink with no host
// round trip between the steps:
//   1. p2p_dispatch_kernel (home): one record per route -- the home token's
//      Q8Activations row (quantized once: a pure function of x, so this
//      equals the reference re-quantizing inside each expert), its block
//      aux and (token, slot, expert, weight) -- stored straight into the
//      owner's receive region for this home; the last CTA writes the count
//      and raises the owner's "records" flag (release, system scope).
//   2. p2p_gather_kernel (owner): waits (bounded) for every home's flag,
//      groups the records by local expert (most records first), and points
//      each record's output row at its home's y_back row (token, slot).
//   3. the streaming expert kernels at k = 1 (weight 1, so their combine
//      stores y itself) write those rows over NVLink as they finish.
//   4. p2p_signal_kernel (owner): raises every home's "y rows" flag.
//   5. p2p_combine_kernel (home): waits (bounded) for every owner's flag,
//      then out[t] = sum over slots s, best first, of w * y_back[t, s],
//      starting from 0 -- the 1-GPU combine order, so the layer output is
//      bit-identical to hale_moe_forward on one GPU.
// Buffers alternate between two halves by call parity. A home only reuses a
// half two calls later, after its combine has seen every owner finish the
// call in between, so no store lands in a half a peer still reads.
// No kernel here waits on another kernel of the same GPU: every wait is on
// a flag another GPU raises (or, with one rank, one the stream has already
// raised).
#pragma once

#include "hale_ep.cuh"

namespace hale {

constexpr int kP2pMaxRanks = 8;

// Offsets inside one rank's exchange block (same on every rank).
struct P2pLayout {
    int R, H, nbp, cap, ytok;  // ranks, hidden, aux pairs per row, records per (half, home), y rows per half
    size_t q, a, m, count, flag, yback, yflag, total;
};

__host__ __device__ inline size_t p2p_align(size_t v) { return (v + 255) & ~(size_t)255; }

__host__ __device__ inline P2pLayout p2p_layout(int R, int H, int nbp, int cap, int ytok) {
    P2pLayout L;
    L.R = R;
    L.H = H;
    L.nbp = nbp;
    L.cap = cap;
    L.ytok = ytok;
    const size_t recs = (size_t)2 * R * cap;
    size_t o = 0;
    L.q = o;
    o = p2p_align(o + recs * H);
    L.a = o;
    o = p2p_align(o + recs * nbp * 8);
    L.m = o;
    o = p2p_align(o + recs * sizeof(EpMeta));
    L.count = o;
    o = p2p_align(o + (size_t)2 * R * 4);
    L.flag = o;
    o = p2p_align(o + (size_t)2 * R * 8);
    L.yback = o;
    o = p2p_align(o + (size_t)2 * ytok * H * 4);
    L.yflag = o;
    o = p2p_align(o + (size_t)2 * R * 8);
    L.total = o;
    return L;
}

// Record (half, home, j) of a block.
__host__ __device__ inline size_t p2p_rec(const P2pLayout& L, int half, int home, int j) {
    return ((size_t)half * L.R + home) * L.cap + j;
}

struct P2pPeers {
    uint8_t* base[kP2pMaxRanks];  // every rank's exchange block, this rank's own included
};

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Bounded spin until *flag == epoch (about a second of clocks); false and
// kErrTimeout on expiry.
__device__ __forceinline__ bool p2p_wait_flag(const unsigned long long* flag, unsigned long long epoch, uint32_t* err) {
    const long long t0 = clock64();
    while (ld_acquire_sys(flag) != epoch) {
        if (clock64() - t0 > (1LL << 31)) {
            raise_error(err, kErrTimeout);
            return false;
        }
        __nanosleep(64);
    }
    return true;
}

struct P2pDispatchArgs {
    P2pPeers peers;
    P2pLayout L;
    int rank, half, k, epr;
    unsigned long long epoch;
    int n;                      // routes = M * k
    const int* elist;           // routes in expert order (owner ranks ascending)
    const int* elist_off;       // [E + 1]
    const int* topk_idx;
    const float* topk_w;
    const int8_t* xq;           // [M, H]
    const int2* xaux;           // [M, nbp]
    unsigned* done;             // CTA counter, zero at launch, reset by the last CTA
};

// One warp per route, in expert-list order: the route's index inside its
// owner's share is its offset from the owner's first expert's list start.
__global__ void __launch_bounds__(256) p2p_dispatch_kernel(P2pDispatchArgs a) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int j = blockIdx.x * (blockDim.x >> 5) + warp;
    const P2pLayout& L = a.L;
    if (j < a.n) {
        const int route = a.elist[j], tok = route / a.k;
        const int e = a.topk_idx[route], owner = e / a.epr;
        const int idx = j - a.elist_off[owner * a.epr];
        uint8_t* blk = a.peers.base[owner];
        const size_t rec = p2p_rec(L, a.half, a.rank, idx);
        const uint4* src = reinterpret_cast<const uint4*>(a.xq + (size_t)tok * L.H);
        uint4* dst = reinterpret_cast<uint4*>(blk + L.q + rec * L.H);
        for (int i = lane; i < L.H / 16; i += 32) dst[i] = __ldg(src + i);
        const int4* asrc = reinterpret_cast<const int4*>(a.xaux + (size_t)tok * L.nbp);
        int4* adst = reinterpret_cast<int4*>(blk + L.a + rec * L.nbp * 8);
        for (int i = lane; i < L.nbp / 2; i += 32) adst[i] = __ldg(asrc + i);
        if (lane == 0) {
            EpMeta m;
            m.token = tok;
            m.slot = route - tok * a.k;
            m.expert = e;
            m.wbits = __float_as_int(a.topk_w[route]);
            reinterpret_cast<EpMeta*>(blk + L.m)[rec] = m;
        }
    }
    __syncthreads();
    __shared__ bool s_last;
    if (threadIdx.x == 0) {
        __threadfence_system();
        s_last = atomicAdd(a.done, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!s_last) return;
    // last CTA: every record of every CTA is out; counts, then the flags
    if (threadIdx.x < L.R) {
        const int r = threadIdx.x;
        __threadfence_system();
        uint8_t* blk = a.peers.base[r];
        const int cnt = a.elist_off[(r + 1) * a.epr] - a.elist_off[r * a.epr];
        reinterpret_cast<int*>(blk + L.count)[a.half * L.R + a.rank] = cnt;
        __threadfence_system();
        st_release_sys(reinterpret_cast<unsigned long long*>(blk + L.flag) + a.half * L.R + a.rank, a.epoch);
    }
    if (threadIdx.x == 0) *a.done = 0u;
}

struct P2pGatherArgs {
    P2pPeers peers;
    P2pLayout L;
    int rank, half, k, expert0, El;
    unsigned long long epoch;
    int* elist_off;   // [El + 1]
    int* elist;       // [R * cap] record ids (home * cap + j)
    int* active;      // [El]
    int* n_active;
    float* ones;      // [R * cap] weight 1 per record
    float** out_rows; // [R * cap] the home's y_back row of each record
    uint32_t* err;
};

// Owner, one CTA: the records of every home for this call, grouped by
// local expert (most records first), each with its output row.
__global__ void __launch_bounds__(1024) p2p_gather_kernel(P2pGatherArgs a) {
    extern __shared__ int s_cnt[];  // [El] then cursors [El]
    __shared__ int s_rc[kP2pMaxRanks];
    const P2pLayout& L = a.L;
    uint8_t* own = a.peers.base[a.rank];
    int* cur = s_cnt + a.El;
    for (int e = threadIdx.x; e < a.El; e += blockDim.x) s_cnt[e] = 0;
    if (threadIdx.x < L.R) {
        const int r = threadIdx.x;
        const bool ok = p2p_wait_flag(reinterpret_cast<unsigned long long*>(own + L.flag) + a.half * L.R + r, a.epoch,
                                      a.err);
        int c = ok ? reinterpret_cast<volatile int*>(own + L.count)[a.half * L.R + r] : 0;
        if (c < 0 || c > L.cap) {
            raise_error(a.err, kErrBounds);
            c = 0;
        }
        s_rc[r] = c;
    }
    __syncthreads();
    const EpMeta* meta = reinterpret_cast<const EpMeta*>(own + L.m);
    for (int r = 0; r < L.R; r++)
        for (int j = threadIdx.x; j < s_rc[r]; j += blockDim.x) {
            const int le = meta[p2p_rec(L, a.half, r, j)].expert - a.expert0;
            if (le < 0 || le >= a.El) {
                raise_error(a.err, kErrBounds);
                continue;
            }
            atomicAdd(&s_cnt[le], 1);
        }
    __syncthreads();
    for (int e = threadIdx.x; e < a.El; e += blockDim.x) {
        const int c = s_cnt[e];
        if (!c) continue;
        int rank = 0;
        for (int e2 = 0; e2 < a.El; e2++) rank += (s_cnt[e2] > c) || (s_cnt[e2] == c && e2 < e);
        a.active[rank] = e;
    }
    if (threadIdx.x == 0) {
        int off = 0, na = 0;
        for (int e = 0; e < a.El; e++) {
            a.elist_off[e] = off;
            cur[e] = off;
            na += s_cnt[e] > 0;
            off += s_cnt[e];
        }
        a.elist_off[a.El] = off;
        *a.n_active = na;
    }
    __syncthreads();
    for (int r = 0; r < L.R; r++)
        for (int j = threadIdx.x; j < s_rc[r]; j += blockDim.x) {
            const int id = r * L.cap + j;
            const EpMeta m = meta[p2p_rec(L, a.half, r, j)];
            const int le = m.expert - a.expert0;
            a.ones[id] = 1.0f;
            if (le < 0 || le >= a.El || m.token < 0 || m.token * a.k + m.slot >= L.ytok || m.slot < 0 ||
                m.slot >= a.k) {
                a.out_rows[id] = nullptr;
                continue;
            }
            a.out_rows[id] = reinterpret_cast<float*>(a.peers.base[r] + L.yback) +
                             ((size_t)a.half * L.ytok + (size_t)m.token * a.k + m.slot) * L.H;
            a.elist[atomicAdd(&cur[le], 1)] = id;
        }
}

// Owner, after its expert kernels: every home's y rows from this rank are
// written; raise each home's flag.
__global__ void p2p_signal_kernel(P2pPeers peers, P2pLayout L, int rank, int half, unsigned long long epoch) {
    const int r = threadIdx.x;
    if (r >= L.R) return;
    __threadfence_system();
    st_release_sys(reinterpret_cast<unsigned long long*>(peers.base[r] + L.yflag) + half * L.R + rank, epoch);
}

// Home: waits for every owner's flag (one thread per CTA), then
// out[t][c] = sum_s w[t, s] * y_back[t, s][c], s best first, from 0.
__global__ void __launch_bounds__(256) p2p_combine_kernel(const uint8_t* own, P2pLayout L, int half,
                                                          unsigned long long epoch, const float* __restrict__ topk_w,
                                                          int M, int k, float* __restrict__ out, uint32_t* err) {
    __shared__ bool s_ok;
    if (threadIdx.x == 0) {
        bool ok = true;
        for (int r = 0; r < L.R; r++)
            ok = p2p_wait_flag(reinterpret_cast<const unsigned long long*>(own + L.yflag) + half * L.R + r, epoch,
                               err) && ok;
        s_ok = ok;
    }
    __syncthreads();
    const int c = blockIdx.x * blockDim.x + threadIdx.x, t = blockIdx.y;
    if (!s_ok || c >= L.H || t >= M) return;
    const float* yb = reinterpret_cast<const float*>(own + L.yback) + (size_t)half * L.ytok * L.H;
    float o = 0.0f;
    for (int s = 0; s < k; s++) {
        const float w = __ldg(topk_w + (size_t)t * k + s);
        const float y = __ldcv(yb + ((size_t)t * k + s) * L.H + c);
        o = fadd(o, fmul(w, y));
    }
    out[(size_t)t * L.H + c] = o;
}

}  // namespace hale
