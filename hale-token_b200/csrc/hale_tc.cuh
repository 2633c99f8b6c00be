// hale_tc.cuh -- tensor-core (tcgen05, kind::i8) expert kernels for batches in
// which an expert sees several tokens.
//
// A CTA owns 128 weight rows of one expert at a time (four 32-row tiles; a
// "unit") and loops over units (persistent: one CTA per SM). Per quantization
// block the integer dot  isum[row, token] = sum_j w[row, j] x[token, j]  is one
// tcgen05.mma (M = 128 rows, N = kTcN token columns, K = 32 = one block) into
// its own TMEM column slab; CUDA cores then apply the reference's float step
//     total += (w_scale * x_scale) * isum
// per block, in block order and unfused, as dot_q8_0 / dot_q4_0 do
// (src/tensor/quant.rs:115-144). Integer products are exact, so results are
// bit-identical to the dp4a kernels in hale_kernels.cuh. q4_0 nibbles are
// unpacked to their signed values (n - 8) before the MMA, which yields the
// reference's block sum directly.
//
// Warp roles (576 threads), connected only by mbarriers:
//   warp 16 (lane 0) producer: weight tiles HBM -> shared-memory ring by
//                    cp.async.bulk, one copy of SB blocks (~9 KB) per tile
//                    per stage -- per-SM copy throughput is bounded by the
//                    number of copies, so copies are made large -- running
//                    ahead across unit boundaries;
//   warps 8-15       transform, two groups of four that own alternate ring
//                    stages (their latencies overlap): per chunk of 4 blocks,
//                    unpack their quadrant's quants in registers into TMEM
//                    with tcgen05.st as the A operand (A never touches shared
//                    memory), stage the chunk's activation bytes as the MMA's
//                    B operand, and hand row and activation scales to the
//                    epilogue through a shared-memory ring;
//   warp 17 (lane 0) MMA issue: 4 MMAs per chunk, commits to the chunk's D
//                    barrier and to its A/B slot's free barrier;
//   warps 0-7        epilogue: two warps per TMEM lane quadrant, each taking
//                    half of the pass's tokens: tcgen05.ld of the D slabs, the
//                    exact float steps, then the layer's per-pass output.
// A/B and D are 4-deep rings of chunk slots and the scales an 8-deep ring,
// so the roles work on different chunks at once.
//
// B operand layout in shared memory: canonical no-swizzle K-major. Core
// matrices of 8 token rows x 16 bytes are 128 contiguous bytes; the two core
// matrices of a block's K are 128 bytes apart (leading byte offset),
// consecutive 8-token groups 256 bytes apart (stride byte offset).
//
// Every wait is bounded. On a timeout a role stops issuing work (epilogue
// warps keep their barrier schedule so none is left waiting), the CTA drains
// what it issued (bounded), frees TMEM and returns; the error word tells the
// host.
#pragma once

#include "hale_kernels.cuh"

namespace hale {

constexpr int kTcN = 16;                 // token columns per MMA (MMA's N)
constexpr int kTcChunk = 4;              // quantization blocks per chunk (MMA / TMEM granularity)
constexpr int kTcMaxStages = 8;          // weight ring depth cap
constexpr int kTcABuf = 4, kTcDBuf = 4;  // A/B and D ring depths (chunks)
constexpr int kTcWsBuf = 8;              // scale ring depth (chunks)
constexpr int kTcDCols = kTcDBuf * kTcChunk * kTcN;  // 256: D slabs
constexpr int kTcACols = kTcABuf * kTcChunk * 8;     // 128: A slabs (32 int8 = 8 columns per block)
constexpr int kTcTmemCols = 512;                     // power of two >= kTcDCols + kTcACols
constexpr int kTcBSlot = kTcChunk * kTcN * 32;       // 2048: one chunk of B (4 blocks x 16 tokens x 32 bytes)
constexpr int kTcEpiWarps = 8, kTcXformWarp0 = 8, kTcProdWarp = 16, kTcMmaWarp = 17;
constexpr int kTcThreads = 576;
// dynamic shared memory the kernels may plan with (their static arrays and
// the 1 KB the runtime reserves stay outside)
constexpr int kTcSmemBudget = 227 * 1024 - 8 * 1024;

// Blocks per tile per ring stage: ~9 KB copies.
template <int QT>
struct TcStage;
template <>
struct TcStage<0> {
    static constexpr int SB = 16;  // 16 x 576 B = 9216 B per tile copy
};
template <>
struct TcStage<1> {
    static constexpr int SB = 8;   // 8 x 1088 B = 8704 B per tile copy
};

// ---- PTX wrappers -----------------------------------------------------------
__device__ __forceinline__ uint64_t tc_smem_desc(const void* p) {
    const uint64_t addr = smem_addr(p);
    return ((addr >> 4) & 0x3FFFull)      // start address
           | ((uint64_t)(128 >> 4) << 16) // leading byte offset: K-direction core-matrix stride
           | ((uint64_t)(256 >> 4) << 32) // stride byte offset: 8-row-group stride
           | (1ull << 46);                // descriptor version for tcgen05; base offset 0, no swizzle
}

// kind::i8, signed A and B, s32 accumulators, both K-major, M = 128, N = kTcN.
constexpr uint32_t kTcIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kTcN >> 3) << 17) |
                              ((uint32_t)(128 >> 4) << 24);

// D[tmem] = A[tmem] x B[smem]^T for one 32-wide K block (no accumulation).
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint32_t a_tmem, uint64_t b) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b), "r"(kTcIdesc), "r"(0)
        : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Whole-warp TMEM allocation of kTcTmemCols columns; the address lands in *slot.
__device__ __forceinline__ void tc_alloc(uint32_t* slot) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(slot)),
                 "n"(kTcTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tc_dealloc(uint32_t taddr) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "n"(kTcTmemCols)
                 : "memory");
}

// This thread's lane (row) of 8 consecutive TMEM columns <- w[0..7].
__device__ __forceinline__ void tc_st8(uint32_t taddr, const uint32_t (&w)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr),
                 "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7])
                 : "memory");
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Loads LW consecutive TMEM columns of this thread's lane; complete after tc_wait_ld().
template <int LW>
__device__ __forceinline__ void tc_ld(uint32_t taddr, int* v);
template <>
__device__ __forceinline__ void tc_ld<4>(uint32_t taddr, int* v) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
                 : "r"(taddr)
                 : "memory");
}
template <>
__device__ __forceinline__ void tc_ld<8>(uint32_t taddr, int* v) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr)
                 : "memory");
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Barrier among the epilogue warps only.
__device__ __forceinline__ void epi_sync() {
    asm volatile("bar.sync 2, %0;" ::"n"(kTcEpiWarps * 32) : "memory");
}

// q4_0: 8 nibble values (low nibbles of 4 bytes, or high) -> signed bytes n - 8.
__device__ __forceinline__ uint32_t q4_signed(uint32_t nib4) {
    return (((nib4 & 0x0F0F0F0Fu) | 0x80808080u) - 0x08080808u) ^ 0x80808080u;
}

// ---- shared-memory plan -------------------------------------------------------
struct TcPlan {
    int stages, stage_bytes, ring_off, b_off, ws_off, xs_off, bar_off, ctl_off, total;
};

// SB: blocks per tile per stage; BB: bytes per block row.
__host__ __device__ inline TcPlan tc_plan(int BB, int SB) {
    TcPlan p;
    p.stage_bytes = 4 * SB * kTileRows * BB;
    const int n_bars = 2 * kTcMaxStages + 2 * kTcABuf + 2 * kTcDBuf + 2 * kTcWsBuf;
    const int fixed = kTcABuf * kTcBSlot + kTcWsBuf * kTcChunk * (128 + kTcN) * 4 + n_bars * 8 + 64 + 4 * 128 + 4096;
    p.stages = (kTcSmemBudget - fixed) / p.stage_bytes;
    if (p.stages > kTcMaxStages) p.stages = kTcMaxStages;
    p.stages &= ~1;  // the two transform groups own the even / odd slots
    p.ring_off = 0;
    p.b_off = (p.stages * p.stage_bytes + 127) & ~127;
    p.ws_off = p.b_off + kTcABuf * kTcBSlot;
    p.xs_off = p.ws_off + kTcWsBuf * kTcChunk * 128 * 4;
    p.bar_off = p.xs_off + kTcWsBuf * kTcChunk * kTcN * 4;
    p.ctl_off = p.bar_off + n_bars * 8;
    // slack keeps every address an operand descriptor can form inside the allocation
    p.total = ((p.ctl_off + 64 + 127) & ~127) + 4096;
    return p;
}

__host__ __device__ inline bool tc_plan_ok(const TcPlan& p) { return p.stages >= 2 && p.total <= kTcSmemBudget; }

struct TcCtl {
    uint32_t tmem;  // TMEM base (written by tcgen05.alloc)
    int abort;      // a wait timed out
    int prod;       // stages issued by the producer
    int mma;        // chunks committed by the MMA thread
};

struct TcCtx {
    uint8_t* ring;
    uint8_t* B;   // [kTcABuf] chunk slots
    float* ws;    // [kTcWsBuf][kTcChunk][128] weight-row scales
    float* xs;    // [kTcWsBuf][kTcChunk][kTcN] activation scales
    int S, SB, stage_bytes;
    uint64_t *full, *empty, *a_full, *a_empty, *d_full, *d_empty, *w_full, *w_empty;
    volatile TcCtl* ctl;
    uint32_t tmem;
    __device__ __forceinline__ uint32_t taddr(int quadrant, int col) const {
        return tmem + ((uint32_t)(quadrant * 32) << 16) + (uint32_t)col;
    }
    __device__ __forceinline__ int d_col(int buf, int bi) const { return (buf * kTcChunk + bi) * kTcN; }
    __device__ __forceinline__ int a_col(int buf, int bi) const { return kTcDCols + (buf * kTcChunk + bi) * 8; }
};

__device__ __forceinline__ void tc_setup(TcCtx& c, uint8_t* smem, const TcPlan& P, int SB) {
    c.ring = smem + P.ring_off;
    c.B = smem + P.b_off;
    c.ws = reinterpret_cast<float*>(smem + P.ws_off);
    c.xs = reinterpret_cast<float*>(smem + P.xs_off);
    c.S = P.stages;
    c.SB = SB;
    c.stage_bytes = P.stage_bytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + P.bar_off);
    c.full = bars;
    c.empty = c.full + kTcMaxStages;
    c.a_full = c.empty + kTcMaxStages;
    c.a_empty = c.a_full + kTcABuf;
    c.d_full = c.a_empty + kTcABuf;
    c.d_empty = c.d_full + kTcDBuf;
    c.w_full = c.d_empty + kTcDBuf;
    c.w_empty = c.w_full + kTcWsBuf;
    c.ctl = reinterpret_cast<volatile TcCtl*>(smem + P.ctl_off);
    if (threadIdx.x == 0) {
        for (int s = 0; s < c.S; s++) {
            mbar_init(&c.full[s], 1);   // producer's expect_tx arrive
            mbar_init(&c.empty[s], 4);  // the owning transform group's warps
        }
        for (int s = 0; s < kTcABuf; s++) {
            mbar_init(&c.a_full[s], 4);   // the chunk's transform group
            mbar_init(&c.a_empty[s], 1);  // MMA commit
        }
        for (int s = 0; s < kTcDBuf; s++) {
            mbar_init(&c.d_full[s], 1);            // MMA commit
            mbar_init(&c.d_empty[s], kTcEpiWarps);  // epilogue warps
        }
        for (int s = 0; s < kTcWsBuf; s++) {
            mbar_init(&c.w_full[s], 4);
            mbar_init(&c.w_empty[s], kTcEpiWarps);
        }
        fence_mbar_init();
        c.ctl->abort = 0;
        c.ctl->prod = c.ctl->mma = 0;
    }
    if ((threadIdx.x >> 5) == 0) tc_alloc(const_cast<uint32_t*>(&c.ctl->tmem));
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    c.tmem = c.ctl->tmem;
}

// Bounded wait that gives up at once when another role has aborted.
__device__ __forceinline__ bool tc_wait(TcCtx& c, uint64_t* bar, uint32_t parity, uint32_t* err) {
    if (c.ctl->abort) return false;
    if (!mbar_wait(bar, parity, err)) {
        c.ctl->abort = 1;
        return false;
    }
    return true;
}

// Drains what is still in flight (bounded), then frees TMEM. All threads.
// MMAs retire in order, so the last commit's barrier covers them; the last
// S stages issued are the only copies that can still be landing, one per
// ring slot.
__device__ __forceinline__ void tc_teardown(TcCtx& c) {
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (c.ctl->abort) {
        if (threadIdx.x == 0 && c.ctl->mma > 0) {
            const int g = c.ctl->mma - 1;
            mbar_wait(&c.d_full[g % kTcDBuf], (g / kTcDBuf) & 1, nullptr, 400000000LL);
        }
        if (threadIdx.x == kTcXformWarp0 * 32)
            for (int gs = max(0, c.ctl->prod - c.S); gs < c.ctl->prod; gs++)
                mbar_wait(&c.full[gs % c.S], (gs / c.S) & 1, nullptr, 400000000LL);
        __syncthreads();
    }
    if ((threadIdx.x >> 5) == 0) tc_dealloc(c.tmem);
}

// A unit: the four 32-row weight tiles one CTA covers, and the tokens routed
// to their expert (slots beg .. beg+T-1 of the expert lists).
struct TcUnit {
    int e, beg, T;
    const uint8_t* tiles[4];
    int out_tile0;  // gate/up: first intermediate tile; down: first H tile
};

// ---- roles ---------------------------------------------------------------------
template <int QT, int PW, class UnitOf>
__device__ void tc_producer(TcCtx& c, int n_units, int nb, UnitOf unit_of, uint32_t* err) {
    constexpr int REC = kTileRows * QFmt<QT>::BB;
    const int SB = c.SB, nst = (nb + SB - 1) / SB;
    int gs = 0;
    for (int u = blockIdx.x; u < n_units; u += gridDim.x) {
        const TcUnit U = unit_of(u);
        const int passes = (U.T + PW - 1) / PW;
        for (int p = 0; p < passes; p++)
            for (int s = 0; s < nst; s++, gs++) {
                const int slot = gs % c.S;
                if (!tc_wait(c, &c.empty[slot], ((gs / c.S) & 1) ^ 1, err)) return;
                const uint32_t bytes = (uint32_t)(min(SB, nb - s * SB) * REC);
                mbar_arrive_expect_tx(&c.full[slot], 4 * bytes);
                for (int w = 0; w < 4; w++)
                    bulk_g2s(c.ring + (size_t)slot * c.stage_bytes + (size_t)w * SB * REC,
                             U.tiles[w] + (size_t)s * SB * REC, bytes, &c.full[slot]);
                c.ctl->prod = gs + 1;
            }
    }
}

// Transform group `grp` (warps kTcXformWarp0 + 4*grp .. +3) handles the
// stages gs with gs % 2 == grp -- ring slots of that parity, since the ring
// depth is even -- and every chunk in them.
template <int QT, int PW, class UnitOf, class RowQ, class RowAux>
__device__ void tc_transform(TcCtx& c, int n_units, int nb, UnitOf unit_of, RowQ row_q, RowAux row_aux,
                             uint32_t* err) {
    constexpr int QB = QFmt<QT>::QB, REC = kTileRows * QFmt<QT>::BB;
    constexpr unsigned FULL = 0xffffffffu;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qd = warp & 3, grp = (warp - kTcXformWarp0) >> 2;
    const int xt = threadIdx.x - (kTcXformWarp0 + 4 * grp) * 32;  // 0..127 within the group
    const int SB = c.SB, nst = (nb + SB - 1) / SB;
    // this thread's share of a chunk's B operand: token bt, 16-byte piece bp
    // (block bp >> 1, K half bp & 1); of its activation scales: token st_t, block st_b
    const int bt = xt >> 3, bp = xt & 7, st_t = xt >> 2, st_b = xt & 3;
    int gs = 0, g = 0;
    for (int u = blockIdx.x; u < n_units; u += gridDim.x) {
        const TcUnit U = unit_of(u);
        const int passes = (U.T + PW - 1) / PW;
        for (int p = 0; p < passes; p++) {
            const int base = p * PW, n = min(PW, U.T - base);
            const int8_t* xrow = bt < n ? row_q(U, base + bt) : nullptr;
            const int2* arow = (xt < 64 && st_t < n) ? row_aux(U, base + st_t) : nullptr;
            for (int s = 0; s < nst; s++, gs++) {
                const int sblk = min(SB, nb - s * SB), nch = (sblk + kTcChunk - 1) / kTcChunk;
                if ((gs & 1) != grp) {
                    g += nch;
                    continue;
                }
                const int slot = gs % c.S;
                if (!__all_sync(FULL, tc_wait(c, &c.full[slot], (gs / c.S) & 1, err))) return;
                const uint8_t* stage = c.ring + (size_t)slot * c.stage_bytes + (size_t)qd * SB * REC;
                for (int ci = 0; ci < nch; ci++, g++) {
                    const int b0 = s * SB + ci * kTcChunk, nblk = min(kTcChunk, nb - b0);
                    const int ab = g % kTcABuf, wb = g % kTcWsBuf;
                    // activation bytes and scales of the chunk (L2-resident rows)
                    uint4 xv = make_uint4(0, 0, 0, 0);
                    if (xrow && (bp >> 1) < nblk)
                        xv = __ldg(reinterpret_cast<const uint4*>(xrow + (b0 + (bp >> 1)) * kQK + (bp & 1) * 16));
                    float xsv = 0.0f;
                    if (arow && st_b < nblk) xsv = __int_as_float(__ldg(&arow[b0 + st_b].x));
                    // weights of this warp's quadrant -> registers
                    uint32_t w[kTcChunk][8];
                    float ws[kTcChunk];
#pragma unroll
                    for (int bi = 0; bi < kTcChunk; bi++) {
                        ws[bi] = 0.0f;
                        if (bi < nblk) {
                            const uint8_t* rec = stage + (ci * kTcChunk + bi) * REC;
                            ws[bi] = half_bits_to_float(
                                *reinterpret_cast<const unsigned short*>(rec + kTileRows * QB + lane * 2));
                            if (QT == 0) {
                                // byte j holds element j (low nibble) and j + 16 (high)
                                const uint4 nib = *reinterpret_cast<const uint4*>(rec + lane * QB);
                                w[bi][0] = q4_signed(nib.x); w[bi][1] = q4_signed(nib.y);
                                w[bi][2] = q4_signed(nib.z); w[bi][3] = q4_signed(nib.w);
                                w[bi][4] = q4_signed(nib.x >> 4); w[bi][5] = q4_signed(nib.y >> 4);
                                w[bi][6] = q4_signed(nib.z >> 4); w[bi][7] = q4_signed(nib.w >> 4);
                            } else {
                                const uint4 q0 = *reinterpret_cast<const uint4*>(rec + lane * QB);
                                const uint4 q1 = *reinterpret_cast<const uint4*>(rec + lane * QB + 16);
                                w[bi][0] = q0.x; w[bi][1] = q0.y; w[bi][2] = q0.z; w[bi][3] = q0.w;
                                w[bi][4] = q1.x; w[bi][5] = q1.y; w[bi][6] = q1.z; w[bi][7] = q1.w;
                            }
                        }
                    }
                    // scales -> the epilogue's ring
                    if (!__all_sync(FULL, tc_wait(c, &c.w_empty[wb], ((g / kTcWsBuf) & 1) ^ 1, err))) return;
#pragma unroll
                    for (int bi = 0; bi < kTcChunk; bi++) c.ws[(wb * kTcChunk + bi) * 128 + qd * 32 + lane] = ws[bi];
                    if (xt < 64) c.xs[(wb * kTcChunk + st_b) * kTcN + st_t] = xsv;
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&c.w_full[wb]);
                    // B slot and A slabs of the chunk
                    if (!__all_sync(FULL, tc_wait(c, &c.a_empty[ab], ((g / kTcABuf) & 1) ^ 1, err))) return;
                    if (bt < kTcN)
                        *reinterpret_cast<uint4*>(c.B + ab * kTcBSlot + (bp >> 1) * (kTcN * 32) + (bt >> 3) * 256 +
                                                  (bp & 1) * 128 + (bt & 7) * 16) = xv;
                    fence_proxy_async_smem();  // generic writes -> visible to the MMA's async reads
                    tc_fence_after();
#pragma unroll
                    for (int bi = 0; bi < kTcChunk; bi++)
                        if (bi < nblk) tc_st8(c.taddr(qd, c.a_col(ab, bi)), w[bi]);
                    tc_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&c.a_full[ab]);
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&c.empty[slot]);  // the stage's quants are all in TMEM
            }
        }
    }
}

template <int PW, class UnitOf>
__device__ void tc_mma_issuer(TcCtx& c, int n_units, int nb, UnitOf unit_of, uint32_t* err) {
    const int nch = (nb + kTcChunk - 1) / kTcChunk;
    int g = 0;
    for (int u = blockIdx.x; u < n_units; u += gridDim.x) {
        const TcUnit U = unit_of(u);
        const int passes = (U.T + PW - 1) / PW;
        for (int p = 0; p < passes; p++) {
            for (int ch = 0; ch < nch; ch++, g++) {
                const int ab = g % kTcABuf, db = g % kTcDBuf;
                const int nblk = min(kTcChunk, nb - ch * kTcChunk);
                if (!tc_wait(c, &c.a_full[ab], (g / kTcABuf) & 1, err)) return;
                if (!tc_wait(c, &c.d_empty[db], ((g / kTcDBuf) & 1) ^ 1, err)) return;
                tc_fence_after();
                for (int bi = 0; bi < nblk; bi++)
                    tc_mma(c.taddr(0, c.d_col(db, bi)), c.taddr(0, c.a_col(ab, bi)),
                           tc_smem_desc(c.B + ab * kTcBSlot + bi * (kTcN * 32)));
                tc_commit(&c.d_full[db]);
                tc_commit(&c.a_empty[ab]);
                c.ctl->mma = g + 1;
            }
        }
    }
}

// Epilogue of one pass for row 32*quadrant + lane and this warp's LW token
// columns tcol .. tcol+LW-1 (nh of them real): acc[t]. `live` goes false
// after an abort; the caller keeps its barrier schedule either way.
template <int LW>
__device__ void tc_epilogue_pass(TcCtx& c, int nb, int nh, int tcol, int& g, float (&acc)[LW], bool& live,
                                 uint32_t* err) {
    constexpr unsigned FULL = 0xffffffffu;
    const int qd = (threadIdx.x >> 5) & 3, lane = threadIdx.x & 31;
    const int nch = (nb + kTcChunk - 1) / kTcChunk;
#pragma unroll
    for (int t = 0; t < LW; t++) acc[t] = 0.0f;
    for (int ch = 0; ch < nch; ch++, g++) {
        const int db = g % kTcDBuf, wb = g % kTcWsBuf;
        const int nblk = min(kTcChunk, nb - ch * kTcChunk);
        live = live && __all_sync(FULL, tc_wait(c, &c.w_full[wb], (g / kTcWsBuf) & 1, err));
        live = live && __all_sync(FULL, tc_wait(c, &c.d_full[db], (g / kTcDBuf) & 1, err));
        if (!live) continue;
        tc_fence_after();
        int v[kTcChunk][LW];
#pragma unroll
        for (int bi = 0; bi < kTcChunk; bi++)
            if (bi < nblk) tc_ld<LW>(c.taddr(qd, c.d_col(db, bi) + tcol), v[bi]);
        float ws[kTcChunk], x[kTcChunk][LW];
#pragma unroll
        for (int bi = 0; bi < kTcChunk; bi++) {
            ws[bi] = c.ws[(wb * kTcChunk + bi) * 128 + qd * 32 + lane];
            const float4* xb = reinterpret_cast<const float4*>(c.xs + (wb * kTcChunk + bi) * kTcN + tcol);
#pragma unroll
            for (int j = 0; j < LW / 4; j++) {
                const float4 f = xb[j];
                x[bi][4 * j] = f.x; x[bi][4 * j + 1] = f.y; x[bi][4 * j + 2] = f.z; x[bi][4 * j + 3] = f.w;
            }
        }
        tc_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
            mbar_arrive(&c.d_empty[db]);  // D slabs and scales now in registers
            mbar_arrive(&c.w_empty[wb]);
        }
#pragma unroll
        for (int bi = 0; bi < kTcChunk; bi++)
            if (bi < nblk)
#pragma unroll
                for (int t = 0; t < LW; t++)
                    if (t < nh) acc[t] = fadd(acc[t], fmul(fmul(ws[bi], x[bi][t]), __int2float_rn(v[bi][t])));
    }
}

// ---- kernels -------------------------------------------------------------------

// Phase 1: units of 64 intermediate rows of one expert -- A rows 0-63 are
// gate rows, 64-127 the matching up rows (quadrants 0,1 gate; 2,3 up) -- so
// h = silu(g) * u and its q8 quantization are formed per pass in-CTA, as in
// expert_gate_up_kernel, and written in slot order.
template <int QT, int PW>
__global__ void __launch_bounds__(kTcThreads, 1) expert_gate_up_tc_kernel(ExpertArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float s_g[2][kTcN][kTileRows];
    constexpr int LW = PW / 2;
    constexpr int REC = kTileRows * QFmt<QT>::BB;
    const int TI = a.I / kTileRows, nbh = a.H / kQK, nbph = aux_stride(nbh), nbpi = aux_stride(a.I / kQK);
    const int upe = TI / 2;
    const int n_units = *a.n_active * upe;
    if ((int)blockIdx.x >= n_units) return;
    const TcPlan P = tc_plan(QFmt<QT>::BB, TcStage<QT>::SB);
    TcCtx c;
    tc_setup(c, smem, P, TcStage<QT>::SB);
    const size_t tile_bytes = (size_t)nbh * REC;
    auto unit_of = [&](int u) {
        TcUnit U;
        const int ai = u / upe, jj = u - ai * upe;
        U.e = a.active[ai];
        U.beg = a.elist_off[U.e];
        U.T = a.elist_off[U.e + 1] - U.beg;
        const uint8_t* eb = expert_base(a, U.e);
        U.tiles[0] = eb + (size_t)(2 * jj) * tile_bytes;
        U.tiles[1] = eb + (size_t)(2 * jj + 1) * tile_bytes;
        U.tiles[2] = eb + (size_t)(TI + 2 * jj) * tile_bytes;
        U.tiles[3] = eb + (size_t)(TI + 2 * jj + 1) * tile_bytes;
        U.out_tile0 = 2 * jj;
        return U;
    };
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp == kTcProdWarp) {
        if (lane == 0) tc_producer<QT, PW>(c, n_units, nbh, unit_of, a.err);
    } else if (warp == kTcMmaWarp) {
        if (lane == 0) tc_mma_issuer<PW>(c, n_units, nbh, unit_of, a.err);
    } else if (warp >= kTcXformWarp0) {
        const int k = a.k;
        tc_transform<QT, PW>(
            c, n_units, nbh, unit_of,
            [&](const TcUnit& U, int j) { return a.xq + (size_t)(a.elist[U.beg + j] / k) * a.H; },
            [&](const TcUnit& U, int j) { return a.xaux + (size_t)(a.elist[U.beg + j] / k) * nbph; }, a.err);
    } else {
        const int qd = warp & 3, tcol = (warp >> 2) * LW;
        bool live = true;
        int g = 0;
        for (int u = blockIdx.x; u < n_units; u += gridDim.x) {
            const TcUnit U = unit_of(u);
            const int passes = (U.T + PW - 1) / PW;
            for (int p = 0; p < passes; p++) {
                const int base = p * PW, nh = min(PW, U.T - base) - tcol;
                float acc[LW];
                tc_epilogue_pass<LW>(c, nbh, nh, tcol, g, acc, live, a.err);
                if (qd < 2)
#pragma unroll
                    for (int t = 0; t < LW; t++) s_g[qd][tcol + t][lane] = acc[t];
                epi_sync();
                if (qd >= 2 && live) {
                    const int tile = U.out_tile0 + (qd - 2);
#pragma unroll
                    for (int t = 0; t < LW; t++) {
                        if (t < nh) {
                            const int slot = U.beg + base + tcol + t;
                            const float h = fmul(silu(s_g[qd - 2][tcol + t][lane]), acc[t]);
                            const float amax = warp_max_abs(h);
                            const float scale = fdiv(amax, 127.0f);
                            const float inv = scale > 0.0f ? fdiv(1.0f, scale) : 0.0f;
                            const int qv = sat_i8(roundf(fmul(h, inv)));
                            const int qs = warp_sum_int(qv);
                            a.hq[(size_t)slot * a.I + tile * kTileRows + lane] = (int8_t)qv;
                            if (lane == 0)
                                a.haux[(size_t)slot * nbpi + tile] = make_int2(__float_as_int(scale), -8 * qs);
                        }
                    }
                }
                epi_sync();  // s_g free for the next pass
            }
        }
    }
    tc_teardown(c);
}

// Phase 2: units of 128 rows of the down projection; y for every route, then
// the best-first combine of expert_down_kernel.
template <int QT, int PW>
__global__ void __launch_bounds__(kTcThreads, 1) expert_down_tc_kernel(ExpertArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int s_last[kTcN];
    constexpr int LW = PW / 2;
    constexpr int REC = kTileRows * QFmt<QT>::BB;
    const int TI = a.I / kTileRows, TH = a.H / kTileRows, nbi = a.I / kQK, nbh = a.H / kQK;
    const int nbpi = aux_stride(nbi);
    const int upe = TH / 4;
    const int n_units = *a.n_active * upe;
    if ((int)blockIdx.x >= n_units) return;
    const TcPlan P = tc_plan(QFmt<QT>::BB, TcStage<QT>::SB);
    TcCtx c;
    tc_setup(c, smem, P, TcStage<QT>::SB);
    const size_t gu_tile = (size_t)nbh * REC, d_tile = (size_t)nbi * REC;
    auto unit_of = [&](int u) {
        TcUnit U;
        const int ai = u / upe, grp = u - ai * upe;
        U.e = a.active[ai];
        U.beg = a.elist_off[U.e];
        U.T = a.elist_off[U.e + 1] - U.beg;
        const uint8_t* db = expert_base(a, U.e) + (size_t)2 * TI * gu_tile;
        for (int w = 0; w < 4; w++) U.tiles[w] = db + (size_t)(4 * grp + w) * d_tile;
        U.out_tile0 = 4 * grp;
        return U;
    };
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp == kTcProdWarp) {
        if (lane == 0) tc_producer<QT, PW>(c, n_units, nbi, unit_of, a.err);
    } else if (warp == kTcMmaWarp) {
        if (lane == 0) tc_mma_issuer<PW>(c, n_units, nbi, unit_of, a.err);
    } else if (warp >= kTcXformWarp0) {
        tc_transform<QT, PW>(
            c, n_units, nbi, unit_of, [&](const TcUnit& U, int j) { return a.hq + (size_t)(U.beg + j) * a.I; },
            [&](const TcUnit& U, int j) { return a.haux + (size_t)(U.beg + j) * nbpi; }, a.err);
    } else {
        const int k = a.k, ng = TH / 4;
        const int qd = warp & 3, tcol = (warp >> 2) * LW;
        bool live = true;
        int g = 0;
        for (int u = blockIdx.x; u < n_units; u += gridDim.x) {
            const TcUnit U = unit_of(u);
            const int grp = U.out_tile0 / 4, tile = U.out_tile0 + qd;
            const int passes = (U.T + PW - 1) / PW;
            const int* routes = a.elist + U.beg;
            for (int p = 0; p < passes; p++) {
                const int base = p * PW, n = min(PW, U.T - base), nh = n - tcol;
                float acc[LW];
                tc_epilogue_pass<LW>(c, nbi, nh, tcol, g, acc, live, a.err);
                if (live) {
#pragma unroll
                    for (int t = 0; t < LW; t++)
                        if (t < nh)
                            a.ybuf[(size_t)routes[base + tcol + t] * a.H + tile * kTileRows + lane] = acc[t];
                }
                __threadfence();
                epi_sync();
                if (threadIdx.x < n) {
                    s_last[threadIdx.x] = 0;
                    if (live) {
                        const int tok = routes[base + threadIdx.x] / k;
                        const unsigned old = atomicAdd(&a.comb_cnt[(size_t)tok * ng + grp], 1u);
                        if (old == (unsigned)(k - 1)) {
                            s_last[threadIdx.x] = 1;
                            a.comb_cnt[(size_t)tok * ng + grp] = 0u;
                        }
                    }
                }
                epi_sync();
                __threadfence();
                for (int j = tcol; j < min(n, tcol + LW); j++) {
                    if (!s_last[j]) continue;
                    const int tok = routes[base + j] / k;
                    float o = 0.0f;
                    for (int s2 = 0; s2 < k; s2++) {
                        const float w = __ldcg(a.topk_w + (size_t)tok * k + s2);
                        const float y = __ldcg(a.ybuf + ((size_t)tok * k + s2) * a.H + tile * kTileRows + lane);
                        o = fadd(o, fmul(w, y));
                    }
                    a.out[(size_t)tok * a.H + tile * kTileRows + lane] = o;
                }
                epi_sync();  // s_last free for the next pass
            }
        }
    }
    tc_teardown(c);
}

}  // namespace hale
