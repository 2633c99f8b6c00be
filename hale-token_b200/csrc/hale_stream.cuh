// hale_stream.cuh -- persistent streaming expert kernels on the warp-level
// int8 MMA.
//
// A CTA owns 128 weight rows of one expert at a time (four 32-row tiles; a
// "unit") and loops over units. One producer thread streams, ahead of the
// compute warps and across unit boundaries:
//   - each pass's activation rows (up to kPassRows tokens of the unit's
//     expert, gathered by bulk copies into a double-buffered stage), and
//   - the unit's weight tiles, SB blocks per tile per ring stage (copies of
//     ~9 KB: per-CTA bulk-copy throughput is bounded by the number of copies,
//     so copies are made large).
// Eight compute warps (two per tile, 16 rows each) read both from shared
// memory: per block, one mma.sync m16n8k32 gives the exact integer block
// sums of 16 rows x 8 tokens (C carries q4_0's -8 * sum(x) and the constant
// of the exact int -> float conversion), then the reference's float step
//     total += (w_scale * x_scale) * isum
// per block in block order (src/tensor/quant.rs:115-144), so results are
// bit-identical to the other expert kernels.
//
// Every wait is bounded. After a timeout the producer stops issuing; compute
// warps stop computing but keep their named-barrier schedule, so none is
// left waiting; the CTA drains the copies it issued (bounded) and returns;
// the error word tells the host.
#pragma once

#include "hale_kernels.cuh"

namespace hale {

constexpr int kPsComputeWarps = 8;
constexpr int kPsThreads = (kPsComputeWarps + 1) * 32;  // + the producer warp
constexpr int kPsMaxStages = 8;

// Blocks per tile per ring stage for `ctas` CTAs per SM: ~9 KB copies with
// one CTA per SM, ~4.5 KB with two (each then has half the shared memory).
__host__ __device__ inline int ps_stage_blocks(int qt, int ctas) { return (qt == 0 ? 16 : 8) / ctas; }

struct PsPlan {
    int stages, stage_bytes, xstride, xq_bytes, nbp, xa_bytes;
    int ring_off, xq_off, xa_off, bar_off, ctl_off, total;
};

// cols: the activation width (H for gate/up, I for down); budget: dynamic
// shared memory for one CTA.
__host__ __device__ inline PsPlan ps_plan(int BB, int SB, int cols, int budget) {
    PsPlan p;
    p.stage_bytes = 4 * SB * kTileRows * BB;
    p.xstride = xstage_stride(cols);
    p.xq_bytes = kPassRows * p.xstride;
    p.nbp = aux_stride(cols / kQK);
    p.xa_bytes = kPassRows * xaux_stride(p.nbp) * 8;
    const int n_bars = 2 * kPsMaxStages + 4;
    const int fixed = 2 * p.xq_bytes + 2 * p.xa_bytes + n_bars * 8 + 64 + 3 * 128;
    p.stages = (budget - fixed) / p.stage_bytes;
    if (p.stages > kPsMaxStages) p.stages = kPsMaxStages;
    p.ring_off = 0;
    p.xq_off = (p.stages * p.stage_bytes + 127) & ~127;
    p.xa_off = (p.xq_off + 2 * p.xq_bytes + 127) & ~127;
    p.bar_off = (p.xa_off + 2 * p.xa_bytes + 15) & ~15;
    p.ctl_off = p.bar_off + n_bars * 8;
    p.total = (p.ctl_off + 64 + 127) & ~127;
    return p;
}

__host__ __device__ inline bool ps_plan_ok(const PsPlan& p, int budget) { return p.stages >= 2 && p.total <= budget; }

struct PsCtl {
    int abort;  // a wait timed out
    int prod;   // weight stages issued
    int xq;     // activation passes issued
};

struct PsCtx {
    uint8_t* ring;
    int8_t* xq;  // [2][kPassRows][xstride]
    int2* xa;    // [2][kPassRows][astride]
    int S, SB, stage_bytes, xstride, nbp, astride, xq_bytes;
    uint64_t *full, *empty, *xfull, *xempty;
    volatile PsCtl* ctl;
};

__device__ __forceinline__ void ps_setup(PsCtx& c, uint8_t* smem, const PsPlan& P, int SB) {
    c.ring = smem + P.ring_off;
    c.xq = reinterpret_cast<int8_t*>(smem + P.xq_off);
    c.xa = reinterpret_cast<int2*>(smem + P.xa_off);
    c.S = P.stages;
    c.SB = SB;
    c.stage_bytes = P.stage_bytes;
    c.xstride = P.xstride;
    c.nbp = P.nbp;
    c.astride = xaux_stride(P.nbp);
    c.xq_bytes = P.xq_bytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + P.bar_off);
    c.full = bars;
    c.empty = bars + kPsMaxStages;
    c.xfull = bars + 2 * kPsMaxStages;
    c.xempty = c.xfull + 2;
    c.ctl = reinterpret_cast<volatile PsCtl*>(smem + P.ctl_off);
    if (threadIdx.x == 0) {
        for (int s = 0; s < c.S; s++) {
            mbar_init(&c.full[s], 1);
            mbar_init(&c.empty[s], kPsComputeWarps);
        }
        for (int s = 0; s < 2; s++) {
            mbar_init(&c.xfull[s], 1);
            mbar_init(&c.xempty[s], kPsComputeWarps);
        }
        fence_mbar_init();
        c.ctl->abort = 0;
        c.ctl->prod = 0;
        c.ctl->xq = 0;
    }
    __syncthreads();
}

__device__ __forceinline__ bool ps_wait(PsCtx& c, uint64_t* bar, uint32_t parity, uint32_t* err) {
    if (c.ctl->abort) return false;
    if (!mbar_wait(bar, parity, err)) {
        c.ctl->abort = 1;
        return false;
    }
    return true;
}

// Drains the copies that can still be landing after an abort (the last S
// weight stages and the last two activation passes issued), bounded. All
// threads.
__device__ __forceinline__ void ps_teardown(PsCtx& c) {
    __syncthreads();
    if (c.ctl->abort && threadIdx.x == 0) {
        for (int gs = max(0, c.ctl->prod - c.S); gs < c.ctl->prod; gs++)
            mbar_wait(&c.full[gs % c.S], (gs / c.S) & 1, nullptr, 400000000LL);
        for (int q = max(0, c.ctl->xq - 2); q < c.ctl->xq; q++)
            mbar_wait(&c.xfull[q & 1], (q >> 1) & 1, nullptr, 400000000LL);
    }
    __syncthreads();
}

// Barrier among the compute warps only.
__device__ __forceinline__ void ps_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kPsComputeWarps * 32) : "memory"); }

// A unit: four 32-row weight tiles of one expert, and the expert's tokens
// (slots beg .. beg+T-1 of the expert lists).
struct PsUnit {
    int e, beg, T;
    const uint8_t* tiles[4];
    int tile0;  // gate/up: first intermediate tile; down: first H tile
};

// The producer (one thread): per pass, the activation rows row_of(U, j)
// (quants from gq with `cols` columns, aux from ga), then the weight stages.
template <int QT, class UnitOf, class RowOf>
__device__ void ps_producer(PsCtx& c, int n_units, int nb, int cols, const int8_t* __restrict__ gq,
                            const int2* __restrict__ ga, UnitOf unit_of, RowOf row_of, uint32_t* err) {
    constexpr int REC = kTileRows * QFmt<QT>::BB;
    const int SB = c.SB, nst = (nb + SB - 1) / SB;
    int gs = 0, q = 0;
    for (int u = blockIdx.x; u < n_units; u += gridDim.x) {
        const PsUnit U = unit_of(u);
        for (int base = 0; base < U.T; base += kPassRows, q++) {
            const int n = min(kPassRows, U.T - base), xb = q & 1;
            if (!ps_wait(c, &c.xempty[xb], ((q >> 1) & 1) ^ 1, err)) return;
            fence_proxy_async_smem();
            mbar_arrive_expect_tx(&c.xfull[xb], (uint32_t)n * (uint32_t)(cols + c.nbp * 8));
            int8_t* xq = c.xq + (size_t)xb * c.xq_bytes;
            int2* xa = c.xa + (size_t)xb * kPassRows * c.astride;
            for (int j = 0; j < n; j++) {
                const int r = row_of(U, base + j);
                bulk_g2s(xq + (size_t)j * c.xstride, gq + (size_t)r * cols, (uint32_t)cols, &c.xfull[xb]);
                bulk_g2s(xa + (size_t)j * c.astride, ga + (size_t)r * c.nbp, (uint32_t)(c.nbp * 8), &c.xfull[xb]);
            }
            c.ctl->xq = q + 1;
            for (int s = 0; s < nst; s++, gs++) {
                const int slot = gs % c.S;
                if (!ps_wait(c, &c.empty[slot], ((gs / c.S) & 1) ^ 1, err)) return;
                const uint32_t bytes = (uint32_t)(min(SB, nb - s * SB) * REC);
                fence_proxy_async_smem();
                mbar_arrive_expect_tx(&c.full[slot], 4 * bytes);
                for (int w = 0; w < 4; w++)
                    bulk_g2s(c.ring + (size_t)slot * c.stage_bytes + (size_t)w * SB * REC,
                             U.tiles[w] + (size_t)s * SB * REC, bytes, &c.full[slot]);
                c.ctl->prod = gs + 1;
            }
        }
    }
}

// One pass of a compute warp: rows 16*half + {g, g+8} of tile `tile`,
// tokens {2t, 2t+1} of the pass: acc[row][token]. gs, q: the warp's global
// stage and pass counters. live goes false after an abort (the caller keeps
// its barrier schedule either way).
template <int QT>
__device__ void ps_pass(PsCtx& c, int nb, int tile, int half, int& gs, int q, float (&acc)[2][2], bool& live,
                        uint32_t* err) {
    constexpr int QB = QFmt<QT>::QB, REC = kTileRows * QFmt<QT>::BB;
    constexpr unsigned FULL = 0xffffffffu;
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int SB = c.SB, nst = (nb + SB - 1) / SB;
    const int xb = q & 1;
    acc[0][0] = acc[0][1] = acc[1][0] = acc[1][1] = 0.0f;
    // ldmatrix row addresses: B -- token (lane & 7), K half (lane >> 3) & 1; A --
    // rows 16*half + (lane & 15), K half lane >> 4 (q8_0), or rows 16*half +
    // (lane & 15) of nibble bytes (q4_0; lanes 16-31 repeat them)
    const int8_t* xrow = c.xq + (size_t)xb * c.xq_bytes + (lane & 7) * c.xstride + ((lane >> 3) & 1) * 16;
    const int2* xa = c.xa + (size_t)xb * kPassRows * c.astride;
    const int2* a0row = xa + (2 * t) * c.astride;
    const int2* a1row = xa + (2 * t + 1) * c.astride;
    const int r0 = half * 16 + g, r1 = r0 + 8;
    live = live && __all_sync(FULL, ps_wait(c, &c.xfull[xb], (q >> 1) & 1, err));
    for (int s = 0; s < nst; s++, gs++) {
        const int slot = gs % c.S;
        live = live && __all_sync(FULL, ps_wait(c, &c.full[slot], (gs / c.S) & 1, err));
        if (!live) continue;
        const uint8_t* stage = c.ring + (size_t)slot * c.stage_bytes + (size_t)tile * SB * REC;
        const int nblk = min(SB, nb - s * SB);
#pragma unroll 4
        for (int bi = 0; bi < nblk; bi++) {
            const int b = s * SB + bi;
            const uint8_t* rec = stage + bi * REC;
            uint32_t bf[2];
            ldsm_x2(bf, xrow + b * kQK);
            const uint32_t bf0 = bf[0], bf1 = bf[1];
            const int2 x0 = a0row[b], x1 = a1row[b];
            const int c0 = ((QT == 0) ? x0.y : 0) + kMagicI, c1 = ((QT == 0) ? x1.y : 0) + kMagicI;
            uint32_t a[4];
            if (QT == 0) {
                // words t of rows r0, r1 -- byte j of a row holds element j (low
                // nibble) and j + 16 (high)
                uint32_t w[2];
                ldsm_x2(w, rec + (half * 16 + (lane & 15)) * QB);
                a[0] = w[0] & 0x0F0F0F0Fu;
                a[1] = w[1] & 0x0F0F0F0Fu;
                a[2] = (w[0] >> 4) & 0x0F0F0F0Fu;
                a[3] = (w[1] >> 4) & 0x0F0F0F0Fu;
            } else {
                ldsm_x4(a, rec + (half * 16 + (lane & 15)) * QB + (lane >> 4) * 16);
            }
            int d[4];
            mma_s8_16832(d, a, bf0, bf1, c0, c1);
            const float ws0 = half_bits_to_float(*reinterpret_cast<const uint16_t*>(rec + kTileRows * QB + r0 * 2));
            const float ws1 = half_bits_to_float(*reinterpret_cast<const uint16_t*>(rec + kTileRows * QB + r1 * 2));
            const float xs0 = __int_as_float(x0.x), xs1 = __int_as_float(x1.x);
            // d: (r0, 2t), (r0, 2t+1), (r1, 2t), (r1, 2t+1)
            acc[0][0] = fadd(acc[0][0], fmul(fmul(ws0, xs0), fsub(__int_as_float(d[0]), kMagicF)));
            acc[0][1] = fadd(acc[0][1], fmul(fmul(ws0, xs1), fsub(__int_as_float(d[1]), kMagicF)));
            acc[1][0] = fadd(acc[1][0], fmul(fmul(ws1, xs0), fsub(__int_as_float(d[2]), kMagicF)));
            acc[1][1] = fadd(acc[1][1], fmul(fmul(ws1, xs1), fsub(__int_as_float(d[3]), kMagicF)));
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&c.empty[slot]);
    }
    __syncwarp();
    if (lane == 0 && live) mbar_arrive(&c.xempty[xb]);  // the pass no longer reads its activation stage
}

// Phase 1: units of 64 intermediate rows -- tiles 0,1 gate rows, 2,3 the
// matching up rows -- so h = silu(g) * u and its q8 quantization are formed
// per pass in-CTA, as in expert_gate_up_kernel, and written in slot order.
template <int QT>
__global__ void __launch_bounds__(kPsThreads, 2) expert_gate_up_ps_kernel(ExpertArgs a, int budget, int sb) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float s_out[4][kPassRows][kTileRows];
    constexpr int REC = kTileRows * QFmt<QT>::BB;
    const int TI = a.I / kTileRows, nbh = a.H / kQK, nbpi = aux_stride(a.I / kQK);
    const int upe = TI / 2;
    const int n_units = *a.n_active * upe;
    if ((int)blockIdx.x >= n_units) return;
    const PsPlan P = ps_plan(QFmt<QT>::BB, sb, a.H, budget);
    PsCtx c;
    ps_setup(c, smem, P, sb);
    const size_t tile_bytes = (size_t)nbh * REC;
    auto unit_of = [&](int u) {
        PsUnit U;
        const int ai = u / upe, jj = u - ai * upe;
        U.e = a.active[ai];
        U.beg = a.elist_off[U.e];
        U.T = a.elist_off[U.e + 1] - U.beg;
        const uint8_t* eb = expert_base(a, U.e);
        U.tiles[0] = eb + (size_t)(2 * jj) * tile_bytes;
        U.tiles[1] = eb + (size_t)(2 * jj + 1) * tile_bytes;
        U.tiles[2] = eb + (size_t)(TI + 2 * jj) * tile_bytes;
        U.tiles[3] = eb + (size_t)(TI + 2 * jj + 1) * tile_bytes;
        U.tile0 = 2 * jj;
        return U;
    };
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp == kPsComputeWarps) {
        if (lane == 0) {
            const int k = a.k;
            ps_producer<QT>(c, n_units, nbh, a.H, a.xq, a.xaux, unit_of,
                            [&](const PsUnit& U, int j) { return a.elist[U.beg + j] / k; }, a.err);
        }
    } else {
        const int tile = warp >> 1, half = warp & 1, g = lane >> 2, t = lane & 3;
        bool live = true;
        int gs = 0, q = 0;
        for (int u = blockIdx.x; u < n_units; u += gridDim.x) {
            const PsUnit U = unit_of(u);
            for (int base = 0; base < U.T; base += kPassRows, q++) {
                const int n = min(kPassRows, U.T - base);
                float acc[2][2];
                ps_pass<QT>(c, nbh, tile, half, gs, q, acc, live, a.err);
#pragma unroll
                for (int h = 0; h < 2; h++)
#pragma unroll
                    for (int j = 0; j < 2; j++) s_out[tile][2 * t + j][half * 16 + h * 8 + g] = acc[h][j];
                ps_sync();
                // (intermediate tile it, token j) pairs: warp w takes w and w + 8
                for (int pr = warp; pr < 2 * kPassRows; pr += kPsComputeWarps) {
                    const int it = pr / kPassRows, j = pr % kPassRows;
                    if (j >= n || !live) continue;
                    const int slot = U.beg + base + j, itile = U.tile0 + it;
                    const float h = fmul(silu(s_out[it][j][lane]), s_out[2 + it][j][lane]);
                    const float amax = warp_max_abs(h);
                    const float scale = fdiv(amax, 127.0f);
                    const float inv = scale > 0.0f ? fdiv(1.0f, scale) : 0.0f;
                    const int qv = sat_i8(roundf(fmul(h, inv)));
                    const int qs = warp_sum_int(qv);
                    a.hq[(size_t)slot * a.I + itile * kTileRows + lane] = (int8_t)qv;
                    if (lane == 0) a.haux[(size_t)slot * nbpi + itile] = make_int2(__float_as_int(scale), -8 * qs);
                }
                ps_sync();  // s_out free for the next pass
            }
        }
    }
    ps_teardown(c);
}

// Phase 2: units of 128 rows of the down projection; y for every route, then
// the best-first combine of expert_down_kernel.
template <int QT>
__global__ void __launch_bounds__(kPsThreads, 2) expert_down_ps_kernel(ExpertArgs a, int budget, int sb) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int s_last[kPassRows];
    constexpr int REC = kTileRows * QFmt<QT>::BB;
    const int TI = a.I / kTileRows, TH = a.H / kTileRows, nbi = a.I / kQK, nbh = a.H / kQK;
    const int upe = TH / 4;
    const int n_units = *a.n_active * upe;
    if ((int)blockIdx.x >= n_units) return;
    const PsPlan P = ps_plan(QFmt<QT>::BB, sb, a.I, budget);
    PsCtx c;
    ps_setup(c, smem, P, sb);
    const size_t gu_tile = (size_t)nbh * REC, d_tile = (size_t)nbi * REC;
    auto unit_of = [&](int u) {
        PsUnit U;
        const int ai = u / upe, grp = u - ai * upe;
        U.e = a.active[ai];
        U.beg = a.elist_off[U.e];
        U.T = a.elist_off[U.e + 1] - U.beg;
        const uint8_t* db = expert_base(a, U.e) + (size_t)2 * TI * gu_tile;
        for (int w = 0; w < 4; w++) U.tiles[w] = db + (size_t)(4 * grp + w) * d_tile;
        U.tile0 = 4 * grp;
        return U;
    };
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp == kPsComputeWarps) {
        if (lane == 0)
            ps_producer<QT>(c, n_units, nbi, a.I, a.hq, a.haux, unit_of,
                            [&](const PsUnit& U, int j) { return U.beg + j; }, a.err);
    } else {
        const int k = a.k, ng = TH / 4;
        const int tile = warp >> 1, half = warp & 1, g = lane >> 2, t = lane & 3;
        const int ct = threadIdx.x;  // 0 .. 255 among the compute warps
        bool live = true;
        int gs = 0, q = 0;
        for (int u = blockIdx.x; u < n_units; u += gridDim.x) {
            const PsUnit U = unit_of(u);
            const int grp = U.tile0 / 4;
            const int* routes = a.elist + U.beg;
            for (int base = 0; base < U.T; base += kPassRows, q++) {
                const int n = min(kPassRows, U.T - base);
                float acc[2][2];
                ps_pass<QT>(c, nbi, tile, half, gs, q, acc, live, a.err);
                if (live) {
#pragma unroll
                    for (int j = 0; j < 2; j++) {
                        const int tok = 2 * t + j;
                        if (tok < n) {
                            float* yrow = a.ybuf + (size_t)routes[base + tok] * a.H + (U.tile0 + tile) * kTileRows;
                            yrow[half * 16 + g] = acc[0][j];
                            yrow[half * 16 + 8 + g] = acc[1][j];
                        }
                    }
                }
                __threadfence();
                ps_sync();
                if (ct < n) {
                    s_last[ct] = 0;
                    if (live) {
                        const int tok = routes[base + ct] / k;
                        const unsigned old = atomicAdd(&a.comb_cnt[(size_t)tok * ng + grp], 1u);
                        if (old == (unsigned)(k - 1)) {
                            s_last[ct] = 1;
                            a.comb_cnt[(size_t)tok * ng + grp] = 0u;
                        }
                    }
                }
                ps_sync();
                __threadfence();
                // combine: the group's 128 rows for each token whose routes are all in
                const int row = ct & 127;
                for (int j = ct >> 7; j < n; j += 2) {
                    if (!s_last[j]) continue;
                    const int tok = routes[base + j] / k;
                    const size_t col = (size_t)U.tile0 * kTileRows + row;
                    float o = 0.0f;
                    for (int s2 = 0; s2 < k; s2++) {
                        const float w = __ldcg(a.topk_w + (size_t)tok * k + s2);
                        const float y = __ldcg(a.ybuf + ((size_t)tok * k + s2) * a.H + col);
                        o = fadd(o, fmul(w, y));
                    }
                    a.out[(size_t)tok * a.H + col] = o;
                }
                ps_sync();  // s_last free for the next pass
            }
        }
    }
    ps_teardown(c);
}

}  // namespace hale
