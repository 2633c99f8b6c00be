// hale_ws.cuh -- warp-specialised streaming expert kernels: TMA tensor loads
// feeding warp-level int8 MMA.
//
// Expert::forward (src/expert/mod.rs:91-103) for every route of a layer,
// grouped by expert so each weight tile is read from HBM once per pass of
// up to kPassRows tokens. Persistent CTAs (CPS per SM) take units from a
// global counter, so CTAs that finish early take more:
//   gate/up: (active expert, 64 rows of the intermediate dimension) -- two
//            32-row tiles of the gate matrix and the same two of up;
//   down:    (active expert, 128 rows of the hidden dimension) -- four tiles.
// One producer thread claims units and keeps a ring of stages in flight. A
// stage is one or two `cp.async.bulk.tensor` loads -- a 4-D box
// [tiles][blocks][record] of the pool's tile layout, no multicast -- and each
// pass's activation rows arrive by bulk copies into a double-buffered stage
// together with the pass descriptor (unit, first token) the consumers follow.
// Four consumer warps read both from shared memory:
//   gate/up: warp w takes rows 16*(w&1) .. +15 of tile w>>1 in BOTH gate and
//            up, so one B fragment and one aux load per block feed two
//            m16n8k32 MMAs, and h = silu(g) * u is formed in registers;
//   down:    warp w takes tile w (two MMAs per block sharing B and aux).
// Per block and token the reference's float step follows the MMA in block
// order, unfused:  total += (w_scale * x_scale) * isum  (quant.rs:115-144);
// the MMA's C operand carries q4_0's -8 * sum(x) and the exact int -> float
// constant. h is quantized per 32-row tile (one q8 block of h: the
// reference's re-quantization before down, matrix.rs:119-121); the two
// warps of a tile combine their amax and quant sums through shared memory.
//
// Every wait is bounded (mbar_wait). After a timeout the error word is set,
// the producer stops issuing, consumers stop computing but keep their
// barrier schedule, and the CTA drains the copies it issued before it
// returns.
#pragma once

#include <cuda.h>

#include "hale_kernels.cuh"

namespace hale {

constexpr int kWsConsumers = 4;
constexpr int kWsThreads = (kWsConsumers + 1) * 32;
constexpr int kWsMaxStages = 6;
constexpr int kWsSB = 4;  // blocks per tile per ring stage

// Dynamic shared memory per CTA with `cps` CTAs per SM (228 KB per SM, less
// the per-CTA reserve and the kernels' static arrays).
__host__ __device__ inline int ws_budget(int cps) {
    return cps >= 4 ? 55 * 1024 : cps == 3 ? 72 * 1024 : 110 * 1024;
}

// Shared-memory plan. boxes: TMA loads per stage (2 for gate/up, 1 for
// down); tiles: 32-row tiles per box; SB: blocks per tile per stage; cols:
// activation width; XB: activation buffers (2: the next pass loads while the
// current one is read; 1: it loads once the consumers release the buffer,
// after the producer has already put the next pass's first weight stages in
// flight -- less shared memory, so more CTAs fit per SM).
struct WsPlan {
    int SB, S, XB, box_bytes, stage_bytes, xstride, astride, xq_bytes, xa_bytes;
    int ring_off, xq_off, xa_off, bar_off, ctl_off, total;
};

__host__ __device__ inline WsPlan ws_plan(int REC, int boxes, int tiles, int SB, int cols, int budget, int XB = 2,
                                          int rows = kPassRows) {
    WsPlan p;
    p.SB = SB;
    p.XB = XB;
    p.box_bytes = tiles * SB * REC;
    p.stage_bytes = boxes * p.box_bytes;
    p.xstride = xstage_stride(cols);
    p.astride = xaux_stride(aux_stride(cols / kQK));
    p.xq_bytes = (rows * p.xstride + 127) & ~127;
    p.xa_bytes = (rows * p.astride * 8 + 127) & ~127;
    const int fixed = XB * p.xq_bytes + XB * p.xa_bytes + (2 * kWsMaxStages + 4) * 8 + 64;
    p.S = (budget - fixed) / p.stage_bytes;
    if (p.S > kWsMaxStages) p.S = kWsMaxStages;
    p.ring_off = 0;
    p.xq_off = p.S * p.stage_bytes;
    p.xa_off = p.xq_off + XB * p.xq_bytes;
    p.bar_off = p.xa_off + XB * p.xa_bytes;
    p.ctl_off = p.bar_off + (2 * kWsMaxStages + 4) * 8;
    p.total = p.ctl_off + 64;  // WsCtl
    return p;
}

// Both TMA destinations and bulk-copy destinations stay 128-byte aligned.
__host__ __device__ inline bool ws_plan_ok(const WsPlan& p, int budget) {
    return p.S >= 2 && p.total <= budget && p.box_bytes % 128 == 0;
}

// 4-D tiled TMA load of one box into shared memory, completing on `bar`.
// Coordinates, innermost first: element of the record (always 0, so the
// copy starts on a record boundary), block, tile, expert slot.
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int c1, int c2, int c3,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
        "%5}], [%6];" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Barriers among the consumer warps (id 1) and between the two warps of one
// gate/up tile (ids 2, 3). The producer warp takes part in neither.
__device__ __forceinline__ void ws_sync_consumers() {
    asm volatile("bar.sync 1, %0;" ::"n"(kWsConsumers * 32) : "memory");
}
__device__ __forceinline__ void ws_sync_pair(int tile) {
    // immediate barrier ids, so the kernel reserves only the ids it names
    if (tile == 0)
        asm volatile("bar.sync 2, 64;" ::: "memory");
    else
        asm volatile("bar.sync 3, 64;" ::: "memory");
}

// bar.red.and over the consumer warps (barrier id 1): one verdict for all.
__device__ __forceinline__ bool ws_consumers_all(bool p) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred a, b;\n\tsetp.ne.u32 a, %1, 0;\n\tbar.red.and.pred b, 1, %2, a;\n\tselp.u32 %0, 1, 0, b;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)p), "n"(kWsConsumers * 32)
        : "memory");
    return r != 0;
}

// Device-scope add with acquire-release order: the release publishes this
// CTA's earlier writes (ordered before it by a CTA barrier); the acquire
// makes other CTAs' writes released the same way visible.
__device__ __forceinline__ unsigned atomic_add_acq_rel(unsigned* p, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

struct WsCtl {
    int abort;   // a wait timed out
    int stages;  // weight stages the producer issued
    int passes;  // activation passes the producer issued
    // per activation buffer, the pass descriptor: first route slot of the
    // unit's expert, the pass's first token, its token count (< 0: no more
    // work) and the unit's first tile
    int pass_beg[2], pass_base[2], pass_n[2], pass_tile0[2];
};

struct WsCtx {
    uint8_t* ring;
    uint8_t* xq;  // [XB][xq_bytes]
    uint8_t* xa;  // [XB][xa_bytes]
    uint64_t *full, *empty, *xfull, *xempty;
    volatile WsCtl* ctl;
    WsPlan P;
};

__device__ __forceinline__ void ws_setup(WsCtx& c, uint8_t* smem, const WsPlan& P) {
    c.P = P;
    c.ring = smem + P.ring_off;
    c.xq = smem + P.xq_off;
    c.xa = smem + P.xa_off;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + P.bar_off);
    c.full = bars;
    c.empty = bars + kWsMaxStages;
    c.xfull = bars + 2 * kWsMaxStages;
    c.xempty = c.xfull + 2;
    c.ctl = reinterpret_cast<volatile WsCtl*>(smem + P.ctl_off);
    if (threadIdx.x == 0) {
        for (int s = 0; s < P.S; s++) {
            mbar_init(&c.full[s], 1);
            mbar_init(&c.empty[s], kWsConsumers);
        }
        for (int s = 0; s < 2; s++) {
            mbar_init(&c.xfull[s], 1);
            mbar_init(&c.xempty[s], kWsConsumers);
        }
        fence_mbar_init();
        c.ctl->abort = 0;
        c.ctl->stages = 0;
        c.ctl->passes = 0;
    }
    __syncthreads();
}

__device__ __forceinline__ bool ws_wait(WsCtx& c, uint64_t* bar, uint32_t parity, uint32_t* err) {
    if (c.ctl->abort) return false;
    if (!mbar_wait(bar, parity, err)) {
        c.ctl->abort = 1;
        return false;
    }
    return true;
}

// After an abort, waits (bounded) for the copies still landing: the last S
// weight stages and the last XB activation passes issued. All threads.
__device__ __forceinline__ void ws_teardown(WsCtx& c) {
    __syncthreads();
    if (c.ctl->abort && threadIdx.x == 0) {
        const int S = c.P.S, gs1 = c.ctl->stages, q1 = c.ctl->passes;
        for (int gs = max(0, gs1 - S); gs < gs1; gs++) mbar_wait(&c.full[gs % S], (gs / S) & 1, nullptr, 400000000LL);
        const int XB = c.P.XB;
        for (int q = max(0, q1 - XB); q < q1; q++)
            mbar_wait(&c.xfull[q % XB], (q / XB) & 1, nullptr, 400000000LL);
    }
    __syncthreads();
}

// A unit: an expert (routes beg .. beg+T-1 of the expert lists, slot
// coordinate cs in the tensor maps) and its first 32-row tile.
struct WsUnit {
    int e, beg, T, cs, tile0;
};

__device__ __forceinline__ int ws_slot(const ExpertArgs& a, int e) {
    return a.slot ? __ldg(a.slot + e) : a.expert0 + e;
}

// The next unit's metadata, fetched one dependent load at a time while the
// current unit's stages are issued, so the producer does not wait on global
// memory between units: step 0 claims a unit (atomic), 1 reads its expert,
// 2 its route range and slot, 3 the rows of its first pass; 4 = ready.
template <int PR>
struct WsNext {
    int u, ai, e, beg, end, cs, step;
    int rows[PR];
};

template <int PR, class RowOf>
__device__ __forceinline__ void ws_next_step(WsNext<PR>& nx, const ExpertArgs& a, unsigned* ctr, int n_units, int upe,
                                             int tpu, RowOf row_of) {
    if (nx.step == 0) {
        nx.u = (int)atomicAdd(ctr, 1u);
        nx.step = nx.u < n_units ? 1 : 4;
    } else if (nx.step == 1) {
        nx.ai = nx.u / upe;
        nx.e = __ldcg(a.active + nx.ai);
        nx.step = 2;
    } else if (nx.step == 2) {
        nx.beg = __ldcg(a.elist_off + nx.e);
        nx.end = __ldcg(a.elist_off + nx.e + 1);
        nx.cs = ws_slot(a, nx.e);
        nx.step = 3;
    } else if (nx.step == 3) {
        WsUnit U{nx.e, nx.beg, nx.end - nx.beg, nx.cs, tpu * (nx.u - nx.ai * upe)};
#pragma unroll
        for (int j = 0; j < PR; j++)
            if (j < U.T) nx.rows[j] = row_of(U, j);
        nx.step = 4;
    }
}

// The producer (one thread): claims units from ctr[0] until they run out;
// per unit and pass, the pass descriptor and activation rows (row_of(U, j)
// of gq / ga, `cols` columns), then the unit's weight stages -- per stage
// `boxes` TMA loads at tile coordinates tile_of(U, box). Ends with a
// descriptor of n = -1. tpu: 32-row tiles per unit; PR: tokens per pass.
template <int PR, class RowOf, class TileOf>
__device__ void ws_produce(WsCtx& c, const ExpertArgs& a, const CUtensorMap* map, int n_units, int upe, int tpu,
                           unsigned* ctr, int nb, int boxes, int cols, const int8_t* __restrict__ gq,
                           const int2* __restrict__ ga, int nbp, RowOf row_of, TileOf tile_of, uint32_t* err) {
    const WsPlan& P = c.P;
    const int nst = (nb + P.SB - 1) / P.SB;
    int gs = 0, q = 0;
    WsNext<PR> nx{};
    while (nx.step < 4) ws_next_step(nx, a, ctr, n_units, upe, tpu, row_of);
    while (nx.u < n_units) {
        const WsUnit U{nx.e, nx.beg, nx.end - nx.beg, nx.cs, tpu * (nx.u - nx.ai * upe)};
        int rows[PR];
#pragma unroll
        for (int j = 0; j < PR; j++) rows[j] = nx.rows[j];
        nx.step = 0;
        for (int base = 0; base < U.T; base += PR, q++) {
            const int n = min(PR, U.T - base), xb = q % P.XB;
            if (base > 0) {
#pragma unroll
                for (int j = 0; j < PR; j++)
                    if (j < n) rows[j] = row_of(U, base + j);
            }
            auto stage = [&](int s) {
                const int slot = gs % P.S;
                if (!ws_wait(c, &c.empty[slot], ((gs / P.S) & 1) ^ 1, err)) return false;
                fence_proxy_async_smem();
                mbar_arrive_expect_tx(&c.full[slot], (uint32_t)P.stage_bytes);
                for (int bx = 0; bx < boxes; bx++)
                    tma_load_4d(c.ring + (size_t)slot * P.stage_bytes + (size_t)bx * P.box_bytes, map, s * P.SB,
                                tile_of(U, bx), U.cs, &c.full[slot]);
                c.ctl->stages = ++gs;
                ws_next_step(nx, a, ctr, n_units, upe, tpu, row_of);  // the next unit, a step per stage
                return true;
            };
            // one activation buffer: the pass's first weight stages go out
            // before the wait for the buffer (their slots free up as the
            // previous pass's stages are consumed, which needs no activations)
            int s = 0;
            if (P.XB == 1)
                for (; s < min(P.S, nst); s++)
                    if (!stage(s)) return;
            if (!ws_wait(c, &c.xempty[xb], ((q / P.XB) & 1) ^ 1, err)) return;
            c.ctl->pass_beg[xb] = U.beg;
            c.ctl->pass_base[xb] = base;
            c.ctl->pass_n[xb] = n;
            c.ctl->pass_tile0[xb] = U.tile0;
            fence_proxy_async_smem();
            mbar_arrive_expect_tx(&c.xfull[xb], (uint32_t)n * (uint32_t)(cols + nbp * 8));
            int8_t* xq = reinterpret_cast<int8_t*>(c.xq + (size_t)xb * P.xq_bytes);
            int2* xa = reinterpret_cast<int2*>(c.xa + (size_t)xb * P.xa_bytes);
#pragma unroll
            for (int j = 0; j < PR; j++) {
                if (j < n) {
                    bulk_g2s(xq + (size_t)j * P.xstride, gq + (size_t)rows[j] * cols, (uint32_t)cols, &c.xfull[xb]);
                    bulk_g2s(xa + (size_t)j * P.astride, ga + (size_t)rows[j] * nbp, (uint32_t)(nbp * 8),
                             &c.xfull[xb]);
                }
            }
            c.ctl->passes = q + 1;
            for (; s < nst; s++)
                if (!stage(s)) return;
        }
        while (nx.step < 4) ws_next_step(nx, a, ctr, n_units, upe, tpu, row_of);
    }
    const int xb = q % P.XB;
    if (!ws_wait(c, &c.xempty[xb], ((q / P.XB) & 1) ^ 1, err)) return;
    c.ctl->pass_n[xb] = -1;
    mbar_arrive(&c.xfull[xb]);
}

// A pass as the consumers see it.
struct WsPass {
    int beg, base, n, tile0;
};

// Consumers: waits for pass q's descriptor and activations; false (for all
// consumer warps alike) when there is no more work or a wait timed out.
__device__ __forceinline__ bool ws_next_pass(WsCtx& c, int q, uint32_t* err, WsPass& d) {
    const int xb = q % c.P.XB;
    bool ok = __all_sync(0xffffffffu, ws_wait(c, &c.xfull[xb], (q / c.P.XB) & 1, err));
    if (ok) {
        d.beg = c.ctl->pass_beg[xb];
        d.base = c.ctl->pass_base[xb];
        d.n = c.ctl->pass_n[xb];
        d.tile0 = c.ctl->pass_tile0[xb];
    }
    ok = ok && d.n > 0 && !c.ctl->abort;
    return ws_consumers_all(ok);
}

// The last CTA to finish resets the unit counter for the next launch.
__device__ __forceinline__ void ws_retire(unsigned* ctr) {
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(ctr + 1, 1u) == gridDim.x - 1) {
            ctr[0] = 0u;
            ctr[1] = 0u;
            __threadfence();
        }
    }
}

// A fragment of rows 16*half + {g, g+8} of a tile record (m16n8k32 layout:
// a0 rows g / K 0-15, a1 rows g+8 / K 0-15, a2 rows g / K 16-31, a3 rows g+8 /
// K 16-31). q4_0: byte j of a row holds element j (low nibble) and j + 16
// (high), so one 16-byte row load gives both K halves.
template <int QT>
__device__ __forceinline__ void ws_a16(uint32_t (&a)[4], const uint8_t* rec, int half, int lane) {
    constexpr int QB = QFmt<QT>::QB;
    if (QT == 0) {
        uint32_t w[2];
        ldsm_x2(w, rec + (half * 16 + (lane & 15)) * QB);
        a[0] = w[0] & 0x0F0F0F0Fu;
        a[1] = w[1] & 0x0F0F0F0Fu;
        a[2] = (w[0] >> 4) & 0x0F0F0F0Fu;
        a[3] = (w[1] >> 4) & 0x0F0F0F0Fu;
    } else {
        ldsm_x4(a, rec + (half * 16 + (lane & 15)) * QB + (lane >> 4) * 16);
    }
}

__device__ __forceinline__ float ws_scale(const uint8_t* rec, int QB, int row) {
    return half_bits_to_float(*reinterpret_cast<const uint16_t*>(rec + kTileRows * QB + row * 2));
}

// Packed f32 pairs (sm_100 f32x2 arithmetic; .rn, one IEEE rounding per
// lane). A packed multiply feeding a packed add can be fused into one
// rounding by the compiler, so the running sums stay scalar adds: measured on
// B200, mul.rn.f32x2 and sub.rn.f32x2 chains equal their scalar __fmul_rn /
// __fsub_rn versions bit for bit, a mul2 -> add2 chain does not.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// acc[i][j] += (w_scale(row i) * x_scale(token j)) * isum, for the lane's
// rows {r0, r1} and tokens {2t, 2t+1}; d from the MMA (biased by kMagicI):
// the same three roundings per product and one per sum as
// fadd(acc, fmul(fmul(w, xs), fsub(d, kMagicF))). xs01 = {xs(2t), xs(2t+1)}.
__device__ __forceinline__ void ws_epilogue(float (&acc)[2][2], const int (&d)[4], float w0, float w1,
                                            uint64_t xs01) {
    const uint64_t magic = f2_pack(kMagicF, kMagicF);
    const uint64_t f0 = f2_sub(f2_pack(__int_as_float(d[0]), __int_as_float(d[1])), magic);
    const uint64_t f1 = f2_sub(f2_pack(__int_as_float(d[2]), __int_as_float(d[3])), magic);
    const uint64_t q0 = f2_mul(f2_mul(f2_pack(w0, w0), xs01), f0);
    const uint64_t q1 = f2_mul(f2_mul(f2_pack(w1, w1), xs01), f1);
    float a, b, c, e;
    f2_unpack(q0, a, b);
    f2_unpack(q1, c, e);
    acc[0][0] = fadd(acc[0][0], a);
    acc[0][1] = fadd(acc[0][1], b);
    acc[1][0] = fadd(acc[1][0], c);
    acc[1][1] = fadd(acc[1][1], e);
}

// ---------------------------------------------------------------------------
// gate/up
// ---------------------------------------------------------------------------
// ctr: two counters (units claimed, CTAs retired), zero at launch. NG token
// groups of 8 per pass: the A fragments and weight scales of a block are
// loaded once and feed NG pairs of MMAs. The library builds NG = 1: wider
// passes stream each weight tile once for more tokens but need the shared
// memory of more CTAs per SM, and measured slower on B200 (Qwen3-30B layer,
// 512 tokens: 306 us gate/up at NG = 4 with two CTAs per SM, 253 us at
// NG = 2 with three, 248 us at NG = 1 with four).
template <int QT, int CPS, int NG>
__global__ void __launch_bounds__(kWsThreads, CPS)
    expert_gate_up_ws_kernel(const __grid_constant__ CUtensorMap map, ExpertArgs a, WsPlan P, unsigned* ctr) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int PR = kPassRows * NG;
    __shared__ float s_amax[2][2][PR];  // [tile][half][token]
    __shared__ int s_qsum[2][2][PR];
    constexpr int QB = QFmt<QT>::QB, REC = kTileRows * QFmt<QT>::BB, SB = kWsSB;
    constexpr unsigned FULL = 0xffffffffu;
    const int TI = a.I / kTileRows, nbh = a.H / kQK, nbph = aux_stride(nbh), nbpi = aux_stride(a.I / kQK);
    const int upe = TI / 2;
    const int n_units = *a.n_active * upe;
    WsCtx c;
    ws_setup(c, smem, P);
    const int k = a.k;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp == kWsConsumers) {
        if (lane == 0) {
            tma_prefetch_desc(&map);
            ws_produce<PR>(
                c, a, &map, n_units, upe, 2, ctr, nbh, 2, a.H, a.xq, a.xaux, nbph,
                [&](const WsUnit& U, int j) { return __ldcg(a.elist + U.beg + j) / k; },
                [&](const WsUnit& U, int bx) { return bx * TI + U.tile0; }, a.err);
        }
    } else {
        const int tw = warp >> 1, half = warp & 1, g = lane >> 2, t = lane & 3;
        const int r0 = half * 16 + g, r1 = r0 + 8;
        const int nst = (nbh + SB - 1) / SB;
        bool live = true;
        int gs = 0;
        WsPass d;
        for (int q = 0; ws_next_pass(c, q, a.err, d); q++) {
            const int base = d.base, n = d.n, xb = q % P.XB;
            // B fragment rows: token (lane & 7), K half (lane >> 3) & 1
            const int8_t* xrow = reinterpret_cast<const int8_t*>(c.xq + (size_t)xb * P.xq_bytes) +
                                 (lane & 7) * P.xstride + ((lane >> 3) & 1) * 16;
            const int2* xa = reinterpret_cast<const int2*>(c.xa + (size_t)xb * P.xa_bytes);
            const int2* a0row = xa + (2 * t) * P.astride;
            const int2* a1row = xa + (2 * t + 1) * P.astride;
            float ag[NG][2][2], au[NG][2][2];
#pragma unroll
            for (int gi = 0; gi < NG; gi++)
#pragma unroll
                for (int i = 0; i < 4; i++) (&ag[gi][0][0])[i] = (&au[gi][0][0])[i] = 0.0f;
            for (int s = 0; s < nst; s++, gs++) {
                const int slot = gs % P.S;
                live = live && __all_sync(FULL, ws_wait(c, &c.full[slot], (gs / P.S) & 1, a.err));
                if (live) {
                    const uint8_t* gst = c.ring + (size_t)slot * P.stage_bytes + (size_t)tw * SB * REC;
                    const uint8_t* ust = gst + P.box_bytes;
                    const int nblk = min(SB, nbh - s * SB);
                    auto block = [&](int bi) {
                        const int b = s * SB + bi;
                        const uint8_t* rg = gst + bi * REC;
                        const uint8_t* ru = ust + bi * REC;
                        uint32_t fg[4], fu[4];
                        ws_a16<QT>(fg, rg, half, lane);
                        ws_a16<QT>(fu, ru, half, lane);
                        const float wg0 = ws_scale(rg, QB, r0), wg1 = ws_scale(rg, QB, r1);
                        const float wu0 = ws_scale(ru, QB, r0), wu1 = ws_scale(ru, QB, r1);
#pragma unroll
                        for (int gi = 0; gi < NG; gi++) {
                            uint32_t bf[2];
                            ldsm_x2(bf, xrow + gi * kPassRows * P.xstride + b * kQK);
                            const int2 x0 = a0row[gi * kPassRows * P.astride + b];
                            const int2 x1 = a1row[gi * kPassRows * P.astride + b];
                            const int c0 = ((QT == 0) ? x0.y : 0) + kMagicI, c1 = ((QT == 0) ? x1.y : 0) + kMagicI;
                            int dg[4], du[4];
                            mma_s8_16832(dg, fg, bf[0], bf[1], c0, c1);
                            mma_s8_16832(du, fu, bf[0], bf[1], c0, c1);
                            const uint64_t xs01 = f2_pack(__int_as_float(x0.x), __int_as_float(x1.x));
                            ws_epilogue(ag[gi], dg, wg0, wg1, xs01);
                            ws_epilogue(au[gi], du, wu0, wu1, xs01);
                        }
                    };
                    if (nblk == SB) {
#pragma unroll
                        for (int bi = 0; bi < SB; bi++) block(bi);
                    } else {
                        for (int bi = 0; bi < nblk; bi++) block(bi);
                    }
                }
                __syncwarp();
                if (lane == 0 && live) mbar_arrive(&c.empty[slot]);
            }
            __syncwarp();
            if (lane == 0 && live) mbar_arrive(&c.xempty[xb]);
            // h = silu(g) * u (expert/mod.rs:100-102) and its q8 quantization
            // per token over the tile's 32 rows (quant.rs:77-93)
            float h[NG][2][2], scale[NG][2];
            int qv[NG][2][2], qs[NG][2];
#pragma unroll
            for (int gi = 0; gi < NG; gi++) {
#pragma unroll
                for (int i = 0; i < 2; i++)
#pragma unroll
                    for (int j = 0; j < 2; j++) h[gi][i][j] = fmul(silu(ag[gi][i][j]), au[gi][i][j]);
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    float m = fmaxf(fmaxf(0.0f, fabsf(h[gi][0][j])), fabsf(h[gi][1][j]));
#pragma unroll
                    for (int o = 4; o < 32; o <<= 1) m = fmaxf(m, __shfl_xor_sync(FULL, m, o));
                    scale[gi][j] = m;  // this warp's 16-row amax, for now
                    if (g == 0) s_amax[tw][half][gi * kPassRows + 2 * t + j] = m;
                }
            }
            ws_sync_pair(tw);
#pragma unroll
            for (int gi = 0; gi < NG; gi++)
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    const float amax = fmaxf(scale[gi][j], s_amax[tw][half ^ 1][gi * kPassRows + 2 * t + j]);
                    scale[gi][j] = fdiv(amax, 127.0f);
                    const float inv = scale[gi][j] > 0.0f ? fdiv(1.0f, scale[gi][j]) : 0.0f;
                    qv[gi][0][j] = sat_i8(roundf(fmul(h[gi][0][j], inv)));
                    qv[gi][1][j] = sat_i8(roundf(fmul(h[gi][1][j], inv)));
                    int sq = qv[gi][0][j] + qv[gi][1][j];
#pragma unroll
                    for (int o = 4; o < 32; o <<= 1) sq += __shfl_xor_sync(FULL, sq, o);
                    qs[gi][j] = sq;
                    if (g == 0) s_qsum[tw][half][gi * kPassRows + 2 * t + j] = sq;
                }
            ws_sync_pair(tw);
            if (live) {
                const int itile = d.tile0 + tw;
#pragma unroll
                for (int gi = 0; gi < NG; gi++)
#pragma unroll
                    for (int j = 0; j < 2; j++) {
                        const int tok = gi * kPassRows + 2 * t + j;
                        if (tok < n) {
                            const size_t slot = (size_t)d.beg + base + tok;
                            int8_t* hrow = a.hq + slot * a.I + itile * kTileRows;
                            hrow[r0] = (int8_t)qv[gi][0][j];
                            hrow[r1] = (int8_t)qv[gi][1][j];
                            if (g == 0 && half == 0)
                                a.haux[slot * nbpi + itile] =
                                    make_int2(__float_as_int(scale[gi][j]), -8 * (qs[gi][j] + s_qsum[tw][1][tok]));
                        }
                    }
            }
        }
    }
    ws_teardown(c);
    ws_retire(ctr);
}

// ---------------------------------------------------------------------------
// down + best-first combine
// ---------------------------------------------------------------------------
template <int QT, int CPS, int NG>
__global__ void __launch_bounds__(kWsThreads, CPS)
    expert_down_ws_kernel(const __grid_constant__ CUtensorMap map, ExpertArgs a, WsPlan P, unsigned* ctr) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int PR = kPassRows * NG;
    __shared__ int s_last[2][PR];
    constexpr int QB = QFmt<QT>::QB, REC = kTileRows * QFmt<QT>::BB, SB = kWsSB;
    constexpr unsigned FULL = 0xffffffffu;
    const int TH = a.H / kTileRows, nbi = a.I / kQK, nbpi = aux_stride(nbi);
    const int upe = TH / 4;
    const int n_units = *a.n_active * upe;
    WsCtx c;
    ws_setup(c, smem, P);
    const int k = a.k;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp == kWsConsumers) {
        if (lane == 0) {
            tma_prefetch_desc(&map);
            ws_produce<PR>(
                c, a, &map, n_units, upe, 4, ctr, nbi, 1, a.I, a.hq, a.haux, nbpi,
                [&](const WsUnit& U, int j) { return U.beg + j; }, [&](const WsUnit& U, int) { return U.tile0; },
                a.err);
        }
    } else {
        const int g = lane >> 2, t = lane & 3, ct = threadIdx.x;  // ct: 0 .. 127
        const int nst = (nbi + SB - 1) / SB;
        bool live = true;
        int gs = 0;
        WsPass d;
        for (int q = 0; ws_next_pass(c, q, a.err, d); q++) {
            const int base = d.base, n = d.n, xb = q % P.XB;
            const int grp = d.tile0 / 4;
            const int* routes = a.elist + d.beg + base;
            // route ids of this lane's y rows (tokens gi*8 + 2t + j) and of the
            // combine thread's token, loaded ahead of the stage loop
            int rt[NG][2];
#pragma unroll
            for (int gi = 0; gi < NG; gi++)
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    const int tok = gi * kPassRows + 2 * t + j;
                    rt[gi][j] = tok < n ? __ldcg(routes + tok) : 0;
                }
            const int rct = ct < n ? __ldcg(routes + ct) : 0;
            const int8_t* xrow = reinterpret_cast<const int8_t*>(c.xq + (size_t)xb * P.xq_bytes) +
                                 (lane & 7) * P.xstride + ((lane >> 3) & 1) * 16;
            const int2* xa = reinterpret_cast<const int2*>(c.xa + (size_t)xb * P.xa_bytes);
            const int2* a0row = xa + (2 * t) * P.astride;
            const int2* a1row = xa + (2 * t + 1) * P.astride;
            float acc[NG][2][2][2];  // [group][16-row half][row g / g+8][token 2t / 2t+1]
#pragma unroll
            for (int i = 0; i < NG * 8; i++) (&acc[0][0][0][0])[i] = 0.0f;
            for (int s = 0; s < nst; s++, gs++) {
                const int slot = gs % P.S;
                live = live && __all_sync(FULL, ws_wait(c, &c.full[slot], (gs / P.S) & 1, a.err));
                if (live) {
                    const uint8_t* st = c.ring + (size_t)slot * P.stage_bytes + (size_t)warp * SB * REC;
                    const int nblk = min(SB, nbi - s * SB);
                    auto block = [&](int bi) {
                        const int b = s * SB + bi;
                        const uint8_t* rec = st + bi * REC;
                        uint32_t fr[2][4];
                        if (QT == 0) {
                            // words t of rows g, g+8, g+16, g+24
                            uint32_t w4[4];
                            ldsm_x4(w4, rec + lane * QB);
#pragma unroll
                            for (int mt = 0; mt < 2; mt++) {
                                fr[mt][0] = w4[2 * mt] & 0x0F0F0F0Fu;
                                fr[mt][1] = w4[2 * mt + 1] & 0x0F0F0F0Fu;
                                fr[mt][2] = (w4[2 * mt] >> 4) & 0x0F0F0F0Fu;
                                fr[mt][3] = (w4[2 * mt + 1] >> 4) & 0x0F0F0F0Fu;
                            }
                        } else {
                            ws_a16<QT>(fr[0], rec, 0, lane);
                            ws_a16<QT>(fr[1], rec, 1, lane);
                        }
                        float wsc[2][2];
#pragma unroll
                        for (int mt = 0; mt < 2; mt++) {
                            wsc[mt][0] = ws_scale(rec, QB, mt * 16 + g);
                            wsc[mt][1] = ws_scale(rec, QB, mt * 16 + 8 + g);
                        }
#pragma unroll
                        for (int gi = 0; gi < NG; gi++) {
                            uint32_t bf[2];
                            ldsm_x2(bf, xrow + gi * kPassRows * P.xstride + b * kQK);
                            const int2 x0 = a0row[gi * kPassRows * P.astride + b];
                            const int2 x1 = a1row[gi * kPassRows * P.astride + b];
                            const int c0 = ((QT == 0) ? x0.y : 0) + kMagicI, c1 = ((QT == 0) ? x1.y : 0) + kMagicI;
                            const uint64_t xs01 = f2_pack(__int_as_float(x0.x), __int_as_float(x1.x));
#pragma unroll
                            for (int mt = 0; mt < 2; mt++) {
                                int dd[4];
                                mma_s8_16832(dd, fr[mt], bf[0], bf[1], c0, c1);
                                ws_epilogue(acc[gi][mt], dd, wsc[mt][0], wsc[mt][1], xs01);
                            }
                        }
                    };
                    if (nblk == SB) {
#pragma unroll
                        for (int bi = 0; bi < SB; bi++) block(bi);
                    } else {
                        for (int bi = 0; bi < nblk; bi++) block(bi);
                    }
                }
                __syncwarp();
                if (lane == 0 && live) mbar_arrive(&c.empty[slot]);
            }
            __syncwarp();
            if (lane == 0 && live) mbar_arrive(&c.xempty[xb]);
            if (live) {
#pragma unroll
                for (int gi = 0; gi < NG; gi++)
#pragma unroll
                    for (int j = 0; j < 2; j++) {
                        const int tok = gi * kPassRows + 2 * t + j;
                        if (tok < n) {
                            float* yrow = a.ybuf + (size_t)rt[gi][j] * a.H + (d.tile0 + warp) * kTileRows;
#pragma unroll
                            for (int mt = 0; mt < 2; mt++) {
                                yrow[mt * 16 + g] = acc[gi][mt][0][j];
                                yrow[mt * 16 + 8 + g] = acc[gi][mt][1][j];
                            }
                        }
                    }
            }
            ws_sync_consumers();  // every y row of the pass is written
            // the last of a token's k routes to land for this 128-row group
            // combines them best-first (moe.rs:63-68)
            int* last = s_last[q & 1];
            if (ct < n) {
                last[ct] = 0;
                if (live) {
                    const int tok = rct / k;
                    unsigned* cnt = a.comb_cnt + (size_t)tok * upe + grp;
                    if (atomic_add_acq_rel(cnt, 1u) == (unsigned)(k - 1)) {
                        last[ct] = 1;
                        *cnt = 0u;
                    }
                }
            }
            ws_sync_consumers();
            for (int j = 0; j < n; j++) {
                if (!last[j]) continue;
                const int tok = __ldcg(routes + j) / k;
                const size_t col = (size_t)d.tile0 * kTileRows + ct;
                float o = 0.0f;
                for (int s2 = 0; s2 < k; s2++) {
                    const float w = __ldcg(a.topk_w + (size_t)tok * k + s2);
                    const float y = __ldcg(a.ybuf + ((size_t)tok * k + s2) * a.H + col);
                    o = fadd(o, fmul(w, y));
                }
                float* orow = out_row(a, tok);
                if (orow) orow[col] = o;
            }
        }
    }
    ws_teardown(c);
    ws_retire(ctr);
}

}  // namespace hale
