// hale_token.cuh -- the MoE layer of one token (batch-1 decode) in one launch.
//
// MoeLayer::forward (src/model/moe.rs:56-70) for a single token: router
// logits (src/model/moe.rs:33-54 via WeightMatrix::matvec), softmax + top-k
// (src/ops/softmax.rs, src/ops/topk.rs:27-35), Expert::forward of the k
// chosen experts (src/expert/mod.rs:91-103) and the best-first combine. Every
// f32 operation is the one router_kernel / expert_gate_up_kernel /
// expert_down_kernel perform, in the same order, so the output, the top-k
// indices and weights are bit-identical to that three-launch path.
//
// At one token those three launches are latency-bound: each moves a few MB
// behind its own ramp-up and drain, and the experts' bytes can only be
// requested once the previous launch has finished. Here one grid, never
// larger than the number of CTAs the GPU holds at once (the host sizes it
// from the occupancy), runs all phases with two grid-wide barriers:
//   A  every CTA stages x and its router rows in shared memory (with
//      norm_w, x = rmsnorm(x + delta): the residual add and RMSNorm in front
//      of the layer, the sum of squares on one thread) and quantizes x for
//      itself; 8-lane groups chain the router logits
//   -- barrier 1 --
//   B  every CTA repeats softmax + top-k over the E logits (the same inputs
//      and operations give the same result everywhere), then issues L2
//      prefetches for its share of the chosen experts' down projections, so
//      those bytes are in flight while the gate/up phase runs
//   C  gate/up units (top-k slot, 32-row tile): 8 warps stream the gate and
//      up tiles by bulk copies (a quarter of the blocks each), form every
//      (row, block) product (ws * xs) * isum in parallel, then one thread per
//      row adds them in block order; h = silu(g) * u and its q8 block
//   -- barrier 2 --
//   D  down units of 8 output rows over all k slots: the products in
//      parallel, the per-(slot, row) sums in block order, then the combine
//      out = sum_s w_s * y_s in top-k order
// Barrier waits are bounded; a wait that runs out raises kErrTimeout and the
// CTA leaves (the host's error check then resets the counters).
#pragma once

#include "hale_kernels.cuh"

// Phase marks for timing probes built from this header; empty in the library.
#ifndef HALE_TOK_MARK
#define HALE_TOK_MARK(i)
#endif

namespace hale {

constexpr int kTokThreads = 256;
constexpr int kTokWarps = kTokThreads / 32;
constexpr int kTokDownRows = 8;            // output rows per down unit
constexpr int kTokChunk = 8;               // blocks per gate/up bulk copy
constexpr uint32_t kTokPrefetch = 16384;   // bytes per L2 prefetch
constexpr int kTokDownLoads = 8;           // down products per thread with loads in flight
constexpr int kTokNormVec = 4;             // float4 of x per thread with the norm folded in (H <= 4096)

struct TokenArgs {
    const void* router;        // [E, H] f32 / f16 / bf16, row-major
    int E, H, I, k, normalize;
    const float* x;            // [H]
    float* logits;             // [E]
    int* topk_idx;             // [k]
    float* topk_w;             // [k]
    int* user_idx;             // nullable [k]
    float* user_w;             // nullable [k]
    unsigned long long* routing_counts;  // nullable [E]
    const uint8_t* experts;    // the layer's E experts, each [gate tiles][up tiles][down tiles]
    size_t expert_stride;
    int8_t* hq;                // [k, I]
    int2* haux;                // [k, I / 32]
    float* out;                // [H]
    unsigned* bar;             // [3] grid barrier counters: 0 at entry, 0 again at exit
    int rpc;                   // router rows per CTA: ceil(E / gridDim.x), <= 32
    int prefetch_all;          // prefetch whole expert records (CTAs take several gate/up units)
    // optional RMSNorm in front of the layer (norm_w non-null): the layer's
    // input is rmsnorm(x + delta) with weights norm_w, and CTA 0 writes the
    // new residual x + delta to x_out (not x: every CTA reads x)
    const float* delta;
    const float* norm_w;
    float eps;
    float* x_out;
    uint32_t* err;
};

// Shared-memory plan (bytes from the dynamic base), the same on host and device.
struct TokPlan {
    int xf, xq, xa, stage, terms, bars, total;
};

__host__ __device__ inline int tok_max(int a, int b) { return a > b ? a : b; }

__host__ __device__ inline TokPlan tok_plan(int BB, int wb, int H, int I, int k, int rpc) {
    TokPlan p;
    const int nbh = H / kQK, nbi = I / kQK;
    int o = 0;
    auto take = [&](int bytes) {
        const int at = o;
        o = (o + bytes + 127) & ~127;
        return at;
    };
    p.xf = take(H * 4);
    p.xq = take(H);
    p.xa = take(nbh * 8);
    // phase A: router rows; phase C: two copy slots per warp; phase D: h rows
    const int ring = kTokWarps * 2 * kTokChunk * kTileRows * BB;
    p.stage = take(tok_max(ring, tok_max(rpc * H * wb, k * I + k * nbi * 8)));
    // phase C: products [2][nbh][32] + sums [2][32]; phase D: products
    // [k][nbi][8] + sums [k][8]
    p.terms = take(tok_max(2 * nbh * kTileRows * 4 + 2 * kTileRows * 4,
                           k * nbi * kTokDownRows * 4 + k * kTokDownRows * 4));
    p.bars = take(kTokWarps * 2 * 8);
    p.total = o;
    return p;
}

#ifdef __CUDACC__
__device__ __forceinline__ unsigned tok_ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned tok_add_acq_rel(unsigned* p, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// Requests `bytes` (a multiple of 16, 16-byte aligned) into L2 without
// waiting for them.
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Grid-wide barrier on a counter that is 0 when the launch starts: after a
// CTA barrier, thread 0 publishes the CTA's writes (fence.acq_rel + relaxed
// add), then polls with acquire loads (bounded, ~1 s) until all gridDim.x
// CTAs have arrived. Returns false (the same verdict in every thread of the
// CTA) if the wait ran out.
__device__ __forceinline__ bool tok_grid_sync(unsigned* cnt, uint32_t* err, int* s_ok) {
    __syncthreads();
    if (threadIdx.x == 0) {
        asm volatile("fence.acq_rel.gpu;\n\tred.relaxed.gpu.global.add.u32 [%0], 1;" ::"l"(cnt) : "memory");
        int ok = 1;
        const long long t0 = clock64();
        while (tok_ld_acquire(cnt) < gridDim.x) {
            if (clock64() - t0 > (1LL << 31)) {
                raise_error(err, kErrTimeout);
                ok = 0;
                break;
            }
        }
        *s_ok = ok;
    }
    __syncthreads();
    return *s_ok != 0;
}

// Integer block sum of one quantized weight row block (lane's 16 nibble bytes
// or 32 quant bytes at wrow) against a q8 activation block xb (shared
// memory); for q4_0 the sum starts at the block's -8 * sum(x), as in tile_dot.
template <int QT>
__device__ __forceinline__ int tok_block_sum(const uint4* w4, const int8_t* xb, int c0) {
    int w[8];
    if (QT == 0) {
        const uint4 nib = w4[0];
        w[0] = nib.x & 0x0F0F0F0F;
        w[1] = nib.y & 0x0F0F0F0F;
        w[2] = nib.z & 0x0F0F0F0F;
        w[3] = nib.w & 0x0F0F0F0F;
        w[4] = (nib.x >> 4) & 0x0F0F0F0F;
        w[5] = (nib.y >> 4) & 0x0F0F0F0F;
        w[6] = (nib.z >> 4) & 0x0F0F0F0F;
        w[7] = (nib.w >> 4) & 0x0F0F0F0F;
    } else {
        const uint4 q0 = w4[0], q1 = w4[1];
        w[0] = q0.x; w[1] = q0.y; w[2] = q0.z; w[3] = q0.w;
        w[4] = q1.x; w[5] = q1.y; w[6] = q1.z; w[7] = q1.w;
    }
    const uint4 xa = reinterpret_cast<const uint4*>(xb)[0];
    const uint4 xc = reinterpret_cast<const uint4*>(xb)[1];
    int s0 = (QT == 0) ? c0 : 0, s1 = 0;
    s0 = __dp4a(w[0], (int)xa.x, s0);
    s1 = __dp4a(w[4], (int)xc.x, s1);
    s0 = __dp4a(w[1], (int)xa.y, s0);
    s1 = __dp4a(w[5], (int)xc.y, s1);
    s0 = __dp4a(w[2], (int)xa.z, s0);
    s1 = __dp4a(w[6], (int)xc.z, s1);
    s0 = __dp4a(w[3], (int)xa.w, s0);
    s1 = __dp4a(w[7], (int)xc.w, s1);
    return s0 + s1;
}

template <int QT, int DT>
__global__ void __launch_bounds__(kTokThreads, 2) moe_token_kernel(TokenArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t s_tab[32];
    __shared__ __align__(16) float s_e[256];
    __shared__ int s_sel[32];
    __shared__ float s_w[32];
    __shared__ int s_ok;
    constexpr int BB = QFmt<QT>::BB, QB = QFmt<QT>::QB, REC = kTileRows * BB;
    constexpr int wb = DT == 0 ? 4 : 2;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, c = blockIdx.x;
    const int H = a.H, I = a.I, E = a.E, k = a.k;
    const int nbh = H / kQK, nbi = I / kQK, TI = I / kTileRows;
    const TokPlan P = tok_plan(BB, wb, H, I, k, a.rpc);
    float* xf = reinterpret_cast<float*>(smem + P.xf);
    int8_t* xq = reinterpret_cast<int8_t*>(smem + P.xq);
    int2* xa = reinterpret_cast<int2*>(smem + P.xa);
    uint8_t* stage = smem + P.stage;
    float* terms = reinterpret_cast<float*>(smem + P.terms);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + P.bars);
    if (tid < 32) s_tab[tid] = kExp2TabDev[tid];
    if (tid < kTokWarps * 2) {
        mbar_init(&bars[tid], 1);
        fence_mbar_init();
    }

    HALE_TOK_MARK(0);
    // ---- A: x, router rows, q8 of x, logits ---------------------------------
    float4 nwv[kTokNormVec];  // this thread's norm weights (norm_w only)
    {
        const float4* x4 = reinterpret_cast<const float4*>(a.x);
        if (a.norm_w) {
            // v = x + delta (the residual add folded into RmsNorm's caller);
            // x, delta and the norm weights requested together, before the
            // router rows (H / 4 <= kTokNormVec * kTokThreads)
            const float4* d4 = reinterpret_cast<const float4*>(a.delta);
            const float4* w4 = reinterpret_cast<const float4*>(a.norm_w);
            float4 xv[kTokNormVec], dv[kTokNormVec];
#pragma unroll
            for (int j = 0; j < kTokNormVec; j++) {
                const int i = tid + j * kTokThreads;
                if (i < H / 4) {
                    xv[j] = __ldg(x4 + i);
                    dv[j] = __ldg(d4 + i);
                    nwv[j] = __ldg(w4 + i);
                }
            }
#pragma unroll
            for (int j = 0; j < kTokNormVec; j++) {
                const int i = tid + j * kTokThreads;
                if (i < H / 4) {
                    const float4 v = make_float4(fadd(xv[j].x, dv[j].x), fadd(xv[j].y, dv[j].y),
                                                 fadd(xv[j].z, dv[j].z), fadd(xv[j].w, dv[j].w));
                    reinterpret_cast<float4*>(xf)[i] = v;
                    if (c == 0) reinterpret_cast<float4*>(a.x_out)[i] = v;
                }
            }
        } else {
            for (int i = tid; i < H / 4; i += kTokThreads) reinterpret_cast<float4*>(xf)[i] = __ldg(x4 + i);
        }
        const int rowv = H * wb / 16;
        for (int r = 0; r < a.rpc; r++) {
            const int e = c + G * r;
            if (e >= E) break;
            const uint4* src =
                reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(a.router) + (size_t)e * H * wb);
            uint4* dst = reinterpret_cast<uint4*>(stage + (size_t)r * H * wb);
            for (int i = tid; i < rowv; i += kTokThreads) dst[i] = __ldg(src + i);
        }
    }
    __syncthreads();
    if (a.norm_w) {
        // RmsNorm::forward (norm.rs): the sum of squares left to right from
        // -0 on one thread (each square formed as the chain reaches it), then
        // x = v * (1 / sqrt(ss / H + eps)) * w
        __shared__ float s_scale;
        if (tid == 0) {
            float ss = -0.0f;
            const float4* v4 = reinterpret_cast<const float4*>(xf);
#pragma unroll 8
            for (int i = 0; i < H / 4; i++) {
                const float4 v = v4[i];
                ss = fadd(fadd(fadd(fadd(ss, fmul(v.x, v.x)), fmul(v.y, v.y)), fmul(v.z, v.z)), fmul(v.w, v.w));
            }
            s_scale = fdiv(1.0f, __fsqrt_rn(fadd(fdiv(ss, (float)H), a.eps)));
        }
        __syncthreads();
        const float scale = s_scale;
#pragma unroll
        for (int j = 0; j < kTokNormVec; j++) {
            const int i = tid + j * kTokThreads;
            if (i < H / 4) {
                float4* p4 = reinterpret_cast<float4*>(xf) + i;
                const float4 v = *p4;
                *p4 = make_float4(fmul(fmul(v.x, scale), nwv[j].x), fmul(fmul(v.y, scale), nwv[j].y),
                                  fmul(fmul(v.z, scale), nwv[j].z), fmul(fmul(v.w, scale), nwv[j].w));
            }
        }
        __syncthreads();
    }
    HALE_TOK_MARK(1);
    // Q8Activations::quantize (quant.rs:77-93), each CTA for its own use, on
    // warps 2.. first so that warp 0 starts the logit chains at once
    for (int b = (tid + kTokThreads - 64) % kTokThreads; b < nbh; b += kTokThreads) {
        float sc;
        int sm;
        quantize_block<true>(xf + b * kQK, xq + b * kQK, &sc, &sm);
        xa[b] = make_int2(__float_as_int(sc), -8 * sm);
    }
    {
        // the router's 8 accumulator lanes per logit, then reduce() and the
        // (empty, H % 8 == 0) tail, as router_kernel
        const int g = tid >> 3, lane8 = tid & 7;
        const int e = c + G * g;
        const bool valid = g < a.rpc && e < E;
        float acc = 0.0f;
        if (valid) {
            // operands of 16 chain steps into registers, then the 16 steps
            const uint8_t* row = stage + (size_t)g * H * wb;
            const int steps = H / 8;
            int i = 0;
            for (; i + 16 <= steps; i += 16) {
                float wv[16], xv[16];
#pragma unroll
                for (int u = 0; u < 16; u++) {
                    wv[u] = smem_w<DT>(row, 8 * (i + u) + lane8);
                    xv[u] = xf[8 * (i + u) + lane8];
                }
#pragma unroll
                for (int u = 0; u < 16; u++) acc = fadd(acc, fmul(wv[u], xv[u]));
            }
            for (; i < steps; i++) acc = fadd(acc, fmul(smem_w<DT>(row, 8 * i + lane8), xf[8 * i + lane8]));
        }
        const float s = fadd(acc, __shfl_down_sync(0xffffffffu, acc, 4, 8));
        const float p = fadd(s, __shfl_down_sync(0xffffffffu, s, 1, 8));
        const float r = fadd(p, __shfl_down_sync(0xffffffffu, p, 2, 8));
        if (valid && lane8 == 0) a.logits[e] = fadd(r, -0.0f);
    }
    HALE_TOK_MARK(2);
    if (!tok_grid_sync(&a.bar[0], a.err, &s_ok)) return;
    HALE_TOK_MARK(3);

    // ---- B: softmax + top-k (every CTA), L2 prefetch -------------------------
    if (warp == 0) {
        float lv[8];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int i = lane + 32 * j;
            lv[j] = i < E ? __ldcg(a.logits + i) : -__int_as_float(0x7f800000);
        }
        float mx = lv[0];
#pragma unroll
        for (int j = 1; j < 8; j++) mx = fmaxf(mx, lv[j]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int i = lane + 32 * j;
            if (i < E) s_e[i] = hale_expf_tab(fsub(lv[j], mx), s_tab);
        }
        __syncwarp();
        float sum = 0.0f;
        if (lane == 0) {
            int i = 0;
            for (; i + 4 <= E; i += 4) {
                const float4 q4 = *reinterpret_cast<const float4*>(&s_e[i]);
                sum = fadd(fadd(fadd(fadd(sum, q4.x), q4.y), q4.z), q4.w);
            }
            for (; i < E; i++) sum = fadd(sum, s_e[i]);
        }
        sum = __shfl_sync(0xffffffffu, sum, 0);
        __syncwarp();
        for (int i = lane; i < E; i += 32) s_e[i] = fdiv(s_e[i], sum);
        __syncwarp();
        unsigned ukey[8];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int i = lane + 32 * j;
            ukey[j] = i < E ? ((unsigned)total_key(s_e[i]) ^ 0x80000000u) : 0u;
        }
        unsigned taken = 0u;
        float chosen_score = 0.0f;
        int chosen_idx = -1;
        float norm = -0.0f;
        for (int kk = 0; kk < k; kk++) {
            unsigned bk = 0u;
            int bj = -1;
#pragma unroll
            for (int j = 0; j < 8; j++)
                if (!(taken & (1u << j)) && lane + 32 * j < E && (bj < 0 || ukey[j] > bk)) { bk = ukey[j]; bj = j; }
            const unsigned wk = __reduce_max_sync(0xffffffffu, bj >= 0 ? bk : 0u);
            const unsigned mine = (bj >= 0 && bk == wk) ? (unsigned)(lane + 32 * bj) : 0xffffffffu;
            const int bi = (int)__reduce_min_sync(0xffffffffu, mine);
            if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
            const float sc = s_e[bi];
            norm = fadd(norm, sc);
            if (lane == kk) { chosen_score = sc; chosen_idx = bi; }
        }
        if (lane < k) {
            const float wv = a.normalize ? fdiv(chosen_score, norm) : fdiv(chosen_score, 1.0f);
            s_sel[lane] = chosen_idx;
            s_w[lane] = wv;
            if (c == 0) {
                a.topk_idx[lane] = chosen_idx;
                a.topk_w[lane] = wv;
                if (a.user_idx) a.user_idx[lane] = chosen_idx;
                if (a.user_w) a.user_w[lane] = wv;
                if (a.routing_counts) a.routing_counts[chosen_idx] += 1ull;
            }
        }
    }
    __syncthreads();
    HALE_TOK_MARK(4);
    const size_t tbh = (size_t)nbh * REC, tbd = (size_t)nbi * REC;
    const size_t down_off = (size_t)2 * TI * tbh;
    {
        // this CTA's share of the chosen experts' bytes, in kTokPrefetch pieces
        const size_t beg = a.prefetch_all ? 0 : down_off, span = a.expert_stride - beg;
        const int per = (int)((span + kTokPrefetch - 1) / kTokPrefetch);
        for (int pc = c + G * tid; pc < k * per; pc += G * kTokThreads) {
            const int s = pc / per;
            const size_t off = (size_t)(pc - s * per) * kTokPrefetch;
            const uint32_t n = (uint32_t)(span - off < kTokPrefetch ? span - off : kTokPrefetch);
            prefetch_l2_bulk(a.experts + (size_t)s_sel[s] * a.expert_stride + beg + off, n);
        }
    }

    HALE_TOK_MARK(5);
    // ---- C: gate/up units ----------------------------------------------------
    {
        const int m = warp >> 2, q = warp & 3;   // m: 0 gate, 1 up; q: quarter of the blocks
        const int nbq = nbh / 4;
        // a warp's blocks fit both slots: one copy; else a ring of 8-block chunks
        const int chb = nbq <= 2 * kTokChunk ? nbq : kTokChunk;
        const int nch = (nbq + chb - 1) / chb;
        uint8_t* wbuf = stage + (size_t)warp * 2 * kTokChunk * REC;
        uint64_t* wbar = bars + warp * 2;
        float* tg = terms;                        // [2][nbh][32]
        float* s_gu = terms + 2 * nbh * kTileRows; // [2][32]
        uint32_t ph = 0;
        for (int u = c; u < k * TI; u += G) {
            const int s = u / TI, t = u - s * TI;
            const uint8_t* src = a.experts + (size_t)s_sel[s] * a.expert_stride + (size_t)(m * TI + t) * tbh +
                                 (size_t)q * nbq * REC;
            auto issue = [&](int ch) {
                const int nb = min(chb, nbq - ch * chb);
                const int slot = ch & 1;
                mbar_arrive_expect_tx(&wbar[slot], (uint32_t)(nb * REC));
                bulk_g2s(wbuf + (size_t)slot * kTokChunk * REC, src + (size_t)ch * chb * REC, (uint32_t)(nb * REC),
                         &wbar[slot]);
            };
            if (lane == 0) {
                fence_proxy_async_smem();  // the stage held router rows / earlier chunks
                for (int ch = 0; ch < min(2, nch); ch++) issue(ch);
            }
            bool ok = true;
            for (int ch = 0; ch < nch; ch++) {
                const int slot = ch & 1;
                if (!__all_sync(0xffffffffu, mbar_wait(&wbar[slot], (ph >> slot) & 1u, a.err))) {
                    ok = false;
                    // copies already issued get a bounded chance to land
                    for (int c2 = ch; c2 < min(ch + 2, nch); c2++)
                        mbar_wait(&wbar[c2 & 1], (ph >> (c2 & 1)) & 1u, nullptr, 400000000LL);
                    break;
                }
                ph ^= 1u << slot;
                const uint8_t* sb = wbuf + (size_t)slot * kTokChunk * REC;
                const int nb = min(chb, nbq - ch * chb);
#pragma unroll 4
                for (int bi = 0; bi < nb; bi++) {
                    const int b = q * nbq + ch * chb + bi;
                    const uint8_t* rec = sb + bi * REC;
                    const float ws =
                        half_bits_to_float(*reinterpret_cast<const uint16_t*>(rec + kTileRows * QB + lane * 2));
                    const int2 ax = xa[b];
                    const int is = tok_block_sum<QT>(reinterpret_cast<const uint4*>(rec + lane * QB), xq + b * kQK,
                                                     ax.y);
                    tg[((size_t)m * nbh + b) * kTileRows + lane] =
                        fmul(fmul(ws, __int_as_float(ax.x)), __int2float_rn(is));
                }
                __syncwarp();
                if (ch + 2 < nch && lane == 0) {
                    fence_proxy_async_smem();
                    issue(ch + 2);
                }
            }
            if (!__syncthreads_and(ok ? 1 : 0)) return;
            if (tid < 2 * kTileRows) {
                // total += (ws * xs) * isum over the blocks in order (tile_dot)
                const float* col = tg + (size_t)(tid >> 5) * nbh * kTileRows + lane;
                float acc = 0.0f;
                for (int b = 0; b < nbh; b++) acc = fadd(acc, col[(size_t)b * kTileRows]);
                s_gu[tid] = acc;
            }
            __syncthreads();
            if (warp == 0) {
                // h = silu(g) * u (expert/mod.rs:100-102), then the 32 rows of
                // the tile as one q8 block (matrix.rs:119-121)
                const float h = fmul(silu(s_gu[lane]), s_gu[kTileRows + lane]);
                const float amax = warp_max_abs(h);
                const float scale = fdiv(amax, 127.0f);
                const float inv = scale > 0.0f ? fdiv(1.0f, scale) : 0.0f;
                const int qv = sat_i8(roundf(fmul(h, inv)));
                const int qs = warp_sum_int(qv);
                a.hq[(size_t)s * I + t * kTileRows + lane] = (int8_t)qv;
                if (lane == 0) a.haux[(size_t)s * nbi + t] = make_int2(__float_as_int(scale), -8 * qs);
            }
            __syncthreads();  // tg / s_gu are reused by the next unit
        }
    }
    HALE_TOK_MARK(6);
    if (!tok_grid_sync(&a.bar[1], a.err, &s_ok)) return;
    HALE_TOK_MARK(7);

    // ---- D: down units of kTokDownRows output rows over all k slots ----------
    const int units_d = H / kTokDownRows;
    if (c < units_d) {
        int8_t* hs = reinterpret_cast<int8_t*>(stage);
        int2* ha = reinterpret_cast<int2*>(stage + (size_t)k * I);
        float* dt = terms;                                   // [k][nbi][8]
        float* ys = terms + (size_t)k * nbi * kTokDownRows;  // [k][8]
        const int items = k * nbi * kTokDownRows;             // (slot, block, row) products
        bool staged = false;
        for (int u = c; u < units_d; u += G) {
            const int r0 = u * kTokDownRows;
            for (int base = 0; base < items; base += kTokDownLoads * kTokThreads) {
                // this thread's weight words first (L2 prefetched), then the
                // h rows (first group only), then the products
                uint4 wq[kTokDownLoads][QT == 1 ? 2 : 1];
                unsigned short wsb[kTokDownLoads];
#pragma unroll
                for (int j = 0; j < kTokDownLoads; j++) {
                    const int it = base + j * kTokThreads + tid;
                    if (it < items) {
                        const int rr = it % kTokDownRows, sb = it / kTokDownRows;
                        const int s = sb / nbi, b = sb - s * nbi;
                        const int r = r0 + rr, ri = r % kTileRows;
                        const uint8_t* rec = a.experts + (size_t)s_sel[s] * a.expert_stride + down_off +
                                             (size_t)(r / kTileRows) * tbd + (size_t)b * REC;
                        wsb[j] = __ldg(reinterpret_cast<const unsigned short*>(rec + kTileRows * QB) + ri);
                        wq[j][0] = __ldg(reinterpret_cast<const uint4*>(rec + ri * QB));
                        if (QT == 1) wq[j][QT] = __ldg(reinterpret_cast<const uint4*>(rec + ri * QB) + 1);
                    }
                }
                if (!staged) {
                    for (int i = tid; i < k * I / 16; i += kTokThreads)
                        reinterpret_cast<uint4*>(hs)[i] = __ldcg(reinterpret_cast<const uint4*>(a.hq) + i);
                    for (int i = tid; i < k * nbi; i += kTokThreads) ha[i] = __ldcg(a.haux + i);
                    __syncthreads();
                    HALE_TOK_MARK(8);
                    staged = true;
                }
#pragma unroll
                for (int j = 0; j < kTokDownLoads; j++) {
                    const int it = base + j * kTokThreads + tid;
                    if (it < items) {
                        const int sb = it / kTokDownRows;
                        const int s = sb / nbi, b = sb - s * nbi;
                        const int2 ax = ha[s * nbi + b];
                        const int is = tok_block_sum<QT>(wq[j], hs + (size_t)s * I + b * kQK, ax.y);
                        dt[it] = fmul(fmul(half_bits_to_float(wsb[j]), __int_as_float(ax.x)), __int2float_rn(is));
                    }
                }
            }
            __syncthreads();
            if (tid < k * kTokDownRows) {
                const float* col = dt + (size_t)(tid / kTokDownRows) * nbi * kTokDownRows + (tid % kTokDownRows);
                float y = 0.0f;
                for (int b = 0; b < nbi; b++) y = fadd(y, col[(size_t)b * kTokDownRows]);
                ys[tid] = y;
            }
            __syncthreads();
            if (tid < kTokDownRows) {
                // out = 0; out += w_s * y_s, s in top-k order (moe.rs:63-68)
                float o = 0.0f;
                for (int s = 0; s < k; s++) o = fadd(o, fmul(s_w[s], ys[s * kTokDownRows + tid]));
                a.out[r0 + tid] = o;
            }
            __syncthreads();
        }
    }
    __syncthreads();
    HALE_TOK_MARK(9);
    if (tid == 0) {
        if (tok_add_acq_rel(&a.bar[2], 1u) == (unsigned)G - 1) {
            // every CTA has passed both barriers: reset for the next launch
            a.bar[0] = 0u;
            a.bar[1] = 0u;
            a.bar[2] = 0u;
        }
    }
}
#endif  // __CUDACC__

}  // namespace hale
