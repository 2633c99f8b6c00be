// hale_attn.cuh -- attention of one decode row spread over the whole GPU.
//
// Attention::forward (attention.rs:59-85) for a single row, in exactly the
// order of attn_gqa_kernel (and the oracle): per query head
//   s_t  = (sum_i q_i k_ti from -0, i ascending) * scale
//   m    = max_t s_t;  e_t = exp(s_t - m);  sum = sum_t e_t from 0, t ascending
//   p_t  = e_t / sum;  ctx_i = sum_t p_t v_ti from 0, t ascending.
// The dependent chains are the score chains (head_dim steps), the denominator
// (seq steps) and each context element (seq steps). attn_gqa_kernel runs a
// head per CTA at one row, so 32 SMs hold the whole step and each pulls a KV
// head's cache through one SM. Here every chain keeps its order but the
// independent ones run on different SMs, in one grid of co-resident CTAs:
//   S  units (kv head, 32 positions): K rows staged in shared memory (with
//      `rope`, the q heads' norms and RoPE done here and the row's new k / v
//      appended to the cache by the unit holding its position), one thread
//      per (query head of the group, position) runs the score chain; scores
//      and each unit's per-head maximum go to global scratch
//   -- grid barrier --
//   P  one unit per query head: the maximum of the partial maxima, the exps,
//      the denominator chain on one thread, p_t = e_t / sum written over the
//      head's scores (positions in chunks of kSplitPC)
//   -- grid barrier --
//   C  units (kv head, 8 head dims): p of the group's heads and the V
//      columns staged in shared memory (chunks of split_chunk(G) positions);
//      all threads form the products p_t v_td, then one thread per (head,
//      dim) adds them in position order.
#pragma once

#include "hale_decoder.cuh"
#include "hale_token.cuh"

// Phase marks for timing probes built from this header; empty in the library.
#ifndef HALE_SPLIT_MARK
#define HALE_SPLIT_MARK(i)
#endif

namespace hale {

constexpr int kSplitPB = 32;   // positions per score unit
constexpr int kSplitD = 8;     // head dims per context unit
constexpr int kSplitPC = 2048; // positions per softmax chunk (one head)

// Positions per softmax / context chunk for G query heads per kv head.
__host__ __device__ inline int split_chunk(int G) {
    const int c = (8192 / G) & ~15;
    return c > 1024 ? 1024 : c;
}
// Row stride of the exps in shared memory: 4 floats of pad put the heads a
// warp's context threads read in different banks.
__host__ __device__ inline int split_es(int G) { return split_chunk(G) + 4; }

// Positions per product block of the context phase: the products p_t v_td
// of all G * kSplitD chains for this many positions sit in shared memory
// (about 64 KB) before the chains add them.
__host__ __device__ inline int split_ps(int G, int ch) {
    int ps = (16384 / (G * kSplitD)) & ~15;
    if (ps < 16) ps = 16;
    return ps > ch ? ch : ps;
}

struct SplitPlan {
    int q, k, e, v, pr, rt, total;  // float offsets in dynamic shared memory
};

__host__ __device__ inline SplitPlan split_plan(int G, int hd) {
    SplitPlan p;
    const int ch = split_chunk(G);
    p.q = 0;
    p.k = p.q + G * hd;
    p.e = p.k + kSplitPB * (hd + 4);
    p.v = p.e + (G * split_es(G) > kSplitPC ? G * split_es(G) : kSplitPC);
    p.pr = p.v + ch * kSplitD;
    p.rt = p.pr + G * kSplitD * (split_ps(G, ch) + 4);  // q / k norm weights, cos, sin at the position
    p.total = p.rt + 3 * hd;
    return p;
}

struct SplitArgs {
    const float* qkv;         // row: [nh | nkv | nkv] heads of hd (q after RoPE)
    int nh, nkv, hd;
    float* kcache;            // this layer's caches: [sequence][position][nkv * hd]
    float* vcache;
    const uint32_t* rows;     // [3]: token, position, sequence
    size_t seq_stride;
    float scale;
    float* sc;                // [nh][sc_stride] scores, then p (sc_stride >= max_len, a multiple of 4)
    float* pm;                // [nh][npm] per-unit maxima, npm = ceil(max_len / kSplitPB)
    int sc_stride, npm;
    float* ctx;               // [nh * hd]
    unsigned* bar;            // [3] grid barrier counters, 0 at entry and exit
    L2Prefetch pf;            // the next kernels' weights, pulled into L2 at the start
    // the row's q/k head RMSNorm + RoPE and the K/V cache append folded in
    // (qk_rope_kernel's work; rope non-zero): q heads are normed and rotated in
    // shared memory by every score unit of their group, the new position's k
    // and v rows by the unit that holds that position
    int rope;
    const float* q_norm;      // nullable: no q/k head norm
    const float* k_norm;
    float eps;
    const float* rope_cos;    // [max_len][hd / 2]
    const float* rope_sin;
    uint32_t* err;
};

// In-place head RMSNorm (when w) and RoPE of one head in shared memory, by one
// warp, as qk_rope_kernel: s = sum x_i^2 left to right from -0 (lane 0),
// x_i *= scale * w_i; then a' = a c - b s, b' = b c + a s on (i, i + hd/2).
__device__ __forceinline__ void split_head_rope(float* x, int hd, const float* w, float eps, const float* c,
                                                const float* sn, int lane) {
    const int half = hd / 2;
    if (w) {
        float scale = 0.0f;
        if (lane == 0) {
            float s = -0.0f;
            const float4* x4 = reinterpret_cast<const float4*>(x);
#pragma unroll 8
            for (int i = 0; i < hd / 4; i++) {
                const float4 v = x4[i];
                s = fadd(fadd(fadd(fadd(s, fmul(v.x, v.x)), fmul(v.y, v.y)), fmul(v.z, v.z)), fmul(v.w, v.w));
            }
            scale = fdiv(1.0f, __fsqrt_rn(fadd(fdiv(s, (float)hd), eps)));
        }
        scale = __shfl_sync(0xffffffffu, scale, 0);
        __syncwarp();
        for (int i = lane; i < hd; i += 32) x[i] = fmul(x[i], fmul(scale, w[i]));
        __syncwarp();
    }
    for (int i = lane; i < half; i += 32) {
        const float av = x[i], bv = x[half + i];
        x[i] = fsub(fmul(av, c[i]), fmul(bv, sn[i]));
        x[half + i] = fadd(fmul(bv, c[i]), fmul(av, sn[i]));
    }
    __syncwarp();
}

#ifdef __CUDACC__
__global__ void __launch_bounds__(256, 1) attn_split_kernel(SplitArgs a) {
    extern __shared__ __align__(16) float s_split[];
    __shared__ uint64_t s_tab[32];
    __shared__ float s_max[32], s_sum[32];
    __shared__ int s_ok;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nh = a.nh, nkv = a.nkv, hd = a.hd, G = nh / nkv, kvd = nkv * hd, q4n = hd >> 2;
    const int seq = (int)a.rows[1] + 1;
    const size_t sbase = (size_t)a.rows[2] * a.seq_stride;
    const SplitPlan P = split_plan(G, hd);
    float* sq = s_split + P.q;
    float* sk = s_split + P.k;
    float* se = s_split + P.e;
    float* sv = s_split + P.v;
    float* spr = s_split + P.pr;
    float* s_qn = s_split + P.rt;     // [hd]
    float* s_kn = s_qn + hd;          // [hd]
    float* s_rc = s_kn + hd;          // [hd / 2]
    float* s_rs = s_rc + hd / 2;      // [hd / 2]
    const int CH = split_chunk(G), ES = split_es(G), kp = hd + 4;
    if (tid < 32) s_tab[tid] = kExp2TabDev[tid];
    const float* qrow = a.qkv;
    const int npb = (seq + kSplitPB - 1) / kSplitPB;
    l2_prefetch_share(a.pf, blockIdx.x, gridDim.x);
    if (a.rope) {
        // the head norms' weights and the position's rotation, for every unit
        // (visible after the first unit's CTA barrier)
        const int half = hd / 2, pos = seq - 1;
        for (int i = tid; i < hd; i += 256) {
            s_qn[i] = a.q_norm ? a.q_norm[i] : 0.0f;
            s_kn[i] = a.k_norm ? a.k_norm[i] : 0.0f;
        }
        for (int i = tid; i < half; i += 256) {
            s_rc[i] = a.rope_cos[(size_t)pos * half + i];
            s_rs[i] = a.rope_sin[(size_t)pos * half + i];
        }
    }
    HALE_SPLIT_MARK(0);

    // ---- S: score chains ------------------------------------------------------
    for (int u = blockIdx.x; u < nkv * npb; u += gridDim.x) {
        const int h = u / npb, pb = u - h * npb;
        const int t0 = pb * kSplitPB, here = min(kSplitPB, seq - t0);
        const float* kb = a.kcache + sbase + (size_t)h * hd;
        // with the rope folded in, the row's own position (seq - 1, in the
        // last unit) is not in the cache yet: it is formed below
        const int cached = (a.rope && pb == npb - 1) ? here - 1 : here;
        for (int j = tid; j < cached * q4n; j += 256) {
            const int tt = j / q4n, c4 = j - tt * q4n;
            cp_async16(sk + tt * kp + 4 * c4, kb + (size_t)(t0 + tt) * kvd + 4 * c4);
        }
        cp_async_commit();
        for (int j = tid; j < G * q4n; j += 256)
            reinterpret_cast<float4*>(sq)[j] = reinterpret_cast<const float4*>(qrow + (size_t)h * G * hd)[j];
        if (a.rope) {
            // this kv head's new k row goes to the stage (and the cache), its v
            // row to the cache, on a warp with no q head if there is one
            const int pos = seq - 1, kw = G < 8 ? G : 7;
            float* kr = sk + (here - 1) * kp;
            if (cached < here && warp == kw) {
                const float* kraw = qrow + (size_t)(nh + h) * hd;
                const float* vraw = qrow + (size_t)(nh + nkv + h) * hd;
                float* vdst = a.vcache + sbase + (size_t)h * hd + (size_t)pos * kvd;
                for (int i = lane; i < hd; i += 32) {
                    kr[i] = kraw[i];
                    vdst[i] = vraw[i];
                }
            }
            __syncthreads();  // q, the k row and the tables staged
            for (int g = warp; g < G; g += 8)
                split_head_rope(sq + g * hd, hd, a.q_norm ? s_qn : nullptr, a.eps, s_rc, s_rs, lane);
            if (cached < here && warp == kw) {
                split_head_rope(kr, hd, a.k_norm ? s_kn : nullptr, a.eps, s_rc, s_rs, lane);
                float* kdst = a.kcache + sbase + (size_t)h * hd + (size_t)pos * kvd;
                for (int i = lane; i < hd; i += 32) kdst[i] = kr[i];
            }
        }
        cp_async_wait<0>();
        __syncthreads();
        for (int g = warp; g < G; g += 8) {
            float sv_ = -__int_as_float(0x7f800000);
            if (lane < here) {
                const float4* k4 = reinterpret_cast<const float4*>(sk + lane * kp);
                const float4* qv = reinterpret_cast<const float4*>(sq + g * hd);
                float acc = -0.0f;
                int i = 0;
                for (; i + 8 <= q4n; i += 8) {
                    float4 kb8[8], qb8[8];
#pragma unroll
                    for (int w = 0; w < 8; w++) {
                        kb8[w] = k4[i + w];
                        qb8[w] = qv[i + w];
                    }
#pragma unroll
                    for (int w = 0; w < 8; w++) {
                        acc = fadd(acc, fmul(qb8[w].x, kb8[w].x));
                        acc = fadd(acc, fmul(qb8[w].y, kb8[w].y));
                        acc = fadd(acc, fmul(qb8[w].z, kb8[w].z));
                        acc = fadd(acc, fmul(qb8[w].w, kb8[w].w));
                    }
                }
                for (; i < q4n; i++) {
                    const float4 k = k4[i], q = qv[i];
                    acc = fadd(acc, fmul(q.x, k.x));
                    acc = fadd(acc, fmul(q.y, k.y));
                    acc = fadd(acc, fmul(q.z, k.z));
                    acc = fadd(acc, fmul(q.w, k.w));
                }
                sv_ = fmul(acc, a.scale);
                a.sc[(size_t)(h * G + g) * a.sc_stride + t0 + lane] = sv_;
            }
            float m = sv_;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            if (lane == 0) a.pm[(size_t)(h * G + g) * a.npm + pb] = m;
        }
        __syncthreads();  // the next unit restages K and q
    }
    HALE_SPLIT_MARK(1);
    if (!tok_grid_sync(&a.bar[0], a.err, &s_ok)) return;
    HALE_SPLIT_MARK(2);

    // ---- P: softmax, one unit per query head ------------------------------------
    // p_t overwrites s_t in the head's score row (only this unit reads it)
    for (int u = blockIdx.x; u < nh; u += gridDim.x) {
        float* row = a.sc + (size_t)u * a.sc_stride;
        // the first chunk's scores are requested together with the partial
        // maxima (one L2 round trip, not two)
        float v0[8];
        const int here0 = min(kSplitPC, seq);
#pragma unroll
        for (int w = 0; w < 8; w++) {
            const int j = w * 256 + tid;
            if (j < here0) v0[w] = __ldcg(row + j);
        }
        if (warp == 0) {
            float m = -__int_as_float(0x7f800000);
            for (int i = lane; i < npb; i += 32) m = fmaxf(m, __ldcg(a.pm + (size_t)u * a.npm + i));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            if (lane == 0) s_max[0] = m;
        }
        __syncthreads();
        const float m = s_max[0];
        // exps of positions [t0, t0 + here) into se (a chunk's scores are 8
        // per thread, all requested before any is used)
        static_assert(kSplitPC == 8 * 256, "a softmax chunk is 8 scores per thread");
        auto exps_of = [&](const float (&v)[8], int here) {
#pragma unroll
            for (int w = 0; w < 8; w++) {
                const int j = w * 256 + tid;
                if (j < here) se[j] = hale_expf_tab(fsub(v[w], m), s_tab);
            }
        };
        auto exps = [&](int t0, int here) {
            if (t0 == 0) {
                exps_of(v0, here);
                return;
            }
            float v[8];
#pragma unroll
            for (int w = 0; w < 8; w++) {
                const int j = w * 256 + tid;
                if (j < here) v[w] = __ldcg(row + t0 + j);
            }
            exps_of(v, here);
        };
        const int nch = (seq + kSplitPC - 1) / kSplitPC;
        float sum = 0.0f;  // thread 0: the denominator, t ascending
        for (int ch = 0; ch < nch; ch++) {
            const int t0 = ch * kSplitPC, here = min(kSplitPC, seq - t0);
            exps(t0, here);
            __syncthreads();
            if (tid == 0) {
                int tt = 0;
                for (; tt + 16 <= here; tt += 16) {
                    const float4 e0 = reinterpret_cast<const float4*>(se + tt)[0];
                    const float4 e1 = reinterpret_cast<const float4*>(se + tt)[1];
                    const float4 e2 = reinterpret_cast<const float4*>(se + tt)[2];
                    const float4 e3 = reinterpret_cast<const float4*>(se + tt)[3];
                    sum = fadd(fadd(fadd(fadd(sum, e0.x), e0.y), e0.z), e0.w);
                    sum = fadd(fadd(fadd(fadd(sum, e1.x), e1.y), e1.z), e1.w);
                    sum = fadd(fadd(fadd(fadd(sum, e2.x), e2.y), e2.z), e2.w);
                    sum = fadd(fadd(fadd(fadd(sum, e3.x), e3.y), e3.z), e3.w);
                }
                for (; tt < here; tt++) sum = fadd(sum, se[tt]);
            }
            __syncthreads();
        }
        if (tid == 0) s_sum[0] = sum;
        __syncthreads();
        const float total = s_sum[0];
        for (int ch = 0; ch < nch; ch++) {
            const int t0 = ch * kSplitPC, here = min(kSplitPC, seq - t0);
            if (nch > 1) {
                exps(t0, here);  // the denominator pass left the last chunk in se
                __syncthreads();
            }
            for (int j = tid; j < here; j += 256) row[t0 + j] = fdiv(se[j], total);
            __syncthreads();
        }
    }
    HALE_SPLIT_MARK(3);
    if (!tok_grid_sync(&a.bar[1], a.err, &s_ok)) return;
    HALE_SPLIT_MARK(5);

    // ---- C: context chains, units (kv head, 8 head dims) ---------------------------
    const int nd = hd / kSplitD;
    const int nch = (seq + CH - 1) / CH;
    const int g = tid / kSplitD, dd = tid - g * kSplitD;
    const bool busy = g < G;  // thread tid runs chain tid = (head g, dim dd)
    // product threads: TPC per chain, thread (pc, pq) takes positions pq, pq + TPC, ...
    const int TPC = 256 / (G * kSplitD), PS = split_ps(G, CH), PR = PS + 4;
    const int pc = tid / TPC, pq = tid - pc * TPC;
    for (int u = blockIdx.x; u < nkv * nd; u += gridDim.x) {
        const int h = u / nd, d0 = (u - h * nd) * kSplitD;
        const float* vb = a.vcache + sbase + (size_t)h * hd + d0;
        const float* pg = a.sc + (size_t)h * G * a.sc_stride;
        float c = 0.0f;
        for (int ch = 0; ch < nch; ch++) {
            const int t0 = ch * CH, here = min(CH, seq - t0), h4 = (here + 3) >> 2;
            // p rows of the group's heads (16-byte copies; rows start 16-byte
            // aligned, the copy of the last partial 4 stays inside the row)
            for (int j = tid; j < G * h4; j += 256) {
                const int gg = j / h4, c4 = j - gg * h4;
                cp_async16(se + gg * ES + 4 * c4, pg + (size_t)gg * a.sc_stride + t0 + 4 * c4);
            }
            for (int j = tid; j < here * (kSplitD / 4); j += 256) {
                const int tt = j / (kSplitD / 4), c4 = j - tt * (kSplitD / 4);
                cp_async16(sv + tt * kSplitD + 4 * c4, vb + (size_t)(t0 + tt) * kvd + 4 * c4);
            }
            cp_async_commit();
            cp_async_wait<0>();
            __syncthreads();
            HALE_SPLIT_MARK(7);
            // ctx[g][d0 + dd] += p_t v_t, t ascending, in blocks of PS positions:
            // every thread forms products (independent), then chain c = tid
            // adds its row of them in order (4 per 16-byte load)
            for (int s0 = 0; s0 < here; s0 += PS) {
                const int n = min(PS, here - s0);
                if (pc < G * kSplitD) {
                    // 8 products' operands loaded before any is formed (one
                    // shared-memory round trip per 8, not per product)
                    const float* pe = se + (pc / kSplitD) * ES + s0;
                    const float* pv = sv + s0 * kSplitD + pc % kSplitD;
                    float* po = spr + pc * PR;
                    int t = pq;
                    for (; t + 7 * TPC < n; t += 8 * TPC) {
                        float ea[8], va[8];
#pragma unroll
                        for (int w = 0; w < 8; w++) {
                            ea[w] = pe[t + w * TPC];
                            va[w] = pv[(t + w * TPC) * kSplitD];
                        }
#pragma unroll
                        for (int w = 0; w < 8; w++) po[t + w * TPC] = fmul(ea[w], va[w]);
                    }
                    for (; t < n; t += TPC) po[t] = fmul(pe[t], pv[t * kSplitD]);
                }
                __syncthreads();
                if (s0 == 0) HALE_SPLIT_MARK(9);
                if (busy) {
                    const float* row = spr + tid * PR;
                    int t = 0;
                    for (; t + 16 <= n; t += 16) {
                        const float4 a0 = reinterpret_cast<const float4*>(row + t)[0];
                        const float4 a1 = reinterpret_cast<const float4*>(row + t)[1];
                        const float4 a2 = reinterpret_cast<const float4*>(row + t)[2];
                        const float4 a3 = reinterpret_cast<const float4*>(row + t)[3];
                        c = fadd(fadd(fadd(fadd(c, a0.x), a0.y), a0.z), a0.w);
                        c = fadd(fadd(fadd(fadd(c, a1.x), a1.y), a1.z), a1.w);
                        c = fadd(fadd(fadd(fadd(c, a2.x), a2.y), a2.z), a2.w);
                        c = fadd(fadd(fadd(fadd(c, a3.x), a3.y), a3.z), a3.w);
                    }
                    for (; t < n; t++) c = fadd(c, row[t]);
                }
                __syncthreads();
                if (s0 == 0) HALE_SPLIT_MARK(10);
            }
            __syncthreads();  // se / sv are restaged by the next chunk or unit
            HALE_SPLIT_MARK(8);
        }
        if (busy) a.ctx[(size_t)(h * G + g) * hd + d0 + dd] = c;
    }
    __syncthreads();
    HALE_SPLIT_MARK(4);
    if (tid == 0) {
        if (tok_add_acq_rel(&a.bar[2], 1u) == gridDim.x - 1) {
            a.bar[0] = 0u;
            a.bar[1] = 0u;
            a.bar[2] = 0u;
        }
    }
}
#endif  // __CUDACC__

}  // namespace hale
