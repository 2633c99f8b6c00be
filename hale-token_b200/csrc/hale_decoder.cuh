// hale_decoder.cuh -- the dense pieces of one decode step of the reference's
// Transformer::forward (src/model/transformer.rs:168-227), around the MoE
// layer: embedding row, RMSNorm, per-head QK-norm and RoPE with the KV-cache
// append, GQA attention over the cache, residual adds, and the float SwiGLU
// of dense layers. Every f32 operation keeps the reference's order, so a
// decode step equals the oracle's bit for bit:
//   - sums that the reference folds left to right (sum of squares in
//     RMSNorm, the softmax denominator, each score's q.k, each context
//     element) run as one sequential chain per output;
//   - order-independent steps (max, elementwise) run in parallel.
// The RoPE cos/sin tables come from the host's libm (the one the reference
// calls), computed once per decoder.
#pragma once

#include "hale_kernels.cuh"

namespace hale {

// A step processes n rows; row r is described in device memory by
// rows[3r .. 3r+2] = token, position, sequence (so a captured step replays
// for any token). Row r's activations sit at row r of every [n, width]
// buffer; sequence s's KV cache of a layer starts at s * seq_stride floats.

// x[r][c] = embed[token_r][c] decoded to f32 (row-major source rows; DT 0
// f32, 1 f16, 2 bf16). Grid: (ceil(H / blockDim), n).
template <int DT>
__global__ void embed_kernel(const void* __restrict__ embed, int H, const uint32_t* __restrict__ rows,
                             float* __restrict__ x) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x, r = blockIdx.y;
    if (c >= H) return;
    const size_t i = (size_t)rows[3 * r] * H + c;
    float* xr = x + (size_t)r * H;
    if (DT == 0) xr[c] = reinterpret_cast<const float*>(embed)[i];
    else if (DT == 1) xr[c] = half_bits_to_float(reinterpret_cast<const uint16_t*>(embed)[i]);
    else xr[c] = __uint_as_float((uint32_t)reinterpret_cast<const uint16_t*>(embed)[i] << 16);
}

// The residual add x += delta (transformer.rs residual; delta nullable), then
// RmsNorm::forward (src/ops/norm.rs:7-28): s = sum of v*v left to right from
// -0; scale = 1 / sqrt(s / n + eps); out = (x * scale) * w. One CTA per row
// (blockIdx.x). All threads stage v and the squares v*v in shared memory, so
// the one sequential chain is FADDs alone over 16-byte shared loads issued
// ahead of it. Dynamic shared memory: 2 n floats.
__global__ void rmsnorm_kernel(float* __restrict__ x, const float* __restrict__ delta, const float* __restrict__ w,
                               float eps, int n, float* __restrict__ out) {
    extern __shared__ __align__(16) float s_v[];  // [n] v, then [n] v*v
    float* s_sq = s_v + n;
    __shared__ float s_scale;
    x += (size_t)blockIdx.x * n;
    out += (size_t)blockIdx.x * n;
    if (delta) delta += (size_t)blockIdx.x * n;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = delta ? fadd(x[i], delta[i]) : x[i];
        if (delta) x[i] = v;
        s_v[i] = v;
        s_sq[i] = fmul(v, v);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float s = -0.0f;
        int i = 0;
        if ((n & 3) == 0) {
            const float4* q4 = reinterpret_cast<const float4*>(s_sq);
#pragma unroll 8
            for (; i < n / 4; i++) {
                const float4 q = q4[i];
                s = fadd(fadd(fadd(fadd(s, q.x), q.y), q.z), q.w);
            }
            i = n;
        }
        for (; i < n; i++) s = fadd(s, s_sq[i]);
        s_scale = fdiv(1.0f, __fsqrt_rn(fadd(fdiv(s, (float)n), eps)));
    }
    __syncthreads();
    const float scale = s_scale;
    for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = fmul(fmul(s_v[i], scale), w[i]);
}

// Per head (one warp each; q heads, then k heads, then v heads): the in-place
// RMSNorm of q/k heads, x = x * (scale * w) (norm.rs:30-37, attention.rs:49-56),
// when the model has it; RoPE (rope.rs:15-43) a' = a c - b s, b' = b c + a s on
// the pairs (i, i + hd/2); k and v rows appended to the row's sequence cache
// at its position. qkv: per row [nh*hd | nkv*hd | nkv*hd] as the fused
// projection wrote it. Grid: (nh + 2 nkv, n).
__global__ void qk_rope_kernel(float* __restrict__ qkv, int nh, int nkv, int hd, const float* __restrict__ q_norm,
                               const float* __restrict__ k_norm, float eps, const float* __restrict__ rope_cos,
                               const float* __restrict__ rope_sin, const uint32_t* __restrict__ rows,
                               float* __restrict__ kcache, float* __restrict__ vcache, size_t seq_stride) {
    const int head = blockIdx.x, lane = threadIdx.x, half = hd / 2, r = blockIdx.y;
    const uint32_t pos = rows[3 * r + 1];
    const size_t seq = rows[3 * r + 2];
    const int kvd = nkv * hd;
    if (head >= nh + 2 * nkv) return;
    qkv += (size_t)r * (nh + 2 * nkv) * hd;
    kcache += seq * seq_stride;
    vcache += seq * seq_stride;
    if (head >= nh + nkv) {  // v head: straight into the cache
        const int vh = head - nh - nkv;
        const float* v = qkv + (size_t)(nh + nkv) * hd + (size_t)vh * hd;
        for (int i = lane; i < hd; i += 32) vcache[(size_t)pos * kvd + vh * hd + i] = v[i];
        return;
    }
    const bool is_k = head >= nh;
    float* x = qkv + (size_t)head * hd;
    const float* w = is_k ? k_norm : q_norm;
    if (w) {
        extern __shared__ float s_h[];  // [hd]: the head, staged for lane 0's chain
        for (int i = lane; i < hd; i += 32) s_h[i] = x[i];
        __syncwarp();
        float scale = 0.0f;
        if (lane == 0) {
            float s = -0.0f;
#pragma unroll 16
            for (int i = 0; i < hd; i++) s = fadd(s, fmul(s_h[i], s_h[i]));
            scale = fdiv(1.0f, __fsqrt_rn(fadd(fdiv(s, (float)hd), eps)));
        }
        scale = __shfl_sync(0xffffffffu, scale, 0);
        __syncwarp();
        for (int i = lane; i < hd; i += 32) x[i] = fmul(x[i], fmul(scale, w[i]));
        __syncwarp();
    }
    const float* c = rope_cos + (size_t)pos * half;
    const float* s = rope_sin + (size_t)pos * half;
    for (int i = lane; i < half; i += 32) {
        const float a = x[i], b = x[half + i];
        x[i] = fsub(fmul(a, c[i]), fmul(b, s[i]));
        x[half + i] = fadd(fmul(b, c[i]), fmul(a, s[i]));
    }
    __syncwarp();
    if (is_k) {
        const int kh = head - nh;
        for (int i = lane; i < hd; i += 32) kcache[(size_t)pos * kvd + kh * hd + i] = x[i];
    }
}

// 16-byte asynchronous global -> shared copies (cp.async, sm_80+).
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    const unsigned sa = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(sa), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// Attention's V staging: kAttnStages stages of attn_v_rows(hd) positions
// (16 KB each).
constexpr int kAttnStages = 3;
__host__ __device__ inline int attn_v_rows(int hd) { return 4096 / hd < 4 ? 4 : 4096 / hd; }

// Copies V rows [tile * vt, +vt) of one kv head (vsrc = its column 0) into
// stage tile % kAttnStages and commits the group (an empty group past the
// last tile keeps the wait count uniform).
__device__ __forceinline__ void attn_stage_v(float* s_v, const float* __restrict__ vsrc, int tile, int n_tiles,
                                             int vt, int seq, int hd, int kvd, int tid) {
    if (tile < n_tiles) {
        float* dst = s_v + (size_t)(tile % kAttnStages) * vt * hd;
        const int t0 = tile * vt, here = min(vt, seq - t0), q4 = hd >> 2;
        for (int j = tid; j < here * q4; j += 256) {
            const int tt = j / q4, c4 = j - tt * q4;
            cp_async16(dst + tt * hd + 4 * c4, vsrc + (size_t)(t0 + tt) * kvd + 4 * c4);
        }
    }
    cp_async_commit();
}

// Attention::forward for the row's token at pos (attention.rs:59-85), one CTA
// per (q head h, row) (kv head h / (nh / nkv)): scores[t] = (sum_i q_i k_ti
// from -0) * scale; softmax over t = 0..pos (activation.rs:11-21); ctx_i =
// sum_t scores[t] v_ti from 0, t ascending, over the row's sequence cache. q
// sits in shared memory and each key row is read 16 bytes at a time ahead of
// its chain; scores live in shared memory when pos + 1 <= smem_scores, else
// in the [n][nh][max_len] scratch; V rows are staged through shared memory
// (vt = attn_v_rows(hd) per stage). Dynamic shared memory: hd +
// round4(smem_scores) + kAttnStages * vt * hd floats. Grid: (nh, n); 256
// threads, each running CMAX context columns.
template <int CMAX>
__global__ void __launch_bounds__(256) attn_decode_kernel(const float* __restrict__ qkv, int nh, int nkv, int hd,
                                                          const float* __restrict__ kcache,
                                                          const float* __restrict__ vcache,
                                                          const uint32_t* __restrict__ rows, int max_len,
                                                          float scale, float* __restrict__ scores,
                                                          float* __restrict__ ctx, int smem_scores,
                                                          size_t seq_stride, int vt) {
    extern __shared__ __align__(16) float s_att[];  // [hd] q, then [smem_scores] scores
    __shared__ float s_red[32];
    __shared__ float s_bc[2];
    const int h = blockIdx.x, tid = threadIdx.x, r = blockIdx.y;
    const int seq = (int)rows[3 * r + 1] + 1, kvd = nkv * hd, off = (h / (nh / nkv)) * hd;
    qkv += (size_t)r * (nh + 2 * nkv) * hd;
    ctx += (size_t)r * nh * hd;
    scores += (size_t)r * nh * max_len;
    kcache += (size_t)rows[3 * r + 2] * seq_stride;
    vcache += (size_t)rows[3 * r + 2] * seq_stride;
    float* s_q = s_att;
    for (int i = tid; i < hd; i += blockDim.x) s_q[i] = qkv[(size_t)h * hd + i];
    float* sc = seq <= smem_scores ? s_att + hd : scores + (size_t)h * max_len;
    __syncthreads();
    float mx = -__int_as_float(0x7f800000);
    for (int t = tid; t < seq; t += blockDim.x) {
        const float4* key = reinterpret_cast<const float4*>(kcache + (size_t)t * kvd + off);
        float s = -0.0f;
#pragma unroll 8
        for (int i4 = 0; i4 < hd / 4; i4++) {
            const float4 k4 = key[i4];
            s = fadd(s, fmul(s_q[4 * i4], k4.x));
            s = fadd(s, fmul(s_q[4 * i4 + 1], k4.y));
            s = fadd(s, fmul(s_q[4 * i4 + 2], k4.z));
            s = fadd(s, fmul(s_q[4 * i4 + 3], k4.w));
        }
        s = fmul(s, scale);
        sc[t] = s;
        mx = fmaxf(mx, s);
    }
    // max is order-independent
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((tid & 31) == 0) s_red[tid >> 5] = mx;
    __syncthreads();
    if (tid == 0) {
        float m = -__int_as_float(0x7f800000);
        for (int w = 0; w < (int)(blockDim.x >> 5); w++) m = fmaxf(m, s_red[w]);
        s_bc[0] = m;
    }
    __syncthreads();
    mx = s_bc[0];
    for (int t = tid; t < seq; t += blockDim.x) sc[t] = hale_expf(fsub(sc[t], mx));
    __syncthreads();
    if (tid == 0) {
        float sum = 0.0f;
#pragma unroll 16
        for (int t = 0; t < seq; t++) sum = fadd(sum, sc[t]);
        s_bc[1] = sum;
    }
    __syncthreads();
    const float sum = s_bc[1];
    for (int t = tid; t < seq; t += blockDim.x) sc[t] = fdiv(sc[t], sum);
    // context: V rows stream through shared memory, vt positions per stage in
    // kAttnStages stages (16-byte cp.async by every thread), while the threads
    // of columns i run their chains over the staged rows in t order
    float* s_v = s_att + hd + ((smem_scores + 3) & ~3);
    const int n_tiles = (seq + vt - 1) / vt;
    const float* vsrc = vcache + off;
#pragma unroll
    for (int st = 0; st < kAttnStages - 1; st++) attn_stage_v(s_v, vsrc, st, n_tiles, vt, seq, hd, kvd, tid);
    float c[CMAX];  // columns tid, tid + 256, ... (CMAX * 256 >= hd)
#pragma unroll
    for (int q = 0; q < CMAX; q++) c[q] = 0.0f;
    for (int tile = 0; tile < n_tiles; tile++) {
        attn_stage_v(s_v, vsrc, tile + kAttnStages - 1, n_tiles, vt, seq, hd, kvd, tid);
        cp_async_wait<kAttnStages - 1>();
        __syncthreads();
        const float* vtile = s_v + (size_t)(tile % kAttnStages) * vt * hd;
        const int t0 = tile * vt, here = min(vt, seq - t0);
#pragma unroll
        for (int q = 0; q < CMAX; q++) {
            const int i = tid + q * 256;
            if (i < hd) {
                float acc = c[q];
#pragma unroll 8
                for (int tt = 0; tt < here; tt++) acc = fadd(acc, fmul(sc[t0 + tt], vtile[tt * hd + i]));
                c[q] = acc;
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int q = 0; q < CMAX; q++) {
        const int i = tid + q * 256;
        if (i < hd) ctx[(size_t)h * hd + i] = c[q];
    }
}

// Attention for GC query heads that share one KV head (GQA group; GC divides
// nh / nkv), one CTA of 256 threads per (head chunk, row): each K and V
// element is read once for the chunk's heads, and every thread runs GC
// independent chains. Per head the arithmetic is Attention::forward's
// (attention.rs:59-85) in attn_decode_kernel's order: scores[t] = (sum_i
// q_i k_ti from -0) * scale; softmax over t = 0..pos; ctx_i = sum_t p_t v_ti
// from 0, t ascending.
//   - V rows start streaming into shared memory (kGqaStages stages of vt
//     rows, 16-byte cp.async) before the scores are computed;
//   - scores: thread per position, 16-byte key loads issued ahead of the GC
//     chains, q of the chunk's heads in shared memory;
//   - context: thread per (column, head subset), scores read four positions
//     at a time.
// Scores live in shared memory ([GC][sc_cap]) when pos + 1 <= sc_cap, else in
// the [n][nh][max_len] scratch. Dynamic shared memory: GC*hd + GC*sc_cap +
// kGqaStages*vt*hd floats (sc_cap a multiple of 4). hd <= 256, hd % 4 == 0.
constexpr int kGqaStages = 4;

// V rows [tile * vt, +vt) of the KV head (vbase = its column 0) into stage
// tile % kGqaStages, then a commit (empty past the last tile).
__device__ __forceinline__ void gqa_stage_v(float* s_v, const float* __restrict__ vbase, int tile, int n_tiles,
                                            int vt, int seq, int hd, int kvd, int tid) {
    if (tile < n_tiles) {
        float* dst = s_v + (size_t)(tile % kGqaStages) * vt * hd;
        const int t0 = tile * vt, here = min(vt, seq - t0), q4n = hd >> 2;
        for (int j = tid; j < here * q4n; j += 256) {
            const int tt = j / q4n, c4 = j - tt * q4n;
            cp_async16(dst + tt * hd + 4 * c4, vbase + (size_t)(t0 + tt) * kvd + 4 * c4);
        }
    }
    cp_async_commit();
}

// Shared-memory score capacity (positions) of attn_gqa_kernel<GC>.
__host__ __device__ inline int gqa_score_cap(int gc) { return gc == 1 ? 8192 : (gc <= 4 ? 4096 : 2048); }
// V rows per stage: 32 KB stages, a multiple of 4 rows (the context loop
// reads scores four positions at a time from 16-byte-aligned offsets).
__host__ __device__ inline int gqa_v_rows(int hd) { return (8192 / hd) & ~3; }

template <int GC>
__global__ void __launch_bounds__(256) attn_gqa_kernel(const float* __restrict__ qkv, int nh, int nkv, int hd,
                                                       const float* __restrict__ kcache,
                                                       const float* __restrict__ vcache,
                                                       const uint32_t* __restrict__ rows, int max_len, float scale,
                                                       float* __restrict__ scores, float* __restrict__ ctx,
                                                       int sc_cap, size_t seq_stride, int vt) {
    extern __shared__ __align__(16) float s_gqa[];
    __shared__ float s_red[8][GC];
    __shared__ float s_mx[GC], s_sum[GC];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, r = blockIdx.y;
    const int h0 = blockIdx.x * GC, G = nh / nkv;
    const int seq = (int)rows[3 * r + 1] + 1, kvd = nkv * hd, off = (h0 / G) * hd, q4n = hd >> 2;
    const size_t sbase = (size_t)rows[3 * r + 2] * seq_stride;
    const float* kbase = kcache + sbase + off;
    const float* vbase = vcache + sbase + off;
    float* s_q = s_gqa;                                   // [GC][hd]
    float* s_sc = s_q + GC * hd;                           // [GC][sc_cap]
    float* s_v = s_sc + (size_t)GC * sc_cap;              // [kGqaStages][vt][hd]
    const bool in_smem = seq <= sc_cap;
    const size_t sc_stride = in_smem ? (size_t)sc_cap : (size_t)max_len;
    float* sc = in_smem ? s_sc : scores + ((size_t)r * nh + h0) * max_len;
    const int n_tiles = (seq + vt - 1) / vt;
    // V prefetch: the first stages are in flight during the score phase
#pragma unroll
    for (int st = 0; st < kGqaStages - 1; st++) gqa_stage_v(s_v, vbase, st, n_tiles, vt, seq, hd, kvd, tid);
    const float* qrow = qkv + (size_t)r * (nh + 2 * nkv) * hd + (size_t)h0 * hd;
    for (int i = tid; i < GC * hd; i += 256) s_q[i] = qrow[i];
    __syncthreads();

    // ---- scores ----
    float mx[GC];
#pragma unroll
    for (int g = 0; g < GC; g++) mx[g] = -__int_as_float(0x7f800000);
    const float4* sq4 = reinterpret_cast<const float4*>(s_q);
    for (int t = tid; t < seq; t += 256) {
        const float4* key = reinterpret_cast<const float4*>(kbase + (size_t)t * kvd);
        float acc[GC];
#pragma unroll
        for (int g = 0; g < GC; g++) acc[g] = -0.0f;
#pragma unroll 8
        for (int i4 = 0; i4 < q4n; i4++) {
            const float4 k4 = key[i4];
#pragma unroll
            for (int g = 0; g < GC; g++) {
                const float4 q = sq4[g * q4n + i4];
                float a = acc[g];
                a = fadd(a, fmul(q.x, k4.x));
                a = fadd(a, fmul(q.y, k4.y));
                a = fadd(a, fmul(q.z, k4.z));
                a = fadd(a, fmul(q.w, k4.w));
                acc[g] = a;
            }
        }
#pragma unroll
        for (int g = 0; g < GC; g++) {
            const float sv = fmul(acc[g], scale);
            sc[(size_t)g * sc_stride + t] = sv;
            mx[g] = fmaxf(mx[g], sv);
        }
    }
    // max per head (order-independent)
#pragma unroll
    for (int g = 0; g < GC; g++) {
        float m = mx[g];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) s_red[warp][g] = m;
    }
    __syncthreads();
    if (tid < GC) {
        float m = -__int_as_float(0x7f800000);
        for (int w = 0; w < 8; w++) m = fmaxf(m, s_red[w][tid]);
        s_mx[tid] = m;
    }
    __syncthreads();
    for (int j = tid; j < GC * seq; j += 256) {
        const int g = j / seq, t = j - g * seq;
        float* p = sc + (size_t)g * sc_stride + t;
        *p = hale_expf(fsub(*p, s_mx[g]));
    }
    __syncthreads();
    // the reference's left-to-right denominator, one thread per head
    if (tid < GC) {
        const float* row = sc + (size_t)tid * sc_stride;
        float sum = 0.0f;
        int t = 0;
        if (in_smem) {
            const float4* r4 = reinterpret_cast<const float4*>(row);
#pragma unroll 8
            for (; t + 4 <= seq; t += 4) {
                const float4 e = r4[t >> 2];
                sum = fadd(fadd(fadd(fadd(sum, e.x), e.y), e.z), e.w);
            }
        }
        for (; t < seq; t++) sum = fadd(sum, row[t]);
        s_sum[tid] = sum;
    }
    __syncthreads();
    for (int j = tid; j < GC * seq; j += 256) {
        const int g = j / seq, t = j - g * seq;
        float* p = sc + (size_t)g * sc_stride + t;
        *p = fdiv(*p, s_sum[g]);
    }

    // ---- context ----
    const int tpc = 256 / hd;            // thread groups over the columns
    const int gi = tid / hd, col = tid - gi * hd;
    constexpr int HPT = GC;              // upper bound of heads per thread
    float c[HPT];
#pragma unroll
    for (int j = 0; j < HPT; j++) c[j] = 0.0f;
    for (int tile = 0; tile < n_tiles; tile++) {
        gqa_stage_v(s_v, vbase, tile + kGqaStages - 1, n_tiles, vt, seq, hd, kvd, tid);
        cp_async_wait<kGqaStages - 1>();
        __syncthreads();
        const float* vt_ = s_v + (size_t)(tile % kGqaStages) * vt * hd + col;
        const int t0 = tile * vt, here = min(vt, seq - t0);
        if (gi < tpc) {
            int tt = 0;
            if (in_smem) {
                for (; tt + 4 <= here; tt += 4) {
                    const float v0 = vt_[tt * hd], v1 = vt_[(tt + 1) * hd], v2 = vt_[(tt + 2) * hd],
                                v3 = vt_[(tt + 3) * hd];
#pragma unroll
                    for (int j = 0; j < HPT; j++) {
                        const int g = gi + j * tpc;
                        if (g < GC) {
                            const float4 p4 = *reinterpret_cast<const float4*>(sc + (size_t)g * sc_stride + t0 + tt);
                            float a = c[j];
                            a = fadd(a, fmul(p4.x, v0));
                            a = fadd(a, fmul(p4.y, v1));
                            a = fadd(a, fmul(p4.z, v2));
                            a = fadd(a, fmul(p4.w, v3));
                            c[j] = a;
                        }
                    }
                }
            }
            for (; tt < here; tt++) {
                const float v = vt_[tt * hd];
#pragma unroll
                for (int j = 0; j < HPT; j++) {
                    const int g = gi + j * tpc;
                    if (g < GC) c[j] = fadd(c[j], fmul(sc[(size_t)g * sc_stride + t0 + tt], v));
                }
            }
        }
        __syncthreads();
    }
    if (gi < tpc) {
        float* out = ctx + (size_t)r * nh * hd + (size_t)h0 * hd;
#pragma unroll
        for (int j = 0; j < HPT; j++) {
            const int g = gi + j * tpc;
            if (g < GC) out[(size_t)g * hd + col] = c[j];
        }
    }
}

// h[j] = silu(g[j]) * u[j] (expert/mod.rs:100 for float dense layers).
__global__ void silu_mul_kernel(const float* __restrict__ g, const float* __restrict__ u, int n,
                                float* __restrict__ h) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j < n) h[j] = fmul(silu(g[j]), u[j]);
}

}  // namespace hale
