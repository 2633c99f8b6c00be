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
// (blockIdx.x). All threads stage v, the squares v*v and w in shared memory
// with every global load issued up front, so the one sequential chain is
// FADDs alone over 16-byte shared loads issued ahead of it and the output
// pass reads no global memory. Dynamic shared memory: 3 n floats.
// Up to two byte ranges to pull into L2 while a latency-bound kernel runs
// (the next kernels' weights). Each range: 16-byte aligned, a multiple of 16
// bytes (or null / 0).
struct L2Prefetch {
    const uint8_t* p[2];
    size_t bytes[2];
};
constexpr uint32_t kL2Piece = 16384;

// CTA `slot` of `slots` prefetch CTAs issues its share of the ranges' pieces
// (cp.async.bulk.prefetch.L2: no destination, nothing to wait for).
__device__ __forceinline__ void l2_prefetch_share(const L2Prefetch& pf, int slot, int slots) {
    for (int r = 0; r < 2; r++) {
        if (!pf.p[r]) continue;
        const size_t n = (pf.bytes[r] + kL2Piece - 1) / kL2Piece;
        for (size_t i = (size_t)slot + (size_t)slots * threadIdx.x; i < n; i += (size_t)slots * blockDim.x) {
            const size_t off = i * kL2Piece;
            const uint32_t len = (uint32_t)(pf.bytes[r] - off < kL2Piece ? pf.bytes[r] - off : kL2Piece);
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(pf.p[r] + off), "r"(len) : "memory");
        }
    }
}

// Rows past the first n of the grid only prefetch (pf) and leave.
__global__ void rmsnorm_kernel(float* __restrict__ x, const float* __restrict__ delta, const float* __restrict__ w,
                               float eps, int n, float* __restrict__ out, int rows, L2Prefetch pf) {
    if ((int)blockIdx.x >= rows) {
        l2_prefetch_share(pf, blockIdx.x - rows, gridDim.x - rows);
        return;
    }
    extern __shared__ __align__(16) float s_v[];  // [n] v, [n] v*v, [n] w
    float* s_sq = s_v + n;
    float* s_w = s_sq + n;
    __shared__ float s_scale;
    x += (size_t)blockIdx.x * n;
    out += (size_t)blockIdx.x * n;
    if (delta) delta += (size_t)blockIdx.x * n;
#pragma unroll 4
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float xv = x[i], dv = delta ? delta[i] : 0.0f, wv = w[i];
        const float v = delta ? fadd(xv, dv) : xv;
        if (delta) x[i] = v;
        s_v[i] = v;
        s_sq[i] = fmul(v, v);
        s_w[i] = wv;
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
    for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = fmul(fmul(s_v[i], scale), s_w[i]);
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
// element is read once for the chunk's heads. Per head the arithmetic is
// Attention::forward's (attention.rs:59-85) in attn_decode_kernel's order:
// scores[t] = (sum_i q_i k_ti from -0) * scale; softmax over t = 0..pos;
// ctx_i = sum_t p_t v_ti from 0, t ascending.
//   - K, then V, stream through kGqaStages shared-memory stages with 16-byte
//     cp.async copies, consecutive threads on consecutive bytes of a row;
//     K rows are padded to hd + 4 floats so the score threads' 16-byte reads
//     of 8 different rows hit distinct banks;
//   - scores: thread (position p of a 64-row tile, head group hg) runs the
//     chains of heads hg, hg + 4, ...; q sits in shared memory;
//   - the first V stages load while the softmax runs;
//   - context: thread (column, head subset), four positions per step with
//     the loads of the next steps issued ahead.
// Scores live in shared memory ([GC][sc_cap]) when pos + 1 <= sc_cap, else in
// the [n][nh][max_len] scratch. hd <= 256, hd % 4 == 0. Dynamic shared
// memory: gqa_smem_floats(gc, cap, hd) floats.
constexpr int kGqaStages = 4;
constexpr int kGqaTK = 64;  // positions per K tile

// Shared-memory score capacity (positions) of attn_gqa_kernel<GC>.
__host__ __device__ inline int gqa_score_cap(int gc) { return gc == 1 ? 8192 : (gc <= 4 ? 4096 : 2048); }
// V rows per stage: 32 KB stages, a multiple of 4 rows (the context loop
// reads scores four positions at a time from 16-byte-aligned offsets).
__host__ __device__ inline int gqa_v_rows(int hd) { return (8192 / hd) & ~3; }
__host__ __device__ inline int gqa_stage_floats(int hd) {
    const int k = kGqaTK * (hd + 4), v = gqa_v_rows(hd) * hd;
    return k > v ? k : v;
}
__host__ __device__ inline size_t gqa_smem_floats(int gc, int cap, int hd) {
    return (size_t)gc * hd + (size_t)gc * cap + (size_t)kGqaStages * gqa_stage_floats(hd);
}

// Rows [tile * rows, +rows) of one KV head (src = its column 0, rows kvd
// floats apart) into stage tile % kGqaStages with destination row pitch
// `pitch` floats, then a commit (an empty group past the last tile keeps the
// wait count uniform). Thread tid copies 16-byte chunk (tid mod q4n) of every
// (256 / q4n)-th row when q4n divides 256.
__device__ __forceinline__ void gqa_stage(float* stages, int sfl, const float* __restrict__ src, int tile,
                                          int n_tiles, int rows, int pitch, int seq, int hd, int kvd, int tid) {
    if (tile < n_tiles) {
        float* dst = stages + (size_t)(tile % kGqaStages) * sfl;
        const int t0 = tile * rows, here = min(rows, seq - t0), q4n = hd >> 2;
        if ((256 % q4n) == 0) {
            const int c4 = tid % q4n, step = 256 / q4n;
            for (int tt = tid / q4n; tt < here; tt += step)
                cp_async16(dst + tt * pitch + 4 * c4, src + (size_t)(t0 + tt) * kvd + 4 * c4);
        } else {
            for (int j = tid; j < here * q4n; j += 256) {
                const int tt = j / q4n, c4 = j - tt * q4n;
                cp_async16(dst + tt * pitch + 4 * c4, src + (size_t)(t0 + tt) * kvd + 4 * c4);
            }
        }
    }
    cp_async_commit();
}

// One score chain step block: 8 key float4 and the matching q float4 of
// each head loaded first, then the 32 chain steps of every head.
template <int HN, int GC>
__device__ __forceinline__ void gqa_score_block(const float4* __restrict__ key, const float4* __restrict__ sq4,
                                                int q4n, int hg, int i0, float (&acc)[HN]) {
    float4 kb[8];
#pragma unroll
    for (int u = 0; u < 8; u++) kb[u] = key[i0 + u];
#pragma unroll
    for (int j = 0; j < HN; j++) {
        const int g = hg + 4 * j;
        if (g < GC) {
            float4 qb[8];
#pragma unroll
            for (int u = 0; u < 8; u++) qb[u] = sq4[g * q4n + i0 + u];
            float a = acc[j];
#pragma unroll
            for (int u = 0; u < 8; u++) {
                a = fadd(a, fmul(qb[u].x, kb[u].x));
                a = fadd(a, fmul(qb[u].y, kb[u].y));
                a = fadd(a, fmul(qb[u].z, kb[u].z));
                a = fadd(a, fmul(qb[u].w, kb[u].w));
            }
            acc[j] = a;
        }
    }
}

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
    __shared__ uint64_t s_tab[32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, r = blockIdx.y;
    const int h0 = blockIdx.x * GC, G = nh / nkv;
    const int seq = (int)rows[3 * r + 1] + 1, kvd = nkv * hd, off = (h0 / G) * hd, q4n = hd >> 2;
    const size_t sbase = (size_t)rows[3 * r + 2] * seq_stride;
    const float* kbase = kcache + sbase + off;
    const float* vbase = vcache + sbase + off;
    const int sfl = gqa_stage_floats(hd), kp = hd + 4;
    float* s_q = s_gqa;                                   // [GC][hd]
    float* s_sc = s_q + GC * hd;                           // [GC][sc_cap]
    float* stages = s_sc + (size_t)GC * sc_cap;           // [kGqaStages][sfl]
    const bool in_smem = seq <= sc_cap;
    float* g_sc = scores + ((size_t)r * nh + h0) * max_len;  // used when !in_smem
    const int nk = (seq + kGqaTK - 1) / kGqaTK;
#pragma unroll
    for (int st = 0; st < kGqaStages - 1; st++) gqa_stage(stages, sfl, kbase, st, nk, kGqaTK, kp, seq, hd, kvd, tid);
    const float* qrow = qkv + (size_t)r * (nh + 2 * nkv) * hd + (size_t)h0 * hd;
    for (int i = tid; i < GC * hd; i += 256) s_q[i] = qrow[i];
    if (tid < 32) s_tab[tid] = kExp2TabDev[tid];

    // ---- scores: thread (p, hg) runs heads hg, hg + 4, ... of position p ----
    const int p = tid & (kGqaTK - 1), hg = tid / kGqaTK;  // a warp has one hg
    constexpr int HN = (GC + 3) / 4;
    float mx[HN];
#pragma unroll
    for (int j = 0; j < HN; j++) mx[j] = -__int_as_float(0x7f800000);
    if (tid < 8 * GC) s_red[tid / GC][tid % GC] = -__int_as_float(0x7f800000);
    const float4* sq4 = reinterpret_cast<const float4*>(s_q);
    for (int tile = 0; tile < nk; tile++) {
        gqa_stage(stages, sfl, kbase, tile + kGqaStages - 1, nk, kGqaTK, kp, seq, hd, kvd, tid);
        cp_async_wait<kGqaStages - 1>();
        __syncthreads();
        const int t = tile * kGqaTK + p;
        if (t < seq && hg < GC) {
            const float4* key = reinterpret_cast<const float4*>(stages + (size_t)(tile % kGqaStages) * sfl + p * kp);
            float acc[HN];
#pragma unroll
            for (int j = 0; j < HN; j++) acc[j] = -0.0f;
            int i0 = 0;
            for (; i0 + 8 <= q4n; i0 += 8) gqa_score_block<HN, GC>(key, sq4, q4n, hg, i0, acc);
            for (; i0 < q4n; i0++) {
                const float4 k4 = key[i0];
#pragma unroll
                for (int j = 0; j < HN; j++) {
                    const int g = hg + 4 * j;
                    if (g < GC) {
                        const float4 q = sq4[g * q4n + i0];
                        float a = acc[j];
                        a = fadd(a, fmul(q.x, k4.x));
                        a = fadd(a, fmul(q.y, k4.y));
                        a = fadd(a, fmul(q.z, k4.z));
                        a = fadd(a, fmul(q.w, k4.w));
                        acc[j] = a;
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < HN; j++) {
                const int g = hg + 4 * j;
                if (g < GC) {
                    const float sv = fmul(acc[j], scale);
                    if (in_smem) s_sc[g * sc_cap + t] = sv;
                    else g_sc[(size_t)g * max_len + t] = sv;
                    mx[j] = fmaxf(mx[j], sv);
                }
            }
        }
        __syncthreads();
    }
    // V streams in while the softmax runs
    const int nv = (seq + vt - 1) / vt;
#pragma unroll
    for (int st = 0; st < kGqaStages - 1; st++) gqa_stage(stages, sfl, vbase, st, nv, vt, hd, seq, hd, kvd, tid);
    // max per head (order-independent): each warp reduces the heads of its hg
#pragma unroll
    for (int j = 0; j < HN; j++) {
        float m = mx[j];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        const int g = hg + 4 * j;
        if (lane == 0 && g < GC) s_red[warp][g] = m;
    }
    __syncthreads();
    if (tid < GC) {
        float m = -__int_as_float(0x7f800000);
        for (int w = 0; w < 8; w++) m = fmaxf(m, s_red[w][tid]);
        s_mx[tid] = m;
    }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < GC; g++) {
        const float m = s_mx[g];
        if (in_smem)
            for (int t = tid; t < seq; t += 256) s_sc[g * sc_cap + t] = hale_expf_tab(fsub(s_sc[g * sc_cap + t], m), s_tab);
        else
            for (int t = tid; t < seq; t += 256)
                g_sc[(size_t)g * max_len + t] = hale_expf_tab(fsub(g_sc[(size_t)g * max_len + t], m), s_tab);
    }
    __syncthreads();
    // the reference's left-to-right denominator, one thread per head
    if (tid < GC) {
        float sum = 0.0f;
        if (in_smem) {
            const float* row = s_sc + tid * sc_cap;
            const float4* r4 = reinterpret_cast<const float4*>(row);
            int t = 0;
            for (; t + 16 <= seq; t += 16) {
                const float4 e0 = r4[t >> 2], e1 = r4[(t >> 2) + 1], e2 = r4[(t >> 2) + 2], e3 = r4[(t >> 2) + 3];
                sum = fadd(fadd(fadd(fadd(sum, e0.x), e0.y), e0.z), e0.w);
                sum = fadd(fadd(fadd(fadd(sum, e1.x), e1.y), e1.z), e1.w);
                sum = fadd(fadd(fadd(fadd(sum, e2.x), e2.y), e2.z), e2.w);
                sum = fadd(fadd(fadd(fadd(sum, e3.x), e3.y), e3.z), e3.w);
            }
            for (; t < seq; t++) sum = fadd(sum, row[t]);
        } else {
            const float* row = g_sc + (size_t)tid * max_len;
            for (int t = 0; t < seq; t++) sum = fadd(sum, row[t]);
        }
        s_sum[tid] = sum;
    }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < GC; g++) {
        const float sm = s_sum[g];
        if (in_smem)
            for (int t = tid; t < seq; t += 256) s_sc[g * sc_cap + t] = fdiv(s_sc[g * sc_cap + t], sm);
        else
            for (int t = tid; t < seq; t += 256) g_sc[(size_t)g * max_len + t] = fdiv(g_sc[(size_t)g * max_len + t], sm);
    }

    // ---- context: thread (col, gi) runs heads gi, gi + tpc, ... ----
    const int tpc = 256 / hd;
    const int gi = tid / hd, col = tid - gi * hd;
    const bool busy = gi < tpc && gi < GC;
    constexpr int HPT = GC;  // upper bound of heads per thread
    float c[HPT];
#pragma unroll
    for (int j = 0; j < HPT; j++) c[j] = 0.0f;
    for (int tile = 0; tile < nv; tile++) {
        gqa_stage(stages, sfl, vbase, tile + kGqaStages - 1, nv, vt, hd, seq, hd, kvd, tid);
        cp_async_wait<kGqaStages - 1>();
        __syncthreads();
        const float* vt_ = stages + (size_t)(tile % kGqaStages) * sfl + col;
        const int t0 = tile * vt, here = min(vt, seq - t0);
        if (busy) {
            int tt = 0;
            if (in_smem) {
                // blocks of 16 positions: the 16 v values and each head's 16
                // scores are loaded before the block's chain steps
                for (; tt + 16 <= here; tt += 16) {
                    float vb[16];
#pragma unroll
                    for (int u = 0; u < 16; u++) vb[u] = vt_[(tt + u) * hd];
#pragma unroll
                    for (int j = 0; j < HPT; j++) {
                        const int g = gi + j * tpc;
                        if (g < GC) {
                            const float4* p4 = reinterpret_cast<const float4*>(s_sc + g * sc_cap + t0 + tt);
                            const float4 a0 = p4[0], a1 = p4[1], a2 = p4[2], a3 = p4[3];
                            float a = c[j];
                            a = fadd(a, fmul(a0.x, vb[0]));  a = fadd(a, fmul(a0.y, vb[1]));
                            a = fadd(a, fmul(a0.z, vb[2]));  a = fadd(a, fmul(a0.w, vb[3]));
                            a = fadd(a, fmul(a1.x, vb[4]));  a = fadd(a, fmul(a1.y, vb[5]));
                            a = fadd(a, fmul(a1.z, vb[6]));  a = fadd(a, fmul(a1.w, vb[7]));
                            a = fadd(a, fmul(a2.x, vb[8]));  a = fadd(a, fmul(a2.y, vb[9]));
                            a = fadd(a, fmul(a2.z, vb[10])); a = fadd(a, fmul(a2.w, vb[11]));
                            a = fadd(a, fmul(a3.x, vb[12])); a = fadd(a, fmul(a3.y, vb[13]));
                            a = fadd(a, fmul(a3.z, vb[14])); a = fadd(a, fmul(a3.w, vb[15]));
                            c[j] = a;
                        }
                    }
                }
                for (; tt < here; tt++) {
                    const float v = vt_[tt * hd];
#pragma unroll
                    for (int j = 0; j < HPT; j++) {
                        const int g = gi + j * tpc;
                        if (g < GC) c[j] = fadd(c[j], fmul(s_sc[g * sc_cap + t0 + tt], v));
                    }
                }
            } else {
                for (; tt < here; tt++) {
                    const float v = vt_[tt * hd];
#pragma unroll
                    for (int j = 0; j < HPT; j++) {
                        const int g = gi + j * tpc;
                        if (g < GC) c[j] = fadd(c[j], fmul(g_sc[(size_t)g * max_len + t0 + tt], v));
                    }
                }
            }
        }
        __syncthreads();
    }
    if (busy) {
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
