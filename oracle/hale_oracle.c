/*
 * hale_oracle.c -- CPU restatement of Hale-Token's MoE / sampling path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA library, never part of
 * it. Build: oracle/build.py (gcc -O2 -ffp-contract=off -fopenmp). Every
 * function cites the Rust file:line it restates (paths inside the reference
 * crate). See hale_oracle.h for the bit-level rules.
 */
#include "hale_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------ */
/* bit helpers                                                               */
/* ------------------------------------------------------------------------ */
static inline uint32_t f_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float bits_f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint16_t rd_u16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* Rust `f as i8`: saturating, NaN -> 0. */
static inline int8_t sat_i8(float f) {
    if (f != f) return 0;
    if (f >= 127.0f) return 127;
    if (f <= -128.0f) return -128;
    return (int8_t)f; /* truncation toward zero; in range */
}
/* Rust `f as i32`: saturating, NaN -> 0. */
static inline int32_t sat_i32(float f) {
    if (f != f) return 0;
    if (f >= 2147483648.0f) return INT32_MAX;
    if (f < -2147483648.0f) return INT32_MIN;
    return (int32_t)f;
}
/* f32::max / f32::min: a NaN operand yields the other operand (C fmaxf). */
static inline float rmax(float a, float b) { return fmaxf(a, b); }

/* ------------------------------------------------------------------------ */
/* half-precision conversions (the `half` crate's IEEE semantics)            */
/* ------------------------------------------------------------------------ */
float ho_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu, man = h & 0x3ffu;
    if (exp == 0) {
        if (man == 0) return bits_f(sign);
        /* subnormal: man * 2^-24, exact in f32 */
        float v = (float)man * 0x1p-24f;
        return bits_f(f_bits(v) | sign);
    }
    if (exp == 31) return bits_f(sign | 0x7f800000u | (man << 13) | (man ? 0x00400000u : 0));
    return bits_f(sign | ((exp + 112u) << 23) | (man << 13));
}

/* Round-to-nearest-even f32 -> f16 from the IEEE definition: keep 11
 * significant bits (fewer for subnormal results), round on the dropped bits. */
uint16_t ho_f32_to_f16(float v) {
    uint32_t x = f_bits(v);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    uint32_t exp = (x >> 23) & 0xffu, man = x & 0x7fffffu;
    if (exp == 0xff) return (uint16_t)(sign | 0x7c00u | (man ? (0x200u | (man >> 13)) : 0));
    int e = (int)exp - 127 + 15; /* biased half exponent */
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        /* subnormal half (or zero): value = sig * 2^-24 */
        if (e < -10) return sign; /* below half of the smallest subnormal */
        uint32_t sig = man | 0x800000u;      /* 24-bit significand */
        uint32_t shift = (uint32_t)(14 - e); /* 14..24 */
        uint32_t q = sig >> shift;
        uint32_t rem = sig & ((1u << shift) - 1u), halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (q & 1u))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t q = ((uint32_t)e << 10) | (man >> 13);
    uint32_t rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++; /* may carry into inf */
    return (uint16_t)(sign | q);
}

uint16_t ho_f32_to_bf16(float v) {
    uint32_t x = f_bits(v);
    if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40u); /* quiet NaN */
    uint32_t round = ((x >> 16) & 1u) + 0x7fffu;
    return (uint16_t)((x + round) >> 16);
}

static inline float bf16_to_f32(uint16_t b) { return bits_f((uint32_t)b << 16); }

/* ------------------------------------------------------------------------ */
/* formats: dtype.rs                                                         */
/* ------------------------------------------------------------------------ */
size_t ho_block_len(int d) { return (d == HO_Q8_0 || d == HO_Q4_0) ? HO_QK : 1; }

size_t ho_block_bytes(int d) {
    switch (d) {
    case HO_F32: return 4;
    case HO_F16:
    case HO_BF16: return 2;
    case HO_Q8_0: return 2 + HO_QK;
    case HO_Q4_0: return 2 + HO_QK / 2;
    }
    return 0;
}

int64_t ho_row_bytes(int d, size_t cols) {
    size_t bl = ho_block_len(d);
    if (ho_block_bytes(d) == 0 || cols % bl != 0) return -1;
    return (int64_t)(cols / bl * ho_block_bytes(d));
}

/* ------------------------------------------------------------------------ */
/* encode / decode: quant.rs:236-321                                         */
/* ------------------------------------------------------------------------ */
/* encode_block_q8_0, quant.rs:295-305 */
static void encode_block_q8_0(const float* b, uint8_t* out) {
    float amax = 0.0f;
    for (int j = 0; j < HO_QK; j++) amax = rmax(amax, fabsf(b[j]));
    float scale = amax / 127.0f;
    float inv = scale > 0.0f ? 1.0f / scale : 0.0f;
    uint16_t h = ho_f32_to_f16(scale);
    out[0] = (uint8_t)(h & 0xff);
    out[1] = (uint8_t)(h >> 8);
    for (int j = 0; j < HO_QK; j++) {
        float r = roundf(b[j] * inv);
        /* .clamp(-127.0, 127.0): NaN stays NaN and then casts to 0 */
        if (r < -127.0f) r = -127.0f;
        if (r > 127.0f) r = 127.0f;
        out[2 + j] = (uint8_t)sat_i8(r);
    }
}

/* encode_block_q4_0, quant.rs:309-321 */
static void encode_block_q4_0(const float* b, uint8_t* out) {
    float extreme = 0.0f;
    for (int j = 0; j < HO_QK; j++)
        if (fabsf(b[j]) > fabsf(extreme)) extreme = b[j];
    float scale = extreme / -8.0f;
    float inv = scale != 0.0f ? 1.0f / scale : 0.0f;
    uint16_t h = ho_f32_to_f16(scale);
    out[0] = (uint8_t)(h & 0xff);
    out[1] = (uint8_t)(h >> 8);
    for (int j = 0; j < HO_QK / 2; j++) {
        int32_t lo = sat_i32(b[j] * inv + 8.5f);
        int32_t hi = sat_i32(b[j + HO_QK / 2] * inv + 8.5f);
        lo = lo < 0 ? 0 : (lo > 15 ? 15 : lo);
        hi = hi < 0 ? 0 : (hi > 15 ? 15 : hi);
        out[2 + j] = (uint8_t)(lo | (hi << 4));
    }
}

/* encode_row, quant.rs:274-292 */
void ho_encode_row(int d, const float* v, size_t n, uint8_t* out) {
    switch (d) {
    case HO_F32:
        memcpy(out, v, n * 4); /* little-endian host */
        break;
    case HO_F16:
        for (size_t i = 0; i < n; i++) {
            uint16_t h = ho_f32_to_f16(v[i]);
            out[2 * i] = (uint8_t)(h & 0xff);
            out[2 * i + 1] = (uint8_t)(h >> 8);
        }
        break;
    case HO_BF16:
        for (size_t i = 0; i < n; i++) {
            uint16_t h = ho_f32_to_bf16(v[i]);
            out[2 * i] = (uint8_t)(h & 0xff);
            out[2 * i + 1] = (uint8_t)(h >> 8);
        }
        break;
    case HO_Q8_0:
        for (size_t b = 0; b < n / HO_QK; b++) encode_block_q8_0(v + b * HO_QK, out + b * 34);
        break;
    case HO_Q4_0:
        for (size_t b = 0; b < n / HO_QK; b++) encode_block_q4_0(v + b * HO_QK, out + b * 18);
        break;
    }
}

/* decode_row, quant.rs:236-269 */
void ho_decode_row(int d, const uint8_t* row, size_t n, float* out) {
    switch (d) {
    case HO_F32:
        memcpy(out, row, n * 4);
        break;
    case HO_F16:
        for (size_t i = 0; i < n; i++) out[i] = ho_f16_to_f32(rd_u16(row + 2 * i));
        break;
    case HO_BF16:
        for (size_t i = 0; i < n; i++) out[i] = bf16_to_f32(rd_u16(row + 2 * i));
        break;
    case HO_Q8_0:
        for (size_t b = 0; b < n / HO_QK; b++) {
            const uint8_t* blk = row + b * 34;
            float s = ho_f16_to_f32(rd_u16(blk));
            for (int j = 0; j < HO_QK; j++) out[b * HO_QK + j] = s * (float)(int8_t)blk[2 + j];
        }
        break;
    case HO_Q4_0:
        for (size_t b = 0; b < n / HO_QK; b++) {
            const uint8_t* blk = row + b * 18;
            float s = ho_f16_to_f32(rd_u16(blk));
            for (int j = 0; j < HO_QK / 2; j++) {
                uint8_t byte = blk[2 + j];
                out[b * HO_QK + j] = s * ((float)(byte & 0x0f) - 8.0f);
                out[b * HO_QK + j + HO_QK / 2] = s * ((float)(byte >> 4) - 8.0f);
            }
        }
        break;
    }
}

/* ------------------------------------------------------------------------ */
/* activation quantization and quantized dots: quant.rs:70-144               */
/* ------------------------------------------------------------------------ */
void ho_quantize_q8(const float* x, size_t n, float* scales, int8_t* quants) {
    for (size_t b = 0; b < n / HO_QK; b++) {
        const float* blk = x + b * HO_QK;
        float amax = 0.0f;
        for (int j = 0; j < HO_QK; j++) amax = rmax(amax, fabsf(blk[j]));
        float scale = amax / 127.0f;
        float inv = scale > 0.0f ? 1.0f / scale : 0.0f;
        scales[b] = scale;
        for (int j = 0; j < HO_QK; j++) quants[b * HO_QK + j] = sat_i8(roundf(blk[j] * inv));
    }
}

/* dot_q8_0, quant.rs:115-127 */
static float dot_q8_0(const uint8_t* row, const float* xs, const int8_t* xq, size_t nb,
                      int32_t* sums) {
    float total = 0.0f;
    for (size_t b = 0; b < nb; b++) {
        const uint8_t* blk = row + b * 34;
        const int8_t* q = xq + b * HO_QK;
        int32_t isum = 0;
        for (int j = 0; j < HO_QK; j++) isum += (int32_t)(int8_t)blk[2 + j] * (int32_t)q[j];
        if (sums) sums[b] = isum;
        float ws = ho_f16_to_f32(rd_u16(blk));
        float t = ws * xs[b];
        t = t * (float)isum;
        total = total + t;
    }
    return total;
}

/* dot_q4_0, quant.rs:129-144 */
static float dot_q4_0(const uint8_t* row, const float* xs, const int8_t* xq, size_t nb,
                      int32_t* sums) {
    float total = 0.0f;
    for (size_t b = 0; b < nb; b++) {
        const uint8_t* blk = row + b * 18;
        const int8_t* q = xq + b * HO_QK;
        int32_t isum = 0;
        for (int j = 0; j < HO_QK / 2; j++) {
            int32_t lo = (int32_t)(blk[2 + j] & 0x0f) - 8;
            int32_t hi = (int32_t)(blk[2 + j] >> 4) - 8;
            isum += lo * (int32_t)q[j] + hi * (int32_t)q[j + HO_QK / 2];
        }
        if (sums) sums[b] = isum;
        float ws = ho_f16_to_f32(rd_u16(blk));
        float t = ws * xs[b];
        t = t * (float)isum;
        total = total + t;
    }
    return total;
}

float ho_dot_quantized(int d, const uint8_t* row, const float* xs, const int8_t* xq, size_t n,
                       int32_t* sums) {
    if (d == HO_Q8_0) return dot_q8_0(row, xs, xq, n / HO_QK, sums);
    if (d == HO_Q4_0) return dot_q4_0(row, xs, xq, n / HO_QK, sums);
    return NAN; /* the reference panics: dot_quantized with a float dtype */
}

/* ------------------------------------------------------------------------ */
/* float dots: quant.rs:32-41 (reduce), 146-202                              */
/* ------------------------------------------------------------------------ */
#define LANES 8
#define DECODE_BLOCK 64

static inline float reduce8(const float* a) {
    float x = (a[0] + a[4]) + (a[1] + a[5]);
    float y = (a[2] + a[6]) + (a[3] + a[7]);
    return x + y;
}

/* dot_lanes, quant.rs:152-160: accumulate whole groups of 8 into acc and
 * return the left-to-right sum of the remainder products. */
static float dot_lanes(const float* w, const float* x, size_t n, float* acc) {
    size_t full = n / LANES * LANES;
    for (size_t i = 0; i < full; i += LANES)
        for (int l = 0; l < LANES; l++) acc[l] = acc[l] + w[i + l] * x[i + l];
    float tail = -0.0f; /* <f32 as Sum>::sum starts at -0.0 */
    for (size_t i = full; i < n; i++) tail = tail + w[i] * x[i];
    return tail;
}

/* dot_decoded, quant.rs:166-184 */
static float dot_decoded(int d, const uint8_t* row, const float* x, size_t n) {
    float acc[LANES] = {0, 0, 0, 0, 0, 0, 0, 0};
    float tail = 0.0f;
    float buf[DECODE_BLOCK];
    size_t bpv = ho_block_bytes(d);
    for (size_t c = 0; c < n; c += DECODE_BLOCK) {
        size_t len = n - c < DECODE_BLOCK ? n - c : DECODE_BLOCK;
        ho_decode_row(d, row + c * bpv, len, buf);
        tail = tail + dot_lanes(buf, x + c, len, acc);
    }
    return reduce8(acc) + tail;
}

float ho_dot(int d, const uint8_t* row, const float* x, size_t n) {
    if (d == HO_F32) {
        /* dot_f32, quant.rs:186-194; the aligned and decoded routes agree */
        if (((uintptr_t)row & 3u) == 0) {
            float acc[LANES] = {0, 0, 0, 0, 0, 0, 0, 0};
            float tail = dot_lanes((const float*)(const void*)row, x, n, acc);
            return reduce8(acc) + tail;
        }
        return dot_decoded(d, row, x, n);
    }
    if (d == HO_F16 || d == HO_BF16) return dot_decoded(d, row, x, n); /* quant.rs:196-202 */
    /* quantized: quantize x on every call, quant.rs:64 */
    size_t nb = n / HO_QK;
    float* xs = (float*)malloc(nb * sizeof(float));
    int8_t* xq = (int8_t*)malloc(n);
    ho_quantize_q8(x, n, xs, xq);
    float r = ho_dot_quantized(d, row, xs, xq, n, NULL);
    free(xs);
    free(xq);
    return r;
}

/* ------------------------------------------------------------------------ */
/* matvec: matrix.rs:115-143                                                 */
/* ------------------------------------------------------------------------ */
#define ROWS_PER_TASK 32 /* matrix.rs:11 */

static void matvec_rows(int d, const uint8_t* w, size_t rows, size_t cols, const float* x,
                        float* out, int parallel, const float* xs, const int8_t* xq) {
    size_t rb = (size_t)ho_row_bytes(d, cols);
    long long n = (long long)rows;
    (void)parallel;
    if (xq) {
#pragma omp parallel for schedule(dynamic, ROWS_PER_TASK) if (parallel && rows >= 2 * ROWS_PER_TASK)
        for (long long r = 0; r < n; r++) out[r] = ho_dot_quantized(d, w + r * rb, xs, xq, cols, NULL);
    } else {
#pragma omp parallel for schedule(dynamic, ROWS_PER_TASK) if (parallel && rows >= 2 * ROWS_PER_TASK)
        for (long long r = 0; r < n; r++) out[r] = ho_dot(d, w + r * rb, x, cols);
    }
}

void ho_matvec(int d, const uint8_t* w, size_t rows, size_t cols, const float* x, float* out,
               int parallel) {
    if (ho_block_len(d) > 1) {
        /* quantize the input once; every row reuses it (matrix.rs:119-121) */
        size_t nb = cols / HO_QK;
        float* xs = (float*)malloc((nb ? nb : 1) * sizeof(float));
        int8_t* xq = (int8_t*)malloc(cols ? cols : 1);
        ho_quantize_q8(x, cols, xs, xq);
        matvec_rows(d, w, rows, cols, x, out, parallel, xs, xq);
        free(xs);
        free(xq);
    } else {
        matvec_rows(d, w, rows, cols, x, out, parallel, NULL, NULL);
    }
}

/* ------------------------------------------------------------------------ */
/* small ops: ops/activation.rs, ops/topk.rs, ops/norm.rs, ops/rope.rs       */
/* ------------------------------------------------------------------------ */
float ho_silu(float v) { return v / (1.0f + expf(-v)); }

void ho_softmax_in_place(float* x, size_t n) {
    float mx = -INFINITY;
    for (size_t i = 0; i < n; i++) mx = rmax(mx, x[i]);
    float sum = 0.0f;
    for (size_t i = 0; i < n; i++) {
        x[i] = expf(x[i] - mx);
        sum = sum + x[i];
    }
    for (size_t i = 0; i < n; i++) x[i] = x[i] / sum;
}

size_t ho_argmax(const float* x, size_t n) {
    size_t best = 0;
    for (size_t i = 0; i < n; i++)
        if (x[i] > x[best]) best = i;
    return best;
}

/* f32::total_cmp key: flip the magnitude bits of negatives so integer order
 * is the IEEE total order. */
static inline int32_t total_key(float f) {
    int32_t b = (int32_t)f_bits(f);
    return b ^ (int32_t)(((uint32_t)(b >> 31)) >> 1);
}
/* true when (sa, ia) ranks strictly before (sb, ib): higher score first,
 * lower index first on equal scores (topk.rs:27-35). */
static inline int ranks_before(float sa, uint32_t ia, float sb, uint32_t ib) {
    int32_t ka = total_key(sa), kb = total_key(sb);
    if (ka != kb) return ka > kb;
    return ia < ib;
}

size_t ho_top_k(const float* scores, size_t n, size_t k, uint32_t* index, float* score) {
    if (k > n) k = n;
    if (k == 0) return 0;
    size_t len = 0;
    /* keep a best-first list of size <= k; the order is total, so this
     * selects exactly what the reference's bounded heap selects */
    for (size_t i = 0; i < n; i++) {
        float s = scores[i];
        if (len == k && !ranks_before(s, (uint32_t)i, score[len - 1], index[len - 1])) continue;
        size_t pos = len < k ? len : k - 1;
        while (pos > 0 && ranks_before(s, (uint32_t)i, score[pos - 1], index[pos - 1])) {
            score[pos] = score[pos - 1];
            index[pos] = index[pos - 1];
            pos--;
        }
        score[pos] = s;
        index[pos] = (uint32_t)i;
        if (len < k) len++;
    }
    return len;
}

static float inverse_rms(const float* x, float eps, size_t n) {
    float s = -0.0f; /* Sum of v*v, left to right (norm.rs:27) */
    for (size_t i = 0; i < n; i++) s = s + x[i] * x[i];
    float mean_sq = s / (float)n;
    return 1.0f / sqrtf(mean_sq + eps);
}

void ho_rms_norm(const float* x, const float* w, float eps, float* out, size_t n) {
    float scale = inverse_rms(x, eps, n);
    for (size_t i = 0; i < n; i++) out[i] = (x[i] * scale) * w[i];
}

void ho_rms_norm_in_place(float* x, const float* w, float eps, size_t n) {
    float scale = inverse_rms(x, eps, n);
    for (size_t i = 0; i < n; i++) x[i] = x[i] * (scale * w[i]);
}

void ho_rope_inv_freq(size_t head_dim, float theta, float* inv_freq) {
    for (size_t i = 0; i < head_dim / 2; i++)
        inv_freq[i] = 1.0f / powf(theta, (float)(2 * i) / (float)head_dim);
}

void ho_rope_angles(const float* inv_freq, size_t half, size_t position, float* c, float* s) {
    for (size_t i = 0; i < half; i++) {
        float angle = (float)position * inv_freq[i];
        c[i] = cosf(angle);
        s[i] = sinf(angle);
    }
}

void ho_rope_apply(float* head, size_t hd, const float* c, const float* s) {
    size_t half = hd / 2;
    for (size_t i = 0; i < half; i++) {
        float a = head[i], b = head[half + i];
        head[i] = a * c[i] - b * s[i];
        head[half + i] = b * c[i] + a * s[i];
    }
}

/* ------------------------------------------------------------------------ */
/* experts and the MoE layer: expert/mod.rs:91-103, model/moe.rs:36-70      */
/* ------------------------------------------------------------------------ */
static void matrix_matvec(const ho_matrix* m, const float* x, float* out, int parallel) {
    ho_matvec(m->dtype, m->data, m->rows, m->cols, x, out, parallel);
}

void ho_expert_forward(const ho_expert* e, const float* x, float* out, int parallel) {
    size_t inter = e->gate.rows;
    float* g = (float*)malloc(inter * sizeof(float));
    float* u = (float*)malloc(inter * sizeof(float));
    /* rayon::join(gate, up): both independent, results identical either way */
    matrix_matvec(&e->gate, x, g, parallel);
    matrix_matvec(&e->up, x, u, parallel);
    for (size_t j = 0; j < inter; j++) g[j] = ho_silu(g[j]) * u[j];
    matrix_matvec(&e->down, g, out, parallel);
    free(g);
    free(u);
}

size_t ho_moe_route(const ho_matrix* router, size_t k, int normalize, const float* x,
                    uint32_t* expert_out, float* weight_out, int parallel) {
    size_t e = router->rows;
    float* probs = (float*)malloc(e * sizeof(float));
    float* score = (float*)malloc((k ? k : 1) * sizeof(float));
    matrix_matvec(router, x, probs, parallel);
    ho_softmax_in_place(probs, e);
    size_t n = ho_top_k(probs, e, k, expert_out, score);
    float norm = 1.0f;
    if (normalize) {
        norm = -0.0f;
        for (size_t i = 0; i < n; i++) norm = norm + score[i];
    }
    for (size_t i = 0; i < n; i++) weight_out[i] = score[i] / norm;
    free(probs);
    free(score);
    return n;
}

void ho_moe_forward(const ho_matrix* router, const ho_expert* experts, size_t n_experts,
                    size_t k, int normalize, const float* x, size_t tokens, float* out,
                    uint32_t* expert_out, float* weight_out, int parallel) {
    size_t h = router->cols;
    uint32_t* idx = (uint32_t*)malloc((k ? k : 1) * sizeof(uint32_t));
    float* w = (float*)malloc((k ? k : 1) * sizeof(float));
    float* tmp = (float*)malloc(h * sizeof(float));
    (void)n_experts;
    for (size_t t = 0; t < tokens; t++) {
        const float* xt = x + t * h;
        float* ot = out + t * h;
        size_t n = ho_moe_route(router, k, normalize, xt, idx, w, parallel);
        for (size_t j = 0; j < h; j++) ot[j] = 0.0f;
        for (size_t r = 0; r < n; r++) {
            ho_expert_forward(&experts[idx[r]], xt, tmp, parallel);
            for (size_t j = 0; j < h; j++) ot[j] = ot[j] + w[r] * tmp[j];
        }
        if (expert_out)
            for (size_t r = 0; r < k; r++) expert_out[t * k + r] = r < n ? idx[r] : 0xffffffffu;
        if (weight_out)
            for (size_t r = 0; r < k; r++) weight_out[t * k + r] = r < n ? w[r] : 0.0f;
    }
    free(idx);
    free(w);
    free(tmp);
}

/* ------------------------------------------------------------------------ */
/* sampling: generate/sampler.rs                                             */
/* ------------------------------------------------------------------------ */
uint64_t ho_xorshift_seed(uint64_t seed) { return seed > 1 ? seed : 1; }

uint64_t ho_xorshift_next_u64(uint64_t* s) {
    uint64_t x = *s;
    x ^= x >> 12;
    x ^= x << 25;
    x ^= x >> 27;
    *s = x;
    return x * 0x2545F4914F6CDD1DULL;
}

float ho_xorshift_next_f32(uint64_t* s) {
    return (float)(ho_xorshift_next_u64(s) >> 40) / (float)(1ULL << 24);
}

void ho_apply_repetition_penalty(float* logits, size_t v, const int32_t* seen, size_t n_seen,
                                 float penalty) {
    if (!seen || n_seen == 0 || penalty == 1.0f) return;
    unsigned char* done = (unsigned char*)calloc(v ? v : 1, 1);
    for (size_t i = 0; i < n_seen; i++) {
        int32_t id = seen[i];
        if (id < 0 || (size_t)id >= v || done[id]) continue;
        done[id] = 1;
        float l = logits[id];
        logits[id] = l > 0.0f ? l / penalty : l * penalty;
    }
    free(done);
}

typedef struct {
    uint32_t index;
    float value;
} cand;

static int cand_cmp(const void* a, const void* b) {
    const cand* x = (const cand*)a;
    const cand* y = (const cand*)b;
    if (ranks_before(x->value, x->index, y->value, y->index)) return -1;
    if (ranks_before(y->value, y->index, x->value, x->index)) return 1;
    return 0;
}

uint32_t ho_sample(const float* logits, size_t v, float temperature, float top_p, size_t top_k,
                   uint64_t* rng, void* scratch) {
    if (temperature <= 0.0f) return (uint32_t)ho_argmax(logits, v); /* sampler.rs:55-61 */
    if (v == 0) return 0;
    cand* c = scratch ? (cand*)scratch : (cand*)malloc(v * sizeof(cand));
    size_t k = top_k == 0 ? v : (top_k < v ? top_k : v);
    size_t n;
    if (k < v) {
        /* select_nth_unstable_by(k-1) + truncate(k): the k best by logit */
        uint32_t* idx = (uint32_t*)malloc(k * sizeof(uint32_t));
        float* sc = (float*)malloc(k * sizeof(float));
        n = ho_top_k(logits, v, k, idx, sc);
        for (size_t i = 0; i < n; i++) {
            c[i].index = idx[i];
            c[i].value = sc[i];
        }
        free(idx);
        free(sc);
    } else {
        for (size_t i = 0; i < v; i++) {
            c[i].index = (uint32_t)i;
            c[i].value = logits[i];
        }
        n = v;
        qsort(c, n, sizeof(cand), cand_cmp);
    }
    /* softmax with temperature over the survivors, sampler.rs:96-101 */
    float mx = c[0].value, total = 0.0f;
    for (size_t i = 0; i < n; i++) {
        c[i].value = expf((c[i].value - mx) / temperature);
        total = total + c[i].value;
    }
    /* nucleus cut, sampler.rs:103-112 */
    float mass = 0.0f;
    size_t keep = n;
    for (size_t i = 0; i < n; i++) {
        mass = mass + c[i].value / total;
        if (mass >= top_p) {
            keep = i + 1;
            break;
        }
    }
    float kept = -0.0f;
    for (size_t i = 0; i < keep; i++) kept = kept + c[i].value;
    float r = ho_xorshift_next_f32(rng) * kept;
    uint32_t out = c[keep - 1].index;
    for (size_t i = 0; i < keep; i++) {
        r = r - c[i].value;
        if (r <= 0.0f) {
            out = c[i].index;
            break;
        }
    }
    if (!scratch) free(c);
    return out;
}

/* ------------------------------------------------------------------------ */
/* full decoder: model/transformer.rs:168-227, model/attention.rs:31-86      */
/* ------------------------------------------------------------------------ */
static void ffn_forward(const ho_model* m, const ho_layer* L, const float* x, float* out,
                        int parallel) {
    if (!L->is_moe) {
        ho_expert_forward(&L->dense, x, out, parallel);
        return;
    }
    ho_moe_forward(&L->router, L->experts, m->n_experts, m->top_k, m->normalize_topk, x, 1, out,
                   NULL, NULL, parallel);
}

static void attention_forward(const ho_model* m, const ho_layer* L, const float* x, size_t pos,
                              const float* cs, const float* sn, float* kc, float* vc, float* out,
                              int parallel) {
    size_t hd = m->head_dim, nh = m->n_heads, kvd = m->n_kv_heads * hd;
    float* q = (float*)malloc(nh * hd * sizeof(float));
    float* k = (float*)malloc(kvd * sizeof(float));
    float* v = (float*)malloc(kvd * sizeof(float));
    matrix_matvec(&L->q, x, q, parallel);
    matrix_matvec(&L->k, x, k, parallel);
    matrix_matvec(&L->v, x, v, parallel);
    for (size_t h = 0; h < nh; h++) {
        if (L->q_norm) ho_rms_norm_in_place(q + h * hd, L->q_norm, m->eps, hd);
        ho_rope_apply(q + h * hd, hd, cs, sn);
    }
    for (size_t h = 0; h < m->n_kv_heads; h++) {
        if (L->k_norm) ho_rms_norm_in_place(k + h * hd, L->k_norm, m->eps, hd);
        ho_rope_apply(k + h * hd, hd, cs, sn);
    }
    memcpy(kc + pos * kvd, k, kvd * sizeof(float));
    memcpy(vc + pos * kvd, v, kvd * sizeof(float));
    size_t seq = pos + 1, group = nh / m->n_kv_heads;
    float scale = 1.0f / sqrtf((float)hd);
    float* ctx = (float*)calloc(nh * hd, sizeof(float));
    float* scores = (float*)malloc(seq * sizeof(float));
    for (size_t h = 0; h < nh; h++) {
        size_t off = (h / group) * hd;
        const float* qh = q + h * hd;
        for (size_t t = 0; t < seq; t++) {
            const float* key = kc + t * kvd + off;
            float s = -0.0f;
            for (size_t i = 0; i < hd; i++) s = s + qh[i] * key[i];
            scores[t] = s * scale;
        }
        ho_softmax_in_place(scores, seq);
        float* c = ctx + h * hd;
        for (size_t t = 0; t < seq; t++) {
            const float* val = vc + t * kvd + off;
            for (size_t i = 0; i < hd; i++) c[i] = c[i] + scores[t] * val[i];
        }
    }
    matrix_matvec(&L->o, ctx, out, parallel);
    free(q);
    free(k);
    free(v);
    free(ctx);
    free(scores);
}

int ho_model_forward(const ho_model* m, uint32_t token, uint32_t position, float* kcache,
                     float* vcache, uint32_t max_len, float* hidden_out, float* logits,
                     int parallel) {
    if (position >= max_len || token >= m->vocab) return -1;
    size_t h = m->hidden, hd = m->head_dim, half = hd / 2, kvd = m->n_kv_heads * hd;
    float* x = (float*)malloc(h * sizeof(float));
    float* normed = (float*)malloc(h * sizeof(float));
    float* delta = (float*)malloc(h * sizeof(float));
    float* inv = (float*)malloc(half * sizeof(float));
    float* cs = (float*)malloc(half * sizeof(float));
    float* sn = (float*)malloc(half * sizeof(float));
    size_t rb = (size_t)ho_row_bytes(m->embed.dtype, h);
    ho_decode_row(m->embed.dtype, m->embed.data + (size_t)token * rb, h, x);
    ho_rope_inv_freq(hd, m->rope_theta, inv);
    ho_rope_angles(inv, half, position, cs, sn);
    for (size_t l = 0; l < m->n_layers; l++) {
        const ho_layer* L = &m->layers[l];
        float* kc = kcache + l * (size_t)max_len * kvd;
        float* vc = vcache + l * (size_t)max_len * kvd;
        ho_rms_norm(x, L->input_norm, m->eps, normed, h);
        attention_forward(m, L, normed, position, cs, sn, kc, vc, delta, parallel);
        for (size_t i = 0; i < h; i++) x[i] = x[i] + delta[i];
        ho_rms_norm(x, L->post_norm, m->eps, normed, h);
        ffn_forward(m, L, normed, delta, parallel);
        for (size_t i = 0; i < h; i++) x[i] = x[i] + delta[i];
    }
    ho_rms_norm(x, m->final_norm, m->eps, normed, h);
    if (hidden_out) memcpy(hidden_out, normed, h * sizeof(float));
    if (logits) matrix_matvec(&m->lm_head, normed, logits, parallel);
    free(x);
    free(normed);
    free(delta);
    free(inv);
    free(cs);
    free(sn);
    return 0;
}

void ho_expf_batch(const float* x, float* y, size_t n) {
    long long nn = (long long)n;
#pragma omp parallel for schedule(static) if (n > 65536)
    for (long long i = 0; i < nn; i++) y[i] = expf(x[i]);
}

int ho_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* Threads of the parallel regions (the reference's rayon pool uses every
 * core; a launcher such as torchrun may have set OMP_NUM_THREADS=1). */
void ho_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}
