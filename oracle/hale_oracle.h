/*
 * hale_oracle.h -- CPU restatement of Hale-Token's MoE / sampling path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker the CUDA path is
 * compared against (tests/, __graft_entry__.smoke(), and bench.py's
 * cpu_baseline / --impl reference legs). Nothing in the product library
 * (libhale_cuda.so) links, loads or calls it.
 *
 * Every function restates the Rust reference (basaanithanaveenkumar/
 * Hale-Token, crate `hale`) and cites the file:line it follows. The bit-level
 * rules that make the restatement exact:
 *   - compiled with -ffp-contract=off and without fast-math: Rust never fuses
 *     a*b+c into an FMA;
 *   - f32::round is round-half-away-from-zero (C roundf);
 *   - Rust `as i8` / `as i32` float casts saturate and send NaN to 0;
 *   - f32::exp/powf/sin/cos come from the platform libm (glibc here);
 *   - iterator sums of f32 fold left to right.
 *
 * Parity pins: tests/test_oracle_*.py restate every reference unit test on
 * this path and check the two reference golden fixtures
 * (tests/fixtures/{tiny-qwen3-moe,tiny-mixtral}/expected.json).
 */
#ifndef HALE_ORACLE_H
#define HALE_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* DType discriminants, src/tensor/dtype.rs:15-25 (declaration order). */
enum { HO_F32 = 0, HO_F16 = 1, HO_BF16 = 2, HO_Q8_0 = 3, HO_Q4_0 = 4 };
#define HO_QK 32 /* src/tensor/dtype.rs:28 */

/* ---- formats: src/tensor/dtype.rs, src/tensor/quant.rs ---------------- */
size_t ho_block_len(int dtype);                 /* dtype.rs:32-37 */
size_t ho_block_bytes(int dtype);               /* dtype.rs:40-47 */
int64_t ho_row_bytes(int dtype, size_t cols);   /* dtype.rs:53-61; -1 = error */
uint16_t ho_f32_to_f16(float v);                /* half::f16::from_f32 (RNE) */
float ho_f16_to_f32(uint16_t h);                /* half::f16::to_f32 */
uint16_t ho_f32_to_bf16(float v);               /* half::bf16::from_f32 (RNE) */
void ho_encode_row(int dtype, const float* values, size_t n, uint8_t* out); /* quant.rs:274-321 */
void ho_decode_row(int dtype, const uint8_t* row, size_t n, float* out);    /* quant.rs:236-269 */

/* Q8Activations::quantize, quant.rs:77-93. scales[n/32], quants[n]. */
void ho_quantize_q8(const float* x, size_t n, float* scales, int8_t* quants);
/* dot_quantized, quant.rs:107-144. block_sums (nullable) receives the
 * per-block int32 sum of each block. */
float ho_dot_quantized(int dtype, const uint8_t* row, const float* xs, const int8_t* xq,
                       size_t n, int32_t* block_sums);
/* dot, quant.rs:59-66 with the float kernels 146-202. */
float ho_dot(int dtype, const uint8_t* row, const float* x, size_t n);

/* WeightMatrix::matvec (parallel over rows, >=32 rows per task) and
 * matvec_serial, matrix.rs:115-143. Results are bit-identical. */
void ho_matvec(int dtype, const uint8_t* w, size_t rows, size_t cols, const float* x,
               float* out, int parallel);

/* ---- small ops: src/ops ------------------------------------------------ */
float ho_silu(float v);                          /* activation.rs:5-7 */
void ho_softmax_in_place(float* x, size_t n);    /* activation.rs:11-21 */
size_t ho_argmax(const float* x, size_t n);      /* activation.rs:24-32 */
/* top_k, topk.rs:44-61 (order: topk.rs:27-35). Returns the count written. */
size_t ho_top_k(const float* scores, size_t n, size_t k, uint32_t* index, float* score);
void ho_rms_norm(const float* x, const float* w, float eps, float* out, size_t n); /* norm.rs:7-15 */
void ho_rms_norm_in_place(float* x, const float* w, float eps, size_t n);          /* norm.rs:18-24 */
void ho_rope_inv_freq(size_t head_dim, float theta, float* inv_freq);              /* rope.rs:15-21 */
void ho_rope_angles(const float* inv_freq, size_t half, size_t position, float* cos_out,
                    float* sin_out);                                               /* rope.rs:26-32 */
void ho_rope_apply(float* head, size_t head_dim, const float* cos_v, const float* sin_v); /* rope.rs:35-43 */

/* ---- MoE: src/model/moe.rs, src/expert/mod.rs --------------------------- */
typedef struct {
    int32_t dtype;
    uint32_t rows, cols;
    const uint8_t* data; /* rows * row_bytes(cols) bytes */
} ho_matrix;

typedef struct {
    ho_matrix gate, up, down; /* [I,H], [I,H], [H,I]: expert/mod.rs:75-83 */
} ho_expert;

/* Expert::forward, expert/mod.rs:91-103. */
void ho_expert_forward(const ho_expert* e, const float* x, float* out, int parallel);
/* MoeLayer::route, moe.rs:36-53. Writes k (expert index, weight) pairs
 * best-first; returns the count. */
size_t ho_moe_route(const ho_matrix* router, size_t k, int normalize_topk, const float* x,
                    uint32_t* expert_out, float* weight_out, int parallel);
/* MoeLayer::forward, moe.rs:56-70, for `tokens` independent rows of x
 * ([tokens, H] -> [tokens, H]). experts[e] is expert e of this layer.
 * expert_out/weight_out (nullable) receive [tokens, k]. */
void ho_moe_forward(const ho_matrix* router, const ho_expert* experts, size_t n_experts,
                    size_t k, int normalize_topk, const float* x, size_t tokens, float* out,
                    uint32_t* expert_out, float* weight_out, int parallel);

/* ---- sampling: src/generate/sampler.rs -------------------------------- */
uint64_t ho_xorshift_next_u64(uint64_t* state); /* sampler.rs:135-140 */
float ho_xorshift_next_f32(uint64_t* state);    /* sampler.rs:143-145 */
uint64_t ho_xorshift_seed(uint64_t seed);       /* sampler.rs:131-133 */
/* Repetition penalty (not in the reference; HF convention, applied to each
 * distinct seen id before temperature). */
void ho_apply_repetition_penalty(float* logits, size_t v, const int32_t* seen, size_t n_seen,
                                 float penalty);
/* SamplingParams::build + Sampler::sample, sampler.rs:55-61, 14-18, 80-123.
 * temperature <= 0 -> greedy. top_k == 0 disables top-k. Tied logits are
 * ordered by lower index first. `scratch` needs 2*v floats + v uint32s
 * worth of bytes (12*v); pass NULL to allocate internally. */
uint32_t ho_sample(const float* logits, size_t v, float temperature, float top_p, size_t top_k,
                   uint64_t* rng_state, void* scratch);

/* ---- full decoder (golden-fixture pin): src/model/ ----------------------- */
typedef struct {
    const float* input_norm;        /* [H] */
    const float* post_norm;         /* [H] */
    ho_matrix q, k, v, o;
    const float* q_norm;            /* [head_dim] or NULL (Mixtral) */
    const float* k_norm;
    int32_t is_moe;
    ho_expert dense;                /* when !is_moe */
    ho_matrix router;               /* when is_moe */
    const ho_expert* experts;       /* [n_experts] when is_moe */
} ho_layer;

typedef struct {
    uint32_t hidden, n_layers, n_heads, n_kv_heads, head_dim, vocab, n_experts, top_k;
    int32_t normalize_topk;
    float eps, rope_theta;
    ho_matrix embed, lm_head;
    const float* final_norm;
    const ho_layer* layers;
} ho_model;

/* Transformer::forward (transformer.rs:168-227) for the token at
 * `position`. kcache/vcache are [n_layers][max_len][n_kv*head_dim] and are
 * appended at `position`. logits (nullable) receives [vocab]. Returns 0, or
 * -1 on a bad token / position. */
int ho_model_forward(const ho_model* m, uint32_t token, uint32_t position, float* kcache,
                     float* vcache, uint32_t max_len, float* hidden_out, float* logits,
                     int parallel);

/* y[i] = expf(x[i]) from this platform's libm: what Rust's f32::exp calls
 * on Linux. Used to check the CUDA library's own exp against. */
void ho_expf_batch(const float* x, float* y, size_t n);

/* Threads OpenMP will use (1 when built without OpenMP). */
int ho_num_threads(void);
void ho_set_num_threads(int n);

#ifdef __cplusplus
}
#endif
#endif
