/*
 * hale_cuda.h -- C ABI of the B200 (sm_100a) implementation of Hale-Token's
 * MoE quantized-expert forward and sampling tail.
 *
 * The entry points replace the Rust reference's operator surface on this
 * path (paths relative to the reference crate):
 *   ExpertProvider / ExpertCache ........ src/expert/mod.rs:128-137, src/expert/cache.rs:124-203
 *   ExpertSource::load (pack record) .... src/expert/pack.rs:264-271
 *   WeightMatrix::new / matvec .......... src/tensor/matrix.rs:29-45, 115-126
 *   Q8Activations::quantize ............. src/tensor/quant.rs:77-93
 *   quant::dot_quantized ................ src/tensor/quant.rs:107-144
 *   MoeLayer::route / forward ........... src/model/moe.rs:36-70
 *   Transformer::logits (lm_head) ....... src/model/transformer.rs:217-221
 *   Sampler::sample / SamplingParams .... src/generate/sampler.rs:7-123
 *
 * Conventions (mirroring the reference):
 *   - Every function returns hale_status: 0 = OK, negative = error. Negative
 *     codes mirror HaleError kinds (src/error.rs:10-57) plus CUDA / timeout
 *     codes. Nothing panics or aborts across this boundary; a message for
 *     the last failure is available from hale_last_error().
 *   - Buffers are caller-owned. Unless a name ends in _host, data pointers
 *     are DEVICE pointers on the context's GPU, and work is enqueued on the
 *     given stream (a cudaStream_t passed as void*; NULL = legacy stream).
 *   - f32 activation buffers (x) start on a 16-byte boundary (any
 *     cudaMalloc / torch allocation does); misaligned ones are rejected.
 *   - A hale_ctx is bound to one GPU. Calls on one ctx must not overlap
 *     (the ctx owns one workspace); use one ctx per host thread / stream.
 *   - Results are deterministic: bit-identical run to run, and bit-identical
 *     to the reference's CPU arithmetic (f32, no FMA contraction, glibc expf)
 *     for the quantized expert path, router top-k and greedy sampling.
 */
#ifndef HALE_CUDA_H
#define HALE_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define HALE_API __attribute__((visibility("default")))
#else
#define HALE_API
#endif

typedef int32_t hale_status;

/* Status codes. The first group mirrors HaleError (src/error.rs:10-57). */
#define HALE_OK 0
#define HALE_E_INVALID_ARGUMENT (-1) /* HaleError::InvalidArgument */
#define HALE_E_BAD_TENSOR (-2)       /* HaleError::BadTensor */
#define HALE_E_IO (-3)               /* HaleError::Io */
#define HALE_E_CONTEXT_OVERFLOW (-4) /* HaleError::ContextOverflow */
#define HALE_E_CUDA (-10)            /* a CUDA runtime call failed */
#define HALE_E_NO_DEVICE (-11)       /* no usable sm_100 device */
#define HALE_E_OUT_OF_MEMORY (-12)   /* device allocation failed */
#define HALE_E_TIMEOUT (-13)         /* a device-side wait hit its bound */
#define HALE_E_DEVICE_CHECK (-14)    /* a device-side bounds check tripped */
#define HALE_E_UNSUPPORTED (-15)     /* valid request this build does not serve */
#define HALE_E_NCCL (-16)            /* an NCCL call failed (communicator set-up) */

/* Storage formats, same discriminants as DType (src/tensor/dtype.rs:15-25). */
typedef enum {
    HALE_F32 = 0,
    HALE_F16 = 1,
    HALE_BF16 = 2,
    HALE_Q8_0 = 3, /* 34-byte blocks: f16 scale + 32 x i8 */
    HALE_Q4_0 = 4  /* 18-byte blocks: f16 scale + 16 B nibbles (j | j+16) */
} hale_dtype;

typedef struct hale_ctx hale_ctx;       /* one GPU + workspace */
typedef struct hale_matrix hale_matrix; /* a WeightMatrix resident in HBM */
typedef struct hale_pool hale_pool;     /* HBM-resident expert store */

/* ---- context ------------------------------------------------------------ */

/* Binds to CUDA device `device` (must be compute capability 10.x). */
HALE_API hale_status hale_ctx_create(int device, hale_ctx** out);
HALE_API void hale_ctx_destroy(hale_ctx* ctx);
/* Copies the message of the last failure on `ctx` (or, with ctx == NULL, of
 * the last failure on this host thread) into buf. Returns its status. */
HALE_API hale_status hale_last_error(const hale_ctx* ctx, char* buf, size_t len);
/* Waits for the ctx's work on `stream` and reports device-side errors
 * (HALE_E_TIMEOUT / HALE_E_DEVICE_CHECK) raised by kernels since the last
 * check; clears them. */
HALE_API hale_status hale_ctx_check(hale_ctx* ctx, void* stream);
/* Number of this library's kernels launched on ctx so far. */
HALE_API uint64_t hale_ctx_launch_count(const hale_ctx* ctx);
/* Expert-kernel family of a context's MoE forwards (default HALE_EXPERT_AUTO:
 * chosen per call from the batch shape). The others force one family wherever
 * the layer's shapes allow it: all give bit-identical results; they differ
 * only in speed. Settings are per context; nothing is read from the process
 * environment. */
#define HALE_EXPERT_AUTO 0 /* by batch shape */
#define HALE_EXPERT_TC 1   /* tcgen05 kind::i8 kernels (TMEM accumulators) */
#define HALE_EXPERT_DP4A 2 /* per-CTA kernels: dp4a, warp MMA from 3 tokens */
#define HALE_EXPERT_PS 3   /* persistent streaming warp-MMA kernels */
#define HALE_EXPERT_WS 4   /* warp-specialised streaming: TMA tensor loads, warp MMA */
HALE_API hale_status hale_ctx_set_expert_kernel(hale_ctx* ctx, int family);
/* Per-kernel timing: while enabled, every launch on ctx is bracketed by a
 * pair of CUDA events on its stream. hale_ctx_profile_read synchronises,
 * and returns the launches and summed device milliseconds recorded for the
 * kernel family `kernel` ("router", "expert_gate_up", "expert_down",
 * "qgemv", "fgemv", "sample", ...) since the last reset, then resets it. */
HALE_API hale_status hale_ctx_profile(hale_ctx* ctx, int enable);
HALE_API hale_status hale_ctx_profile_read(hale_ctx* ctx, const char* kernel, uint64_t* launches,
                                           double* total_ms);

/* ---- formats (src/tensor/dtype.rs) ---------------------------------------- */

/* DType::row_bytes (dtype.rs:53-61); returns -1 when cols is not a
 * multiple of the block length or dtype is unknown. */
HALE_API int64_t hale_row_bytes(hale_dtype dtype, uint64_t cols);

/* ---- weight matrices (src/tensor/matrix.rs) ------------------------------- */

/* WeightMatrix::new (matrix.rs:29-45): takes `rows` encoded rows (the
 * reference byte layout: row-major, GGML blocks for q8_0/q4_0) from
 * `encoded` (device memory when on_device != 0, else host memory), checks
 * the byte count and repacks them into the GPU tile layout. */
HALE_API hale_status hale_matrix_create(hale_ctx* ctx, hale_dtype dtype, uint32_t rows, uint32_t cols,
                               const void* encoded, uint64_t encoded_bytes, int on_device,
                               hale_matrix** out);
HALE_API void hale_matrix_destroy(hale_matrix* m);

/* WeightMatrix::matvec (matrix.rs:115-126) for `m_rows` independent inputs:
 * out[t, r] = dot(row r, x[t, :]). x is [m_rows, cols] f32, out is
 * [m_rows, rows] f32 (device). Quantized matrices quantize each x row once
 * (quant.rs:77-93), exactly like the reference. block_sums (nullable,
 * quantized only) receives the int32 block dot products
 * [m_rows, rows, cols/32] -- the bit-exact intermediate of dot_q8_0 /
 * dot_q4_0 (quant.rs:115-144). */
HALE_API hale_status hale_matrix_matvec(hale_ctx* ctx, const hale_matrix* m, const float* x,
                               uint32_t m_rows, float* out, int32_t* block_sums, void* stream);

/* quant::dot_quantized applied to every row with caller-supplied quantized
 * activations (Q8Activations: scales [m_rows, cols/32] f32 and quants
 * [m_rows, cols] i8, device). Same outputs as hale_matrix_matvec. */
HALE_API hale_status hale_matrix_matvec_q8(hale_ctx* ctx, const hale_matrix* m, const float* x_scales,
                                  const int8_t* x_quants, uint32_t m_rows, float* out,
                                  int32_t* block_sums, void* stream);

/* Q8Activations::quantize (quant.rs:77-93) for [m_rows, cols] f32 rows. */
HALE_API hale_status hale_quantize_q8(hale_ctx* ctx, const float* x, uint32_t m_rows, uint32_t cols,
                             float* scales, int8_t* quants, void* stream);

/* ---- expert pool: ExpertProvider (src/expert/mod.rs:128-137) -------------- */

/* CacheStats (src/expert/cache.rs:15-33). Every expert of the pool lives in
 * HBM, so requests are served from the pinned tier; `misses` counts requests
 * for experts that were never uploaded (which fail). */
typedef struct {
    uint64_t pinned_hits;
    uint64_t lru_hits;
    uint64_t misses;
    uint64_t bytes_loaded;   /* bytes uploaded into HBM */
    double load_seconds;     /* host wall time spent uploading */
    uint64_t pinned_experts; /* experts resident in HBM */
    uint64_t pinned_bytes;
    uint64_t lru_experts;
    uint64_t lru_bytes;
    uint64_t lru_capacity_bytes;
    int32_t passthrough;
} hale_cache_stats;

/* ExpertKey (src/expert/mod.rs:50-62). */
typedef struct {
    uint32_t layer;
    uint32_t expert;
} hale_expert_key;

/* Device view of one resident expert, returned by hale_pool_fetch. */
typedef struct {
    const void* gate; /* tiled [I, H] */
    const void* up;   /* tiled [I, H] */
    const void* down; /* tiled [H, I] */
} hale_expert_view;

/* Creates an HBM store for n_layers x n_experts SwiGLU experts of shape
 * gate/up [inter, hidden], down [hidden, inter] in `dtype` (q8_0 or q4_0).
 * hidden and inter must be multiples of 32. */
HALE_API hale_status hale_pool_create(hale_ctx* ctx, hale_dtype dtype, uint32_t hidden, uint32_t inter,
                             uint32_t n_layers, uint32_t n_experts, hale_pool** out);
HALE_API void hale_pool_destroy(hale_pool* pool);

/* Uploads one expert from a pack record -- gate | up | down in the pack's
 * byte layout, exactly what PackExpertSource::load reads (pack.rs:264-271,
 * decode_record 125-133). `record` is host memory (on_device = 0) or device
 * memory (on_device != 0); the record is repacked into the tile layout. */
HALE_API hale_status hale_pool_upload_expert(hale_pool* pool, uint32_t layer, uint32_t expert,
                                    const void* record, uint64_t record_bytes, int on_device,
                                    void* stream);

/* ExpertProvider::fetch (mod.rs:128-137, cache.rs:124-194): resolves keys in
 * request order, records routing counts and cache counters. */
HALE_API hale_status hale_pool_fetch(hale_pool* pool, const hale_expert_key* keys, uint64_t n,
                            hale_expert_view* out);
/* ExpertProvider::stats (cache.rs:196-198). Includes routes served by
 * hale_moe_forward on device (read back, which synchronises the ctx). */
HALE_API hale_status hale_pool_stats(hale_pool* pool, hale_cache_stats* out);
/* ExpertProvider::routing_stats: counts[n_layers * n_experts] (u64). */
HALE_API hale_status hale_pool_routing_counts(hale_pool* pool, uint64_t* counts, uint64_t n);
/* Bytes of one expert record (ExpertSource::expert_bytes). */
HALE_API uint64_t hale_pool_expert_bytes(const hale_pool* pool);

/* ---- tiered expert pool: ExpertCache (src/expert/cache.rs:66-194) --------- */

/* CachePolicy (cache.rs:58-64): keys kept in HBM for the pool's life (tier 0)
 * and the byte budget of the HBM LRU tier (tier 1), counted in record bytes
 * like LruCache's weights (cache.rs:178, lru.rs:97-125). */
typedef struct {
    const hale_expert_key* pinned;
    uint64_t n_pinned;
    uint64_t lru_bytes;
} hale_cache_policy;

/* A pool for experts that do not all fit in HBM. hale_pool_upload_expert
 * fills the cold tier: every expert's tiled bytes in pinned host memory (the
 * pack read once into page-locked RAM; PackExpertSource, pack.rs:211-271, is
 * the reference's tier 2). HBM holds the policy's pinned experts, an LRU of
 * the others, and one forward's working set. hale_moe_forward then reads the
 * routes back, resolves them through the tiers with ExpertCache::fetch's
 * counters (one request per token, top-k order) and brings misses in with
 * asynchronous host-to-device copies on a side stream before the expert
 * kernels, which read every expert through a slot table: results are
 * identical to a resident pool's. Tiered forwards block the calling thread
 * until the routes are known and cannot be captured into a CUDA graph.
 * Device views from hale_pool_fetch stay valid until the next fetch or
 * forward on the pool. */
HALE_API hale_status hale_pool_create_tiered(hale_ctx* ctx, hale_dtype dtype, uint32_t hidden, uint32_t inter,
                                    uint32_t n_layers, uint32_t n_experts, const hale_cache_policy* policy,
                                    hale_pool** out);
/* ExpertSource::load (src/expert/mod.rs:110-124) for a tiered pool: when a
 * request names an expert that was never uploaded, the pool calls
 * fn(user, layer, expert, record, record_bytes) on the calling thread to
 * fill `record` with that expert's pack record (gate | up | down, the bytes
 * PackExpertSource::load returns, pack.rs:264-271) and return 0; the record
 * then enters the host tier as hale_pool_upload_expert would put it there.
 * A nonzero return fails the forward (or fetch) with HALE_E_IO before any
 * cache counter or slot changes, and the next request asks the source again.
 * fn NULL removes the source (never-uploaded experts are then an error). */
typedef int32_t (*hale_expert_source_fn)(void* user, uint32_t layer, uint32_t expert, void* record,
                                         uint64_t record_bytes);
HALE_API hale_status hale_pool_set_source(hale_pool* pool, hale_expert_source_fn fn, void* user);
/* Number of HBM expert slots of a pool (n_layers * n_experts when resident). */
HALE_API uint64_t hale_pool_hbm_slots(const hale_pool* pool);

/* ---- the MoE layer (src/model/moe.rs:25-70) ---------------------------- */

/* Router description for MoeLayer (moe.rs:25-32): `router` is the [E, H]
 * router matrix in reference encoding (f32 / f16 / bf16 rows, device). */
typedef struct {
    uint32_t layer;
    const void* router;
    hale_dtype router_dtype;
    uint32_t n_experts;
    uint32_t top_k;
    int32_t normalize_topk;
} hale_moe_layer;

/* MoeLayer::forward (moe.rs:56-70) for m_tokens independent tokens:
 * out[t] = sum over the top-k routes of weight * Expert(x[t]), combined in
 * best-first order. x, out: [m_tokens, H] f32 (device). topk_idx / topk_w
 * (nullable): [m_tokens, top_k] expert ids (i32) and weights (f32), the
 * output of MoeLayer::route (moe.rs:36-53). */
HALE_API hale_status hale_moe_forward(hale_ctx* ctx, hale_pool* pool, const hale_moe_layer* layer,
                             const float* x, uint32_t m_tokens, float* out, int32_t* topk_idx,
                             float* topk_w, void* stream);
/* Same with host buffers: copies x in, runs, copies out, and synchronises. */
HALE_API hale_status hale_moe_forward_host(hale_ctx* ctx, hale_pool* pool, const hale_moe_layer* layer,
                                  const float* x_host, uint32_t m_tokens, float* out_host,
                                  int32_t* topk_idx_host, float* topk_w_host, void* stream);
/* MoeLayer::route only (moe.rs:36-53): top-k expert ids and weights. */
HALE_API hale_status hale_moe_route(hale_ctx* ctx, const hale_moe_layer* layer, uint32_t hidden,
                           const float* x, uint32_t m_tokens, int32_t* topk_idx, float* topk_w,
                           float* probs, void* stream);

/* Routing that allocates nothing. No counterpart in the reference: it exists
 * for hosts that cannot call cudaMalloc on the routing path -- a serving loop
 * that must not add the device-wide synchronisation an allocation can cause
 * in the middle of a decode step, or an embedding that hands all device
 * memory to its own fixed arena up front. Same arguments and results as
 * hale_moe_route, without a context: it runs on the calling thread's current
 * device. Its scratch (router logits and a few counters) is a fixed 1 MiB
 * array inside this library, held on every GPU that loads the library until
 * the process exits, so m_tokens * n_experts must be at most 261,888 and
 * m_tokens at most 1016 (larger requests are rejected with
 * HALE_E_INVALID_ARGUMENT). The first call on a device looks up that array's
 * device address and keeps it for the life of the device's primary context
 * (a host that resets the device must not call this entry point again in
 * the same process); make that first call before any stream capture. Calls
 * share the array: calls that overlap on the GPU race, so keep them on one
 * stream. Errors are reported through hale_last_error(NULL, ...); a
 * device-side wait that times out is not reported by this entry point. */
HALE_API hale_status hale_moe_route_noalloc(const void* router, hale_dtype router_dtype,
                                            uint32_t n_experts, uint32_t top_k,
                                            int32_t normalize_topk, uint32_t hidden,
                                            const float* x, uint32_t m_tokens, int32_t* topk_idx,
                                            float* topk_w, float* probs, void* stream);

/* ---- expert parallelism ----------------------------------------------------
 * MoeLayer::forward (moe.rs:56-70) over n_ranks ranks, each owning a
 * contiguous block of n_experts / n_ranks experts per layer (rank r owns
 * [r * E/R, (r+1) * E/R)). The reference runs on one host and has no such
 * split; these three calls are the device work around the two all-to-all-v
 * exchanges the host performs with its own communicator:
 *   1. hale_ep_dispatch (home): route m_tokens tokens, quantize each once,
 *      pack one record per route, grouped by owner rank;
 *   2. send the records; hale_ep_experts (owner) on what arrived; send the
 *      y rows back in the order they came;
 *   3. hale_ep_combine (home): best-first weighted sum per token.
 * The result is bit-identical to hale_moe_forward on one GPU. Records:
 *   q    [n, hidden] int8      -- Q8Activations quants of the home token
 *   aux  [n, 2 * hale_q8_aux_pairs(hidden)] int32 -- per block: f32 scale bits,
 *                                -8 * sum of the block's quants
 *   meta [n, 4] int32          -- home token, route slot (0 = best), global
 *                                expert, routing weight (f32 bits)
 * Device buffers must be 16-byte aligned. */

/* Pairs of int32 per aux row: (cols / 32) rounded up to even. */
HALE_API int32_t hale_q8_aux_pairs(uint32_t cols);

/* Home side. Records for all m_tokens * top_k routes in send order (owner
 * rank ascending, then expert ascending); counts_host[r] = records for rank
 * r (host memory; the call synchronizes the stream). topk_idx / topk_w
 * (nullable): as hale_moe_forward. */
HALE_API hale_status hale_ep_dispatch(hale_ctx* ctx, const hale_moe_layer* layer, uint32_t hidden,
                                      const float* x, uint32_t m_tokens, uint32_t n_ranks, int8_t* send_q,
                                      int32_t* send_aux, int32_t* send_meta, uint64_t* counts_host,
                                      int32_t* topk_idx, float* topk_w, void* stream);

/* Owner side: y[j, :] = Expert(record j) for the n received records (any
 * source order), with this rank's experts in `pool` as local ids
 * 0 .. pool experts - 1 = global ids expert0 .. ; a record naming another
 * expert raises HALE_E_DEVICE_CHECK at the next hale_ctx_check. */
HALE_API hale_status hale_ep_experts(hale_ctx* ctx, hale_pool* pool, uint32_t layer, uint32_t expert0,
                                     const int8_t* recv_q, const int32_t* recv_aux, const int32_t* recv_meta,
                                     uint32_t n, float* y, void* stream);

/* Home side: out[t, :] = sum over s = 0 .. top_k-1 of w * y_back[record of
 * (t, s)], starting from 0 (moe.rs:63-68). send_meta: as packed by
 * hale_ep_dispatch; y_back [m_tokens * top_k, hidden]: y of each record in
 * send order. */
HALE_API hale_status hale_ep_combine(hale_ctx* ctx, const int32_t* send_meta, const float* y_back,
                                     uint32_t m_tokens, uint32_t top_k, uint32_t hidden, float* out,
                                     void* stream);

/* ---- expert parallelism over NVLink, one call per layer --------------------
 * MoeLayer::forward (moe.rs:56-70) with the layer's experts split over
 * n_ranks GPUs of one node, one process (and hale_ctx) per GPU; rank r owns
 * experts [r * E/R, (r+1) * E/R), held in a resident pool with local ids.
 * Each rank brings its own tokens. hale_moe_forward_ep routes them, stores
 * one record per route (the token's q8 row, its block aux and the route)
 * straight into the owner rank's memory over NVLink, runs this rank's
 * experts on what every rank sent, stores each y row straight back into its
 * home rank's memory, and combines best-first -- kernels and peer stores
 * only, no host synchronisation inside the call. out is bit-identical to
 * hale_moe_forward with all E experts on one GPU. The reference runs on one
 * host and has no such split; the surface it replaces is the same
 * MoeLayer::forward / ExpertProvider::fetch (src/expert/mod.rs:128-137). */
typedef struct hale_comm hale_comm;
#define HALE_COMM_ID_BYTES 128

/* A fresh communicator id (an ncclUniqueId, 128 bytes), made on one rank and
 * handed to every rank by the caller's own means (a TCP store, MPI, ...). */
HALE_API hale_status hale_comm_unique_id(void* id);

/* Collective over the n_ranks ranks (every rank calls it with the same id
 * and shape). Allocates this rank's exchange block -- two halves of
 * n_ranks * max_tokens * min(top_k, E / n_ranks) record slots plus
 * max_tokens * top_k f32 rows of `hidden` -- and maps every peer's block
 * through CUDA IPC (NCCL all-gathers the handles; NCCL is loaded at run
 * time, libnccl.so.2). With n_ranks = 1 there is no NCCL and id may be NULL.
 * Up to 8 ranks; n_experts must divide by n_ranks. */
HALE_API hale_status hale_comm_create(hale_ctx* ctx, uint32_t n_ranks, uint32_t rank, const void* id,
                                      uint32_t hidden, uint32_t n_experts, uint32_t top_k, uint32_t max_tokens,
                                      hale_comm** out);
/* Collective: waits for every rank, then frees the block and unmaps peers. */
HALE_API hale_status hale_comm_destroy(hale_comm* comm);

/* One expert-parallel layer call on every rank (collective: each rank makes
 * the same sequence of calls, with its own m_tokens <= max_tokens, possibly
 * 0). pool: this rank's E / n_ranks experts (HBM-resident) at pool layer
 * layer->layer; layer: the full router (all E experts), replicated.
 * x, out: [m_tokens, hidden] f32 (device); topk_idx / topk_w (nullable) as
 * hale_moe_forward. Waits on peers are bounded (about a second): a rank that
 * never arrives shows up as HALE_E_TIMEOUT at the next hale_ctx_check. */
HALE_API hale_status hale_moe_forward_ep(hale_ctx* ctx, hale_comm* comm, hale_pool* pool,
                                         const hale_moe_layer* layer, const float* x, uint32_t m_tokens, float* out,
                                         int32_t* topk_idx, float* topk_w, void* stream);

/* ---- decode step of the whole model ----------------------------------------
 * Transformer::forward (transformer.rs:168-227) for one token: embedding
 * row, then per layer RMSNorm -> attention (q/k/v projections, per-head
 * q/k RMSNorm when present, RoPE, KV-cache append, GQA softmax attention,
 * o projection) -> residual -> RMSNorm -> MoE layer or dense SwiGLU ->
 * residual; final RMSNorm and lm_head. Bit-identical to the reference's
 * arithmetic (the RoPE tables come from the host libm the reference calls).
 * Matrices are given as host row-major buffers in the reference's encodings
 * (tensor/dtype.rs); dense matrices must be float (f32, f16, bf16). */
typedef struct {
    int32_t dtype;       /* hale_dtype */
    uint32_t rows, cols;
    const void* data;    /* rows * hale_row_bytes(dtype, cols) bytes, host memory */
} hale_host_matrix;

typedef struct {
    const float* input_norm;   /* [hidden], host */
    const float* post_norm;    /* [hidden] */
    const float* q_norm;       /* [head_dim] or NULL (Mixtral) */
    const float* k_norm;       /* [head_dim] or NULL */
    hale_host_matrix q, k, v, o;                 /* [nh*hd, H], [nkv*hd, H] x2, [H, nh*hd] */
    int32_t is_moe;
    hale_host_matrix router;                     /* is_moe: [n_experts, H], float */
    hale_host_matrix dense_gate, dense_up, dense_down;  /* !is_moe: [I, H], [I, H], [H, I] */
} hale_decoder_layer;

typedef struct {
    uint32_t hidden, n_layers, n_heads, n_kv_heads, head_dim, vocab, n_experts, top_k;
    int32_t normalize_topk;
    float eps, rope_theta;
    hale_host_matrix embed;    /* [vocab, hidden], float */
    hale_host_matrix lm_head;  /* [vocab, hidden], float */
    const float* final_norm;   /* [hidden], host */
} hale_decoder_desc;

typedef struct hale_decoder hale_decoder;

/* Builds the decoder on ctx's GPU. experts: the routed experts of the MoE
 * layers in order (pool layer j = the j-th MoE layer), already uploaded;
 * NULL when the model has no MoE layer. max_len: KV-cache positions. */
HALE_API hale_status hale_decoder_create(hale_ctx* ctx, const hale_decoder_desc* desc,
                                         const hale_decoder_layer* layers, hale_pool* experts,
                                         uint32_t max_len, hale_decoder** out);
HALE_API void hale_decoder_destroy(hale_decoder* dec);
/* One step for `token` at `position` (KV cache appended there). logits
 * [vocab] / hidden [hidden] (the final-normed state): device, nullable. */
HALE_API hale_status hale_decoder_forward(hale_ctx* ctx, hale_decoder* dec, uint32_t token, uint32_t position,
                                          float* logits, float* hidden, void* stream);

/* A decoder with n_seqs independent KV caches whose steps take up to
 * max_batch rows (hale_decoder_create is n_seqs = max_batch = 1). */
HALE_API hale_status hale_decoder_create_batched(hale_ctx* ctx, const hale_decoder_desc* desc,
                                                 const hale_decoder_layer* layers, hale_pool* experts,
                                                 uint32_t max_len, uint32_t n_seqs, uint32_t max_batch,
                                                 hale_decoder** out);
/* One step over n rows (host arrays): row r is tokens[r] at positions[r] of
 * sequence seqs[r] (seqs NULL = all sequence 0). Every row's K/V is appended
 * before any row attends, and row r attends to positions 0..positions[r] of
 * its sequence, so a prompt's consecutive positions in one step (batched
 * prefill) or one row per sequence (batched decode) give each row exactly
 * the logits of token-by-token Transformer::forward (transformer.rs:168-239):
 * the MoE layers run all rows through the grouped expert kernels, every
 * other op applies the one-row arithmetic to each row. Two rows may not
 * write the same (sequence, position). logits: [n, vocab], or [1, vocab] for
 * the last row when last_logits_only; hidden: [n, hidden]; both device,
 * nullable. Not capturable into a CUDA graph. */
HALE_API hale_status hale_decoder_step(hale_ctx* ctx, hale_decoder* dec, const uint32_t* tokens,
                                       const uint32_t* positions, const uint32_t* seqs, uint32_t n,
                                       float* logits, int32_t last_logits_only, float* hidden, void* stream);

/* Expert-parallel decoding: the decoder's MoE layers run through
 * hale_moe_forward_ep over `comm`, with the decoder's pool holding this
 * rank's n_experts / n_ranks experts of every MoE layer (HBM-resident);
 * attention and the dense layers stay on this rank for its own sequences
 * (data-parallel). Every rank must then make the same sequence of decoder
 * calls (collective per MoE layer; its own rows each time; a rank with no
 * rows calls hale_decoder_step with n = 0, which still joins every MoE
 * layer's exchange), which run eagerly (no graph replay). comm NULL returns to single-GPU layers.
 * comm's max_tokens must cover the decoder's max_batch. Such a decoder is
 * created with the rank's pool (n_experts / n_ranks experts per layer);
 * until its comm is set, its MoE calls fail with HALE_E_INVALID_ARGUMENT. */
HALE_API hale_status hale_decoder_set_comm(hale_decoder* dec, hale_comm* comm);

/* ---- sampling tail -------------------------------------------------------- */

/* Transformer::logits (transformer.rs:217-221): logits[b, :] = lm_head .
 * hidden[b, :] for b < batch, with lm_head a float hale_matrix [V, H]. */
HALE_API hale_status hale_lm_head(hale_ctx* ctx, const hale_matrix* lm_head, const float* hidden,
                         uint32_t batch, float* logits, void* stream);

/* SamplingParams (sampler.rs:22-43) plus a repetition penalty, which the
 * reference does not have (1.0 disables it; HF convention: a seen id's
 * logit l becomes l / p when l > 0, else l * p, before temperature). */
typedef struct {
    float temperature; /* <= 0: greedy argmax */
    float top_p;       /* 1.0 disables the nucleus cut */
    uint32_t top_k;    /* 0 disables top-k */
    float repetition_penalty;
} hale_sampling_params;

/* Sampler::sample (sampler.rs:14-18, 80-123) for `batch` rows of logits
 * [batch, vocab] (device). Up to 1024 candidates (top_k <= 1024, or a vocab
 * of at most 1024) are selected and sorted in one kernel per row; more
 * (top_k = 0 with a larger vocab, which keeps every token, or a larger
 * top_k) are ranked by a segmented radix sort in the ctx's scratch memory,
 * with the reference's softmax, nucleus and draw sums run over the sorted
 * order exactly. rng_state [batch] u64 (device) holds each row's
 * XorShift64 state (seed.max(1) initially, sampler.rs:131-133) and is
 * advanced in place. seen_ids [batch, n_seen] i32 (nullable; entries < 0
 * are ignored) feeds the repetition penalty. out_tokens [batch] i32. */
HALE_API hale_status hale_sample(hale_ctx* ctx, const float* logits, uint32_t batch, uint32_t vocab,
                        const hale_sampling_params* params, uint64_t* rng_state,
                        const int32_t* seen_ids, uint32_t n_seen, int32_t* out_tokens,
                        void* stream);

/* generate() (src/generate/generator.rs:55-94) on a decoder: the prompt is
 * prefilled into sequence 0 from position 0 (steps of up to max_batch rows,
 * only the last row's logits computed), then each round samples the next
 * token from the device logits (hale_sample with `params`; the XorShift64
 * state starts at seed.max(1), sampler.rs:131-133; a repetition penalty
 * other than 1 sees the prompt and the tokens generated so far), appends it
 * to out_tokens and, unless it is in stop_tokens or the round is the last,
 * runs the one-row step for it at the next position. *n_out = tokens
 * written (<= max_new_tokens). Each round reads the token back to the host
 * for the stop check, as the reference's loop does. prefill_ms / decode_ms
 * (nullable): CUDA-event times of the prefill and of the rounds, the split
 * GenerationStats reports. n_prompt + max_new_tokens beyond the decoder's
 * positions: HALE_E_CONTEXT_OVERFLOW (HaleError::ContextOverflow). Not for an
 * expert-parallel decoder (HALE_E_UNSUPPORTED). No reference counterpart for
 * the timing outputs. */
HALE_API hale_status hale_decoder_generate(hale_ctx* ctx, hale_decoder* dec, const uint32_t* prompt, uint32_t n_prompt,
                                           const hale_sampling_params* params, uint64_t seed, uint32_t max_new_tokens,
                                           const uint32_t* stop_tokens, uint32_t n_stop, uint32_t* out_tokens,
                                           uint32_t* n_out, float* prefill_ms, float* decode_ms, void* stream);

/* ---- self-checks ----------------------------------------------------------- */

/* The exp used by the device kernels, evaluated on the host from the same
 * source (y[i] = exp(x[i]) for i < n). It restates glibc's expf so softmax
 * and SiLU match the reference's CPU results bit for bit. */
HALE_API void hale_expf_host(const float* x, float* y, uint64_t n);

#ifdef __cplusplus
}
#endif
#endif /* HALE_CUDA_H */
