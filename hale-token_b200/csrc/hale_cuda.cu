// hale_cuda.cu -- C ABI (include/hale_cuda.h) over the sm_100a kernels.
//
// Host orchestration only: argument checks mirroring the reference's
// assertions and HaleError cases, workspace management, and launches. The
// arithmetic lives in hale_kernels.cuh.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <cub/device/device_segmented_radix_sort.cuh>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <set>
#include <string>
#include <tuple>
#include <vector>

#include "../../include/hale_cuda.h"
#include "hale_kernels.cuh"
#include "hale_tc.cuh"
#include "hale_stream.cuh"
#include "hale_ws.cuh"
#include "hale_token.cuh"
#include "hale_ep.cuh"
#include "hale_p2p.cuh"
#include "hale_decoder.cuh"
#include "hale_attn.cuh"
#include "hale_tier.h"

using namespace hale;

// ---------------------------------------------------------------------------
// errors
// ---------------------------------------------------------------------------
namespace {
thread_local std::string g_thread_msg;
thread_local hale_status g_thread_status = HALE_OK;
}  // namespace

struct hale_ctx {
    int device = 0;
    // objects made on this context; destroying the context detaches them
    // (their own destroy then frees their memory on their device)
    std::set<hale_matrix*> matrices;
    std::set<hale_pool*> pools;
    std::set<hale_decoder*> decoders;
    std::set<hale_comm*> comms;
    int sm_count = 0;
    // expert kernel family (hale_ctx_set_expert_kernel): HALE_EXPERT_AUTO =
    // by batch shape, _TC = tcgen05 kernels, _DP4A = per-CTA kernels (dp4a /
    // warp MMA), _PS = persistent streaming warp-MMA kernels; each where the
    // shapes allow, else the per-CTA kernels
    int expert_kernel = 0;
    std::string msg;
    hale_status status = HALE_OK;
    uint32_t* d_err = nullptr;
    // MoE / route workspace (capacity-based layout; counters first)
    void* ws = nullptr;
    size_t ws_bytes = 0;
    int capM = 0, capE = 0, capK = 0, capH = 0, capI = 0;
    // scratch for unit-level calls
    void* scratch = nullptr;
    size_t scratch_bytes = 0;
    // bumped whenever ws or scratch is reallocated: CUDA graphs captured
    // before hold the old addresses and must not be replayed
    uint64_t ws_gen = 1;
    // hale_moe_forward_host replays: one captured graph per (pool, layer,
    // M, host buffers), valid while ws_gen matches
    struct HostGraph {
        const hale_pool* pool;
        hale_moe_layer layer;
        uint32_t M;
        const void *x, *out, *idx, *w;
        uint64_t gen;
        cudaGraphExec_t exec;
    };
    std::vector<HostGraph> host_graphs;
    cudaStream_t cap_st = nullptr;
    uint32_t* h_err = nullptr;  // page-locked copy of d_err
    uint64_t launches = 0;
    // per-kernel event timing (hale_ctx_profile)
    bool profiling = false;
    struct Mark {
        std::string name;
        cudaEvent_t a, b;
    };
    std::vector<Mark> marks;
    std::vector<cudaEvent_t> spare;
    std::map<std::string, std::pair<uint64_t, double>> totals;
};

struct hale_matrix {
    hale_ctx* ctx;
    int device = 0;
    hale_dtype dtype;
    uint32_t rows, cols, rows_pad;
    uint32_t nb;     // quantized: blocks per row; float: steps of 8
    uint8_t* data;
    size_t bytes;
    bool lanes = false;  // float, lane-major layout (fgemv_lanes_kernel); rows_pad = rows rounded to 4
};

struct hale_pool {
    hale_ctx* ctx;
    int device = 0;
    hale_dtype dtype;
    uint32_t H, I, L, E;
    size_t expert_stride;   // tiled bytes per expert
    size_t record_bytes;    // reference pack record bytes per expert
    uint8_t* data = nullptr;                   // resident: [L * E] experts; tiered: [n_slots]
    uint8_t* staging = nullptr;
    unsigned long long* d_routing = nullptr;  // [L * E]
    std::vector<uint8_t> resident;             // [L * E] uploaded
    std::vector<uint32_t> layer_resident;      // count per layer
    std::vector<uint64_t> host_routing;        // fetch() records
    hale_cache_stats stats{};
    // tiered pools (hale_pool_create_tiered)
    bool tiered = false;
    uint8_t* host_tier = nullptr;          // [L * E] tiled experts, page-locked host memory
    uint8_t* scratch = nullptr;            // one tiled expert (upload of an unpinned key)
    hale_tier::Book book;                  // slots, LRU and counters (hale_tier.h)
    int32_t* d_slot = nullptr;             // [L * E] slot table read by the expert kernels
    int32_t* h_slot = nullptr;             // page-locked staging of one layer's row [E]
    int32_t* h_routes = nullptr;           // page-locked read-back of a forward's routes
    size_t h_routes_cap = 0;
    cudaStream_t copy_st = nullptr;
    cudaEvent_t ev_issue = nullptr, ev_t0 = nullptr, ev_t1 = nullptr;
    cudaEvent_t ev_done = nullptr;         // after the last tiered forward's expert kernels
    bool done_recorded = false;
    bool timing_pending = false;
    // ExpertSource (hale_pool_set_source): fills the host tier on first use
    hale_expert_source_fn source = nullptr;
    void* source_user = nullptr;
    std::vector<uint8_t> source_buf;  // one pack record
    // TMA tensor maps over the tile layout of every expert slot (the
    // warp-specialised streaming kernels): gate/up tiles and down tiles
    bool ws_maps = false;
    CUtensorMap map_gu, map_d;
};

static hale_status fail(hale_ctx* ctx, hale_status st, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_thread_msg = buf;
    g_thread_status = st;
    if (ctx) {
        ctx->msg = buf;
        ctx->status = st;
    }
    return st;
}

#define CUDA_TRY(ctx, call)                                                                    \
    do {                                                                                       \
        cudaError_t e_ = (call);                                                               \
        if (e_ != cudaSuccess)                                                                 \
            return fail((ctx), e_ == cudaErrorMemoryAllocation ? HALE_E_OUT_OF_MEMORY : HALE_E_CUDA, \
                        "%s: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, __LINE__);  \
    } while (0)

static hale_status check_launch(hale_ctx* ctx, const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(ctx, HALE_E_CUDA, "launch of %s failed: %s", what, cudaGetErrorString(e));
    ctx->launches++;
    return HALE_OK;
}

static inline cudaStream_t S(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Opts a kernel into more than 48 KB of dynamic shared memory (once per
// kernel and size; the attribute is per function, not per launch).
// Static shared memory counts toward the same 48 KB default, so the opt-in
// is made for every dynamic size, cached per device and function.
template <class F>
static cudaError_t allow_smem(F* func, size_t bytes) {
    if (bytes == 0) return cudaSuccess;
    static std::mutex mu;
    static std::map<std::pair<int, const void*>, size_t> granted;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    size_t& g = granted[{dev, reinterpret_cast<const void*>(func)}];
    if (bytes <= g) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e == cudaSuccess) g = bytes;
    return e;
}

static cudaEvent_t take_event(hale_ctx* ctx) {
    if (!ctx->spare.empty()) {
        cudaEvent_t e = ctx->spare.back();
        ctx->spare.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}

// Brackets one launch with events when profiling is on.
struct ProfScope {
    hale_ctx* ctx;
    const char* name;
    cudaStream_t st;
    cudaEvent_t a = nullptr;
    ProfScope(hale_ctx* c, const char* n, cudaStream_t s) : ctx(c), name(n), st(s) {
        if (ctx->profiling) {
            a = take_event(ctx);
            cudaEventRecord(a, st);
        }
    }
    ~ProfScope() {
        if (a) {
            cudaEvent_t b = take_event(ctx);
            cudaEventRecord(b, st);
            ctx->marks.push_back({name, a, b});
        }
    }
};

static void drain_marks(hale_ctx* ctx) {
    for (auto& m : ctx->marks) {
        float ms = 0.0f;
        if (cudaEventSynchronize(m.b) == cudaSuccess && cudaEventElapsedTime(&ms, m.a, m.b) == cudaSuccess) {
            auto& t = ctx->totals[m.name];
            t.first++;
            t.second += ms;
        }
        ctx->spare.push_back(m.a);
        ctx->spare.push_back(m.b);
    }
    ctx->marks.clear();
    cudaGetLastError();
}

static bool stream_capturing(void* stream) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(S(stream), &cs) != cudaSuccess) return false;
    return cs != cudaStreamCaptureStatusNone;
}

static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
static bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }
// Dynamic shared memory one CTA may ask for on sm_100 (227 KB).
static constexpr size_t kMaxDynSmem = 227 * 1024;

static bool is_quant(hale_dtype d) { return d == HALE_Q8_0 || d == HALE_Q4_0; }
static bool is_float(hale_dtype d) { return d == HALE_F32 || d == HALE_F16 || d == HALE_BF16; }
static int block_len(hale_dtype d) { return is_quant(d) ? 32 : 1; }
static int block_bytes(hale_dtype d) {
    switch (d) {
    case HALE_F32: return 4;
    case HALE_F16:
    case HALE_BF16: return 2;
    case HALE_Q8_0: return 34;
    case HALE_Q4_0: return 18;
    }
    return 0;
}
static int float_code(hale_dtype d) { return d == HALE_F32 ? 0 : (d == HALE_F16 ? 1 : 2); }

extern "C" int64_t hale_row_bytes(hale_dtype dtype, uint64_t cols) {
    int bb = block_bytes(dtype);
    if (bb == 0) return -1;
    uint64_t bl = (uint64_t)block_len(dtype);
    if (cols % bl) return -1;
    return (int64_t)(cols / bl * (uint64_t)bb);
}

// ---------------------------------------------------------------------------
// context
// ---------------------------------------------------------------------------
extern "C" hale_status hale_ctx_create(int device, hale_ctx** out) {
    if (!out) return fail(nullptr, HALE_E_INVALID_ARGUMENT, "hale_ctx_create: out is NULL");
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        return fail(nullptr, HALE_E_NO_DEVICE, "no CUDA device is visible");
    }
    if (device < 0 || device >= n)
        return fail(nullptr, HALE_E_INVALID_ARGUMENT, "device %d out of range (%d devices)", device, n);
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess)
        return fail(nullptr, HALE_E_CUDA, "cudaGetDeviceProperties failed");
    if (prop.major != 10)
        return fail(nullptr, HALE_E_NO_DEVICE,
                    "device %d is compute capability %d.%d; this library is built for sm_100a (B200)",
                    device, prop.major, prop.minor);
    hale_ctx* c = new hale_ctx();
    c->device = device;
    c->sm_count = prop.multiProcessorCount;
    if (cudaSetDevice(device) != cudaSuccess || cudaMalloc(&c->d_err, 4) != cudaSuccess ||
        cudaMemset(c->d_err, 0, 4) != cudaSuccess) {
        delete c;
        return fail(nullptr, HALE_E_CUDA, "context setup failed on device %d", device);
    }
    *out = c;
    return HALE_OK;
}

static void drop_host_graphs(hale_ctx* ctx, const hale_pool* pool) {
    for (size_t i = 0; i < ctx->host_graphs.size();) {
        if (!pool || ctx->host_graphs[i].pool == pool) {
            cudaGraphExecDestroy(ctx->host_graphs[i].exec);
            ctx->host_graphs.erase(ctx->host_graphs.begin() + (long)i);
        } else {
            i++;
        }
    }
}

static void ctx_detach_children(hale_ctx* ctx);

extern "C" void hale_ctx_destroy(hale_ctx* ctx) {
    if (!ctx) return;
    ctx_detach_children(ctx);
    cudaSetDevice(ctx->device);
    cudaDeviceSynchronize();
    drop_host_graphs(ctx, nullptr);
    if (ctx->cap_st) cudaStreamDestroy(ctx->cap_st);
    cudaFreeHost(ctx->h_err);
    cudaFree(ctx->d_err);
    cudaFree(ctx->ws);
    cudaFree(ctx->scratch);
    drain_marks(ctx);
    for (cudaEvent_t e : ctx->spare) cudaEventDestroy(e);
    delete ctx;
}

extern "C" hale_status hale_ctx_set_expert_kernel(hale_ctx* ctx, int family) {
    if (!ctx) return fail(nullptr, HALE_E_INVALID_ARGUMENT, "hale_ctx_set_expert_kernel: ctx is NULL");
    if (family < HALE_EXPERT_AUTO || family > HALE_EXPERT_WS)
        return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_ctx_set_expert_kernel: unknown family %d", family);
    ctx->expert_kernel = family;
    return HALE_OK;
}

extern "C" hale_status hale_ctx_profile(hale_ctx* ctx, int enable) {
    if (!ctx) return fail(nullptr, HALE_E_INVALID_ARGUMENT, "hale_ctx_profile: ctx is NULL");
    ctx->profiling = enable != 0;
    return HALE_OK;
}

extern "C" hale_status hale_ctx_profile_read(hale_ctx* ctx, const char* kernel, uint64_t* launches,
                                             double* total_ms) {
    if (!ctx || !kernel) return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_ctx_profile_read: NULL argument");
    CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    drain_marks(ctx);
    auto it = ctx->totals.find(kernel);
    uint64_t n = it == ctx->totals.end() ? 0 : it->second.first;
    double ms = it == ctx->totals.end() ? 0.0 : it->second.second;
    if (launches) *launches = n;
    if (total_ms) *total_ms = ms;
    if (it != ctx->totals.end()) ctx->totals.erase(it);
    return HALE_OK;
}

extern "C" hale_status hale_last_error(const hale_ctx* ctx, char* buf, size_t len) {
    const std::string& m = ctx ? ctx->msg : g_thread_msg;
    if (buf && len) {
        size_t n = std::min(len - 1, m.size());
        memcpy(buf, m.data(), n);
        buf[n] = 0;
    }
    return ctx ? ctx->status : g_thread_status;
}

extern "C" uint64_t hale_ctx_launch_count(const hale_ctx* ctx) { return ctx ? ctx->launches : 0; }

// Counter region of the MoE workspace (zero between calls).
struct MoeLayout {
    size_t tile_cnt, grid_cnt, comb_cnt, ws_cnt, tok_bar, counters_end;
    size_t logits, topk_idx, topk_w, xq, xaux, elist_off, elist, active, n_active;
    size_t hq, haux, ybuf, total;
};

static MoeLayout moe_layout(int M, int E, int k, int H, int I) {
    MoeLayout L{};
    size_t o = 0;
    auto take = [&](size_t bytes) {
        size_t at = o;
        o = align_up(o + bytes, 256);
        return at;
    };
    const size_t nbph = (size_t)aux_stride(std::max(H / 32, 1)), nbpi = (size_t)aux_stride(std::max(I / 32, 1));
    L.tile_cnt = take((size_t)(M + kRouterTT - 1) / kRouterTT * 4);
    L.grid_cnt = take(4);
    L.comb_cnt = take((size_t)M * ((H + 127) / 128) * 4);
    L.ws_cnt = take(4 * 4);
    L.tok_bar = take(4 * 4);
    L.counters_end = o;
    L.logits = take((size_t)M * E * 4);
    L.topk_idx = take((size_t)M * k * 4);
    L.topk_w = take((size_t)M * k * 4);
    L.xq = take((size_t)M * H);
    L.xaux = take((size_t)M * nbph * 8);
    L.elist_off = take((size_t)(E + 1) * 4);
    L.elist = take((size_t)M * k * 4);
    L.active = take((size_t)E * 4);
    L.n_active = take(4);
    L.hq = take((size_t)M * k * I);
    L.haux = take((size_t)M * k * nbpi * 8);
    L.ybuf = take((size_t)M * k * H * 4);
    L.total = o;
    return L;
}

// Ensures the MoE workspace covers (M, E, k, H, I); the layout is computed
// from the capacities so counters never move between calls.
static hale_status ensure_moe_ws(hale_ctx* ctx, int M, int E, int k, int H, int I, void* stream,
                                 MoeLayout* out) {
    if (M <= ctx->capM && E <= ctx->capE && k <= ctx->capK && H <= ctx->capH && I <= ctx->capI && ctx->ws) {
        *out = moe_layout(ctx->capM, ctx->capE, ctx->capK, ctx->capH, ctx->capI);
        return HALE_OK;
    }
    if (stream_capturing(stream))
        return fail(ctx, HALE_E_INVALID_ARGUMENT,
                    "workspace must grow (M=%d) while the stream is being captured; run one call "
                    "of the largest shape before capturing", M);
    int cM = std::max(M, ctx->capM), cE = std::max(E, ctx->capE), cK = std::max(k, ctx->capK);
    int cH = std::max(H, ctx->capH), cI = std::max(I, ctx->capI);
    MoeLayout L = moe_layout(cM, cE, cK, cH, cI);
    CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    CUDA_TRY(ctx, cudaDeviceSynchronize());
    cudaFree(ctx->ws);
    ctx->ws = nullptr;
    ctx->ws_gen++;
    CUDA_TRY(ctx, cudaMalloc(&ctx->ws, L.total));
    CUDA_TRY(ctx, cudaMemset(ctx->ws, 0, L.total));
    ctx->ws_bytes = L.total;
    ctx->capM = cM; ctx->capE = cE; ctx->capK = cK; ctx->capH = cH; ctx->capI = cI;
    *out = L;
    return HALE_OK;
}

static hale_status ensure_scratch(hale_ctx* ctx, size_t bytes, void* stream) {
    if (bytes <= ctx->scratch_bytes && ctx->scratch) return HALE_OK;
    if (stream_capturing(stream))
        return fail(ctx, HALE_E_INVALID_ARGUMENT, "scratch must grow while the stream is being captured");
    CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    CUDA_TRY(ctx, cudaDeviceSynchronize());
    cudaFree(ctx->scratch);
    ctx->scratch = nullptr;
    ctx->ws_gen++;
    size_t b = align_up(std::max(bytes, (size_t)1 << 20), 1 << 20);
    CUDA_TRY(ctx, cudaMalloc(&ctx->scratch, b));
    ctx->scratch_bytes = b;
    return HALE_OK;
}

extern "C" hale_status hale_ctx_check(hale_ctx* ctx, void* stream) {
    if (!ctx) return fail(nullptr, HALE_E_INVALID_ARGUMENT, "hale_ctx_check: ctx is NULL");
    CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    CUDA_TRY(ctx, cudaStreamSynchronize(S(stream)));
    uint32_t err = 0;
    CUDA_TRY(ctx, cudaMemcpy(&err, ctx->d_err, 4, cudaMemcpyDeviceToHost));
    if (!err) return HALE_OK;
    CUDA_TRY(ctx, cudaMemset(ctx->d_err, 0, 4));
    if (ctx->ws) {  // a kernel stopped early: counters may be stale
        MoeLayout L = moe_layout(ctx->capM, ctx->capE, ctx->capK, ctx->capH, ctx->capI);
        CUDA_TRY(ctx, cudaMemset(ctx->ws, 0, L.counters_end));
    }
    if (err & kErrTimeout) return fail(ctx, HALE_E_TIMEOUT, "a device-side wait exceeded its bound");
    return fail(ctx, HALE_E_DEVICE_CHECK, "a device-side bounds check failed (0x%x)", err);
}

// ---------------------------------------------------------------------------
// repack launches
// ---------------------------------------------------------------------------
static hale_status launch_repack(hale_ctx* ctx, hale_dtype dt, const uint8_t* src, uint8_t* dst,
                                 uint32_t rows, uint32_t cols, cudaStream_t st) {
    uint32_t rows_pad = (rows + 31) / 32 * 32;
    if (is_quant(dt)) {
        int nb = (int)(cols / 32);
        long long total = (long long)rows_pad * nb;
        int bb = block_bytes(dt), qb = dt == HALE_Q4_0 ? 16 : 32;
        repack_quant_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(src, dst, (int)rows, (int)rows_pad, nb, bb, qb);
    } else {
        int steps = (int)((cols + 7) / 8);
        long long total = (long long)rows_pad * steps;
        repack_float_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(src, dst, (int)rows, (int)rows_pad,
                                                                               (int)cols, steps, block_bytes(dt));
    }
    return check_launch(ctx, "repack");
}

static size_t tiled_bytes(hale_dtype dt, uint32_t rows, uint32_t cols) {
    size_t rows_pad = (rows + 31) / 32 * 32;
    if (is_quant(dt)) return rows_pad * (cols / 32) * block_bytes(dt);
    return rows_pad * ((cols + 7) / 8) * 8 * block_bytes(dt);
}

// ---------------------------------------------------------------------------
// matrices
// ---------------------------------------------------------------------------
extern "C" hale_status hale_matrix_create(hale_ctx* ctx, hale_dtype dtype, uint32_t rows, uint32_t cols,
                                          const void* encoded, uint64_t encoded_bytes, int on_device,
                                          hale_matrix** out) {
    if (!ctx || !out) return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_matrix_create: NULL argument");
    *out = nullptr;
    int64_t rb = hale_row_bytes(dtype, cols);
    if (rb < 0)
        return fail(ctx, HALE_E_INVALID_ARGUMENT, "dtype %d needs row length divisible by %d, got %u",
                    (int)dtype, block_len(dtype), cols);
    if (rows == 0 || cols == 0) return fail(ctx, HALE_E_INVALID_ARGUMENT, "matrix %ux%u is empty", rows, cols);
    if ((uint64_t)rows * (uint64_t)rb != encoded_bytes)
        return fail(ctx, HALE_E_INVALID_ARGUMENT, "matrix %ux%u dtype %d needs %llu bytes, got %llu", rows,
                    cols, (int)dtype, (unsigned long long)rows * (unsigned long long)rb,
                    (unsigned long long)encoded_bytes);
    if (!encoded) return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_matrix_create: data is NULL");
    CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    hale_matrix* m = new hale_matrix();
    m->ctx = ctx;
    m->device = ctx->device;
    ctx->matrices.insert(m);
    m->dtype = dtype;
    m->rows = rows;
    m->cols = cols;
    m->rows_pad = (rows + 31) / 32 * 32;
    m->nb = is_quant(dtype) ? cols / 32 : (cols + 7) / 8;
    m->bytes = tiled_bytes(dtype, rows, cols);
    if (cudaMalloc(&m->data, m->bytes) != cudaSuccess) {
        delete m;
        return fail(ctx, HALE_E_OUT_OF_MEMORY, "cannot allocate %zu bytes for a matrix", m->bytes);
    }
    const uint8_t* src = static_cast<const uint8_t*>(encoded);
    uint8_t* tmp = nullptr;
    if (!on_device) {
        if (cudaMalloc(&tmp, encoded_bytes) != cudaSuccess ||
            cudaMemcpy(tmp, encoded, encoded_bytes, cudaMemcpyHostToDevice) != cudaSuccess) {
            cudaFree(tmp);
            cudaFree(m->data);
            delete m;
            return fail(ctx, HALE_E_CUDA, "cannot stage %llu bytes of matrix data", (unsigned long long)encoded_bytes);
        }
        src = tmp;
    }
    hale_status st = launch_repack(ctx, dtype, src, m->data, rows, cols, 0);
    cudaError_t e = cudaDeviceSynchronize();
    cudaFree(tmp);
    if (st != HALE_OK || e != cudaSuccess) {
        cudaFree(m->data);
        delete m;
        return st != HALE_OK ? st : fail(ctx, HALE_E_CUDA, "repack failed: %s", cudaGetErrorString(e));
    }
    *out = m;
    return HALE_OK;
}

extern "C" void hale_matrix_destroy(hale_matrix* m) {
    if (!m) return;
    if (m->ctx) m->ctx->matrices.erase(m);
    cudaSetDevice(m->device);
    cudaFree(m->data);
    delete m;
}

// Bulk-copy ring depth per warp (stages of 8 blocks: 4.6 KB for q4_0,
// 8.7 KB for q8_0). Large batches keep 2 stages in flight per warp, which
// leaves room for 3 CTAs per SM; small batches launch few CTAs, so each warp
// keeps (up to) its whole 2048-column tile in flight to cover HBM latency.
static int ring_stages(hale_dtype dt, uint32_t m_rows) {
    if (m_rows <= 2) return dt == HALE_Q4_0 ? 8 : 4;
    if (m_rows <= 16) return 4;
    return 2;
}

template <int QT>
static hale_status qgemv_go(hale_ctx* ctx, const hale_matrix* m, const int8_t* xq, const int2* xaux, uint32_t M,
                            float* out, int32_t* dbg, int S_, cudaStream_t st) {
    SmemPlan P = smem_plan(QFmt<QT>::BB, S_, 4, (int)m->cols);
    CUDA_TRY(ctx, allow_smem(qgemv_kernel<QT>, (size_t)P.total));
    unsigned grid = (m->rows_pad / 32 + 3) / 4;
    qgemv_kernel<QT><<<grid, 128, P.total, st>>>(m->data, (int)m->rows, (int)m->nb, xq, xaux, (int)M, out, dbg,
                                                 S_, ctx->d_err);
    return HALE_OK;
}

static hale_status qgemv_launch(hale_ctx* ctx, const hale_matrix* m, const int8_t* xq, const int2* xaux,
                                uint32_t M, float* out, int32_t* dbg, cudaStream_t st) {
    int S_ = std::min(ring_stages(m->dtype, M), ((int)m->nb + kStageBlocks - 1) / kStageBlocks);
    hale_status r;
    {
        ProfScope ps_(ctx, "qgemv", st);
        r = m->dtype == HALE_Q4_0 ? qgemv_go<0>(ctx, m, xq, xaux, M, out, dbg, S_, st)
                                  : qgemv_go<1>(ctx, m, xq, xaux, M, out, dbg, S_, st);
    }
    if (r) return r;
    return check_launch(ctx, "qgemv");
}

template <int DT>
static void fgemv_dispatch(const hale_matrix* m, const float* x, uint32_t M, float* out, int vec, cudaStream_t st) {
    unsigned grid = (m->rows_pad / 32 + 3) / 4;
    if (M <= 1)
        fgemv_kernel<DT, 1><<<grid, 128, 0, st>>>(m->data, (int)m->rows, (int)m->cols, (int)m->nb, x, (int)M, out, vec);
    else if (M <= 2)
        fgemv_kernel<DT, 2><<<grid, 128, 0, st>>>(m->data, (int)m->rows, (int)m->cols, (int)m->nb, x, (int)M, out, vec);
    else if (M <= 4)
        fgemv_kernel<DT, 4><<<grid, 128, 0, st>>>(m->data, (int)m->rows, (int)m->cols, (int)m->nb, x, (int)M, out, vec);
    else
        fgemv_kernel<DT, 8><<<grid, 128, 0, st>>>(m->data, (int)m->rows, (int)m->cols, (int)m->nb, x, (int)M, out, vec);
}

// Blocks a kernel keeps resident per SM at `smem` bytes and `threads`
// threads (cached per device, kernel and configuration).
template <class F>
static int kernel_occupancy(F* kern, int threads, size_t smem) {
    static std::mutex mu;
    static std::map<std::tuple<int, const void*, int, size_t>, int> memo;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    const auto key = std::make_tuple(dev, reinterpret_cast<const void*>(kern), threads, smem);
    auto it = memo.find(key);
    if (it != memo.end()) return it->second;
    int n = 0;
    if (allow_smem(kern, smem) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, threads, smem) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
    }
    memo[key] = n;
    return n;
}

// Warps per CTA of the single-row lane-major kernels: 8 (32 rows) when that
// still gives every SM two CTAs, else 4 so a decode-size matrix spreads over
// more SMs.
static unsigned lanes_warps(const hale_ctx* ctx, const hale_matrix* m) {
    return m->rows_pad / 32 >= 2u * (unsigned)ctx->sm_count ? 8u : 4u;
}

// Weight-ring depth of a single-row lane-major launch: the deepest (up to 4
// stages, no more than a warp's region has) that keeps the whole grid in one
// wave; grids of several waves take 2 (more CTAs per SM). 0: nothing fits.
template <class F>
static int lanes_pick_ns(const hale_ctx* ctx, F* kern, int act_bytes, uint32_t cols, int stage_bytes, unsigned wpc,
                         unsigned grid, size_t* smem_out) {
    const int nst = (int)((cols / 64 + kLanesSB - 1) / kLanesSB);
    int fallback = 0;
    size_t fb_smem = 0;
    for (int ns = std::min(4, std::max(nst, 1)); ns >= 1; ns--) {
        const size_t smem = lanes_smem(act_bytes, (int)wpc, ns * stage_bytes, ns);
        if (smem > kMaxDynSmem) continue;
        const int occ = kernel_occupancy(kern, (int)(32 * wpc), smem);
        if (occ <= 0) continue;
        if ((long long)occ * ctx->sm_count >= (long long)grid) {
            *smem_out = smem;
            return ns;
        }
        if (fallback == 0 || ns == 2) {
            fallback = ns;
            fb_smem = smem;
        }
    }
    *smem_out = fb_smem;
    return fallback;
}

static hale_status fgemv_launch(hale_ctx* ctx, const hale_matrix* m, const float* x, uint32_t M, float* out,
                                cudaStream_t st) {
    ProfScope ps_(ctx, "fgemv", st);
    if (m->lanes && M > 1) {
        // several activation rows: each weight step read once per chunk of NB rows
        const unsigned gx = (m->rows_pad / 4 + 7) / 8;
        // rows per chunk: 96 KB of staged activations at most (two or more CTAs per SM)
        const int NB = m->cols <= 3072 ? 8 : (m->cols <= 6144 ? 4 : 2);
        const dim3 grid(gx, (M + NB - 1) / NB);
        const size_t smem = (size_t)NB * m->cols * 4;
        hale_status r = HALE_OK;
        auto go = [&](auto kern) {
            cudaError_t e = allow_smem(kern, smem);
            if (e != cudaSuccess) {
                r = fail(ctx, HALE_E_CUDA, "fgemv_lanes_batch: %s", cudaGetErrorString(e));
                return;
            }
            kern<<<grid, 256, smem, st>>>(m->data, (int)m->rows, (int)m->cols, x, (int)M, out);
        };
        switch (m->dtype) {
        case HALE_F32:
            NB == 8 ? go(fgemv_lanes_batch_kernel<0, 8>) : NB == 4 ? go(fgemv_lanes_batch_kernel<0, 4>) : go(fgemv_lanes_batch_kernel<0, 2>);
            break;
        case HALE_F16:
            NB == 8 ? go(fgemv_lanes_batch_kernel<1, 8>) : NB == 4 ? go(fgemv_lanes_batch_kernel<1, 4>) : go(fgemv_lanes_batch_kernel<1, 2>);
            break;
        default:
            NB == 8 ? go(fgemv_lanes_batch_kernel<2, 8>) : NB == 4 ? go(fgemv_lanes_batch_kernel<2, 4>) : go(fgemv_lanes_batch_kernel<2, 2>);
            break;
        }
        if (r) return r;
        return check_launch(ctx, "fgemv_lanes_batch");
    }
    if (m->lanes) {
        const unsigned wpc = lanes_warps(ctx, m), grid = (m->rows_pad / 4 + wpc - 1) / wpc, threads = 32 * wpc;
        auto go = [&](auto kern, int ring_stage) -> cudaError_t {
            size_t smem = 0;
            const int ns = lanes_pick_ns(ctx, kern, (int)m->cols * 4, m->cols, ring_stage, wpc, grid, &smem);
            if (ns == 0) return cudaErrorInvalidConfiguration;
            cudaError_t e = allow_smem(kern, smem);
            if (e != cudaSuccess) return e;
            for (uint32_t t = 0; t < M; t++)
                kern<<<grid, threads, smem, st>>>(m->data, (int)m->rows, (int)m->cols, x + (size_t)t * m->cols,
                                                  out + (size_t)t * m->rows, ns, ctx->d_err);
            return cudaSuccess;
        };
        cudaError_t e = m->dtype == HALE_F32 ? go(fgemv_lanes_kernel<0>, lanes_stage_bytes<0>())
                        : m->dtype == HALE_F16 ? go(fgemv_lanes_kernel<1>, lanes_stage_bytes<1>())
                                               : go(fgemv_lanes_kernel<2>, lanes_stage_bytes<2>());
        if (e != cudaSuccess) return fail(ctx, HALE_E_CUDA, "fgemv_lanes: %s", cudaGetErrorString(e));
        return check_launch(ctx, "fgemv_lanes");
    }
    int vec = (m->cols % 4 == 0) && (((uintptr_t)x & 15) == 0);
    switch (m->dtype) {
    case HALE_F32: fgemv_dispatch<0>(m, x, M, out, vec, st); break;
    case HALE_F16: fgemv_dispatch<1>(m, x, M, out, vec, st); break;
    default: fgemv_dispatch<2>(m, x, M, out, vec, st); break;
    }
    return check_launch(ctx, "fgemv");
}

// One activation row through a lane-major float matrix with the RMSNorm in
// front folded in (fgemv_lanes_norm_kernel); false in *done when the matrix
// or buffers do not fit that kernel (nothing launched).
static hale_status fgemv_norm_launch(hale_ctx* ctx, const hale_matrix* m, const float* x, const float* delta,
                                     const float* nw, float eps, float* x_out, float* out, cudaStream_t st,
                                     bool* done) {
    *done = false;
    if (!m->lanes || m->cols % 64 || !aligned16(x) || (delta && (!aligned16(delta) || !aligned16(x_out))))
        return HALE_OK;
    const unsigned wpc = lanes_warps(ctx, m), grid = (m->rows_pad / 4 + wpc - 1) / wpc, threads = 32 * wpc;
    if (m->cols > 4u * kLanesNormVec * threads) return HALE_OK;
    ProfScope ps_(ctx, "fgemv", st);
    bool skip = false;
    auto go = [&](auto kern, int ring_stage) -> cudaError_t {
        size_t smem = 0;
        const int ns = lanes_pick_ns(ctx, kern, (int)m->cols * 8, m->cols, ring_stage, wpc, grid, &smem);
        if (ns == 0) {
            skip = true;
            return cudaSuccess;
        }
        cudaError_t e = allow_smem(kern, smem);
        if (e != cudaSuccess) return e;
        kern<<<grid, threads, smem, st>>>(m->data, (int)m->rows, (int)m->cols, x, delta, nw, eps, x_out, out, ns,
                                          ctx->d_err);
        return cudaSuccess;
    };
    cudaError_t e = m->dtype == HALE_F32 ? go(fgemv_lanes_norm_kernel<0>, lanes_stage_bytes<0>())
                    : m->dtype == HALE_F16 ? go(fgemv_lanes_norm_kernel<1>, lanes_stage_bytes<1>())
                                           : go(fgemv_lanes_norm_kernel<2>, lanes_stage_bytes<2>());
    if (e != cudaSuccess) return fail(ctx, HALE_E_CUDA, "fgemv_lanes_norm: %s", cudaGetErrorString(e));
    if (skip) return HALE_OK;
    hale_status r = check_launch(ctx, "fgemv_lanes_norm");
    if (!r) *done = true;
    return r;
}

extern "C" hale_status hale_quantize_q8(hale_ctx* ctx, const float* x, uint32_t m_rows, uint32_t cols,
                                        float* scales, int8_t* quants, void* stream) {
    if (!ctx) return fail(nullptr, HALE_E_INVALID_ARGUMENT, "hale_quantize_q8: ctx is NULL");
    if (cols % 32) return fail(ctx, HALE_E_INVALID_ARGUMENT, "activation length must be a multiple of 32, got %u", cols);
    if (m_rows == 0) return HALE_OK;
    if (!x || !scales || !quants) return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_quantize_q8: NULL buffer");
    if (!aligned16(x) || !aligned16(quants))
        return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_quantize_q8: x and quants must be 16-byte aligned");
    CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    unsigned grid = (m_rows * 32 + 255) / 256;
    ProfScope ps_(ctx, "quantize", S(stream));
    quantize_rows_kernel<<<grid, 256, 0, S(stream)>>>(x, (int)m_rows, (int)cols, quants, scales, nullptr);
    return check_launch(ctx, "quantize");
}

extern "C" hale_status hale_matrix_matvec(hale_ctx* ctx, const hale_matrix* m, const float* x, uint32_t m_rows,
                                          float* out, int32_t* block_sums, void* stream) {
    if (!ctx || !m) return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_matrix_matvec: NULL argument");
    if (m_rows == 0) return HALE_OK;
    if (!x || !out) return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_matrix_matvec: NULL buffer");
    CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    cudaStream_t st = S(stream);
    if (is_float(m->dtype)) {
        if (block_sums) return fail(ctx, HALE_E_INVALID_ARGUMENT, "block sums exist only for quantized matrices");
        return fgemv_launch(ctx, m, x, m_rows, out, st);
    }
    if (!aligned16(x)) return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_matrix_matvec: x must be 16-byte aligned");
    size_t qbytes = align_up((size_t)m_rows * m->cols, 256);
    size_t abytes = (size_t)m_rows * aux_stride((int)m->nb) * 8;
    hale_status rs = ensure_scratch(ctx, qbytes + abytes, stream);
    if (rs) return rs;
    int8_t* xq = static_cast<int8_t*>(ctx->scratch);
    int2* xaux = reinterpret_cast<int2*>(static_cast<uint8_t*>(ctx->scratch) + qbytes);
    unsigned grid = (m_rows * 32 + 255) / 256;
    {
        ProfScope ps_(ctx, "quantize", st);
        quantize_rows_kernel<<<grid, 256, 0, st>>>(x, (int)m_rows, (int)m->cols, xq, nullptr, xaux);
    }
    hale_status r = check_launch(ctx, "quantize");
    if (r) return r;
    return qgemv_launch(ctx, m, xq, xaux, m_rows, out, block_sums, st);
}

extern "C" hale_status hale_matrix_matvec_q8(hale_ctx* ctx, const hale_matrix* m, const float* x_scales,
                                             const int8_t* x_quants, uint32_t m_rows, float* out,
                                             int32_t* block_sums, void* stream) {
    if (!ctx || !m) return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_matrix_matvec_q8: NULL argument");
    if (!is_quant(m->dtype))
        return fail(ctx, HALE_E_INVALID_ARGUMENT, "dot_quantized called with float dtype %d", (int)m->dtype);
    if (m_rows == 0) return HALE_OK;
    if (!x_scales || !x_quants || !out) return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_matrix_matvec_q8: NULL buffer");
    CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    cudaStream_t st = S(stream);
    hale_status rs = ensure_scratch(ctx, (size_t)m_rows * aux_stride((int)m->nb) * 8, stream);
    if (rs) return rs;
    int2* xaux = static_cast<int2*>(ctx->scratch);
    long long n = (long long)m_rows * m->nb;
    aux_from_q8_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(x_scales, x_quants, (int)m_rows, (int)m->cols, xaux);
    hale_status r = check_launch(ctx, "aux");
    if (r) return r;
    if (((uintptr_t)x_quants & 15) != 0)
        return fail(ctx, HALE_E_INVALID_ARGUMENT, "x_quants must be 16-byte aligned");
    return qgemv_launch(ctx, m, x_quants, xaux, m_rows, out, block_sums, st);
}

// ---------------------------------------------------------------------------
// TMA tensor maps over the pool's tile layout
// ---------------------------------------------------------------------------
// cuTensorMapEncodeTiled, reached through the runtime's driver entry point
// (no link-time dependency on the driver library).
static PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
    static std::mutex mu;
    static bool tried = false;
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    std::lock_guard<std::mutex> lk(mu);
    if (!tried) {
        tried = true;
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
        else
            cudaGetLastError();
    }
    return fn;
}

// A 4-D map over `n_slots` experts' region starting `offset` bytes into each
// expert: [slot][tile][block][record as u64], boxes of box_tiles tiles x SB
// blocks (whole records, so every copy starts on a 16-byte boundary).
static bool pool_tensor_map(CUtensorMap* m, uint8_t* data, size_t offset, int rec, int nb, int tiles, size_t n_slots,
                            size_t stride, int box_tiles, int SB) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = tmap_encoder();
    if (!enc || rec % 16 || rec / 8 > 256 || ((uintptr_t)(data + offset) & 15) || stride % 16) return false;
    cuuint64_t dims[4] = {(cuuint64_t)(rec / 8), (cuuint64_t)nb, (cuuint64_t)tiles, (cuuint64_t)n_slots};
    cuuint64_t strides[3] = {(cuuint64_t)rec, (cuuint64_t)nb * rec, (cuuint64_t)stride};
    cuuint32_t box[4] = {(cuuint32_t)(rec / 8), (cuuint32_t)SB, (cuuint32_t)box_tiles, 1u};
    cuuint32_t es[4] = {1u, 1u, 1u, 1u};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT64, 4, data + offset, dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// CTAs per SM and activation buffers of the streaming kernels for these
// shapes: the first configuration, in preference order, whose shared-memory
// plans fit for both kernels with at least three weight stages in flight
// (two for the last resort); cps 0 = the shapes do not suit them. Measured
// on B200 at the Qwen3-30B layer shape: four CTAs per SM with one activation
// buffer are fastest from ~2 routes per active expert on (M = 64: 71.5 vs
// 72.9 us gate/up; M = 512: 248 vs 252 us gate/up, 176 vs 199 us down);
// smaller batches, where a CTA sees about one unit, keep three CTAs with
// double-buffered activations (M = 8: 45 vs 53 us gate/up).
struct WsCfg {
    int cps, xb;
};
static constexpr WsCfg kWsWide[] = {{4, 1}, {3, 2}, {3, 1}, {2, 2}, {2, 1}};
static constexpr WsCfg kWsNarrow[] = {{3, 2}, {4, 1}, {3, 1}, {2, 2}, {2, 1}};

static WsCfg ws_config(hale_dtype dt, int H, int I, bool narrow = false) {
    const int rec = 32 * block_bytes(dt);
    for (int min_s : {3, 2})
        for (const WsCfg& c : narrow ? kWsNarrow : kWsWide) {
            const int budget = ws_budget(c.cps);
            const WsPlan a = ws_plan(rec, 2, 2, kWsSB, H, budget, c.xb), b = ws_plan(rec, 1, 4, kWsSB, I, budget, c.xb);
            if (ws_plan_ok(a, budget) && ws_plan_ok(b, budget) && a.S >= min_s && b.S >= min_s) return c;
        }
    return {0, 0};
}

static int ws_ctas_per_sm(hale_dtype dt, int H, int I) { return ws_config(dt, H, I).cps; }

// Builds the pool's maps (gate/up: H/32 blocks per tile, 2 * I/32 tiles;
// down: I/32 blocks per tile, H/32 tiles) when its shapes suit the
// streaming kernels; otherwise they are left unused.
static void pool_build_maps(hale_pool* p, size_t n_slots) {
    p->ws_maps = false;
    const int H = (int)p->H, I = (int)p->I, rec = 32 * block_bytes(p->dtype);
    if (I % 64 || H % 128 || !ws_ctas_per_sm(p->dtype, H, I)) return;
    const int nbh = H / 32, nbi = I / 32, TI = I / 32, TH = H / 32;
    const size_t gu = 2 * tiled_bytes(p->dtype, p->I, p->H);
    p->ws_maps = pool_tensor_map(&p->map_gu, p->data, 0, rec, nbh, 2 * TI, n_slots, p->expert_stride, 2, kWsSB) &&
                 pool_tensor_map(&p->map_d, p->data, gu, rec, nbi, TH, n_slots, p->expert_stride, 4, kWsSB);
}

// ---------------------------------------------------------------------------
// expert pool
// ---------------------------------------------------------------------------
extern "C" hale_status hale_pool_create(hale_ctx* ctx, hale_dtype dtype, uint32_t hidden, uint32_t inter,
                                        uint32_t n_layers, uint32_t n_experts, hale_pool** out) {
    if (!ctx || !out) return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_pool_create: NULL argument");
    *out = nullptr;
    if (!is_quant(dtype)) return fail(ctx, HALE_E_INVALID_ARGUMENT, "expert pool dtype must be q8_0 or q4_0");
    if (hidden == 0 || inter == 0 || hidden % 32 || inter % 32)
        return fail(ctx, HALE_E_INVALID_ARGUMENT, "hidden (%u) and intermediate (%u) must be non-zero multiples of 32",
                    hidden, inter);
    if (n_layers == 0 || n_experts == 0 || n_experts > 256)
        return fail(ctx, HALE_E_INVALID_ARGUMENT, "need 1..256 experts and >= 1 layer (got %u, %u)", n_experts, n_layers);
    CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    hale_pool* p = new hale_pool();
    p->ctx = ctx;
    p->device = ctx->device;
    ctx->pools.insert(p);
    p->dtype = dtype;
    p->H = hidden;
    p->I = inter;
    p->L = n_layers;
    p->E = n_experts;
    p->expert_stride = 2 * tiled_bytes(dtype, inter, hidden) + tiled_bytes(dtype, hidden, inter);
    p->record_bytes = 2 * (size_t)inter * hale_row_bytes(dtype, hidden) + (size_t)hidden * hale_row_bytes(dtype, inter);
    size_t total = p->expert_stride * n_layers * n_experts;
    if (cudaMalloc(&p->data, total) != cudaSuccess || cudaMalloc(&p->staging, p->record_bytes) != cudaSuccess ||
        cudaMalloc(&p->d_routing, (size_t)n_layers * n_experts * 8) != cudaSuccess ||
        cudaMemset(p->d_routing, 0, (size_t)n_layers * n_experts * 8) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(p->data);
        cudaFree(p->staging);
        cudaFree(p->d_routing);
        delete p;
        return fail(ctx, HALE_E_OUT_OF_MEMORY, "cannot allocate %zu bytes of expert pool", total);
    }
    p->resident.assign((size_t)n_layers * n_experts, 0);
    p->layer_resident.assign(n_layers, 0);
    p->host_routing.assign((size_t)n_layers * n_experts, 0);
    pool_build_maps(p, (size_t)n_layers * n_experts);
    *out = p;
    return HALE_OK;
}

extern "C" void hale_pool_destroy(hale_pool* p) {
    if (!p) return;
    cudaSetDevice(p->device);
    if (p->ctx) {
        drop_host_graphs(p->ctx, p);
        p->ctx->pools.erase(p);
    }
    if (p->copy_st) cudaStreamSynchronize(p->copy_st);
    cudaFree(p->data);
    cudaFree(p->staging);
    cudaFree(p->d_routing);
    cudaFree(p->scratch);
    cudaFree(p->d_slot);
    cudaFreeHost(p->host_tier);
    cudaFreeHost(p->h_slot);
    cudaFreeHost(p->h_routes);
    if (p->copy_st) cudaStreamDestroy(p->copy_st);
    if (p->ev_issue) cudaEventDestroy(p->ev_issue);
    if (p->ev_t0) cudaEventDestroy(p->ev_t0);
    if (p->ev_t1) cudaEventDestroy(p->ev_t1);
    if (p->ev_done) cudaEventDestroy(p->ev_done);
    delete p;
}

extern "C" hale_status hale_pool_create_tiered(hale_ctx* ctx, hale_dtype dtype, uint32_t hidden, uint32_t inter,
                                               uint32_t n_layers, uint32_t n_experts, const hale_cache_policy* policy,
                                               hale_pool** out) {
    if (!ctx || !out || !policy) return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_pool_create_tiered: NULL argument");
    *out = nullptr;
    if (policy->n_pinned && !policy->pinned)
        return fail(ctx, HALE_E_INVALID_ARGUMENT, "policy lists %llu pinned keys but no key array",
                    (unsigned long long)policy->n_pinned);
    if (!is_quant(dtype)) return fail(ctx, HALE_E_INVALID_ARGUMENT, "expert pool dtype must be q8_0 or q4_0");
    if (hidden == 0 || inter == 0 || hidden % 32 || inter % 32)
        return fail(ctx, HALE_E_INVALID_ARGUMENT, "hidden (%u) and intermediate (%u) must be non-zero multiples of 32",
                    hidden, inter);
    if (n_layers == 0 || n_experts == 0 || n_experts > 256)
        return fail(ctx, HALE_E_INVALID_ARGUMENT, "need 1..256 experts and >= 1 layer (got %u, %u)", n_experts, n_layers);
    const size_t nk = (size_t)n_layers * n_experts;
    for (uint64_t i = 0; i < policy->n_pinned; i++)
        if (policy->pinned[i].layer >= n_layers || policy->pinned[i].expert >= n_experts)
            return fail(ctx, HALE_E_INVALID_ARGUMENT, "pinned expert L%uE%u out of range", policy->pinned[i].layer,
                        policy->pinned[i].expert);
    CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    hale_pool* p = new hale_pool();
    p->ctx = ctx;
    p->device = ctx->device;
    ctx->pools.insert(p);
    p->dtype = dtype;
    p->H = hidden;
    p->I = inter;
    p->L = n_layers;
    p->E = n_experts;
    p->tiered = true;
    p->expert_stride = 2 * tiled_bytes(dtype, inter, hidden) + tiled_bytes(dtype, hidden, inter);
    p->record_bytes = 2 * (size_t)inter * hale_row_bytes(dtype, hidden) + (size_t)hidden * hale_row_bytes(dtype, inter);
    std::vector<int64_t> pinned(policy->n_pinned);
    for (uint64_t i = 0; i < policy->n_pinned; i++)
        pinned[i] = (int64_t)policy->pinned[i].layer * n_experts + policy->pinned[i].expert;
    // slots: the pinned tier, the LRU at full budget, and one forward's
    // distinct experts (at most one layer's E) held while the LRU evicts them
    std::vector<uint8_t> seen(nk, 0);
    uint64_t n_pinned = 0;
    for (int64_t k : pinned)
        if (!seen[k]) {
            seen[k] = 1;
            n_pinned++;
        }
    const uint32_t n_slots = hale_tier::Book::slots_needed(nk, n_pinned, policy->lru_bytes, p->record_bytes, n_experts);
    const size_t dev_bytes = p->expert_stride * n_slots;
    bool ok = cudaMalloc(&p->data, dev_bytes) == cudaSuccess &&
              cudaMalloc(&p->staging, p->record_bytes) == cudaSuccess &&
              cudaMalloc(&p->scratch, p->expert_stride) == cudaSuccess &&
              cudaMalloc(&p->d_routing, nk * 8) == cudaSuccess && cudaMemset(p->d_routing, 0, nk * 8) == cudaSuccess &&
              cudaMalloc(&p->d_slot, nk * 4) == cudaSuccess && cudaMemset(p->d_slot, 0xff, nk * 4) == cudaSuccess &&
              cudaHostAlloc(&p->host_tier, p->expert_stride * nk, cudaHostAllocPortable) == cudaSuccess &&
              cudaHostAlloc(&p->h_slot, (size_t)n_experts * 4, cudaHostAllocPortable) == cudaSuccess &&
              cudaStreamCreateWithFlags(&p->copy_st, cudaStreamNonBlocking) == cudaSuccess &&
              cudaEventCreateWithFlags(&p->ev_issue, cudaEventDisableTiming) == cudaSuccess &&
              cudaEventCreate(&p->ev_t0) == cudaSuccess && cudaEventCreate(&p->ev_t1) == cudaSuccess &&
              cudaEventCreateWithFlags(&p->ev_done, cudaEventDisableTiming) == cudaSuccess;
    if (!ok) {
        cudaGetLastError();
        const size_t host_bytes = p->expert_stride * nk;
        hale_pool_destroy(p);
        return fail(ctx, HALE_E_OUT_OF_MEMORY, "cannot allocate a tiered pool (%zu bytes of HBM, %zu of host memory)",
                    dev_bytes, host_bytes);
    }
    p->resident.assign(nk, 0);
    p->layer_resident.assign(n_layers, 0);
    p->host_routing.assign(nk, 0);
    p->book.init(nk, pinned, policy->lru_bytes, p->record_bytes, n_slots);  // pinned keys take the first slots
    // CacheStats at construction (cache.rs:96-103)
    p->stats.pinned_experts = n_pinned;
    p->stats.pinned_bytes = n_pinned * p->record_bytes;
    p->stats.lru_capacity_bytes = policy->lru_bytes;
    pool_build_maps(p, n_slots);
    *out = p;
    return HALE_OK;
}

extern "C" uint64_t hale_pool_hbm_slots(const hale_pool* p) {
    return p ? (p->tiered ? p->book.n_slots : (uint64_t)p->L * p->E) : 0;
}

// ---- tier bookkeeping (host) ------------------------------------------------

// Folds the device-timed duration of the last batch of tier loads into
// load_seconds once it has completed.
static void tier_collect_timing(hale_pool* p) {
    if (!p->timing_pending) return;
    float ms = 0.f;
    if (cudaEventSynchronize(p->ev_t1) == cudaSuccess && cudaEventElapsedTime(&ms, p->ev_t0, p->ev_t1) == cudaSuccess)
        p->stats.load_seconds += ms * 1e-3;
    cudaGetLastError();
    p->timing_pending = false;
}

// The previous request's kernels have completed (waited for here): its held
// slots are released (hale_tier::Book::release).
static void tier_release(hale_pool* p) {
    if (p->done_recorded) {
        cudaEventSynchronize(p->ev_done);  // the previous forward may have run on another stream
        p->done_recorded = false;
    }
    p->book.release();
    tier_collect_timing(p);
}

// One ExpertCache::fetch request through the book; copies to issue go to
// `loads`.
static hale_status tier_request(hale_pool* p, const int64_t* keys, size_t n,
                                std::vector<std::pair<int32_t, int64_t>>& loads) {
    if (!p->book.request(keys, n, loads))
        return fail(p->ctx, HALE_E_OUT_OF_MEMORY, "tiered pool ran out of HBM slots (%u): one request names more "
                    "distinct experts than a layer has", p->book.n_slots);
    return HALE_OK;
}

// Host tier -> HBM slots on the copy stream, after the work already queued on
// `st`; `st` waits for the copies.
static hale_status tier_issue(hale_pool* p, const std::vector<std::pair<int32_t, int64_t>>& loads, cudaStream_t st) {
    hale_ctx* ctx = p->ctx;
    if (loads.empty()) return HALE_OK;
    CUDA_TRY(ctx, cudaEventRecord(p->ev_issue, st));
    CUDA_TRY(ctx, cudaStreamWaitEvent(p->copy_st, p->ev_issue, 0));
    CUDA_TRY(ctx, cudaEventRecord(p->ev_t0, p->copy_st));
    for (const auto& ld : loads)
        CUDA_TRY(ctx, cudaMemcpyAsync(p->data + (size_t)ld.first * p->expert_stride,
                                      p->host_tier + (size_t)ld.second * p->expert_stride, p->expert_stride,
                                      cudaMemcpyHostToDevice, p->copy_st));
    CUDA_TRY(ctx, cudaEventRecord(p->ev_t1, p->copy_st));
    CUDA_TRY(ctx, cudaStreamWaitEvent(st, p->ev_t1, 0));
    p->timing_pending = true;
    return HALE_OK;
}

extern "C" uint64_t hale_pool_expert_bytes(const hale_pool* p) { return p ? p->record_bytes : 0; }

extern "C" hale_status hale_pool_upload_expert(hale_pool* p, uint32_t layer, uint32_t expert, const void* record,
                                               uint64_t record_bytes, int on_device, void* stream) {
    if (!p) return fail(nullptr, HALE_E_INVALID_ARGUMENT, "hale_pool_upload_expert: pool is NULL");
    hale_ctx* ctx = p->ctx;
    if (!ctx) return fail(nullptr, HALE_E_INVALID_ARGUMENT, "the pool's context was destroyed");
    if (layer >= p->L || expert >= p->E)
        return fail(ctx, HALE_E_INVALID_ARGUMENT, "expert L%uE%u out of range", layer, expert);
    if (!record) return fail(ctx, HALE_E_INVALID_ARGUMENT, "record is NULL");
    if (record_bytes != p->record_bytes)
        return fail(ctx, HALE_E_BAD_TENSOR, "L%uE%u: record is %llu bytes, expected %zu", layer, expert,
                    (unsigned long long)record_bytes, p->record_bytes);
    auto t0 = std::chrono::steady_clock::now();
    CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    cudaStream_t st = S(stream);
    const uint8_t* src = static_cast<const uint8_t*>(record);
    if (!on_device) {
        CUDA_TRY(ctx, cudaMemcpyAsync(p->staging, record, record_bytes, cudaMemcpyHostToDevice, st));
        src = p->staging;
    }
    const size_t i = (size_t)layer * p->E + expert;
    // tiered: a pinned key is tiled straight into its slot, any other through
    // the scratch expert; both then land in the host tier
    uint8_t* dst = !p->tiered ? p->data + i * p->expert_stride
                              : (p->book.pinned_key[i] ? p->data + (size_t)p->book.slot_of[i] * p->expert_stride
                                                       : p->scratch);
    size_t proj = (size_t)p->I * hale_row_bytes(p->dtype, p->H);
    size_t gu_tiled = tiled_bytes(p->dtype, p->I, p->H);
    hale_status r;
    if ((r = launch_repack(ctx, p->dtype, src, dst, p->I, p->H, st))) return r;
    if ((r = launch_repack(ctx, p->dtype, src + proj, dst + gu_tiled, p->I, p->H, st))) return r;
    if ((r = launch_repack(ctx, p->dtype, src + 2 * proj, dst + 2 * gu_tiled, p->H, p->I, st))) return r;
    if (p->tiered) {
        CUDA_TRY(ctx, cudaMemcpyAsync(p->host_tier + i * p->expert_stride, dst, p->expert_stride,
                                      cudaMemcpyDeviceToHost, st));
        if (!p->book.pinned_key[i] && p->book.slot_of[i] >= 0)
            CUDA_TRY(ctx, cudaMemcpyAsync(p->data + (size_t)p->book.slot_of[i] * p->expert_stride, dst, p->expert_stride,
                                          cudaMemcpyDeviceToDevice, st));
    }
    CUDA_TRY(ctx, cudaStreamSynchronize(st));
    if (p->tiered) {
        // the cold tier is filled before serving; CacheStats counts only the
        // loads of fetch() (cache.rs:185-188)
        if (!p->resident[i]) {
            p->resident[i] = 1;
            p->layer_resident[layer]++;
        }
        return HALE_OK;
    }
    if (!p->resident[i]) {
        p->resident[i] = 1;
        p->layer_resident[layer]++;
        p->stats.pinned_experts++;
        p->stats.pinned_bytes += p->record_bytes;
    }
    p->stats.bytes_loaded += record_bytes;
    p->stats.load_seconds += std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    return HALE_OK;
}

static hale_status source_fill(hale_pool* p, const int64_t* keys, size_t n, cudaStream_t st);

extern "C" hale_status hale_pool_fetch(hale_pool* p, const hale_expert_key* keys, uint64_t n, hale_expert_view* out) {
    if (!p) return fail(nullptr, HALE_E_INVALID_ARGUMENT, "hale_pool_fetch: pool is NULL");
    hale_ctx* ctx = p->ctx;
    if (!ctx) return fail(nullptr, HALE_E_INVALID_ARGUMENT, "the pool's context was destroyed");
    if (n && (!keys || !out)) return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_pool_fetch: NULL buffer");
    if (p->tiered) {
        std::vector<int64_t> ks(n);
        for (uint64_t i = 0; i < n; i++) {
            if (keys[i].layer >= p->L || keys[i].expert >= p->E)
                return fail(ctx, HALE_E_INVALID_ARGUMENT, "expert L%uE%u out of range", keys[i].layer, keys[i].expert);
            ks[i] = (int64_t)keys[i].layer * p->E + keys[i].expert;
        }
        CUDA_TRY(ctx, cudaSetDevice(ctx->device));
        // the slots of the previous request may still be read by queued work
        CUDA_TRY(ctx, cudaDeviceSynchronize());
        hale_status rs = source_fill(p, ks.data(), n, nullptr);
        if (rs) return rs;
        tier_release(p);
        std::vector<std::pair<int32_t, int64_t>> loads;
        hale_status r = tier_request(p, ks.data(), n, loads);
        if (r) return r;
        if ((r = tier_issue(p, loads, p->copy_st))) return r;
        CUDA_TRY(ctx, cudaStreamSynchronize(p->copy_st));
        const size_t gu_tiled = tiled_bytes(p->dtype, p->I, p->H);
        for (uint64_t i = 0; i < n; i++) {
            const uint8_t* base = p->data + (size_t)p->book.slot_of[ks[i]] * p->expert_stride;
            out[i].gate = base;
            out[i].up = base + gu_tiled;
            out[i].down = base + 2 * gu_tiled;
        }
        return HALE_OK;
    }
    // routing is recorded before lookup, like ExpertCache::fetch (cache.rs:125-128)
    for (uint64_t i = 0; i < n; i++)
        if (keys[i].layer < p->L && keys[i].expert < p->E) p->host_routing[(size_t)keys[i].layer * p->E + keys[i].expert]++;
    uint64_t hits = 0;
    for (uint64_t i = 0; i < n; i++) {
        const hale_expert_key k = keys[i];
        if (k.layer >= p->L || k.expert >= p->E) {
            p->stats.misses++;
            return fail(ctx, HALE_E_INVALID_ARGUMENT, "expert L%uE%u out of range", k.layer, k.expert);
        }
        size_t idx = (size_t)k.layer * p->E + k.expert;
        if (!p->resident[idx]) {
            p->stats.misses++;
            return fail(ctx, HALE_E_INVALID_ARGUMENT, "expert L%uE%u is not resident in the pool", k.layer, k.expert);
        }
        const uint8_t* base = p->data + idx * p->expert_stride;
        size_t gu_tiled = tiled_bytes(p->dtype, p->I, p->H);
        out[i].gate = base;
        out[i].up = base + gu_tiled;
        out[i].down = base + 2 * gu_tiled;
        hits++;
    }
    p->stats.pinned_hits += hits;
    return HALE_OK;
}

extern "C" hale_status hale_pool_routing_counts(hale_pool* p, uint64_t* counts, uint64_t n) {
    if (!p || !counts) return fail(p ? p->ctx : nullptr, HALE_E_INVALID_ARGUMENT, "hale_pool_routing_counts: NULL");
    if (!p->ctx) return fail(nullptr, HALE_E_INVALID_ARGUMENT, "the pool's context was destroyed");
    size_t total = (size_t)p->L * p->E;
    if (n < total) return fail(p->ctx, HALE_E_INVALID_ARGUMENT, "counts needs %zu entries", total);
    CUDA_TRY(p->ctx, cudaSetDevice(p->ctx->device));
    std::vector<uint64_t> dev(total);
    CUDA_TRY(p->ctx, cudaDeviceSynchronize());
    CUDA_TRY(p->ctx, cudaMemcpy(dev.data(), p->d_routing, total * 8, cudaMemcpyDeviceToHost));
    for (size_t i = 0; i < total; i++)
        counts[i] = dev[i] + p->host_routing[i] + (p->tiered ? p->book.routing[i] : 0);
    return HALE_OK;
}

extern "C" hale_status hale_pool_stats(hale_pool* p, hale_cache_stats* out) {
    if (!p || !out) return fail(p ? p->ctx : nullptr, HALE_E_INVALID_ARGUMENT, "hale_pool_stats: NULL");
    if (!p->ctx) return fail(nullptr, HALE_E_INVALID_ARGUMENT, "the pool's context was destroyed");
    size_t total = (size_t)p->L * p->E;
    std::vector<uint64_t> dev(total);
    CUDA_TRY(p->ctx, cudaSetDevice(p->ctx->device));
    CUDA_TRY(p->ctx, cudaDeviceSynchronize());
    CUDA_TRY(p->ctx, cudaMemcpy(dev.data(), p->d_routing, total * 8, cudaMemcpyDeviceToHost));
    if (p->tiered) {
        // routes were counted on the host as they were resolved
        tier_collect_timing(p);
        *out = p->stats;
        out->pinned_hits = p->book.c.pinned_hits;
        out->lru_hits = p->book.c.lru_hits;
        out->misses = p->book.c.misses;
        out->bytes_loaded = p->book.c.bytes_loaded;
        out->lru_experts = p->book.lru.count;
        out->lru_bytes = p->book.lru.used;
        return HALE_OK;
    }
    *out = p->stats;
    for (size_t i = 0; i < total; i++) out->pinned_hits += dev[i];
    return HALE_OK;
}

// ---------------------------------------------------------------------------
// MoE layer
// ---------------------------------------------------------------------------
static hale_status check_layer(hale_ctx* ctx, const hale_moe_layer* ly, uint32_t H) {
    if (!ly) return fail(ctx, HALE_E_INVALID_ARGUMENT, "layer is NULL");
    if (!ly->router) return fail(ctx, HALE_E_INVALID_ARGUMENT, "router weights are NULL");
    if (!is_float(ly->router_dtype))
        return fail(ctx, HALE_E_INVALID_ARGUMENT, "router dtype must be f32, f16 or bf16");
    if (ly->n_experts == 0 || ly->n_experts > 256)
        return fail(ctx, HALE_E_INVALID_ARGUMENT, "router has %u experts (1..256 supported)", ly->n_experts);
    if (ly->top_k == 0 || ly->top_k > ly->n_experts || ly->top_k > 32)
        return fail(ctx, HALE_E_INVALID_ARGUMENT, "num_experts_per_tok (%u) must be in 1..=%u", ly->top_k,
                    std::min(ly->n_experts, 32u));
    if (H == 0) return fail(ctx, HALE_E_INVALID_ARGUMENT, "hidden size is 0");
    return HALE_OK;
}

static hale_status launch_router(hale_ctx* ctx, const hale_moe_layer* ly, uint32_t H, const float* x, uint32_t M,
                                 const MoeLayout& L, bool full, int32_t* user_idx, float* user_w, float* probs,
                                 unsigned long long* routing, cudaStream_t st) {
    uint8_t* ws = static_cast<uint8_t*>(ctx->ws);
    RouterArgs a{};
    a.w = ly->router;
    a.wdtype = float_code(ly->router_dtype);
    a.E = (int)ly->n_experts;
    a.H = (int)H;
    a.M = (int)M;
    a.k = (int)ly->top_k;
    a.normalize = ly->normalize_topk ? 1 : 0;
    // rows stream through shared memory when they are 16-byte aligned spans
    a.staged = (H % 8 == 0 && aligned16(x) && aligned16(ly->router)) ? 1 : 0;
    a.x = x;
    a.logits = reinterpret_cast<float*>(ws + L.logits);
    a.probs_out = probs;
    a.topk_idx = reinterpret_cast<int*>(ws + L.topk_idx);
    a.topk_w = reinterpret_cast<float*>(ws + L.topk_w);
    a.user_idx = user_idx;
    a.user_w = user_w;
    a.xq = full ? reinterpret_cast<int8_t*>(ws + L.xq) : nullptr;
    a.xaux = reinterpret_cast<int2*>(ws + L.xaux);
    a.elist_off = full ? reinterpret_cast<int*>(ws + L.elist_off) : nullptr;
    a.elist = reinterpret_cast<int*>(ws + L.elist);
    a.active = reinterpret_cast<int*>(ws + L.active);
    a.n_active = reinterpret_cast<int*>(ws + L.n_active);
    a.routing_counts = routing;
    a.tile_cnt = reinterpret_cast<unsigned*>(ws + L.tile_cnt);
    a.grid_cnt = reinterpret_cast<unsigned*>(ws + L.grid_cnt);
    a.err = ctx->d_err;
    dim3 grid((M + kRouterTT - 1) / kRouterTT, (a.E + kRouterET - 1) / kRouterET);
    const int nslots = std::min<int>(((int)H + kRouterCH - 1) / kRouterCH, kRouterSlots);
    size_t smem = a.staged ? (size_t)nslots * router_slot_bytes(a.wdtype == 0 ? 4 : 2) + 8 * nslots : 0;
    auto* kern = a.wdtype == 0 ? router_kernel<0> : (a.wdtype == 1 ? router_kernel<1> : router_kernel<2>);
    CUDA_TRY(ctx, allow_smem(kern, smem));
    ProfScope ps_(ctx, "router", st);
    kern<<<grid, 256, smem, st>>>(a);
    return check_launch(ctx, "router");
}

extern "C" hale_status hale_moe_route(hale_ctx* ctx, const hale_moe_layer* ly, uint32_t hidden, const float* x,
                                      uint32_t M, int32_t* topk_idx, float* topk_w, float* probs, void* stream) {
    if (!ctx) return fail(nullptr, HALE_E_INVALID_ARGUMENT, "hale_moe_route: ctx is NULL");
    hale_status r = check_layer(ctx, ly, hidden);
    if (r) return r;
    if (M == 0) return HALE_OK;
    if (!x || !topk_idx || !topk_w) return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_moe_route: NULL buffer");
    CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    MoeLayout L;
    int Hq = (int)((hidden + 31) / 32 * 32);
    if ((r = ensure_moe_ws(ctx, (int)M, (int)ly->n_experts, (int)ly->top_k, Hq, ctx->capI > 0 ? ctx->capI : 32, stream, &L)))
        return r;
    return launch_router(ctx, ly, hidden, x, M, L, false, topk_idx, topk_w, probs, nullptr, S(stream));
}

// Tensor-core expert kernels (hale_tc.cuh). A kind::i8 tcgen05.mma of K = 32
// (one quantization block) costs ~190 cycles of issue on B200 whatever its N
// (16..256), so with one MMA per 128 rows x 1 block they only pay off once
// experts see many tokens each; measured on the layer shapes here they are not
// yet faster than the dp4a kernels at any batch size, so "auto" keeps dp4a
// and HALE_EXPERT_KERNEL=tc selects them.
static constexpr uint32_t kTcMinTokens = 1u << 30;
static bool use_tc(const hale_ctx* ctx, hale_dtype dt, uint32_t M, int H, int I) {
    if ((ctx->expert_kernel != HALE_EXPERT_TC && ctx->expert_kernel != HALE_EXPERT_AUTO) || I % 64 != 0 ||
        H % 128 != 0)
        return false;
    if (ctx->expert_kernel == HALE_EXPERT_AUTO && M < kTcMinTokens) return false;
    return tc_plan_ok(dt == HALE_Q4_0 ? tc_plan(QFmt<0>::BB, TcStage<0>::SB) : tc_plan(QFmt<1>::BB, TcStage<1>::SB));
}

// Persistent launches: one CTA per SM (each holds 512 TMEM columns and most of
// the shared memory), looping over the (expert, 128-row) units.
template <int QT, int PW>
static hale_status expert_go_tc(hale_ctx* ctx, const ExpertArgs& a, unsigned max_active, cudaStream_t st) {
    const int TI = a.I / 32, TH = a.H / 32;
    const TcPlan P = tc_plan(QFmt<QT>::BB, TcStage<QT>::SB);
    CUDA_TRY(ctx, allow_smem(expert_gate_up_tc_kernel<QT, PW>, (size_t)P.total));
    CUDA_TRY(ctx, allow_smem(expert_down_tc_kernel<QT, PW>, (size_t)P.total));
    const unsigned sms = (unsigned)ctx->sm_count;
    unsigned g1 = std::min(max_active * (unsigned)(TI / 2), sms), g2 = std::min(max_active * (unsigned)(TH / 4), sms);
    {
        ProfScope ps_(ctx, "expert_gate_up", st);
        expert_gate_up_tc_kernel<QT, PW><<<g1, kTcThreads, P.total, st>>>(a);
    }
    hale_status r = check_launch(ctx, "expert_gate_up_tc");
    if (r) return r;
    {
        ProfScope ps_(ctx, "expert_down", st);
        expert_down_tc_kernel<QT, PW><<<g2, kTcThreads, P.total, st>>>(a);
    }
    return check_launch(ctx, "expert_down_tc");
}

// Persistent streaming kernels (hale_stream.cuh): kPsCtas CTAs per SM, each
// with its share of shared memory, so one CTA's per-pass epilogue overlaps
// another's streaming.
static constexpr int kPsCtas = 2;
static constexpr int kPsBudget = (kPsCtas == 1 ? 219 : 104) * 1024;
static bool use_ps(const hale_ctx* ctx, hale_dtype dt, uint32_t M, int H, int I) {
    if (ctx->expert_kernel != HALE_EXPERT_PS || I % 64 != 0 || H % 128 != 0) return false;
    const int bb = block_bytes(dt), sb = ps_stage_blocks(dt == HALE_Q4_0 ? 0 : 1, kPsCtas);
    return ps_plan_ok(ps_plan(bb, sb, H, kPsBudget), kPsBudget) && ps_plan_ok(ps_plan(bb, sb, I, kPsBudget), kPsBudget);
}

template <int QT>
static hale_status expert_go_ps(hale_ctx* ctx, const ExpertArgs& a, unsigned max_active, cudaStream_t st) {
    const int TI = a.I / 32, TH = a.H / 32, sb = ps_stage_blocks(QT, kPsCtas);
    const PsPlan P1 = ps_plan(QFmt<QT>::BB, sb, a.H, kPsBudget);
    const PsPlan P2 = ps_plan(QFmt<QT>::BB, sb, a.I, kPsBudget);
    CUDA_TRY(ctx, allow_smem(expert_gate_up_ps_kernel<QT>, (size_t)P1.total));
    CUDA_TRY(ctx, allow_smem(expert_down_ps_kernel<QT>, (size_t)P2.total));
    const unsigned slots = (unsigned)(ctx->sm_count * kPsCtas);
    unsigned g1 = std::min(max_active * (unsigned)(TI / 2), slots), g2 = std::min(max_active * (unsigned)(TH / 4), slots);
    {
        ProfScope ps_(ctx, "expert_gate_up", st);
        expert_gate_up_ps_kernel<QT><<<g1, kPsThreads, P1.total, st>>>(a, kPsBudget, sb);
    }
    hale_status r = check_launch(ctx, "expert_gate_up_ps");
    if (r) return r;
    {
        ProfScope ps_(ctx, "expert_down", st);
        expert_down_ps_kernel<QT><<<g2, kPsThreads, P2.total, st>>>(a, kPsBudget, sb);
    }
    return check_launch(ctx, "expert_down_ps");
}

// Warp-specialised streaming kernels (hale_ws.cuh): two persistent CTAs per
// SM, weights by TMA tensor loads through the pool's maps. "auto" takes them
// from kWsMinTokens tokens (the per-CTA kernels keep the smallest batches,
// where more CTAs per expert win).
static constexpr uint32_t kWsMinTokens = 3;
static bool use_ws(const hale_ctx* ctx, const hale_pool* p, uint32_t M, int k, int E) {
    (void)k;
    (void)E;
    if (!p->ws_maps || (ctx->expert_kernel != HALE_EXPERT_AUTO && ctx->expert_kernel != HALE_EXPERT_WS)) return false;
    return ctx->expert_kernel == HALE_EXPERT_WS || M >= kWsMinTokens;
}

template <int QT, int CPS, int NG>
static hale_status expert_go_ws(hale_ctx* ctx, const hale_pool* p, const ExpertArgs& a, unsigned max_active,
                                unsigned* ctr, int xb, cudaStream_t st) {
    const int TI = a.I / 32, TH = a.H / 32, rec = 32 * QFmt<QT>::BB, budget = ws_budget(CPS), rows = kPassRows * NG;
    const WsPlan P1 = ws_plan(rec, 2, 2, kWsSB, a.H, budget, xb, rows);
    const WsPlan P2 = ws_plan(rec, 1, 4, kWsSB, a.I, budget, xb, rows);
    CUDA_TRY(ctx, allow_smem(expert_gate_up_ws_kernel<QT, CPS, NG>, (size_t)P1.total));
    CUDA_TRY(ctx, allow_smem(expert_down_ws_kernel<QT, CPS, NG>, (size_t)P2.total));
    const unsigned slots = (unsigned)(ctx->sm_count * CPS);
    const unsigned g1 = std::min(max_active * (unsigned)(TI / 2), slots);
    const unsigned g2 = std::min(max_active * (unsigned)(TH / 4), slots);
    {
        ProfScope ps_(ctx, "expert_gate_up", st);
        expert_gate_up_ws_kernel<QT, CPS, NG><<<g1, kWsThreads, P1.total, st>>>(p->map_gu, a, P1, ctr);
    }
    hale_status r = check_launch(ctx, "expert_gate_up_ws");
    if (r) return r;
    {
        ProfScope ps_(ctx, "expert_down", st);
        expert_down_ws_kernel<QT, CPS, NG><<<g2, kWsThreads, P2.total, st>>>(p->map_d, a, P2, ctr + 2);
    }
    return check_launch(ctx, "expert_down_ws");
}

template <int QT>
static hale_status expert_go_ws_cfg(hale_ctx* ctx, const hale_pool* p, const ExpertArgs& a, unsigned max_active,
                                    uint32_t M, int k, int E, cudaStream_t st) {
    // routes per active expert the batch can have on average
    const long long routes = (long long)M * k, experts = std::min<long long>(E, routes);
    const bool narrow = experts > 0 && routes < 2 * experts;
    const WsCfg c = ws_config(p->dtype, a.H, a.I, narrow);
    unsigned* ctr = a.ws_cnt;
    if (c.cps == 4) return expert_go_ws<QT, 4, 1>(ctx, p, a, max_active, ctr, c.xb, st);
    if (c.cps == 3) return expert_go_ws<QT, 3, 1>(ctx, p, a, max_active, ctr, c.xb, st);
    return expert_go_ws<QT, 2, 1>(ctx, p, a, max_active, ctr, c.xb, st);
}

template <int QT, int RT>
static hale_status expert_go(hale_ctx* ctx, const ExpertArgs& a, unsigned max_active, cudaStream_t st) {
    const int TI = a.I / 32, TH = a.H / 32;
    SmemPlan P1 = smem_plan(QFmt<QT>::BB, a.S1, 2 * RT, a.H);
    SmemPlan P2 = smem_plan(QFmt<QT>::BB, a.S2, 4, a.I);
    CUDA_TRY(ctx, allow_smem(expert_gate_up_kernel<QT, RT>, (size_t)P1.total));
    CUDA_TRY(ctx, allow_smem(expert_down_kernel<QT>, (size_t)P2.total));
    unsigned g1 = max_active * (unsigned)((TI + RT - 1) / RT), g2 = max_active * (unsigned)((TH + 3) / 4);
    {
        ProfScope ps_(ctx, "expert_gate_up", st);
        expert_gate_up_kernel<QT, RT><<<g1, 64 * RT, P1.total, st>>>(a);
    }
    hale_status r = check_launch(ctx, "expert_gate_up");
    if (r) return r;
    {
        ProfScope ps_(ctx, "expert_down", st);
        expert_down_kernel<QT><<<g2, 128, P2.total, st>>>(a);
    }
    return check_launch(ctx, "expert_down");
}

static hale_status launch_experts(hale_ctx* ctx, const hale_pool* p, ExpertArgs& a, uint32_t M, int k, int E,
                                  cudaStream_t st);

// ExpertSource::load (src/expert/mod.rs:110-124) for the keys of a request
// whose experts were never uploaded: the source hands over the pack record,
// which goes through hale_pool_upload_expert into the host tier. Runs before
// the request touches the cache book, so a failed load leaves the pool as it
// was; it comes back as HALE_E_IO (the reference's HaleError::Io).
static hale_status source_fill(hale_pool* p, const int64_t* keys, size_t n, cudaStream_t st) {
    hale_ctx* ctx = p->ctx;
    for (size_t i = 0; i < n; i++) {
        const int64_t key = keys[i];
        if (p->resident[key]) continue;
        const uint32_t layer = (uint32_t)(key / p->E), expert = (uint32_t)(key % p->E);
        if (!p->source)
            return fail(ctx, HALE_E_INVALID_ARGUMENT, "expert L%uE%u was never uploaded and the pool has no source",
                        layer, expert);
        p->source_buf.resize(p->record_bytes);
        const int32_t rc = p->source(p->source_user, layer, expert, p->source_buf.data(), p->record_bytes);
        if (rc != 0)
            return fail(ctx, HALE_E_IO, "ExpertSource::load failed for L%uE%u (source returned %d)", layer, expert,
                        rc);
        hale_status r = hale_pool_upload_expert(p, layer, expert, p->source_buf.data(), p->record_bytes, 0, st);
        if (r) return r;
    }
    return HALE_OK;
}

extern "C" hale_status hale_pool_set_source(hale_pool* p, hale_expert_source_fn fn, void* user) {
    if (!p || !p->ctx) return fail(nullptr, HALE_E_INVALID_ARGUMENT, "hale_pool_set_source: bad pool");
    if (!p->tiered) return fail(p->ctx, HALE_E_UNSUPPORTED, "an HBM-resident pool holds every expert; no source");
    p->source = fn;
    p->source_user = user;
    return HALE_OK;
}

// A tiered pool's forward: read the routes back (the calling thread waits for
// the router), resolve them one token at a time in top-k order, copy the
// misses into HBM slots on the side stream and publish this layer's slot row
// for the expert kernels, which `st` orders after the copies.
static hale_status tier_forward(hale_pool* p, uint32_t layer, const int* d_routes, uint32_t M, int k,
                                cudaStream_t st) {
    hale_ctx* ctx = p->ctx;
    const size_t n = (size_t)M * k;
    if (n > p->h_routes_cap) {
        cudaFreeHost(p->h_routes);
        p->h_routes = nullptr;
        p->h_routes_cap = 0;
        CUDA_TRY(ctx, cudaHostAlloc(&p->h_routes, n * 4, cudaHostAllocPortable));
        p->h_routes_cap = n;
    }
    CUDA_TRY(ctx, cudaMemcpyAsync(p->h_routes, d_routes, n * 4, cudaMemcpyDeviceToHost, st));
    // also completes every earlier forward's kernels, so held slots can go
    CUDA_TRY(ctx, cudaStreamSynchronize(st));
    {
        std::vector<int64_t> ks(n);
        for (size_t i = 0; i < n; i++) {
            const int e = p->h_routes[i];
            if (e < 0 || (uint32_t)e >= p->E) return fail(ctx, HALE_E_DEVICE_CHECK, "route %d out of range", e);
            ks[i] = (int64_t)layer * p->E + e;
        }
        hale_status r = source_fill(p, ks.data(), n, st);
        if (r) return r;
    }
    tier_release(p);
    std::vector<std::pair<int32_t, int64_t>> loads;
    std::vector<int64_t> keys(k);
    for (uint32_t t = 0; t < M; t++) {
        for (int j = 0; j < k; j++) {
            const int e = p->h_routes[(size_t)t * k + j];
            if (e < 0 || (uint32_t)e >= p->E) return fail(ctx, HALE_E_DEVICE_CHECK, "route %d out of range", e);
            keys[j] = (int64_t)layer * p->E + e;
        }
        hale_status r = tier_request(p, keys.data(), (size_t)k, loads);
        if (r) return r;
    }
    hale_status r = tier_issue(p, loads, st);
    if (r) return r;
    for (uint32_t e = 0; e < p->E; e++) p->h_slot[e] = p->book.slot_of[(size_t)layer * p->E + e];
    CUDA_TRY(ctx, cudaMemcpyAsync(p->d_slot + (size_t)layer * p->E, p->h_slot, (size_t)p->E * 4,
                                  cudaMemcpyHostToDevice, st));
    return HALE_OK;
}

// One token through an HBM-resident pool: the whole layer in one launch
// (moe_token_kernel). "auto" only; the other families keep their kernels.
static bool use_token(const hale_ctx* ctx, const hale_pool* p, const hale_moe_layer* ly, uint32_t M) {
    return M == 1 && !p->tiered && ctx->expert_kernel == HALE_EXPERT_AUTO && p->H % 128 == 0 && p->I % 32 == 0 &&
           aligned16(ly->router) && ly->top_k <= 32 && ly->n_experts <= 256 &&
           (p->dtype == HALE_Q4_0 || p->dtype == HALE_Q8_0);
}

// CTAs of moe_token_kernel one SM holds at `smem` bytes (cached per device
// and size; the grid must never exceed what the GPU holds at once, since its
// CTAs wait for one another).
template <class F>
static int token_occupancy(F* kern, size_t smem) {
    static std::mutex mu;
    static std::map<std::pair<int, std::pair<const void*, size_t>>, int> memo;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    auto key = std::make_pair(dev, std::make_pair(reinterpret_cast<const void*>(kern), smem));
    auto it = memo.find(key);
    if (it != memo.end()) return it->second;
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kTokThreads, smem) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
    }
    memo[key] = n;
    return n;
}

template <int QT, int DT>
static hale_status token_go(hale_ctx* ctx, TokenArgs a, cudaStream_t st, bool* done) {
    auto* kern = moe_token_kernel<QT, DT>;
    constexpr int wb = DT == 0 ? 4 : 2;
    const int need = std::max(std::max(a.k * (a.I / 32), a.H / kTokDownRows), a.E);
    int rpc = 1, G = 0;
    size_t smem = 0;
    for (int pass = 0; pass < 3; pass++) {
        smem = (size_t)tok_plan(QFmt<QT>::BB, wb, a.H, a.I, a.k, rpc).total;
        if (smem > 200 * 1024) return HALE_OK;  // not this kernel's shapes: the three-launch path
        CUDA_TRY(ctx, allow_smem(kern, smem));
        const int occ = token_occupancy(kern, smem);
        G = std::min(need, ctx->sm_count * occ);
        if (G <= 0) return HALE_OK;
        const int r2 = (a.E + G - 1) / G;
        if (r2 == rpc) break;
        rpc = r2;
        G = 0;
    }
    if (G <= 0 || rpc > 32) return HALE_OK;
    a.rpc = rpc;
    a.prefetch_all = a.k * (a.I / 32) > G ? 1 : 0;
    {
        ProfScope ps_(ctx, "moe_token", st);
        kern<<<G, kTokThreads, smem, st>>>(a);
    }
    hale_status r = check_launch(ctx, "moe_token");
    if (!r) *done = true;
    return r;
}

// RMSNorm folded in front of a one-token layer (the decoder's post-attention
// norm): input = rmsnorm(x + delta) * w; x + delta goes to x_out.
struct TokNorm {
    const float* delta;
    const float* w;
    float eps;
    float* x_out;
};

static hale_status launch_token(hale_ctx* ctx, const hale_pool* p, const hale_moe_layer* ly, const float* x,
                                const MoeLayout& L, float* out, int32_t* topk_idx, float* topk_w, cudaStream_t st,
                                bool* done, const TokNorm* norm = nullptr) {
    uint8_t* ws = static_cast<uint8_t*>(ctx->ws);
    TokenArgs a{};
    a.router = ly->router;
    a.E = (int)p->E;
    a.H = (int)p->H;
    a.I = (int)p->I;
    a.k = (int)ly->top_k;
    a.normalize = ly->normalize_topk ? 1 : 0;
    a.x = x;
    a.logits = reinterpret_cast<float*>(ws + L.logits);
    a.topk_idx = reinterpret_cast<int*>(ws + L.topk_idx);
    a.topk_w = reinterpret_cast<float*>(ws + L.topk_w);
    a.user_idx = topk_idx;
    a.user_w = topk_w;
    a.routing_counts = p->d_routing + (size_t)ly->layer * p->E;
    a.experts = p->data + (size_t)ly->layer * p->E * p->expert_stride;
    a.expert_stride = p->expert_stride;
    a.hq = reinterpret_cast<int8_t*>(ws + L.hq);
    a.haux = reinterpret_cast<int2*>(ws + L.haux);
    a.out = out;
    a.bar = reinterpret_cast<unsigned*>(ws + L.tok_bar);
    a.err = ctx->d_err;
    if (norm) {
        a.delta = norm->delta;
        a.norm_w = norm->w;
        a.eps = norm->eps;
        a.x_out = norm->x_out;
    }
    const int dt = float_code(ly->router_dtype);
    if (p->dtype == HALE_Q4_0)
        return dt == 0 ? token_go<0, 0>(ctx, a, st, done)
                       : (dt == 1 ? token_go<0, 1>(ctx, a, st, done) : token_go<0, 2>(ctx, a, st, done));
    return dt == 0 ? token_go<1, 0>(ctx, a, st, done)
                   : (dt == 1 ? token_go<1, 1>(ctx, a, st, done) : token_go<1, 2>(ctx, a, st, done));
}

extern "C" hale_status hale_moe_forward(hale_ctx* ctx, hale_pool* p, const hale_moe_layer* ly, const float* x,
                                        uint32_t M, float* out, int32_t* topk_idx, float* topk_w, void* stream) {
    if (!ctx || !p) return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_moe_forward: NULL ctx or pool");
    if (p->ctx != ctx) return fail(ctx, HALE_E_INVALID_ARGUMENT, "pool belongs to another context");
    hale_status r = check_layer(ctx, ly, p->H);
    if (r) return r;
    if (ly->layer >= p->L) return fail(ctx, HALE_E_INVALID_ARGUMENT, "layer %u has no experts in the pool", ly->layer);
    if (ly->n_experts != p->E)
        return fail(ctx, HALE_E_INVALID_ARGUMENT, "router has %u experts, pool has %u", ly->n_experts, p->E);
    if (p->layer_resident[ly->layer] != p->E && !(p->tiered && p->source))
        return fail(ctx, HALE_E_INVALID_ARGUMENT, "layer %u: only %u of %u experts are resident", ly->layer,
                    p->layer_resident[ly->layer], p->E);
    if (M == 0) return HALE_OK;
    if (!x || !out) return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_moe_forward: NULL buffer");
    if (!aligned16(x)) return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_moe_forward: x must be 16-byte aligned");
    CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    const int E = (int)p->E, k = (int)ly->top_k, H = (int)p->H, I = (int)p->I;
    MoeLayout L;
    if ((r = ensure_moe_ws(ctx, (int)M, E, k, H, I, stream, &L))) return r;
    cudaStream_t st = S(stream);
    if (p->tiered && stream_capturing(stream))
        return fail(ctx, HALE_E_UNSUPPORTED, "a tiered pool resolves routes on the host; its forward cannot be captured");
    if (use_token(ctx, p, ly, M)) {
        bool done = false;
        if ((r = launch_token(ctx, p, ly, x, L, out, topk_idx, topk_w, st, &done))) return r;
        if (done) return HALE_OK;
    }
    if ((r = launch_router(ctx, ly, p->H, x, M, L, true, topk_idx, topk_w, nullptr,
                           p->tiered ? nullptr : p->d_routing + (size_t)ly->layer * p->E, st)))
        return r;
    uint8_t* ws = static_cast<uint8_t*>(ctx->ws);
    ExpertArgs a{};
    if (p->tiered) {
        if ((r = tier_forward(p, ly->layer, reinterpret_cast<const int*>(ws + L.topk_idx), M, k, st))) return r;
        a.experts = p->data;
        a.slot = p->d_slot + (size_t)ly->layer * p->E;
    } else {
        a.experts = p->data + (size_t)ly->layer * p->E * p->expert_stride;
        a.expert0 = (int)(ly->layer * p->E);
    }
    a.expert_stride = p->expert_stride;
    a.H = H;
    a.I = I;
    a.k = k;
    a.M = (int)M;
    a.elist_off = reinterpret_cast<int*>(ws + L.elist_off);
    a.elist = reinterpret_cast<int*>(ws + L.elist);
    a.active = reinterpret_cast<int*>(ws + L.active);
    a.n_active = reinterpret_cast<int*>(ws + L.n_active);
    a.xq = reinterpret_cast<int8_t*>(ws + L.xq);
    a.xaux = reinterpret_cast<int2*>(ws + L.xaux);
    a.hq = reinterpret_cast<int8_t*>(ws + L.hq);
    a.haux = reinterpret_cast<int2*>(ws + L.haux);
    a.ybuf = reinterpret_cast<float*>(ws + L.ybuf);
    a.comb_cnt = reinterpret_cast<unsigned*>(ws + L.comb_cnt);
    a.ws_cnt = reinterpret_cast<unsigned*>(ws + L.ws_cnt);
    a.topk_w = reinterpret_cast<float*>(ws + L.topk_w);
    a.out = out;
    a.err = ctx->d_err;
    r = launch_experts(ctx, p, a, M, k, E, st);
    if (!r && p->tiered) {
        CUDA_TRY(ctx, cudaEventRecord(p->ev_done, st));
        p->done_recorded = true;
    }
    return r;
}

// The decoder's post-attention RMSNorm and a one-token MoE layer in one
// launch when the token kernel serves the layer (*done), else nothing is
// launched and the caller runs the two separately.
static hale_status moe_token_norm(hale_ctx* ctx, hale_pool* p, const hale_moe_layer* ly, const float* x,
                                  const TokNorm& norm, float* out, cudaStream_t st, bool* done) {
    *done = false;
    if (!use_token(ctx, p, ly, 1) || p->H > 4u * kTokNormVec * kTokThreads || ly->layer >= p->L ||
        ly->n_experts != p->E ||
        p->layer_resident[ly->layer] != p->E || !aligned16(x) || !aligned16(norm.delta) || !aligned16(norm.x_out))
        return HALE_OK;
    MoeLayout L;
    hale_status r = ensure_moe_ws(ctx, 1, (int)p->E, (int)ly->top_k, (int)p->H, (int)p->I, st, &L);
    if (r) return r;
    return launch_token(ctx, p, ly, x, L, out, nullptr, nullptr, st, done, &norm);
}

// The expert kernels over the routes in a (expert lists built, activations
// quantized): the family by context setting and batch shape.
static hale_status launch_experts(hale_ctx* ctx, const hale_pool* p, ExpertArgs& a, uint32_t M, int k, int E,
                                  cudaStream_t st) {
    const hale_dtype dt = p->dtype;
    const int H = a.H, I = a.I;
    // ring depth, capped at the stages one tile has
    // ring depth: deep rings only for a single token, where a CTA's whole
    // tile stream fits in flight; from two tokens on, two stages per warp
    // keep more CTAs resident (measured faster at 2, 4, 8, 64 and 512 tokens)
    const int depth = M <= 1 ? ring_stages(dt, M) : 2;
    a.S1 = std::min(depth, (H / 32 + kStageBlocks - 1) / kStageBlocks);
    a.S2 = std::min(depth, (I / 32 + kStageBlocks - 1) / kStageBlocks);
    unsigned max_active = (unsigned)std::min<long long>(E, (long long)M * k);
    if (use_ws(ctx, p, M, k, E))
        return dt == HALE_Q4_0 ? expert_go_ws_cfg<0>(ctx, p, a, max_active, M, k, E, st)
                               : expert_go_ws_cfg<1>(ctx, p, a, max_active, M, k, E, st);
    if (use_tc(ctx, dt, M, H, I)) {
        // 16-token passes once experts average ~16 tokens; 8-token passes below
        const bool wide = (long long)M * k >= 16LL * E;
        if (dt == HALE_Q4_0)
            return wide ? expert_go_tc<0, 16>(ctx, a, max_active, st) : expert_go_tc<0, 8>(ctx, a, max_active, st);
        return wide ? expert_go_tc<1, 16>(ctx, a, max_active, st) : expert_go_tc<1, 8>(ctx, a, max_active, st);
    }
    if (use_ps(ctx, dt, M, H, I))
        return dt == HALE_Q4_0 ? expert_go_ps<0>(ctx, a, max_active, st) : expert_go_ps<1>(ctx, a, max_active, st);
    // small batches: one row tile per CTA pair of warps, for more CTAs
    bool small = M <= 2;
    if (dt == HALE_Q4_0)
        return small ? expert_go<0, 1>(ctx, a, max_active, st) : expert_go<0, 2>(ctx, a, max_active, st);
    return small ? expert_go<1, 1>(ctx, a, max_active, st) : expert_go<1, 2>(ctx, a, max_active, st);
}

// The host-buffer call's work on stream st: x in, the layer, results out.
static hale_status moe_forward_host_enqueue(hale_ctx* ctx, hale_pool* p, const hale_moe_layer* ly,
                                            const float* x_host, uint32_t M, float* out_host, int32_t* idx_host,
                                            float* w_host, cudaStream_t st) {
    const size_t xb = (size_t)M * p->H * 4, kb = (size_t)M * ly->top_k * 4;
    uint8_t* s = static_cast<uint8_t*>(ctx->scratch);
    float* dx = reinterpret_cast<float*>(s);
    float* dout = reinterpret_cast<float*>(s + align_up(xb, 256));
    int32_t* didx = reinterpret_cast<int32_t*>(s + 2 * align_up(xb, 256));
    float* dw = reinterpret_cast<float*>(s + 2 * align_up(xb, 256) + align_up(kb, 256));
    CUDA_TRY(ctx, cudaMemcpyAsync(dx, x_host, xb, cudaMemcpyHostToDevice, st));
    hale_status r = hale_moe_forward(ctx, p, ly, dx, M, dout, idx_host ? didx : nullptr, w_host ? dw : nullptr, st);
    if (r) return r;
    CUDA_TRY(ctx, cudaMemcpyAsync(out_host, dout, xb, cudaMemcpyDeviceToHost, st));
    if (idx_host) CUDA_TRY(ctx, cudaMemcpyAsync(idx_host, didx, kb, cudaMemcpyDeviceToHost, st));
    if (w_host) CUDA_TRY(ctx, cudaMemcpyAsync(w_host, dw, kb, cudaMemcpyDeviceToHost, st));
    return HALE_OK;
}

static bool host_pinned(const void* p) {
    if (!p) return true;
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeHost;
}

static bool same_layer(const hale_moe_layer& a, const hale_moe_layer& b) {
    return a.layer == b.layer && a.router == b.router && a.router_dtype == b.router_dtype &&
           a.n_experts == b.n_experts && a.top_k == b.top_k && a.normalize_topk == b.normalize_topk;
}

extern "C" hale_status hale_moe_forward_host(hale_ctx* ctx, hale_pool* p, const hale_moe_layer* ly,
                                             const float* x_host, uint32_t M, float* out_host,
                                             int32_t* idx_host, float* w_host, void* stream) {
    if (!ctx || !p) return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_moe_forward_host: NULL ctx or pool");
    if (M == 0) return HALE_OK;
    if (!x_host || !out_host) return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_moe_forward_host: NULL buffer");
    hale_status r = check_layer(ctx, ly, p->H);
    if (r) return r;
    CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    size_t xb = (size_t)M * p->H * 4, kb = (size_t)M * ly->top_k * 4;
    size_t need = 2 * align_up(xb, 256) + 2 * align_up(kb, 256);
    if ((r = ensure_scratch(ctx, need, stream))) return r;
    cudaStream_t st = S(stream);
    // Repeated calls with the same pool, layer, size and page-locked buffers
    // replay one CUDA graph of the whole call (copies, three kernels, the
    // error word): one launch instead of eight. Tiered pools resolve routes
    // on the host mid-call and always run step by step.
    const bool graphable = !p->tiered && !ctx->profiling && !stream_capturing(stream);
    if (graphable) {
        for (const auto& g : ctx->host_graphs)
            if (g.pool == p && same_layer(g.layer, *ly) && g.M == M && g.x == x_host && g.out == out_host &&
                g.idx == idx_host && g.w == w_host && g.gen == ctx->ws_gen) {
                CUDA_TRY(ctx, cudaGraphLaunch(g.exec, st));
                CUDA_TRY(ctx, cudaStreamSynchronize(st));
                if (*ctx->h_err == 0) return HALE_OK;
                return hale_ctx_check(ctx, stream);
            }
    }
    if ((r = moe_forward_host_enqueue(ctx, p, ly, x_host, M, out_host, idx_host, w_host, st))) return r;
    r = hale_ctx_check(ctx, stream);
    if (r || !graphable) return r;
    // this call sized the workspaces: capture it for the next ones
    if (!host_pinned(x_host) || !host_pinned(out_host) || !host_pinned(idx_host) || !host_pinned(w_host))
        return HALE_OK;
    if (!ctx->cap_st && cudaStreamCreateWithFlags(&ctx->cap_st, cudaStreamNonBlocking) != cudaSuccess) {
        cudaGetLastError();
        ctx->cap_st = nullptr;
        return HALE_OK;
    }
    if (!ctx->h_err && cudaHostAlloc(reinterpret_cast<void**>(&ctx->h_err), 4, cudaHostAllocDefault) != cudaSuccess) {
        cudaGetLastError();
        ctx->h_err = nullptr;
        return HALE_OK;
    }
    const uint64_t gen = ctx->ws_gen;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    if (cudaStreamBeginCapture(ctx->cap_st, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        cudaGetLastError();
        return HALE_OK;
    }
    hale_status cr = moe_forward_host_enqueue(ctx, p, ly, x_host, M, out_host, idx_host, w_host, ctx->cap_st);
    const bool copied = cudaMemcpyAsync(ctx->h_err, ctx->d_err, 4, cudaMemcpyDeviceToHost, ctx->cap_st) == cudaSuccess;
    const cudaError_t ec = cudaStreamEndCapture(ctx->cap_st, &graph);
    if (cr || !copied || ec != cudaSuccess || !graph || gen != ctx->ws_gen ||
        cudaGraphInstantiate(&exec, graph, 0) != cudaSuccess) {
        cudaGetLastError();
        if (exec) cudaGraphExecDestroy(exec);
        exec = nullptr;
        g_thread_status = HALE_OK;
    }
    if (graph) cudaGraphDestroy(graph);
    if (exec) {
        if (ctx->host_graphs.size() >= 8) {
            cudaGraphExecDestroy(ctx->host_graphs.front().exec);
            ctx->host_graphs.erase(ctx->host_graphs.begin());
        }
        ctx->host_graphs.push_back({p, *ly, M, x_host, out_host, idx_host, w_host, gen, exec});
    }
    return HALE_OK;
}

// ---------------------------------------------------------------------------
// sampling tail
// ---------------------------------------------------------------------------
// ---------------------------------------------------------------------------
// Expert parallelism (hale_ep.cuh): the device work on either side of the
// two all-to-all-v exchanges the host performs.
// ---------------------------------------------------------------------------
extern "C" int32_t hale_q8_aux_pairs(uint32_t cols) { return aux_stride((int)(cols / 32)); }

extern "C" hale_status hale_ep_dispatch(hale_ctx* ctx, const hale_moe_layer* ly, uint32_t hidden, const float* x,
                                        uint32_t M, uint32_t n_ranks, int8_t* send_q, int32_t* send_aux,
                                        int32_t* send_meta, uint64_t* counts_host, int32_t* topk_idx, float* topk_w,
                                        void* stream) {
    if (!ctx) return fail(nullptr, HALE_E_INVALID_ARGUMENT, "hale_ep_dispatch: ctx is NULL");
    hale_status r = check_layer(ctx, ly, hidden);
    if (r) return r;
    if (hidden % 32 != 0) return fail(ctx, HALE_E_INVALID_ARGUMENT, "hidden (%u) must be a multiple of 32", hidden);
    if (n_ranks == 0 || ly->n_experts % n_ranks != 0)
        return fail(ctx, HALE_E_INVALID_ARGUMENT, "%u experts do not split evenly over %u ranks", ly->n_experts,
                    n_ranks);
    if (!counts_host) return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_ep_dispatch: counts is NULL");
    if (M == 0) {
        for (uint32_t i = 0; i < n_ranks; i++) counts_host[i] = 0;
        return HALE_OK;
    }
    if (!x || !send_q || !send_aux || !send_meta)
        return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_ep_dispatch: NULL buffer");
    if (!aligned16(x) || !aligned16(send_q) || !aligned16(send_aux) || !aligned16(send_meta))
        return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_ep_dispatch: buffers must be 16-byte aligned");
    CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    const int E = (int)ly->n_experts, k = (int)ly->top_k, H = (int)hidden;
    MoeLayout L;
    if ((r = ensure_moe_ws(ctx, (int)M, E, k, H, ctx->capI > 0 ? ctx->capI : 32, stream, &L))) return r;
    if ((r = ensure_scratch(ctx, (size_t)n_ranks * 8, stream))) return r;
    cudaStream_t st = S(stream);
    if ((r = launch_router(ctx, ly, hidden, x, M, L, true, topk_idx, topk_w, nullptr, nullptr, st))) return r;
    uint8_t* ws = static_cast<uint8_t*>(ctx->ws);
    const int n = (int)M * k, nbp = aux_stride(H / 32);
    {
        ProfScope ps_(ctx, "ep_pack", st);
        ep_pack_kernel<<<(n + 7) / 8, 256, 0, st>>>(
            reinterpret_cast<const int*>(ws + L.elist), reinterpret_cast<const int*>(ws + L.topk_idx),
            reinterpret_cast<const float*>(ws + L.topk_w), reinterpret_cast<const int8_t*>(ws + L.xq),
            reinterpret_cast<const int2*>(ws + L.xaux), n, k, H, nbp, send_q, reinterpret_cast<int2*>(send_aux),
            reinterpret_cast<EpMeta*>(send_meta));
    }
    if ((r = check_launch(ctx, "ep_pack"))) return r;
    auto* d_counts = static_cast<unsigned long long*>(ctx->scratch);
    ep_rank_counts_kernel<<<1, 256, 0, st>>>(reinterpret_cast<const int*>(ws + L.elist_off), (int)n_ranks,
                                             E / (int)n_ranks, d_counts);
    if ((r = check_launch(ctx, "ep_rank_counts"))) return r;
    CUDA_TRY(ctx, cudaMemcpyAsync(counts_host, d_counts, (size_t)n_ranks * 8, cudaMemcpyDeviceToHost, st));
    CUDA_TRY(ctx, cudaStreamSynchronize(st));
    return HALE_OK;
}

extern "C" hale_status hale_ep_experts(hale_ctx* ctx, hale_pool* p, uint32_t layer, uint32_t expert0,
                                       const int8_t* recv_q, const int32_t* recv_aux, const int32_t* recv_meta,
                                       uint32_t n, float* y, void* stream) {
    if (!ctx || !p) return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_ep_experts: NULL ctx or pool");
    if (p->ctx != ctx) return fail(ctx, HALE_E_INVALID_ARGUMENT, "pool belongs to another context");
    if (p->tiered) return fail(ctx, HALE_E_UNSUPPORTED, "hale_ep_experts needs an HBM-resident pool");
    if (layer >= p->L) return fail(ctx, HALE_E_INVALID_ARGUMENT, "layer %u has no experts in the pool", layer);
    if (p->layer_resident[layer] != p->E)
        return fail(ctx, HALE_E_INVALID_ARGUMENT, "layer %u: only %u of %u experts are resident", layer,
                    p->layer_resident[layer], p->E);
    if (n == 0) return HALE_OK;
    if (!recv_q || !recv_aux || !recv_meta || !y)
        return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_ep_experts: NULL buffer");
    if (!aligned16(recv_q) || !aligned16(recv_aux) || !aligned16(recv_meta))
        return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_ep_experts: buffers must be 16-byte aligned");
    CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    const int El = (int)p->E, H = (int)p->H, I = (int)p->I;
    MoeLayout L;
    hale_status r;
    if ((r = ensure_moe_ws(ctx, (int)n, El, 1, H, I, stream, &L))) return r;
    cudaStream_t st = S(stream);
    uint8_t* ws = static_cast<uint8_t*>(ctx->ws);
    const EpMeta* meta = reinterpret_cast<const EpMeta*>(recv_meta);
    int* cursor = reinterpret_cast<int*>(ws + L.logits);  // [El], free on this side
    ep_count_kernel<<<1, 1024, (size_t)El * 4, st>>>(meta, (int)n, (int)expert0, El,
                                                      reinterpret_cast<int*>(ws + L.elist_off), cursor,
                                                      reinterpret_cast<int*>(ws + L.active),
                                                      reinterpret_cast<int*>(ws + L.n_active), ctx->d_err);
    if ((r = check_launch(ctx, "ep_count"))) return r;
    ep_scatter_kernel<<<(n + 255) / 256, 256, 0, st>>>(meta, (int)n, (int)expert0, El,
                                                        reinterpret_cast<const int*>(ws + L.elist_off), cursor,
                                                        reinterpret_cast<int*>(ws + L.elist),
                                                        reinterpret_cast<float*>(ws + L.topk_w));
    if ((r = check_launch(ctx, "ep_scatter"))) return r;
    // every record is one token with one route of weight 1: the combine of
    // the expert kernels then writes y itself (0 + 1 * y == y)
    ExpertArgs a{};
    a.experts = p->data + (size_t)layer * p->E * p->expert_stride;
    a.expert0 = (int)(layer * p->E);
    a.expert_stride = p->expert_stride;
    a.H = H;
    a.I = I;
    a.k = 1;
    a.M = (int)n;
    a.elist_off = reinterpret_cast<int*>(ws + L.elist_off);
    a.elist = reinterpret_cast<int*>(ws + L.elist);
    a.active = reinterpret_cast<int*>(ws + L.active);
    a.n_active = reinterpret_cast<int*>(ws + L.n_active);
    a.xq = recv_q;
    a.xaux = reinterpret_cast<const int2*>(recv_aux);
    a.hq = reinterpret_cast<int8_t*>(ws + L.hq);
    a.haux = reinterpret_cast<int2*>(ws + L.haux);
    a.ybuf = reinterpret_cast<float*>(ws + L.ybuf);
    a.comb_cnt = reinterpret_cast<unsigned*>(ws + L.comb_cnt);
    a.ws_cnt = reinterpret_cast<unsigned*>(ws + L.ws_cnt);
    a.topk_w = reinterpret_cast<float*>(ws + L.topk_w);
    a.out = y;
    a.err = ctx->d_err;
    return launch_experts(ctx, p, a, n, 1, El, st);
}

extern "C" hale_status hale_ep_combine(hale_ctx* ctx, const int32_t* send_meta, const float* y_back, uint32_t M,
                                       uint32_t top_k, uint32_t hidden, float* out, void* stream) {
    if (!ctx) return fail(nullptr, HALE_E_INVALID_ARGUMENT, "hale_ep_combine: ctx is NULL");
    if (M == 0) return HALE_OK;
    if (!send_meta || !y_back || !out) return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_ep_combine: NULL buffer");
    if (top_k == 0 || top_k > 32 || hidden == 0)
        return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_ep_combine: top_k %u / hidden %u out of range", top_k, hidden);
    CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    hale_status r;
    const size_t n = (size_t)M * top_k;
    if ((r = ensure_scratch(ctx, n * 4, stream))) return r;
    cudaStream_t st = S(stream);
    int* pos = static_cast<int*>(ctx->scratch);
    CUDA_TRY(ctx, cudaMemsetAsync(pos, 0xFF, n * 4, st));
    const EpMeta* meta = reinterpret_cast<const EpMeta*>(send_meta);
    ep_pos_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(meta, (int)n, (int)M, (int)top_k, pos, ctx->d_err);
    if ((r = check_launch(ctx, "ep_pos"))) return r;
    {
        ProfScope ps_(ctx, "ep_combine", st);
        ep_combine_kernel<<<dim3((hidden + 255) / 256, M), 256, 0, st>>>(meta, pos, y_back, (int)n, (int)M,
                                                                          (int)top_k, (int)hidden, out, ctx->d_err);
    }
    return check_launch(ctx, "ep_combine");
}

// ---------------------------------------------------------------------------
// Expert parallelism over NVLink peer memory (hale_p2p.cuh)
// ---------------------------------------------------------------------------
// NCCL serves only the communicator's set-up: the ranks all-gather their
// exchange blocks' CUDA IPC handles. It is loaded at run time, so the
// library has no link-time dependency on it and one-GPU use never loads it.
struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*destroy)(ncclComm_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
    bool ok = false;
};

static const NcclApi& nccl_api() {
    static std::once_flag once;
    static NcclApi api;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
        api.init_rank = reinterpret_cast<decltype(api.init_rank)>(dlsym(h, "ncclCommInitRank"));
        api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
        api.destroy = reinterpret_cast<decltype(api.destroy)>(dlsym(h, "ncclCommDestroy"));
        api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
        api.ok = api.get_unique_id && api.init_rank && api.all_gather && api.destroy && api.error_string;
    });
    return api;
}

static_assert(sizeof(ncclUniqueId) == HALE_COMM_ID_BYTES, "ncclUniqueId size");

struct hale_comm {
    hale_ctx* ctx = nullptr;
    int device = 0;
    uint32_t R = 1, rank = 0, H = 0, E = 0, k = 0, max_tokens = 0, epr = 0;
    P2pLayout L{};
    uint8_t* block = nullptr;          // this rank's exchange block
    P2pPeers peers{};
    std::vector<uint8_t*> opened;      // peers' blocks mapped through IPC
    ncclComm_t nccl = nullptr;
    uint8_t* d_setup = nullptr;        // handle all-gather buffer
    unsigned* d_done = nullptr;        // dispatch CTA counter
    // owner-side lists of one call (kept apart from the ctx workspace, whose
    // route arrays the home's combine still needs)
    float* d_ones = nullptr;           // [R * cap]
    float** d_out_rows = nullptr;      // [R * cap]
    int* d_elist = nullptr;            // [R * cap]
    int* d_lists = nullptr;            // elist_off [epr + 1], active [epr], n_active
    unsigned long long epoch = 0;
};

extern "C" hale_status hale_comm_unique_id(void* id) {
    if (!id) return fail(nullptr, HALE_E_INVALID_ARGUMENT, "hale_comm_unique_id: NULL buffer");
    const NcclApi& api = nccl_api();
    if (!api.ok) return fail(nullptr, HALE_E_UNSUPPORTED, "NCCL (libnccl.so.2) is not loadable");
    ncclUniqueId u;
    const ncclResult_t r = api.get_unique_id(&u);
    if (r != ncclSuccess) return fail(nullptr, HALE_E_NCCL, "ncclGetUniqueId: %s", api.error_string(r));
    std::memcpy(id, &u, sizeof u);
    return HALE_OK;
}

static void comm_free(hale_comm* c) {
    if (c->ctx) c->ctx->comms.erase(c);
    for (uint8_t* p : c->opened) cudaIpcCloseMemHandle(p);
    c->opened.clear();
    cudaFree(c->block);
    cudaFree(c->d_setup);
    cudaFree(c->d_done);
    cudaFree(c->d_ones);
    cudaFree(c->d_out_rows);
    cudaFree(c->d_elist);
    cudaFree(c->d_lists);
    if (c->nccl) nccl_api().destroy(c->nccl);
    delete c;
}

// Per rank, in the set-up all-gather: the block's IPC handle and the shape
// every rank must agree on.
struct CommSlot {
    cudaIpcMemHandle_t handle;
    uint32_t shape[8];
    uint8_t pad[32];
};
static_assert(sizeof(CommSlot) == 128, "CommSlot");

extern "C" hale_status hale_comm_create(hale_ctx* ctx, uint32_t n_ranks, uint32_t rank, const void* unique_id,
                                        uint32_t hidden, uint32_t n_experts, uint32_t top_k, uint32_t max_tokens,
                                        hale_comm** out) {
    if (!ctx || !out) return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_comm_create: NULL argument");
    *out = nullptr;
    if (n_ranks == 0 || n_ranks > (uint32_t)kP2pMaxRanks || rank >= n_ranks)
        return fail(ctx, HALE_E_INVALID_ARGUMENT, "rank %u of %u ranks (1..%d ranks supported)", rank, n_ranks,
                    kP2pMaxRanks);
    if (n_experts == 0 || n_experts > 256 || n_experts % n_ranks)
        return fail(ctx, HALE_E_INVALID_ARGUMENT, "%u experts do not split evenly over %u ranks", n_experts, n_ranks);
    if (hidden == 0 || hidden % 32 || top_k == 0 || top_k > n_experts || top_k > 32 || max_tokens == 0 ||
        max_tokens > 65536)
        return fail(ctx, HALE_E_INVALID_ARGUMENT, "bad shape (hidden %u, top_k %u, max_tokens %u)", hidden, top_k,
                    max_tokens);
    if (n_ranks > 1 && !unique_id) return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_comm_create: NULL unique id");
    CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    hale_comm* c = new hale_comm();
    c->ctx = ctx;
    c->device = ctx->device;
    ctx->comms.insert(c);
    c->R = n_ranks;
    c->rank = rank;
    c->H = hidden;
    c->E = n_experts;
    c->k = top_k;
    c->max_tokens = max_tokens;
    c->epr = n_experts / n_ranks;
    const int cap = (int)(max_tokens * std::min(top_k, c->epr));
    c->L = p2p_layout((int)n_ranks, (int)hidden, aux_stride((int)hidden / 32), cap, (int)(max_tokens * top_k));
    const size_t nrec = (size_t)n_ranks * cap;
    bool ok = cudaMalloc(&c->block, c->L.total) == cudaSuccess && cudaMemset(c->block, 0, c->L.total) == cudaSuccess &&
              cudaMalloc(&c->d_done, 4) == cudaSuccess && cudaMemset(c->d_done, 0, 4) == cudaSuccess &&
              cudaMalloc(&c->d_ones, nrec * 4) == cudaSuccess &&
              cudaMalloc(&c->d_out_rows, nrec * sizeof(float*)) == cudaSuccess &&
              cudaMalloc(&c->d_elist, nrec * 4) == cudaSuccess &&
              cudaMalloc(&c->d_lists, (2 * (size_t)c->epr + 2) * 4) == cudaSuccess &&
              cudaMalloc(&c->d_setup, (size_t)n_ranks * sizeof(CommSlot)) == cudaSuccess;
    if (!ok) {
        cudaGetLastError();
        comm_free(c);
        return fail(ctx, HALE_E_OUT_OF_MEMORY, "cannot allocate the %zu-byte exchange block", (size_t)c->L.total);
    }
    c->peers.base[rank] = c->block;
    if (n_ranks > 1) {
        const NcclApi& api = nccl_api();
        if (!api.ok) {
            comm_free(c);
            return fail(ctx, HALE_E_UNSUPPORTED, "NCCL (libnccl.so.2) is not loadable");
        }
        ncclUniqueId uid;
        std::memcpy(&uid, unique_id, sizeof uid);
        ncclResult_t nr = api.init_rank(&c->nccl, (int)n_ranks, uid, (int)rank);
        if (nr != ncclSuccess) {
            c->nccl = nullptr;
            comm_free(c);
            return fail(ctx, HALE_E_NCCL, "ncclCommInitRank: %s", api.error_string(nr));
        }
        CommSlot mine{};
        if (cudaIpcGetMemHandle(&mine.handle, c->block) != cudaSuccess) {
            cudaGetLastError();
            comm_free(c);
            return fail(ctx, HALE_E_CUDA, "cudaIpcGetMemHandle of the exchange block failed");
        }
        const uint32_t shape[8] = {n_ranks, hidden, n_experts, top_k, max_tokens, 0x48414c45u, 1u, 0u};
        std::memcpy(mine.shape, shape, sizeof shape);
        std::vector<CommSlot> all(n_ranks);
        cudaStream_t st = nullptr;
        ok = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) == cudaSuccess &&
             cudaMemcpy(c->d_setup + (size_t)rank * sizeof(CommSlot), &mine, sizeof mine, cudaMemcpyHostToDevice) ==
                 cudaSuccess;
        if (ok) {
            nr = api.all_gather(c->d_setup + (size_t)rank * sizeof(CommSlot), c->d_setup, sizeof(CommSlot), ncclUint8,
                                c->nccl, st);
            ok = nr == ncclSuccess && cudaStreamSynchronize(st) == cudaSuccess &&
                 cudaMemcpy(all.data(), c->d_setup, all.size() * sizeof(CommSlot), cudaMemcpyDeviceToHost) ==
                     cudaSuccess;
        }
        if (st) cudaStreamDestroy(st);
        if (!ok) {
            cudaGetLastError();
            comm_free(c);
            return fail(ctx, HALE_E_NCCL, "exchange of IPC handles failed");
        }
        for (uint32_t r = 0; r < n_ranks; r++)
            if (std::memcmp(all[r].shape, shape, sizeof shape) != 0) {
                comm_free(c);
                return fail(ctx, HALE_E_INVALID_ARGUMENT, "rank %u created its communicator with another shape", r);
            }
        for (uint32_t r = 0; r < n_ranks; r++) {
            if (r == rank) continue;
            void* p = nullptr;
            if (cudaIpcOpenMemHandle(&p, all[r].handle, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
                cudaGetLastError();
                comm_free(c);
                return fail(ctx, HALE_E_CUDA, "cannot map rank %u's exchange block (peer access over NVLink)", r);
            }
            c->opened.push_back(static_cast<uint8_t*>(p));
            c->peers.base[r] = static_cast<uint8_t*>(p);
        }
    }
    // weight 1 for every record: the expert kernels' combine then stores y
    std::vector<float> ones(nrec, 1.0f);
    if (cudaMemcpy(c->d_ones, ones.data(), nrec * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
        cudaGetLastError();
        comm_free(c);
        return fail(ctx, HALE_E_CUDA, "communicator set-up copy failed");
    }
    *out = c;
    return HALE_OK;
}

extern "C" hale_status hale_comm_destroy(hale_comm* c) {
    if (!c) return HALE_OK;
    cudaSetDevice(c->device);
    cudaDeviceSynchronize();
    hale_status r = HALE_OK;
    if (c->R > 1 && c->nccl) {
        // every rank is past its last call before any block goes away
        const NcclApi& api = nccl_api();
        cudaStream_t st = nullptr;
        if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) == cudaSuccess) {
            const ncclResult_t nr = api.all_gather(c->d_setup + (size_t)c->rank * sizeof(CommSlot), c->d_setup,
                                                   sizeof(CommSlot), ncclUint8, c->nccl, st);
            if (nr != ncclSuccess || cudaStreamSynchronize(st) != cudaSuccess)
                r = fail(c->ctx, HALE_E_NCCL, "hale_comm_destroy: closing barrier failed");
            cudaStreamDestroy(st);
        }
    }
    comm_free(c);
    return r;
}

extern "C" hale_status hale_moe_forward_ep(hale_ctx* ctx, hale_comm* c, hale_pool* p, const hale_moe_layer* ly,
                                           const float* x, uint32_t M, float* out, int32_t* topk_idx, float* topk_w,
                                           void* stream) {
    if (!ctx || !c || !p) return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_moe_forward_ep: NULL ctx, comm or pool");
    if (c->ctx != ctx || p->ctx != ctx)
        return fail(ctx, HALE_E_INVALID_ARGUMENT, "communicator or pool belongs to another context");
    hale_status r = check_layer(ctx, ly, p->H);
    if (r) return r;
    if (p->tiered) return fail(ctx, HALE_E_UNSUPPORTED, "expert parallelism needs an HBM-resident pool");
    if (ly->n_experts != c->E || ly->top_k != c->k || p->H != c->H || p->E != c->epr)
        return fail(ctx, HALE_E_INVALID_ARGUMENT,
                    "layer (%u experts, top-%u), pool (%u experts, hidden %u) and communicator (%u experts over %u "
                    "ranks, top-%u, hidden %u) disagree",
                    ly->n_experts, ly->top_k, p->E, p->H, c->E, c->R, c->k, c->H);
    if (ly->layer >= p->L || p->layer_resident[ly->layer] != p->E)
        return fail(ctx, HALE_E_INVALID_ARGUMENT, "layer %u: this rank's experts are not all resident", ly->layer);
    if (M > c->max_tokens)
        return fail(ctx, HALE_E_INVALID_ARGUMENT, "%u tokens exceed the communicator's %u", M, c->max_tokens);
    if (M > 0 && (!x || !out)) return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_moe_forward_ep: NULL buffer");
    if (M > 0 && !aligned16(x)) return fail(ctx, HALE_E_INVALID_ARGUMENT, "x must be 16-byte aligned");
    CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    const int H = (int)p->H, I = (int)p->I, k = (int)c->k, E = (int)c->E, El = (int)c->epr;
    const int nrec = (int)c->R * c->L.cap;
    // one workspace plan for both sides, so nothing reallocates mid-call
    MoeLayout L;
    if ((r = ensure_moe_ws(ctx, std::max<int>((int)M, nrec), E, k, H, I, stream, &L))) return r;
    cudaStream_t st = S(stream);
    uint8_t* ws = static_cast<uint8_t*>(ctx->ws);
    const unsigned long long epoch = ++c->epoch;
    const int half = (int)(epoch & 1);
    // 1. home: route and quantize this rank's tokens, records to their owners
    if (M > 0) {
        if ((r = launch_router(ctx, ly, p->H, x, M, L, true, topk_idx, topk_w, nullptr, nullptr, st))) return r;
    }
    {
        P2pDispatchArgs d{};
        d.peers = c->peers;
        d.L = c->L;
        d.rank = (int)c->rank;
        d.half = half;
        d.k = k;
        d.epr = El;
        d.epoch = epoch;
        d.n = (int)M * k;
        d.elist = reinterpret_cast<const int*>(ws + L.elist);
        d.elist_off = reinterpret_cast<const int*>(ws + L.elist_off);
        d.topk_idx = reinterpret_cast<const int*>(ws + L.topk_idx);
        d.topk_w = reinterpret_cast<const float*>(ws + L.topk_w);
        d.xq = reinterpret_cast<const int8_t*>(ws + L.xq);
        d.xaux = reinterpret_cast<const int2*>(ws + L.xaux);
        d.done = c->d_done;
        if (M == 0) {
            // no routes: the counts are zero -- elist_off of an empty call
            CUDA_TRY(ctx, cudaMemsetAsync(ws + L.elist_off, 0, (size_t)(E + 1) * 4, st));
        }
        ProfScope ps_(ctx, "ep_dispatch", st);
        p2p_dispatch_kernel<<<std::max(1u, (unsigned)((d.n + 7) / 8)), 256, 0, st>>>(d);
    }
    if ((r = check_launch(ctx, "p2p_dispatch"))) return r;
    // 2. owner: every home's records for this call, grouped by local expert
    int* elist_off = c->d_lists;
    int* active = c->d_lists + El + 1;
    int* n_active = c->d_lists + 2 * El + 1;
    {
        P2pGatherArgs g{};
        g.peers = c->peers;
        g.L = c->L;
        g.rank = (int)c->rank;
        g.half = half;
        g.k = k;
        g.expert0 = (int)c->rank * El;
        g.El = El;
        g.epoch = epoch;
        g.elist_off = elist_off;
        g.elist = c->d_elist;
        g.active = active;
        g.n_active = n_active;
        g.ones = c->d_ones;
        g.out_rows = c->d_out_rows;
        g.err = ctx->d_err;
        CUDA_TRY(ctx, allow_smem(p2p_gather_kernel, (size_t)2 * El * 4));
        ProfScope ps_(ctx, "ep_gather", st);
        p2p_gather_kernel<<<1, 1024, (size_t)2 * El * 4, st>>>(g);
    }
    if ((r = check_launch(ctx, "p2p_gather"))) return r;
    // 3. owner: the local experts at k = 1; each record's y goes to its home
    {
        ExpertArgs a{};
        a.experts = p->data + (size_t)ly->layer * p->E * p->expert_stride;
        a.expert0 = (int)(ly->layer * p->E);
        a.expert_stride = p->expert_stride;
        a.H = H;
        a.I = I;
        a.k = 1;
        a.M = nrec;
        a.elist_off = elist_off;
        a.elist = c->d_elist;
        a.active = active;
        a.n_active = n_active;
        a.xq = reinterpret_cast<const int8_t*>(c->block + c->L.q + (size_t)half * nrec * H);
        a.xaux = reinterpret_cast<const int2*>(c->block + c->L.a + (size_t)half * nrec * c->L.nbp * 8);
        a.hq = reinterpret_cast<int8_t*>(ws + L.hq);
        a.haux = reinterpret_cast<int2*>(ws + L.haux);
        a.ybuf = reinterpret_cast<float*>(ws + L.ybuf);
        a.comb_cnt = reinterpret_cast<unsigned*>(ws + L.comb_cnt);
        a.ws_cnt = reinterpret_cast<unsigned*>(ws + L.ws_cnt);
        a.topk_w = c->d_ones;
        a.out = nullptr;
        a.out_rows = c->d_out_rows;
        a.err = ctx->d_err;
        // the families whose combine honours out_rows: streaming, else per-CTA
        const int saved = ctx->expert_kernel;
        ctx->expert_kernel = p->ws_maps ? HALE_EXPERT_WS : HALE_EXPERT_DP4A;
        r = launch_experts(ctx, p, a, (uint32_t)nrec, 1, El, st);
        ctx->expert_kernel = saved;
        if (r) return r;
    }
    // 4. owner -> homes: this rank's y rows are all written
    p2p_signal_kernel<<<1, 32, 0, st>>>(c->peers, c->L, (int)c->rank, half, epoch);
    if ((r = check_launch(ctx, "p2p_signal"))) return r;
    // 5. home: best-first combine once every owner has signalled
    {
        ProfScope ps_(ctx, "ep_combine", st);
        p2p_combine_kernel<<<dim3((unsigned)((H + 255) / 256), std::max(1u, M)), 256, 0, st>>>(
            c->block, c->L, half, epoch, reinterpret_cast<const float*>(ws + L.topk_w), (int)M, k, out, ctx->d_err);
    }
    return check_launch(ctx, "p2p_combine");
}

// ---------------------------------------------------------------------------
// Decode step of the whole model (hale_decoder.cuh)
// ---------------------------------------------------------------------------
// A float matrix in the lane-major layout (fgemv_lanes_kernel): cols a
// multiple of 64, at most 12288 (its activation row is staged in shared
// memory). Host row-major data in.
static hale_status matrix_create_lanes(hale_ctx* ctx, hale_dtype dt, uint32_t rows, uint32_t cols, const void* host,
                                       hale_matrix** out) {
    *out = nullptr;
    const int es = dt == HALE_F32 ? 4 : 2;
    hale_matrix* m = new hale_matrix();
    m->ctx = ctx;
    m->device = ctx->device;
    ctx->matrices.insert(m);
    m->dtype = dt;
    m->rows = rows;
    m->cols = cols;
    m->rows_pad = (rows + 3) / 4 * 4;
    m->nb = cols / 8;
    m->lanes = true;
    m->bytes = (size_t)m->rows_pad * cols * es;
    uint8_t* tmp = nullptr;
    const size_t src_bytes = (size_t)rows * cols * es;
    if (cudaMalloc(&m->data, m->bytes) != cudaSuccess || cudaMalloc(&tmp, src_bytes) != cudaSuccess ||
        cudaMemcpy(tmp, host, src_bytes, cudaMemcpyHostToDevice) != cudaSuccess) {
        cudaFree(tmp);
        cudaFree(m->data);
        delete m;
        return fail(ctx, HALE_E_OUT_OF_MEMORY, "cannot stage a %ux%u float matrix", rows, cols);
    }
    const unsigned grid = (unsigned)std::min<size_t>((m->bytes / es + 255) / 256, 65535);
    if (es == 4) repack_lanes_kernel<4><<<grid, 256>>>(tmp, m->data, (int)rows, (int)m->rows_pad, (int)cols);
    else repack_lanes_kernel<2><<<grid, 256>>>(tmp, m->data, (int)rows, (int)m->rows_pad, (int)cols);
    const cudaError_t e1 = cudaGetLastError(), e2 = cudaDeviceSynchronize();
    cudaFree(tmp);
    if (e1 != cudaSuccess || e2 != cudaSuccess) {
        cudaFree(m->data);
        delete m;
        return fail(ctx, HALE_E_CUDA, "lane-major repack failed: %s", cudaGetErrorString(e1 ? e1 : e2));
    }
    *out = m;
    return HALE_OK;
}

static bool lanes_ok(hale_dtype dt, uint32_t cols) { return is_float(dt) && cols % 64 == 0 && cols <= 12288; }

struct hale_decoder {
    struct Layer {
        float *in_norm = nullptr, *post_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
        hale_matrix *qkv = nullptr, *o = nullptr, *gate = nullptr, *up = nullptr, *down = nullptr;
        int is_moe = 0;
        void* router = nullptr;
        hale_dtype router_dtype = HALE_F32;
        uint32_t pool_layer = 0, inter = 0;
    };
    hale_ctx* ctx = nullptr;
    int device = 0;
    hale_pool* pool = nullptr;
    hale_comm* comm = nullptr;  // set: MoE layers run expert-parallel (hale_moe_forward_ep)
    uint32_t H = 0, L = 0, nh = 0, nkv = 0, hd = 0, V = 0, E = 0, k = 0, max_len = 0;
    uint32_t n_seqs = 1, max_batch = 1;
    size_t seq_stride = 0;  // floats per sequence in one layer's K (or V) cache
    int normalize = 0;
    float eps = 0.0f, scale = 0.0f;
    std::vector<Layer> layers;
    void* embed = nullptr;
    hale_dtype embed_dtype = HALE_F32;
    hale_matrix* lm_head = nullptr;
    float* final_norm = nullptr;
    float *rope_cos = nullptr, *rope_sin = nullptr, *kcache = nullptr, *vcache = nullptr;
    float *x = nullptr, *normed = nullptr, *delta = nullptr, *qkv = nullptr, *attn = nullptr;
    float* x2 = nullptr;  // second residual buffer: norms folded into their consumers write x + delta here
    float* moe_out = nullptr;  // a fused norm + MoE layer writes its output here (it reads delta)
    float *g = nullptr, *u = nullptr, *h = nullptr, *scores = nullptr;
    std::vector<void*> allocs;
    // step rows (token, position, sequence) through device memory from a
    // pinned slot, so a captured step replays for any token
    uint32_t* d_rows = nullptr;
    uint32_t* h_rows = nullptr;
    cudaEvent_t ev_copied = nullptr;
    bool copied_recorded = false;
    cudaStream_t cap = nullptr;
    cudaGraphExec_t exec = nullptr;
    float *g_logits = nullptr, *g_hidden = nullptr;
    uint64_t g_gen = 0;  // ctx->ws_gen the graph was captured against
    bool no_graph = false;
    uint32_t smem_scores = 0;  // attention scores kept in shared memory up to this many positions
    size_t attn_smem = 0;      // attention's dynamic shared memory
    // GQA-grouped attention (head_dim <= 256): heads per CTA at one row and in
    // batched steps, and each variant's shared-memory layout
    bool gqa = false;
    int gc_one = 1, gc_batch = 1;
    int gqa_cap[9] = {0};
    size_t gqa_smem[9] = {0};
    // hale_decoder_generate's buffers, made on its first call: logits [V],
    // sampler state, sampled token, seen ids [max_len]; the token's pinned
    // host copy; events around prefill and decode
    float* gen_logits = nullptr;
    uint64_t* gen_rng = nullptr;
    int32_t* gen_tok = nullptr;
    int32_t* gen_seen = nullptr;
    int32_t* h_tok = nullptr;
    cudaEvent_t gen_ev[3] = {nullptr, nullptr, nullptr};
    // single-row attention over the whole GPU (attn_split_kernel)
    bool split = false;
    int split_grid = 0, split_npm = 0;
    size_t split_smem = 0;
    float *split_sc = nullptr, *split_pm = nullptr;
    unsigned* split_bar = nullptr;
};

extern "C" void hale_decoder_destroy(hale_decoder* d) {
    if (!d) return;
    if (d->ctx) d->ctx->decoders.erase(d);
    cudaSetDevice(d->device);
    cudaDeviceSynchronize();
    if (d->exec) cudaGraphExecDestroy(d->exec);
    if (d->cap) cudaStreamDestroy(d->cap);
    if (d->ev_copied) cudaEventDestroy(d->ev_copied);
    if (d->h_rows) cudaFreeHost(d->h_rows);
    if (d->h_tok) cudaFreeHost(d->h_tok);
    for (cudaEvent_t e : d->gen_ev)
        if (e) cudaEventDestroy(e);
    for (auto& ly : d->layers)
        for (hale_matrix* m : {ly.qkv, ly.o, ly.gate, ly.up, ly.down})
            if (m) hale_matrix_destroy(m);
    if (d->lm_head) hale_matrix_destroy(d->lm_head);
    for (void* p : d->allocs) cudaFree(p);
    delete d;
}

extern "C" hale_status hale_decoder_set_comm(hale_decoder* d, hale_comm* c) {
    if (!d || !d->ctx) return fail(nullptr, HALE_E_INVALID_ARGUMENT, "hale_decoder_set_comm: bad decoder");
    hale_ctx* ctx = d->ctx;
    if (!c) {
        d->comm = nullptr;
        return HALE_OK;
    }
    if (c->ctx != ctx) return fail(ctx, HALE_E_INVALID_ARGUMENT, "communicator belongs to another context");
    if (!d->pool) return fail(ctx, HALE_E_INVALID_ARGUMENT, "decoder has no MoE layers");
    if (c->E != d->E || c->k != d->k || c->H != d->H || d->pool->E != c->epr || d->pool->tiered)
        return fail(ctx, HALE_E_INVALID_ARGUMENT,
                    "communicator (%u experts over %u ranks, top-%u, hidden %u) does not match the decoder "
                    "(%u experts, top-%u, hidden %u) and its pool of %u resident experts per layer",
                    c->E, c->R, c->k, c->H, d->E, d->k, d->H, d->pool->E);
    if (c->max_tokens < d->max_batch)
        return fail(ctx, HALE_E_INVALID_ARGUMENT, "communicator takes %u tokens per call, decoder steps up to %u",
                    c->max_tokens, d->max_batch);
    d->comm = c;
    // every call advances the exchange's epoch: steps run eagerly
    d->no_graph = true;
    if (d->exec) {
        cudaGraphExecDestroy(d->exec);
        d->exec = nullptr;
    }
    return HALE_OK;
}

static hale_status dec_alloc(hale_ctx* ctx, hale_decoder* d, size_t bytes, void** out) {
    if (cudaMalloc(out, std::max(bytes, (size_t)16)) != cudaSuccess)
        return fail(ctx, HALE_E_OUT_OF_MEMORY, "decoder: cannot allocate %zu bytes", bytes);
    d->allocs.push_back(*out);
    CUDA_TRY(ctx, cudaMemset(*out, 0, bytes));
    return HALE_OK;
}

static hale_status dec_upload(hale_ctx* ctx, hale_decoder* d, const void* host, size_t bytes, void** out) {
    hale_status r = dec_alloc(ctx, d, bytes, out);
    if (r) return r;
    CUDA_TRY(ctx, cudaMemcpy(*out, host, bytes, cudaMemcpyHostToDevice));
    return HALE_OK;
}

static hale_status dec_matrix(hale_ctx* ctx, const hale_host_matrix& m, uint32_t rows, uint32_t cols,
                              const char* what, hale_matrix** out) {
    if (!is_float((hale_dtype)m.dtype))
        return fail(ctx, HALE_E_INVALID_ARGUMENT, "decoder: %s must be f32, f16 or bf16", what);
    if (m.rows != rows || m.cols != cols || !m.data)
        return fail(ctx, HALE_E_INVALID_ARGUMENT, "decoder: %s is %ux%u, expected %ux%u", what, m.rows, m.cols, rows,
                    cols);
    if (lanes_ok((hale_dtype)m.dtype, cols)) return matrix_create_lanes(ctx, (hale_dtype)m.dtype, rows, cols, m.data, out);
    const int64_t rb = hale_row_bytes((hale_dtype)m.dtype, cols);
    return hale_matrix_create(ctx, (hale_dtype)m.dtype, rows, cols, m.data, (uint64_t)rows * rb, 0, out);
}

extern "C" hale_status hale_decoder_create_batched(hale_ctx* ctx, const hale_decoder_desc* ds,
                                                   const hale_decoder_layer* lys, hale_pool* pool, uint32_t max_len,
                                                   uint32_t n_seqs, uint32_t max_batch, hale_decoder** out) {
    if (!ctx || !ds || !lys || !out) return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_decoder_create: NULL argument");
    *out = nullptr;
    if (n_seqs == 0 || max_batch == 0 || max_batch > 4096)
        return fail(ctx, HALE_E_INVALID_ARGUMENT, "decoder: need 1 or more sequences and 1..4096 rows per step (got %u, %u)",
                    n_seqs, max_batch);
    const uint32_t H = ds->hidden, nh = ds->n_heads, nkv = ds->n_kv_heads, hd = ds->head_dim;
    if (!H || !ds->n_layers || !nh || !nkv || !hd || !ds->vocab || !max_len || nh % nkv || hd % 4 || hd > 1024)
        return fail(ctx, HALE_E_INVALID_ARGUMENT,
                    "decoder: bad shape (hidden %u, layers %u, heads %u/%u, head_dim %u, vocab %u, max_len %u)", H,
                    ds->n_layers, nh, nkv, hd, ds->vocab, max_len);
    if (!ds->final_norm) return fail(ctx, HALE_E_INVALID_ARGUMENT, "decoder: final_norm is NULL");
    CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    hale_decoder* d = new hale_decoder();
    d->ctx = ctx;
    d->device = ctx->device;
    ctx->decoders.insert(d);
    d->pool = pool;
    // a tiered pool resolves each MoE layer's routes on the host mid-step
    d->no_graph = pool && pool->tiered;
    d->H = H;
    d->L = ds->n_layers;
    d->nh = nh;
    d->nkv = nkv;
    d->hd = hd;
    d->V = ds->vocab;
    d->E = ds->n_experts;
    d->k = ds->top_k;
    d->normalize = ds->normalize_topk;
    d->eps = ds->eps;
    d->max_len = max_len;
    d->n_seqs = n_seqs;
    d->max_batch = max_batch;
    d->scale = 1.0f / sqrtf((float)hd);  // attention.rs: 1 / sqrt(head_dim)
    hale_status r = HALE_OK;
    auto bail = [&](hale_status st) {
        hale_decoder_destroy(d);
        return st;
    };
    const uint32_t kvd = nkv * hd, qkv_rows = (nh + 2 * nkv) * hd;
    uint32_t moe_layers = 0, max_inter = 1;
    d->layers.resize(d->L);
    for (uint32_t l = 0; l < d->L; l++) {
        const hale_decoder_layer& s = lys[l];
        auto& ly = d->layers[l];
        if (!s.input_norm || !s.post_norm) return bail(fail(ctx, HALE_E_INVALID_ARGUMENT, "layer %u: norm is NULL", l));
        // q, k, v rows of one dtype go into one fused projection (rows are independent dots)
        if (s.q.dtype != s.k.dtype || s.q.dtype != s.v.dtype)
            return bail(fail(ctx, HALE_E_INVALID_ARGUMENT, "layer %u: q/k/v dtypes differ", l));
        if (s.q.rows != nh * hd || s.k.rows != kvd || s.v.rows != kvd || s.q.cols != H || s.k.cols != H ||
            s.v.cols != H || !s.q.data || !s.k.data || !s.v.data)
            return bail(fail(ctx, HALE_E_INVALID_ARGUMENT, "layer %u: q/k/v shapes", l));
        if (!is_float((hale_dtype)s.q.dtype))
            return bail(fail(ctx, HALE_E_INVALID_ARGUMENT, "layer %u: q/k/v must be float", l));
        const size_t rb = (size_t)hale_row_bytes((hale_dtype)s.q.dtype, H);
        std::vector<uint8_t> cat((size_t)qkv_rows * rb);
        std::memcpy(cat.data(), s.q.data, (size_t)nh * hd * rb);
        std::memcpy(cat.data() + (size_t)nh * hd * rb, s.k.data, (size_t)kvd * rb);
        std::memcpy(cat.data() + (size_t)(nh + nkv) * hd * rb, s.v.data, (size_t)kvd * rb);
        r = lanes_ok((hale_dtype)s.q.dtype, H)
                ? matrix_create_lanes(ctx, (hale_dtype)s.q.dtype, qkv_rows, H, cat.data(), &ly.qkv)
                : hale_matrix_create(ctx, (hale_dtype)s.q.dtype, qkv_rows, H, cat.data(), cat.size(), 0, &ly.qkv);
        if (r) return bail(r);
        if ((r = dec_matrix(ctx, s.o, H, nh * hd, "o_proj", &ly.o))) return bail(r);
        if ((r = dec_upload(ctx, d, s.input_norm, H * 4, reinterpret_cast<void**>(&ly.in_norm)))) return bail(r);
        if ((r = dec_upload(ctx, d, s.post_norm, H * 4, reinterpret_cast<void**>(&ly.post_norm)))) return bail(r);
        if (s.q_norm && (r = dec_upload(ctx, d, s.q_norm, hd * 4, reinterpret_cast<void**>(&ly.q_norm)))) return bail(r);
        if (s.k_norm && (r = dec_upload(ctx, d, s.k_norm, hd * 4, reinterpret_cast<void**>(&ly.k_norm)))) return bail(r);
        ly.is_moe = s.is_moe ? 1 : 0;
        if (ly.is_moe) {
            // all E experts, or one rank's share of them (E / R, for hale_decoder_set_comm)
            if (!pool || pool->ctx != ctx || pool->H != H || !pool->E || d->E % pool->E || moe_layers >= pool->L)
                return bail(fail(ctx, HALE_E_INVALID_ARGUMENT, "layer %u: the expert pool does not hold MoE layer %u "
                                 "(%u experts of hidden %u)", l, moe_layers, d->E, H));
            if (!is_float((hale_dtype)s.router.dtype) || s.router.rows != d->E || s.router.cols != H || !s.router.data)
                return bail(fail(ctx, HALE_E_INVALID_ARGUMENT, "layer %u: router must be float [%u, %u]", l, d->E, H));
            ly.router_dtype = (hale_dtype)s.router.dtype;
            if ((r = dec_upload(ctx, d, s.router.data, (size_t)d->E * hale_row_bytes(ly.router_dtype, H), &ly.router)))
                return bail(r);
            ly.pool_layer = moe_layers++;
        } else {
            const uint32_t I = s.dense_gate.rows;
            if ((r = dec_matrix(ctx, s.dense_gate, I, H, "dense gate", &ly.gate))) return bail(r);
            if ((r = dec_matrix(ctx, s.dense_up, I, H, "dense up", &ly.up))) return bail(r);
            if ((r = dec_matrix(ctx, s.dense_down, H, I, "dense down", &ly.down))) return bail(r);
            ly.inter = I;
            max_inter = std::max(max_inter, I);
        }
    }
    const hale_dtype edt = (hale_dtype)ds->embed.dtype;
    if (!is_float(edt) || ds->embed.rows != d->V || ds->embed.cols != H || !ds->embed.data)
        return bail(fail(ctx, HALE_E_INVALID_ARGUMENT, "decoder: embedding must be float [%u, %u]", d->V, H));
    d->embed_dtype = edt;
    if ((r = dec_upload(ctx, d, ds->embed.data, (size_t)d->V * hale_row_bytes(edt, H), &d->embed))) return bail(r);
    if ((r = dec_matrix(ctx, ds->lm_head, d->V, H, "lm_head", &d->lm_head))) return bail(r);
    if ((r = dec_upload(ctx, d, ds->final_norm, H * 4, reinterpret_cast<void**>(&d->final_norm)))) return bail(r);
    // RoPE tables with the host libm (rope.rs:15-30): inv_freq_i = 1 / theta^(2i / hd),
    // angle = position * inv_freq_i
    const uint32_t half = hd / 2;
    std::vector<float> inv(half), cs((size_t)max_len * half), sn((size_t)max_len * half);
    for (uint32_t i = 0; i < half; i++) inv[i] = 1.0f / powf(ds->rope_theta, (float)(2 * i) / (float)hd);
    for (uint32_t p = 0; p < max_len; p++)
        for (uint32_t i = 0; i < half; i++) {
            const float angle = (float)p * inv[i];
            cs[(size_t)p * half + i] = cosf(angle);
            sn[(size_t)p * half + i] = sinf(angle);
        }
    if ((r = dec_upload(ctx, d, cs.data(), cs.size() * 4, reinterpret_cast<void**>(&d->rope_cos)))) return bail(r);
    if ((r = dec_upload(ctx, d, sn.data(), sn.size() * 4, reinterpret_cast<void**>(&d->rope_sin)))) return bail(r);
    // KV cache: [layer][sequence][position][kv heads * head_dim] f32
    d->seq_stride = (size_t)max_len * kvd;
    const size_t cache = (size_t)d->L * n_seqs * d->seq_stride * 4;
    if ((r = dec_alloc(ctx, d, cache, reinterpret_cast<void**>(&d->kcache)))) return bail(r);
    if ((r = dec_alloc(ctx, d, cache, reinterpret_cast<void**>(&d->vcache)))) return bail(r);
    // attention keeps q and up to 8192 scores in shared memory (below 48 KB);
    // longer contexts keep scores in a [rows][heads][max_len] scratch
    d->smem_scores = std::min<uint32_t>(max_len, 8192u);
    d->attn_smem = ((size_t)hd + ((d->smem_scores + 3) & ~3u) + (size_t)kAttnStages * attn_v_rows((int)hd) * hd) * 4;
    // attn_decode_kernel serves head_dim > 256 only (attn_gqa_kernel the rest)
    if (allow_smem(rmsnorm_kernel, (size_t)H * 12) != cudaSuccess ||
        allow_smem(attn_decode_kernel<4>, d->attn_smem) != cudaSuccess)
        return bail(fail(ctx, HALE_E_CUDA, "decoder: attention needs %zu bytes of shared memory", d->attn_smem));
    const size_t B = max_batch;
    // GQA-grouped attention: one CTA per head at one row (most CTAs for a
    // single token), the whole group (up to 8 heads) in batched steps (each
    // K/V element read once per group)
    d->gqa = hd <= 256 && hd % 4 == 0;
    uint32_t min_cap = d->smem_scores;
    if (d->gqa) {
        const uint32_t G = nh / nkv;
        int gmax = 1;
        for (int g : {8, 4, 2})
            if (G % g == 0) { gmax = g; break; }
        d->gc_batch = gmax;
        d->gc_one = 0;  // 0: chosen per step from the row count
        // group sizes whose shared-memory plan fits (wide heads may fit none:
        // then attn_decode_kernel serves every step)
        int fit = 0;
        for (int gc : {1, 2, 4, 8}) {
            if (G % gc != 0 || gc > gmax) continue;
            const int cap = (int)std::min<uint32_t>((uint32_t)gqa_score_cap(gc), (max_len + 3) & ~3u);
            const size_t sm = gqa_smem_floats(gc, cap, (int)hd) * 4;
            if (sm > kMaxDynSmem) break;
            cudaError_t e = gc == 1 ? allow_smem(attn_gqa_kernel<1>, sm)
                          : gc == 2 ? allow_smem(attn_gqa_kernel<2>, sm)
                          : gc == 4 ? allow_smem(attn_gqa_kernel<4>, sm)
                                    : allow_smem(attn_gqa_kernel<8>, sm);
            if (e != cudaSuccess)
                return bail(fail(ctx, HALE_E_CUDA, "decoder: attention needs %zu bytes of shared memory", sm));
            d->gqa_cap[gc] = cap;
            d->gqa_smem[gc] = sm;
            min_cap = std::min<uint32_t>(min_cap, (uint32_t)cap);
            fit = gc;
        }
        if (fit == 0) d->gqa = false;
        d->gc_batch = std::min(d->gc_batch, std::max(fit, 1));
    }
    // one-row steps: attention spread over the GPU when the group fits its
    // shared-memory plan (up to 32 query heads per kv head, head_dim % 8 == 0)
    if (nh % nkv == 0 && nh / nkv <= 32 && hd % kSplitD == 0 &&
        (size_t)split_plan((int)(nh / nkv), (int)hd).total * 4 <= kMaxDynSmem) {
        const int G = (int)(nh / nkv);
        d->split_smem = (size_t)split_plan(G, (int)hd).total * 4;
        int occ = 0;
        if (allow_smem(attn_split_kernel, d->split_smem) == cudaSuccess &&
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, attn_split_kernel, 256, d->split_smem) ==
                cudaSuccess &&
            occ > 0) {
            d->split_npm = (int)((max_len + kSplitPB - 1) / kSplitPB);
            const int units = std::max((int)nkv * d->split_npm, (int)(nkv * hd / kSplitD));
            d->split_grid = std::min(ctx->sm_count * occ, units);
            d->split = true;
            if ((r = dec_alloc(ctx, d, (size_t)nh * ((max_len + 3) & ~3u) * 4, reinterpret_cast<void**>(&d->split_sc))) ||
                (r = dec_alloc(ctx, d, (size_t)nh * d->split_npm * 4, reinterpret_cast<void**>(&d->split_pm))) ||
                (r = dec_alloc(ctx, d, 16, reinterpret_cast<void**>(&d->split_bar))))
                return bail(r);
        } else {
            cudaGetLastError();
        }
    }
    const size_t score_floats = max_len > min_cap ? B * nh * max_len : 4;
    struct { float** p; size_t n; } bufs[] = {{&d->x, B * H}, {&d->x2, B * H}, {&d->moe_out, B * H},
                                               {&d->normed, B * H}, {&d->delta, B * H},
                                               {&d->qkv, B * qkv_rows}, {&d->attn, B * nh * hd},
                                               {&d->g, B * max_inter}, {&d->u, B * max_inter},
                                               {&d->h, B * max_inter}, {&d->scores, score_floats}};
    for (auto& b : bufs)
        if ((r = dec_alloc(ctx, d, b.n * 4, reinterpret_cast<void**>(b.p)))) return bail(r);
    if ((r = dec_alloc(ctx, d, B * 12, reinterpret_cast<void**>(&d->d_rows)))) return bail(r);
    if (H > 12000) return bail(fail(ctx, HALE_E_INVALID_ARGUMENT, "decoder: hidden %u above 12000", H));
    if (cudaHostAlloc(reinterpret_cast<void**>(&d->h_rows), B * 12, cudaHostAllocDefault) != cudaSuccess ||
        cudaEventCreateWithFlags(&d->ev_copied, cudaEventDisableTiming) != cudaSuccess ||
        cudaStreamCreateWithFlags(&d->cap, cudaStreamNonBlocking) != cudaSuccess)
        return bail(fail(ctx, HALE_E_CUDA, "decoder: cannot create its step resources"));
    *out = d;
    return HALE_OK;
}

// L2 prefetch descriptor of up to two device ranges (a range that is not
// 16-byte aligned is skipped; lengths round down to 16 bytes).
static L2Prefetch l2_ranges(const void* a, size_t an, const void* b, size_t bn) {
    L2Prefetch pf{};
    if (a && aligned16(a)) { pf.p[0] = static_cast<const uint8_t*>(a); pf.bytes[0] = an & ~(size_t)15; }
    if (b && aligned16(b)) { pf.p[1] = static_cast<const uint8_t*>(b); pf.bytes[1] = bn & ~(size_t)15; }
    return pf;
}
// CTAs an RMSNorm launch adds for the L2 prefetch.
static constexpr uint32_t kNormPrefetchCtas = 32;

// One step of n rows on stream st: the row descriptors' copy from the pinned
// slot, then every kernel of the step. logits: [n, V], or [1, V] for the last
// row only when last_logits.
static hale_status decoder_enqueue(hale_ctx* ctx, hale_decoder* d, uint32_t n, float* logits, bool last_logits,
                                   float* hidden, cudaStream_t st) {
    void* stream = st;
    CUDA_TRY(ctx, cudaMemcpyAsync(d->d_rows, d->h_rows, (size_t)n * 12, cudaMemcpyHostToDevice, st));
    hale_status r;
    const int H = (int)d->H, hb = (H + 255) / 256;
    const size_t lstride = (size_t)d->n_seqs * d->seq_stride;
    const dim3 eg(hb, n);
    {
    ProfScope ps_(ctx, "embed", st);
    switch (d->embed_dtype) {
    case HALE_F32: embed_kernel<0><<<eg, 256, 0, st>>>(d->embed, H, d->d_rows, d->x); break;
    case HALE_F16: embed_kernel<1><<<eg, 256, 0, st>>>(d->embed, H, d->d_rows, d->x); break;
    default: embed_kernel<2><<<eg, 256, 0, st>>>(d->embed, H, d->d_rows, d->x); break;
    }
    }
    if ((r = check_launch(ctx, "embed"))) return r;
    // the residual stream: norms folded into their consumer read xr and write
    // xr + delta to the other buffer (other CTAs of the launch still read xr)
    float* xr = d->x;
    float* xo = d->x2;
    // the layer output buffer (dl) and its spare: a fused norm + MoE layer
    // reads dl and writes dspare, which then becomes dl
    float* dl = d->delta;
    float* dspare = d->moe_out;
    for (uint32_t l = 0; l < d->L; l++) {
        const auto& ly = d->layers[l];
        float* kc = d->kcache + (size_t)l * lstride;
        float* vc = d->vcache + (size_t)l * lstride;
        // the previous layer's FFN residual folds into this norm; one row: the
        // norm runs inside the q/k/v matvec
        bool fused = false;
        if (n == 1 && (r = fgemv_norm_launch(ctx, ly.qkv, xr, l ? dl : nullptr, ly.in_norm, d->eps,
                                             l ? xo : nullptr, d->qkv, st, &fused)))
            return r;
        if (fused) {
            if (l) std::swap(xr, xo);
        } else {
            {
                // spare CTAs pull this layer's attention weights into L2
                ProfScope ps_(ctx, "rmsnorm", st);
                const L2Prefetch pf = l2_ranges(ly.qkv->data, ly.qkv->bytes, ly.o->data, ly.o->bytes);
                rmsnorm_kernel<<<n + kNormPrefetchCtas, 256, (size_t)H * 12, st>>>(
                    xr, l ? dl : nullptr, ly.in_norm, d->eps, H, d->normed, (int)n, pf);
            }
            if ((r = check_launch(ctx, "rmsnorm"))) return r;
            if ((r = hale_matrix_matvec(ctx, ly.qkv, d->normed, n, d->qkv, nullptr, stream))) return r;
        }
        // one row: attn_split_kernel does this itself
        if (!(n == 1 && d->split)) {
            {
                ProfScope ps_(ctx, "qk_rope", st);
                qk_rope_kernel<<<dim3(d->nh + 2 * d->nkv, n), 32, (size_t)d->hd * 4, st>>>(
                    d->qkv, (int)d->nh, (int)d->nkv, (int)d->hd, ly.q_norm, ly.k_norm, d->eps, d->rope_cos,
                    d->rope_sin, d->d_rows, kc, vc, d->seq_stride);
            }
            if ((r = check_launch(ctx, "qk_rope"))) return r;
        }
        {
            ProfScope ps_(ctx, "attention", st);
            if (n == 1 && d->split) {
                SplitArgs sa{};
                sa.qkv = d->qkv;
                sa.nh = (int)d->nh;
                sa.nkv = (int)d->nkv;
                sa.hd = (int)d->hd;
                sa.kcache = kc;
                sa.vcache = vc;
                sa.rows = d->d_rows;
                sa.seq_stride = d->seq_stride;
                sa.scale = d->scale;
                sa.sc = d->split_sc;
                sa.pm = d->split_pm;
                sa.sc_stride = (int)((d->max_len + 3) & ~3u);
                sa.npm = d->split_npm;
                sa.ctx = d->attn;
                sa.bar = d->split_bar;
                sa.pf = l2_ranges(ly.o->data, ly.o->bytes, nullptr, 0);
                sa.rope = 1;
                sa.q_norm = ly.q_norm;
                sa.k_norm = ly.k_norm;
                sa.eps = d->eps;
                sa.rope_cos = d->rope_cos;
                sa.rope_sin = d->rope_sin;
                sa.err = ctx->d_err;
                attn_split_kernel<<<d->split_grid, 256, d->split_smem, st>>>(sa);
            } else if (d->gqa) {
                // the most heads per CTA (each K/V element read once per group)
                // that still gives about two thirds of the SMs a CTA
                int gc = d->gc_one;
                if (gc == 0) {
                    gc = 1;
                    for (int g = d->gc_batch; g > 1; g /= 2)
                        if ((d->nh / d->nkv) % g == 0 && (size_t)n * d->nh / g >= 96) { gc = g; break; }
                }
                const dim3 grid(d->nh / gc, n);
                const size_t sm = d->gqa_smem[gc];
                const int cap = d->gqa_cap[gc], vt = gqa_v_rows((int)d->hd);
#define HALE_GQA(GCV)                                                                                               \
    attn_gqa_kernel<GCV><<<grid, 256, sm, st>>>(d->qkv, (int)d->nh, (int)d->nkv, (int)d->hd, kc, vc, d->d_rows,   \
                                                (int)d->max_len, d->scale, d->scores, d->attn, cap, d->seq_stride, vt)
                if (gc == 1) HALE_GQA(1);
                else if (gc == 2) HALE_GQA(2);
                else if (gc == 4) HALE_GQA(4);
                else HALE_GQA(8);
#undef HALE_GQA
            } else {
                attn_decode_kernel<4><<<dim3(d->nh, n), 256, d->attn_smem, st>>>(
                    d->qkv, (int)d->nh, (int)d->nkv, (int)d->hd, kc, vc, d->d_rows, (int)d->max_len, d->scale,
                    d->scores, d->attn, (int)d->smem_scores, d->seq_stride, attn_v_rows((int)d->hd));
            }
        }
        if ((r = check_launch(ctx, "attn_decode"))) return r;
        if ((r = hale_matrix_matvec(ctx, ly.o, d->attn, n, dl, nullptr, stream))) return r;
        hale_moe_layer m{};
        if (ly.is_moe) {
            m.layer = ly.pool_layer;
            m.router = ly.router;
            m.router_dtype = ly.router_dtype;
            m.n_experts = d->E;
            m.top_k = d->k;
            m.normalize_topk = d->normalize;
        }
        // one row through a resident pool: the post-attention norm runs inside
        // the one-launch MoE layer (its output, the layer's delta, replaces
        // the attention delta it read)
        fused = false;
        if (ly.is_moe && n == 1 && !d->comm && !d->pool->tiered) {
            const TokNorm tn{dl, ly.post_norm, d->eps, xo};
            if ((r = moe_token_norm(ctx, d->pool, &m, xr, tn, dspare, st, &fused))) return r;
            if (fused) {
                std::swap(xr, xo);
                std::swap(dl, dspare);
                continue;
            }
        }
        {
            ProfScope ps_(ctx, "rmsnorm", st);
            // spare CTAs: the router (MoE) or the dense FFN's gate and up rows
            const L2Prefetch pf =
                ly.is_moe ? l2_ranges(ly.router, (size_t)d->E * H * (ly.router_dtype == HALE_F32 ? 4 : 2), nullptr, 0)
                          : l2_ranges(ly.gate->data, ly.gate->bytes, ly.up->data, ly.up->bytes);
            rmsnorm_kernel<<<n + kNormPrefetchCtas, 256, (size_t)H * 12, st>>>(xr, dl, ly.post_norm, d->eps,
                                                                              H, d->normed, (int)n, pf);
        }
        if ((r = check_launch(ctx, "rmsnorm"))) return r;
        if (ly.is_moe) {
            if (d->comm)
                r = hale_moe_forward_ep(ctx, d->comm, d->pool, &m, d->normed, n, dl, nullptr, nullptr, stream);
            else
                r = hale_moe_forward(ctx, d->pool, &m, d->normed, n, dl, nullptr, nullptr, stream);
            if (r) return r;
        } else {
            if ((r = hale_matrix_matvec(ctx, ly.gate, d->normed, n, d->g, nullptr, stream))) return r;
            if ((r = hale_matrix_matvec(ctx, ly.up, d->normed, n, d->u, nullptr, stream))) return r;
            const int cnt = (int)(n * ly.inter);
            silu_mul_kernel<<<(cnt + 255) / 256, 256, 0, st>>>(d->g, d->u, cnt, d->h);
            if ((r = check_launch(ctx, "silu_mul"))) return r;
            if ((r = hale_matrix_matvec(ctx, ly.down, d->h, n, dl, nullptr, stream))) return r;
        }
    }
    {
        ProfScope ps_(ctx, "rmsnorm", st);
        rmsnorm_kernel<<<n, 256, (size_t)H * 12, st>>>(xr, dl, d->final_norm, d->eps, H, d->normed, (int)n,
                                                     l2_ranges(nullptr, 0, nullptr, 0));
    }
    if ((r = check_launch(ctx, "rmsnorm"))) return r;
    if (hidden) CUDA_TRY(ctx, cudaMemcpyAsync(hidden, d->normed, (size_t)n * H * 4, cudaMemcpyDeviceToDevice, st));
    if (logits) {
        ProfScope ps_(ctx, "lm_head", st);
        if (last_logits) return hale_matrix_matvec(ctx, d->lm_head, d->normed + (size_t)(n - 1) * H, 1, logits, nullptr, stream);
        return hale_matrix_matvec(ctx, d->lm_head, d->normed, n, logits, nullptr, stream);
    }
    return HALE_OK;
}

extern "C" hale_status hale_decoder_create(hale_ctx* ctx, const hale_decoder_desc* ds, const hale_decoder_layer* lys,
                                           hale_pool* pool, uint32_t max_len, hale_decoder** out) {
    return hale_decoder_create_batched(ctx, ds, lys, pool, max_len, 1, 1, out);
}

extern "C" hale_status hale_decoder_forward(hale_ctx* ctx, hale_decoder* d, uint32_t token, uint32_t position,
                                            float* logits, float* hidden, void* stream) {
    if (!ctx || !d || d->ctx != ctx) return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_decoder_forward: bad handle");
    if (token >= d->V) return fail(ctx, HALE_E_INVALID_ARGUMENT, "token %u out of vocabulary (%u)", token, d->V);
    if (position >= d->max_len)
        return fail(ctx, HALE_E_CONTEXT_OVERFLOW, "position %u exceeds the KV cache (%u positions)", position,
                    d->max_len);
    CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    cudaStream_t st = S(stream);
    // the previous step must have read the slot before it is rewritten
    if (d->copied_recorded) CUDA_TRY(ctx, cudaEventSynchronize(d->ev_copied));
    d->h_rows[0] = token;
    d->h_rows[1] = position;
    d->h_rows[2] = 0;
    const bool capturing = stream_capturing(stream);
    d->copied_recorded = !capturing;
    // per-kernel profiling (hale_ctx_profile) times eager launches only
    if (d->exec && d->g_logits == logits && d->g_hidden == hidden && d->g_gen == ctx->ws_gen && !capturing &&
        !ctx->profiling) {
        CUDA_TRY(ctx, cudaGraphLaunch(d->exec, st));
        CUDA_TRY(ctx, cudaEventRecord(d->ev_copied, st));
        return HALE_OK;
    }
    hale_status r = decoder_enqueue(ctx, d, 1, logits, false, hidden, st);
    if (!r && !capturing) CUDA_TRY(ctx, cudaEventRecord(d->ev_copied, st));
    if (r || capturing || d->no_graph || ctx->profiling) return r;
    // capture the step for the following calls with these outputs
    if (d->exec) {
        cudaGraphExecDestroy(d->exec);
        d->exec = nullptr;
    }
    cudaGraph_t graph = nullptr;
    if (cudaStreamBeginCapture(d->cap, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        cudaGetLastError();
        d->no_graph = true;
        return HALE_OK;
    }
    r = decoder_enqueue(ctx, d, 1, logits, false, hidden, d->cap);
    const cudaError_t ec = cudaStreamEndCapture(d->cap, &graph);
    if (r || ec != cudaSuccess || !graph || cudaGraphInstantiate(&d->exec, graph, 0) != cudaSuccess) {
        cudaGetLastError();
        d->exec = nullptr;
        d->no_graph = true;  // keep launching step by step
        g_thread_status = HALE_OK;
    }
    if (graph) cudaGraphDestroy(graph);
    d->g_logits = logits;
    d->g_hidden = hidden;
    d->g_gen = ctx->ws_gen;
    return HALE_OK;
}

extern "C" hale_status hale_decoder_step(hale_ctx* ctx, hale_decoder* d, const uint32_t* tokens,
                                         const uint32_t* positions, const uint32_t* seqs, uint32_t n, float* logits,
                                         int32_t last_logits_only, float* hidden, void* stream) {
    if (!ctx || !d || d->ctx != ctx) return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_decoder_step: bad handle");
    if (n == 0) {
        // an expert-parallel rank with no rows still takes part in every
        // layer's exchange (the other ranks' tokens may route to its experts)
        if (!d->comm) return HALE_OK;
        CUDA_TRY(ctx, cudaSetDevice(d->device));
        for (const auto& ly : d->layers) {
            if (!ly.is_moe) continue;
            hale_moe_layer m{};
            m.layer = ly.pool_layer;
            m.router = ly.router;
            m.router_dtype = ly.router_dtype;
            m.n_experts = d->E;
            m.top_k = d->k;
            m.normalize_topk = d->normalize;
            hale_status r = hale_moe_forward_ep(ctx, d->comm, d->pool, &m, nullptr, 0, nullptr, nullptr, nullptr, stream);
            if (r) return r;
        }
        return HALE_OK;
    }
    if (!tokens || !positions) return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_decoder_step: NULL tokens or positions");
    if (n > d->max_batch)
        return fail(ctx, HALE_E_INVALID_ARGUMENT, "step of %u rows exceeds the decoder's %u", n, d->max_batch);
    for (uint32_t i = 0; i < n; i++) {
        const uint32_t sq = seqs ? seqs[i] : 0;
        if (tokens[i] >= d->V) return fail(ctx, HALE_E_INVALID_ARGUMENT, "token %u out of vocabulary (%u)", tokens[i], d->V);
        if (sq >= d->n_seqs) return fail(ctx, HALE_E_INVALID_ARGUMENT, "sequence %u out of range (%u)", sq, d->n_seqs);
        if (positions[i] >= d->max_len)
            return fail(ctx, HALE_E_CONTEXT_OVERFLOW, "position %u exceeds the KV cache (%u positions)", positions[i],
                        d->max_len);
    }
    {
        // a (sequence, position) slot is written by at most one row of a step
        std::vector<uint64_t> keys(n);
        for (uint32_t i = 0; i < n; i++) keys[i] = ((uint64_t)(seqs ? seqs[i] : 0) << 32) | positions[i];
        std::sort(keys.begin(), keys.end());
        for (uint32_t i = 1; i < n; i++)
            if (keys[i] == keys[i - 1])
                return fail(ctx, HALE_E_INVALID_ARGUMENT, "two rows write sequence %u position %u",
                            (unsigned)(keys[i] >> 32), (unsigned)(keys[i] & 0xffffffffu));
    }
    if (stream_capturing(stream))
        return fail(ctx, HALE_E_UNSUPPORTED, "hale_decoder_step is not captured; hale_decoder_forward replays a graph");
    CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    cudaStream_t st = S(stream);
    if (d->copied_recorded) CUDA_TRY(ctx, cudaEventSynchronize(d->ev_copied));
    for (uint32_t i = 0; i < n; i++) {
        d->h_rows[3 * i] = tokens[i];
        d->h_rows[3 * i + 1] = positions[i];
        d->h_rows[3 * i + 2] = seqs ? seqs[i] : 0;
    }
    hale_status r = decoder_enqueue(ctx, d, n, logits, last_logits_only != 0, hidden, st);
    if (!r) {
        CUDA_TRY(ctx, cudaEventRecord(d->ev_copied, st));
        d->copied_recorded = true;
    }
    return r;
}

extern "C" hale_status hale_lm_head(hale_ctx* ctx, const hale_matrix* lm_head, const float* hidden, uint32_t batch,
                                    float* logits, void* stream) {
    if (!ctx || !lm_head) return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_lm_head: NULL argument");
    if (!is_float(lm_head->dtype)) return fail(ctx, HALE_E_INVALID_ARGUMENT, "lm_head must be f32, f16 or bf16");
    return hale_matrix_matvec(ctx, lm_head, hidden, batch, logits, nullptr, stream);
}

// More than kSampleMaxK candidates: every row's candidates ranked by unique
// 64-bit keys (logit total order, then index), sorted by CUB's segmented
// radix sort (compiled from the toolkit's headers), then the reference's
// exact sums over the sorted order (sample_exp_kernel, sample_tail_kernel).
// Scratch: two key buffers, exp and probability rows, segment offsets and
// the sort's temporary storage.
static hale_status sample_full(hale_ctx* ctx, const SampleArgs& a, uint32_t batch, size_t bitmap_smem,
                               cudaStream_t st) {
    const size_t n = (size_t)batch * a.V;
    if (n > (size_t)INT32_MAX) return fail(ctx, HALE_E_UNSUPPORTED, "batch x vocab above 2^31 candidates");
    size_t temp = 0;
    CUDA_TRY(ctx, cub::DeviceSegmentedRadixSort::SortKeysDescending(
                      nullptr, temp, (const unsigned long long*)nullptr, (unsigned long long*)nullptr, (int)n,
                      (int)batch, (const int*)nullptr, (const int*)nullptr, 0, 64, st));
    const size_t o_keys2 = align_up(n * 8, 256), o_e = o_keys2 + align_up(n * 8, 256);
    const size_t o_q = o_e + align_up(n * 4, 256), o_off = o_q + align_up(n * 4, 256);
    const size_t o_tmp = o_off + align_up(((size_t)batch + 1) * 4, 256), total = o_tmp + temp;
    hale_status r = ensure_scratch(ctx, total, st);
    if (r) return r;
    uint8_t* sc = static_cast<uint8_t*>(ctx->scratch);
    auto* keys = reinterpret_cast<unsigned long long*>(sc);
    auto* sorted = reinterpret_cast<unsigned long long*>(sc + o_keys2);
    float* e = reinterpret_cast<float*>(sc + o_e);
    float* q = reinterpret_cast<float*>(sc + o_q);
    int* off = reinterpret_cast<int*>(sc + o_off);
    if (bitmap_smem > 48 * 1024)
        CUDA_TRY(ctx, cudaFuncSetAttribute(sample_keys_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)bitmap_smem));
    ProfScope ps_(ctx, "sample", st);
    sample_keys_kernel<<<batch, 1024, bitmap_smem, st>>>(a, keys, off);
    if ((r = check_launch(ctx, "sample_keys"))) return r;
    CUDA_TRY(ctx, cub::DeviceSegmentedRadixSort::SortKeysDescending(sc + o_tmp, temp, keys, sorted, (int)n,
                                                                    (int)batch, off, off + 1, 0, 64, st));
    sample_exp_kernel<<<dim3((unsigned)((a.top_k + 255) / 256), batch), 256, 0, st>>>(sorted, a.V, a.top_k,
                                                                                      a.temperature, e);
    if ((r = check_launch(ctx, "sample_exp"))) return r;
    sample_tail_kernel<<<batch, 1024, 0, st>>>(sorted, e, q, a.V, a.top_k, a.top_p, a.rng, a.out);
    return check_launch(ctx, "sample_tail");
}

extern "C" hale_status hale_sample(hale_ctx* ctx, const float* logits, uint32_t batch, uint32_t vocab,
                                   const hale_sampling_params* prm, uint64_t* rng_state, const int32_t* seen_ids,
                                   uint32_t n_seen, int32_t* out_tokens, void* stream) {
    if (!ctx || !prm) return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_sample: NULL argument");
    if (batch == 0) return HALE_OK;
    if (!logits || !out_tokens) return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_sample: NULL buffer");
    if (vocab == 0 || vocab > (1u << 30)) return fail(ctx, HALE_E_INVALID_ARGUMENT, "vocab %u out of range", vocab);
    float pen = prm->repetition_penalty;
    if (!(pen > 0.0f)) return fail(ctx, HALE_E_INVALID_ARGUMENT, "repetition_penalty must be > 0");
    int K = (int)vocab;
    if (prm->temperature > 0.0f) {
        if (!rng_state) return fail(ctx, HALE_E_INVALID_ARGUMENT, "rng_state is NULL");
        K = prm->top_k == 0 ? (int)vocab : (int)std::min<uint32_t>(prm->top_k, vocab);
    }
    CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    SampleArgs a{};
    a.logits = logits;
    a.V = (int)vocab;
    a.temperature = prm->temperature;
    a.top_p = prm->top_p;
    a.penalty = pen;
    a.top_k = K;
    a.rng = rng_state;
    a.seen = seen_ids;
    a.n_seen = (int)n_seen;
    a.out = out_tokens;
    size_t smem = (seen_ids && n_seen && pen != 1.0f) ? (size_t)((vocab + 31) / 32) * 4 : 0;
    if (smem > 200 * 1024) return fail(ctx, HALE_E_UNSUPPORTED, "vocab %u too large for the penalty bitmap", vocab);
    if (prm->temperature > 0.0f && K > kSampleMaxK) return sample_full(ctx, a, batch, smem, S(stream));
    if (smem > 48 * 1024) CUDA_TRY(ctx, cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    ProfScope ps_(ctx, "sample", S(stream));
    sample_kernel<<<batch, kSampleThreads, smem, S(stream)>>>(a);
    return check_launch(ctx, "sample");
}

// ---------------------------------------------------------------------------
// allocation-free routing (hale_moe_route_noalloc)
//
// For hosts that cannot call cudaMalloc on the routing path (graph replay,
// fixed device-memory arenas). The router's scratch lives in a fixed array of
// this file; every GPU that loads the library holds it until exit.
// Layout: [0, 1024) counters -- up to 254 token-tile counters, the grid
// counter and a device error word -- then the [M, E] f32 router logits.
// ---------------------------------------------------------------------------
constexpr size_t kNoAllocScratchBytes = (size_t)1 << 20;
constexpr size_t kNoAllocCounterBytes = 1024;
constexpr uint32_t kNoAllocMaxTiles = 254;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch, looked up once per device with that
// device current (in host code the symbol is only a stand-in, never a device
// address).
static hale_status noalloc_scratch(int device, uint8_t** out) {
    static std::mutex mu;
    static std::map<int, uint8_t*> addr;
    std::lock_guard<std::mutex> lock(mu);
    auto it = addr.find(device);
    if (it != addr.end()) {
        *out = it->second;
        return HALE_OK;
    }
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
        return fail(nullptr, HALE_E_CUDA, "cudaGetSymbolAddress of the routing scratch failed on device %d: %s",
                    device, cudaGetErrorString(e));
    addr[device] = static_cast<uint8_t*>(p);
    *out = static_cast<uint8_t*>(p);
    return HALE_OK;
}


// generate() (src/generate/generator.rs:55-94): the prompt prefilled as
// steps of up to max_batch rows (the last one computing only its last row's
// logits), then Sampler::sample on the device logits and a one-row step per
// token. Each round reads the sampled token back for the stop check, as the
// reference's loop checks it on the host.
extern "C" hale_status hale_decoder_generate(hale_ctx* ctx, hale_decoder* d, const uint32_t* prompt,
                                             uint32_t n_prompt, const hale_sampling_params* params, uint64_t seed,
                                             uint32_t max_new_tokens, const uint32_t* stop_tokens, uint32_t n_stop,
                                             uint32_t* out_tokens, uint32_t* n_out, float* prefill_ms,
                                             float* decode_ms, void* stream) {
    if (!ctx || !d || d->ctx != ctx) return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_decoder_generate: bad handle");
    if (!prompt || n_prompt == 0 || !params || !out_tokens || !n_out || (n_stop && !stop_tokens))
        return fail(ctx, HALE_E_INVALID_ARGUMENT, "hale_decoder_generate: NULL argument or empty prompt");
    *n_out = 0;
    if (d->comm)
        return fail(ctx, HALE_E_UNSUPPORTED,
                    "hale_decoder_generate: an expert-parallel decoder steps in lockstep with its peers; drive it "
                    "with hale_decoder_step");
    const uint64_t needed = (uint64_t)n_prompt + max_new_tokens;
    if (needed > d->max_len)
        return fail(ctx, HALE_E_CONTEXT_OVERFLOW, "prompt + new tokens (%llu) exceed the KV cache (%u positions)",
                    (unsigned long long)needed, d->max_len);
    if (max_new_tokens == 0) return HALE_OK;
    CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    cudaStream_t st = S(stream);
    hale_status r;
    if (!d->gen_logits) {
        if ((r = dec_alloc(ctx, d, (size_t)d->V * 4, reinterpret_cast<void**>(&d->gen_logits))) ||
            (r = dec_alloc(ctx, d, 8, reinterpret_cast<void**>(&d->gen_rng))) ||
            (r = dec_alloc(ctx, d, 4, reinterpret_cast<void**>(&d->gen_tok))) ||
            (r = dec_alloc(ctx, d, (size_t)d->max_len * 4, reinterpret_cast<void**>(&d->gen_seen))))
            return r;
        if (cudaHostAlloc(reinterpret_cast<void**>(&d->h_tok), 4, cudaHostAllocDefault) != cudaSuccess)
            return fail(ctx, HALE_E_OUT_OF_MEMORY, "hale_decoder_generate: cannot allocate a pinned token slot");
        for (cudaEvent_t& e : d->gen_ev) CUDA_TRY(ctx, cudaEventCreate(&e));
    }
    // XorShift64 state seed.max(1) (sampler.rs:131-133); seen ids = the
    // sequence so far (only the repetition penalty reads them)
    const uint64_t s0 = seed > 1 ? seed : 1;
    CUDA_TRY(ctx, cudaMemcpyAsync(d->gen_rng, &s0, 8, cudaMemcpyHostToDevice, st));
    const bool penalty = params->repetition_penalty != 1.0f;
    if (penalty) {
        std::vector<int32_t> ids(prompt, prompt + n_prompt);
        CUDA_TRY(ctx, cudaMemcpyAsync(d->gen_seen, ids.data(), (size_t)n_prompt * 4, cudaMemcpyHostToDevice, st));
        CUDA_TRY(ctx, cudaStreamSynchronize(st));  // ids leaves scope
    }
    CUDA_TRY(ctx, cudaEventRecord(d->gen_ev[0], st));
    std::vector<uint32_t> pos(d->max_batch);
    for (uint32_t b = 0; b < n_prompt; b += d->max_batch) {
        const uint32_t n = std::min(d->max_batch, n_prompt - b);
        for (uint32_t i = 0; i < n; i++) pos[i] = b + i;
        const bool last = b + n == n_prompt;
        if ((r = hale_decoder_step(ctx, d, prompt + b, pos.data(), nullptr, n, last ? d->gen_logits : nullptr, 1,
                                   nullptr, stream)))
            return r;
    }
    CUDA_TRY(ctx, cudaEventRecord(d->gen_ev[1], st));
    uint32_t count = 0;
    for (uint32_t step = 0; step < max_new_tokens; step++) {
        if ((r = hale_sample(ctx, d->gen_logits, 1, d->V, params, d->gen_rng, penalty ? d->gen_seen : nullptr,
                             penalty ? n_prompt + step : 0, d->gen_tok, stream)))
            return r;
        CUDA_TRY(ctx, cudaMemcpyAsync(d->h_tok, d->gen_tok, 4, cudaMemcpyDeviceToHost, st));
        CUDA_TRY(ctx, cudaStreamSynchronize(st));
        const uint32_t tok = (uint32_t)*d->h_tok;
        out_tokens[count++] = tok;
        bool stop = step + 1 == max_new_tokens;
        for (uint32_t i = 0; i < n_stop && !stop; i++) stop = stop_tokens[i] == tok;
        if (stop) break;
        if (penalty)
            CUDA_TRY(ctx, cudaMemcpyAsync(d->gen_seen + n_prompt + step, d->gen_tok, 4, cudaMemcpyDeviceToDevice, st));
        if ((r = hale_decoder_forward(ctx, d, tok, n_prompt + step, d->gen_logits, nullptr, stream))) return r;
    }
    CUDA_TRY(ctx, cudaEventRecord(d->gen_ev[2], st));
    CUDA_TRY(ctx, cudaEventSynchronize(d->gen_ev[2]));
    *n_out = count;
    if (prefill_ms) CUDA_TRY(ctx, cudaEventElapsedTime(prefill_ms, d->gen_ev[0], d->gen_ev[1]));
    if (decode_ms) CUDA_TRY(ctx, cudaEventElapsedTime(decode_ms, d->gen_ev[1], d->gen_ev[2]));
    return HALE_OK;
}

extern "C" hale_status hale_moe_route_noalloc(const void* router, hale_dtype router_dtype, uint32_t n_experts,
                                              uint32_t top_k, int32_t normalize_topk, uint32_t hidden,
                                              const float* x, uint32_t M, int32_t* topk_idx, float* topk_w,
                                              float* probs, void* stream) {
    hale_moe_layer ly{0, router, router_dtype, n_experts, top_k, normalize_topk};
    hale_status r = check_layer(nullptr, &ly, hidden);
    if (r) return r;
    if (M == 0) return HALE_OK;
    if (!x || !topk_idx || !topk_w) return fail(nullptr, HALE_E_INVALID_ARGUMENT, "hale_moe_route_noalloc: NULL buffer");
    const uint32_t tiles = (M + kRouterTT - 1) / kRouterTT;
    const size_t logit_bytes = (size_t)M * n_experts * 4;
    if (tiles > kNoAllocMaxTiles || logit_bytes > kNoAllocScratchBytes - kNoAllocCounterBytes)
        return fail(nullptr, HALE_E_INVALID_ARGUMENT,
                    "hale_moe_route_noalloc: %u tokens x %u experts exceeds the fixed scratch "
                    "(tokens <= %u and tokens * experts <= %zu)",
                    M, n_experts, kNoAllocMaxTiles * kRouterTT,
                    (kNoAllocScratchBytes - kNoAllocCounterBytes) / 4);
    int device = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return fail(nullptr, HALE_E_NO_DEVICE, "no current CUDA device: %s", cudaGetErrorString(e));
    uint8_t* scratch = nullptr;
    if ((r = noalloc_scratch(device, &scratch))) return r;
    cudaStream_t st = S(stream);
    // the counters must start at zero; the previous call may have stopped early
    e = cudaMemsetAsync(scratch, 0, kNoAllocCounterBytes, st);
    if (e != cudaSuccess) return fail(nullptr, HALE_E_CUDA, "clearing the routing scratch failed: %s", cudaGetErrorString(e));
    unsigned* counters = reinterpret_cast<unsigned*>(scratch);
    RouterArgs a{};
    a.w = router;
    a.wdtype = float_code(router_dtype);
    a.E = (int)n_experts;
    a.H = (int)hidden;
    a.M = (int)M;
    a.k = (int)top_k;
    a.normalize = normalize_topk ? 1 : 0;
    a.staged = (hidden % 8 == 0 && aligned16(x) && aligned16(router)) ? 1 : 0;
    a.x = x;
    a.logits = reinterpret_cast<float*>(scratch + kNoAllocCounterBytes);
    a.probs_out = probs;
    a.topk_idx = topk_idx;
    a.topk_w = topk_w;
    a.tile_cnt = counters;
    a.grid_cnt = counters + kNoAllocMaxTiles;
    a.err = counters + kNoAllocMaxTiles + 1;
    dim3 grid(tiles, (n_experts + kRouterET - 1) / kRouterET);
    const int nslots = std::min<int>(((int)hidden + kRouterCH - 1) / kRouterCH, kRouterSlots);
    size_t smem = a.staged ? (size_t)nslots * router_slot_bytes(a.wdtype == 0 ? 4 : 2) + 8 * nslots : 0;
    auto* kern = a.wdtype == 0 ? router_kernel<0> : (a.wdtype == 1 ? router_kernel<1> : router_kernel<2>);
    e = allow_smem(kern, smem);
    if (e != cudaSuccess) return fail(nullptr, HALE_E_CUDA, "router shared-memory opt-in failed: %s", cudaGetErrorString(e));
    kern<<<grid, 256, smem, st>>>(a);
    e = cudaGetLastError();
    if (e != cudaSuccess) return fail(nullptr, HALE_E_CUDA, "launch of router failed: %s", cudaGetErrorString(e));
    return HALE_OK;
}

// ---------------------------------------------------------------------------
// self-check
// ---------------------------------------------------------------------------
extern "C" void hale_expf_host(const float* x, float* y, uint64_t n) {
    for (uint64_t i = 0; i < n; i++) y[i] = hale::hale_expf(x[i]);
}

// Detaches every object made on ctx (hale_ctx_destroy): each keeps its own
// device and frees its memory there when it is destroyed later.
static void ctx_detach_children(hale_ctx* ctx) {
    for (hale_matrix* m : ctx->matrices) m->ctx = nullptr;
    for (hale_pool* p : ctx->pools) p->ctx = nullptr;
    for (hale_decoder* d : ctx->decoders) d->ctx = nullptr;
    for (hale_comm* c : ctx->comms) c->ctx = nullptr;
    ctx->matrices.clear();
    ctx->pools.clear();
    ctx->decoders.clear();
    ctx->comms.clear();
}
