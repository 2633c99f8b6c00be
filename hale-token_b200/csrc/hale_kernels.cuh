// hale_kernels.cuh -- the B200 kernels of the MoE expert path and the
// sampling tail. Each kernel names the reference code it reproduces (paths
// inside the Rust reference crate).
//
// Quantized weight layout in HBM ("row tiles"). A matrix of R rows x C cols
// (nb = C/32 blocks per row) is cut into tiles of 32 consecutive rows. Tile
// g holds, for every block b in order, a 32*BB-byte record:
//     [32 rows x QB bytes of quants][32 rows x 2 bytes f16 scale]
// with BB = 18 (q4_0; QB = 16 nibble bytes, same j / j+16 pairing as the
// reference) or 34 (q8_0; QB = 32). A tile is nb * 32 * BB bytes -- the same
// bytes as the reference's 32 rows, reordered so that a warp (lane = row)
// reads one block of all 32 rows as one contiguous 512 B / 1 KiB run, and a
// stage of consecutive blocks is one contiguous span for a bulk async copy.
//
// Float matrices (router excluded, which is read row-major) use
//     tile g, step i: [32 rows x 8 elements]
// so a thread owning row r reads the 8 elements of step i that feed the
// reference's 8 accumulator lanes, and a warp reads 32 rows contiguously.
#pragma once

#include "hale_device.cuh"

namespace hale {

constexpr int kTileRows = 32;
constexpr int kQK = 32;
constexpr int kStageBlocks = 8;  // blocks per bulk-copy stage

template <int QT>
struct QFmt;
template <>
struct QFmt<0> {  // q4_0
    static constexpr int BB = 18, QB = 16;
};
template <>
struct QFmt<1> {  // q8_0
    static constexpr int BB = 34, QB = 32;
};

// ---------------------------------------------------------------------------
// repack: reference row-major encoding -> row tiles
// ---------------------------------------------------------------------------
__global__ void repack_quant_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                    int rows, int rows_pad, int nb, int BB, int QB) {
    long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    long long total = (long long)rows_pad * nb;
    if (idx >= total) return;
    int r = (int)(idx / nb), b = (int)(idx % nb);
    int g = r / kTileRows, lane = r % kTileRows;
    size_t tile_bytes = (size_t)nb * kTileRows * BB;
    uint8_t* rec = dst + (size_t)g * tile_bytes + (size_t)b * kTileRows * BB;
    uint8_t* q = rec + lane * QB;
    uint8_t* s = rec + kTileRows * QB + lane * 2;
    if (r < rows) {
        const uint8_t* blk = src + (size_t)r * nb * BB + (size_t)b * BB;
        s[0] = blk[0];
        s[1] = blk[1];
        for (int j = 0; j < QB; j++) q[j] = blk[2 + j];
    } else {
        s[0] = 0;
        s[1] = 0;
        for (int j = 0; j < QB; j++) q[j] = 0;
    }
}

__global__ void repack_float_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                    int rows, int rows_pad, int cols, int steps, int esize) {
    long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    long long total = (long long)rows_pad * steps;
    if (idx >= total) return;
    int r = (int)(idx / steps), i = (int)(idx % steps);
    int g = r / kTileRows, lane = r % kTileRows;
    uint8_t* d = dst + (((size_t)g * steps + i) * kTileRows + lane) * 8 * esize;
    for (int l = 0; l < 8; l++) {
        int c = i * 8 + l;
        for (int k = 0; k < esize; k++)
            d[l * esize + k] = (r < rows && c < cols) ? src[((size_t)r * cols + c) * esize + k] : 0;
    }
}

// ---------------------------------------------------------------------------
// Q8Activations::quantize (src/tensor/quant.rs:77-93), one warp per row.
// Writes quants [rows, cols] i8 and, per block, the f32 scale (scales,
// nullable) and aux = (scale bits, -8 * sum of the block's quants) (aux,
// nullable; row stride nbp = nb rounded up to even so every aux row starts
// on a 16-byte boundary for bulk copies). The -8*sum term turns the nibble
// dot into the reference's sum of (n - 8) * x exactly (integer arithmetic).
// ---------------------------------------------------------------------------
__host__ __device__ __forceinline__ int aux_stride(int nb) { return (nb + 1) & ~1; }

// One block of Q8Activations::quantize by one thread: the 32 values come in
// with eight 16-byte loads and leave with two 16-byte stores (xb, q 16-byte
// aligned: rows of a multiple of 32 elements).
// SMEM: xb points into shared memory (plain loads instead of the read-only
// global path).
template <bool SMEM = false>
__device__ __forceinline__ void quantize_block(const float* __restrict__ xb, int8_t* __restrict__ q,
                                               float* scale_out, int* sum_out) {
    float v[kQK];
#pragma unroll
    for (int j = 0; j < kQK / 4; j++) {
        float4 f = SMEM ? reinterpret_cast<const float4*>(xb)[j] : __ldg(reinterpret_cast<const float4*>(xb) + j);
        v[4 * j] = f.x; v[4 * j + 1] = f.y; v[4 * j + 2] = f.z; v[4 * j + 3] = f.w;
    }
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < kQK; j++) amax = fmaxf(amax, fabsf(v[j]));
    float scale = fdiv(amax, 127.0f);
    float inv = scale > 0.0f ? fdiv(1.0f, scale) : 0.0f;
    int s = 0;
    uint32_t packed[kQK / 4];
#pragma unroll
    for (int j = 0; j < kQK / 4; j++) {
        uint32_t w = 0;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            int qv = sat_i8(roundf(fmul(v[4 * j + i], inv)));
            s += qv;
            w |= ((uint32_t)qv & 0xffu) << (8 * i);
        }
        packed[j] = w;
    }
    reinterpret_cast<uint4*>(q)[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    reinterpret_cast<uint4*>(q)[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
    *scale_out = scale;
    *sum_out = s;
}

__global__ void quantize_rows_kernel(const float* __restrict__ x, int rows, int cols,
                                     int8_t* __restrict__ quants, float* __restrict__ scales,
                                     int2* __restrict__ aux) {
    int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= rows) return;
    int nb = cols / kQK, nbp = aux_stride(nb);
    const float* xr = x + (size_t)warp * cols;
    for (int b = lane; b < nb; b += 32) {
        float sc;
        int sm;
        quantize_block(xr + b * kQK, quants + (size_t)warp * cols + b * kQK, &sc, &sm);
        if (scales) scales[(size_t)warp * nb + b] = sc;
        if (aux) aux[(size_t)warp * nbp + b] = make_int2(__float_as_int(sc), -8 * sm);
    }
}

// aux from caller-supplied Q8Activations (scales + quants).
__global__ void aux_from_q8_kernel(const float* __restrict__ scales,
                                   const int8_t* __restrict__ quants, int rows, int cols,
                                   int2* __restrict__ aux) {
    long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    int nb = cols / kQK;
    if (idx >= (long long)rows * nb) return;
    int r = (int)(idx / nb), b = (int)(idx % nb);
    const int8_t* q = quants + (size_t)r * cols + b * kQK;
    int s = 0;
    for (int j = 0; j < kQK; j++) s += q[j];
    aux[(size_t)r * aux_stride(nb) + b] = make_int2(__float_as_int(scales[idx]), -8 * s);
}

// ---------------------------------------------------------------------------
// The quantized row-tile dot product (dot_q8_0 / dot_q4_0, quant.rs:115-144)
// for one warp: lane = row of the tile, TG activation rows at once.
//
// Weights stream HBM -> shared memory with cp.async.bulk (the TMA engine)
// through a per-warp ring of S stages of kStageBlocks blocks, each landing
// on its own mbarrier; lane 0 issues, the warp consumes. The activation rows
// of the pass sit in shared memory (XStage, gathered by bulk copies once per
// CTA and pass). Per block and activation row the integer dot is 8 dp4a
// (exact int32); then the reference's float step
//     total += (w_scale * x_scale) * isum,
// in block order and unfused.
// ---------------------------------------------------------------------------
constexpr int kPassRows = 8;  // activation rows per pass

struct Ring {
    uint8_t* buf;      // S * stage_bytes
    uint64_t* bars;    // S mbarriers
    int S;
    int stage_bytes;   // kStageBlocks * 32 * BB
    uint32_t phase;    // bit s = parity of the next completion of slot s
};

template <int QT>
__device__ __forceinline__ void ring_issue(Ring& rg, const uint8_t* gtile, int nb, int st) {
    constexpr int REC = kTileRows * QFmt<QT>::BB;
    int slot = st % rg.S;
    int nblk = min(kStageBlocks, nb - st * kStageBlocks);
    uint32_t bytes = (uint32_t)(nblk * REC);
    mbar_arrive_expect_tx(&rg.bars[slot], bytes);
    bulk_g2s(rg.buf + (size_t)slot * rg.stage_bytes, gtile + (size_t)st * kStageBlocks * REC, bytes,
             &rg.bars[slot]);
}

__device__ __forceinline__ void ring_init(Ring& rg, uint8_t* buf, uint64_t* bars, int S, int stage_bytes) {
    rg.buf = buf;
    rg.bars = bars;
    rg.S = S;
    rg.stage_bytes = stage_bytes;
    rg.phase = 0;
    if ((threadIdx.x & 31) == 0) {
        for (int s = 0; s < S; s++) mbar_init(&rg.bars[s], 1);
        fence_mbar_init();
    }
    __syncwarp();
}

// Activation rows of one pass, in shared memory: quants [kPassRows][stride]
// with stride = cols + 16 (the pad puts the 8 rows an MMA B fragment reads
// in distinct banks), and aux [kPassRows][xaux_stride(nbp)].
struct XStage {
    int8_t* q;
    int2* a;
    uint64_t* bar;
    uint32_t phase;
};

__host__ __device__ inline int xstage_stride(int cols) { return cols + 16; }

// Row stride (int2 units) of the staged aux rows: nbp padded so that
// stride / 2 is odd, which puts the four token pairs (2t, 2t+1) an MMA lane
// group reads in distinct banks.
__host__ __device__ inline int xaux_stride(int nbp) {
    const int s = nbp + 2;
    return (s % 4 == 0) ? s + 2 : s;
}

__device__ __forceinline__ void xstage_init(XStage& xs, int8_t* q, int2* a, uint64_t* bar) {
    xs.q = q;
    xs.a = a;
    xs.bar = bar;
    xs.phase = 0;
    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
}

// Gathers activation rows row_of(base .. base+n-1) into the stage (all
// threads call; thread 0 issues). contiguous: the rows are consecutive in
// global memory (one copy for the aux rows).
template <class RowOf>
__device__ bool xstage_load(XStage& xs, const int8_t* __restrict__ gq, const int2* __restrict__ ga,
                            int cols, int nbp, int base, int n, bool contiguous, RowOf row_of,
                            uint32_t* err) {
    __syncthreads();  // every warp is done with the previous pass
    if (threadIdx.x == 0) {
        const int stride = xstage_stride(cols);
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(xs.bar, (uint32_t)n * (uint32_t)(cols + nbp * 8));
        const int astride = xaux_stride(nbp);
        for (int j = 0; j < n; j++) {
            const int r = contiguous ? row_of(base) + j : row_of(base + j);
            bulk_g2s(xs.q + (size_t)j * stride, gq + (size_t)r * cols, (uint32_t)cols, xs.bar);
            bulk_g2s(xs.a + (size_t)j * astride, ga + (size_t)r * nbp, (uint32_t)(nbp * 8), xs.bar);
        }
    }
    bool ok = mbar_wait(xs.bar, xs.phase, err);
    xs.phase ^= 1u;
    return __syncthreads_and(ok ? 1 : 0) != 0;  // one verdict for the whole CTA
}

// acc[j] = dot(row `lane` of the tile, staged activation row j), j < TG.
// dbg (nullable): block sums of staged row j at dbg[j * dbg_stride + lane*nb + b]
// for j < nvalid. Returns false if a wait timed out.
template <int QT, int TG>
__device__ bool tile_dot(Ring& rg, const uint8_t* __restrict__ gtile, int nb, const XStage& xs,
                         int cols, int nbp, float (&acc)[TG], int32_t* dbg, size_t dbg_stride,
                         int nvalid, uint32_t* err) {
    constexpr int BB = QFmt<QT>::BB, QB = QFmt<QT>::QB, REC = kTileRows * BB;
    const int lane = threadIdx.x & 31;
    const int nst = (nb + kStageBlocks - 1) / kStageBlocks;
#pragma unroll
    for (int j = 0; j < TG; j++) acc[j] = 0.0f;
    if (lane == 0) {
        fence_proxy_async_smem();  // earlier passes read these slots
        for (int st = 0; st < min(rg.S, nst); st++) ring_issue<QT>(rg, gtile, nb, st);
    }
    bool ok = true;
    for (int st = 0; st < nst; st++) {
        int slot = st % rg.S;
        if (!__all_sync(0xffffffffu, mbar_wait(&rg.bars[slot], (rg.phase >> slot) & 1u, err))) {
            ok = false;
            // drain: give the copies already issued a bounded chance to land
            for (int s2 = st; s2 < min(st + rg.S, nst); s2++)
                mbar_wait(&rg.bars[s2 % rg.S], (rg.phase >> (s2 % rg.S)) & 1u, nullptr, 400000000LL);
            break;
        }
        rg.phase ^= 1u << slot;
        const uint8_t* sbuf = rg.buf + (size_t)slot * rg.stage_bytes;
        const int nblk = min(kStageBlocks, nb - st * kStageBlocks);
#pragma unroll 2
        for (int bi = 0; bi < nblk; bi++) {
            const int b = st * kStageBlocks + bi;
            const uint8_t* rec = sbuf + bi * REC;
            float ws = half_bits_to_float(*reinterpret_cast<const uint16_t*>(rec + kTileRows * QB + lane * 2));
            int w[8];
            if (QT == 0) {
                uint4 nib = *reinterpret_cast<const uint4*>(rec + lane * QB);
                w[0] = nib.x & 0x0F0F0F0F;
                w[1] = nib.y & 0x0F0F0F0F;
                w[2] = nib.z & 0x0F0F0F0F;
                w[3] = nib.w & 0x0F0F0F0F;
                w[4] = (nib.x >> 4) & 0x0F0F0F0F;
                w[5] = (nib.y >> 4) & 0x0F0F0F0F;
                w[6] = (nib.z >> 4) & 0x0F0F0F0F;
                w[7] = (nib.w >> 4) & 0x0F0F0F0F;
            } else {
                uint4 q0 = *reinterpret_cast<const uint4*>(rec + lane * QB);
                uint4 q1 = *reinterpret_cast<const uint4*>(rec + lane * QB + 16);
                w[0] = q0.x; w[1] = q0.y; w[2] = q0.z; w[3] = q0.w;
                w[4] = q1.x; w[5] = q1.y; w[6] = q1.z; w[7] = q1.w;
            }
#pragma unroll
            for (int j = 0; j < TG; j++) {
                const int8_t* xp = xs.q + j * xstage_stride(cols) + b * kQK;
                uint4 xa = *reinterpret_cast<const uint4*>(xp);
                uint4 xb = *reinterpret_cast<const uint4*>(xp + 16);
                int2 ax = xs.a[j * xaux_stride(nbp) + b];
                // two independent dp4a chains (integer sums are exact in any order)
                int s0 = (QT == 0) ? ax.y : 0, s1 = 0;
                s0 = __dp4a(w[0], (int)xa.x, s0);
                s1 = __dp4a(w[4], (int)xb.x, s1);
                s0 = __dp4a(w[1], (int)xa.y, s0);
                s1 = __dp4a(w[5], (int)xb.y, s1);
                s0 = __dp4a(w[2], (int)xa.z, s0);
                s1 = __dp4a(w[6], (int)xb.z, s1);
                s0 = __dp4a(w[3], (int)xa.w, s0);
                s1 = __dp4a(w[7], (int)xb.w, s1);
                const int s = s0 + s1;
                if (dbg && j < nvalid) dbg[(size_t)j * dbg_stride + (size_t)lane * nb + b] = s;
                acc[j] = fadd(acc[j], fmul(fmul(ws, __int_as_float(ax.x)), __int2float_rn(s)));
            }
        }
        __syncwarp();
        if (st + rg.S < nst && lane == 0) {
            fence_proxy_async_smem();
            ring_issue<QT>(rg, gtile, nb, st + rg.S);
        }
    }
    __syncwarp();
    return ok;
}

// Exact int -> float of a biased block sum through the f32 significand: for
// |v| < 2^22 the bits (kMagicI + v) read as a float equal 1.5 * 2^23 + v
// exactly, and subtracting 1.5 * 2^23 leaves v. Block sums are bounded by
// 32 * 128 * 127 < 2^22.
constexpr int kMagicI = 0x4B400000;
constexpr float kMagicF = 12582912.0f;

// D = A(16x32 s8, row) x B(32x8 s8, col) + C (s32), warp-wide. A pure
// function of its operands (not volatile), so the compiler may overlap the
// MMAs and loads of consecutive blocks.
__device__ __forceinline__ void mma_s8_16832(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1, int c0,
                                             int c1) {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(c0), "r"(c1), "r"(c0), "r"(c1));
}

// ldmatrix: lane L supplies the shared-memory address of row L % 8 of matrix
// L / 8 (16 contiguous bytes); lane 4 g + t receives, from each matrix, the
// 4 bytes 4t .. 4t+3 of its row g -- the m16n8k32 fragment layout.
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* row_addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_addr(row_addr)));
}
__device__ __forceinline__ void ldsm_x2(uint32_t (&r)[2], const void* row_addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
                 : "=r"(r[0]), "=r"(r[1])
                 : "r"(smem_addr(row_addr)));
}

// The same dot products as tile_dot for a pass of up to kPassRows tokens, on
// the warp-level tensor-core MMA: per block, one m16n8k32 per 16 rows gives
// the integer block sums of 16 rows x 8 tokens; C carries q4_0's -8 * sum(x)
// and kMagicI, so D reads as the biased sum the exact conversion needs. Then
// the reference's float step per (row, token), in block order.
// Lane = 4 g + t holds rows {g, g+8, g+16, g+24} x tokens {2t, 2t+1}. The
// results land in the warp's ring buffer as float [kPassRows][32] (token,
// row), which is free once every stage has been consumed.
template <int QT>
__device__ bool tile_dot_mma(Ring& rg, const uint8_t* __restrict__ gtile, int nb, const XStage& xs, int cols,
                             int nbp, uint32_t* err) {
    constexpr int BB = QFmt<QT>::BB, QB = QFmt<QT>::QB, REC = kTileRows * BB;
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int nst = (nb + kStageBlocks - 1) / kStageBlocks;
    float acc[2][2][2];  // [16-row half][row g or g+8][token 2t or 2t+1]
#pragma unroll
    for (int i = 0; i < 8; i++) (&acc[0][0][0])[i] = 0.0f;
    if (lane == 0) {
        fence_proxy_async_smem();  // earlier passes read these slots
        for (int st = 0; st < min(rg.S, nst); st++) ring_issue<QT>(rg, gtile, nb, st);
    }
    // ldmatrix row addresses: B -- token (lane & 7), K half (lane >> 3) & 1;
    // A -- row `lane` of the tile (q4_0: its 16 nibble bytes; q8_0: first or
    // second 16 bytes of rows (lane & 15) + 16 * mt, half lane >> 4)
    const int8_t* xrow = xs.q + (lane & 7) * xstage_stride(cols) + ((lane >> 3) & 1) * 16;
    const int2* a0row = xs.a + (2 * t) * xaux_stride(nbp);
    const int2* a1row = xs.a + (2 * t + 1) * xaux_stride(nbp);
    bool ok = true;
    for (int st = 0; st < nst; st++) {
        int slot = st % rg.S;
        if (!__all_sync(0xffffffffu, mbar_wait(&rg.bars[slot], (rg.phase >> slot) & 1u, err))) {
            ok = false;
            for (int s2 = st; s2 < min(st + rg.S, nst); s2++)
                mbar_wait(&rg.bars[s2 % rg.S], (rg.phase >> (s2 % rg.S)) & 1u, nullptr, 400000000LL);
            break;
        }
        rg.phase ^= 1u << slot;
        const uint8_t* sbuf = rg.buf + (size_t)slot * rg.stage_bytes;
        const int nblk = min(kStageBlocks, nb - st * kStageBlocks);
#pragma unroll 2
        for (int bi = 0; bi < nblk; bi++) {
            const int b = st * kStageBlocks + bi;
            const uint8_t* rec = sbuf + bi * REC;
            uint32_t bf[2];
            ldsm_x2(bf, xrow + b * kQK);
            const uint32_t bf0 = bf[0], bf1 = bf[1];
            const int2 x0 = a0row[b], x1 = a1row[b];
            const int c0 = ((QT == 0) ? x0.y : 0) + kMagicI, c1 = ((QT == 0) ? x1.y : 0) + kMagicI;
            const float xs0 = __int_as_float(x0.x), xs1 = __int_as_float(x1.x);
            // words t of rows g, g+8, g+16, g+24 (q4_0) -- byte j of a row holds
            // element j (low nibble) and j + 16 (high)
            uint32_t w4[4];
            if (QT == 0) ldsm_x4(w4, rec + lane * QB);
#pragma unroll
            for (int mt = 0; mt < 2; mt++) {
                const int r0 = mt * 16 + g, r1 = r0 + 8;
                uint32_t a[4];
                if (QT == 0) {
                    a[0] = w4[2 * mt] & 0x0F0F0F0Fu;
                    a[1] = w4[2 * mt + 1] & 0x0F0F0F0Fu;
                    a[2] = (w4[2 * mt] >> 4) & 0x0F0F0F0Fu;
                    a[3] = (w4[2 * mt + 1] >> 4) & 0x0F0F0F0Fu;
                } else {
                    // matrices (rows 0-7, K 0-15), (rows 8-15, K 0-15), (rows 0-7,
                    // K 16-31), (rows 8-15, K 16-31) of this half: a0 .. a3
                    ldsm_x4(a, rec + (mt * 16 + (lane & 15)) * QB + (lane >> 4) * 16);
                }
                int d[4];
                mma_s8_16832(d, a, bf0, bf1, c0, c1);
                const float ws0 = half_bits_to_float(*reinterpret_cast<const uint16_t*>(rec + kTileRows * QB + r0 * 2));
                const float ws1 = half_bits_to_float(*reinterpret_cast<const uint16_t*>(rec + kTileRows * QB + r1 * 2));
                // d: (r0, 2t), (r0, 2t+1), (r1, 2t), (r1, 2t+1)
                acc[mt][0][0] = fadd(acc[mt][0][0], fmul(fmul(ws0, xs0), fsub(__int_as_float(d[0]), kMagicF)));
                acc[mt][0][1] = fadd(acc[mt][0][1], fmul(fmul(ws0, xs1), fsub(__int_as_float(d[1]), kMagicF)));
                acc[mt][1][0] = fadd(acc[mt][1][0], fmul(fmul(ws1, xs0), fsub(__int_as_float(d[2]), kMagicF)));
                acc[mt][1][1] = fadd(acc[mt][1][1], fmul(fmul(ws1, xs1), fsub(__int_as_float(d[3]), kMagicF)));
            }
        }
        __syncwarp();
        if (st + rg.S < nst && lane == 0) {
            fence_proxy_async_smem();
            ring_issue<QT>(rg, gtile, nb, st + rg.S);
        }
    }
    __syncwarp();
    if (ok) {
        float* outb = reinterpret_cast<float*>(rg.buf);  // every issued stage was consumed
#pragma unroll
        for (int mt = 0; mt < 2; mt++)
#pragma unroll
            for (int h = 0; h < 2; h++)
#pragma unroll
                for (int j = 0; j < 2; j++) outb[(2 * t + j) * kTileRows + mt * 16 + h * 8 + g] = acc[mt][h][j];
    }
    __syncwarp();
    return ok;
}

// Passes of at least this many rows go through tile_dot_mma.
constexpr int kMmaMinRows = 3;

// Runs tile_dot with the pass width equal to the pass's row count n (1..8,
// each width its own unrolled instance) and hands the results to
// emit(j, value).
template <int QT, int TG, class Emit>
__device__ __forceinline__ bool tile_dot_w(Ring& rg, const uint8_t* gtile, int nb, const XStage& xs, int cols,
                                           int nbp, int32_t* dbg, size_t dbg_stride, uint32_t* err, Emit& emit) {
    float acc[TG];
    bool ok = tile_dot<QT, TG>(rg, gtile, nb, xs, cols, nbp, acc, dbg, dbg_stride, TG, err);
    if (ok)
#pragma unroll
        for (int j = 0; j < TG; j++) emit(j, acc[j]);
    return ok;
}

// use_mma (uniform across the CTA): passes of kMmaMinRows or more rows take
// the tensor-core path; the block-sum debug output needs use_mma false.
template <int QT, class Emit>
__device__ bool tile_dot_n(Ring& rg, const uint8_t* gtile, int nb, const XStage& xs, int cols, int nbp,
                           int n, int32_t* dbg, size_t dbg_stride, bool use_mma, uint32_t* err, Emit emit) {
    if (use_mma && n >= kMmaMinRows) {
        const bool ok = tile_dot_mma<QT>(rg, gtile, nb, xs, cols, nbp, err);
        if (ok) {
            const float* res = reinterpret_cast<const float*>(rg.buf);
            const int lane = threadIdx.x & 31;
            for (int j = 0; j < n; j++) emit(j, res[j * kTileRows + lane]);
        }
        __syncwarp();  // results read before the next pass's copies reuse the ring
        return ok;
    }
    switch (n) {
    case 1: return tile_dot_w<QT, 1>(rg, gtile, nb, xs, cols, nbp, dbg, dbg_stride, err, emit);
    case 2: return tile_dot_w<QT, 2>(rg, gtile, nb, xs, cols, nbp, dbg, dbg_stride, err, emit);
    case 3: return tile_dot_w<QT, 3>(rg, gtile, nb, xs, cols, nbp, dbg, dbg_stride, err, emit);
    case 4: return tile_dot_w<QT, 4>(rg, gtile, nb, xs, cols, nbp, dbg, dbg_stride, err, emit);
    case 5: return tile_dot_w<QT, 5>(rg, gtile, nb, xs, cols, nbp, dbg, dbg_stride, err, emit);
    case 6: return tile_dot_w<QT, 6>(rg, gtile, nb, xs, cols, nbp, dbg, dbg_stride, err, emit);
    case 7: return tile_dot_w<QT, 7>(rg, gtile, nb, xs, cols, nbp, dbg, dbg_stride, err, emit);
    default: return tile_dot_w<QT, 8>(rg, gtile, nb, xs, cols, nbp, dbg, dbg_stride, err, emit);
    }
}

// Shared-memory plan of the GEMV kernels: per-warp rings, then the
// activation stage, then the barriers.
struct SmemPlan {
    int stage_bytes, ring_bytes, xq_off, xa_off, bars_off, total;
};

__host__ __device__ inline SmemPlan smem_plan(int BB, int S, int warps, int cols) {
    SmemPlan p;
    p.stage_bytes = kStageBlocks * kTileRows * BB;
    p.ring_bytes = S * p.stage_bytes;
    p.xq_off = warps * p.ring_bytes;
    int nbp = aux_stride(cols / kQK);
    p.xa_off = p.xq_off + kPassRows * xstage_stride(cols);
    p.bars_off = p.xa_off + kPassRows * xaux_stride(nbp) * 8;
    p.total = p.bars_off + (warps * S + 1) * 8;
    return p;
}

// ---------------------------------------------------------------------------
// WeightMatrix::matvec for quantized matrices (matrix.rs:115-126): a CTA of
// 4 warps covers 4 row tiles (128 rows); activation rows go in passes of 8.
// dbg: block sums [M, rows, nb].
// ---------------------------------------------------------------------------
template <int QT>
__global__ void __launch_bounds__(128) qgemv_kernel(const uint8_t* __restrict__ W, int rows, int nb,
                                                    const int8_t* __restrict__ xq,
                                                    const int2* __restrict__ xaux, int M,
                                                    float* __restrict__ out, int32_t* dbg,
                                                    int S, uint32_t* err) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, cols = nb * kQK, nbp = aux_stride(nb);
    const SmemPlan P = smem_plan(QFmt<QT>::BB, S, 4, cols);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + P.bars_off);
    Ring rg;
    ring_init(rg, smem + warp * P.ring_bytes, bars + warp * S, S, P.stage_bytes);
    XStage xs;
    xstage_init(xs, reinterpret_cast<int8_t*>(smem + P.xq_off), reinterpret_cast<int2*>(smem + P.xa_off),
                 bars + 4 * S);
    const int ntiles = (rows + kTileRows - 1) / kTileRows;
    const int g = blockIdx.x * 4 + warp;
    const int row = g * kTileRows + lane;
    const uint8_t* gtile = W + (size_t)g * nb * kTileRows * QFmt<QT>::BB;
    for (int base = 0; base < M; base += kPassRows) {
        const int n = min(kPassRows, M - base);
        if (!xstage_load(xs, xq, xaux, cols, nbp, base, n, true, [](int j) { return j; }, err)) return;
        if (g >= ntiles) continue;
        int32_t* d = (dbg && row < rows) ? dbg + (size_t)base * rows * nb + (size_t)g * kTileRows * nb : nullptr;
        tile_dot_n<QT>(rg, gtile, nb, xs, cols, nbp, n, d, (size_t)rows * nb, dbg == nullptr, err, [&](int j, float v) {
            if (row < rows) out[(size_t)(base + j) * rows + row] = v;
        });
    }
}

// ---------------------------------------------------------------------------
// Router: MoeLayer::route (src/model/moe.rs:36-53).
//
// Logits: each (token, expert) pair is 8 threads, thread l owning the
// reference's accumulator lane l (quant.rs:152-160): acc += w[8i+l]*x[8i+l]
// over i in order, then reduce() (quant.rs:37-41) and the tail. A CTA covers
// 4 tokens x 8 experts; the router rows and token rows stream into shared
// memory in column chunks by bulk copies (two-slot ring), so the 8-lane
// chains run from shared memory. The last CTA to finish a token tile then
// runs softmax (activation.rs:11-21), top-k with (score desc, index asc)
// (topk.rs:27-61) and the weight normalisation, and quantizes the tile's
// activation rows. The last such CTA of the grid groups the routes by
// expert for the expert kernels.
// ---------------------------------------------------------------------------
constexpr int kRouterTT = 4, kRouterET = 8, kRouterCH = 1024, kRouterPad = 8;  // pad: 8-bank row skew
constexpr int kRouterSlots = 4;

struct RouterArgs {
    const void* w;
    int wdtype;  // 0 f32, 1 f16, 2 bf16
    int E, H, M, k, normalize;
    int staged;             // rows stream through shared memory (H % 8 == 0)
    const float* x;
    float* logits;          // [M, E]
    float* probs_out;       // [M, E] nullable
    int* topk_idx;          // [M, k]
    float* topk_w;          // [M, k]
    int* user_idx;          // nullable copies for the caller
    float* user_w;
    int8_t* xq;             // [M, H] nullable (route-only calls skip it)
    int2* xaux;             // [M, nbp(H)]
    int* elist_off;         // [E + 1]   (nullable: route-only)
    int* elist;             // [M * k]
    int* active;            // [E]
    int* n_active;          // [1]
    unsigned long long* routing_counts;  // [E] nullable
    unsigned* tile_cnt;     // [ceil(M / TT)]
    unsigned* grid_cnt;     // [1]
    uint32_t* err;
};

// Router weight element c (DT: 0 f32, 1 f16, 2 bf16) -- a compile-time
// format, so the chains' loads can be issued ahead of the adds.
template <int DT>
__device__ __forceinline__ float load_w(const void* w, size_t i) {
    if (DT == 0) return __ldg(reinterpret_cast<const float*>(w) + i);
    uint16_t h = __ldg(reinterpret_cast<const unsigned short*>(w) + i);
    if (DT == 2) return __uint_as_float((uint32_t)h << 16);
    return half_bits_to_float(h);
}

template <int DT>
__device__ __forceinline__ float smem_w(const uint8_t* row, int c) {
    if (DT == 0) return reinterpret_cast<const float*>(row)[c];
    uint16_t h = reinterpret_cast<const uint16_t*>(row)[c];
    if (DT == 2) return __uint_as_float((uint32_t)h << 16);
    return half_bits_to_float(h);
}

__host__ __device__ inline int router_slot_bytes(int wbytes) {
    return kRouterET * (kRouterCH + kRouterPad) * wbytes + kRouterTT * (kRouterCH + kRouterPad) * 4;
}

// Phase marks for timing probes built from this header; empty in the library.
#ifndef HALE_ROUTER_MARK
#define HALE_ROUTER_MARK(i)
#endif

template <int DT>
__global__ void __launch_bounds__(256) router_kernel(RouterArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ unsigned s_flag;
    __shared__ uint64_t s_tab[32];
    __shared__ __align__(16) float s_e[8][256];
    __shared__ int s_cnt[256];
    __shared__ int s_cur[256];
    const int tid = threadIdx.x, lane8 = tid & 7, pair = tid >> 3;
    const int tl = pair / kRouterET, el = pair % kRouterET;
    const int t = blockIdx.x * kRouterTT + tl;
    const int e = blockIdx.y * kRouterET + el;
    const bool valid = t < a.M && e < a.E;
    const int full = a.H / 8;
    constexpr int wb = DT == 0 ? 4 : 2;
    if (tid < 32) s_tab[tid] = kExp2TabDev[tid];  // exp table for the tail (read after barriers)
    HALE_ROUTER_MARK(0);
    float acc = 0.0f;
    if (a.staged) {
        // ring of column chunks [8 router rows][4 token rows]; with up to
        // kRouterSlots slots every chunk of a 2048-wide row is in flight at once
        const int slot_bytes = router_slot_bytes(wb);
        const int nch = (a.H + kRouterCH - 1) / kRouterCH;
        const int NS = min(nch, kRouterSlots);
        uint64_t* bars = reinterpret_cast<uint64_t*>(smem + NS * slot_bytes);
        const int rpitch = (kRouterCH + kRouterPad) * wb, xpitch = (kRouterCH + kRouterPad) * 4;
        if (tid == 0) {
            for (int q = 0; q < NS; q++) mbar_init(&bars[q], 1);
            fence_mbar_init();
        }
        __syncthreads();
        auto issue = [&](int c) {
            const int q = c % NS;
            uint8_t* slot = smem + q * slot_bytes;
            const int c0 = c * kRouterCH, len = min(kRouterCH, a.H - c0);
            const int nr = min(kRouterET, a.E - (int)blockIdx.y * kRouterET);
            const int nt = min(kRouterTT, a.M - (int)blockIdx.x * kRouterTT);
            fence_proxy_async_smem();
            mbar_arrive_expect_tx(&bars[q], (uint32_t)(nr * len * wb + nt * len * 4));
            for (int r = 0; r < nr; r++)
                bulk_g2s(slot + r * rpitch,
                         reinterpret_cast<const uint8_t*>(a.w) + ((size_t)(blockIdx.y * kRouterET + r) * a.H + c0) * wb,
                         (uint32_t)(len * wb), &bars[q]);
            for (int r = 0; r < nt; r++)
                bulk_g2s(slot + kRouterET * rpitch + r * xpitch,
                         a.x + (size_t)(blockIdx.x * kRouterTT + r) * a.H + c0, (uint32_t)(len * 4),
                         &bars[q]);
        };
        if (tid == 0)
            for (int c = 0; c < NS; c++) issue(c);
        uint32_t phase = 0;
        bool ok = true;
        for (int c = 0; c < nch; c++) {
            const int q = c % NS;
            // every chunk is waited on (bounded) even after a timeout, so no
            // copy is still landing when the CTA moves on
            ok = mbar_wait(&bars[q], (phase >> q) & 1u, a.err) && ok;
            phase ^= 1u << q;
            const uint8_t* slot = smem + q * slot_bytes;
            const uint8_t* wrow = slot + el * rpitch;
            const float* xrow = reinterpret_cast<const float*>(slot + kRouterET * rpitch + tl * xpitch);
            const int steps = min(kRouterCH, a.H - c * kRouterCH) / 8;
            if (valid && ok) {
#pragma unroll 8
                for (int i = 0; i < steps; i++)
                    acc = fadd(acc, fmul(smem_w<DT>(wrow, 8 * i + lane8), xrow[8 * i + lane8]));
            }
            __syncthreads();
            if (tid == 0 && c + NS < nch) issue(c + NS);
        }
    } else if (valid) {
        const float* xt = a.x + (size_t)t * a.H;
        size_t wrow = (size_t)e * a.H;
#pragma unroll 8
        for (int i = 0; i < full; i++) {
            int c = 8 * i + lane8;
            acc = fadd(acc, fmul(load_w<DT>(a.w, wrow + c), __ldg(xt + c)));
        }
    }
    // reduce(): ((l0+l4)+(l1+l5)) + ((l2+l6)+(l3+l7))
    float s = fadd(acc, __shfl_down_sync(0xffffffffu, acc, 4, 8));
    float p = fadd(s, __shfl_down_sync(0xffffffffu, s, 1, 8));
    float r = fadd(p, __shfl_down_sync(0xffffffffu, p, 2, 8));
    if (valid && lane8 == 0) {
        float tail = -0.0f;
        const float* xt = a.x + (size_t)t * a.H;
        for (int c = full * 8; c < a.H; c++)
            tail = fadd(tail, fmul(load_w<DT>(a.w, (size_t)e * a.H + c), xt[c]));
        a.logits[(size_t)t * a.E + e] = fadd(r, tail);
    }
    HALE_ROUTER_MARK(1);
    __threadfence();
    __syncthreads();
    if (tid == 0) s_flag = (atomicAdd(&a.tile_cnt[blockIdx.x], 1u) == gridDim.y - 1) ? 1u : 0u;
    __syncthreads();
    if (!s_flag) return;
    __threadfence();
    HALE_ROUTER_MARK(2);

    // ---- last CTA of this token tile: softmax, top-k, quantize ----------
    // warps 0 .. kRouterTT-1: softmax and top-k of one token each; the other
    // warps quantize the tile's activation rows meanwhile
    const int warp = tid >> 5, lane = tid & 31;
    static_assert(kRouterTT < 8, "the router tail needs warps left for quantization");
    if (warp >= kRouterTT && a.xq) {
        // Q8Activations::quantize of the tile's tokens (quant.rs:77-93)
        const int nb = a.H / kQK, nbp = aux_stride(nb);
        const int nt = min(kRouterTT, a.M - (int)blockIdx.x * kRouterTT);
        for (int i = tid - kRouterTT * 32; i < nt * nb; i += (8 - kRouterTT) * 32) {
            const int tt = i / nb, b = i - tt * nb;
            const int tok = blockIdx.x * kRouterTT + tt;
            float sc;
            int sm;
            quantize_block(a.x + (size_t)tok * a.H + b * kQK, a.xq + (size_t)tok * a.H + b * kQK, &sc, &sm);
            a.xaux[(size_t)tok * nbp + b] = make_int2(__float_as_int(sc), -8 * sm);
        }
    }
    for (int tt = warp; tt < kRouterTT; tt += 8) {
        const int tok = blockIdx.x * kRouterTT + tt;
        if (tok >= a.M) break;
        const float* lg = a.logits + (size_t)tok * a.E;
        // the token's logits (E <= 256) read once into registers
        float lv[8];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int i = lane + 32 * j;
            lv[j] = i < a.E ? __ldcg(lg + i) : -__int_as_float(0x7f800000);
        }
        float mx = lv[0];
#pragma unroll
        for (int j = 1; j < 8; j++) mx = fmaxf(mx, lv[j]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int i = lane + 32 * j;
            if (i < a.E) s_e[warp][i] = hale_expf_tab(fsub(lv[j], mx), s_tab);
        }
        __syncwarp();
        // the reference's left-to-right sum, on one lane, loads batched 4 wide
        float sum = 0.0f;
        if (lane == 0) {
            int i = 0;
            for (; i + 4 <= a.E; i += 4) {
                float4 q4 = *reinterpret_cast<const float4*>(&s_e[warp][i]);
                sum = fadd(fadd(fadd(fadd(sum, q4.x), q4.y), q4.z), q4.w);
            }
            for (; i < a.E; i++) sum = fadd(sum, s_e[warp][i]);
        }
        sum = __shfl_sync(0xffffffffu, sum, 0);
        __syncwarp();
        for (int i = lane; i < a.E; i += 32) {
            float pv = fdiv(s_e[warp][i], sum);
            s_e[warp][i] = pv;
            if (a.probs_out) a.probs_out[(size_t)tok * a.E + i] = pv;
        }
        __syncwarp();
        // top-k by (total_cmp desc, index asc): keys in registers as unsigned
        // total-order keys; each round a warp max over keys, then the lowest
        // index holding it (topk.rs:27-35)
        unsigned ukey[8];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int i = lane + 32 * j;
            ukey[j] = i < a.E ? ((unsigned)total_key(s_e[warp][i]) ^ 0x80000000u) : 0u;
        }
        unsigned taken = 0u;  // bit j: element lane + 32 j selected (E <= 256)
        float chosen_score = 0.0f;
        int chosen_idx = -1;
        float norm = -0.0f;
        for (int kk = 0; kk < a.k; kk++) {
            unsigned bk = 0u;
            int bj = -1;
#pragma unroll
            for (int j = 0; j < 8; j++)
                if (!(taken & (1u << j)) && lane + 32 * j < a.E && (bj < 0 || ukey[j] > bk)) { bk = ukey[j]; bj = j; }
            const unsigned wk = __reduce_max_sync(0xffffffffu, bj >= 0 ? bk : 0u);
            const unsigned mine = (bj >= 0 && bk == wk) ? (unsigned)(lane + 32 * bj) : 0xffffffffu;
            const int bi = (int)__reduce_min_sync(0xffffffffu, mine);
            if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
            float sc = s_e[warp][bi];
            norm = fadd(norm, sc);
            if (lane == kk) { chosen_score = sc; chosen_idx = bi; }
        }
        if (lane < a.k) {
            float wv = a.normalize ? fdiv(chosen_score, norm) : fdiv(chosen_score, 1.0f);
            a.topk_idx[(size_t)tok * a.k + lane] = chosen_idx;
            a.topk_w[(size_t)tok * a.k + lane] = wv;
            if (a.user_idx) a.user_idx[(size_t)tok * a.k + lane] = chosen_idx;
            if (a.user_w) a.user_w[(size_t)tok * a.k + lane] = wv;
        }
        __syncwarp();
    }
    HALE_ROUTER_MARK(3);
    if (gridDim.x == 1) {
        // one token tile: this CTA is also the last of the grid, and its own
        // writes are visible to all its threads after the barrier
        __syncthreads();
        if (tid == 0) a.tile_cnt[blockIdx.x] = 0u;
        if (!a.elist_off) return;
    } else {
        __threadfence();
        __syncthreads();
        if (tid == 0) {
            a.tile_cnt[blockIdx.x] = 0u;
            s_flag = (atomicAdd(a.grid_cnt, 1u) == gridDim.x - 1) ? 1u : 0u;
        }
        __syncthreads();
        if (!s_flag || !a.elist_off) {
            if (s_flag && tid == 0) *a.grid_cnt = 0u;
            return;
        }
        __threadfence();
    }

    // ---- last CTA of the grid: group routes by expert ----------------------
    HALE_ROUTER_MARK(4);
    const int R = a.M * a.k;
    for (int i = tid; i < a.E; i += blockDim.x) s_cnt[i] = 0;
    __syncthreads();
    for (int i = tid; i < R; i += blockDim.x) atomicAdd(&s_cnt[__ldcg(a.topk_idx + i)], 1);
    __syncthreads();
    // exclusive scans over the (<= 256) experts: route offsets and the
    // compacted list of experts with work; one expert per thread
    {
        const int c = tid < a.E ? s_cnt[tid] : 0;
        int incl = c, act = c > 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int u = __shfl_up_sync(0xffffffffu, incl, o), v = __shfl_up_sync(0xffffffffu, act, o);
            if (lane >= o) { incl += u; act += v; }
        }
        __shared__ int w_sum[8], w_act[8];
        if (lane == 31) { w_sum[warp] = incl; w_act[warp] = act; }
        __syncthreads();
        int base_s = 0, base_a = 0;
        for (int w2 = 0; w2 < warp; w2++) { base_s += w_sum[w2]; base_a += w_act[w2]; }
        if (tid < a.E) {
            const int off = base_s + incl - c;
            a.elist_off[tid] = off;
            s_cur[tid] = off;
            if (c > 0) {
                // experts with work, most routes first (ties: lower id): the
                // persistent kernels claim work in this order, so the longest
                // units start first and the tail is short
                int rank = 0;
                for (int e2 = 0; e2 < a.E; e2++) {
                    const int c2 = s_cnt[e2];
                    rank += (c2 > c) || (c2 == c && e2 < tid);
                }
                a.active[rank] = tid;
                if (a.routing_counts) a.routing_counts[tid] += (unsigned long long)c;
            }
        }
        if (tid == a.E - 1) {
            a.elist_off[a.E] = base_s + incl;
            *a.n_active = base_a + act;
        }
    }
    __syncthreads();
    for (int i = tid; i < R; i += blockDim.x) {
        int ex = __ldcg(a.topk_idx + i);
        int pos = atomicAdd(&s_cur[ex], 1);
        a.elist[pos] = i;
    }
    if (tid == 0) *a.grid_cnt = 0u;
    HALE_ROUTER_MARK(5);
}

// ---------------------------------------------------------------------------
// Expert kernels: Expert::forward (src/expert/mod.rs:91-103) for every route
// of the layer, grouped by expert so each weight tile is read from HBM once
// for all tokens routed to it.
// ---------------------------------------------------------------------------
struct ExpertArgs {
    const uint8_t* experts;   // layer base: E experts, each [gate tiles][up tiles][down tiles]
    size_t expert_stride;     // bytes per expert
    const int* slot;          // nullable [E]: expert e lives at experts + slot[e] * stride (tiered pools)
    int H, I, k, M;
    const int* elist_off;     // [E + 1]: routes of expert e are slots off[e] .. off[e+1]-1
    const int* elist;         // [M * k]: route id (token * k + s) of each slot
    const int* active;
    const int* n_active;
    const int8_t* xq;         // [M, H]
    const int2* xaux;         // [M, nbp(H)]
    int8_t* hq;               // [M*k slots, I]   (slot order)
    int2* haux;               // [M*k slots, nbp(I)]
    float* ybuf;              // [M*k routes, H]  (route order)
    unsigned* comb_cnt;       // [M, ceil(H / 128)]
    unsigned* ws_cnt;         // [4]: streaming kernels' unit / retire counters
    const float* topk_w;      // [M, k]
    float* out;               // [M, H]
    float* const* out_rows;   // nullable [M]: token t's output row (else out + t * H); NULL entry = drop
    int S1, S2;               // ring depths of the gate/up and down kernels
    int expert0;              // tensor-map slot of expert 0 of the layer (resident pools)
    uint32_t* err;
};

// Output row of token t of the combine.
__device__ __forceinline__ float* out_row(const ExpertArgs& a, int t) {
    return a.out_rows ? a.out_rows[t] : a.out + (size_t)t * a.H;
}

// Tiled weights of expert e: its own position in a resident pool's layer, or
// the HBM slot a tiered pool placed it in for this forward.
__device__ __forceinline__ const uint8_t* expert_base(const ExpertArgs& a, int e) {
    return a.experts + (size_t)(a.slot ? __ldg(a.slot + e) : e) * a.expert_stride;
}

// Phase 1: one CTA per (active expert, RT consecutive 32-row tiles of the
// intermediate dimension). Warps 0..RT-1 take the gate tiles, RT..2RT-1 the
// matching up tiles. After each pass the gate warps hand g to the up warps
// through shared memory, which form h = silu(g) * u (expert/mod.rs:100-102)
// and quantize it: the 32 rows of a tile are exactly one q8 block of h,
// which the reference re-quantizes before the down projection
// (matrix.rs:119-121). h is written in slot order, so each expert's rows are
// contiguous for phase 2.
template <int QT, int RT>
__global__ void __launch_bounds__(64 * RT) expert_gate_up_kernel(ExpertArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float s_g[RT][kPassRows][kTileRows];
    constexpr int REC = kTileRows * QFmt<QT>::BB;
    constexpr int W = 2 * RT;
    const int TI = a.I / kTileRows, nbh = a.H / kQK, nbph = aux_stride(nbh), nbpi = aux_stride(a.I / kQK);
    const int units = (TI + RT - 1) / RT;
    const int ai = blockIdx.x / units;
    if (ai >= *a.n_active) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m = warp / RT, tl = warp % RT;           // m: 0 gate, 1 up
    const int tile = (blockIdx.x % units) * RT + tl;    // tile of the intermediate dim
    const int e = a.active[ai];
    const int beg = a.elist_off[e], T = a.elist_off[e + 1] - beg;
    const SmemPlan P = smem_plan(QFmt<QT>::BB, a.S1, W, a.H);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + P.bars_off);
    Ring rg;
    ring_init(rg, smem + warp * P.ring_bytes, bars + warp * a.S1, a.S1, P.stage_bytes);
    XStage xs;
    xstage_init(xs, reinterpret_cast<int8_t*>(smem + P.xq_off), reinterpret_cast<int2*>(smem + P.xa_off),
                bars + W * a.S1);
    const size_t tile_bytes = (size_t)nbh * REC;
    const uint8_t* gtile = expert_base(a, e) + (size_t)(m * TI + tile) * tile_bytes;
    const int* routes = a.elist + beg;
    const int k = a.k;
    const bool live = tile < TI;
    for (int base = 0; base < T; base += kPassRows) {
        const int n = min(kPassRows, T - base);
        if (!xstage_load(xs, a.xq, a.xaux, a.H, nbph, base, n, false, [&](int j) { return routes[j] / k; }, a.err))
            return;
        float myv[kPassRows];
#pragma unroll
        for (int j = 0; j < kPassRows; j++) myv[j] = 0.0f;
        bool ok = true;
        if (live)
            ok = tile_dot_n<QT>(rg, gtile, nbh, xs, a.H, nbph, n, nullptr, 0, true, a.err, [&](int j, float v) {
#pragma unroll
                for (int q = 0; q < kPassRows; q++) if (q == j) myv[q] = v;
            });
        if (m == 0 && live)
#pragma unroll
            for (int j = 0; j < kPassRows; j++) s_g[tl][j][lane] = myv[j];
        if (!__syncthreads_and(ok ? 1 : 0)) return;  // also publishes s_g
        if (m == 1 && live) {
            for (int j = 0; j < n; j++) {
                const int slot = beg + base + j;
                float h = fmul(silu(s_g[tl][j][lane]), myv[j]);
                float amax = warp_max_abs(h);
                float scale = fdiv(amax, 127.0f);
                float inv = scale > 0.0f ? fdiv(1.0f, scale) : 0.0f;
                int q = sat_i8(roundf(fmul(h, inv)));
                int qs = warp_sum_int(q);
                a.hq[(size_t)slot * a.I + tile * kTileRows + lane] = (int8_t)q;
                if (lane == 0) a.haux[(size_t)slot * nbpi + tile] = make_int2(__float_as_int(scale), -8 * qs);
            }
        }
    }
}

// Phase 2: one CTA (4 warps) per (active expert, 4 consecutive 32-row tiles
// of the down projection); y for every route of the expert. The last of a
// token's k routes to land for a 128-row group combines them in best-first
// order (moe.rs:63-68): out = 0; out += w_s * y_s for s = 0..k-1, unfused.
template <int QT>
__global__ void __launch_bounds__(128) expert_down_kernel(ExpertArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int s_last[kPassRows];
    constexpr int REC = kTileRows * QFmt<QT>::BB;
    const int TI = a.I / kTileRows, TH = a.H / kTileRows, nbi = a.I / kQK, nbh = a.H / kQK;
    const int nbpi = aux_stride(nbi);
    const int groups = (TH + 3) / 4;
    const int ai = blockIdx.x / groups, grp = blockIdx.x % groups;
    if (ai >= *a.n_active) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tile = grp * 4 + warp;
    const bool live = tile < TH;
    const int e = a.active[ai];
    const int beg = a.elist_off[e], T = a.elist_off[e + 1] - beg;
    const SmemPlan P = smem_plan(QFmt<QT>::BB, a.S2, 4, a.I);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + P.bars_off);
    Ring rg;
    ring_init(rg, smem + warp * P.ring_bytes, bars + warp * a.S2, a.S2, P.stage_bytes);
    XStage xs;
    xstage_init(xs, reinterpret_cast<int8_t*>(smem + P.xq_off), reinterpret_cast<int2*>(smem + P.xa_off),
                bars + 4 * a.S2);
    const size_t gu_tile = (size_t)nbh * REC, d_tile = (size_t)nbi * REC;
    const uint8_t* gtile = expert_base(a, e) + (size_t)2 * TI * gu_tile + (size_t)tile * d_tile;
    const int* routes = a.elist + beg;
    const int k = a.k;
    for (int base = 0; base < T; base += kPassRows) {
        const int n = min(kPassRows, T - base);
        if (!xstage_load(xs, a.hq, a.haux, a.I, nbpi, beg + base, n, true, [](int j) { return j; }, a.err))
            return;
        bool ok = true;
        if (live)
            ok = tile_dot_n<QT>(rg, gtile, nbi, xs, a.I, nbpi, n, nullptr, 0, true, a.err, [&](int j, float v) {
                a.ybuf[(size_t)routes[base + j] * a.H + tile * kTileRows + lane] = v;
            });
        __threadfence();
        if (!__syncthreads_and(ok ? 1 : 0)) return;
        if (threadIdx.x < n) {
            const int tok = routes[base + threadIdx.x] / k;
            unsigned old = atomicAdd(&a.comb_cnt[(size_t)tok * groups + grp], 1u);
            s_last[threadIdx.x] = old == (unsigned)(k - 1);
            if (old == (unsigned)(k - 1)) a.comb_cnt[(size_t)tok * groups + grp] = 0u;
        }
        __syncthreads();
        __threadfence();
        for (int j = 0; j < n; j++) {
            if (!s_last[j] || !live) continue;
            const int tok = routes[base + j] / k;
            float o = 0.0f;
            for (int s2 = 0; s2 < k; s2++) {
                float w = __ldcg(a.topk_w + (size_t)tok * k + s2);
                float y = __ldcg(a.ybuf + ((size_t)tok * k + s2) * a.H + tile * kTileRows + lane);
                o = fadd(o, fmul(w, y));
            }
            float* orow = out_row(a, tok);
            if (orow) orow[tile * kTileRows + lane] = o;
        }
    }
}

// ---------------------------------------------------------------------------
// Float GEMV (quant.rs:146-202 via matrix.rs:115-126): lm_head and float
// WeightMatrix::matvec. One thread per row owning all 8 accumulator lanes;
// steps i over the full groups of 8 in order, then reduce() + tail.
// ---------------------------------------------------------------------------
template <int DT>
__device__ __forceinline__ void load8(const uint8_t* p, float (&w)[8]) {
    if (DT == 0) {
        float4 a = __ldg(reinterpret_cast<const float4*>(p));
        float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
        w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w;
        w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
    } else {
        uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
        uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int q = 0; q < 4; q++) {
            uint16_t lo = (uint16_t)(u[q] & 0xffffu), hi = (uint16_t)(u[q] >> 16);
            if (DT == 2) {
                w[2 * q] = __uint_as_float((uint32_t)lo << 16);
                w[2 * q + 1] = __uint_as_float((uint32_t)hi << 16);
            } else {
                w[2 * q] = half_bits_to_float(lo);
                w[2 * q + 1] = half_bits_to_float(hi);
            }
        }
    }
}

// Raw 16-byte words of one lane's 8 weights (DT 1/2: one uint4 of 8 halves;
// DT 0: two uint4 of 4 floats), loaded ahead and decoded when used.
template <int DT>
struct Raw8 {
    uint4 a, b;
};
template <int DT>
__device__ __forceinline__ void raw8_load(const uint8_t* p, Raw8<DT>& r) {
    r.a = __ldg(reinterpret_cast<const uint4*>(p));
    if (DT == 0) r.b = __ldg(reinterpret_cast<const uint4*>(p) + 1);
}
template <int DT>
__device__ __forceinline__ void raw8_decode(const Raw8<DT>& r, float (&w)[8]) {
    if (DT == 0) {
        w[0] = __uint_as_float(r.a.x); w[1] = __uint_as_float(r.a.y);
        w[2] = __uint_as_float(r.a.z); w[3] = __uint_as_float(r.a.w);
        w[4] = __uint_as_float(r.b.x); w[5] = __uint_as_float(r.b.y);
        w[6] = __uint_as_float(r.b.z); w[7] = __uint_as_float(r.b.w);
    } else {
        const uint32_t u[4] = {r.a.x, r.a.y, r.a.z, r.a.w};
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const uint16_t lo = (uint16_t)(u[q] & 0xffffu), hi = (uint16_t)(u[q] >> 16);
            if (DT == 2) {
                w[2 * q] = __uint_as_float((uint32_t)lo << 16);
                w[2 * q + 1] = __uint_as_float((uint32_t)hi << 16);
            } else {
                w[2 * q] = half_bits_to_float(lo);
                w[2 * q + 1] = half_bits_to_float(hi);
            }
        }
    }
}

template <int DT, int TG>
__global__ void __launch_bounds__(128) fgemv_kernel(const uint8_t* __restrict__ W, int rows,
                                                    int cols, int steps,
                                                    const float* __restrict__ x, int M,
                                                    float* __restrict__ out, int vec_x) {
    constexpr int ES = DT == 0 ? 4 : 2;
    const int g = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    const int rows_pad = (rows + 31) / 32 * 32;
    if (g * kTileRows >= rows_pad) return;
    const int row = g * kTileRows + lane;
    const int full = cols / 8, rem = cols % 8;
    const uint8_t* base = W + ((size_t)g * steps * kTileRows + lane) * 8 * ES;
    for (int t0 = 0; t0 < M; t0 += TG) {
        float acc[TG][8];
#pragma unroll
        for (int j = 0; j < TG; j++)
#pragma unroll
            for (int l = 0; l < 8; l++) acc[j][l] = 0.0f;
#pragma unroll 2
        for (int i = 0; i < full; i++) {
            float w[8];
            load8<DT>(base + (size_t)i * kTileRows * 8 * ES, w);
#pragma unroll
            for (int j = 0; j < TG; j++) {
                const float* xp = x + (size_t)min(t0 + j, M - 1) * cols + 8 * i;
                float xv[8];
                if (vec_x) {
                    float4 a = __ldg(reinterpret_cast<const float4*>(xp));
                    float4 b = __ldg(reinterpret_cast<const float4*>(xp) + 1);
                    xv[0] = a.x; xv[1] = a.y; xv[2] = a.z; xv[3] = a.w;
                    xv[4] = b.x; xv[5] = b.y; xv[6] = b.z; xv[7] = b.w;
                } else {
#pragma unroll
                    for (int l = 0; l < 8; l++) xv[l] = __ldg(xp + l);
                }
#pragma unroll
                for (int l = 0; l < 8; l++) acc[j][l] = fadd(acc[j][l], fmul(w[l], xv[l]));
            }
        }
        float wt[8];
        if (rem) load8<DT>(base + (size_t)full * kTileRows * 8 * ES, wt);
#pragma unroll
        for (int j = 0; j < TG; j++) {
            if (t0 + j >= M) break;
            float tail = -0.0f;
            const float* xp = x + (size_t)(t0 + j) * cols + 8 * full;
            for (int l = 0; l < rem; l++) tail = fadd(tail, fmul(wt[l], __ldg(xp + l)));
            float a0 = fadd(fadd(acc[j][0], acc[j][4]), fadd(acc[j][1], acc[j][5]));
            float a1 = fadd(fadd(acc[j][2], acc[j][6]), fadd(acc[j][3], acc[j][7]));
            if (row < rows) out[(size_t)(t0 + j) * rows + row] = fadd(fadd(a0, a1), tail);
        }
    }
}

// Activation staging for the lane-major kernels: element c = (8 s + j) 8 + l
// (step s, accumulator lane l, j-th value of the lane's step) goes to
// shared-memory float (s << 6) | ((j >> 2) << 5) | (l << 2) | (j & 3), so
// lane l reads its step's 8 values as two 16-byte words, and the 8 lanes of a
// quarter-warp read 128 contiguous bytes.
__device__ __forceinline__ int lanes_x_slot(int c) {
    const int s = c >> 6, j = (c >> 3) & 7, l = c & 7;
    return (s << 6) | ((j >> 2) << 5) | (l << 2) | (j & 3);
}

// Float matvec for one activation row in the lane-major layout (cols a
// multiple of 64): in each group of 4 rows, for each group of 8 steps (a step
// = 8 columns), row rr's lane l holds its 8 consecutive step values
// contiguously -- offset ((q * S8 + s) * 4 + rr) * 64 + l * 8 + j elements for
// row 4q + rr, column 8 (8 s + j) + l. A warp covers 4 rows x 8 lanes: thread
// (rr, l) runs the reference's accumulator lane l of row 4q + rr
// (acc += w * x over the steps in order, quant.rs:152-160), and reduce()
// ((a0+a4)+(a1+a5))+((a2+a6)+(a3+a7)) (quant.rs:37-41) combines the 8
// threads; the (empty) tail adds -0. 8x the row parallelism of
// fgemv_kernel, with 512-byte warp loads.
// Single-row lane-major matvec: each warp's 4 rows are one contiguous
// region (S8 groups of [4 rows][64 columns]); the warp streams it through a
// ring of `ns` shared-memory stages of kLanesSB groups by bulk copies (lane 0
// issues every stage it can at once, then refills), so the whole region is
// in flight from the kernel's start -- under the RMSNorm chain when the norm
// is folded in. Shared memory after the staged activations:
// lanes_ring_bytes<DT>(ns) per warp, then ns mbarriers per warp.
constexpr int kLanesSB = 8;  // 64-column groups per stage

// Phase marks for timing probes built from this header; empty in the library.
#ifndef HALE_LANES_MARK
#define HALE_LANES_MARK(i)
#endif

template <int DT>
__host__ __device__ constexpr int lanes_stage_bytes() { return kLanesSB * 4 * 64 * (DT == 0 ? 4 : 2); }
template <int DT>
__host__ __device__ inline int lanes_ring_bytes(int ns) { return ns * lanes_stage_bytes<DT>(); }

// Issue stages [st0, st1) of this warp's region (lane 0 only).
template <int DT>
__device__ __forceinline__ void lanes_issue(const uint8_t* wq, int S8, uint8_t* ring, uint64_t* bars, int ns,
                                            int st0, int st1) {
    constexpr int ES = DT == 0 ? 4 : 2, STB = lanes_stage_bytes<DT>();
    for (int st = st0; st < st1; st++) {
        const int slot = st % ns, groups = min(kLanesSB, S8 - st * kLanesSB);
        const uint32_t bytes = (uint32_t)(groups * 4 * 64 * ES);
        mbar_arrive_expect_tx(&bars[slot], bytes);
        bulk_g2s(ring + (size_t)slot * STB, wq + (size_t)st * STB, bytes, &bars[slot]);
    }
}

// Starts this warp's weight stream (barrier init + the first ns stages).
// Returns false for warps past the last row (nothing issued).
template <int DT>
__device__ __forceinline__ bool lanes_start(const uint8_t* __restrict__ W, int rows, int cols, uint8_t* ring,
                                            uint64_t* bars, int ns) {
    constexpr int ES = DT == 0 ? 4 : 2;
    const int q = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (q * 4 >= rows) return false;
    const int S8 = cols / 64, nst = (S8 + kLanesSB - 1) / kLanesSB;
    if (lane == 0) {
        for (int i = 0; i < ns; i++) mbar_init(&bars[i], 1);
        fence_mbar_init();
        const uint8_t* wq = W + (size_t)q * 4 * cols * ES;
        // the first min(ns, nst) stages are contiguous in the region and in
        // the ring: one copy on the first stage's barrier
        const uint32_t first = (uint32_t)(min(ns * kLanesSB, S8) * 4 * 64 * ES);
        mbar_arrive_expect_tx(&bars[0], first);
        bulk_g2s(ring, wq, first, &bars[0]);
        if (nst > ns) {
            // the stages the ring cannot hold yet: into L2, for the refills
            const size_t done = (size_t)ns * lanes_stage_bytes<DT>(), total = (size_t)4 * cols * ES;
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(wq + done), "r"((uint32_t)(total - done))
                         : "memory");
        }
    }
    __syncwarp();
    return true;
}

// The matvec proper over activations already staged in s_x (lanes order),
// consuming the stream lanes_start began.
template <int DT>
__device__ __forceinline__ void lanes_gemv(const uint8_t* __restrict__ W, int rows, int cols, const float* s_x,
                                           float* __restrict__ out, uint8_t* ring, uint64_t* bars, int ns,
                                           uint32_t* err) {
    constexpr int ES = DT == 0 ? 4 : 2, STB = lanes_stage_bytes<DT>();
    const float4* s_x4 = reinterpret_cast<const float4*>(s_x);
    const int q = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    const int rr = lane >> 3, l = lane & 7, S8 = cols / 64, nst = (S8 + kLanesSB - 1) / kLanesSB;
    const uint8_t* wq = W + (size_t)q * 4 * cols * ES;
    float acc = 0.0f;
    uint32_t ph = 0;
    const int first = min(ns, nst);  // stages of the first copy (all on bars[0])
    for (int st = 0; st < nst; st++) {
        const int slot = st % ns;
        if (st == 0 || st >= first) {
            if (!__all_sync(0xffffffffu, mbar_wait(&bars[slot], (ph >> slot) & 1u, err))) {
                // copies still in flight get a bounded chance to land: the
                // first copy (st 0), else the refills of stages st ..
                if (st == 0) mbar_wait(&bars[0], 0u, nullptr, 400000000LL);
                for (int s2 = max(st, first); s2 < min(st + ns, nst); s2++)
                    mbar_wait(&bars[s2 % ns], (ph >> (s2 % ns)) & 1u, nullptr, 400000000LL);
                return;
            }
            ph ^= 1u << slot;
        }
        if (st == 0) HALE_LANES_MARK(5);
        if (st == 1) HALE_LANES_MARK(6);
        if (st == 3) HALE_LANES_MARK(7);
        const uint8_t* sb = ring + (size_t)slot * STB;
        const int groups = min(kLanesSB, S8 - st * kLanesSB);
        if (groups == kLanesSB) {
            // a full stage: every group's weights into registers first, so no
            // add waits on a shared-memory load
            Raw8<DT> rw[kLanesSB];
#pragma unroll
            for (int u = 0; u < kLanesSB; u++) {
                const uint4* src = reinterpret_cast<const uint4*>(sb + ((u * 4 + rr) * 64 + l * 8) * ES);
                rw[u].a = src[0];
                if (DT == 0) rw[u].b = src[1];
            }
#pragma unroll
            for (int u = 0; u < kLanesSB; u++) {
                const int s = st * kLanesSB + u;
                float w[8];
                raw8_decode<DT>(rw[u], w);
                const float4 xa = s_x4[(s << 4) + l], xb = s_x4[(s << 4) + 8 + l];
                acc = fadd(acc, fmul(w[0], xa.x)); acc = fadd(acc, fmul(w[1], xa.y));
                acc = fadd(acc, fmul(w[2], xa.z)); acc = fadd(acc, fmul(w[3], xa.w));
                acc = fadd(acc, fmul(w[4], xb.x)); acc = fadd(acc, fmul(w[5], xb.y));
                acc = fadd(acc, fmul(w[6], xb.z)); acc = fadd(acc, fmul(w[7], xb.w));
            }
        } else {
#pragma unroll
        for (int u = 0; u < kLanesSB; u++) {
            if (u < groups) {
                const int s = st * kLanesSB + u;
                Raw8<DT> rw;
                const uint4* src = reinterpret_cast<const uint4*>(sb + ((u * 4 + rr) * 64 + l * 8) * ES);
                rw.a = src[0];
                if (DT == 0) rw.b = src[1];
                float w[8];
                raw8_decode<DT>(rw, w);
                const float4 xa = s_x4[(s << 4) + l], xb = s_x4[(s << 4) + 8 + l];
                acc = fadd(acc, fmul(w[0], xa.x)); acc = fadd(acc, fmul(w[1], xa.y));
                acc = fadd(acc, fmul(w[2], xa.z)); acc = fadd(acc, fmul(w[3], xa.w));
                acc = fadd(acc, fmul(w[4], xb.x)); acc = fadd(acc, fmul(w[5], xb.y));
                acc = fadd(acc, fmul(w[6], xb.z)); acc = fadd(acc, fmul(w[7], xb.w));
            }
        }
        }
        __syncwarp();
        if (lane == 0 && st + ns < nst) {
            fence_proxy_async_smem();
            lanes_issue<DT>(wq, S8, ring, bars, ns, st + ns, st + ns + 1);
        }
    }
    const float s1 = fadd(acc, __shfl_down_sync(0xffffffffu, acc, 4, 8));
    const float p = fadd(s1, __shfl_down_sync(0xffffffffu, s1, 1, 8));
    const float r = fadd(p, __shfl_down_sync(0xffffffffu, p, 2, 8));
    const int row = q * 4 + rr;
    if (l == 0 && row < rows) out[row] = fadd(r, -0.0f);
}

// Shared memory of the single-row kernels: `act` bytes of staged
// activations (and norm scratch), then each warp's ring, then its barriers.
__host__ __device__ inline size_t lanes_smem(int act_bytes, int warps, int ring_bytes, int ns) {
    return (size_t)act_bytes + (size_t)warps * ring_bytes + (size_t)warps * ns * 8;
}

template <int DT>
__global__ void __launch_bounds__(256) fgemv_lanes_kernel(const uint8_t* __restrict__ W, int rows, int cols,
                                                          const float* __restrict__ x, float* __restrict__ out,
                                                          int ns, uint32_t* err) {
    extern __shared__ __align__(128) float s_x[];  // [cols], rings, barriers
    const int warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
    uint8_t* rings = reinterpret_cast<uint8_t*>(s_x) + (size_t)cols * 4;
    uint8_t* ring = rings + (size_t)warp * lanes_ring_bytes<DT>(ns);
    uint64_t* bars = reinterpret_cast<uint64_t*>(rings + (size_t)warps * lanes_ring_bytes<DT>(ns)) + warp * ns;
    const bool live = lanes_start<DT>(W, rows, cols, ring, bars, ns);
    if ((reinterpret_cast<uintptr_t>(x) & 15) == 0) {
        const float4* x4 = reinterpret_cast<const float4*>(x);
#pragma unroll 4
        for (int i = threadIdx.x; i < cols / 4; i += blockDim.x) {
            const float4 v = x4[i];
            s_x[lanes_x_slot(4 * i)] = v.x;
            s_x[lanes_x_slot(4 * i + 1)] = v.y;
            s_x[lanes_x_slot(4 * i + 2)] = v.z;
            s_x[lanes_x_slot(4 * i + 3)] = v.w;
        }
    } else {
        for (int i = threadIdx.x; i < cols; i += blockDim.x) s_x[lanes_x_slot(i)] = x[i];
    }
    __syncthreads();
    if (live) lanes_gemv<DT>(W, rows, cols, s_x, out, ring, bars, ns, err);
}

// RMSNorm folded into the matvec that consumes it (one activation row):
// every CTA forms v = x (+ delta), runs the norm's sum of squares (the
// reference's left-to-right chain, as rmsnorm_kernel) on one thread, and
// stages v * scale * w in lanes order; CTA 0 also writes the new residual v
// to x_out (x_out != x: other CTAs read x meanwhile). The warps' weight
// streams start before the chain. cols % 64 == 0, x / delta 16-byte aligned.
// float4 of x (and delta, norm weights) a thread of the norm kernel holds:
// cols <= 4 * kLanesNormVec * blockDim.x (4096 at 128 threads).
constexpr int kLanesNormVec = 8;

template <int DT>
__global__ void __launch_bounds__(256) fgemv_lanes_norm_kernel(const uint8_t* __restrict__ W, int rows, int cols,
                                                               const float* __restrict__ x,
                                                               const float* __restrict__ delta,
                                                               const float* __restrict__ nw, float eps,
                                                               float* __restrict__ x_out, float* __restrict__ out,
                                                               int ns, uint32_t* err) {
    extern __shared__ __align__(128) float s_x[];  // [cols] staged, [cols] v, rings, barriers
    float* s_v = s_x + cols;
    __shared__ float s_scale;
    const int warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
    uint8_t* rings = reinterpret_cast<uint8_t*>(s_x) + (size_t)cols * 8;
    uint8_t* ring = rings + (size_t)warp * lanes_ring_bytes<DT>(ns);
    uint64_t* bars = reinterpret_cast<uint64_t*>(rings + (size_t)warps * lanes_ring_bytes<DT>(ns)) + warp * ns;
    HALE_LANES_MARK(0);
    // x, delta and the norm weights are requested before the weight streams,
    // so they are not queued behind them (cols / 4 <= kLanesNormVec * blockDim.x)
    float4 xv[kLanesNormVec], dv[kLanesNormVec], wv[kLanesNormVec];
    const float4* x4 = reinterpret_cast<const float4*>(x);
    const float4* d4 = reinterpret_cast<const float4*>(delta);
    const float4* w4 = reinterpret_cast<const float4*>(nw);
#pragma unroll
    for (int j = 0; j < kLanesNormVec; j++) {
        const int i = threadIdx.x + j * blockDim.x;
        if (i < cols / 4) {
            xv[j] = x4[i];
            if (delta) dv[j] = d4[i];
            wv[j] = w4[i];
        }
    }
    const bool live = lanes_start<DT>(W, rows, cols, ring, bars, ns);
    float* s_w = s_x;  // the norm weights wait in s_x until the staging reads them
#pragma unroll
    for (int j = 0; j < kLanesNormVec; j++) {
        const int i = threadIdx.x + j * blockDim.x;
        if (i < cols / 4) {
            float4 v = xv[j];
            if (delta) {
                v = make_float4(fadd(v.x, dv[j].x), fadd(v.y, dv[j].y), fadd(v.z, dv[j].z), fadd(v.w, dv[j].w));
                if (blockIdx.x == 0) reinterpret_cast<float4*>(x_out)[i] = v;
            }
            reinterpret_cast<float4*>(s_v)[i] = v;
            reinterpret_cast<float4*>(s_w)[i] = wv[j];
        }
    }
    __syncthreads();
    HALE_LANES_MARK(1);
    if (threadIdx.x == 0) {
        // RmsNorm::forward (norm.rs): sum of squares left to right from -0
        // (the squares are independent of the chain)
        float s = -0.0f;
        const float4* v4 = reinterpret_cast<const float4*>(s_v);
#pragma unroll 8
        for (int i = 0; i < cols / 4; i++) {
            const float4 v = v4[i];
            s = fadd(fadd(fadd(fadd(s, fmul(v.x, v.x)), fmul(v.y, v.y)), fmul(v.z, v.z)), fmul(v.w, v.w));
        }
        s_scale = fdiv(1.0f, __fsqrt_rn(fadd(fdiv(s, (float)cols), eps)));
    }
    __syncthreads();
    HALE_LANES_MARK(2);
    const float scale = s_scale;
    // normed values into registers first: s_x holds the norm weights until
    // every thread has read its own
    float nv[4 * kLanesNormVec];
#pragma unroll
    for (int j = 0; j < 4 * kLanesNormVec; j++) {
        const int i = threadIdx.x + j * blockDim.x;
        if (i < cols) nv[j] = fmul(fmul(s_v[i], scale), s_w[i]);
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < 4 * kLanesNormVec; j++) {
        const int i = threadIdx.x + j * blockDim.x;
        if (i < cols) s_x[lanes_x_slot(i)] = nv[j];
    }
    __syncthreads();
    HALE_LANES_MARK(3);
    if (live) lanes_gemv<DT>(W, rows, cols, s_x, out, ring, bars, ns, err);
    HALE_LANES_MARK(4);
}

// The same matvec for n activation rows, NB per CTA (blockIdx.y = chunk):
// each weight step is loaded once and applied to the chunk's rows, staged in
// shared memory ([NB][cols], rows past n zero-filled and never stored). Per
// activation row the operations and their order are fgemv_lanes_kernel's, so
// every row's result has the same bits as a one-row launch.
template <int DT, int NB>
__global__ void __launch_bounds__(256) fgemv_lanes_batch_kernel(const uint8_t* __restrict__ W, int rows, int cols,
                                                                const float* __restrict__ x, int n,
                                                                float* __restrict__ out) {
    extern __shared__ __align__(16) float s_xb[];  // [NB][cols], each row in lanes_x_slot order
    constexpr int ES = DT == 0 ? 4 : 2;
    const int b0 = blockIdx.y * NB;
    const int nb = min(NB, n - b0);
    const bool x16 = (reinterpret_cast<uintptr_t>(x) & 15) == 0;  // cols % 64 == 0: every row aligned
#pragma unroll 1
    for (int b = 0; b < NB; b++) {
        const float* xr = x + (size_t)(b0 + b) * cols;
        float* dst = s_xb + b * cols;
        if (x16) {
            const float4* x4 = reinterpret_cast<const float4*>(xr);
#pragma unroll 4
            for (int i = threadIdx.x; i < cols / 4; i += blockDim.x) {
                const float4 v = b < nb ? x4[i] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                dst[lanes_x_slot(4 * i)] = v.x;
                dst[lanes_x_slot(4 * i + 1)] = v.y;
                dst[lanes_x_slot(4 * i + 2)] = v.z;
                dst[lanes_x_slot(4 * i + 3)] = v.w;
            }
        } else {
            for (int c = threadIdx.x; c < cols; c += blockDim.x) dst[lanes_x_slot(c)] = b < nb ? xr[c] : 0.0f;
        }
    }
    __syncthreads();
    const int q = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (q * 4 >= rows) return;
    const int rr = lane >> 3, l = lane & 7, S8 = cols / 64;
    const uint8_t* base = W + (((size_t)q * S8 * 4 + rr) * 64 + l * 8) * ES;
    const float4* s_x4 = reinterpret_cast<const float4*>(s_xb);
    const int c4 = cols >> 2;  // float4 per staged row
    float acc[NB];
#pragma unroll
    for (int b = 0; b < NB; b++) acc[b] = 0.0f;
#pragma unroll 2
    for (int s = 0; s < S8; s++) {
        float w[8];
        load8<DT>(base + (size_t)s * 4 * 64 * ES, w);
#pragma unroll
        for (int b = 0; b < NB; b++) {
            const float4 xa = s_x4[b * c4 + (s << 4) + l], xb = s_x4[b * c4 + (s << 4) + 8 + l];
            float a = acc[b];
            a = fadd(a, fmul(w[0], xa.x)); a = fadd(a, fmul(w[1], xa.y));
            a = fadd(a, fmul(w[2], xa.z)); a = fadd(a, fmul(w[3], xa.w));
            a = fadd(a, fmul(w[4], xb.x)); a = fadd(a, fmul(w[5], xb.y));
            a = fadd(a, fmul(w[6], xb.z)); a = fadd(a, fmul(w[7], xb.w));
            acc[b] = a;
        }
    }
    const int row = q * 4 + rr;
#pragma unroll
    for (int b = 0; b < NB; b++) {
        const float s1 = fadd(acc[b], __shfl_down_sync(0xffffffffu, acc[b], 4, 8));
        const float p = fadd(s1, __shfl_down_sync(0xffffffffu, s1, 1, 8));
        const float r = fadd(p, __shfl_down_sync(0xffffffffu, p, 2, 8));
        if (l == 0 && row < rows && b < nb) out[(size_t)(b0 + b) * rows + row] = fadd(r, -0.0f);
    }
}

// Row-major float rows -> the lane-major layout (rows padded to 4 with 0).
template <int ES>
__global__ void repack_lanes_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int rows,
                                    int rows_pad, int cols) {
    const size_t n = (size_t)rows_pad * cols;
    const int S8 = cols / 64;
    for (size_t o = blockIdx.x * (size_t)blockDim.x + threadIdx.x; o < n; o += (size_t)gridDim.x * blockDim.x) {
        const int j = (int)(o & 7), l = (int)((o >> 3) & 7), rr = (int)((o >> 6) & 3);
        const size_t qs = o >> 8;
        const int s = (int)(qs % S8), q = (int)(qs / S8);
        const int r = q * 4 + rr, c = 8 * (8 * s + j) + l;
        uint8_t* d = dst + o * ES;
        if (r < rows) {
            const uint8_t* sp = src + ((size_t)r * cols + c) * ES;
            for (int b = 0; b < ES; b++) d[b] = sp[b];
        } else {
            for (int b = 0; b < ES; b++) d[b] = 0;
        }
    }
}

// ---------------------------------------------------------------------------
// Sampler (src/generate/sampler.rs): one CTA of 1024 threads per row.
//   temperature <= 0: argmax, first maximum wins (activation.rs:24-32).
//   otherwise (sampler.rs:80-123): the top_k best logits (ties: lower index
//   first), sorted best-first; e_i = exp((l_i - max) / T) summed in order;
//   nucleus cut at the first prefix whose running mass reaches top_p; draw
//   r = next_f32() * kept_total and walk down. xorshift64* state per row.
// Repetition penalty (extension) is applied to each seen id first.
// ---------------------------------------------------------------------------
constexpr int kSampleThreads = 1024;
constexpr int kSampleMaxK = 1024;

struct SampleArgs {
    const float* logits;
    int V;
    float temperature, top_p, penalty;
    int top_k;  // already clamped: 1..min(V, kSampleMaxK), or V when V <= kSampleMaxK
    uint64_t* rng;
    const int32_t* seen;
    int n_seen;
    int32_t* out;
};

__device__ __forceinline__ float penalized(const float* lg, const uint32_t* bits, int i, float p) {
    float l = lg[i];
    if (bits && (bits[i >> 5] >> (i & 31)) & 1u) l = l > 0.0f ? fdiv(l, p) : fmul(l, p);
    return l;
}

__global__ void __launch_bounds__(kSampleThreads) sample_kernel(SampleArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    // layout: [penalty bitmap (V/32 words, when used)] ...
    __shared__ unsigned s_hist[256];
    __shared__ int s_ctl[8];
    __shared__ unsigned long long s_key[kSampleMaxK];
    __shared__ float s_val[kSampleMaxK];
    const int row = blockIdx.x, tid = threadIdx.x, V = a.V;
    const float* lg = a.logits + (size_t)row * V;
    uint32_t* bits = nullptr;
    if (a.seen && a.n_seen > 0 && a.penalty != 1.0f) {
        bits = reinterpret_cast<uint32_t*>(smem);
        for (int i = tid; i < (V + 31) / 32; i += blockDim.x) bits[i] = 0u;
        __syncthreads();
        for (int i = tid; i < a.n_seen; i += blockDim.x) {
            int id = a.seen[(size_t)row * a.n_seen + i];
            if (id >= 0 && id < V) atomicOr(&bits[id >> 5], 1u << (id & 31));
        }
    }
    __syncthreads();

    if (a.temperature <= 0.0f) {
        // argmax: strict '>' scan from index 0; NaN never wins, and a NaN at
        // index 0 is never beaten.
        float bv = -__int_as_float(0x7f800000);
        int bi = INT_MAX;
        for (int i = tid; i < V; i += blockDim.x) {
            float v = penalized(lg, bits, i, a.penalty);
            if (v == v && (bi == INT_MAX || v > bv)) { bv = v; bi = i; }
        }
        // block reduce: larger value, then lower index
        __shared__ float r_v[32];
        __shared__ int r_i[32];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (oi != INT_MAX && (bi == INT_MAX || ov > bv || (ov == bv && oi < bi))) { bv = ov; bi = oi; }
        }
        if ((tid & 31) == 0) { r_v[tid >> 5] = bv; r_i[tid >> 5] = bi; }
        __syncthreads();
        if (tid < 32) {
            bv = r_v[tid];
            bi = r_i[tid];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (oi != INT_MAX && (bi == INT_MAX || ov > bv || (ov == bv && oi < bi))) { bv = ov; bi = oi; }
            }
            if (tid == 0) {
                float v0 = penalized(lg, bits, 0, a.penalty);
                a.out[row] = (v0 != v0 || bi == INT_MAX) ? 0 : bi;
            }
        }
        return;
    }

    // ---- candidates: the top_k by (key desc, index asc) ---------------------
    const int K = a.top_k;
    // Radix-select the K-th largest ordered key (uk = key ^ 0x80000000).
    unsigned prefix = 0u, pmask = 0u;
    int need = K;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = tid; i < 256; i += blockDim.x) s_hist[i] = 0u;
        __syncthreads();
        for (int i = tid; i < V; i += blockDim.x) {
            unsigned uk = (unsigned)total_key(penalized(lg, bits, i, a.penalty)) ^ 0x80000000u;
            if ((uk & pmask) == prefix) atomicAdd(&s_hist[(uk >> shift) & 255u], 1u);
        }
        __syncthreads();
        if (tid == 0) {
            int acc = 0, d = 255;
            for (; d > 0; d--) {
                if (acc + (int)s_hist[d] >= need) break;
                acc += (int)s_hist[d];
            }
            s_ctl[0] = d;
            s_ctl[1] = need - acc;
        }
        __syncthreads();
        prefix |= (unsigned)s_ctl[0] << shift;
        pmask |= 255u << shift;
        need = s_ctl[1];
        __syncthreads();
    }
    // Threshold key `prefix`; take every key above it and the `need` lowest
    // indices equal to it. Contiguous chunks per thread keep index order.
    const int chunk = (V + blockDim.x - 1) / blockDim.x;
    const int lo = tid * chunk, hi = min(V, lo + chunk);
    int n_gt = 0, n_eq = 0;
    for (int i = lo; i < hi; i++) {
        unsigned uk = (unsigned)total_key(penalized(lg, bits, i, a.penalty)) ^ 0x80000000u;
        n_gt += uk > prefix;
        n_eq += uk == prefix;
    }
    // exclusive scans of n_gt and n_eq over threads (in index order)
    __shared__ int w_gt[32], w_eq[32];
    int lane = tid & 31, warp = tid >> 5;
    int sg = n_gt, se = n_eq;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int tg = __shfl_up_sync(0xffffffffu, sg, o), te = __shfl_up_sync(0xffffffffu, se, o);
        if (lane >= o) { sg += tg; se += te; }
    }
    if (lane == 31) { w_gt[warp] = sg; w_eq[warp] = se; }
    __syncthreads();
    if (tid == 0) {
        int cg = 0, ce = 0;
        for (int w = 0; w < (int)(blockDim.x >> 5); w++) {
            int tg = w_gt[w], te = w_eq[w];
            w_gt[w] = cg; w_eq[w] = ce;
            cg += tg; ce += te;
        }
        s_ctl[2] = cg;  // total strictly greater
    }
    __syncthreads();
    int pos_gt = w_gt[warp] + sg - n_gt, pos_eq = w_eq[warp] + se - n_eq;
    const int total_gt = s_ctl[2];
    for (int i = lo; i < hi; i++) {
        float v = penalized(lg, bits, i, a.penalty);
        unsigned uk = (unsigned)total_key(v) ^ 0x80000000u;
        int slot = -1;
        if (uk > prefix) slot = pos_gt++;
        else if (uk == prefix) { if (pos_eq < need) slot = total_gt + pos_eq; pos_eq++; }
        if (slot >= 0 && slot < K) {
            // sort key: ordered key high, inverted index low -> descending
            s_key[slot] = ((unsigned long long)uk << 32) | (unsigned)(0x7fffffff - i);
            s_val[slot] = v;
        }
    }
    // pad to a power of two for the bitonic sort
    int P = 1;
    while (P < K) P <<= 1;
    for (int i = K + tid; i < P; i += blockDim.x) { s_key[i] = 0ull; s_val[i] = 0.0f; }
    __syncthreads();
    // bitonic sort, descending by s_key
    for (int size = 2; size <= P; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = tid; i < P; i += blockDim.x) {
                int j = i ^ stride;
                if (j > i) {
                    bool desc = (i & size) == 0;
                    unsigned long long ki = s_key[i], kj = s_key[j];
                    if (desc ? (ki < kj) : (ki > kj)) {
                        s_key[i] = kj; s_key[j] = ki;
                        float t = s_val[i]; s_val[i] = s_val[j]; s_val[j] = t;
                    }
                }
            }
            __syncthreads();
        }
    }
    // softmax with temperature over the survivors (sampler.rs:96-101)
    const float mx = s_val[0];
    for (int i = tid; i < K; i += blockDim.x) s_val[i] = hale_expf(fdiv(fsub(s_val[i], mx), a.temperature));
    __syncthreads();
    if (tid == 0) {
        float total = 0.0f;
        for (int i = 0; i < K; i++) total = fadd(total, s_val[i]);
        float mass = 0.0f;
        int keep = K;
        for (int i = 0; i < K; i++) {
            mass = fadd(mass, fdiv(s_val[i], total));
            if (mass >= a.top_p) { keep = i + 1; break; }
        }
        float kept = -0.0f;
        for (int i = 0; i < keep; i++) kept = fadd(kept, s_val[i]);
        uint64_t st = a.rng[row];
        st ^= st >> 12;
        st ^= st << 25;
        st ^= st >> 27;
        a.rng[row] = st;
        uint64_t u = st * 0x2545F4914F6CDD1DULL;
        float r = fmul(fdiv((float)(u >> 40), 16777216.0f), kept);
        int pick = 0x7fffffff - (int)(unsigned)(s_key[keep - 1] & 0xffffffffull);
        for (int i = 0; i < keep; i++) {
            r = fsub(r, s_val[i]);
            if (r <= 0.0f) {
                pick = 0x7fffffff - (int)(unsigned)(s_key[i] & 0xffffffffull);
                break;
            }
        }
        a.out[row] = pick;
    }
}

// ---------------------------------------------------------------------------
// Sampling with more than kSampleMaxK candidates (top_k = 0 keeps the whole
// vocabulary, sampler.rs:84-93): every candidate is ranked by a unique 64-bit
// key -- the logit's total-order key, then the inverted index, so the
// descending key order is the reference's (logit desc, index asc) order --
// and the keys of each row are sorted by a segmented radix sort. The
// reference's sums then run in that order, one thread per row, exactly:
// softmax total over the K best, nucleus mass, kept mass, the draw.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float key_to_float(unsigned long long key) {
    const int32_t k = (int32_t)((uint32_t)(key >> 32) ^ 0x80000000u);
    return __int_as_float(k >= 0 ? k : (k ^ 0x7fffffff));
}
__device__ __forceinline__ int key_to_index(unsigned long long key) {
    return 0x7fffffff - (int)(uint32_t)(key & 0xffffffffull);
}

// keys[row * V + i]; offsets[row] = row * V (segment starts, offsets[B] = B * V).
__global__ void __launch_bounds__(1024) sample_keys_kernel(SampleArgs a, unsigned long long* __restrict__ keys,
                                                           int* __restrict__ offsets) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int row = blockIdx.x, tid = threadIdx.x, V = a.V;
    const float* lg = a.logits + (size_t)row * V;
    uint32_t* bits = nullptr;
    if (a.seen && a.n_seen > 0 && a.penalty != 1.0f) {
        bits = reinterpret_cast<uint32_t*>(smem);
        for (int i = tid; i < (V + 31) / 32; i += blockDim.x) bits[i] = 0u;
        __syncthreads();
        for (int i = tid; i < a.n_seen; i += blockDim.x) {
            const int id = a.seen[(size_t)row * a.n_seen + i];
            if (id >= 0 && id < V) atomicOr(&bits[id >> 5], 1u << (id & 31));
        }
    }
    __syncthreads();
    for (int i = tid; i < V; i += blockDim.x) {
        const unsigned uk = (unsigned)total_key(penalized(lg, bits, i, a.penalty)) ^ 0x80000000u;
        keys[(size_t)row * V + i] = ((unsigned long long)uk << 32) | (unsigned)(0x7fffffff - i);
    }
    if (tid == 0) {
        offsets[row] = row * V;
        if (row == gridDim.x - 1) offsets[row + 1] = (row + 1) * V;
    }
}

// e[row * V + j] = exp((v_j - v_0) / T) over the K best (sampler.rs:96-101).
__global__ void sample_exp_kernel(const unsigned long long* __restrict__ sorted, int V, int K, float temperature,
                                  float* __restrict__ e) {
    const int row = blockIdx.y, j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= K) return;
    const unsigned long long* ks = sorted + (size_t)row * V;
    const float mx = key_to_float(__ldg(ks));
    e[(size_t)row * V + j] = hale_expf(fdiv(fsub(key_to_float(__ldg(ks + j)), mx), temperature));
}

constexpr int kSampleChunk = 4096;

// Streams x[0 .. n) through shared memory in chunks (threads 1.. load the
// next chunk while thread 0 folds the current one): thread 0 calls
// step(value, j) in order until it returns false. All threads call this.
template <class Step>
__device__ void sample_scan(const float* __restrict__ x, int n, float (*buf)[kSampleChunk], Step step) {
    const int tid = threadIdx.x;
    // go[i & 1]: whether chunk i is still wanted; written by thread 0 one
    // chunk ahead, read by everyone after the barrier that follows
    __shared__ int s_go[2];
    if (tid == 0) s_go[0] = 1;
    for (int j = tid; j < min(n, kSampleChunk); j += blockDim.x) buf[0][j] = __ldcg(x + j);
    __syncthreads();
    for (int c0 = 0, it = 0; c0 < n; c0 += kSampleChunk, it++) {
        if (!s_go[it & 1]) break;
        const int c1 = c0 + kSampleChunk, ci = it & 1;
        if (tid == 0) {
            int go = 1;
            const int m = min(kSampleChunk, n - c0);
            for (int j = 0; j < m; j++)
                if (!step(buf[ci][j], c0 + j)) {
                    go = 0;
                    break;
                }
            s_go[(it + 1) & 1] = go;
        } else {
            for (int j = c1 + tid - 1; j < min(n, c1 + kSampleChunk); j += blockDim.x - 1)
                buf[ci ^ 1][j - c1] = __ldcg(x + j);
        }
        __syncthreads();
    }
    __syncthreads();
}

// One CTA per row: the reference's tail of TopPSampler::sample
// (sampler.rs:96-123) over the sorted candidates, in its order.
__global__ void __launch_bounds__(1024) sample_tail_kernel(const unsigned long long* __restrict__ sorted,
                                                           float* __restrict__ e, float* __restrict__ q, int V,
                                                           int K, float top_p, uint64_t* __restrict__ rng,
                                                           int32_t* __restrict__ out) {
    __shared__ float buf[2][kSampleChunk];
    __shared__ float s_total;
    __shared__ int s_keep;
    const int row = blockIdx.x, tid = threadIdx.x;
    const float* er = e + (size_t)row * V;
    float* qr = q + (size_t)row * V;
    // total: sequential over the K best; once a term leaves the sum unchanged
    // every later (smaller or equal) one does too
    float total = 0.0f;
    sample_scan(er, K, buf, [&](float v, int) {
        const float t = fadd(total, v);
        if (t == total) return false;
        total = t;
        return true;
    });
    if (tid == 0) s_total = total;
    __syncthreads();
    total = s_total;
    for (int j = tid; j < K; j += blockDim.x) qr[j] = fdiv(__ldcg(er + j), total);
    __syncthreads();
    // nucleus cut (sampler.rs:103-112)
    float mass = 0.0f;
    int keep = K;
    sample_scan(qr, K, buf, [&](float v, int j) {
        mass = fadd(mass, v);
        if (mass >= top_p) {
            keep = j + 1;
            return false;
        }
        return true;
    });
    if (tid == 0) s_keep = keep;
    __syncthreads();
    keep = s_keep;
    float kept = -0.0f;
    sample_scan(er, keep, buf, [&](float v, int) {
        kept = fadd(kept, v);
        return true;
    });
    // the draw (sampler.rs:114-122, XorShift64 :128-146)
    __shared__ float s_r;
    if (tid == 0) {
        uint64_t st = rng[row];
        st ^= st >> 12;
        st ^= st << 25;
        st ^= st >> 27;
        rng[row] = st;
        const uint64_t u = st * 0x2545F4914F6CDD1DULL;
        s_r = fmul(fdiv((float)(u >> 40), 16777216.0f), kept);
    }
    __syncthreads();
    float r = s_r;
    int pick = keep - 1;
    sample_scan(er, keep, buf, [&](float v, int j) {
        r = fsub(r, v);
        if (r <= 0.0f) {
            pick = j;
            return false;
        }
        return true;
    });
    if (tid == 0) out[row] = key_to_index(__ldg(sorted + (size_t)row * V + pick));
}

}  // namespace hale
