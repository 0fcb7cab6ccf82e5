// gemv.cu — grouped GEMV for decode-sized groups (work items of at most kGemvMaxRows token
// rows), bound by HBM bandwidth.  Same work items and tile format as the tensor-core path.
//
// CTA = 128 threads on one (group, 128-row block, <= 8 token rows) item.  Thread 0 streams
// the item's weight tiles along K through a kRing-slot ring of 1-D bulk copies
// (cp.async.bulk, mbarrier transaction counts), so every CTA keeps kRing tiles (Q8_0:
// 8 x 8.7 KB) in flight - the depth HBM needs.  Each thread owns two (row, GGUF block)
// entries of every tile: it dequantises them exactly in fp32 ((q - 8) or q via the 2^23
// magic number), accumulates each block's dot product with the fp16 activations in fp32 and
// scales it by the block's d once.  gate_up items end with the SwiGLU (silu of rows 0..63
// times rows 64..127) and write fp16; down items write fp32.
#include "common.cuh"
#include "kernels.h"

namespace hymoe {

namespace {

constexpr int kGemvThreads = 128;
constexpr int kRing = 8;

template <int WT>
struct RawBlock;

template <>
struct RawBlock<W_Q4_0> {
    uint4 q;
    float d;
    __device__ __forceinline__ void load(const uint8_t* tile, int e) {
        d = __half2float(*reinterpret_cast<const __half*>(tile + 2 * e));
        q = *reinterpret_cast<const uint4*>(tile + 512 + 16 * e);
    }
    __device__ __forceinline__ void values(float (&v)[32]) const {
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const uint32_t byte = (w[i >> 2] >> (8 * (i & 3))) & 0xFFu;
            v[i] = __int_as_float(0x4B000000 | (byte & 0xFu)) - 8388616.0f;
            v[i + 16] = __int_as_float(0x4B000000 | (byte >> 4)) - 8388616.0f;
        }
    }
};

template <>
struct RawBlock<W_Q8_0> {
    uint4 q0, q1;
    float d;
    __device__ __forceinline__ void load(const uint8_t* tile, int e) {
        d = __half2float(*reinterpret_cast<const __half*>(tile + 2 * e));
        q0 = *reinterpret_cast<const uint4*>(tile + 512 + 32 * e);
        q1 = *reinterpret_cast<const uint4*>(tile + 512 + 32 * e + 16);
    }
    __device__ __forceinline__ void values(float (&v)[32]) const {
        const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const uint32_t byte = (w[i >> 2] >> (8 * (i & 3))) & 0xFFu;
            v[i] = __int_as_float(0x4B000000 | (byte ^ 0x80u)) - 8388736.0f;
        }
    }
};

template <>
struct RawBlock<W_F16> {
    uint4 h[4];
    float d;
    __device__ __forceinline__ void load(const uint8_t* tile, int e) {
        const int r = e >> 1, b = e & 1;
        const uint4* p = reinterpret_cast<const uint4*>(tile + r * 128 + b * 64);
#pragma unroll
        for (int i = 0; i < 4; ++i) h[i] = p[i];
        d = 1.0f;
    }
    __device__ __forceinline__ void values(float (&v)[32]) const {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const __half2* hp = reinterpret_cast<const __half2*>(&h[i]);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float2 f = __half22float2(hp[j]);
                v[8 * i + 2 * j] = f.x;
                v[8 * i + 2 * j + 1] = f.y;
            }
        }
    }
};

template <int WT>
__global__ __launch_bounds__(kGemvThreads) void gemv_kernel(const int4* __restrict__ items,
                                                            const int* __restrict__ n_items,
                                                            const uint8_t* const* __restrict__ wtiles,
                                                            int n_ks, int glu,
                                                            const __half* __restrict__ act, int act_ld,
                                                            void* __restrict__ out, int out_ld,
                                                            int* err) {
    constexpr int TB = tile_bytes(WT);
    extern __shared__ __align__(128) uint8_t gsm[];
    uint8_t* ring = gsm;                                            // kRing x TB
    uint64_t* full = reinterpret_cast<uint64_t*>(ring + kRing * TB);
    float* G = reinterpret_cast<float*>(full + kRing);             // [128][kGemvMaxRows + 1]
    if (static_cast<int>(blockIdx.x) >= *n_items) return;
    const int4 it = items[blockIdx.x];
    const int g = it.x, rb = it.y, row0 = it.z, nrows = min(it.w, kGemvMaxRows);
    const int tid = threadIdx.x;
    const uint8_t* wt = wtiles[g] + static_cast<size_t>(rb) * n_ks * TB;

    if (tid == 0) {
        for (int s = 0; s < kRing; ++s) mbar_init(&full[s], 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0)
        for (int s = 0; s < kRing && s < n_ks; ++s) {
            mbar_arrive_expect_tx(&full[s], TB);
            bulk_load(ring + s * TB, wt + static_cast<size_t>(s) * TB, TB, &full[s]);
        }

    float acc[2][kGemvMaxRows];
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int n = 0; n < kGemvMaxRows; ++n) acc[h][n] = 0.f;

    // `ok` stays uniform across the CTA (__syncthreads_and), so every thread takes the same
    // path; after a failed (timed-out) wait no further copies are issued and the copies
    // still in flight, tiles [fail_ks, issued), are waited for (bounded) before returning.
    bool ok = true;
    int issued = min(kRing, n_ks), fail_ks = -1;
    for (int ks = 0; ks < n_ks; ++ks) {
        const int s = ks % kRing;
        const bool got = ok && mbar_wait(&full[s], (ks / kRing) & 1, err, DEVERR_TIMEOUT_DEQUANT);
        if (got) {
            const uint8_t* tile = ring + s * TB;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int e = tid + h * kGemvThreads;  // entry (row e >> 1, block e & 1)
                RawBlock<WT> blk;
                blk.load(tile, e);
                float v[32];
                blk.values(v);
                const int k0 = ks * kTileK + (e & 1) * 32;
#pragma unroll
                for (int n = 0; n < kGemvMaxRows; ++n) {
                    if (n >= nrows) break;
                    const uint4* xr = reinterpret_cast<const uint4*>(act + static_cast<size_t>(row0 + n) * act_ld + k0);
                    float sum = 0.f;
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const uint4 xv = __ldg(xr + c);
                        const __half2* hp = reinterpret_cast<const __half2*>(&xv);
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const float2 f = __half22float2(hp[j]);
                            sum = fmaf(v[8 * c + 2 * j], f.x, sum);
                            sum = fmaf(v[8 * c + 2 * j + 1], f.y, sum);
                        }
                    }
                    acc[h][n] = fmaf(blk.d, sum, acc[h][n]);
                }
            }
        }
        const bool was_ok = ok;
        ok = __syncthreads_and(got) != 0;  // also: every thread is done with slot s
        if (was_ok && !ok) fail_ks = ks;
        if (ok && ks + kRing < n_ks) {
            if (tid == 0) {
                mbar_arrive_expect_tx(&full[s], TB);
                bulk_load(ring + s * TB, wt + static_cast<size_t>(ks + kRing) * TB, TB, &full[s]);
            }
            issued = ks + kRing + 1;
        }
    }
    if (!ok) {
        if (tid == 0)
            for (int t = fail_ks; t < issued; ++t) mbar_drain(&full[t % kRing], (t / kRing) & 1);
        __syncthreads();
        return;
    }
    // Entries 2r and 2r+1 (blocks 0 and 1 of row r) sit in adjacent lanes for h = 0, 1.
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int n = 0; n < kGemvMaxRows; ++n) acc[h][n] += __shfl_xor_sync(0xffffffffu, acc[h][n], 1);
    if ((tid & 1) == 0)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int r = (tid + h * kGemvThreads) >> 1;
#pragma unroll
            for (int n = 0; n < kGemvMaxRows; ++n) G[r * (kGemvMaxRows + 1) + n] = acc[h][n];
        }
    __syncthreads();
    if (glu) {
        __half* o = static_cast<__half*>(out);
        for (int i = tid; i < kGluHalf * nrows; i += kGemvThreads) {
            const int j = i % kGluHalf, n = i / kGluHalf;
            o[static_cast<size_t>(row0 + n) * out_ld + rb * kGluHalf + j] =
                __float2half_rn(silu_mul(G[j * (kGemvMaxRows + 1) + n],
                                         G[(kGluHalf + j) * (kGemvMaxRows + 1) + n]));
        }
    } else {
        float* o = static_cast<float*>(out);
        for (int i = tid; i < kTileRows * nrows; i += kGemvThreads) {
            const int r = i % kTileRows, n = i / kTileRows;
            o[static_cast<size_t>(row0 + n) * out_ld + rb * kTileRows + r] = G[r * (kGemvMaxRows + 1) + n];
        }
    }
}

template <int WT>
cudaError_t launch_t(const int4* items, const int* n_items, int max_items,
                     const uint8_t* const* wtiles, int n_ks, int glu, const __half* act, int act_ld,
                     void* out, int out_ld, int* err, cudaStream_t st) {
    const size_t smem = static_cast<size_t>(kRing) * tile_bytes(WT) + kRing * 8 +
                        sizeof(float) * kTileRows * (kGemvMaxRows + 1);
    cudaError_t e = cudaFuncSetAttribute(gemv_kernel<WT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    gemv_kernel<WT><<<max_items, kGemvThreads, smem, st>>>(items, n_items, wtiles, n_ks, glu, act,
                                                           act_ld, out, out_ld, err);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gemv(const int4* items, const int* n_items, int max_items,
                        const uint8_t* const* wtiles, int wtype, int n_ks, int glu,
                        const __half* act, int act_ld, void* out, int out_ld, int* err,
                        cudaStream_t st) {
    if (max_items <= 0) return cudaSuccess;
    switch (wtype) {
        case W_Q4_0: return launch_t<W_Q4_0>(items, n_items, max_items, wtiles, n_ks, glu, act, act_ld, out, out_ld, err, st);
        case W_Q8_0: return launch_t<W_Q8_0>(items, n_items, max_items, wtiles, n_ks, glu, act, act_ld, out, out_ld, err, st);
        default: return launch_t<W_F16>(items, n_items, max_items, wtiles, n_ks, glu, act, act_ld, out, out_ld, err, st);
    }
}

}  // namespace hymoe
