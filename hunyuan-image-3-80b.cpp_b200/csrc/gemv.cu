// gemv.cu — grouped GEMV for decode-sized groups (at most kGemvMaxRows token rows per
// expert), HBM-bound.  Same work items and tile format as the tensor-core path.
//
// CTA = 256 threads on one (group, 128-row block) work item; thread (r, b) owns tile row r
// and GGUF block b of every 64-column tile along K.  Quantised weights are dequantised to
// fp32 exactly ((q - 8) or q via the 2^23 magic-number trick), each block's dot product is
// accumulated in fp32 and scaled by the block's d once.  The next tile's bytes are loaded
// before the current tile is consumed (register double buffering) so every thread keeps
// loads in flight.  gate_up work items end with the SwiGLU (silu of rows 0..63 times
// rows 64..127) and write fp16; down work items write fp32.
#include "common.cuh"
#include "kernels.h"

namespace hymoe {

namespace {

template <int WT>
struct RawBlock;

template <>
struct RawBlock<W_Q4_0> {
    uint4 q;
    uint16_t d;
    __device__ __forceinline__ void load(const uint8_t* tile, int e) {
        d = *reinterpret_cast<const uint16_t*>(tile + 2 * e);
        q = __ldg(reinterpret_cast<const uint4*>(tile + 512 + 16 * e));
    }
    // v[j] = (q_j - 8), element j of the block
    __device__ __forceinline__ void values(float (&v)[32]) const {
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const uint32_t byte = (w[i >> 2] >> (8 * (i & 3))) & 0xFFu;
            v[i] = __int_as_float(0x4B000000 | (byte & 0xFu)) - 8388616.0f;
            v[i + 16] = __int_as_float(0x4B000000 | (byte >> 4)) - 8388616.0f;
        }
    }
    __device__ __forceinline__ float scale() const { return __half2float(__ushort_as_half(d)); }
};

template <>
struct RawBlock<W_Q8_0> {
    uint4 q0, q1;
    uint16_t d;
    __device__ __forceinline__ void load(const uint8_t* tile, int e) {
        d = *reinterpret_cast<const uint16_t*>(tile + 2 * e);
        q0 = __ldg(reinterpret_cast<const uint4*>(tile + 512 + 32 * e));
        q1 = __ldg(reinterpret_cast<const uint4*>(tile + 512 + 32 * e + 16));
    }
    __device__ __forceinline__ void values(float (&v)[32]) const {
        const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const uint32_t byte = (w[i >> 2] >> (8 * (i & 3))) & 0xFFu;
            v[i] = __int_as_float(0x4B000000 | (byte ^ 0x80u)) - 8388736.0f;
        }
    }
    __device__ __forceinline__ float scale() const { return __half2float(__ushort_as_half(d)); }
};

template <>
struct RawBlock<W_F16> {
    uint4 h[4];
    __device__ __forceinline__ void load(const uint8_t* tile, int e) {
        const int r = e >> 1, b = e & 1;
        const uint4* p = reinterpret_cast<const uint4*>(tile + r * 128 + b * 64);
#pragma unroll
        for (int i = 0; i < 4; ++i) h[i] = __ldg(p + i);
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
    __device__ __forceinline__ float scale() const { return 1.0f; }
};

template <int WT>
__global__ __launch_bounds__(256) void gemv_kernel(const int4* __restrict__ items,
                                                   const int* __restrict__ n_items,
                                                   const uint8_t* const* __restrict__ wtiles,
                                                   int n_ks, int glu,
                                                   const __half* __restrict__ act, int act_ld,
                                                   void* __restrict__ out, int out_ld) {
    constexpr int TB = tile_bytes(WT);
    if (static_cast<int>(blockIdx.x) >= *n_items) return;
    const int4 it = items[blockIdx.x];
    const int g = it.x, rb = it.y, row0 = it.z, nrows = min(it.w, kGemvMaxRows);
    const int e = threadIdx.x, r = e >> 1, b = e & 1;
    const uint8_t* wt = wtiles[g] + static_cast<size_t>(rb) * n_ks * TB;

    float acc[kGemvMaxRows];
#pragma unroll
    for (int n = 0; n < kGemvMaxRows; ++n) acc[n] = 0.f;

    RawBlock<WT> cur, nxt;
    cur.load(wt, e);
    for (int ks = 0; ks < n_ks; ++ks) {
        if (ks + 1 < n_ks) nxt.load(wt + static_cast<size_t>(ks + 1) * TB, e);
        float v[32];
        cur.values(v);
        const float d = cur.scale();
        const int k0 = ks * kTileK + b * 32;
#pragma unroll
        for (int n = 0; n < kGemvMaxRows; ++n) {
            if (n >= nrows) break;
            const uint4* xr = reinterpret_cast<const uint4*>(act + static_cast<size_t>(row0 + n) * act_ld + k0);
            float s = 0.f;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const uint4 xv = __ldg(xr + c);
                const __half2* hp = reinterpret_cast<const __half2*>(&xv);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float2 f = __half22float2(hp[j]);
                    s = fmaf(v[8 * c + 2 * j], f.x, s);
                    s = fmaf(v[8 * c + 2 * j + 1], f.y, s);
                }
            }
            acc[n] = fmaf(d, s, acc[n]);
        }
        cur = nxt;
    }
#pragma unroll
    for (int n = 0; n < kGemvMaxRows; ++n) acc[n] += __shfl_xor_sync(0xffffffffu, acc[n], 1);

    if (glu) {
        __shared__ float G[kTileRows][kGemvMaxRows + 1];
        if (b == 0)
#pragma unroll
            for (int n = 0; n < kGemvMaxRows; ++n) G[r][n] = acc[n];
        __syncthreads();
        __half* o = static_cast<__half*>(out);
        for (int i = threadIdx.x; i < kGluHalf * nrows; i += blockDim.x) {
            const int j = i % kGluHalf, n = i / kGluHalf;
            o[static_cast<size_t>(row0 + n) * out_ld + rb * kGluHalf + j] =
                __float2half_rn(silu_mul(G[j][n], G[kGluHalf + j][n]));
        }
    } else if (b == 0) {
        float* o = static_cast<float*>(out);
        for (int n = 0; n < nrows; ++n)
            o[static_cast<size_t>(row0 + n) * out_ld + rb * kTileRows + r] = acc[n];
    }
}

}  // namespace

cudaError_t launch_gemv(const int4* items, const int* n_items, int max_items,
                        const uint8_t* const* wtiles, int wtype, int n_ks, int glu,
                        const __half* act, int act_ld, void* out, int out_ld, cudaStream_t st) {
    if (max_items <= 0) return cudaSuccess;
    switch (wtype) {
        case W_Q4_0:
            gemv_kernel<W_Q4_0><<<max_items, 256, 0, st>>>(items, n_items, wtiles, n_ks, glu, act,
                                                           act_ld, out, out_ld);
            break;
        case W_Q8_0:
            gemv_kernel<W_Q8_0><<<max_items, 256, 0, st>>>(items, n_items, wtiles, n_ks, glu, act,
                                                           act_ld, out, out_ld);
            break;
        default:
            gemv_kernel<W_F16><<<max_items, 256, 0, st>>>(items, n_items, wtiles, n_ks, glu, act,
                                                          act_ld, out, out_ld);
            break;
    }
    return cudaGetLastError();
}

}  // namespace hymoe
