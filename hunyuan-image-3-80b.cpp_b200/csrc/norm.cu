// norm.cu — the decoder layer's post-attention RMSNorm ahead of the MoE block
// (rms_norm_f32, src/rms_norm.cpp:9-33, applied at src/decoder_layer.cpp:34), with the
// reference's rounding: each token's sum of squares is one sequential chain in column order
// (every product rounded, then added: no fused multiply-add), rms = 1 / sqrt(sum / H + eps)
// with IEEE-rounded division and square root, and out = (x * rms) * w[j] rounded left to right.
//
// The chain is inherently serial per token (H dependent adds), so tokens run in parallel:
// a CTA owns 32 tokens, one chain per lane of warp 0, fed from shared memory.  All 256 threads
// stage 32 x 128-column chunks with coalesced 16-byte loads, the next chunk's loads in flight
// (registers) while warp 0 sums the current one; rows are padded to 132 floats so the 32
// chain lanes' 16-byte reads hit distinct banks.  The normalised rows are then written by all
// threads (x re-read through L2).  HBM bound: 8 bytes per element (x read, out written).
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace hymoe {
namespace {

constexpr int kNormTok = 32;            // tokens per CTA
constexpr int kNormCols = 128;          // columns per staged chunk
constexpr int kNormLd = kNormCols + 4;  // padded row stride (floats)
constexpr int kNormThreads = 256;
constexpr int kNormLoads = kNormTok * kNormCols / 4 / kNormThreads;  // float4 per thread per chunk

__global__ __launch_bounds__(kNormThreads) void rmsnorm_kernel(const float* __restrict__ x,
                                                               const float* __restrict__ w, float eps,
                                                               int T, int H, float* __restrict__ out) {
    __shared__ __align__(16) float tile[2][kNormTok * kNormLd];
    __shared__ float rms_s[kNormTok];
    const int t0 = blockIdx.x * kNormTok;
    const int tid = threadIdx.x;
    float4 r[kNormLoads];
    auto load = [&](int c0) {
#pragma unroll
        for (int i = 0; i < kNormLoads; ++i) {
            const int idx = tid + i * kNormThreads;
            const int row = idx / (kNormCols / 4), q = idx % (kNormCols / 4);
            const int t = t0 + row;
            r[i] = t < T ? __ldg(reinterpret_cast<const float4*>(x + static_cast<size_t>(t) * H + c0) + q)
                         : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    };
    auto store = [&](int buf) {
#pragma unroll
        for (int i = 0; i < kNormLoads; ++i) {
            const int idx = tid + i * kNormThreads;
            const int row = idx / (kNormCols / 4), q = idx % (kNormCols / 4);
            *reinterpret_cast<float4*>(&tile[buf][row * kNormLd + 4 * q]) = r[i];
        }
    };
    float ss = 0.f;
    const int n_chunks = H / kNormCols;
    load(0);
    for (int c = 0; c < n_chunks; ++c) {
        // buffer c&1 was last read by warp 0 in chunk c-2, which it finished before the
        // barrier of chunk c-1
        store(c & 1);
        __syncthreads();
        if (c + 1 < n_chunks) load((c + 1) * kNormCols);
        if (tid < kNormTok) {
            const float* row = &tile[c & 1][tid * kNormLd];
#pragma unroll 8
            for (int j = 0; j < kNormCols; j += 4) {
                const float4 v = *reinterpret_cast<const float4*>(row + j);
                ss = __fadd_rn(ss, __fmul_rn(v.x, v.x));
                ss = __fadd_rn(ss, __fmul_rn(v.y, v.y));
                ss = __fadd_rn(ss, __fmul_rn(v.z, v.z));
                ss = __fadd_rn(ss, __fmul_rn(v.w, v.w));
            }
        }
    }
    if (tid < kNormTok)
        rms_s[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(H)), eps)));
    __syncthreads();
    const int n4 = H / 4;
    for (int i = tid; i < kNormTok * n4; i += kNormThreads) {
        const int row = i / n4, q = i - row * n4;
        const int t = t0 + row;
        if (t >= T) break;  // rows grow with i
        const float4 v = __ldg(reinterpret_cast<const float4*>(x + static_cast<size_t>(t) * H) + q);
        const float4 g = __ldg(reinterpret_cast<const float4*>(w) + q);
        const float s = rms_s[row];
        float4 o;
        o.x = __fmul_rn(__fmul_rn(v.x, s), g.x);
        o.y = __fmul_rn(__fmul_rn(v.y, s), g.y);
        o.z = __fmul_rn(__fmul_rn(v.z, s), g.z);
        o.w = __fmul_rn(__fmul_rn(v.w, s), g.w);
        reinterpret_cast<float4*>(out + static_cast<size_t>(t) * H)[q] = o;
    }
}

}  // namespace

cudaError_t launch_rmsnorm(const float* x, const float* w, float eps, int T, int H, float* out,
                           cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    if (H % kNormCols != 0) return cudaErrorInvalidValue;
    rmsnorm_kernel<<<(T + kNormTok - 1) / kNormTok, kNormThreads, 0, st>>>(x, w, eps, T, H, out);
    return cudaGetLastError();
}

}  // namespace hymoe
