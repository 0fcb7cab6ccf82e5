// norm.cu — the decoder layer's post-attention RMSNorm ahead of the MoE block
// (rms_norm_f32, src/rms_norm.cpp:9-33, applied at src/decoder_layer.cpp:34), with the
// reference's rounding: each token's sum of squares is one sequential chain in column order
// (every product rounded, then added: no fused multiply-add), rms = 1 / sqrt(sum / H + eps)
// with IEEE-rounded division and square root, and out = (x * rms) * w[j] rounded left to right.
//
// The chain is inherently serial per token (H dependent adds), so tokens run in parallel: a CTA
// owns 16 tokens, one chain per lane of its first half-warp, fed from shared memory.  All 256
// threads copy 16 x 128-column chunks into a 4-stage ring with 16-byte cp.async (three chunks in
// flight while the current one is summed); rows are padded to 132 floats so the chain lanes'
// 16-byte reads hit distinct banks.  The normalised rows are then written by all threads, four
// independent 16-byte loads in flight per thread (x re-read, mostly from L2).  HBM bound: 8 bytes
// per element (x read once from HBM, out written).
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace hymoe {
namespace {

constexpr int kNormTok = 16;            // tokens per CTA
constexpr int kNormCols = 128;          // columns per staged chunk
constexpr int kNormLd = kNormCols + 4;  // padded row stride (floats)
constexpr int kNormStages = 4;
constexpr int kNormThreads = 256;
constexpr int kNormCopies = kNormTok * kNormCols / 4 / kNormThreads;  // 16-byte copies per thread per chunk
constexpr int kNormUnroll = 4;

// out == nullptr: only the per-token factor, into rms_out[T] (the consumers apply it).
__global__ __launch_bounds__(kNormThreads) void rmsnorm_kernel(const float* __restrict__ x,
                                                               const float* __restrict__ w, float eps,
                                                               int T, int H, float* __restrict__ out,
                                                               float* __restrict__ rms_out) {
    __shared__ __align__(16) float tile[kNormStages][kNormTok * kNormLd];
    __shared__ float rms_s[kNormTok];
    const int t0 = blockIdx.x * kNormTok;
    const int tid = threadIdx.x;
    const int n_chunks = H / kNormCols;
    auto issue = [&](int c) {
        float* dst = tile[c % kNormStages];
#pragma unroll
        for (int i = 0; i < kNormCopies; ++i) {
            const int idx = tid + i * kNormThreads;
            const int row = idx / (kNormCols / 4), q = idx % (kNormCols / 4);
            const int t = min(t0 + row, T - 1);  // rows past T copy a valid row; never written out
            cp_async16(dst + row * kNormLd + 4 * q, x + static_cast<size_t>(t) * H + c * kNormCols + 4 * q);
        }
    };
#pragma unroll
    for (int c = 0; c < kNormStages - 1; ++c) {
        if (c < n_chunks) issue(c);
        cp_async_commit();
    }
    float ss = 0.f;
    for (int c = 0; c < n_chunks; ++c) {
        cp_async_wait<kNormStages - 2>();  // this thread's copies of chunk c have landed
        // every thread's copies of chunk c have landed, and the chain lanes are done with chunk
        // c-1, whose stage the next issue reuses
        __syncthreads();
        if (c + kNormStages - 1 < n_chunks) issue(c + kNormStages - 1);
        cp_async_commit();  // possibly empty: keeps the group count per iteration fixed
        if (tid < kNormTok) {
            const float* row = &tile[c % kNormStages][tid * kNormLd];
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
    cp_async_wait<0>();
    if (tid < kNormTok)
        rms_s[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(H)), eps)));
    if (out == nullptr) {
        if (tid < kNormTok && t0 + tid < T) rms_out[t0 + tid] = rms_s[tid];
        return;
    }
    __syncthreads();
    const int n4 = H / 4;
    const int rows = min(kNormTok, T - t0);
    const int total = rows * n4;
    for (int base = tid; base < total; base += kNormUnroll * kNormThreads) {
        float4 v[kNormUnroll], g[kNormUnroll];
#pragma unroll
        for (int u = 0; u < kNormUnroll; ++u) {
            const int i = base + u * kNormThreads;
            if (i < total) {
                const int row = i / n4, q = i - row * n4;
                v[u] = __ldg(reinterpret_cast<const float4*>(x + static_cast<size_t>(t0 + row) * H) + q);
                g[u] = __ldg(reinterpret_cast<const float4*>(w) + q);
            }
        }
#pragma unroll
        for (int u = 0; u < kNormUnroll; ++u) {
            const int i = base + u * kNormThreads;
            if (i < total) {
                const int row = i / n4, q = i - row * n4;
                const float s = rms_s[row];
                float4 o;
                o.x = __fmul_rn(__fmul_rn(v[u].x, s), g[u].x);
                o.y = __fmul_rn(__fmul_rn(v[u].y, s), g[u].y);
                o.z = __fmul_rn(__fmul_rn(v[u].z, s), g[u].z);
                o.w = __fmul_rn(__fmul_rn(v[u].w, s), g[u].w);
                reinterpret_cast<float4*>(out + static_cast<size_t>(t0 + row) * H)[q] = o;
            }
        }
    }
}

}  // namespace

cudaError_t launch_rmsnorm(const float* x, const float* w, float eps, int T, int H, float* out,
                           cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    if (H % kNormCols != 0) return cudaErrorInvalidValue;
    rmsnorm_kernel<<<(T + kNormTok - 1) / kNormTok, kNormThreads, 0, st>>>(x, w, eps, T, H, out, nullptr);
    return cudaGetLastError();
}

cudaError_t launch_rms(const float* x, float eps, int T, int H, float* rms, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    if (H % kNormCols != 0) return cudaErrorInvalidValue;
    rmsnorm_kernel<<<(T + kNormTok - 1) / kNormTok, kNormThreads, 0, st>>>(x, nullptr, eps, T, H, nullptr, rms);
    return cudaGetLastError();
}

}  // namespace hymoe
