// norm.cu — the per-token factor of the decoder layer's post-attention RMSNorm
// (rms_norm_f32, src/rms_norm.cpp:9-33, applied at src/decoder_layer.cpp:34):
//   rms[t] = 1 / sqrt(sum_j x[t,j]^2 / H + eps)
// with the reference's rounding: the sum of squares is one sequential chain in column order
// (every product rounded, then added: no fused multiply-add), then IEEE-rounded division and
// square root.  The kernels that read the token rows (router, dispatch, expert-parallel sends)
// apply (x * rms[t]) * w[j] as they load them (RowNorm), so the normalised rows are never
// written: the norm costs one 4 * T * H byte read.
//
// The chain is serial per token (H dependent adds, ~4 cycles each), so its latency bounds the
// kernel and tokens run in parallel: a CTA is ONE warp owning 32 tokens, a lane per token.  The
// warp streams 64-column chunks of its 32 rows through an 8-stage cp.async ring (each copy
// instruction covers 256 contiguous bytes of two rows: coalesced), waits with its own
// cp.async groups plus a warp barrier (no CTA barrier), and each lane runs its token's chain
// over the chunk.  Rows are padded to 68 floats so the lanes' 16-byte reads of 32 different
// rows take the minimum 4 shared-memory wavefronts.  Seven chunks (61 KB) in flight per warp
// keep its HBM stream ahead of the chain.
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace hymoe {
namespace {

constexpr int kRmsTok = 32;             // tokens per CTA (one warp, a lane each)
constexpr int kRmsCols = 64;            // columns per chunk
constexpr int kRmsLd = kRmsCols + 4;    // padded row stride (floats)
constexpr int kRmsStages = 8;
constexpr int kRmsCopies = kRmsTok * kRmsCols / 4 / 32;  // 16-byte copies per lane per chunk (16)
constexpr size_t kRmsSmem = sizeof(float) * kRmsStages * kRmsTok * kRmsLd;

__global__ __launch_bounds__(32) void rms_kernel(const float* __restrict__ x, float eps, int T, int H,
                                                 float* __restrict__ rms) {
    extern __shared__ float4 rms_smem4[];
    float* tile = reinterpret_cast<float*>(rms_smem4);  // [stages][32 rows][kRmsLd]
    const int lane = threadIdx.x;
    const int t0 = blockIdx.x * kRmsTok;
    const int n_chunks = H / kRmsCols;
    // copy i of a chunk: rows 2i and 2i + 1, lanes 0-15 and 16-31, 16 bytes each
    const int sub = lane >> 4, q = lane & 15;
    auto issue = [&](int c) {
        float* dst = tile + (c % kRmsStages) * kRmsTok * kRmsLd;
#pragma unroll
        for (int i = 0; i < kRmsCopies; ++i) {
            const int row = 2 * i + sub;
            const int t = min(t0 + row, T - 1);  // rows past T copy a valid row; never written out
            cp_async16(dst + row * kRmsLd + 4 * q, x + static_cast<size_t>(t) * H + c * kRmsCols + 4 * q);
        }
    };
#pragma unroll
    for (int c = 0; c < kRmsStages - 1; ++c) {
        if (c < n_chunks) issue(c);
        cp_async_commit();
    }
    float ss = 0.f;
    for (int c = 0; c < n_chunks; ++c) {
        cp_async_wait<kRmsStages - 2>();  // this lane's copies of chunk c have landed
        // every lane's copies of chunk c have landed, and every lane is done with chunk c - 1,
        // whose stage the next issue reuses
        __syncwarp();
        if (c + kRmsStages - 1 < n_chunks) issue(c + kRmsStages - 1);
        cp_async_commit();  // possibly empty: keeps the group count per iteration fixed
        const float* row = tile + (c % kRmsStages) * kRmsTok * kRmsLd + lane * kRmsLd;
#pragma unroll
        for (int j = 0; j < kRmsCols; j += 4) {
            const float4 v = *reinterpret_cast<const float4*>(row + j);
            ss = __fadd_rn(ss, __fmul_rn(v.x, v.x));
            ss = __fadd_rn(ss, __fmul_rn(v.y, v.y));
            ss = __fadd_rn(ss, __fmul_rn(v.z, v.z));
            ss = __fadd_rn(ss, __fmul_rn(v.w, v.w));
        }
    }
    cp_async_wait<0>();
    if (t0 + lane < T)
        rms[t0 + lane] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(H)), eps)));
}

}  // namespace

cudaError_t launch_rms(const float* x, float eps, int T, int H, float* rms, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    if (H % kRmsCols != 0) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(rms_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kRmsSmem));
    if (e != cudaSuccess) return e;
    rms_kernel<<<(T + kRmsTok - 1) / kRmsTok, 32, kRmsSmem, st>>>(x, eps, T, H, rms);
    return cudaGetLastError();
}

}  // namespace hymoe
