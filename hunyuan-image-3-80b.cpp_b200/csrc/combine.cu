// combine.cu — weighted combine of the routed expert outputs, plus the shared expert and
// the residual, in the reference's operation order:
//   routed = 0; for k: routed += w[t,k] * y_k        (src/attention.cpp:296-298)
//   moe    = shared + routed                         (src/attention.cpp:306-309)
//   out    = residual + moe                          (src/decoder_layer.cpp:42)
// Each element is a chain of separately rounded IEEE multiplies and adds in that order.
// Routed expert results arrive as fp16 (the down projection stores them rounded once); the
// shared expert's result and everything after are fp32.
#include "common.cuh"
#include "kernels.h"

namespace hymoe {

namespace {

// Grid (H / 1024, T), 128 threads x 8 columns.  All K routed rows are loaded before the
// arithmetic starts (K <= 8), so the loads overlap instead of following the FP chain.
__global__ __launch_bounds__(128, 10) void combine_kernel(const float* __restrict__ y_shared,
                                                      const __half* __restrict__ y_routed,
                                                      const int* __restrict__ slot_pos,
                                                      const float* __restrict__ topk_w,
                                                      const float* resid, float* out, int T,
                                                      int H, int K) {
    griddep_wait();
    griddep_launch_dependents();
    const int t = blockIdx.y;
    const int j = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
    if (j >= H) return;
    uint4 u[8];  // raw fp16 rows (converted inside the sum: fewer live registers)
    float w[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        if (k < K) {
            const int pos = __ldg(slot_pos + t * K + k);  // < 0: a pair dropped by the capacity
            w[k] = __ldg(topk_w + t * K + k);
            u[k] = pos >= 0 ? *reinterpret_cast<const uint4*>(y_routed + static_cast<size_t>(pos) * H + j)
                            : make_uint4(0u, 0u, 0u, 0u);
        }
    }
    const float* sr = y_shared + static_cast<size_t>(t) * H + j;
    const float4 s0 = *reinterpret_cast<const float4*>(sr), s1 = *reinterpret_cast<const float4*>(sr + 4);
    const float s[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    float h[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (resid != nullptr) {
        const float* hr = resid + static_cast<size_t>(t) * H + j;
        const float4 h0 = *reinterpret_cast<const float4*>(hr), h1 = *reinterpret_cast<const float4*>(hr + 4);
        h[0] = h0.x; h[1] = h0.y; h[2] = h0.z; h[3] = h0.w;
        h[4] = h1.x; h[5] = h1.y; h[6] = h1.z; h[7] = h1.w;
    }
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        float r = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            if (k < K && w[k] != 0.f) {  // a dropped pair (weight 0) adds nothing
                const uint32_t wd = i < 2 ? u[k].x : i < 4 ? u[k].y : i < 6 ? u[k].z : u[k].w;
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&wd));
                r = __fadd_rn(r, __fmul_rn(w[k], (i & 1) ? f.y : f.x));
            }
        }
        o[i] = __fadd_rn(s[i], r);
        if (resid != nullptr) o[i] = __fadd_rn(h[i], o[i]);
    }
    float* orow = out + static_cast<size_t>(t) * H + j;
    *reinterpret_cast<float4*>(orow) = make_float4(o[0], o[1], o[2], o[3]);
    *reinterpret_cast<float4*>(orow + 4) = make_float4(o[4], o[5], o[6], o[7]);
}

}  // namespace

cudaError_t launch_combine(const float* y_shared, const __half* y_routed, const int* slot_pos,
                           const float* topk_w, const float* resid, float* out, int T, int H,
                           int K, cudaStream_t st, bool pdl) {
    if (K > 8) return cudaErrorInvalidValue;
    dim3 grid((H / 8 + 127) / 128, T);
    return launch_kernel(pdl, combine_kernel, grid, dim3(128), 0, st, y_shared, y_routed, slot_pos, topk_w, resid,
                         out, T, H, K);
}

}  // namespace hymoe
