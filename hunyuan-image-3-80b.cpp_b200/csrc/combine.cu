// combine.cu — weighted combine of the routed expert outputs, plus the shared expert and
// the residual, in the reference's operation order:
//   routed = 0; for k: routed += w[t,k] * y_k        (src/attention.cpp:296-298)
//   moe    = shared + routed                         (src/attention.cpp:306-309)
//   out    = residual + moe                          (src/decoder_layer.cpp:42)
// Each element is a chain of separately rounded IEEE multiplies and adds in that order.
#include "common.cuh"
#include "kernels.h"

namespace hymoe {

namespace {

// Grid (H / 512, T), 128 threads x 4 columns.  All K routed rows are loaded before the
// arithmetic starts (K <= 8), so the loads overlap instead of following the FP chain.
__global__ __launch_bounds__(128) void combine_kernel(const float* __restrict__ y_shared,
                                                      const float* __restrict__ y_routed,
                                                      const int* __restrict__ slot_pos,
                                                      const float* __restrict__ topk_w,
                                                      const float* resid, float* out, int T,
                                                      int H, int K) {
    const int t = blockIdx.y;
    const int j = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (j >= H) return;
    float4 v[8];
    float w[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        if (k < K) {
            const int pos = __ldg(slot_pos + t * K + k);
            w[k] = __ldg(topk_w + t * K + k);
            v[k] = *reinterpret_cast<const float4*>(y_routed + static_cast<size_t>(pos) * H + j);
        }
    }
    const float4 s = *reinterpret_cast<const float4*>(y_shared + static_cast<size_t>(t) * H + j);
    float4 h = make_float4(0.f, 0.f, 0.f, 0.f);
    if (resid != nullptr) h = *reinterpret_cast<const float4*>(resid + static_cast<size_t>(t) * H + j);
    float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        if (k < K) {
            r.x = __fadd_rn(r.x, __fmul_rn(w[k], v[k].x));
            r.y = __fadd_rn(r.y, __fmul_rn(w[k], v[k].y));
            r.z = __fadd_rn(r.z, __fmul_rn(w[k], v[k].z));
            r.w = __fadd_rn(r.w, __fmul_rn(w[k], v[k].w));
        }
    }
    float4 o = make_float4(__fadd_rn(s.x, r.x), __fadd_rn(s.y, r.y), __fadd_rn(s.z, r.z),
                           __fadd_rn(s.w, r.w));
    if (resid != nullptr)
        o = make_float4(__fadd_rn(h.x, o.x), __fadd_rn(h.y, o.y), __fadd_rn(h.z, o.z),
                        __fadd_rn(h.w, o.w));
    *reinterpret_cast<float4*>(out + static_cast<size_t>(t) * H + j) = o;
}

}  // namespace

cudaError_t launch_combine(const float* y_shared, const float* y_routed, const int* slot_pos,
                           const float* topk_w, const float* resid, float* out, int T, int H,
                           int K, cudaStream_t st) {
    if (K > 8) return cudaErrorInvalidValue;
    dim3 grid((H / 4 + 127) / 128, T);
    combine_kernel<<<grid, 128, 0, st>>>(y_shared, y_routed, slot_pos, topk_w, resid, out, T, H, K);
    return cudaGetLastError();
}

}  // namespace hymoe
