// router_chain.cuh — the router logit as the reference computes it (src/attention.cpp:213-222):
// one sequential chain of separately rounded multiplies and adds in column order, and the
// on-the-fly RMSNorm of staged token slabs (src/rms_norm.cpp:9-33).  Used by the router
// kernels (router.cu) and the one-kernel decode path (decode.cu).
#pragma once

#include "common.cuh"
#include "kernels.h"

namespace hymoe {
namespace rchain {

// Two IEEE single-precision products, each rounded to nearest, in one packed instruction
// (sm_100 f32x2): the same results as two __fmul_rn.
__device__ __forceinline__ float2 mul2_rn(float ax, float ay, float bx, float by) {
    unsigned long long a, b, p;
    asm("mov.b64 %0, {%1, %2};" : "=l"(a) : "f"(ax), "f"(ay));
    asm("mov.b64 %0, {%1, %2};" : "=l"(b) : "f"(bx), "f"(by));
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(p) : "l"(a), "l"(b));
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(p));
    return r;
}

// acc + a.x*b.x + a.y*b.y + a.z*b.z + a.w*b.w, every product and sum separately rounded, in
// that order (the reference's loop).
__device__ __forceinline__ float chain4(float acc, float4 a, float4 b) {
    const float2 p01 = mul2_rn(a.x, a.y, b.x, b.y);
    const float2 p23 = mul2_rn(a.z, a.w, b.z, b.w);
    acc = __fadd_rn(acc, p01.x);
    acc = __fadd_rn(acc, p01.y);
    acc = __fadd_rn(acc, p23.x);
    return __fadd_rn(acc, p23.y);
}

// Token rows normalised on the fly (RowNorm): each landed stage of the token slab is
// normalised in place, x * rms[row] * w[col] rounded left to right, from the per-token factors
// and the stage's slice of the norm weights, both staged in shared memory with the slab (no
// global load on the stage's critical path).  cols % 4 == 0, ld % 4 == 0.
__device__ __forceinline__ void norm_slab(float* xs, int rows, int cols, int ld, const float* rs,
                                          const float* ws, int nthreads) {
    const int q = cols / 4;
    for (int i = threadIdx.x; i < rows * q; i += nthreads) {
        const int r = i / q, c = 4 * (i - r * q);
        float4 v = *reinterpret_cast<float4*>(xs + r * ld + c);
        const float4 g = *reinterpret_cast<const float4*>(ws + c);
        const float s = rs[r];
        v.x = __fmul_rn(__fmul_rn(v.x, s), g.x);
        v.y = __fmul_rn(__fmul_rn(v.y, s), g.y);
        v.z = __fmul_rn(__fmul_rn(v.z, s), g.z);
        v.w = __fmul_rn(__fmul_rn(v.w, s), g.w);
        *reinterpret_cast<float4*>(xs + r * ld + c) = v;
    }
}

}  // namespace rchain
}  // namespace hymoe
