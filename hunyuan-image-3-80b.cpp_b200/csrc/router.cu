// router.cu — router GEMV + softmax + top-K + renormalisation, fused.
//
// Restates src/attention.cpp:213-276 on the device:
//   logits[t,e] = sum_h x[t,h] * Wr[e,h]           (:213-222; + bias[e], no reference counterpart)
//   probs       = softmax(logits)                   (:224-240)
//   top-K by probability, ties -> lower expert id   (:242-265, insertion with strict '<')
//   w_k         = p_k / sum_{k'<K} p_k'              (:267-275)
// Each logit is one thread's sequential chain of separately rounded multiplies and adds in
// h order, the same operations the reference performs, so logits match it bit for bit;
// the softmax sum is likewise taken in expert order.  Only expf may differ from the host
// libm in the last place.
//
// One CTA = 16 tokens (one dispatch chunk).  Phase 1 computes the 16 x E logit block with
// the router matrix streamed through shared memory in 64-column slabs; phase 2 gives each
// warp two tokens and does the softmax and the top-K selection with warp shuffles.  The CTA
// also emits its per-expert token counts for the dispatch prefix scan.
#include <math.h>

#include "common.cuh"
#include "kernels.h"

namespace hymoe {

namespace {

constexpr int kRT = kRouterTok;  // tokens per CTA
constexpr int kMaxE = 64;

__global__ __launch_bounds__(256) void router_kernel(const float* __restrict__ x, int T, int H,
                                                     const float* __restrict__ Wr, int E, int K,
                                                     const float* __restrict__ bias,
                                                     float* __restrict__ logits_out,
                                                     float* __restrict__ probs_out,
                                                     float* __restrict__ topk_w,
                                                     int* __restrict__ topk_idx,
                                                     int* __restrict__ chunk_counts) {
    __shared__ float xs[kRT][64];
    __shared__ float ws[kMaxE][65];
    __shared__ float lg[kRT][kMaxE];
    __shared__ int cnt[kMaxE];

    const int tid = threadIdx.x;
    const int t0 = blockIdx.x * kRT;
    const int e = tid & 63;        // expert of this thread's four outputs
    const int tg = tid >> 6;       // tokens 4 tg .. 4 tg + 3
    float acc[4] = {0.f, 0.f, 0.f, 0.f};

    for (int k0 = 0; k0 < H; k0 += 64) {
        for (int i = tid; i < kRT * 64; i += 256) {
            const int tt = i >> 6, kk = i & 63, t = t0 + tt;
            xs[tt][kk] = t < T ? x[static_cast<size_t>(t) * H + k0 + kk] : 0.f;
        }
        for (int i = tid; i < kMaxE * 64; i += 256) {
            const int ee = i >> 6, kk = i & 63;
            ws[ee][kk] = ee < E ? Wr[static_cast<size_t>(ee) * H + k0 + kk] : 0.f;
        }
        __syncthreads();
#pragma unroll 8
        for (int kk = 0; kk < 64; ++kk) {
            const float w = ws[e][kk];
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[i] = __fadd_rn(acc[i], __fmul_rn(xs[4 * tg + i][kk], w));
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float v = acc[i];
        if (bias != nullptr && e < E) v = __fadd_rn(v, bias[e]);
        lg[4 * tg + i][e] = v;
    }
    if (tid < kMaxE) cnt[tid] = 0;
    __syncthreads();

    const int warp = tid >> 5, lane = tid & 31;
    for (int j = 0; j < 2; ++j) {
        const int tt = 2 * warp + j, t = t0 + tt;
        if (t >= T) continue;  // warp-uniform
        const bool v0 = lane < E, v1 = lane + 32 < E;
        const float l0 = v0 ? lg[tt][lane] : -INFINITY;
        const float l1 = v1 ? lg[tt][lane + 32] : -INFINITY;
        if (logits_out != nullptr) {
            if (v0) logits_out[static_cast<size_t>(t) * E + lane] = l0;
            if (v1) logits_out[static_cast<size_t>(t) * E + lane + 32] = l1;
        }
        float m = fmaxf(l0, l1);
#pragma unroll
        for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float p0 = v0 ? expf(__fsub_rn(l0, m)) : 0.f;
        float p1 = v1 ? expf(__fsub_rn(l1, m)) : 0.f;
        __syncwarp();
        lg[tt][lane] = p0;
        lg[tt][lane + 32] = p1;
        __syncwarp();
        float s = 0.f;
        if (lane == 0)
            for (int ee = 0; ee < E; ++ee) s = __fadd_rn(s, lg[tt][ee]);
        s = __shfl_sync(0xffffffffu, s, 0);
        p0 = __fdiv_rn(p0, s);
        p1 = __fdiv_rn(p1, s);
        if (probs_out != nullptr) {
            if (v0) probs_out[static_cast<size_t>(t) * E + lane] = p0;
            if (v1) probs_out[static_cast<size_t>(t) * E + lane + 32] = p1;
        }
        bool taken0 = !v0, taken1 = !v1;
        float selp[8];
        int sele[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            if (k >= K) break;
            float bv;
            int bi;
            if (!taken0 && (taken1 || p0 >= p1)) {
                bv = p0;
                bi = lane;
            } else if (!taken1) {
                bv = p1;
                bi = lane + 32;
            } else {
                bv = -1.f;
                bi = 1 << 30;
            }
#pragma unroll
            for (int o = 16; o; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (ov > bv || (ov == bv && oi < bi)) {
                    bv = ov;
                    bi = oi;
                }
            }
            if (bi == lane) taken0 = true;
            if (bi == lane + 32) taken1 = true;
            selp[k] = bv;
            sele[k] = bi;
        }
        if (lane == 0) {
            float sw = 0.f;
            for (int k = 0; k < K; ++k) sw = __fadd_rn(sw, selp[k]);
            for (int k = 0; k < K; ++k) {
                topk_w[static_cast<size_t>(t) * K + k] = __fdiv_rn(selp[k], sw);
                topk_idx[static_cast<size_t>(t) * K + k] = sele[k];
                atomicAdd(&cnt[sele[k]], 1);
            }
        }
    }
    __syncthreads();
    if (tid < E) chunk_counts[static_cast<size_t>(blockIdx.x) * E + tid] = cnt[tid];
}

}  // namespace

cudaError_t launch_router(const float* x, int T, int H, const float* Wr, int E, int K,
                          const float* bias, float* logits, float* probs, float* topk_w,
                          int* topk_idx, int* chunk_counts, cudaStream_t st) {
    const int blocks = (T + kRT - 1) / kRT;
    router_kernel<<<blocks, 256, 0, st>>>(x, T, H, Wr, E, K, bias, logits, probs, topk_w,
                                          topk_idx, chunk_counts);
    return cudaGetLastError();
}

}  // namespace hymoe
