// router.cu — router GEMV, softmax, top-K selection and renormalisation.
//
// Restates src/attention.cpp:213-276 on the device:
//   logits[t,e] = sum_h x[t,h] * Wr[e,h]           (:213-222; + bias[e], no reference counterpart)
//   probs       = softmax(logits)                   (:224-240)
//   top-K by probability, ties -> lower expert id   (:242-265, insertion with strict '<')
//   w_k         = p_k / sum_{k'<K} p_k'              (:267-275)
//
// router_logits_kernel: every logit is one thread's sequential chain of separately rounded
// multiplies and adds in h order - the operations the reference performs - so the logits
// equal the reference's bit for bit.  A CTA covers 32 tokens x 8 experts (one chain per
// thread); x and Wr are streamed through the read-only path with 16-byte loads (a row of x
// is shared by the 8 expert threads of a token, a router row by the 32 token threads).
// The chain's add latency bounds a call at roughly 4 x H cycles regardless of T.
//
// router_topk_kernel: one warp per token (16 tokens = one dispatch chunk per CTA): softmax
// with the sum taken in expert order, K rounds of warp-shuffle arg-max (ties to the lower
// expert), renormalisation in rank order, and the chunk's per-expert token counts for the
// dispatch prefix scan.  Only expf may differ from the host libm in the last place.
#include <math.h>

#include "common.cuh"
#include "kernels.h"

namespace hymoe {

namespace {

constexpr int kLogitTok = 32;  // tokens per logits CTA
constexpr int kLogitExp = 8;   // experts per logits CTA
constexpr int kMaxE = 64;

__global__ __launch_bounds__(256) void router_logits_kernel(const float* __restrict__ x, int T,
                                                            int H, const float* __restrict__ Wr,
                                                            int E, const float* __restrict__ bias,
                                                            float* __restrict__ logits) {
    const int t = blockIdx.x * kLogitTok + (threadIdx.x >> 3);
    const int e = blockIdx.y * kLogitExp + (threadIdx.x & 7);
    if (t >= T || e >= E) return;
    const float4* xr = reinterpret_cast<const float4*>(x + static_cast<size_t>(t) * H);
    const float4* wr = reinterpret_cast<const float4*>(Wr + static_cast<size_t>(e) * H);
    float acc = 0.f;
    const int n4 = H / 4;
    int i = 0;
    for (; i + 4 <= n4; i += 4) {
        float4 xv[4], wv[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            xv[u] = __ldg(xr + i + u);
            wv[u] = __ldg(wr + i + u);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            acc = __fadd_rn(acc, __fmul_rn(xv[u].x, wv[u].x));
            acc = __fadd_rn(acc, __fmul_rn(xv[u].y, wv[u].y));
            acc = __fadd_rn(acc, __fmul_rn(xv[u].z, wv[u].z));
            acc = __fadd_rn(acc, __fmul_rn(xv[u].w, wv[u].w));
        }
    }
    for (; i < n4; ++i) {
        const float4 xv = __ldg(xr + i), wv = __ldg(wr + i);
        acc = __fadd_rn(acc, __fmul_rn(xv.x, wv.x));
        acc = __fadd_rn(acc, __fmul_rn(xv.y, wv.y));
        acc = __fadd_rn(acc, __fmul_rn(xv.z, wv.z));
        acc = __fadd_rn(acc, __fmul_rn(xv.w, wv.w));
    }
    if (bias != nullptr) acc = __fadd_rn(acc, bias[e]);
    logits[static_cast<size_t>(t) * E + e] = acc;
}

__global__ __launch_bounds__(32 * kRouterTok) void router_topk_kernel(
    const float* __restrict__ logits, int T, int E, int K, float* __restrict__ probs_out,
    float* __restrict__ topk_w, int* __restrict__ topk_idx, int* __restrict__ chunk_counts) {
    __shared__ float pbuf[kRouterTok][kMaxE];
    __shared__ int cnt[kMaxE];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x < kMaxE) cnt[threadIdx.x] = 0;
    __syncthreads();
    const int t = blockIdx.x * kRouterTok + warp;
    if (t < T) {
        const bool v0 = lane < E, v1 = lane + 32 < E;
        const float l0 = v0 ? logits[static_cast<size_t>(t) * E + lane] : -INFINITY;
        const float l1 = v1 ? logits[static_cast<size_t>(t) * E + lane + 32] : -INFINITY;
        float m = fmaxf(l0, l1);
#pragma unroll
        for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float p0 = v0 ? expf(__fsub_rn(l0, m)) : 0.f;
        float p1 = v1 ? expf(__fsub_rn(l1, m)) : 0.f;
        pbuf[warp][lane] = p0;
        pbuf[warp][lane + 32] = p1;
        __syncwarp();
        float s = 0.f;
        if (lane == 0)
            for (int ee = 0; ee < E; ++ee) s = __fadd_rn(s, pbuf[warp][ee]);
        s = __shfl_sync(0xffffffffu, s, 0);
        p0 = __fdiv_rn(p0, s);
        p1 = __fdiv_rn(p1, s);
        if (probs_out != nullptr) {
            if (v0) probs_out[static_cast<size_t>(t) * E + lane] = p0;
            if (v1) probs_out[static_cast<size_t>(t) * E + lane + 32] = p1;
        }
        bool taken0 = !v0, taken1 = !v1;
        float selp = 0.f;  // lane k keeps the k-th selection
        int sele = 0;
        for (int k = 0; k < K; ++k) {
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
            if (lane == k) {
                selp = bv;
                sele = bi;
            }
        }
        // renormalise in rank order: sum_{k<K} p_k sequentially
        float sw = 0.f;
        for (int k = 0; k < K; ++k) sw = __fadd_rn(sw, __shfl_sync(0xffffffffu, selp, k));
        if (lane < K) {
            topk_w[static_cast<size_t>(t) * K + lane] = __fdiv_rn(selp, sw);
            topk_idx[static_cast<size_t>(t) * K + lane] = sele;
            atomicAdd(&cnt[sele], 1);
        }
    }
    __syncthreads();
    if (threadIdx.x < E) chunk_counts[static_cast<size_t>(blockIdx.x) * E + threadIdx.x] = cnt[threadIdx.x];
}

}  // namespace

cudaError_t launch_router(const float* x, int T, int H, const float* Wr, int E, int K,
                          const float* bias, float* logits, float* probs, float* topk_w,
                          int* topk_idx, int* chunk_counts, cudaStream_t st) {
    dim3 g1((T + kLogitTok - 1) / kLogitTok, (E + kLogitExp - 1) / kLogitExp);
    router_logits_kernel<<<g1, 256, 0, st>>>(x, T, H, Wr, E, bias, logits);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    router_topk_kernel<<<(T + kRouterTok - 1) / kRouterTok, 32 * kRouterTok, 0, st>>>(
        logits, T, E, K, probs, topk_w, topk_idx, chunk_counts);
    return cudaGetLastError();
}

}  // namespace hymoe
