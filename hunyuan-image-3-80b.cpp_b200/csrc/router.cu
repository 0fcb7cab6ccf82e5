// router.cu — router GEMV, softmax, top-K selection and renormalisation.
//
// Restates src/attention.cpp:213-276 on the device:
//   logits[t,e] = sum_h x[t,h] * Wr[e,h]           (:213-222; + bias[e], no reference counterpart)
//   probs       = softmax(logits)                   (:224-240)
//   top-K by probability, ties -> lower expert id   (:242-265, insertion with strict '<')
//   w_k         = p_k / sum_{k'<K} p_k'              (:267-275)
//
// Logits: every logit is one thread's sequential chain of separately rounded multiplies
// and adds in h order - the operations the reference performs - so the logits equal the
// reference's bit for bit.  The add chain bounds a call at roughly 4 x H cycles; beyond
// that the kernels are organised for operand reuse:
//   router_logits_tiled_kernel (T > 8): CTA = 16 tokens x 32 experts, 128 threads with
//     2 tokens x 2 experts (4 independent chains) each; x and Wr slabs of 128 columns
//     stream through a 3-stage cp.async ring in shared memory.
//   router_logits_decode_kernel (T <= 8): CTA = one expert; its router row and the T
//     token rows are staged in shared memory once, then T threads run their chains.
// router_topk_kernel: one warp per token (16 tokens = one dispatch chunk per CTA): softmax
// with the sum taken in expert order, K rounds of warp-shuffle arg-max (ties to the lower
// expert), renormalisation in rank order, and the chunk's per-expert token counts for the
// dispatch prefix scan.  Only expf may differ from the host libm in the last place.
#include <math.h>

#include "common.cuh"
#include "kernels.h"

namespace hymoe {

namespace {

constexpr int kMaxE = 64;
constexpr int kTT = 16;     // tokens per tiled CTA
constexpr int kTE = 32;     // experts per tiled CTA
constexpr int kKC = 128;    // columns per stage
constexpr int kLd = kKC + 4;  // padded smem row (floats): 16-byte rows offset by 4 banks
constexpr int kStages = 3;
constexpr int kDecodeMaxT = 8;

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ float chain4(float acc, float4 a, float4 b) {
    acc = __fadd_rn(acc, __fmul_rn(a.x, b.x));
    acc = __fadd_rn(acc, __fmul_rn(a.y, b.y));
    acc = __fadd_rn(acc, __fmul_rn(a.z, b.z));
    return __fadd_rn(acc, __fmul_rn(a.w, b.w));
}

__global__ __launch_bounds__(128) void router_logits_tiled_kernel(
    const float* __restrict__ x, int T, int H, const float* __restrict__ Wr, int E,
    const float* __restrict__ bias, float* __restrict__ logits) {
    extern __shared__ float4 rsm4[];
    float* sm = reinterpret_cast<float*>(rsm4);
    float* Xs = sm;                          // [stages][kTT][kLd]
    float* Ws = sm + kStages * kTT * kLd;    // [stages][kTE][kLd]
    const int tid = threadIdx.x;
    const int t0 = blockIdx.x * kTT, e0 = blockIdx.y * kTE;
    const int tq = tid >> 4, eq = tid & 15;  // tokens 2tq, 2tq+1; experts eq, eq+16
    const int nst = H / kKC;

    auto load_stage = [&](int st, int ks) {
        float* xs = Xs + st * kTT * kLd;
        float* ws = Ws + st * kTE * kLd;
        const int c0 = ks * kKC;
        for (int i = tid; i < kTT * (kKC / 4); i += 128) {
            const int r = i / (kKC / 4), c = (i % (kKC / 4)) * 4;
            const int t = min(t0 + r, T - 1);
            cp_async16(xs + r * kLd + c, x + static_cast<size_t>(t) * H + c0 + c);
        }
        for (int i = tid; i < kTE * (kKC / 4); i += 128) {
            const int r = i / (kKC / 4), c = (i % (kKC / 4)) * 4;
            const int e = min(e0 + r, E - 1);
            cp_async16(ws + r * kLd + c, Wr + static_cast<size_t>(e) * H + c0 + c);
        }
    };

    float a00 = 0.f, a01 = 0.f, a10 = 0.f, a11 = 0.f;  // [token][expert]
#pragma unroll
    for (int s = 0; s < kStages - 1; ++s) {
        if (s < nst) load_stage(s, s);
        cp_async_commit();
    }
    for (int ks = 0; ks < nst; ++ks) {
        cp_async_wait<kStages - 2>();
        __syncthreads();
        if (ks + kStages - 1 < nst) load_stage((ks + kStages - 1) % kStages, ks + kStages - 1);
        cp_async_commit();
        const int st = ks % kStages;
        const float* x0 = Xs + st * kTT * kLd + (2 * tq) * kLd;
        const float* x1 = x0 + kLd;
        const float* w0 = Ws + st * kTE * kLd + eq * kLd;
        const float* w1 = w0 + 16 * kLd;
#pragma unroll 8
        for (int k = 0; k < kKC; k += 4) {
            const float4 xa = *reinterpret_cast<const float4*>(x0 + k);
            const float4 xb = *reinterpret_cast<const float4*>(x1 + k);
            const float4 wa = *reinterpret_cast<const float4*>(w0 + k);
            const float4 wb = *reinterpret_cast<const float4*>(w1 + k);
            a00 = chain4(a00, xa, wa);
            a01 = chain4(a01, xa, wb);
            a10 = chain4(a10, xb, wa);
            a11 = chain4(a11, xb, wb);
        }
    }
    cp_async_wait<0>();
    const int ta = t0 + 2 * tq, ea = e0 + eq;
    const float b0 = (bias != nullptr && ea < E) ? bias[ea] : 0.f;
    const float b1 = (bias != nullptr && ea + 16 < E) ? bias[ea + 16] : 0.f;
    auto put = [&](int t, int e, float v, float b) {
        if (t < T && e < E) logits[static_cast<size_t>(t) * E + e] = bias ? __fadd_rn(v, b) : v;
    };
    put(ta, ea, a00, b0);
    put(ta, ea + 16, a01, b1);
    put(ta + 1, ea, a10, b0);
    put(ta + 1, ea + 16, a11, b1);
}

__global__ __launch_bounds__(128) void router_logits_decode_kernel(
    const float* __restrict__ x, int T, int H, const float* __restrict__ Wr, int E,
    const float* __restrict__ bias, float* __restrict__ logits) {
    extern __shared__ float4 rsm4[];
    float* ws = reinterpret_cast<float*>(rsm4);  // [H]
    float* xs = ws + H;                           // [T][H]
    const int e = blockIdx.x;
    for (int i = threadIdx.x * 4; i < H; i += 128 * 4)
        cp_async16(ws + i, Wr + static_cast<size_t>(e) * H + i);
    for (int i = threadIdx.x * 4; i < T * H; i += 128 * 4) cp_async16(xs + i, x + i);
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    const int t = threadIdx.x;
    if (t >= T) return;
    const float* xr = xs + static_cast<size_t>(t) * H;
    float acc = 0.f;
#pragma unroll 8
    for (int k = 0; k < H; k += 4)
        acc = chain4(acc, *reinterpret_cast<const float4*>(xr + k), *reinterpret_cast<const float4*>(ws + k));
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
    cudaError_t e;
    if (T <= kDecodeMaxT) {
        const size_t smem = sizeof(float) * static_cast<size_t>(H) * (1 + T);
        e = cudaFuncSetAttribute(router_logits_decode_kernel,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        router_logits_decode_kernel<<<E, 128, smem, st>>>(x, T, H, Wr, E, bias, logits);
    } else {
        const size_t smem = sizeof(float) * kStages * (kTT + kTE) * kLd;
        e = cudaFuncSetAttribute(router_logits_tiled_kernel,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        dim3 g((T + kTT - 1) / kTT, (E + kTE - 1) / kTE);
        router_logits_tiled_kernel<<<g, 128, smem, st>>>(x, T, H, Wr, E, bias, logits);
    }
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    router_topk_kernel<<<(T + kRouterTok - 1) / kRouterTok, 32 * kRouterTok, 0, st>>>(
        logits, T, E, K, probs, topk_w, topk_idx, chunk_counts);
    return cudaGetLastError();
}

}  // namespace hymoe
