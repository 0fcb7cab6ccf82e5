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
//   router_logits_wide_kernel (T > 64): CTA = 16 tokens x all experts, 128 threads; warp w
//     owns 4 tokens, lane l experts l and l + 32 (8 independent chains per lane); token slabs
//     broadcast, router rows by conflict-free lane reads, 2 stages of 128 columns in shared
//     memory (an earlier 16 x 32 tile with 4 chains per thread was shared-memory-latency
//     bound: 163 us against 0.137 ms for this kernel plus the top-K at 4096 tokens).
//   router_logits_rows_kernel (8 < T <= 64): CTA = one warp owning 4 tokens x 8 experts, one
//     chain per lane; its 12 rows are staged whole (4 column chunks of cp.async groups, the
//     chains starting on the first), so only warp barriers interrupt the chains: the call is
//     the chain's latency (~17 us at H = 4096) plus the first chunk's load.  An earlier
//     8 x 8-thread CTA streaming 256-column stages through a 6-stage ring with a CTA barrier
//     per stage took 40 us at 64 tokens.  router_logits_small_kernel keeps that form for
//     hidden sizes whose rows do not fit in shared memory.
//   router_logits_decode_kernel (T <= 8): CTA = one expert; its router row and the T
//     token rows are staged in shared memory once, then T threads run their chains.
// router_topk_kernel: one warp per token (16 tokens = one dispatch chunk per CTA): softmax
// with the sum taken in expert order, K rounds of warp-shuffle arg-max (ties to the lower
// expert), renormalisation in rank order, and the chunk's per-expert token counts for the
// dispatch prefix scan.  Only expf may differ from the host libm in the last place.
#include <math.h>

#include "common.cuh"
#include "kernels.h"
#include "router_chain.cuh"
#include "topk.cuh"

namespace hymoe {

namespace {

using namespace rchain;

constexpr int kKC = 128;    // columns per stage
constexpr int kLd = kKC + 4;  // padded smem row (floats): 16-byte rows offset by 4 banks
constexpr int kSmallMaxT = 64;

// T > 64: CTA = 16 tokens (one dispatch chunk) x all E experts, 4 warps; warp w owns tokens
// 4w..4w+3 and lane l experts l and l + 32 (8 independent chains per lane).  Token slabs are
// read by broadcast, router rows by conflict-free 16-byte lane reads (rows padded to 132
// floats); two stages of 128 columns (84 KB: two CTAs per SM, the whole grid in one wave at
// 4096 tokens).
constexpr int kWTok = 16, kWExp = 64, kWStages = 2;

__global__ __launch_bounds__(128) void router_logits_wide_kernel(
    const float* __restrict__ x, int T, int H, const float* __restrict__ Wr, int E,
    const float* __restrict__ bias, float* __restrict__ logits, RowNorm nrm) {
    extern __shared__ float4 rsm4[];
    float* sm = reinterpret_cast<float*>(rsm4);
    float* Xs = sm;
    float* Ws = sm + kWStages * kWTok * kLd;
    float* Ns = Ws + kWStages * kWExp * kLd;  // [stages][kKC] norm weights of the stage's columns
    __shared__ float rs[kWTok];                // the slab's per-token norm factors
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t0 = blockIdx.x * kWTok;
    const int nst = H / kKC;
    const bool norm = nrm.rms != nullptr;
    if (norm && tid < kWTok) rs[tid] = nrm.rms[min(t0 + tid, T - 1)];
    auto load_stage = [&](int st, int ks) {
        float* xs = Xs + st * kWTok * kLd;
        float* ws = Ws + st * kWExp * kLd;
        const int c0 = ks * kKC;
        for (int i = tid; i < kWTok * (kKC / 4); i += 128) {
            const int r = i / (kKC / 4), c = (i % (kKC / 4)) * 4;
            cp_async16(xs + r * kLd + c, x + static_cast<size_t>(min(t0 + r, T - 1)) * H + c0 + c);
        }
        for (int i = tid; i < E * (kKC / 4); i += 128) {
            const int r = i / (kKC / 4), c = (i % (kKC / 4)) * 4;
            cp_async16(ws + r * kLd + c, Wr + static_cast<size_t>(r) * H + c0 + c);
        }
        if (norm && tid < kKC / 4) cp_async16(Ns + st * kKC + 4 * tid, nrm.w + c0 + 4 * tid);
    };
    float acc[4][2];
#pragma unroll
    for (int u = 0; u < 4; ++u) acc[u][0] = acc[u][1] = 0.f;
    load_stage(0, 0);
    cp_async_commit();
    for (int ks = 0; ks < nst; ++ks) {
        if (ks + 1 < nst) load_stage((ks + 1) % kWStages, ks + 1);
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        const int st = ks % kWStages;
        if (norm) {
            norm_slab(Xs + st * kWTok * kLd, kWTok, kKC, kLd, rs, Ns + st * kKC, 128);
            __syncthreads();
        }
        const float* xs = Xs + st * kWTok * kLd + (4 * warp) * kLd;
        const float* w0 = Ws + st * kWExp * kLd + lane * kLd;
        const float* w1 = w0 + 32 * kLd;
#pragma unroll 4
        for (int k = 0; k < kKC; k += 4) {
            const float4 wa = *reinterpret_cast<const float4*>(w0 + k);
            const float4 wb = *reinterpret_cast<const float4*>(w1 + k);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const float4 xv = *reinterpret_cast<const float4*>(xs + u * kLd + k);
                acc[u][0] = chain4(acc[u][0], xv, wa);
                acc[u][1] = chain4(acc[u][1], xv, wb);
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const int t = t0 + 4 * warp + u;
        if (t >= T) continue;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int e = lane + 32 * h;
            if (e < E) logits[static_cast<size_t>(t) * E + e] = bias != nullptr ? __fadd_rn(acc[u][h], bias[e]) : acc[u][h];
        }
    }
}

// T <= 8: CTA = one expert; its router row and the T token rows are staged in shared memory
// once, then T threads run their chains without further synchronisation.
__global__ __launch_bounds__(128) void router_logits_decode_kernel(
    const float* __restrict__ x, int T, int H, const float* __restrict__ Wr, int E,
    const float* __restrict__ bias, float* __restrict__ logits, RowNorm nrm) {
    extern __shared__ float4 rsm4[];
    float* ws = reinterpret_cast<float*>(rsm4);  // [H]
    float* xs = ws + H;                           // [T][H]
    float* ns = xs + static_cast<size_t>(T) * H;  // [H] norm weights (pre-norm calls)
    __shared__ float rs[kDecodeMaxT];
    const int e = blockIdx.x;
    const bool norm = nrm.rms != nullptr;
    // The router row before the programmatic-launch wait (it depends on no earlier launch); the
    // token rows and the per-token norm factors after it.
    for (int i = threadIdx.x * 4; i < H; i += 128 * 4)
        cp_async16(ws + i, Wr + static_cast<size_t>(e) * H + i);
    griddep_wait();
    griddep_launch_dependents();
    for (int i = threadIdx.x * 4; i < T * H; i += 128 * 4) cp_async16(xs + i, x + i);
    if (norm) {
        for (int i = threadIdx.x * 4; i < H; i += 128 * 4) cp_async16(ns + i, nrm.w + i);
        if (threadIdx.x < T) rs[threadIdx.x] = nrm.rms[threadIdx.x];
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    if (norm) {
        norm_slab(xs, T, H, H, rs, ns, 128);
        __syncthreads();
    }
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

// 8 < T <= 64: CTA = 8 tokens x 8 experts, 64 threads with one chain each (the chains are
// latency-bound, so they are spread over (T / 8) x (E / 8) CTAs).  x and Wr slabs of 256
// columns stream through a 6-stage cp.async ring.
constexpr int kSmallTT = 8, kSmallTE = 8;
constexpr int kSmallKC = 256, kSmallLd = kSmallKC + 4, kSmallStages = 6;

__global__ __launch_bounds__(64) void router_logits_small_kernel(
    const float* __restrict__ x, int T, int H, const float* __restrict__ Wr, int E,
    const float* __restrict__ bias, float* __restrict__ logits, RowNorm nrm) {
    extern __shared__ float4 rsm4[];
    float* sm = reinterpret_cast<float*>(rsm4);
    float* Xs = sm;                                 // [stages][kSmallTT][kSmallLd]
    float* Ws = sm + kSmallStages * kSmallTT * kSmallLd;      // [stages][kSmallTE][kSmallLd]
    float* Ns = Ws + kSmallStages * kSmallTE * kSmallLd;      // [stages][kSmallKC] norm weights
    __shared__ float rs[kSmallTT];
    const int tid = threadIdx.x;
    const int t0 = blockIdx.x * kSmallTT, e0 = blockIdx.y * kSmallTE;
    const int nt = min(kSmallTT, T - t0), ne = min(kSmallTE, E - e0);
    const int tt = tid / kSmallTE, ee = tid % kSmallTE;
    const int nst = (H + kSmallKC - 1) / kSmallKC;  // H is a multiple of 128
    const bool norm = nrm.rms != nullptr;
    if (norm && tid < kSmallTT) rs[tid] = nrm.rms[min(t0 + tid, T - 1)];

    auto load_stage = [&](int st, int ks) {
        float* xs = Xs + st * kSmallTT * kSmallLd;
        float* ws = Ws + st * kSmallTE * kSmallLd;
        const int c0 = ks * kSmallKC, q = min(kSmallKC, H - c0) / 4;  // float4 per row
        for (int i = tid; i < nt * q; i += 64) {
            const int r = i / q, c = (i % q) * 4;
            cp_async16(xs + r * kSmallLd + c, x + static_cast<size_t>(t0 + r) * H + c0 + c);
        }
        for (int i = tid; i < ne * q; i += 64) {
            const int r = i / q, c = (i % q) * 4;
            cp_async16(ws + r * kSmallLd + c, Wr + static_cast<size_t>(e0 + r) * H + c0 + c);
        }
        if (norm)
            for (int i = tid; i < q; i += 64) cp_async16(Ns + st * kSmallKC + 4 * i, nrm.w + c0 + 4 * i);
    };

    float acc = 0.f;
#pragma unroll
    for (int s = 0; s < kSmallStages - 1; ++s) {
        if (s < nst) load_stage(s, s);
        cp_async_commit();
    }
    for (int ks = 0; ks < nst; ++ks) {
        cp_async_wait<kSmallStages - 2>();
        __syncthreads();
        if (ks + kSmallStages - 1 < nst) load_stage((ks + kSmallStages - 1) % kSmallStages, ks + kSmallStages - 1);
        cp_async_commit();
        const int st = ks % kSmallStages;
        if (norm) {
            norm_slab(Xs + st * kSmallTT * kSmallLd, nt, min(kSmallKC, H - ks * kSmallKC), kSmallLd, rs,
                      Ns + st * kSmallKC, 64);
            __syncthreads();
        }
        const float* xr = Xs + st * kSmallTT * kSmallLd + tt * kSmallLd;
        const float* wr = Ws + st * kSmallTE * kSmallLd + ee * kSmallLd;
        const int ncol = min(kSmallKC, H - ks * kSmallKC);
#pragma unroll 8
        for (int k = 0; k < ncol; k += 4)
            acc = chain4(acc, *reinterpret_cast<const float4*>(xr + k), *reinterpret_cast<const float4*>(wr + k));
    }
    cp_async_wait<0>();
    if (tt < nt && ee < ne) {
        const int t = t0 + tt, e = e0 + ee;
        logits[static_cast<size_t>(t) * E + e] = bias != nullptr ? __fadd_rn(acc, bias[e]) : acc;
    }
}

// 8 < T <= 64: CTA = one warp, lane = 8 * token + expert over 4 tokens x 8 experts.  The warp's
// 4 token rows and 8 router rows (rows padded by 4 floats: the 8 router rows' 16-byte lane reads
// hit distinct banks) and the norm weights are staged whole in 4 column chunks, one cp.async
// group each; each chunk is normalised (pre-norm calls) and chained as soon as it has landed.
constexpr int kRowsTT = 4, kRowsTE = 8, kRowsChunks = 4;

size_t rows_smem(int H) { return sizeof(float) * (static_cast<size_t>(kRowsTT + kRowsTE) * (H + 4) + H); }

__global__ __launch_bounds__(32) void router_logits_rows_kernel(
    const float* __restrict__ x, int T, int H, const float* __restrict__ Wr, int E,
    const float* __restrict__ bias, float* __restrict__ logits, RowNorm nrm) {
    griddep_wait();
    griddep_launch_dependents();
    extern __shared__ float4 rsm4[];
    const int ld = H + 4;
    float* xs = reinterpret_cast<float*>(rsm4);  // [4][ld]
    float* ws = xs + kRowsTT * ld;                // [8][ld]
    float* ns = ws + kRowsTE * ld;                // [H]
    __shared__ float rs[kRowsTT];
    const int lane = threadIdx.x, tt = lane >> 3, ee = lane & 7;
    const int t0 = blockIdx.x * kRowsTT, e0 = blockIdx.y * kRowsTE;
    const int nt = min(kRowsTT, T - t0), ne = min(kRowsTE, E - e0);
    const bool norm = nrm.rms != nullptr;
    if (norm && lane < kRowsTT) rs[lane] = nrm.rms[min(t0 + lane, T - 1)];
    const int cc = H / kRowsChunks;  // columns of a chunk
#pragma unroll
    for (int c = 0; c < kRowsChunks; ++c) {
        const int c0 = c * cc;
        for (int r = 0; r < nt; ++r) {
            const float* src = x + static_cast<size_t>(t0 + r) * H;
            for (int j = c0 + 4 * lane; j < c0 + cc; j += 128) cp_async16(xs + r * ld + j, src + j);
        }
        for (int r = 0; r < ne; ++r) {
            const float* src = Wr + static_cast<size_t>(e0 + r) * H;
            for (int j = c0 + 4 * lane; j < c0 + cc; j += 128) cp_async16(ws + r * ld + j, src + j);
        }
        if (norm)
            for (int j = c0 + 4 * lane; j < c0 + cc; j += 128) cp_async16(ns + j, nrm.w + j);
        cp_async_commit();
    }
    const float* xr = xs + tt * ld;
    const float* wr = ws + ee * ld;
    float acc = 0.f;
#pragma unroll
    for (int c = 0; c < kRowsChunks; ++c) {
        if (c == 0) cp_async_wait<kRowsChunks - 1>();
        else if (c == 1) cp_async_wait<kRowsChunks - 2>();
        else if (c == 2) cp_async_wait<kRowsChunks - 3>();
        else cp_async_wait<0>();
        __syncwarp();  // every lane's copies of chunk c are visible
        const int c0 = c * cc;
        if (norm) {
            norm_slab(xs + c0, nt, cc, ld, rs, ns + c0, 32);
            __syncwarp();
        }
#pragma unroll 8
        for (int k = c0; k < c0 + cc; k += 4)
            acc = chain4(acc, *reinterpret_cast<const float4*>(xr + k), *reinterpret_cast<const float4*>(wr + k));
    }
    if (tt < nt && ee < ne) {
        const int t = t0 + tt, e = e0 + ee;
        logits[static_cast<size_t>(t) * E + e] = bias != nullptr ? __fadd_rn(acc, bias[e]) : acc;
    }
}

__global__ __launch_bounds__(32 * kRouterTok) void router_topk_kernel(
    const float* __restrict__ logits, int T, int E, int K, float* __restrict__ probs_out,
    float* __restrict__ topk_w, int* __restrict__ topk_idx, int* __restrict__ chunk_counts,
    const int* __restrict__ slot_of, RouteMode mode) {
    griddep_wait();
    griddep_launch_dependents();
    __shared__ float pbuf[kRouterTok][kMaxE];
    __shared__ int cnt[kMaxE];
    const int warp = threadIdx.x >> 5;
    if (threadIdx.x < kMaxE) cnt[threadIdx.x] = 0;
    __syncthreads();
    const int t = blockIdx.x * kRouterTok + warp;
    if (t < T) topk_token(logits, t, E, K, probs_out, topk_w, topk_idx, pbuf[warp], cnt, slot_of, mode);
    __syncthreads();
    if (threadIdx.x < E) chunk_counts[static_cast<size_t>(blockIdx.x) * E + threadIdx.x] = cnt[threadIdx.x];
}

}  // namespace

cudaError_t launch_router(const float* x, int T, int H, const float* Wr, int E, int K,
                          const float* bias, float* logits, float* probs, float* topk_w,
                          int* topk_idx, int* chunk_counts, const int* slot_of,
                          const RouteMode& mode, bool topk, cudaStream_t st, const RowNorm& nrm, bool pdl) {
    cudaError_t e;
    if (T <= kDecodeMaxT) {
        const size_t smem = sizeof(float) * static_cast<size_t>(H) * (2 + T);
        e = cudaFuncSetAttribute(router_logits_decode_kernel,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        e = launch_kernel(pdl, router_logits_decode_kernel, dim3(E), dim3(128), smem, st, x, T, H, Wr, E, bias,
                          logits, nrm);
        if (e != cudaSuccess) return e;
    } else if (T <= kSmallMaxT && H % (4 * kRowsChunks) == 0 && rows_smem(H) <= 227u * 1024u) {
        const size_t smem = rows_smem(H);
        e = cudaFuncSetAttribute(router_logits_rows_kernel,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        dim3 g((T + kRowsTT - 1) / kRowsTT, (E + kRowsTE - 1) / kRowsTE);
        e = launch_kernel(pdl, router_logits_rows_kernel, g, dim3(32), smem, st, x, T, H, Wr, E, bias, logits, nrm);
        if (e != cudaSuccess) return e;
    } else if (T <= kSmallMaxT) {
        const size_t smem = sizeof(float) * kSmallStages * ((kSmallTT + kSmallTE) * kSmallLd + kSmallKC);
        e = cudaFuncSetAttribute(router_logits_small_kernel,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        dim3 g((T + kSmallTT - 1) / kSmallTT, (E + kSmallTE - 1) / kSmallTE);
        router_logits_small_kernel<<<g, 64, smem, st>>>(x, T, H, Wr, E, bias, logits, nrm);
    } else {
        const size_t smem = sizeof(float) * kWStages * ((kWTok + kWExp) * kLd + kKC);
        e = cudaFuncSetAttribute(router_logits_wide_kernel,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        router_logits_wide_kernel<<<(T + kWTok - 1) / kWTok, 128, smem, st>>>(x, T, H, Wr, E, bias, logits, nrm);
    }
    e = cudaGetLastError();
    if (e != cudaSuccess || !topk) return e;
    // the top-K kernel waits for the logits kernel like every kernel of a programmatic chain
    return launch_kernel(pdl, router_topk_kernel, dim3((T + kRouterTok - 1) / kRouterTok), dim3(32 * kRouterTok), 0,
                         st, logits, T, E, K, probs, topk_w, topk_idx, chunk_counts, slot_of, mode);
}

}  // namespace hymoe
