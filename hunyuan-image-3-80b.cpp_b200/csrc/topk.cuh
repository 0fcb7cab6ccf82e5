// topk.cuh — per-token routing step shared by the top-K kernel and the fused decode
// top-K + plan kernel: softmax with the sum taken in expert order, K rounds of warp-shuffle
// arg-max (ties to the lower expert), renormalisation in rank order (src/attention.cpp:224-275).
// Only expf may differ from the host libm in the last place.
#pragma once

#include <math.h>

#include "common.cuh"
#include "kernels.h"

namespace hymoe {

constexpr int kMaxE = 64;

// One warp routes token t.  pbuf: this warp's kMaxE floats of shared memory.  cnt: shared
// per-slot counters of the caller's chunk (incremented for the token's K selections).
// slot_of: expert -> placement slot (nullptr: slot = expert).  Selection, ties and weights are
// decided on expert ids; topk_idx and cnt receive the selected experts' slots, so every later
// step (sort, dispatch, GEMM groups, combine) works in slot order.  mode: the routing variant.
__device__ __forceinline__ void topk_token(const float* __restrict__ logits, int t, int E, int K,
                                           float* __restrict__ probs_out, float* __restrict__ topk_w,
                                           int* __restrict__ topk_idx, float* pbuf, int* cnt,
                                           const int* __restrict__ slot_of, const RouteMode& mode) {
    const int lane = threadIdx.x & 31;
    const bool v0 = lane < E, v1 = lane + 32 < E;
    const float l0 = v0 ? logits[static_cast<size_t>(t) * E + lane] : -INFINITY;
    const float l1 = v1 ? logits[static_cast<size_t>(t) * E + lane + 32] : -INFINITY;
    float m = fmaxf(l0, l1);
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float p0 = v0 ? expf(__fsub_rn(l0, m)) : 0.f;
    float p1 = v1 ? expf(__fsub_rn(l1, m)) : 0.f;
    pbuf[lane] = p0;
    pbuf[lane + 32] = p1;
    __syncwarp();
    float s = 0.f;
    if (lane == 0)
        for (int ee = 0; ee < E; ++ee) s = __fadd_rn(s, pbuf[ee]);
    s = __shfl_sync(0xffffffffu, s, 0);
    p0 = __fdiv_rn(p0, s);
    p1 = __fdiv_rn(p1, s);
    if (probs_out != nullptr) {
        if (v0) probs_out[static_cast<size_t>(t) * E + lane] = p0;
        if (v1) probs_out[static_cast<size_t>(t) * E + lane + 32] = p1;
    }
    if (mode.n_group > 0) {
        // Group-limited greedy (src/hunyuan_moe_full.cpp:137-170): groups of gs experts scored
        // by their largest probability (at least 0); the topk_group best (ties: lower group)
        // keep their probabilities, every other expert's becomes 0.  probs_out keeps the
        // unmasked softmax, as the reference's router_probs does.
        const int gs = E / mode.n_group;
        __syncwarp();  // lane 0 is done reading the exponentials
        pbuf[lane] = p0;
        pbuf[lane + 32] = p1;
        __syncwarp();
        float sc = 0.f;
        if (lane < mode.n_group)
            for (int e = 0; e < gs; ++e) {
                const float v = pbuf[lane * gs + e];
                if (v > sc) sc = v;
            }
        bool gtaken = lane >= mode.n_group, gsel = false;
        for (int r = 0; r < mode.topk_group; ++r) {
            float bv = gtaken ? -1.f : sc;
            int bi = gtaken ? (1 << 30) : lane;
#pragma unroll
            for (int o = 16; o; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (ov > bv || (ov == bv && oi < bi)) {
                    bv = ov;
                    bi = oi;
                }
            }
            if (bi == lane) gtaken = gsel = true;
        }
        const unsigned kept = __ballot_sync(0xffffffffu, gsel);  // bit g: group g kept
        if (v0 && !((kept >> (lane / gs)) & 1u)) p0 = 0.f;
        if (v1 && !((kept >> ((lane + 32) / gs)) & 1u)) p1 = 0.f;
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
        float wv;
        if (mode.norm)
            wv = __fdiv_rn(selp, mode.clamp && sw < 1e-8f ? 1e-8f : sw);
        else
            wv = __fmul_rn(selp, mode.scale);
        topk_w[static_cast<size_t>(t) * K + lane] = wv;
        const int slot = slot_of != nullptr ? __ldg(slot_of + sele) : sele;
        topk_idx[static_cast<size_t>(t) * K + lane] = slot;
        atomicAdd(&cnt[slot], 1);
    }
}

// Exclusive prefix sum of n <= 96 ints held in shared memory (in place, total returned in
// out_total), computed by the calling warp (all 32 lanes).
__device__ __forceinline__ int warp_exclusive_scan(int* v, int n) {
    const int lane = threadIdx.x & 31;
    int a[3], loc = 0;
#pragma unroll
    for (int i = 0; i < 3; ++i) {
        const int idx = 3 * lane + i;
        a[i] = idx < n ? v[idx] : 0;
        loc += a[i];
    }
    int inc = loc;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += u;
    }
    int run = inc - loc;
#pragma unroll
    for (int i = 0; i < 3; ++i) {
        const int idx = 3 * lane + i;
        if (idx < n) v[idx] = run;
        run += a[i];
    }
    return __shfl_sync(0xffffffffu, inc, 31);
}

}  // namespace hymoe
