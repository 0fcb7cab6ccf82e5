// decode.cu — the MoE block for decode calls (1 to 8 tokens, one GPU, Q4_0 / Q8_0 experts) as
// ONE persistent cooperative kernel (src/attention.cpp:191-313 for a handful of tokens).
//
// At one token the block reads ~361 MB of weights (8 routed experts + the shared one) and does
// almost no arithmetic, so the call is a weight stream at HBM speed plus whatever keeps the
// stream from starting or finishing: the router's 4096-long add chain (~8 us, bit-exact with
// the reference), top-K, plan, dispatch and combine, and the gaps between their launches.  Here
// all of it is one grid of one 8-warp CTA per SM, and kernel boundaries become counters in a
// small device block (DecodeSync):
//
//   router CTAs (the last min(32, E)): stage their experts' router rows and the T token rows
//     (normalised on the fly for pre-norm calls), run one sequential chain per (token, expert)
//     - the router kernels' arithmetic, so the logits are the same bits - and count themselves
//     done; the last one to finish runs the top-K of every token (topk_token, the same routing
//     step as the multi-kernel path), lists the routed slots hit (in slot order) and publishes
//     the plan with a release store.
//   one CTA writes the fp16 token rows (the only activation of every gate_up item) and
//     publishes them.
//   every CTA walks its share of one work list, position p = blockIdx.x + i * gridDim.x:
//     [shared gate_up row blocks][shared down][routed gate_up, slot-major][routed down]
//     The shared expert needs no routing, so its weights stream while the router chains run;
//     routed items wait for the plan, and a down item of group g waits until all of g's
//     gate_up items are done (per-group counter).  Positions only ever wait on earlier
//     positions and every CTA takes its positions in order, so with all CTAs resident
//     (cooperative launch) every wait ends.
//   item = one 128-row weight block of one group against all T token rows (one 8-row
//     activation box): the persistent streaming kernel's scheme (gemv.cu), warp w streaming
//     k-tiles w, w + 8, ... through a private ring, partials summed in warp order.  Tokens that
//     did not select a routed expert are computed too (their columns cost nothing in the MMA)
//     and never stored, so no dispatch or sort is needed: a token's column does not depend on
//     the other columns, and the results equal the multi-kernel path's bit for bit.
//   combine: the CTA that finishes the last group of a down row block combines that block for
//     every token, in the reference's order (combine.cu).
//
// Ring: weights are issued as soon as an item is known (shared items at once, so their stream
// starts before the router is done); the activation box of a tile joins the same mbarrier when
// its producer has published it.  Lane 0 of each warp issues; a tile about to be consumed is
// issued blockingly, later tiles only when ready, so a warp never waits on work behind its own.
// Every wait is bounded (DEVERR_TIMEOUT_DECODE); on an error every CTA stops at its next item
// boundary, lets its copies land and leaves.  The last CTA to leave zeroes DecodeSync for the
// next call.
#include "common.cuh"
#include "gemv_frags.cuh"
#include "kernels.h"
#include "router_chain.cuh"
#include "topk.cuh"

namespace hymoe {

namespace {

using namespace gemvf;
using namespace rchain;

constexpr int kDThreads = 256, kDWarps = 8;
constexpr int kDRedLd = 9;        // token pitch (floats) of the cross-warp partials
constexpr int kDRouterCtas = 32;  // router CTAs (E / this many experts each)
constexpr int kDSpecCtas = 32;    // CTAs of the certified routing pass
// Certified selection: the K-th selected logit's lower bound must exceed every other expert's
// upper bound by this much (covers the softmax's roundings, see certify_token) and lie within
// this distance of the largest logit (probabilities stay normal numbers).
constexpr double kSpecMargin = 3e-5;
constexpr double kSpecRange = 80.0;

__device__ __forceinline__ uint32_t ld_acquire_gpu_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_gpu_u32(uint32_t* p, uint32_t v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_relaxed_gpu_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// A relaxed load that saw a released value, then this fence: an acquire.
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
__device__ __forceinline__ void red_release_gpu_add(uint32_t* p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t atom_acq_rel_gpu_add(uint32_t* p, uint32_t v) {
    uint32_t old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// Bounded wait until *p >= v (acquire).  false: the budget ran out (error recorded) or another
// CTA already reported an error.
__device__ __noinline__ bool wait_geq(const uint32_t* p, uint32_t v, int* err) {
    const uint64_t t0 = globaltimer_ns();
    uint32_t spins = 0;
    while (ld_acquire_gpu_u32(p) < v) {
        if (spins > 8) __nanosleep(64);  // many warps poll one line: back off after a few tries
        if ((++spins & 31u) == 0) {
            if (*(volatile int*)err != 0) return false;
            if (globaltimer_ns() - t0 > kWaitBudgetNs) {
                atomicOr(err, DEVERR_TIMEOUT_DECODE);
                return false;
            }
        }
    }
    return true;
}

struct Item {
    int kind;  // 0 gate_up, 1 down
    int g;     // group: 0 shared, 1 + j routed
    int rb;    // 128-row weight block
};

template <int WT, int R>
__global__ __launch_bounds__(kDThreads, 1) void decode_kernel(const __grid_constant__ DecodeMaps maps,
                                                              const __grid_constant__ DecodeArgs a) {
    constexpr int TB = tile_bytes(WT);
    extern __shared__ uint8_t dsm_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* xbox = base;                                                // [8 warps][R][1024]
    uint8_t* wbuf = base + kDWarps * R * 1024;                           // [8 warps][R][TB]
    float* red = reinterpret_cast<float*>(wbuf + kDWarps * R * TB);      // [8][128][kDRedLd]
    // The router CTAs stage their rows over the ring before it runs: the barriers live apart.
    __shared__ __align__(8) uint64_t bars[kDWarps * R];
    __shared__ int s_abort, s_last, s_comb, s_claim;
    __shared__ int s_pos[2];  // list positions (tickets) of the current and the next item
    __shared__ int s_cnt[kMaxE];
    __shared__ float s_rs[kDecodeMaxT];
    __shared__ float s_pbuf[kDWarps][kMaxE];
    __shared__ float s_logit[kDecodeMaxT * kMaxE];
    // The weight tile pointers of every slot and (per warp, once the plan is seen) the active
    // slots: the issue path never waits on a global load for them.
    __shared__ const uint8_t* s_wgu[kDecodeMaxE + 1];
    __shared__ const uint8_t* s_wdn[kDecodeMaxE + 1];
    __shared__ int s_act[kDWarps][kDecodeMaxE];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int gq = lane >> 2, c4 = lane & 3;
    const int G = gridDim.x, cta = blockIdx.x;
    const int T = a.T, H = a.H, I = a.I, E = a.E;
    const int NGU = 2 * I / kTileRows, NDN = H / kTileRows, NSH = NGU + NDN;
    const int ks_gu = H / kTileK, ks_dn = I / kTileK;
    DecodeSync* sy = a.sync;
    const int n_router = min(kDRouterCtas, E);
    const int epc = (E + n_router - 1) / n_router;
    const int router0 = G - n_router;      // router CTAs: [router0, G)
    const int xp_cta = NSH % router0;      // writes the fp16 token rows
    // CTAs of the certified routing pass: [spec0, router0), below the router CTAs and above the
    // fp16-row CTA (plain top-K only: the group-limited variants wait for the chains).
    const int n_spec = a.mode.n_group > 0 ? 0 : max(0, min(kDSpecCtas, router0 - xp_cta - 1));
    const int spec0 = router0 - n_spec;

    uint64_t* wb = bars + warp * R;
    uint8_t* wx = xbox + warp * R * 1024;
    uint8_t* ww = wbuf + static_cast<size_t>(warp) * R * TB;
    if (tid == 0) {
        s_abort = 0;
        s_last = 0;
        s_comb = 0;
    }
    if (tid <= a.el) {
        s_wgu[tid] = a.gu[tid];
        s_wdn[tid] = a.dn[tid];
    }
    if (lane == 0)
        for (int r = 0; r < R; ++r) mbar_init(&wb[r], 1);
    fence_mbar_init();
    __syncthreads();

    // ---------------------------------------------------------------- router CTAs
    if (cta >= router0) {
        float* rw = reinterpret_cast<float*>(base);         // [epc][H]
        float* xs = rw + static_cast<size_t>(epc) * H;      // [T][H]
        float* ns = xs + static_cast<size_t>(T) * H;        // [H]
        const int e0 = (cta - router0) * epc;
        const int ne = max(0, min(epc, E - e0));
        const bool norm = a.nrm.rms != nullptr;
        for (int i = tid * 4; i < ne * H; i += kDThreads * 4)
            cp_async16(rw + i, a.Wr + static_cast<size_t>(e0) * H + i);
        for (int i = tid * 4; i < T * H; i += kDThreads * 4) cp_async16(xs + i, a.x + i);
        if (norm) {
            for (int i = tid * 4; i < H; i += kDThreads * 4) cp_async16(ns + i, a.nrm.w + i);
            if (tid < T) s_rs[tid] = a.nrm.rms[tid];
        }
        cp_async_commit();
        cp_async_wait<0>();
        __syncthreads();
        if (norm) {
            norm_slab(xs, T, H, H, s_rs, ns, kDThreads);
            __syncthreads();
        }
        if (warp < ne && lane < T) {
            const float* xr = xs + static_cast<size_t>(lane) * H;
            const float* wr = rw + static_cast<size_t>(warp) * H;
            float acc = 0.f;
#pragma unroll 8
            for (int k = 0; k < H; k += 4)
                acc = chain4(acc, *reinterpret_cast<const float4*>(xr + k), *reinterpret_cast<const float4*>(wr + k));
            const int e = e0 + warp;
            if (a.bias != nullptr) acc = __fadd_rn(acc, a.bias[e]);
            a.logits[static_cast<size_t>(lane) * E + e] = acc;
        }
        __syncthreads();
        if (tid == 0)  // release of this CTA's logits; the last one acquires every CTA's
            s_last = atom_acq_rel_gpu_add(&sy->router_done, 1u) == static_cast<uint32_t>(n_router - 1);
        __syncthreads();
        if (s_last) {
            // Every router CTA is done: the top-K of every token, then the plan.
            for (int i = tid; i < T * E; i += kDThreads) s_logit[i] = __ldcg(a.logits + i);
            if (tid < kMaxE) s_cnt[tid] = 0;
            __syncthreads();
            if (warp < T)
                topk_token(s_logit, warp, E, a.K, a.probs, a.topk_w, a.topk_idx, s_pbuf[warp], s_cnt, a.slot_of,
                           a.mode);
            __syncthreads();
            // The plan comes from here unless the certified pass has published it already; then
            // the chains' selection must be the certified one.
            if (tid == 0) s_claim = static_cast<int>(atomicCAS(&sy->plan_claim, 0u, 2u));
            __syncthreads();
            if (s_claim == 0) {
                if (warp == 0) {  // the routed slots hit, in slot order (el <= 64: two ballots)
                    int n = 0;
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int sl = lane + 32 * h;
                        const bool hit = sl < a.el && s_cnt[sl] > 0;
                        const unsigned b = __ballot_sync(0xffffffffu, hit);
                        const int rank = n + __popc(b & ((1u << lane) - 1u));
                        if (sl < a.el) {
                            sy->j_of[sl] = hit ? rank : -1;
                            if (hit) sy->act_slot[rank] = sl;
                        }
                        n += __popc(b);
                    }
                    if (lane == 0) sy->n_act = static_cast<uint32_t>(n);
                    __syncwarp();
                    // release of the warp's stores and (through the barrier) the top-K outputs
                    if (lane == 0) st_release_gpu_u32(&sy->plan_ready, 1u);
                }
            } else if (warp < T) {
                // the certified pass published the plan (its masks happen before plan_ready)
                bool ok = true;
                if (lane == 0) ok = wait_geq(&sy->plan_ready, 1u, a.err);
                if (__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) {
                    const int sl = lane < a.K ? __ldcg(a.topk_idx + warp * a.K + lane) : -1;
                    uint64_t bit = sl >= 0 ? (1ull << sl) : 0ull;
#pragma unroll
                    for (int o = 16; o; o >>= 1) bit |= __shfl_xor_sync(0xffffffffu, bit, o);
                    if (lane == 0 && bit != __ldcg(reinterpret_cast<const unsigned long long*>(sy->spec_mask + warp)))
                        atomicOr(a.err, DEVERR_SPEC_MISMATCH);
                }
            }
            __syncthreads();
            if (tid == 0) st_release_gpu_u32(&sy->weights_ready, 1u);  // after every top-K store
        }
        // The staging area becomes the ring: order these generic accesses before the copies.
        fence_proxy_async_smem();
        __syncthreads();
    }

    // ---------------------------------------------------------------- certified routing
    // Speculation without risk: every (token, expert) logit is computed in fp64 from the same
    // rounded products the chain adds (x * w rounded to fp32; pre-norm rows normalised with the
    // same roundings), together with a bound on how far the chain's recursive fp32 sum can lie
    // from it: |chain - sum| <= u/(1-u) * sum_k |partial_k| (each rounding of an add is at most
    // u times the rounded partial sum), the partial sums bounded by the fp64 prefix sums plus
    // H*gamma_H*sum|p| (u = 2^-24, gamma_H = H u / (1 - H u)), plus one rounding of the bias add.
    // A token whose K-th selected lower bound exceeds every other upper bound by kSpecMargin has
    // the chains' selection for certain: softmax is monotone, and two logits that far apart
    // (both within kSpecRange of the largest) keep distinct probabilities through fl(l - m), expf
    // (2 ulp) and the division.  If every token is certified, the plan is published from here,
    // long before the chains end; the chains then only supply the weights and their rank order
    // (and check the selection).  A warp per (token, expert) pair, lanes over 32 column chunks.
    if (cta >= spec0 && cta < router0) {
        // Unit = one token x 8 experts: the token row, the 8 router rows (and the norm weights)
        // are staged in shared memory, then warp w takes expert e0 + w, lane l the columns
        // [l * per, (l + 1) * per) in order.  Rows are padded by 4 floats after every per
        // columns so that the lanes' chunk reads spread over the banks.
        const int per = H / 32;                 // columns per lane (H % 128 == 0)
        const int ldp = H + 128;                // padded row (floats)
        const bool norm = a.nrm.rms != nullptr;
        float* sx = reinterpret_cast<float*>(base);  // [ldp] token row
        float* sw = sx + ldp;                        // [8][ldp] router rows
        float* sn = sw + 8 * ldp;                    // [ldp] norm weights
        const int egroups = (E + 7) / 8, n_units = T * egroups;
        for (int un = cta - spec0; un < n_units; un += n_spec) {
            const int t = un / egroups, e0 = (un - t * egroups) * 8, ne = min(8, E - e0);
            for (int i = tid; i < H / 4; i += kDThreads) {
                const int c = 4 * i, pc = c + 4 * (c / per);
                cp_async16(sx + pc, a.x + static_cast<size_t>(t) * H + c);
                if (norm) cp_async16(sn + pc, a.nrm.w + c);
                for (int r = 0; r < ne; ++r) cp_async16(sw + r * ldp + pc, a.Wr + static_cast<size_t>(e0 + r) * H + c);
            }
            cp_async_commit();
            cp_async_wait<0>();
            __syncthreads();
            if (warp < ne) {
                const int e = e0 + warp;
                const int cl = lane * (per + 4);  // this lane's chunk, padded
                const float rms = norm ? __ldg(a.nrm.rms + t) : 1.f;
                auto prod4 = [&](int k, float (&p)[4]) {
                    float4 xv = *reinterpret_cast<const float4*>(sx + cl + k);
                    const float4 wv = *reinterpret_cast<const float4*>(sw + warp * ldp + cl + k);
                    if (norm) {
                        const float4 g = *reinterpret_cast<const float4*>(sn + cl + k);
                        xv = make_float4(__fmul_rn(__fmul_rn(xv.x, rms), g.x), __fmul_rn(__fmul_rn(xv.y, rms), g.y),
                                         __fmul_rn(__fmul_rn(xv.z, rms), g.z), __fmul_rn(__fmul_rn(xv.w, rms), g.w));
                    }
                    p[0] = __fmul_rn(xv.x, wv.x);
                    p[1] = __fmul_rn(xv.y, wv.y);
                    p[2] = __fmul_rn(xv.z, wv.z);
                    p[3] = __fmul_rn(xv.w, wv.w);
                };
                double loc = 0.0, pabs = 0.0;
                for (int k = 0; k < per; k += 4) {
                    float p[4];
                    prod4(k, p);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        loc += static_cast<double>(p[i]);
                        pabs += fabs(static_cast<double>(p[i]));
                    }
                }
                double inc = loc;  // inclusive prefix of the chunk sums over lanes (column order)
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const double v = __shfl_up_sync(0xffffffffu, inc, o);
                    if (lane >= o) inc += v;
                }
                double run = inc - loc, sabs = 0.0;
                for (int k = 0; k < per; k += 4) {
                    float p[4];
                    prod4(k, p);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        run += static_cast<double>(p[i]);
                        sabs += fabs(run);
                    }
                }
#pragma unroll
                for (int o = 16; o; o >>= 1) {
                    pabs += __shfl_xor_sync(0xffffffffu, pabs, o);
                    sabs += __shfl_xor_sync(0xffffffffu, sabs, o);
                }
                const double L = __shfl_sync(0xffffffffu, inc, 31);
                int last = 0;
                if (lane == 0) {
                    const double u = 5.9604644775390625e-8;  // 2^-24
                    const double gH = H * u / (1.0 - H * u);
                    const double bc = u / (1.0 - u) * (sabs + H * gH * pabs) + 1e-9 * (pabs + fabs(L));
                    const double lb = L + (a.bias != nullptr ? static_cast<double>(a.bias[e]) : 0.0);
                    sy->spec_lb[t * E + e] = lb;
                    sy->spec_bd[t * E + e] = bc + u * (fabs(lb) + bc) + 1e-12 * (fabs(lb) + 1.0);
                    last = atom_acq_rel_gpu_add(sy->spec_tok + t, 1u) == static_cast<uint32_t>(E - 1);
                }
                if (__shfl_sync(0xffffffffu, last, 0)) {
                    // This warp completed token t's bounds: certify its selection.
                    double lb0 = -1e300, lb1 = -1e300, bd0 = 0.0, bd1 = 0.0;
                    if (lane < E) {
                        lb0 = __ldcg(sy->spec_lb + t * E + lane);
                        bd0 = __ldcg(sy->spec_bd + t * E + lane);
                    }
                    if (lane + 32 < E) {
                        lb1 = __ldcg(sy->spec_lb + t * E + lane + 32);
                        bd1 = __ldcg(sy->spec_bd + t * E + lane + 32);
                    }
                    bool sel0 = false, sel1 = false;
                    for (int k = 0; k < a.K; ++k) {  // K rounds of arg-max, ties to the lower expert
                        double bv = -1e300;
                        int bi = 1 << 30;
                        if (!sel0 && lane < E) {
                            bv = lb0;
                            bi = lane;
                        }
                        if (!sel1 && lane + 32 < E && (lb1 > bv || bi == (1 << 30))) {
                            bv = lb1;
                            bi = lane + 32;
                        }
#pragma unroll
                        for (int o = 16; o; o >>= 1) {
                            const double ov = __shfl_xor_sync(0xffffffffu, bv, o);
                            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                            if (ov > bv || (ov == bv && oi < bi)) {
                                bv = ov;
                                bi = oi;
                            }
                        }
                        if (bi == lane) sel0 = true;
                        if (bi == lane + 32) sel1 = true;
                    }
                    double lo = 1e300, hi = -1e300, top = -1e300;
                    if (lane < E) {
                        top = lb0 + bd0;
                        if (sel0) lo = lb0 - bd0;
                        else hi = lb0 + bd0;
                    }
                    if (lane + 32 < E) {
                        top = fmax(top, lb1 + bd1);
                        if (sel1) lo = fmin(lo, lb1 - bd1);
                        else hi = fmax(hi, lb1 + bd1);
                    }
#pragma unroll
                    for (int o = 16; o; o >>= 1) {
                        lo = fmin(lo, __shfl_xor_sync(0xffffffffu, lo, o));
                        hi = fmax(hi, __shfl_xor_sync(0xffffffffu, hi, o));
                        top = fmax(top, __shfl_xor_sync(0xffffffffu, top, o));
                    }
                    const bool ok = lo - hi > kSpecMargin && lo - top > -kSpecRange;
                    uint64_t mask = 0;
                    if (sel0) mask |= 1ull << (a.slot_of != nullptr ? __ldg(a.slot_of + lane) : lane);
                    if (sel1) mask |= 1ull << (a.slot_of != nullptr ? __ldg(a.slot_of + lane + 32) : lane + 32);
#pragma unroll
                    for (int o = 16; o; o >>= 1) mask |= __shfl_xor_sync(0xffffffffu, mask, o);
                    int all = 0;
                    if (lane == 0) {
                        sy->spec_mask[t] = mask;
                        if (!ok) atomicOr(&sy->spec_fail, 1u);
                        all = atom_acq_rel_gpu_add(&sy->spec_cert, 1u) == static_cast<uint32_t>(T - 1);
                        // every token decided, none failed, and the chains have not published yet
                        if (all) all = __ldcg(&sy->spec_fail) == 0 && atomicCAS(&sy->plan_claim, 0u, 1u) == 0u;
                    }
                    if (__shfl_sync(0xffffffffu, all, 0)) {
                        // Publish the plan: the union of the certified selections, in slot order.
                        uint64_t uni = 0;
                        for (int tt = 0; tt < T; ++tt)
                            uni |= __ldcg(reinterpret_cast<const unsigned long long*>(sy->spec_mask + tt));
                        int n = 0;
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const int sl = lane + 32 * h;
                            const bool hit = sl < a.el && ((uni >> sl) & 1ull);
                            const unsigned b = __ballot_sync(0xffffffffu, hit);
                            const int rank = n + __popc(b & ((1u << lane) - 1u));
                            if (sl < a.el) {
                                sy->j_of[sl] = hit ? rank : -1;
                                if (hit) sy->act_slot[rank] = sl;
                            }
                            n += __popc(b);
                        }
                        if (lane == 0) sy->n_act = static_cast<uint32_t>(n);
                        __syncwarp();
                        if (lane == 0) st_release_gpu_u32(&sy->plan_ready, 1u);
                    }
                }
            }
            __syncthreads();  // the staged rows are reused by the next unit
        }
        // The staging area becomes the ring: order these generic accesses before the copies.
        fence_proxy_async_smem();
        __syncthreads();
    }

    // ---------------------------------------------------------------- fp16 token rows
    if (cta == xp_cta) {
        const int n4 = T * H / 4;
        for (int i = tid; i < n4; i += kDThreads) {
            const int t = (4 * i) / H, j = 4 * i - t * H;
            const float4 v = norm_row4(__ldg(reinterpret_cast<const float4*>(a.x) + i), a.nrm, t, j);
            const __half2 lo = __floats2half2_rn(v.x, v.y), hi = __floats2half2_rn(v.z, v.w);
            uint2 u;
            u.x = *reinterpret_cast<const uint32_t*>(&lo);
            u.y = *reinterpret_cast<const uint32_t*>(&hi);
            *reinterpret_cast<uint2*>(a.xp + static_cast<size_t>(t) * H + j) = u;
        }
        fence_proxy_async_global();
        __syncthreads();
        if (tid == 0) st_release_gpu_u32(&sy->xp_ready, 1u);
    }

    // ---------------------------------------------------------------- the work list
    // Positions are handed out by a ticket counter in list order: the shared expert's items
    // (no routing needed), then routed gate_up (slot-major), then routed down.  A CTA holds two
    // tickets, the item it works on and the next one, so its warps prefetch the next item's
    // tiles during the current one, and CTAs that finish early take more items.  Items wait
    // only on earlier positions, so with all CTAs resident every wait ends.
    //
    // Lane 0 state: the plan (n_act < 0: not seen yet), readiness caches, and two stream
    // cursors over this CTA's items (weights issued, activations issued; tiles consumed: cq);
    // a tile's slot is its stream count % R.  Readiness that is not known yet is polled once per
    // consumed tile, the flag's load issued before the tile's math and its value used after it;
    // only a tile about to be consumed waits.
    struct Cur {
        int i;             // CTA item index
        int m;             // tile of the item (this warp's share)
        int n;             // this warp's tiles of the item
        int state;         // 1 known, 0 end of the list, -1 not known yet
        Item it;
        const uint8_t* w;  // weight tiles of the item (weight cursor; nullptr: not looked up)
    };
    int n_act = -1;
    bool xp_ok = false;
    bool sh_ok = false;  // the shared expert's gate_up items are known to be done
    uint64_t gu_ok = 0;  // routed groups known done: bit g - 1 for group g (1..64)
    int wq = 0, xq = 0, cq = 0;
    Cur wc{0, 0, 0, -1, {0, 0, 0}, nullptr};
    Cur xc = wc;
    int cur_i = 0;  // this CTA's current item; s_pos holds the tickets of cur_i and cur_i + 1

    auto tiles_of = [&](int kind) {
        const int n = kind ? ks_dn : ks_gu;
        return n > warp ? (n - warp + kDWarps - 1) / kDWarps : 0;
    };
    // position -> item; 1: exists, 0: past the end of the list, -1: unknown until the plan
    auto item_at = [&](int p, Item& it) -> int {
        if (p < NGU) {
            it = {0, 0, p};
            return 1;
        }
        if (p < NSH) {
            it = {1, 0, p - NGU};
            return 1;
        }
        if (n_act < 0) return -1;
        int q = p - NSH;
        if (q < n_act * NGU) {
            it = {0, 1 + q / NGU, q % NGU};
            return 1;
        }
        q -= n_act * NGU;
        if (q < n_act * NDN) {
            it = {1, 1 + q / NDN, q % NDN};
            return 1;
        }
        return 0;
    };
    // Moves a cursor (at the start of item c.i) to the first item with tiles for this warp.
    auto resolve = [&](Cur& c) {
        while (true) {
            if (c.i > cur_i + 1) {  // no ticket yet
                c.state = -1;
                return;
            }
            c.state = item_at(s_pos[c.i & 1], c.it);
            if (c.state != 1) return;
            c.n = tiles_of(c.it.kind);
            c.w = nullptr;
            if (c.n > 0) return;
            ++c.i;
        }
    };
    auto advance = [&](Cur& c) {
        if (++c.m >= c.n) {
            ++c.i;
            c.m = 0;
            resolve(c);
        }
    };
    auto take_plan = [&]() {
        n_act = static_cast<int>(__ldcg(reinterpret_cast<const int*>(&sy->n_act)));
        for (int j = 0; j < n_act; ++j) s_act[warp][j] = __ldcg(sy->act_slot + j);
        if (wc.state < 0) resolve(wc);
        if (xc.state < 0) resolve(xc);
    };
    auto see_plan = [&]() -> bool {  // blocking; false: the wait failed
        if (n_act >= 0) return true;
        if (!wait_geq(&sy->plan_ready, 1u, a.err)) return false;
        take_plan();
        return true;
    };
    // Weights of the weight cursor's tile into its slot (known item, free slot).
    auto issue_w = [&]() {
        if (wc.w == nullptr) {
            const int slot = wc.it.g == 0 ? a.el : s_act[warp][wc.it.g - 1];
            const int nks = wc.it.kind ? ks_dn : ks_gu;
            wc.w = (wc.it.kind ? s_wdn[slot] : s_wgu[slot]) + static_cast<size_t>(wc.it.rb) * nks * TB;
        }
        const int s = wq % R, k = warp + kDWarps * wc.m;
        mbar_arrive_expect_tx(&wb[s], TB + 1024u);
        bulk_load(ww + s * TB, wc.w + static_cast<size_t>(k) * TB, TB, &wb[s]);
        ++wq;
        advance(wc);
    };
    auto x_ready = [&](const Item& it) {
        return it.kind == 0 ? xp_ok : it.g == 0 ? sh_ok : ((gu_ok >> (it.g - 1)) & 1ull) != 0;
    };
    // Activation box of the activation cursor's tile (its weights are issued: xq < wq): 1 issued,
    // 0 its producer has not published it yet (as far as this lane knows), -1 a blocking wait
    // failed.  force: issue without the check (only to let a barrier complete before an early
    // exit; the box then holds stale rows).
    auto issue_x = [&](bool block, bool force) -> int {
        const Item& it = xc.it;
        if (!force && !x_ready(it)) {
            if (!block) return 0;
            if (it.kind == 0) {
                if (!wait_geq(&sy->xp_ready, 1u, a.err)) return -1;
                xp_ok = true;
            } else {
                if (!wait_geq(sy->gu_done + it.g, static_cast<uint32_t>(NGU), a.err)) return -1;
                if (it.g == 0) sh_ok = true;
                else gu_ok |= 1ull << (it.g - 1);
            }
            fence_proxy_async_global();  // the producers' generic stores before this lane's TMA reads
        }
        const int s = xq % R, k = warp + kDWarps * xc.m;
        if (it.kind == 0)
            tma_load_2d(wx + s * 1024, &maps.x, &wb[s], k * kTileK, 0);
        else
            tma_load_2d(wx + s * 1024, &maps.h, &wb[s], k * kTileK, 8 * it.g);
        ++xq;
        advance(xc);
        return 1;
    };
    auto top_up = [&]() {  // lane 0, never blocks
        while (wq < cq + R && wc.state == 1) issue_w();
        while (xq < wq && issue_x(false, false) == 1) {
        }
    };
    // The flag whose value would let top_up go further (nullptr: none), and its target.
    auto poll_target = [&](uint32_t& target) -> const uint32_t* {
        if (xq < wq && !x_ready(xc.it)) {
            target = xc.it.kind == 0 ? 1u : static_cast<uint32_t>(NGU);
            return xc.it.kind == 0 ? &sy->xp_ready : sy->gu_done + xc.it.g;
        }
        if (n_act < 0 && wc.state < 0 && wc.i <= cur_i + 1 && wq < cq + R) {
            target = 1u;
            return &sy->plan_ready;
        }
        return nullptr;
    };
    auto poll_apply = [&](const uint32_t* p, uint32_t target, uint32_t v) {
        if (p == nullptr || v < target) return;
        fence_acq_rel_gpu();
        if (p == &sy->plan_ready) {
            take_plan();
            return;
        }
        if (p == &sy->xp_ready) xp_ok = true;
        else if (p == sy->gu_done) sh_ok = true;
        else gu_ok |= 1ull << static_cast<int>(p - sy->gu_done - 1);
        fence_proxy_async_global();  // the producers' generic stores before this lane's TMA reads
    };

    const int tok_b = col_token<WT>(gq);
    const int t0 = col_token<WT>(2 * c4), t1 = col_token<WT>(2 * c4 + 1);
    for (;; ++cur_i) {
        // Tickets: this item's (taken one item earlier) and the next one's.
        if (tid == 0) {
            if (cur_i == 0) s_pos[0] = static_cast<int>(atomicAdd(&sy->ticket, 1u));
            s_pos[(cur_i + 1) & 1] = static_cast<int>(atomicAdd(&sy->ticket, 1u));
        }
        __syncthreads();
        // The item (the same in every warp: all read the same plan).
        int v = 0;
        Item it{0, 0, 0};
        if (lane == 0) {
            if (wc.state < 0) resolve(wc);
            if (xc.state < 0) resolve(xc);
            v = item_at(s_pos[cur_i & 1], it);
            if (v < 0) v = see_plan() ? item_at(s_pos[cur_i & 1], it) : -2;
            if (v == 1) top_up();
        }
        v = __shfl_sync(0xffffffffu, v, 0);
        it.kind = __shfl_sync(0xffffffffu, it.kind, 0);
        it.g = __shfl_sync(0xffffffffu, it.g, 0);
        it.rb = __shfl_sync(0xffffffffu, it.rb, 0);
        if (__syncthreads_or(v == -2 || s_abort)) break;
        if (v == 0) break;

        float acc[8][4];
#pragma unroll
        for (int g = 0; g < 8; ++g)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[g][j] = 0.f;
        const int per = tiles_of(it.kind);
        bool failed = false;
        for (int m = 0; m < per; ++m) {
            int got = 1;
            const uint32_t* pp = nullptr;
            uint32_t ptarget = 0, pv = 0;
            if (lane == 0) {
                // This tile now: blocking is safe, every earlier item of this CTA is complete.
                while (got && wq <= cq) {
                    if (wc.state == 1) issue_w();
                    else got = 0;  // cannot happen: the current item is known
                }
                while (got && xq <= cq) got = issue_x(true, false) == 1;
                pp = poll_target(ptarget);
                if (pp != nullptr) pv = ld_relaxed_gpu_u32(pp);  // used after the math
                if (got) got = mbar_wait(&wb[cq % R], (cq / R) & 1, a.err, DEVERR_TIMEOUT_DECODE) ? 1 : 0;
            }
            if (!__shfl_sync(0xffffffffu, got, 0)) {
                failed = true;
                break;
            }
            // The tile's words into registers, then the slot goes back to the copy engine
            // (the next copy overlaps this tile's conversion and MMAs).
            const int s = cq % R;  // cq: lane 0's count, the same in every lane here
            const uint8_t* tile = ww + s * TB;
            uint32_t bx[2][2][2];
            x_frags<WT>(wx + s * 1024 + 128 * tok_b, tok_b & 7, c4, bx);
            RawGroup<WT> raw[8];
#pragma unroll
            for (int g = 0; g < 8; ++g) tile_raw<WT>(tile, 16 * g + gq, c4, raw[g]);
            __syncwarp();  // every lane has read the slot
            ++cq;
            if (lane == 0) {
                poll_apply(pp, ptarget, pv);
                top_up();
            }
#pragma unroll
            for (int g = 0; g < 8; ++g) {
                uint32_t af[2][2][4];
                float d[2][2];
                raw_frags<WT>(raw[g], af, d);
#pragma unroll
                for (int b = 0; b < 2; ++b) {
                    float blk[4] = {0.f, 0.f, 0.f, 0.f};
                    mma16816(blk, af[b][0], bx[b][0][0], bx[b][0][1]);
                    mma16816(blk, af[b][1], bx[b][1][0], bx[b][1][1]);
                    acc[g][0] = fmaf(d[b][0], blk[0], acc[g][0]);
                    acc[g][1] = fmaf(d[b][0], blk[1], acc[g][1]);
                    acc[g][2] = fmaf(d[b][1], blk[2], acc[g][2]);
                    acc[g][3] = fmaf(d[b][1], blk[3], acc[g][3]);
                }
            }
        }
        if (failed && lane == 0) s_abort = 1;
        float* rwp = red + warp * kTileRows * kDRedLd;
#pragma unroll
        for (int g = 0; g < 8; ++g) {
            const int r0 = 16 * g + gq;
            rwp[r0 * kDRedLd + t0] = acc[g][0];
            rwp[r0 * kDRedLd + t1] = acc[g][1];
            rwp[(r0 + 8) * kDRedLd + t0] = acc[g][2];
            rwp[(r0 + 8) * kDRedLd + t1] = acc[g][3];
        }
        __syncthreads();
        if (s_abort) break;
        auto sum = [&](int r, int n) {
            float vv = 0.f;
#pragma unroll
            for (int w = 0; w < kDWarps; ++w) vv += red[(w * kTileRows + r) * kDRedLd + n];
            return vv;
        };
        if (it.kind == 0) {
            __half* o = a.hb + static_cast<size_t>(8 * it.g) * I + it.rb * kGluHalf;
            for (int e = tid; e < kGluHalf * T; e += kDThreads) {
                const int j = e % kGluHalf, n = e / kGluHalf;
                o[static_cast<size_t>(n) * I + j] = __float2half_rn(silu_mul(sum(glu_gate_row(j), n), sum(glu_up_row(j), n)));
            }
        } else if (it.g == 0) {
            float* o = a.ysh + it.rb * kTileRows;
            for (int e = tid; e < kTileRows * T; e += kDThreads) {
                const int r = e % kTileRows, n = e / kTileRows;
                o[static_cast<size_t>(n) * H + r] = sum(r, n);
            }
        } else {
            __half* o = a.yr + static_cast<size_t>(8 * (it.g - 1)) * H + it.rb * kTileRows;
            for (int e = tid; e < kTileRows * T; e += kDThreads) {
                const int r = e % kTileRows, n = e / kTileRows;
                o[static_cast<size_t>(n) * H + r] = __float2half_rn(sum(r, n));
            }
        }
        __syncthreads();
        if (tid == 0) {
            // Release of every thread's outputs (ordered before by the barrier).
            if (it.kind == 0) {
                red_release_gpu_add(sy->gu_done + it.g, 1u);
            } else {
                // The last group of this row block combines it (the plan gives the group count).
                if (!see_plan()) {
                    s_abort = 1;
                } else {
                    s_comb = atom_acq_rel_gpu_add(sy->dn_done + it.rb, 1u) == static_cast<uint32_t>(n_act);
                }
            }
        }
        __syncthreads();
        if (s_abort) break;
        if (s_comb) {
            // out = resid + (shared + sum_k w_k y_k), each step rounded (combine.cu's order).  The
            // weights and their rank order come from the chains.
            if (tid == 0 && !wait_geq(&sy->weights_ready, 1u, a.err)) s_abort = 1;
            __syncthreads();
            if (s_abort) break;
            const int K = a.K;
            for (int e = tid; e < kTileRows * T; e += kDThreads) {
                const int r = e % kTileRows, t = e / kTileRows;
                const int col = it.rb * kTileRows + r;
                float rsum = 0.f;
                for (int k = 0; k < K; ++k) {
                    const float w = __ldcg(a.topk_w + t * K + k);
                    if (w != 0.f) {
                        const int j = __ldcg(sy->j_of + __ldcg(a.topk_idx + t * K + k));
                        const __half y = __ldcg(a.yr + (static_cast<size_t>(8 * j) + t) * H + col);
                        rsum = __fadd_rn(rsum, __fmul_rn(w, __half2float(y)));
                    }
                }
                float o = __fadd_rn(__ldcg(a.ysh + static_cast<size_t>(t) * H + col), rsum);
                if (a.resid != nullptr) o = __fadd_rn(a.resid[static_cast<size_t>(t) * H + col], o);
                a.out[static_cast<size_t>(t) * H + col] = o;
            }
            __syncthreads();
            if (tid == 0) s_comb = 0;
        }
        __syncthreads();  // red is free again
    }

    // ---------------------------------------------------------------- leave
    if (lane == 0) {
        // On an early exit: copies issued but not consumed land first (a tile whose weights
        // are in flight gets its activation box too, so that its barrier completes).
        while (xq < wq) issue_x(false, true);
        for (int q = cq; q < wq; ++q) mbar_drain(&wb[q % R], (q / R) & 1);
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        if (atomicAdd(&sy->exit_cnt, 1u) == static_cast<uint32_t>(G - 1)) {
            // Every CTA is done with the block: zero it for the next call.
            sy->router_done = 0;
            sy->xp_ready = 0;
            sy->plan_ready = 0;
            sy->n_act = 0;
            sy->ticket = 0;
            sy->plan_claim = 0;
            sy->weights_ready = 0;
            sy->spec_cert = 0;
            sy->spec_fail = 0;
            for (int t = 0; t < kDecodeMaxT; ++t) sy->spec_tok[t] = 0;
            for (int g = 0; g <= a.el && g <= kDecodeMaxE; ++g) sy->gu_done[g] = 0;
            for (int rb = 0; rb < NDN; ++rb) sy->dn_done[rb] = 0;
            sy->exit_cnt = 0;
            __threadfence();
        }
    }
}

template <int WT, int R>
size_t ring_smem() {
    return static_cast<size_t>(kDWarps) * R * (1024 + tile_bytes(WT)) + sizeof(float) * kDWarps * kTileRows * kDRedLd;
}

template <int WT, int R>
cudaError_t launch_t(const DecodeMaps& maps, const DecodeArgs& a, size_t smem, int n_sms, cudaStream_t st) {
    auto* fn = decode_kernel<WT, R>;
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kDThreads, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorNotSupported;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(n_sms);
    cfg.blockDim = dim3(kDThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, fn, maps, a);
}

}  // namespace

size_t decode_smem(int wtype, int T, int H, int E) {
    if (T < 1 || T > kDecodeMaxT || E < 1 || E > kDecodeMaxE || H % kTileRows != 0 || H / kTileRows > kDecodeMaxRb)
        return 0;
    size_t ring = 0;
    if (wtype == W_Q8_0) ring = ring_smem<W_Q8_0, 2>();
    else if (wtype == W_Q4_0) ring = ring_smem<W_Q4_0, 3>();
    else return 0;
    const int n_router = E < kDRouterCtas ? E : kDRouterCtas;
    const int epc = (E + n_router - 1) / n_router;
    const size_t router = sizeof(float) * static_cast<size_t>(epc + T + 1) * H;
    const size_t spec = sizeof(float) * 10u * static_cast<size_t>(H + 128);
    size_t need = ring > router ? ring : router;
    need = 1024 + (need > spec ? need : spec);
    return need <= 227u * 1024u ? need : 0;
}

cudaError_t launch_decode(const DecodeMaps& maps, const DecodeArgs& a, int wtype, int n_sms, cudaStream_t st) {
    const size_t smem = decode_smem(wtype, a.T, a.H, a.E);
    if (smem == 0 || a.K > 8 || a.el > kDecodeMaxE || (2 * a.I) % kTileRows != 0) return cudaErrorInvalidValue;
    // every position below the routed items must belong to a non-router CTA
    const int n_router = a.E < kDRouterCtas ? a.E : kDRouterCtas;
    if (n_sms - n_router < 1) return cudaErrorNotSupported;
    if (wtype == W_Q8_0) return launch_t<W_Q8_0, 2>(maps, a, smem, n_sms, st);
    return launch_t<W_Q4_0, 3>(maps, a, smem, n_sms, st);
}

}  // namespace hymoe
