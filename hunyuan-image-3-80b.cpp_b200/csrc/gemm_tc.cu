// gemm_tc.cu — grouped expert GEMM on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Replaces the per-(token, expert) matrix-vector loops of swiglu_ffn_f32
// (src/rms_norm.cpp:55-63 gate_up, :81-89 down) with one persistent grouped GEMM per
// projection over all experts (and the shared expert as one more group).
//
// Orientation ("swap AB"): weight rows are the MMA's M dimension and a group's token rows
// are N (16..256, multiple of 16), so a group's last, ragged token tile costs at most 15
// padding columns instead of a padded 128-row M tile.
//
// 2-SM pairs (tcgen05 cta_group::2, clusters of two CTAs on neighbouring SMs): a pair
// tile is 256 weight rows x N tokens x 64 K per stage.  Each CTA dequantises its own
// 128-row weight tile (A half) and TMA-loads its own N/2 token rows (B half); the leader
// CTA issues
//   D[256, N] (fp32, TMEM; each CTA holds its 128 rows) += A[256, 64] * B[N, 64]^T
// as four K=16 tcgen05.mma.cta_group::2.kind::f16 instructions, and its commits arrive
// on both CTAs' barriers.  Per SM this halves the token-operand traffic (L2 -> SMEM and
// SMEM -> tensor core) of a 128 x N single-SM tile.
//
// Warp roles (512 threads per CTA, one CTA per SM, persistent over the work list; warp w
// runs on SM sub-partition w % 4):
//   warp 0      producer: TMA 2-D load of this CTA's B half (128B swizzle) + one bulk copy
//               of its raw GGUF weight tile, both completing on the local full[s]
//   warp 1      TMEM allocation for the pair; in the leader, the MMA issuer
//   warps 2..5  epilogue: tcgen05.ld of this CTA's accumulator rows straight to registers
//               (lane = output row of the tile): gate_up pairs each gate row with its up row
//               in the same warp (tile row order of glu_gate_row / glu_up_row) by one
//               shuffle per token pair, SwiGLU -> fp16; down stores fp32 (shared expert) or
//               fp16 (routed) rows; one coalesced segment per token, no shared memory
//   warps 6-8, 10-12, 14, 15  dequantisers, two groups of four on alternate stages: GGUF
//               Q4_0/Q8_0/F16 tile -> fp16 A half in the canonical K-major 128B-swizzled
//               layout, two (row, GGUF block) entries per thread; then arrive on the leader's
//               a_ready[s].  None runs on sub-partition 1: the MMA issuer (warp 1) shares it
//               only with an epilogue warp and two idle warps (9, 13), because with two
//               dequantisers beside it the issuer's instruction slots, not the tensor core,
//               set the stage period of full tiles (0.448 against 0.352 us per stage)
//   warps 16, 18, 19, 20 (fused expert parallel only, 672 threads; warp 17 idle, again to keep
//               sub-partition 1 to the MMA issuer) communication, beside the MMA
//               pipeline: in gate_up they store this rank's token rows owned by other ranks
//               into the owners' activation matrices (NVLink peer stores), and the producer
//               loads a remote source's rows only after that source's delivery flag; in down
//               they copy each finished item's routed result rows back to the source rank
//               (peer stores into its return matrix), then raise this rank's ready flag.
// Barriers: full[s] (local), a_ready[s] (leader, 8 warp arrivals: the 4 dequant warps of
// the stage's group in each CTA),
// empty[s] / acc_full[b] (both CTAs, from the leader's multicast commits), acc_empty[b]
// (leader, 8 epilogue warp arrivals).  Every wait is bounded in time; on expiry the CTA
// records an error code, unwinds, lets in-flight copies land and releases tensor memory.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>

// Optional pipeline trace (compiled only with -DHYMOE_TRACE): global-timer stamps of the
// first kTraceIters stage iterations of cluster 0, read back by hymoe_trace_read.
#ifdef HYMOE_TRACE
constexpr int kTraceIters = 1024;
__device__ unsigned long long g_trace[2][8][kTraceIters];
#define HY_TRACE(ev, it)                                                   \
    do {                                                                   \
        if (blockIdx.x < 2 && (it) < static_cast<uint32_t>(kTraceIters))   \
            g_trace[blockIdx.x][ev][it] = globaltimer_ns();                \
    } while (0)
extern "C" int hymoe_trace_read(void* host, size_t bytes) {
    return static_cast<int>(cudaMemcpyFromSymbol(host, g_trace, bytes < sizeof(g_trace) ? bytes : sizeof(g_trace)));
}
// Per-item stamps of every pair's MMA issuer in gate_up launches: [pair][item of the pair]
// {first MMA issue, last commit issue, item token rows}.
constexpr int kTracePairs = 80, kTraceItems = 256;
__device__ unsigned long long g_trace_items[kTracePairs][kTraceItems][3];
#define HY_ITEM(glu, cid, j, k, v)                                        \
    do {                                                                 \
        if ((glu) && (cid) < kTracePairs && (j) < kTraceItems)           \
            g_trace_items[cid][j][k] = (v);                              \
    } while (0)
extern "C" int hymoe_trace_items_read(void* host, size_t bytes) {
    return static_cast<int>(cudaMemcpyFromSymbol(host, g_trace_items,
                                                 bytes < sizeof(g_trace_items) ? bytes : sizeof(g_trace_items)));
}
#else
#define HY_TRACE(ev, it) \
    do {                 \
    } while (0)
#define HY_ITEM(glu, cid, j, k, v) \
    do {                           \
    } while (0)
#endif

namespace hymoe {

namespace {

constexpr int kThreads = 512;
constexpr int kEpThreads = 672;    // + four communication warps (fused expert parallel) and an idle one
constexpr int kEpSendCols = 1024;  // columns per send work unit: 128 threads x 8 fp16
constexpr int kABytes = kTileRows * 128;        // 16 KB fp16 A half
constexpr int kBBytes = kMaxBoxRows * 128;      // 16 KB fp16 B half (largest box)
constexpr int kAccCols = 256;
constexpr int kTmemCols = 512;

// Dequantiser index 0..7 of warps 6, 7, 8, 10, 11, 12, 14, 15 (-1 for other warps): the
// dequantisers keep off sub-partition 1, where the MMA issuer runs.
__device__ __forceinline__ int dequant_index(int warp) {
    const int d = warp - 6;
    return (d < 0 || d > 9 || (warp & 3) == 1) ? -1 : d - d / 4;
}

// Communication warp index 0..3 of warps 16, 18, 19, 20 (-1 for other warps).
__device__ __forceinline__ int comm_index(int warp) {
    return warp == 16 ? 0 : (warp >= 18 && warp <= 20) ? warp - 17 : -1;
}

__device__ __forceinline__ bool named_bar_and(int id, int n, bool p) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred pi, po;\n\t"
        "setp.ne.u32 pi, %1, 0;\n\t"
        "bar.red.and.pred po, %2, %3, pi;\n\t"
        "selp.u32 %0, 1, 0, po;\n\t}"
        : "=r"(r)
        : "r"(static_cast<uint32_t>(p)), "r"(id), "r"(n)
        : "memory");
    return r != 0;
}

// Item of round j for SM pair cid of ncl: rounds deal consecutive runs of ncl items, in
// alternating direction ("snake"), so with a size-ordered list every pair's total work stays
// close to the mean.  Every role of a pair walks the same sequence.
__device__ __forceinline__ int gemm_item(int j, int cid, int ncl) {
    return j * ncl + ((j & 1) ? ncl - 1 - cid : cid);
}

// Pair tile width: the item's token count rounded up to the MMA's granularity (16).
__device__ __forceinline__ int pair_n(int rows) {
    const int n = (rows + 15) & ~15;
    return n < 16 ? 16 : (n > 2 * kMaxBoxRows ? 2 * kMaxBoxRows : n);
}

// Smallest TMA box (rows) covering this CTA's half of the pair tile.
__device__ __forceinline__ int box_index(int half) {
    return half <= box_rows(0) ? 0 : half <= box_rows(1) ? 1 : 2;
}

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// ---- dequantisers: entry e = 2 r + b of the raw tile -> row r, chunks 4b..4b+3 of A.

template <int WT>
__device__ __forceinline__ void dequant_entry(const uint8_t* raw, uint8_t* A, int e);

template <>
__device__ __forceinline__ void dequant_entry<W_Q4_0>(const uint8_t* raw, uint8_t* A, int e) {
    const int r = e >> 1, b = e & 1;
    const __half2 d2 = __half2half2(*reinterpret_cast<const __half*>(raw + 2 * e));
    const uint4 q = *reinterpret_cast<const uint4*>(raw + 512 + 16 * e);
    const __half2 off = __float2half2_rn(1032.0f);  // 1024 magic + 8 offset
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
    uint32_t lo[8], hi[8];  // half2 pairs of elements (2i, 2i+1) and (16+2i, 17+2i)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t p0 = __byte_perm(w[i], 0, 0x4140);  // bytes 4i, 4i+1 -> halves
        const uint32_t p1 = __byte_perm(w[i], 0, 0x4342);  // bytes 4i+2, 4i+3
        lo[2 * i] = (p0 & 0x000F000Fu) | 0x64006400u;
        hi[2 * i] = ((p0 >> 4) & 0x000F000Fu) | 0x64006400u;
        lo[2 * i + 1] = (p1 & 0x000F000Fu) | 0x64006400u;
        hi[2 * i + 1] = ((p1 >> 4) & 0x000F000Fu) | 0x64006400u;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        lo[i] = h2_bits(__hmul2(__hsub2(bits_h2(lo[i]), off), d2));
        hi[i] = h2_bits(__hmul2(__hsub2(bits_h2(hi[i]), off), d2));
    }
    uint8_t* row = A;
    *reinterpret_cast<uint4*>(row + sw128_offset(r, 4 * b + 0)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    *reinterpret_cast<uint4*>(row + sw128_offset(r, 4 * b + 1)) = make_uint4(lo[4], lo[5], lo[6], lo[7]);
    *reinterpret_cast<uint4*>(row + sw128_offset(r, 4 * b + 2)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<uint4*>(row + sw128_offset(r, 4 * b + 3)) = make_uint4(hi[4], hi[5], hi[6], hi[7]);
}

template <>
__device__ __forceinline__ void dequant_entry<W_Q8_0>(const uint8_t* raw, uint8_t* A, int e) {
    const int r = e >> 1, b = e & 1;
    const __half2 d2 = __half2half2(*reinterpret_cast<const __half*>(raw + 2 * e));
    const uint4* qp = reinterpret_cast<const uint4*>(raw + 512 + 32 * e);
    const uint4 q0 = qp[0], q1 = qp[1];
    const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    const __half2 off = __float2half2_rn(1152.0f);  // 1024 magic + 128 sign offset
    uint32_t h[16];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        // excess-128 bytes u = q + 128 -> halves 1024 + u (high byte 0x64 from the constant)
        const uint32_t p0 = __byte_perm(w[i], 0x64u, 0x4140);
        const uint32_t p1 = __byte_perm(w[i], 0x64u, 0x4342);
        h[2 * i] = h2_bits(__hmul2(__hsub2(bits_h2(p0), off), d2));
        h[2 * i + 1] = h2_bits(__hmul2(__hsub2(bits_h2(p1), off), d2));
    }
#pragma unroll
    for (int c = 0; c < 4; ++c)
        *reinterpret_cast<uint4*>(A + sw128_offset(r, 4 * b + c)) =
            make_uint4(h[4 * c], h[4 * c + 1], h[4 * c + 2], h[4 * c + 3]);
}

template <>
__device__ __forceinline__ void dequant_entry<W_F16>(const uint8_t* raw, uint8_t* A, int e) {
    const int r = e >> 1, b = e & 1;
    const uint4* src = reinterpret_cast<const uint4*>(raw + r * 128 + b * 64);
#pragma unroll
    for (int c = 0; c < 4; ++c) *reinterpret_cast<uint4*>(A + sw128_offset(r, 4 * b + c)) = src[c];
}


// ---- fused expert parallel: communication warps (128 threads, named barrier 2)

// Bounded wait for a system-scope flag to reach `epoch` (another GPU raises it).
__device__ bool wait_flag_sys(const uint32_t* flag, uint32_t epoch, uint64_t budget_ns, int* err) {
    const uint64_t t0 = globaltimer_ns();
    uint32_t spins = 0;
    while (ld_acquire_sys_u32(flag) < epoch) {
        if ((++spins & 255u) == 0) {
            if (*(volatile int*)err != 0) return false;
            if (globaltimer_ns() - t0 > budget_ns) {
                atomicOr(err, DEVERR_TIMEOUT_PEER);
                return false;
            }
        }
    }
    return true;
}

// gate_up: this rank's pairs owned by other ranks, as fp16 rows of x, into the owners' xp at
// their receive rows  T_d + sum_{s < me} sum_{le} C[s][d * el + le] + p - goff[d * el]
// (p = slot_pos, the pair's expert-sorted position).  Work units: (16-token router chunk,
// 1024-column slice), spread over the grid's CTAs; each thread moves 8 columns of 4 tokens
// at a time (loads first, then the stores).
__device__ void ep_send_rows(const EpFuse& f, int ct, int cta, int n_ctas, int* base_s) {
    const int* C = f.peers.meta[f.me] + kEpCountOff;
    const int ld = f.E + 1;
    if (ct < f.N) {
        int b = C[ct * ld + f.E];  // T of rank ct: its shared rows come first
        for (int s = 0; s < f.me; ++s)
            for (int le = 0; le < f.el; ++le) b += C[s * ld + ct * f.el + le];
        base_s[ct] = b - f.goff[ct * f.el];
    }
    named_bar_sync(2, 128);
    const int n_chunks = (f.T + kRouterTok - 1) / kRouterTok;
    const int n_sl = (f.H + kEpSendCols - 1) / kEpSendCols;
    for (int vb = cta; vb < n_chunks * n_sl; vb += n_ctas) {
        const int c = vb / n_sl, sl = vb - c * n_sl;
        const int t0 = c * kRouterTok, nt = min(kRouterTok, f.T - t0);
        const int j = sl * kEpSendCols + ct * 8;
        if (j >= f.H) continue;
        for (int tb = 0; tb < nt; tb += 4) {
            float4 xv[4][2];
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (tb + u < nt) {
                    const float4* xr = reinterpret_cast<const float4*>(f.x + static_cast<size_t>(t0 + tb + u) * f.H + j);
                    xv[u][0] = norm_row4(xr[0], f.nrm, t0 + tb + u, j);
                    xv[u][1] = norm_row4(xr[1], f.nrm, t0 + tb + u, j + 4);
                }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                if (tb + u >= nt) break;
                const int t = t0 + tb + u;
                const __half2 h0 = __floats2half2_rn(xv[u][0].x, xv[u][0].y), h1 = __floats2half2_rn(xv[u][0].z, xv[u][0].w);
                const __half2 h2 = __floats2half2_rn(xv[u][1].x, xv[u][1].y), h3 = __floats2half2_rn(xv[u][1].z, xv[u][1].w);
                uint4 v;
                v.x = *reinterpret_cast<const uint32_t*>(&h0);
                v.y = *reinterpret_cast<const uint32_t*>(&h1);
                v.z = *reinterpret_cast<const uint32_t*>(&h2);
                v.w = *reinterpret_cast<const uint32_t*>(&h3);
                for (int k = 0; k < f.K; ++k) {
                    const int sl = __ldg(f.topk_idx + t * f.K + k);
                    if (sl & kDroppedPair) continue;  // a pair dropped by the capacity takes no row
                    const int d = sl / f.el;
                    if (d == f.me) continue;
                    const int row = base_s[d] + __ldg(f.slot_pos + t * f.K + k);
                    *reinterpret_cast<uint4*>(f.peers.xp[d] + static_cast<size_t>(row) * f.H + j) = v;
                }
            }
        }
    }
}

// down: after the epilogue has finished item tc (4 warp arrivals on done_items per item), its
// routed result rows [row0, row0 + rows) x this CTA's 128 columns go from yr to the source's
// yret at the source's expert-sorted positions (aux.y + r).  Shared-expert rows stay local.
__device__ bool ep_push_results(const GemmArgs& a, const EpFuse& f, int ct, int cid, int ncl, int rank,
                                int n_items, const uint32_t* done_items, int* err) {
    uint32_t tc = 0;
    for (int w; (w = gemm_item(static_cast<int>(tc), cid, ncl)) < n_items; ++tc) {
        const uint64_t t0 = globaltimer_ns();
        uint32_t spins = 0;
        while (ld_acquire_cta_u32(done_items) < 4u * (tc + 1)) {
            if ((++spins & 63u) == 0) {
                if (*(volatile int*)err != 0) return false;
                if (globaltimer_ns() - t0 > kWaitBudgetNs) {
                    atomicOr(err, DEVERR_TIMEOUT_EPILOGUE);
                    return false;
                }
            }
            __nanosleep(100);
        }
        const int4 item = a.items[w];
        const int rb = 2 * item.y + rank;
        if (rb >= a.n_rb || item.z < a.shared_rows) continue;
        const int2 ax = f.aux[w];
        const __half* src = a.out_r + static_cast<size_t>(item.z) * a.out_ld + rb * kTileRows;
        __half* dst = f.peers.yret[ax.x] + static_cast<size_t>(ax.y) * a.out_ld + rb * kTileRows;
        const int n16 = item.w * (kTileRows / 8);
        for (int i = ct; i < n16; i += 128) {
            const int r = i >> 4, col = (i & 15) * 8;
            const uint4 v = __ldcg(reinterpret_cast<const uint4*>(src + static_cast<size_t>(r) * a.out_ld + col));
            *reinterpret_cast<uint4*>(dst + static_cast<size_t>(r) * a.out_ld + col) = v;
        }
    }
    return true;
}

// Every CTA's communication warps are done: the last CTA raises this rank's flag at
// flag_off on every rank (after a system-scope fence of every CTA's peer stores).
__device__ void ep_finish(const EpFuse& f, int ct, int n_ctas, int flag_off, int* last_s) {
    __threadfence_system();
    named_bar_sync(2, 128);
    if (ct == 0) *last_s = atomicAdd(f.done, 1u) == static_cast<unsigned>(n_ctas - 1);
    named_bar_sync(2, 128);
    if (*last_s) {
        __threadfence_system();
        if (ct < f.N) st_release_sys_u32(reinterpret_cast<uint32_t*>(f.peers.meta[ct]) + flag_off + f.me, f.epoch);
        if (ct == 0) *f.done = 0u;  // every CTA of this launch has counted
    }
}

template <int WT, int STAGES, bool EP>
__global__ void __launch_bounds__(EP ? kEpThreads : kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ GemmMaps maps, const GemmArgs a, const __grid_constant__ EpFuse ep) {
    constexpr int RAW = tile_bytes(WT);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint8_t* sA = smem;
    uint8_t* sB = sA + STAGES * kABytes;
    uint8_t* sRaw = sB + STAGES * kBBytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sRaw + STAGES * RAW);
    uint64_t* full = bars;
    uint64_t* aready = full + STAGES;
    uint64_t* empty = aready + STAGES;
    uint64_t* acc_full = empty + STAGES;
    uint64_t* acc_empty = acc_full + 2;
    uint64_t* mma_done = acc_empty + 2;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(mma_done + 1);
    uint32_t* done_items = tmem_holder + 1;  // epilogue warp arrivals (fused down: 4 per item)
    int* comm_s = reinterpret_cast<int*>(tmem_holder + 2);  // [kEpMaxRanks + 1] comm scratch

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&aready[s], 8);  // 4 dequant warps of each CTA
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 8);
        }
        mbar_init(mma_done, 1);
        if constexpr (EP) *done_items = 0u;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc_2sm(tmem_holder, kTmemCols);
        tmem_relinquish_2sm();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    const int n_items = *a.n_items;
    const int cid = blockIdx.x >> 1, ncl = gridDim.x >> 1;
    int* err = a.err;

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            uint32_t delivered = 0;  // sources whose rows of this call have landed (fused gate_up)
            for (int j = 0, w; ok && (w = gemm_item(j, cid, ncl)) < n_items; ++j) {
                const int4 item = a.items[w];
                if constexpr (EP) {
                    if (a.ep_mode == 1) {
                        const int src = ep.aux[w].x;
                        if (src != ep.me && !((delivered >> src) & 1u)) {
                            const uint32_t* flag = reinterpret_cast<const uint32_t*>(ep.peers.meta[ep.me]) +
                                                   kEpFlagDeliver + src;
                            if (!wait_flag_sys(flag, ep.epoch, ep.budget_ns, err)) {
                                ok = false;
                                break;
                            }
                            fence_proxy_async_global();
                            delivered |= 1u << src;
                        }
                    }
                }
                const int rb = 2 * item.y + static_cast<int>(rank);
                const bool has_tile = rb < a.n_rb;
                const int n = pair_n(item.w), half = n >> 1;
                const int bi = box_index(half);
                const uint32_t bbytes = static_cast<uint32_t>(box_rows(bi)) * 128u;
                const uint8_t* wt = a.wtiles[item.x] + static_cast<size_t>(has_tile ? rb : 0) * a.n_ks * RAW;
                for (int ks = 0; ks < a.n_ks; ++ks, ++it) {
                    const int s = it % STAGES;
                    const uint32_t ph = (it / STAGES) & 1;
                    if (!mbar_wait_poll(&empty[s], ph ^ 1, err, DEVERR_TIMEOUT_PRODUCER)) {
                        ok = false;
                        break;
                    }
                    HY_TRACE(0, it);
                    mbar_arrive_expect_tx(&full[s], bbytes + (has_tile ? RAW : 0));
                    tma_load_2d(sB + s * kBBytes, &maps.b[bi], &full[s], ks * kTileK,
                                item.z + static_cast<int>(rank) * half);
                    if (has_tile)
                        bulk_load(sRaw + s * RAW, wt + static_cast<size_t>(ks) * RAW, RAW, &full[s]);
                }
            }
            // Let every copy this CTA issued land before shared memory goes away.
            const uint32_t first = it > static_cast<uint32_t>(STAGES) ? it - STAGES : 0;
            for (uint32_t j = first; j < it; ++j) mbar_drain(&full[j % STAGES], (j / STAGES) & 1);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer (leader)
        if (leader && lane == 0) {
            uint32_t it = 0, tc = 0;
            bool ok = true;
            for (int w; ok && (w = gemm_item(static_cast<int>(tc), cid, ncl)) < n_items; ++tc) {
                const int4 item = a.items[w];
                const uint32_t idesc = idesc_f16_f32(2 * kTileRows, pair_n(item.w));
                const uint32_t ab = tc & 1, aph = (tc >> 1) & 1;
                if (!mbar_wait(&acc_empty[ab], aph ^ 1, err, DEVERR_TIMEOUT_MMA)) break;
                HY_TRACE(4, tc);
                tc_fence_after();
                const uint32_t d_tmem = tmem + ab * kAccCols;
                for (int ks = 0; ks < a.n_ks; ++ks, ++it) {
                    const int s = it % STAGES;
                    const uint32_t ph = (it / STAGES) & 1;
                    if (!mbar_wait_poll(&aready[s], ph, err, DEVERR_TIMEOUT_MMA)) {
                        ok = false;
                        break;
                    }
                    HY_TRACE(3, it);
                    if (ks == 0) HY_ITEM(a.glu, cid, tc, 0, globaltimer_ns());
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(sA + s * kABytes);
                    const uint32_t b_addr = smem_u32(sB + s * kBBytes);
#pragma unroll
                    for (int kk = 0; kk < kTileK / 16; ++kk)
                        mma_f16_ss_2sm(d_tmem, sw128_kmajor_desc(a_addr + kk * 32),
                                       sw128_kmajor_desc(b_addr + kk * 32), idesc,
                                       (ks | kk) != 0 ? 1u : 0u);
                    mma_commit_2sm_mc(&empty[s], 0x3);
                }
                if (!ok) break;
                mma_commit_2sm_mc(&acc_full[ab], 0x3);
                HY_ITEM(a.glu, cid, tc, 1, globaltimer_ns());
                HY_ITEM(a.glu, cid, tc, 2, static_cast<unsigned long long>(item.w));
            }
            // All pair MMAs complete before either CTA releases tensor memory.
            mma_commit_2sm(mma_done);
            mbar_drain(mma_done, 0);
        }
        __syncwarp();
    } else if (warp < 6) {
        // ------------------------------------------------------------ epilogue
        const int q = warp & 3;            // TMEM lane quarter this warp may access
        const int et = tid - 64;           // 0..127
        const uint32_t acc_empty_leader0 = mapa_shared(&acc_empty[0], 0);
        const uint32_t acc_empty_leader1 = mapa_shared(&acc_empty[1], 0);
        uint32_t tc = 0;
        for (int w; (w = gemm_item(static_cast<int>(tc), cid, ncl)) < n_items; ++tc) {
            const int4 item = a.items[w];
            const int rb = 2 * item.y + static_cast<int>(rank);
            const bool has_tile = rb < a.n_rb;
            const int row0 = item.z, nrows = item.w;
            const uint32_t ab = tc & 1, aph = (tc >> 1) & 1;
            const bool got = mbar_wait(&acc_full[ab], aph, err, DEVERR_TIMEOUT_EPILOGUE);
            if (et == 0) HY_TRACE(5, tc);
            if (!named_bar_and(1, 128, got)) break;
            tc_fence_after();
            const uint32_t d_tmem = tmem + ab * kAccCols + (static_cast<uint32_t>(q * 32) << 16);
            const int nchunks = (nrows + 31) / 32;
            for (int ch = 0; ch < nchunks; ++ch) {
                uint32_t v[32];
                tmem_ld_32x32b_x32(d_tmem + ch * 32, v);
                tmem_ld_wait();
                if (ch == nchunks - 1) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_cluster(ab ? acc_empty_leader1 : acc_empty_leader0);
                }
                if (!has_tile) continue;  // warp-uniform; no staging barrier below either
                if (!a.glu) {
                    // down projection: lane = output column, so for every token the warp's 32
                    // lanes store 32 consecutive values straight from the registers — fp32 for
                    // the shared expert's rows, fp16 for routed results
                    const size_t base = static_cast<size_t>(row0 + ch * 32) * a.out_ld + rb * kTileRows + q * 32 + lane;
                    const int nj = min(32, nrows - ch * 32);
                    if (row0 < a.shared_rows) {
                        float* o = static_cast<float*>(a.out) + base;
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (j < nj) o[static_cast<size_t>(j) * a.out_ld] = __uint_as_float(v[j]);
                    } else {
                        __half* o = a.out_r + base;
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (j < nj) o[static_cast<size_t>(j) * a.out_ld] = __float2half_rn(__uint_as_float(v[j]));
                    }
                    continue;
                }
                // gate_up: lanes 0-15 hold gate rows (output column 16q + lane), lanes 16-31 the
                // matching up rows.  Lanes < 16 finish tokens 0-15 of the chunk, lanes >= 16
                // tokens 16-31; one shuffle per token pair swaps the missing halves.
                const bool gate_lane = lane < 16;
                __half* o = static_cast<__half*>(a.out) + static_cast<size_t>(row0 + ch * 32) * a.out_ld +
                            rb * kGluHalf + 16 * q + (lane & 15);
                const int nj = min(32, nrows - ch * 32);
#pragma unroll
                for (int k = 0; k < 16; ++k) {
                    const float send = __uint_as_float(gate_lane ? v[16 + k] : v[k]);
                    const float recv = __shfl_xor_sync(0xffffffffu, send, 16);
                    const float gt = gate_lane ? __uint_as_float(v[k]) : recv;
                    const float up = gate_lane ? recv : __uint_as_float(v[16 + k]);
                    const int t = gate_lane ? k : 16 + k;
                    if (t < nj) o[static_cast<size_t>(t) * a.out_ld] = __float2half_rn(silu_mul(gt, up));
                }
            }
            if constexpr (EP) {
                if (a.ep_mode == 2) {  // this item's result rows are written: hand them to the comm warps
                    __threadfence_block();
                    __syncwarp();
                    if (lane == 0) red_release_cta_add(done_items, 1u);
                }
            }
        }
    } else if (dequant_index(warp) >= 0) {
        // ------------------------------------------------------------ dequantisers
        // Two groups of four warps take alternate stage slots (slot s to group s & 1), so two
        // stages are converted concurrently; each thread converts entries e and e + 128 of its
        // stage.  Each slot belongs to one group, which therefore waits for the slot's phases
        // strictly in order (with an odd slot count, a split by iteration parity would let
        // both groups use every slot, and a group two phases ahead would pass the parity wait
        // of a phase that has not completed).
        const int dq = dequant_index(warp) * 32 + lane;  // 0..255
        const uint32_t grp = static_cast<uint32_t>(dq >> 7);
        const int e = dq & 127;
        uint32_t it = 0;
        bool ok = true;
        for (int j = 0, w; ok && (w = gemm_item(j, cid, ncl)) < n_items; ++j) {
            const int4 item = a.items[w];
            const bool has_tile = 2 * item.y + static_cast<int>(rank) < a.n_rb;
            for (int ks = 0; ks < a.n_ks; ++ks, ++it) {
                if ((static_cast<uint32_t>(it % STAGES) & 1u) != grp) continue;
                const int s = it % STAGES;
                const uint32_t ph = (it / STAGES) & 1;
                if (!mbar_wait(&full[s], ph, err, DEVERR_TIMEOUT_DEQUANT)) {
                    ok = false;
                    break;
                }
                if (e == 0) HY_TRACE(1, it);
                if (has_tile) {
                    dequant_entry<WT>(sRaw + s * RAW, sA + s * kABytes, e);
                    dequant_entry<WT>(sRaw + s * RAW, sA + s * kABytes, e + 128);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (e == 0) HY_TRACE(2, it);
                if (lane == 0) mbar_arrive_cluster(mapa_shared(&aready[s], 0));
            }
        }
    } else if (comm_index(warp) >= 0) {
        // ------------------------------------------------------------ communication (EP)
        if constexpr (EP) {
            const int ct = comm_index(warp) * 32 + lane;  // 0..127
            if (a.ep_mode == 1) {
                ep_send_rows(ep, ct, blockIdx.x, gridDim.x, comm_s);
                ep_finish(ep, ct, gridDim.x, kEpFlagDeliver, comm_s + kEpMaxRanks);
            } else if (a.ep_mode == 2) {
                // every wait inside is bounded, so all 128 threads arrive here; they agree before
                // the completion barriers (a thread that gave up must not leave the others waiting)
                const bool pushed = ep_push_results(a, ep, ct, cid, ncl, static_cast<int>(rank), n_items,
                                                    done_items, err);
                if (named_bar_and(2, 128, pushed)) ep_finish(ep, ct, gridDim.x, kEpFlagReady, comm_s + kEpMaxRanks);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_2sm(tmem, kTmemCols);
    }
}

template <int WT, int STAGES>
constexpr size_t smem_bytes() {
    // tiles, barriers, then tmem_holder, done_items and the comm scratch (kEpMaxRanks + 1 ints)
    return 1024 + STAGES * (kABytes + kBBytes + tile_bytes(WT)) +
           (3 * STAGES + 5) * 8 + 8 + 4 * (kEpMaxRanks + 1);
}

template <int WT, int STAGES, bool EP>
cudaError_t launch_typed(const GemmMaps& maps, const GemmArgs& a, const EpFuse& ep, int n_sms, cudaStream_t st) {
    constexpr size_t smem = smem_bytes<WT, STAGES>();
    static_assert(smem <= 232448, "shared memory budget");
    auto kern = gemm_tc_kernel<WT, STAGES, EP>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(EP ? kEpThreads : kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    // Persistent grid: as many pairs as can be resident at once.
    static int max_clusters[2][16] = {};
    int& mc = max_clusters[EP ? 1 : 0][WT & 15];
    if (mc == 0) {
        cfg.gridDim = dim3(2 * (n_sms / 2));
        if (cudaOccupancyMaxActiveClusters(&mc, kern, &cfg) != cudaSuccess || mc <= 0) {
            cudaGetLastError();
            mc = n_sms / 2;
        }
    }
    cfg.gridDim = dim3(2 * std::min(mc, n_sms / 2));
    e = cudaLaunchKernelEx(&cfg, kern, maps, a, ep);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gemm_tc(const GemmMaps& maps, const GemmArgs& a, int n_sms, cudaStream_t st,
                           const EpFuse* ep) {
    if (a.ep_mode != 0) {
        if (!ep || ep->N > kEpMaxRanks || ep->K > 8 || ep->aux == nullptr) return cudaErrorInvalidValue;
        switch (a.wtype) {
            case W_Q4_0: return launch_typed<W_Q4_0, 6, true>(maps, a, *ep, n_sms, st);
            case W_Q8_0: return launch_typed<W_Q8_0, 5, true>(maps, a, *ep, n_sms, st);
            case W_F16: return launch_typed<W_F16, 4, true>(maps, a, *ep, n_sms, st);
            default: return cudaErrorInvalidValue;
        }
    }
    const EpFuse none{};
    switch (a.wtype) {
        case W_Q4_0: return launch_typed<W_Q4_0, 6, false>(maps, a, none, n_sms, st);
        case W_Q8_0: return launch_typed<W_Q8_0, 5, false>(maps, a, none, n_sms, st);
        case W_F16: return launch_typed<W_F16, 4, false>(maps, a, none, n_sms, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace hymoe
