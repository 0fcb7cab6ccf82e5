// ep_p2p.cu — expert-parallel dispatch and combine over NVLink peer memory.
//
// Every rank maps the other ranks' activation matrix (xp, fp16), routed-result matrix (yr,
// fp16), return matrix (yret, fp16) and metadata block (count matrix + flags) into its address
// space (CUDA IPC).  One call, on every rank:
//
//   ep_counts_kernel    my per-expert pair counts and my token count -> C[me] of every rank;
//                       count flag; wait for every rank's count flag (bounded)
//   dispatch            each pair's token row (fp16) goes straight into its owner's xp at its
//                       final receive row (P2P stores), then this rank's delivery flag is
//                       raised on every rank.  Tensor-core calls: ep_local_kernel writes the
//                       local rows before the GEMM and the gate_up GEMM's communication warps
//                       send the rest while it computes; decode-size calls: ep_scatter_kernel
//   (local GEMMs over rows [0, T + received); the tensor-core producer waits per source for
//    its delivery flag, the decode path waits for all of them first, ep_wait_kernel)
//   return              each routed result row goes back into its source's yret at the
//                       source's expert-sorted position of the pair, then this rank's ready
//                       flag is raised on every rank: the down GEMM's communication warps
//                       (tensor core) or ep_push_kernel (decode)
//   combine             wait for every rank's ready flag (bounded), then the local combine
//                       over yret (the same kernel and operation order as on one GPU)
//
// Receive layout: rows [0, T) the shared expert's local tokens, then the rows of source rank
// 0, 1, ..., each in (local expert, source token) order.  A source places its pair (t, k)
// with slot e (owner d = e / el) and expert-sorted position p at
//   base(d, me) + p - goff[d * el],  base(d, me) = T_d + sum_{s < me} sum_{le} C[s][d * el + le]
// Flags carry the call's epoch (strictly increasing, the same on every rank) and are compared
// with >=, so they never need resetting.  Ordering between calls needs no extra flags: a rank
// starts writing a peer's xp (next call) only after its own combine of this call, which waited
// for every rank's ready flag, raised after that rank's GEMMs read their xp; an owner writes a
// source's yret in the next call only for rows that source delivered in the next call, i.e.
// after that source's combine of this call.
#include "common.cuh"
#include "kernels.h"

namespace hymoe {

namespace {

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded wait until flags[i] >= epoch for i in [0, n).  Returns false (and records
// DEVERR_TIMEOUT_PEER) when the budget runs out or another waiter already failed.
__device__ bool wait_flags(const uint32_t* flags, int n, uint32_t epoch, uint64_t budget_ns, int* err) {
    const uint64_t t0 = globaltimer_ns();
    for (int i = 0; i < n; ++i) {
        uint32_t spins = 0;
        while (ld_acquire_sys(flags + i) < epoch) {
            if ((++spins & 255u) == 0) {
                if (*(volatile int*)err != 0) return false;
                if (globaltimer_ns() - t0 > budget_ns) {
                    atomicOr(err, DEVERR_TIMEOUT_PEER);
                    return false;
                }
            }
        }
    }
    return true;
}

__global__ void ep_counts_kernel(EpPeers peers, int N, int me, int E, int T, const int* __restrict__ gcnt,
                                 uint32_t epoch, uint64_t budget_ns, int* err) {
    const int tid = threadIdx.x;
    for (int d = 0; d < N; ++d) {
        int* dst = peers.meta[d] + kEpCountOff + me * (E + 1);
        for (int e = tid; e <= E; e += blockDim.x) dst[e] = e < E ? gcnt[e] : T;
    }
    __threadfence_system();
    __syncthreads();
    if (tid < N) st_release_sys(reinterpret_cast<uint32_t*>(peers.meta[tid]) + kEpFlagCount + me, epoch);
    if (tid == 0) {
        const uint32_t* mine = reinterpret_cast<const uint32_t*>(peers.meta[me]) + kEpFlagCount;
        wait_flags(mine, N, epoch, budget_ns, err);
    }
}

// This rank's choice record (pairs per (choice k, slot), then its token count) into `rec`
// (one CTA; shared-memory counters).
__device__ void choice_record(const int* __restrict__ topk_idx, int T, int K, int E, int* rec) {
    __shared__ int cnt[kEpMaxK * 64];
    for (int i = threadIdx.x; i < kEpMaxK * E; i += blockDim.x) cnt[i] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < T * K; i += blockDim.x) atomicAdd(&cnt[(i % K) * E + topk_idx[i]], 1);
    __syncthreads();
    for (int i = threadIdx.x; i < kEpMaxK * E; i += blockDim.x) rec[i] = cnt[i];
    if (threadIdx.x == 0) rec[kEpMaxK * E] = T;
}

__global__ void choice_record_kernel(const int* __restrict__ topk_idx, int T, int K, int E, int* rec) {
    choice_record(topk_idx, T, K, E, rec);
}

// Peer memory: the record goes to every rank's choice records (slot `me`), then this rank's
// choice flag is raised on every rank and every rank's flag is awaited (bounded).
__global__ void ep_choice_kernel(EpPeers peers, int N, int me, int E, int K, int T, const int* __restrict__ topk_idx,
                                 uint32_t epoch, uint64_t budget_ns, int* err) {
    const int rl = ep_choice_rec(E);
    int* mine = peers.meta[me] + ep_choice_off(E) + me * rl;
    choice_record(topk_idx, T, K, E, mine);
    __syncthreads();
    for (int d = 0; d < N; ++d) {
        if (d == me) continue;
        int* dst = peers.meta[d] + ep_choice_off(E) + me * rl;
        for (int i = threadIdx.x; i < rl; i += blockDim.x) dst[i] = mine[i];
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x < N)
        st_release_sys(reinterpret_cast<uint32_t*>(peers.meta[threadIdx.x]) + kEpFlagChoice + me, epoch);
    if (threadIdx.x == 0) {
        const uint32_t* flags = reinterpret_cast<const uint32_t*>(peers.meta[me]) + kEpFlagChoice;
        wait_flags(flags, N, epoch, budget_ns, err);
    }
}

// Grid (router chunk of 16 tokens, column slice of 256); 128 threads.  slot_pos[t, k]
// receives the pair's expert-sorted position (its row in this rank's yret).
constexpr int kEpCols = 256;

__global__ __launch_bounds__(128) void ep_scatter_kernel(
    EpPeers peers, int N, int me, int E, int el, int T, int H, int K, const float* __restrict__ x,
    const int* __restrict__ topk_idx, const int* __restrict__ chunk_base, const int* __restrict__ goff,
    int* __restrict__ slot_pos, unsigned int* done_ctas, uint32_t epoch, RowNorm nrm) {
    __shared__ int sidx[kRouterTok][8];
    __shared__ int srow[kRouterTok][8];
    __shared__ int base[kEpMaxRanks];
    __shared__ bool last;
    const int c = blockIdx.x, t0 = c * kRouterTok, tid = threadIdx.x;
    const int nt = min(kRouterTok, T - t0);
    const int* C = peers.meta[me] + kEpCountOff;  // [N][E + 1], every rank's counts (local copy)
    if (tid < N) {
        int b = C[tid * (E + 1) + E];  // T of rank tid: its shared rows come first
        for (int s = 0; s < me; ++s)
            for (int le = 0; le < el; ++le) b += C[s * (E + 1) + tid * el + le];
        base[tid] = b;
    }
    {
        const int tt = tid >> 3, k = tid & 7;
        const int v = (tt < nt && k < K) ? topk_idx[(t0 + tt) * K + k] : -1;
        sidx[tt][k] = v >= 0 && (v & kDroppedPair) ? -1 : v;  // a dropped pair takes no row
    }
    __syncthreads();
    {
        const int tt = tid >> 3, k = tid & 7;
        if (tt < nt && k < K) {
            const int e = sidx[tt][k];
            int pos = -1;
            srow[tt][k] = -1;
            if (e >= 0) {
                int rank = 0;
                for (int p = 0; p < tt; ++p)
                    for (int kk = 0; kk < K; ++kk) rank += sidx[p][kk] == e;
                const int d = e / el;
                pos = chunk_base[c * E + e] + rank;  // expert-sorted position of the pair
                srow[tt][k] = base[d] + pos - goff[d * el];
            }
            if (blockIdx.y == 0) slot_pos[(t0 + tt) * K + k] = pos;
        }
    }
    __syncthreads();
    const int j = blockIdx.y * kEpCols + (tid & 31) * 8;
    if (j < H) {
        for (int tt = tid >> 5; tt < nt; tt += 4) {
            const float* xr = x + static_cast<size_t>(t0 + tt) * H;
            const float4 a = norm_row4(*reinterpret_cast<const float4*>(xr + j), nrm, t0 + tt, j);
            const float4 b = norm_row4(*reinterpret_cast<const float4*>(xr + j + 4), nrm, t0 + tt, j + 4);
            const __half2 h0 = __floats2half2_rn(a.x, a.y), h1 = __floats2half2_rn(a.z, a.w);
            const __half2 h2 = __floats2half2_rn(b.x, b.y), h3 = __floats2half2_rn(b.z, b.w);
            uint4 v;
            v.x = *reinterpret_cast<const uint32_t*>(&h0);
            v.y = *reinterpret_cast<const uint32_t*>(&h1);
            v.z = *reinterpret_cast<const uint32_t*>(&h2);
            v.w = *reinterpret_cast<const uint32_t*>(&h3);
            for (int k = 0; k < K; ++k) {
                if (sidx[tt][k] < 0) continue;
                const int d = sidx[tt][k] / el;
                *reinterpret_cast<uint4*>(peers.xp[d] + static_cast<size_t>(srow[tt][k]) * H + j) = v;
            }
            *reinterpret_cast<uint4*>(peers.xp[me] + static_cast<size_t>(t0 + tt) * H + j) = v;
        }
    }
    // Delivery: the last CTA to finish raises this rank's flag on every rank.
    __threadfence_system();
    __syncthreads();
    if (tid == 0) last = atomicAdd(done_ctas, 1u) == gridDim.x * gridDim.y - 1;
    __syncthreads();
    if (last) {
        __threadfence_system();
        if (tid < N) st_release_sys(reinterpret_cast<uint32_t*>(peers.meta[tid]) + kEpFlagDeliver + me, epoch);
        if (tid == 0) *done_ctas = 0u;  // every CTA of this launch has counted
    }
}

// Fused expert parallel, before the GEMMs.  Grid (router chunk, column slice of 256), 128
// threads.  slot_pos[t, k] = the pair's expert-sorted position p (the row its result returns
// to in this rank's yret); every token row goes to rows [0, T) of this rank's xp (the shared
// expert's rows) and each pair this rank owns to its receive row
//   T + sum_{s < me} sum_{le} C[s][me * el + le] + p - goff[me * el];
// pairs owned elsewhere are sent by the gate_up GEMM's communication warps.
__global__ __launch_bounds__(128) void ep_local_kernel(
    EpPeers peers, int N, int me, int E, int el, int T, int H, int K, const float* __restrict__ x,
    const int* __restrict__ topk_idx, const int* __restrict__ chunk_base, const int* __restrict__ goff,
    int* __restrict__ slot_pos, RowNorm nrm) {
    __shared__ int sidx[kRouterTok][8];
    __shared__ int srow[kRouterTok][8];
    __shared__ int base;
    const int c = blockIdx.x, t0 = c * kRouterTok, tid = threadIdx.x;
    const int nt = min(kRouterTok, T - t0);
    if (tid == 0) {
        const int* C = peers.meta[me] + kEpCountOff;
        int b = T;
        for (int s = 0; s < me; ++s)
            for (int le = 0; le < el; ++le) b += C[s * (E + 1) + me * el + le];
        base = b - goff[me * el];
    }
    {
        const int tt = tid >> 3, k = tid & 7;
        const int v = (tt < nt && k < K) ? topk_idx[(t0 + tt) * K + k] : -1;
        sidx[tt][k] = v >= 0 && (v & kDroppedPair) ? -1 : v;  // a dropped pair takes no row
    }
    __syncthreads();
    {
        const int tt = tid >> 3, k = tid & 7;
        if (tt < nt && k < K) {
            const int e = sidx[tt][k];
            int pos = -1;
            srow[tt][k] = -1;
            if (e >= 0) {
                int rank = 0;
                for (int p = 0; p < tt; ++p)
                    for (int kk = 0; kk < K; ++kk) rank += sidx[p][kk] == e;
                pos = chunk_base[c * E + e] + rank;
                srow[tt][k] = e / el == me ? base + pos : -1;
            }
            if (blockIdx.y == 0) slot_pos[(t0 + tt) * K + k] = pos;
        }
    }
    __syncthreads();
    const int j = blockIdx.y * kEpCols + (tid & 31) * 8;
    if (j >= H) return;
    __half* xp = peers.xp[me];
    for (int tt = tid >> 5; tt < nt; tt += 4) {
        const float* xr = x + static_cast<size_t>(t0 + tt) * H;
        const float4 a = norm_row4(*reinterpret_cast<const float4*>(xr + j), nrm, t0 + tt, j);
        const float4 b = norm_row4(*reinterpret_cast<const float4*>(xr + j + 4), nrm, t0 + tt, j + 4);
        const __half2 h0 = __floats2half2_rn(a.x, a.y), h1 = __floats2half2_rn(a.z, a.w);
        const __half2 h2 = __floats2half2_rn(b.x, b.y), h3 = __floats2half2_rn(b.z, b.w);
        uint4 v;
        v.x = *reinterpret_cast<const uint32_t*>(&h0);
        v.y = *reinterpret_cast<const uint32_t*>(&h1);
        v.z = *reinterpret_cast<const uint32_t*>(&h2);
        v.w = *reinterpret_cast<const uint32_t*>(&h3);
        for (int k = 0; k < K; ++k) {
            const int row = srow[tt][k];
            if (row >= 0) *reinterpret_cast<uint4*>(xp + static_cast<size_t>(row) * H + j) = v;
        }
        *reinterpret_cast<uint4*>(xp + static_cast<size_t>(t0 + tt) * H + j) = v;
    }
}

__global__ void ep_wait_kernel(EpPeers peers, int N, int me, int flag_off, uint32_t epoch, uint64_t budget_ns,
                               int* err) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    wait_flags(reinterpret_cast<const uint32_t*>(peers.meta[me]) + flag_off, N, epoch, budget_ns, err);
}

// Raise this rank's flag at flag_off on every rank, after all its earlier work on the stream.
__global__ void ep_raise_kernel(EpPeers peers, int N, int me, int flag_off, uint32_t epoch) {
    __threadfence_system();
    if (threadIdx.x < N)
        st_release_sys(reinterpret_cast<uint32_t*>(peers.meta[threadIdx.x]) + flag_off + me, epoch);
}

// Decode-size calls: every received segment's result rows (yr, fp16) into its source's yret
// at the source's expert-sorted positions (seg_ret), then the last CTA raises this rank's ready
// flag on every rank.  segs[0] is the shared expert's (local, not returned).
__global__ __launch_bounds__(256) void ep_push_kernel(EpPeers peers, int N, int me, const int4* __restrict__ segs,
                                                      const int* __restrict__ seg_ret,
                                                      const int* __restrict__ n_segs, int H,
                                                      unsigned int* done_ctas, uint32_t epoch) {
    __shared__ bool last;
    const int ns = *n_segs;
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (int i = 1; i < ns; ++i) {
        const int4 sg = segs[i];
        const uint4* src = reinterpret_cast<const uint4*>(peers.yr[me] + static_cast<size_t>(sg.y) * H);
        uint4* dst = reinterpret_cast<uint4*>(peers.yret[sg.w] + static_cast<size_t>(seg_ret[i]) * H);
        const size_t n16 = static_cast<size_t>(sg.z) * H / 8;
        for (size_t q = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; q < n16; q += stride)
            dst[q] = __ldcg(src + q);
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(done_ctas, 1u) == gridDim.x - 1;
    __syncthreads();
    if (last) {
        __threadfence_system();
        if (threadIdx.x < N) st_release_sys(reinterpret_cast<uint32_t*>(peers.meta[threadIdx.x]) + kEpFlagReady + me, epoch);
        if (threadIdx.x == 0) *done_ctas = 0u;
    }
}

}  // namespace

cudaError_t launch_ep_counts(const EpPeers& p, int N, int me, int E, int T, const int* gcnt, uint32_t epoch,
                             uint64_t budget_ns, int* err, cudaStream_t st) {
    if (N > kEpMaxRanks) return cudaErrorInvalidValue;
    ep_counts_kernel<<<1, 128, 0, st>>>(p, N, me, E, T, gcnt, epoch, budget_ns, err);
    return cudaGetLastError();
}

cudaError_t launch_ep_choice_counts(const EpPeers& p, int N, int me, int E, int K, int T, const int* topk_idx,
                                    uint32_t epoch, uint64_t budget_ns, int* err, cudaStream_t st) {
    if (E > 64 || K > kEpMaxK || N > kEpMaxRanks) return cudaErrorInvalidValue;
    ep_choice_kernel<<<1, 256, 0, st>>>(p, N, me, E, K, T, topk_idx, epoch, budget_ns, err);
    return cudaGetLastError();
}

cudaError_t launch_choice_record(const int* topk_idx, int T, int K, int E, int* rec, cudaStream_t st) {
    if (E > 64 || K > kEpMaxK) return cudaErrorInvalidValue;
    choice_record_kernel<<<1, 256, 0, st>>>(topk_idx, T, K, E, rec);
    return cudaGetLastError();
}

cudaError_t launch_ep_scatter(const EpPeers& p, int N, int me, int E, int el, int T, int H, int K, const float* x,
                              const int* topk_idx, const int* chunk_base, const int* goff, int* slot_pos,
                              unsigned int* done_ctas, uint32_t epoch, cudaStream_t st, const RowNorm& nrm) {
    if (T <= 0) return cudaErrorInvalidValue;  // a rank without tokens raises its flag directly
    dim3 grid((T + kRouterTok - 1) / kRouterTok, (H + kEpCols - 1) / kEpCols);
    ep_scatter_kernel<<<grid, 128, 0, st>>>(p, N, me, E, el, T, H, K, x, topk_idx, chunk_base, goff, slot_pos,
                                            done_ctas, epoch, nrm);
    return cudaGetLastError();
}

cudaError_t launch_ep_local(const EpPeers& p, int N, int me, int E, int el, int T, int H, int K, const float* x,
                            const int* topk_idx, const int* chunk_base, const int* goff, int* slot_pos,
                            cudaStream_t st, const RowNorm& nrm) {
    (void)N;
    if (T <= 0) return cudaSuccess;
    dim3 grid((T + kRouterTok - 1) / kRouterTok, (H + kEpCols - 1) / kEpCols);
    ep_local_kernel<<<grid, 128, 0, st>>>(p, N, me, E, el, T, H, K, x, topk_idx, chunk_base, goff, slot_pos, nrm);
    return cudaGetLastError();
}

cudaError_t launch_ep_wait(const EpPeers& p, int N, int me, int flag_off, uint32_t epoch, uint64_t budget_ns,
                           int* err, cudaStream_t st) {
    ep_wait_kernel<<<1, 32, 0, st>>>(p, N, me, flag_off, epoch, budget_ns, err);
    return cudaGetLastError();
}

cudaError_t launch_ep_raise(const EpPeers& p, int N, int me, int flag_off, uint32_t epoch, cudaStream_t st) {
    ep_raise_kernel<<<1, 32, 0, st>>>(p, N, me, flag_off, epoch);
    return cudaGetLastError();
}

cudaError_t launch_ep_push(const EpPeers& p, int N, int me, const int4* segs, const int* seg_ret, const int* n_segs,
                           int H, unsigned int* done_ctas, uint32_t epoch, int n_sms, cudaStream_t st) {
    ep_push_kernel<<<n_sms, 256, 0, st>>>(p, N, me, segs, seg_ret, n_segs, H, done_ctas, epoch);
    return cudaGetLastError();
}

}  // namespace hymoe
