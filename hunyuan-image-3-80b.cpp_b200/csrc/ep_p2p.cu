// ep_p2p.cu — expert-parallel dispatch and combine over NVLink peer memory.
//
// Every rank maps the other ranks' activation matrix (xp, fp16), routed-result matrix (yr,
// fp16) and metadata block (count matrix + flags) into its address space (CUDA IPC).  One call:
//
//   ep_counts_kernel    my per-expert pair counts and my token count -> C[me] of every rank;
//                       count flag; wait for every rank's count flag (bounded)
//   ep_scatter_kernel   each token row, converted to fp16 once, goes straight into the
//                       owner's xp at its final row (P2P stores); the last CTA raises this
//                       rank's delivery flag on every rank
//   ep_wait_kernel      wait for every rank's delivery flag (bounded): xp is complete
//   (local GEMMs over rows [0, T + received))
//   ep_raise_kernel     raise this rank's "results ready" flag on every rank
//   ep_combine_kernel   wait for every owner's ready flag (bounded), then the weighted sum
//                       reads each routed result directly from its owner's yr (P2P loads)
//
// Receive layout (same as the NCCL path): rows [0, T) the shared expert's local tokens, then
// the rows of source rank 0, 1, ..., each in (local expert, source token) order.  A source
// places its pair (t, k) with expert e (owner d = e / el) at
//   base(d, me) + (sorted position of the pair among my pairs) - goff[d * el]
//   base(d, me) = T_d + sum_{s < me} sum_{le} C[s][d * el + le]
// Flags carry the call's epoch (strictly increasing, the same on every rank) and are compared
// with >=, so they never need resetting.  Ordering between calls needs no extra flags: a rank
// starts writing a peer's xp (next call) only after its own combine finished reading every
// owner's yr, which waited for every owner's ready flag, raised after that owner's GEMMs.
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

// Grid (router chunk of 16 tokens, column slice of 256); 128 threads.  slot_pos[t, k]
// receives the pair's row in its owner's matrices.
constexpr int kEpCols = 256;

__global__ __launch_bounds__(128) void ep_scatter_kernel(
    EpPeers peers, int N, int me, int E, int el, int T, int H, int K, const float* __restrict__ x,
    const int* __restrict__ topk_idx, const int* __restrict__ chunk_base, const int* __restrict__ goff,
    int* __restrict__ slot_pos, unsigned int* done_ctas, uint32_t epoch) {
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
        sidx[tt][k] = (tt < nt && k < K) ? topk_idx[(t0 + tt) * K + k] : -1;
    }
    __syncthreads();
    {
        const int tt = tid >> 3, k = tid & 7;
        if (tt < nt && k < K) {
            const int e = sidx[tt][k];
            int rank = 0;
            for (int p = 0; p < tt; ++p)
                for (int kk = 0; kk < K; ++kk) rank += sidx[p][kk] == e;
            const int d = e / el;
            const int row = base[d] + chunk_base[c * E + e] + rank - goff[d * el];
            srow[tt][k] = row;
            if (blockIdx.y == 0) slot_pos[(t0 + tt) * K + k] = row;
        }
    }
    __syncthreads();
    const int j = blockIdx.y * kEpCols + (tid & 31) * 8;
    if (j < H) {
        for (int tt = tid >> 5; tt < nt; tt += 4) {
            const float* xr = x + static_cast<size_t>(t0 + tt) * H;
            const float4 a = *reinterpret_cast<const float4*>(xr + j);
            const float4 b = *reinterpret_cast<const float4*>(xr + j + 4);
            const __half2 h0 = __floats2half2_rn(a.x, a.y), h1 = __floats2half2_rn(a.z, a.w);
            const __half2 h2 = __floats2half2_rn(b.x, b.y), h3 = __floats2half2_rn(b.z, b.w);
            uint4 v;
            v.x = *reinterpret_cast<const uint32_t*>(&h0);
            v.y = *reinterpret_cast<const uint32_t*>(&h1);
            v.z = *reinterpret_cast<const uint32_t*>(&h2);
            v.w = *reinterpret_cast<const uint32_t*>(&h3);
            for (int k = 0; k < K; ++k) {
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

// out[t] = resid[t] + (y_shared[t] + sum_k w[t,k] * yr_owner(k)[slot_pos[t,k]]), the owners'
// fp16 rows read over NVLink (16 bytes per load); the same operation order as combine_kernel.
// Grid (H / 1024, T), 128 threads x 8 columns.
__global__ __launch_bounds__(128) void ep_combine_kernel(EpPeers peers, int N, int me, int el,
                                                         const int* __restrict__ topk_idx,
                                                         const int* __restrict__ slot_pos,
                                                         const float* __restrict__ topk_w,
                                                         const float* __restrict__ y_shared,
                                                         const float* resid, float* out, int H, int K,
                                                         uint32_t epoch, uint64_t budget_ns, int* err) {
    __shared__ int ok;
    if (threadIdx.x == 0)
        ok = wait_flags(reinterpret_cast<const uint32_t*>(peers.meta[me]) + kEpFlagReady, N, epoch, budget_ns, err)
                 ? 1 : 0;
    __syncthreads();
    if (!ok) return;
    const int t = blockIdx.y;
    const int j = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
    if (j >= H) return;
    uint4 u[8];
    float w[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        if (k < K) {
            const int d = __ldg(topk_idx + t * K + k) / el;
            const int row = __ldg(slot_pos + t * K + k);
            w[k] = __ldg(topk_w + t * K + k);
            u[k] = *reinterpret_cast<const uint4*>(peers.yr[d] + static_cast<size_t>(row) * H + j);
        }
    }
    const float* sr = y_shared + static_cast<size_t>(t) * H + j;
    const float4 s0 = *reinterpret_cast<const float4*>(sr), s1 = *reinterpret_cast<const float4*>(sr + 4);
    const float s[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    float h[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (resid != nullptr) {
        const float* hr = resid + static_cast<size_t>(t) * H + j;
        const float4 h0 = *reinterpret_cast<const float4*>(hr), h1 = *reinterpret_cast<const float4*>(hr + 4);
        h[0] = h0.x; h[1] = h0.y; h[2] = h0.z; h[3] = h0.w;
        h[4] = h1.x; h[5] = h1.y; h[6] = h1.z; h[7] = h1.w;
    }
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        float r = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            if (k < K) {
                const uint32_t wd = i < 2 ? u[k].x : i < 4 ? u[k].y : i < 6 ? u[k].z : u[k].w;
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&wd));
                r = __fadd_rn(r, __fmul_rn(w[k], (i & 1) ? f.y : f.x));
            }
        }
        o[i] = __fadd_rn(s[i], r);
        if (resid != nullptr) o[i] = __fadd_rn(h[i], o[i]);
    }
    float* orow = out + static_cast<size_t>(t) * H + j;
    *reinterpret_cast<float4*>(orow) = make_float4(o[0], o[1], o[2], o[3]);
    *reinterpret_cast<float4*>(orow + 4) = make_float4(o[4], o[5], o[6], o[7]);
}

}  // namespace

cudaError_t launch_ep_counts(const EpPeers& p, int N, int me, int E, int T, const int* gcnt, uint32_t epoch,
                             uint64_t budget_ns, int* err, cudaStream_t st) {
    if (N > kEpMaxRanks) return cudaErrorInvalidValue;
    ep_counts_kernel<<<1, 128, 0, st>>>(p, N, me, E, T, gcnt, epoch, budget_ns, err);
    return cudaGetLastError();
}

cudaError_t launch_ep_scatter(const EpPeers& p, int N, int me, int E, int el, int T, int H, int K, const float* x,
                              const int* topk_idx, const int* chunk_base, const int* goff, int* slot_pos,
                              unsigned int* done_ctas, uint32_t epoch, cudaStream_t st) {
    if (T <= 0) return cudaErrorInvalidValue;  // a rank without tokens raises its flag directly
    dim3 grid((T + kRouterTok - 1) / kRouterTok, (H + kEpCols - 1) / kEpCols);
    ep_scatter_kernel<<<grid, 128, 0, st>>>(p, N, me, E, el, T, H, K, x, topk_idx, chunk_base, goff, slot_pos,
                                            done_ctas, epoch);
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

cudaError_t launch_ep_combine(const EpPeers& p, int N, int me, int el, const int* topk_idx, const int* slot_pos,
                              const float* topk_w, const float* y_shared, const float* resid, float* out, int T,
                              int H, int K, uint32_t epoch, uint64_t budget_ns, int* err, cudaStream_t st) {
    if (K > 8) return cudaErrorInvalidValue;
    dim3 grid((H / 8 + 127) / 128, T);
    ep_combine_kernel<<<grid, 128, 0, st>>>(p, N, me, el, topk_idx, slot_pos, topk_w, y_shared, resid, out, H, K,
                                            epoch, budget_ns, err);
    return cudaGetLastError();
}

}  // namespace hymoe
