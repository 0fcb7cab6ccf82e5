// dispatch.cu — token permutation: per-expert prefix scan, GEMM segments and work lists,
// and the scatter/gather of token rows into expert-sorted order.
//
// The reference has no explicit dispatch: its loop calls the FFN once per (token, rank)
// pair (src/attention.cpp:285-299).  Here the T*K (token, rank) pairs are counting-sorted
// by global expert id, stably by token.  Expert e's pairs become rows
// [goff[e], goff[e] + count_e) of the routed-row matrix; since expert-parallel ranks own
// consecutive experts, that order is also destination-rank-major.
//
// GEMM input layout (one fp16 matrix per call):
//   rows [0, T)        the shared expert's rows (every local token, in order)
//   rows [T, T + R)    routed rows: on one GPU the sorted pairs themselves; with expert
//                      parallelism the rows received from every rank (source-major,
//                      then local expert)
// A segment {weight group, first row, rows} names a run of rows that one expert's weights
// multiply; work items tile segments into (row-block, up to tile_n rows) pieces.
#include "common.cuh"
#include "kernels.h"
#include "topk.cuh"

namespace hymoe {

namespace {

// Work items from segments (executed by a whole CTA; `seg` in shared memory, pre: shared
// scratch of kMaxSegs + 1 ints): segment-major, then row block, then token tile, so an
// expert's tiles run close together while its weights are in L2, and concurrently running
// CTAs share weight tiles (with expert parallelism the local source's rows come first).  The
// GEMM deals the list to its SM pairs in snake order (gemm_item).  A list ordered by tile size
// (every expert's partial tile last) balanced the pairs' rows better but made every expert's
// weights come from DRAM twice (gate_up at 4096 tokens: 2.25 GB per launch instead of 1.46 GB)
// for a 1 % shorter kernel, so it is not used.
__device__ void build_items(const int4* seg, int ns, const ItemsArgs& a, int* pre) {
    const int tid = threadIdx.x;
    const int tn = a.gemv ? kGemvMaxRows : a.tile_n;
    for (int i = tid; i < ns; i += blockDim.x) {
        const int cnt = seg[i].z;
        pre[i] = cnt <= 0 ? 0 : (cnt + tn - 1) / tn;  // token tiles of segment i
    }
    __syncthreads();
    if (tid < 32) {
        const int tot = warp_exclusive_scan(pre, ns);  // pre[i] = tiles before segment i
        if (tid == 0) {
            pre[ns] = tot;
            a.n_items[0] = tot * a.n_rb_gu;
            a.n_items[1] = tot * a.n_rb_dn;
        }
    }
    __syncthreads();
    for (int which = 0; which < 2; ++which) {
        const int n_rb = which ? a.n_rb_dn : a.n_rb_gu;
        int4* items = which ? a.items_dn : a.items_gu;
        const int total = pre[ns] * n_rb;
        for (int i = tid; i < total; i += blockDim.x) {
            const int key = i / n_rb;
            int lo = 0, hi = ns - 1;  // last segment with pre <= key
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (pre[mid] <= key) lo = mid;
                else hi = mid - 1;
            }
            const int4 sg = seg[lo];
            const int local = i - pre[lo] * n_rb;
            const int ntt = pre[lo + 1] - pre[lo];
            const int rb = local / ntt, tt = local - rb * ntt;
            items[i] = make_int4(sg.x, rb, sg.y + tt * tn, min(tn, sg.z - tt * tn));
            int2* aux = which ? a.aux_dn : a.aux_gu;
            if (aux != nullptr) aux[i] = make_int2(sg.w, a.seg_ret[lo] + tt * tn);
        }
    }
}

__global__ __launch_bounds__(1024) void items_kernel(ItemsArgs a) {
    __shared__ int4 seg[kMaxSegs];
    __shared__ int pre[kMaxSegs + 1];
    const int ns = min(*a.n_segs, kMaxSegs);
    for (int i = threadIdx.x; i < ns; i += blockDim.x) seg[i] = a.segs[i];
    __syncthreads();
    build_items(seg, ns, a, pre);
}

// Single-GPU segments (shared expert first, then one segment per routed expert) and their
// work items.  goff_s / gcnt_s: the routed-row offsets and counts in shared memory.
__device__ void single_gpu_items(const PlanArgs& a, const int* goff_s, const int* gcnt_s) {
    __shared__ int4 seg[kMaxSegs];
    __shared__ int pre[kMaxSegs + 1];
    const int tid = threadIdx.x;
    const int s0 = a.shared_apart ? 0 : 1;  // the shared segment, unless it runs apart
    const int ns = a.E + s0;
    if (tid == 0) {
        if (s0) seg[0] = make_int4(a.E, 0, a.T, 0);
        *a.n_segs = ns;
    }
    for (int g = tid; g < a.E; g += blockDim.x) seg[s0 + g] = make_int4(g, a.T + goff_s[g], gcnt_s[g], 0);
    __syncthreads();
    for (int i = tid; i < ns; i += blockDim.x) a.segs[i] = seg[i];
    build_items(seg, ns, a.items, pre);
}

// One CTA of 1024 threads.  (expert, part) = (tid / 16, tid % 16) owns a contiguous run of
// at most kMaxChunksPerPart router chunks; its counts stay in registers between the column
// sum and the base write-out.
constexpr int kMaxChunksPerPart = 32;  // 16 parts x 32 chunks x 16 tokens = 8192 tokens

__global__ __launch_bounds__(1024) void plan_kernel(PlanArgs a) {
    griddep_wait();
    griddep_launch_dependents();
    __shared__ int part_sum[64][17];
    __shared__ int gcnt_s[64], goff_s[kMaxSegs + 1];
    const int tid = threadIdx.x;
    const int e = tid >> 4, part = tid & 15;
    const int cpp = (a.n_chunks + 15) / 16;
    const int c_lo = min(a.n_chunks, part * cpp), c_hi = min(a.n_chunks, c_lo + cpp);
    int cnt[kMaxChunksPerPart];
    int s = 0;
#pragma unroll
    for (int i = 0; i < kMaxChunksPerPart; ++i) {
        const int c = c_lo + i;
        cnt[i] = (e < a.E && c < c_hi) ? a.chunk_counts[c * a.E + e] : 0;
        s += cnt[i];
    }
    part_sum[e][part] = s;
    __syncthreads();
    if (tid < 64) {
        int tot = 0;
        for (int p = 0; p < 16; ++p) tot += part_sum[tid][p];
        gcnt_s[tid] = tid < a.E ? tot : 0;
        goff_s[tid] = gcnt_s[tid];
    }
    __syncthreads();
    if (tid < 32) {
        const int tot = warp_exclusive_scan(goff_s, a.E);
        if (tid == 0) goff_s[a.E] = tot;  // == T * K
    }
    __syncthreads();
    for (int g = tid; g <= a.E; g += blockDim.x) a.goff[g] = goff_s[g];
    for (int g = tid; g < a.E; g += blockDim.x) a.gcnt[g] = gcnt_s[g];
    if (e < a.E) {
        int base = goff_s[e];
        for (int p = 0; p < part; ++p) base += part_sum[e][p];
#pragma unroll
        for (int i = 0; i < kMaxChunksPerPart; ++i) {
            const int c = c_lo + i;
            if (c < c_hi) a.chunk_base[c * a.E + e] = base;
            base += cnt[i];
        }
    }
    // Single-GPU segments and their work items, in this same launch.
    if (a.segs != nullptr) single_gpu_items(a, goff_s, gcnt_s);
}

// Decode front end for T <= 16 (one router chunk): top-K of every token (warp t routes token
// t) followed by the plan of that single chunk, in one launch.
__global__ __launch_bounds__(1024) void topk_plan_kernel(const float* __restrict__ logits, int T, int K,
                                                         float* __restrict__ probs_out,
                                                         float* __restrict__ topk_w,
                                                         int* __restrict__ topk_idx, PlanArgs a) {
    griddep_wait();
    griddep_launch_dependents();
    __shared__ float pbuf[kRouterTok][kMaxE];
    __shared__ int gcnt_s[kMaxE], goff_s[kMaxSegs + 1];
    const int tid = threadIdx.x, warp = tid >> 5;
    if (tid < kMaxE) gcnt_s[tid] = 0;
    __syncthreads();
    if (warp < T) topk_token(logits, warp, a.E, K, probs_out, topk_w, topk_idx, pbuf[warp], gcnt_s, a.slot_of, a.mode);
    __syncthreads();
    if (tid < 64) goff_s[tid] = tid < a.E ? gcnt_s[tid] : 0;
    __syncthreads();
    if (tid < 32) {
        const int tot = warp_exclusive_scan(goff_s, a.E);
        if (tid == 0) goff_s[a.E] = tot;
    }
    __syncthreads();
    for (int g = tid; g <= a.E; g += blockDim.x) a.goff[g] = goff_s[g];
    for (int g = tid; g < a.E; g += blockDim.x) {
        a.gcnt[g] = gcnt_s[g];
        a.chunk_base[g] = goff_s[g];  // the only chunk starts at each expert's offset
    }
    if (a.segs != nullptr) single_gpu_items(a, goff_s, gcnt_s);
}

// Grid (router chunk of 16 tokens, column slice of kScatterCols).  Position of pair (t, k)
// with expert e:
//   chunk_base[c][e] + #{earlier tokens of the chunk that also chose e}
// which is the stable (token-ordered) counting sort (every slice recomputes it; slice 0
// publishes slot_pos).  Then each token row slice is converted to fp16 once and written to
// its K routed rows and its shared-expert row.
constexpr int kScatterCols = 256;

__global__ __launch_bounds__(128) void scatter_gather_kernel(
    const float* __restrict__ x, int T, int H, int E, int K, const int* __restrict__ topk_idx,
    const int* __restrict__ chunk_base, int* __restrict__ slot_pos, __half* __restrict__ xp_routed,
    __half* __restrict__ xp_shared, RowNorm nrm) {
    griddep_wait();
    griddep_launch_dependents();
    __shared__ int sidx[kRouterTok][8];
    __shared__ int spos[kRouterTok][8];
    const int c = blockIdx.x, t0 = c * kRouterTok, tid = threadIdx.x;
    const int nt = min(kRouterTok, T - t0);
    {
        const int tt = tid >> 3, k = tid & 7;  // 128 threads = 16 tokens x 8 ranks
        const int v = (tt < nt && k < K) ? topk_idx[(t0 + tt) * K + k] : -1;
        sidx[tt][k] = v >= 0 && (v & kDroppedPair) ? -1 : v;  // a dropped pair takes no row
    }
    __syncthreads();
    {
        const int tt = tid >> 3, k = tid & 7;
        if (tt < nt && k < K) {
            const int e = sidx[tt][k];
            int pos = -1;
            if (e >= 0) {
                int rank = 0;
                for (int p = 0; p < tt; ++p)
                    for (int kk = 0; kk < K; ++kk) rank += sidx[p][kk] == e;
                pos = chunk_base[c * E + e] + rank;
            }
            spos[tt][k] = pos;
            if (blockIdx.y == 0) slot_pos[(t0 + tt) * K + k] = pos;
        }
    }
    __syncthreads();
    // 128 threads x 8 columns = 4 token rows of the slice per pass
    const int j = blockIdx.y * kScatterCols + (tid & 31) * 8;
    if (j >= H) return;
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
        for (int k = 0; k < K; ++k)
            if (spos[tt][k] >= 0) *reinterpret_cast<uint4*>(xp_routed + static_cast<size_t>(spos[tt][k]) * H + j) = v;
        if (xp_shared != nullptr) *reinterpret_cast<uint4*>(xp_shared + static_cast<size_t>(t0 + tt) * H + j) = v;
    }
}

// One CTA: the shared expert's fp16 rows and its work items (decode sizes, T <= 8).
__global__ __launch_bounds__(256) void shared_prep_kernel(const float* __restrict__ x, int T, int H,
                                                          __half* __restrict__ xp, int group, int n_rb_gu,
                                                          int n_rb_dn, int4* items_gu, int4* items_dn,
                                                          int* n_items, RowNorm nrm) {
    const int tid = threadIdx.x;
    for (int i = tid; i < n_rb_gu; i += blockDim.x) items_gu[i] = make_int4(group, i, 0, T);
    for (int i = tid; i < n_rb_dn; i += blockDim.x) items_dn[i] = make_int4(group, i, 0, T);
    if (tid == 0) {
        n_items[0] = n_rb_gu;
        n_items[1] = n_rb_dn;
    }
    for (int i = tid * 4; i < T * H; i += blockDim.x * 4) {
        const float4 a = norm_row4(*reinterpret_cast<const float4*>(x + i), nrm, i / H, i % H);
        const __half2 h0 = __floats2half2_rn(a.x, a.y), h1 = __floats2half2_rn(a.z, a.w);
        uint2 v;
        v.x = *reinterpret_cast<const uint32_t*>(&h0);
        v.y = *reinterpret_cast<const uint32_t*>(&h1);
        *reinterpret_cast<uint2*>(xp + i) = v;
    }
}

// Expert-parallel receive segments from the gathered count matrix C[N][E]: the shared
// expert over the local rows first, then (source s, local expert le) runs in source-major
// order starting at row T.  Single thread: at most E + 1 segments.
__global__ void ep_segments_kernel(const int* __restrict__ C, int ld, int N, int rank, int el,
                                   int T, int4* __restrict__ segs, int* __restrict__ n_segs) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    segs[0] = make_int4(el, 0, T, 0);
    int row = T, n = 1;
    for (int s = 0; s < N; ++s)
        for (int le = 0; le < el; ++le) {
            const int cnt = C[s * ld + rank * el + le];
            segs[n++] = make_int4(le, row, cnt, 0);
            row += cnt;
        }
    *n_segs = n;
}

// Fused expert parallel: the receive segments of ep_segments_kernel (rows stay source-major)
// listed shared first, then this rank's own rows, then sources rank-1, rank-2, ...; each with
// its source rank (w) and, in seg_ret, the source's expert-sorted position of its first row:
// sum of the source's counts of every slot before this rank's local expert le.
__global__ void ep_segments_fused_kernel(const int* __restrict__ C, int ld, int N, int rank, int el,
                                         int T, int4* __restrict__ segs, int* __restrict__ seg_ret,
                                         int* __restrict__ n_segs) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    segs[0] = make_int4(el, 0, T, rank);
    seg_ret[0] = 0;
    int n = 1;
    for (int j = 0; j < N; ++j) {
        const int s = (rank - j + N) % N;
        int row = T;  // first row of source s: after the rows of sources 0..s-1
        for (int s2 = 0; s2 < s; ++s2)
            for (int le = 0; le < el; ++le) row += C[s2 * ld + rank * el + le];
        int ret = 0;  // source s's pairs of slots before rank * el
        for (int e = 0; e < rank * el; ++e) ret += C[s * ld + e];
        for (int le = 0; le < el; ++le) {
            const int cnt = C[s * ld + rank * el + le];
            segs[n] = make_int4(le, row, cnt, s);
            seg_ret[n++] = ret;
            row += cnt;
            ret += cnt;
        }
    }
    *n_segs = n;
}

__global__ void unmap_slots_kernel(int* __restrict__ idx, const int* __restrict__ expert_of_slot, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int slot = idx[i] & ~kDroppedPair;
    idx[i] = expert_of_slot != nullptr ? __ldg(expert_of_slot + slot) : slot;
}

// k-major priorities (one CTA of 1024 threads).  For each choice k, tokens in blocks of 1024:
// a lane's rank among its warp's lanes of the same slot (warp match), plus the counts of the
// same slot in earlier warps of the block, plus the slot's running count over earlier blocks
// and earlier choices.  Over an expert-parallel job (recs != nullptr) the running count of
// choice k starts at the job's pairs of earlier choices plus earlier ranks' pairs of choice k
// (the job's tokens are rank 0's, then rank 1's, ...), and the capacity comes from the job's
// token count.
__global__ __launch_bounds__(1024) void capacity_kernel(int* __restrict__ topk_idx, float* __restrict__ topk_w,
                                                        int* __restrict__ chunk_counts, int T, int K, int E,
                                                        int capacity, const int* __restrict__ recs, int N, int me,
                                                        float cf, int min_capacity) {
    __shared__ int run[kMaxE];
    __shared__ int wcnt[32][kMaxE];
    __shared__ int cap_s;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rl = ep_choice_rec(E);
    if (tid < kMaxE) run[tid] = 0;
    if (tid == 0) {
        int cap = capacity;
        if (recs != nullptr) {
            int t_job = 0;
            for (int r = 0; r < N; ++r) t_job += recs[r * rl + kEpMaxK * E];
            const float f = __fdiv_rn(__fmul_rn(__fmul_rn(cf, static_cast<float>(K)), static_cast<float>(t_job)),
                                      static_cast<float>(E));
            const uint32_t fu = f >= 4294967296.f ? 0xffffffffu : static_cast<uint32_t>(f);
            cap = max(max(static_cast<int>(min(fu, 1u << 30)), K), min_capacity);
        }
        cap_s = cap;
    }
    __syncthreads();
    const int cap = cap_s;
    const unsigned lt = (1u << lane) - 1u;
    for (int k = 0; k < K; ++k) {
        if (recs != nullptr && tid < E) {
            int b = 0;
            for (int r = 0; r < N; ++r) {
                for (int k2 = 0; k2 < k; ++k2) b += recs[r * rl + k2 * E + tid];
                if (r < me) b += recs[r * rl + k * E + tid];
            }
            run[tid] = b;
        }
        __syncthreads();
        for (int t0 = 0; t0 < T; t0 += 1024) {
            const int t = t0 + tid;
            const bool valid = t < T;
            const int slot = valid ? topk_idx[t * K + k] : -1;
            const unsigned peers = __match_any_sync(0xffffffffu, slot);
            for (int e = lane; e < kMaxE; e += 32) wcnt[warp][e] = 0;
            __syncwarp();
            if (valid && (peers & lt) == 0) wcnt[warp][slot] = __popc(peers);
            __syncthreads();
            if (tid < E) {  // exclusive scan over the block's warps, continued from `run`
                int acc = run[tid];
                for (int w = 0; w < 32; ++w) {
                    const int cnt = wcnt[w][tid];
                    wcnt[w][tid] = acc;
                    acc += cnt;
                }
                run[tid] = acc;
            }
            __syncthreads();
            if (valid && wcnt[warp][slot] + __popc(peers & lt) >= cap) {
                topk_idx[t * K + k] = slot | kDroppedPair;
                topk_w[t * K + k] = 0.f;
                atomicSub(chunk_counts + static_cast<size_t>(t / kRouterTok) * E + slot, 1);
            }
            __syncthreads();  // wcnt (and run, next choice) are rewritten
        }
    }
}

}  // namespace

cudaError_t launch_plan(const PlanArgs& a, cudaStream_t st, bool pdl) {
    return launch_kernel(pdl, plan_kernel, dim3(1), dim3(1024), 0, st, a);
}

cudaError_t launch_topk_plan(const float* logits, int T, int K, float* probs, float* topk_w,
                             int* topk_idx, const PlanArgs& a, cudaStream_t st, bool pdl) {
    if (T > kRouterTok || a.n_chunks != 1) return cudaErrorInvalidValue;
    return launch_kernel(pdl, topk_plan_kernel, dim3(1), dim3(1024), 0, st, logits, T, K, probs, topk_w, topk_idx, a);
}

cudaError_t launch_items(const ItemsArgs& a, cudaStream_t st) {
    items_kernel<<<1, 1024, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_capacity(int* topk_idx, float* topk_w, int* chunk_counts, int T, int K, int E, int capacity,
                            cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    if (E > kMaxE) return cudaErrorInvalidValue;
    capacity_kernel<<<1, 1024, 0, st>>>(topk_idx, topk_w, chunk_counts, T, K, E, capacity, nullptr, 1, 0, 0.f, 0);
    return cudaGetLastError();
}

cudaError_t launch_capacity_job(int* topk_idx, float* topk_w, int* chunk_counts, int T, int K, int E,
                                const int* recs, int N, int me, float cf, int min_capacity, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    if (E > kMaxE || K > kEpMaxK || N > kEpMaxRanks) return cudaErrorInvalidValue;
    capacity_kernel<<<1, 1024, 0, st>>>(topk_idx, topk_w, chunk_counts, T, K, E, 0, recs, N, me, cf, min_capacity);
    return cudaGetLastError();
}

cudaError_t launch_unmap_slots(int* idx, const int* expert_of_slot, int n, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    unmap_slots_kernel<<<(n + 255) / 256, 256, 0, st>>>(idx, expert_of_slot, n);
    return cudaGetLastError();
}

cudaError_t launch_scatter_gather(const float* x, int T, int H, int E, int K, const int* topk_idx,
                                  const int* chunk_base, int* slot_pos, __half* xp_routed,
                                  __half* xp_shared, cudaStream_t st, const RowNorm& nrm, bool pdl) {
    dim3 grid((T + kRouterTok - 1) / kRouterTok, (H + kScatterCols - 1) / kScatterCols);
    return launch_kernel(pdl, scatter_gather_kernel, grid, dim3(128), 0, st, x, T, H, E, K, topk_idx, chunk_base,
                         slot_pos, xp_routed, xp_shared, nrm);
}

cudaError_t launch_shared_prep(const float* x, int T, int H, __half* xp, int group, int n_rb_gu,
                               int n_rb_dn, int4* items_gu, int4* items_dn, int* n_items, cudaStream_t st,
                               const RowNorm& nrm) {
    shared_prep_kernel<<<1, 256, 0, st>>>(x, T, H, xp, group, n_rb_gu, n_rb_dn, items_gu, items_dn, n_items, nrm);
    return cudaGetLastError();
}

cudaError_t launch_ep_segments_fused(const int* C, int ld, int N, int rank, int el, int T, int4* segs,
                                     int* seg_ret, int* n_segs, cudaStream_t st) {
    ep_segments_fused_kernel<<<1, 32, 0, st>>>(C, ld, N, rank, el, T, segs, seg_ret, n_segs);
    return cudaGetLastError();
}

cudaError_t launch_ep_segments(const int* C, int ld, int N, int rank, int el, int E, int T, int4* segs,
                               int* n_segs, cudaStream_t st) {
    (void)E;
    ep_segments_kernel<<<1, 32, 0, st>>>(C, ld, N, rank, el, T, segs, n_segs);
    return cudaGetLastError();
}

}  // namespace hymoe
