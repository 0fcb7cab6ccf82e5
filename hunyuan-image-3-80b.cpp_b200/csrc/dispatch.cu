// dispatch.cu — token permutation: per-expert prefix scan, GEMM work lists, and the
// scatter/gather of token rows into expert-sorted order.
//
// The reference has no explicit dispatch: its loop calls the FFN once per (token, rank)
// pair (src/attention.cpp:285-299).  Here the T*K (token, rank) pairs are counting-sorted
// by expert, stably by token, so every expert's tokens form one contiguous row range of
// the fp16 activation matrix `xp` that the grouped GEMMs read.  Row ranges:
//   group e < E : [goff[e], goff[e] + count_e)  routed expert e
//   group E     : [T*K, T*K + T)                shared expert (every token, in order)
#include "common.cuh"
#include "kernels.h"

namespace hymoe {

namespace {

// One CTA of 1024 threads.  (expert, part) = (tid / 16, tid % 16) owns a contiguous run of
// at most kMaxChunksPerPart router chunks; its counts stay in registers between the column
// sum and the base write-out.
constexpr int kMaxChunksPerPart = 32;  // 16 parts x 32 chunks x 16 tokens = 8192 tokens

__global__ __launch_bounds__(1024) void plan_kernel(PlanArgs a) {
    __shared__ int part_sum[64][17];
    __shared__ int gcnt[66], goff_s[67], ioff_gu[67], ioff_dn[67], ntt_s[66];
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
        gcnt[tid] = tid < a.E ? tot : 0;
    }
    __syncthreads();
    if (tid == 0) {
        gcnt[a.E] = a.T;  // shared expert: every token
        int off = 0, ngu = 0, ndn = 0;
        for (int g = 0; g <= a.E; ++g) {
            goff_s[g] = off;
            off += gcnt[g];
            const int ntt = a.gemv ? (gcnt[g] > 0) : (gcnt[g] + a.tile_n - 1) / a.tile_n;
            ntt_s[g] = ntt;
            ioff_gu[g] = ngu;
            ioff_dn[g] = ndn;
            ngu += ntt * a.n_rb_gu;
            ndn += ntt * a.n_rb_dn;
        }
        goff_s[a.E + 1] = off;
        ioff_gu[a.E + 1] = ngu;
        ioff_dn[a.E + 1] = ndn;
        a.n_items[0] = ngu;
        a.n_items[1] = ndn;
    }
    __syncthreads();
    for (int g = tid; g < a.E + 2; g += blockDim.x) a.goff[g] = goff_s[g];
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
    // Work items, group-major then row block then token tile: consecutive items share a
    // weight tile, so concurrently running CTAs hit it in L2.  Flat loop over all items;
    // the group of an item is found by binary search over the item offsets.
    for (int which = 0; which < 2; ++which) {
        const int* ioff = which ? ioff_dn : ioff_gu;
        const int nrb = which ? a.n_rb_dn : a.n_rb_gu;
        int4* items = which ? a.items_dn : a.items_gu;
        const int total = ioff[a.E + 1];
        for (int i = tid; i < total; i += blockDim.x) {
            int lo = 0, hi = a.E;  // find g with ioff[g] <= i < ioff[g + 1]
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (ioff[mid] <= i) lo = mid;
                else hi = mid - 1;
            }
            const int g = lo, local = i - ioff[g];
            const int ntt = ntt_s[g];
            const int rb = local / ntt, tt = local - rb * ntt;
            const int tn = a.gemv ? gcnt[g] : a.tile_n;
            items[i] = make_int4(g, rb, goff_s[g] + tt * tn, min(tn, gcnt[g] - tt * tn));
            (void)nrb;
        }
    }
}

// One CTA per router chunk of 16 tokens.  Position of pair (t, k) with expert e:
//   chunk_base[c][e] + #{earlier tokens of the chunk that also chose e}
// which is the stable (token-ordered) counting sort.  Then each token row is converted
// to fp16 once and written to its K routed rows and its shared-expert row.
__global__ __launch_bounds__(256) void scatter_gather_kernel(
    const float* __restrict__ x, int T, int H, int E, int K, const int* __restrict__ topk_idx,
    const int* __restrict__ chunk_base, const int* __restrict__ goff, int* __restrict__ slot_pos,
    __half* __restrict__ xp) {
    __shared__ int sidx[kRouterTok][8];
    __shared__ int spos[kRouterTok][9];
    const int c = blockIdx.x, t0 = c * kRouterTok, tid = threadIdx.x;
    const int nt = min(kRouterTok, T - t0);
    if (tid < kRouterTok * 8) {
        const int tt = tid >> 3, k = tid & 7;
        sidx[tt][k] = (tt < nt && k < K) ? topk_idx[(t0 + tt) * K + k] : -1;
    }
    __syncthreads();
    if (tid < kRouterTok * 8) {
        const int tt = tid >> 3, k = tid & 7;
        if (tt < nt && k < K) {
            const int e = sidx[tt][k];
            int rank = 0;
            for (int p = 0; p < tt; ++p)
                for (int kk = 0; kk < K; ++kk) rank += sidx[p][kk] == e;
            const int pos = chunk_base[c * E + e] + rank;
            spos[tt][k] = pos;
            slot_pos[(t0 + tt) * K + k] = pos;
        }
    }
    if (tid < kRouterTok) spos[tid][8] = goff[E] + t0 + tid;
    __syncthreads();
    for (int tt = 0; tt < nt; ++tt) {
        const float* xr = x + static_cast<size_t>(t0 + tt) * H;
        for (int j = tid * 8; j < H; j += 256 * 8) {
            const float4 a = *reinterpret_cast<const float4*>(xr + j);
            const float4 b = *reinterpret_cast<const float4*>(xr + j + 4);
            const __half2 h0 = __floats2half2_rn(a.x, a.y), h1 = __floats2half2_rn(a.z, a.w);
            const __half2 h2 = __floats2half2_rn(b.x, b.y), h3 = __floats2half2_rn(b.z, b.w);
            uint4 v;
            v.x = *reinterpret_cast<const uint32_t*>(&h0);
            v.y = *reinterpret_cast<const uint32_t*>(&h1);
            v.z = *reinterpret_cast<const uint32_t*>(&h2);
            v.w = *reinterpret_cast<const uint32_t*>(&h3);
            for (int k = 0; k < K; ++k)
                *reinterpret_cast<uint4*>(xp + static_cast<size_t>(spos[tt][k]) * H + j) = v;
            *reinterpret_cast<uint4*>(xp + static_cast<size_t>(spos[tt][8]) * H + j) = v;
        }
    }
}

}  // namespace

cudaError_t launch_plan(const PlanArgs& a, cudaStream_t st) {
    plan_kernel<<<1, 1024, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_scatter_gather(const float* x, int T, int H, int E, int K, const int* topk_idx,
                                  const int* chunk_base, const int* goff, int* slot_pos,
                                  __half* xp, cudaStream_t st) {
    const int blocks = (T + kRouterTok - 1) / kRouterTok;
    scatter_gather_kernel<<<blocks, 256, 0, st>>>(x, T, H, E, K, topk_idx, chunk_base, goff,
                                                  slot_pos, xp);
    return cudaGetLastError();
}

}  // namespace hymoe
