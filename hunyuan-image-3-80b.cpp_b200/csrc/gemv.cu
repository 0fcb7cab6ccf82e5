// gemv.cu — grouped weight-streaming kernel for decode-sized groups (work items of at most
// kGemvMaxRows = 64 token rows), bound by HBM bandwidth.  Same work items and weight tile
// format as the tensor-core path.
//
// CTA = 256 threads (8 warps) on one (group, 128-row block, <= 64 token rows) item.  Thread 0
// streams the item's weight tiles along K through a ring of `slots` stages: each stage is one
// 1-D bulk copy of two consecutive raw GGUF tiles plus, per tile, one 2-D TMA load of the
// matching activation slice (64 halves x 8/16/32/64 token rows, 128-byte swizzle), all
// completing on the stage's mbarrier.  Several stages per CTA and several CTAs per SM keep
// enough bytes in flight for HBM; one CTA barrier per stage (two tiles) keeps the
// bookkeeping per byte small.
//
// Math: mma.sync m16n8k16 (fp16 x fp16, fp32 accumulate), weights as A (warp w owns the
// 16-row group w of the tile), token rows as B in n-tiles of 8.  The quants become exact
// fp16 integers (q - 8 or q, via the 0x6400 magic-number trick); the block scale d is applied
// to each block's fp32 partial sums for items of up to 16 rows, or folded into the fp16
// weights (the tensor-core path's rounding) for larger items.  A k-permutation shared by A and B (each thread's MMA k positions
// 2c, 2c+1, 2c+8, 2c+9, c = lane % 4, hold four CONSECUTIVE quants of a GGUF block) lets each
// thread build its A fragments from wide shared-memory loads of raw quants; B columns are
// token rows permuted so that the swizzled activation loads are free of bank conflicts too.
// gate_up items end with the SwiGLU (silu of each gate row times its up row) and write fp16;
// down items write fp32.
#include "common.cuh"
#include "gemv_frags.cuh"
#include "kernels.h"

namespace hymoe {

namespace {

using namespace gemvf;

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kStageTiles = 2;  // k-tiles per pipeline stage (one barrier round each)
constexpr int kGL = kGemvMaxRows + 1;  // row pitch (floats) of the result staging G

__host__ __device__ __forceinline__ int box_index(int nrows) {
    return nrows <= 8 ? 0 : nrows <= 16 ? 1 : nrows <= 32 ? 2 : 3;
}

struct GemvItem {
    int rb, row0, nrows, n_ks, slots, xb_max, glu, out_ld;
    const uint8_t* wt;  // first weight tile of the item's row block
    const CUtensorMap* xmap;
    void* out;
    __half* out_r;    // down projection: routed rows (>= shared_rows), fp16
    int shared_rows;
    int* err;
};

// One work item with NT n-tiles of 8 token rows (NT * 8 = the activation box height).
// Thread 0 alone polls the stage barriers (its acquire of the completed phase, followed by
// the CTA barrier, orders every thread's reads after the copies); the same CTA barrier
// tells thread 0 that the previous stage has been consumed, so it can be refilled.
// Up to 16 token rows the block scales are applied to each block's fp32 partial sums
// (exact weights); from 17 rows on they are folded into the fp16 weights once per tile,
// which costs fewer instructions than per-token scaling there.
template <int WT, int NT>
__device__ __forceinline__ void run_item(const GemvItem& p, uint8_t* base, uint64_t* full) {
    constexpr int TB = tile_bytes(WT);
    const int xs_bytes = kStageTiles * p.xb_max;          // activation part of a stage
    uint8_t* xring = base;                                 // slots x xs_bytes
    uint8_t* wring = base + static_cast<size_t>(p.slots) * xs_bytes;  // slots x kStageTiles x TB
    float* G = reinterpret_cast<float*>(base);  // [128][kGL], reuses the ring afterwards
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int gq = lane >> 2, c = lane & 3;
    const int r0 = 16 * warp + gq;
    const int slots = p.slots, n_ks = p.n_ks;
    const int n_st = (n_ks + kStageTiles - 1) / kStageTiles;

    // Stage j: k-tiles [kStageTiles j, kStageTiles j + cnt): one bulk copy of the (contiguous)
    // weight tiles and one activation box per tile, all on the stage's barrier.
    auto issue = [&](int stage, int j) {
        const int t0 = kStageTiles * j, cnt = min(kStageTiles, n_ks - t0);
        mbar_arrive_expect_tx(&full[stage], static_cast<uint32_t>(cnt) * (TB + NT * 1024u));
        bulk_load(wring + static_cast<size_t>(stage) * kStageTiles * TB, p.wt + static_cast<size_t>(t0) * TB,
                  static_cast<uint32_t>(cnt) * TB, &full[stage]);
        for (int i = 0; i < cnt; ++i)
            tma_load_2d(xring + static_cast<size_t>(stage) * xs_bytes + i * p.xb_max, p.xmap, &full[stage],
                        (t0 + i) * kTileK, p.row0);
    };
    int issued = min(slots, n_st);  // stages issued; meaningful in thread 0 only
    if (tid == 0)
        for (int j = 0; j < issued; ++j) issue(j, j);

    float acc[NT][4];
#pragma unroll
    for (int i = 0; i < NT; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
    const int tok_b = col_token<WT>(gq);  // token row (within an n-tile) of this lane's B column

    int s = 0, fail_st = -1;
    uint32_t phase = 0;
    for (int j = 0; j < n_st; ++j) {
        const bool got = tid != 0 || mbar_wait(&full[s], phase, p.err, DEVERR_TIMEOUT_DEQUANT);
        if (!__syncthreads_and(got)) {  // uniform: every thread leaves the loop here
            fail_st = j;
            break;
        }
        // Every thread has finished stage j - 1: its slot takes stage j - 1 + slots.
        if (tid == 0 && j > 0 && j - 1 + slots < n_st) {
            issue(s == 0 ? slots - 1 : s - 1, j - 1 + slots);
            issued = j + slots;
        }
        const int cnt = min(kStageTiles, n_ks - kStageTiles * j);
        const uint8_t* wst = wring + static_cast<size_t>(s) * kStageTiles * TB;
        const uint8_t* xst = xring + static_cast<size_t>(s) * xs_bytes;
#pragma unroll
        for (int i = 0; i < kStageTiles; ++i) {
            if (i < cnt) {
                constexpr bool kPre = NT >= 4;
                uint32_t a[2][2][4];
                float d[2][2];
                tile_frags<WT, kPre>(wst + i * TB, r0, c, a, d);
                const uint8_t* xt = xst + i * p.xb_max;
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    const int n = 8 * nt + tok_b;
                    uint32_t bx[2][2][2];
                    x_frags<WT>(xt + 128 * n, n & 7, c, bx);
#pragma unroll
                    for (int b = 0; b < 2; ++b) {
                        if constexpr (kPre) {
                            mma16816(acc[nt], a[b][0], bx[b][0][0], bx[b][0][1]);
                            mma16816(acc[nt], a[b][1], bx[b][1][0], bx[b][1][1]);
                        } else {
                            float blk[4] = {0.f, 0.f, 0.f, 0.f};
                            mma16816(blk, a[b][0], bx[b][0][0], bx[b][0][1]);
                            mma16816(blk, a[b][1], bx[b][1][0], bx[b][1][1]);
                            acc[nt][0] = fmaf(d[b][0], blk[0], acc[nt][0]);
                            acc[nt][1] = fmaf(d[b][0], blk[1], acc[nt][1]);
                            acc[nt][2] = fmaf(d[b][1], blk[2], acc[nt][2]);
                            acc[nt][3] = fmaf(d[b][1], blk[3], acc[nt][3]);
                        }
                    }
                }
            }
        }
        if (++s == slots) {
            s = 0;
            phase ^= 1u;
        }
    }
    if (fail_st >= 0) {
        // Copies still in flight, stages [fail_st, issued), land before the exit.
        if (tid == 0)
            for (int t = fail_st; t < issued; ++t) mbar_drain(&full[t % slots], (t / slots) & 1);
        __syncthreads();
        return;
    }
    __syncthreads();  // every thread is done with the ring: it becomes G
    const int t0 = col_token<WT>(2 * c), t1 = col_token<WT>(2 * c + 1);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        G[r0 * kGL + 8 * nt + t0] = acc[nt][0];
        G[r0 * kGL + 8 * nt + t1] = acc[nt][1];
        G[(r0 + 8) * kGL + 8 * nt + t0] = acc[nt][2];
        G[(r0 + 8) * kGL + 8 * nt + t1] = acc[nt][3];
    }
    __syncthreads();
    const int nrows = p.nrows;
    if (p.glu) {
        __half* o = static_cast<__half*>(p.out);
        for (int i = tid; i < kGluHalf * nrows; i += kGemvThreads) {
            const int j = i % kGluHalf, n = i / kGluHalf;
            o[static_cast<size_t>(p.row0 + n) * p.out_ld + p.rb * kGluHalf + j] =
                __float2half_rn(silu_mul(G[glu_gate_row(j) * kGL + n], G[glu_up_row(j) * kGL + n]));
        }
    } else if (p.row0 < p.shared_rows) {
        float* o = static_cast<float*>(p.out);
        for (int i = tid; i < kTileRows * nrows; i += kGemvThreads) {
            const int r = i % kTileRows, n = i / kTileRows;
            o[static_cast<size_t>(p.row0 + n) * p.out_ld + p.rb * kTileRows + r] = G[r * kGL + n];
        }
    } else {
        for (int i = tid; i < kTileRows * nrows; i += kGemvThreads) {
            const int r = i % kTileRows, n = i / kTileRows;
            p.out_r[static_cast<size_t>(p.row0 + n) * p.out_ld + p.rb * kTileRows + r] = __float2half_rn(G[r * kGL + n]);
        }
    }
}

template <int WT>
__global__ __launch_bounds__(kGemvThreads, 3) void gemv_kernel(const __grid_constant__ GemvMaps maps,
                                                            const int4* __restrict__ items,
                                                            const int* __restrict__ n_items,
                                                            const uint8_t* const* __restrict__ wtiles,
                                                            int n_ks, int glu, int slots, int xb_max,
                                                            void* __restrict__ out, int out_ld,
                                                            __half* __restrict__ out_r, int shared_rows,
                                                            int* err) {
    griddep_wait();
    griddep_launch_dependents();
    constexpr int TB = tile_bytes(WT);
    extern __shared__ uint8_t gsm_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gsm_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(base + static_cast<size_t>(slots) * kStageTiles * (xb_max + TB));
    if (static_cast<int>(blockIdx.x) >= *n_items) return;
    const int4 it = items[blockIdx.x];
    // The host sizes the activation box (xb_max / 128 rows) from the largest group.
    if (it.w > (xb_max >> 7)) {
        if (threadIdx.x == 0) atomicOr(err, DEVERR_BAD_ITEM);
        return;
    }
    const int bi = box_index(it.w);
    GemvItem p;
    p.rb = it.y;
    p.row0 = it.z;
    p.nrows = it.w;
    p.n_ks = n_ks;
    p.slots = slots;
    p.xb_max = xb_max;
    p.glu = glu;
    p.out_ld = out_ld;
    p.wt = wtiles[it.x] + static_cast<size_t>(it.y) * n_ks * TB;
    p.xmap = &maps.x[bi];
    p.out = out;
    p.out_r = out_r;
    p.shared_rows = shared_rows;
    p.err = err;
    if (threadIdx.x == 0) {
        for (int s = 0; s < slots; ++s) mbar_init(&full[s], 1);
        fence_mbar_init();
    }
    __syncthreads();
    switch (bi) {
        case 0: run_item<WT, 1>(p, base, full); break;
        case 1: run_item<WT, 2>(p, base, full); break;
        case 2: run_item<WT, 4>(p, base, full); break;
        default: run_item<WT, 8>(p, base, full); break;
    }
}

// ---- persistent streaming variant for items of at most 8 token rows (Q4_0 / Q8_0).
//
// One CTA per SM; the CTA takes items blockIdx.x, blockIdx.x + gridDim.x, ...  Warp w owns
// k-tiles w, w + 8, ... of every item and streams them, one bulk copy of the weight tile and
// one 8-row activation box per tile, through a private ring of R slots: no barrier is shared
// between warps inside an item, and the ring runs on into the next item.  Each warp
// accumulates all 128 rows of the tile (8 row groups, exact block scales); at the item's end
// the 8 warp partials meet in shared memory and are summed in warp order (deterministic), and
// the item's output is written.
constexpr int kRedLd = 9;  // token pitch (floats) of the partial buffer: conflict-free sums
constexpr int kStreamItems = 64;

template <int WT, int R>
__global__ __launch_bounds__(kGemvThreads, 1) void gemv_stream_kernel(
    const __grid_constant__ GemvMaps maps, const int4* __restrict__ items, const int* __restrict__ n_items,
    const uint8_t* const* __restrict__ wtiles, int n_ks, int glu, void* __restrict__ out, int out_ld,
    __half* __restrict__ out_r, int shared_rows, int* err) {
    // Programmatic dependent launch: everything up to griddep_wait reads only what was complete
    // before this grid could be scheduled (the work list, written by the plan two or more
    // launches back, and the weights); the activation rows come from the predecessor.
    constexpr int TB = tile_bytes(WT);
    extern __shared__ uint8_t gsm_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gsm_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* xbox = base;                                           // [8 warps][R][1024] (1024-aligned)
    uint8_t* wbuf = base + kGemvWarps * R * 1024;                  // [8 warps][R][TB]
    float* red = reinterpret_cast<float*>(wbuf + kGemvWarps * R * TB);  // [8][128][kRedLd]
    uint64_t* bars = reinterpret_cast<uint64_t*>(red + kGemvWarps * kTileRows * kRedLd);  // [8][R]
    __shared__ int abort_flag;
    // This CTA's items and their weight row blocks, staged once (the issue path must not wait
    // on global loads); more than kStreamItems items fall back to global reads.
    __shared__ int4 s_item[kStreamItems];
    __shared__ const uint8_t* s_wt[kStreamItems];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int gq = lane >> 2, c = lane & 3;
    const int n_it = *n_items, G = gridDim.x;
    const int per_item = warp < n_ks ? (n_ks - warp + kGemvWarps - 1) / kGemvWarps : 0;
    const int my_items = static_cast<int>(blockIdx.x) < n_it ? (n_it - blockIdx.x + G - 1) / G : 0;
    const int total = my_items * per_item;  // this warp's tiles
    uint64_t* wb = bars + warp * R;
    uint8_t* wx = xbox + warp * R * 1024;
    uint8_t* ww = wbuf + static_cast<size_t>(warp) * R * TB;
    if (lane == 0)
        for (int r = 0; r < R; ++r) mbar_init(&wb[r], 1);
    if (tid == 0) abort_flag = 0;
    for (int i = tid; i < min(my_items, kStreamItems); i += kGemvThreads) {
        const int4 it = items[blockIdx.x + i * G];
        s_item[i] = it;
        s_wt[i] = wtiles[it.x] + static_cast<size_t>(it.y) * n_ks * TB;
    }
    fence_mbar_init();
    __syncthreads();
    auto item_at = [&](int i) {
        return i < kStreamItems ? s_item[i] : items[blockIdx.x + i * G];
    };

    auto issue_w = [&](int q) {  // lane 0: weights of tile q of this warp's stream
        const int i = q / per_item, m = q - i * per_item;
        const int4 it = item_at(i);
        const uint8_t* wt = i < kStreamItems ? s_wt[i] : wtiles[it.x] + static_cast<size_t>(it.y) * n_ks * TB;
        const int k = warp + kGemvWarps * m, slot = q % R;
        mbar_arrive_expect_tx(&wb[slot], TB + 1024u);
        bulk_load(ww + slot * TB, wt + static_cast<size_t>(k) * TB, TB, &wb[slot]);
    };
    auto issue_x = [&](int q) {  // lane 0: the activation box of tile q (same barrier)
        const int i = q / per_item, m = q - i * per_item;
        const int k = warp + kGemvWarps * m, slot = q % R;
        tma_load_2d(wx + slot * 1024, &maps.x[0], &wb[slot], k * kTileK, item_at(i).z);
    };
    auto issue = [&](int q) {
        issue_w(q);
        issue_x(q);
    };
    int issued = 0, done = 0;  // lane 0's stream positions
    const int first = min(R, total);
    if (lane == 0)
        for (int q = 0; q < first; ++q) issue_w(q);
    griddep_wait();
    griddep_launch_dependents();
    if (lane == 0)
        for (; issued < first; ++issued) issue_x(issued);

    const int tok_b = col_token<WT>(gq);
    const int t0 = col_token<WT>(2 * c), t1 = col_token<WT>(2 * c + 1);
    for (int i = 0; i < my_items; ++i) {
        const int4 it = item_at(i);
        float acc[8][4];
#pragma unroll
        for (int g = 0; g < 8; ++g)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[g][j] = 0.f;
        bool failed = false;
        for (int m = 0; m < per_item; ++m) {
            const int q = i * per_item + m, slot = q % R;
            int got = 1;
            if (lane == 0) got = mbar_wait(&wb[slot], (q / R) & 1, err, DEVERR_TIMEOUT_DEQUANT) ? 1 : 0;
            __syncwarp();
            if (!__shfl_sync(0xffffffffu, got, 0)) {
                failed = true;
                break;
            }
            // The tile's words into registers, then the slot goes back to the copy engine (the
            // next copy overlaps this tile's conversion and MMAs).
            const uint8_t* tile = ww + slot * TB;
            uint32_t bx[2][2][2];
            x_frags<WT>(wx + slot * 1024 + 128 * tok_b, tok_b & 7, c, bx);
            RawGroup<WT> raw[8];
#pragma unroll
            for (int g = 0; g < 8; ++g) tile_raw<WT>(tile, 16 * g + gq, c, raw[g]);
            __syncwarp();  // every lane has read the slot
            if (lane == 0) {
                done = q + 1;
                if (issued < total) issue(issued++);
            }
#pragma unroll
            for (int g = 0; g < 8; ++g) {
                uint32_t a[2][2][4];
                float d[2][2];
                raw_frags<WT>(raw[g], a, d);
#pragma unroll
                for (int b = 0; b < 2; ++b) {
                    float blk[4] = {0.f, 0.f, 0.f, 0.f};
                    mma16816(blk, a[b][0], bx[b][0][0], bx[b][0][1]);
                    mma16816(blk, a[b][1], bx[b][1][0], bx[b][1][1]);
                    acc[g][0] = fmaf(d[b][0], blk[0], acc[g][0]);
                    acc[g][1] = fmaf(d[b][0], blk[1], acc[g][1]);
                    acc[g][2] = fmaf(d[b][1], blk[2], acc[g][2]);
                    acc[g][3] = fmaf(d[b][1], blk[3], acc[g][3]);
                }
            }
        }
        if (failed && lane == 0) abort_flag = 1;
        // this warp's partial -> red[warp]
        float* rw = red + warp * kTileRows * kRedLd;
#pragma unroll
        for (int g = 0; g < 8; ++g) {
            const int r0 = 16 * g + gq;
            rw[r0 * kRedLd + t0] = acc[g][0];
            rw[r0 * kRedLd + t1] = acc[g][1];
            rw[(r0 + 8) * kRedLd + t0] = acc[g][2];
            rw[(r0 + 8) * kRedLd + t1] = acc[g][3];
        }
        __syncthreads();
        if (abort_flag) break;
        const int nrows = min(it.w, 8), row0 = it.z, rb = it.y;
        auto sum = [&](int r, int n) {
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < kGemvWarps; ++w) v += red[(w * kTileRows + r) * kRedLd + n];
            return v;
        };
        if (glu) {
            __half* o = static_cast<__half*>(out);
            for (int e = tid; e < kGluHalf * nrows; e += kGemvThreads) {
                const int j = e % kGluHalf, n = e / kGluHalf;
                o[static_cast<size_t>(row0 + n) * out_ld + rb * kGluHalf + j] =
                    __float2half_rn(silu_mul(sum(glu_gate_row(j), n), sum(glu_up_row(j), n)));
            }
        } else if (row0 < shared_rows) {
            float* o = static_cast<float*>(out);
            for (int e = tid; e < kTileRows * nrows; e += kGemvThreads) {
                const int r = e % kTileRows, n = e / kTileRows;
                o[static_cast<size_t>(row0 + n) * out_ld + rb * kTileRows + r] = sum(r, n);
            }
        } else {
            for (int e = tid; e < kTileRows * nrows; e += kGemvThreads) {
                const int r = e % kTileRows, n = e / kTileRows;
                out_r[static_cast<size_t>(row0 + n) * out_ld + rb * kTileRows + r] = __float2half_rn(sum(r, n));
            }
        }
        __syncthreads();  // red is free again
    }
    if (abort_flag) {
        // Copies this warp issued but did not consume land before the exit (bounded waits).
        if (lane == 0)
            for (int q = done; q < issued; ++q) mbar_drain(&wb[q % R], (q / R) & 1);
        __syncwarp();
    }
}

template <int WT, int R>
size_t stream_smem() {
    return 1024 + static_cast<size_t>(kGemvWarps) * R * (1024 + tile_bytes(WT)) +
           sizeof(float) * kGemvWarps * kTileRows * kRedLd + 8u * kGemvWarps * R;
}

template <int WT, int R>
cudaError_t launch_stream(const GemvMaps& maps, const int4* items, const int* n_items, int n_sms,
                          const uint8_t* const* wtiles, int n_ks, int glu, void* out, int out_ld, __half* out_r,
                          int shared_rows, int* err, cudaStream_t st, bool pdl) {
    const size_t smem = stream_smem<WT, R>();
    cudaError_t e = cudaFuncSetAttribute(gemv_stream_kernel<WT, R>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    return launch_kernel(pdl, gemv_stream_kernel<WT, R>, dim3(n_sms), dim3(kGemvThreads), smem, st, maps, items,
                         n_items, wtiles, n_ks, glu, out, out_ld, out_r, shared_rows, err);
}

// Stages per CTA: as many as fit in ~72 KB (three CTAs per SM), at least 2 and at most 4;
// the ring must also hold the result staging G.
template <int WT>
void gemv_smem(int max_box, int* slots, int* xb_max, size_t* smem) {
    *xb_max = 1024 << max_box;
    const size_t stage = static_cast<size_t>(kStageTiles) * (tile_bytes(WT) + *xb_max);
    int s = static_cast<int>((72u * 1024u) / stage);
    s = s < 2 ? 2 : s > 4 ? 4 : s;
    const size_t g_bytes = sizeof(float) * kTileRows * kGL;
    while (static_cast<size_t>(s) * stage < g_bytes) ++s;
    *slots = s;
    *smem = 1024 + static_cast<size_t>(s) * stage + 8u * s;
}

template <int WT>
cudaError_t launch_t(const GemvMaps& maps, const int4* items, const int* n_items, int max_items,
                     const uint8_t* const* wtiles, int n_ks, int glu, int max_rows, void* out,
                     int out_ld, __half* out_r, int shared_rows, int* err, cudaStream_t st, bool pdl) {
    int slots = 0, xb_max = 0;
    size_t smem = 0;
    gemv_smem<WT>(box_index(max_rows), &slots, &xb_max, &smem);
    cudaError_t e = cudaFuncSetAttribute(gemv_kernel<WT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    return launch_kernel(pdl, gemv_kernel<WT>, dim3(max_items), dim3(kGemvThreads), smem, st, maps, items, n_items,
                         wtiles, n_ks, glu, slots, xb_max, out, out_ld, out_r, shared_rows, err);
}

}  // namespace

cudaError_t launch_gemv(const GemvMaps& maps, const int4* items, const int* n_items, int max_items,
                        const uint8_t* const* wtiles, int wtype, int n_ks, int glu, int max_rows,
                        void* out, int out_ld, __half* out_r, int shared_rows, int* err, int n_sms,
                        cudaStream_t st, bool pdl) {
    if (max_items <= 0) return cudaSuccess;
    if (max_rows < 1 || max_rows > kGemvMaxRows) return cudaErrorInvalidValue;
    if (max_rows <= 8 && wtype == W_Q8_0)
        return launch_stream<W_Q8_0, 2>(maps, items, n_items, n_sms, wtiles, n_ks, glu, out, out_ld, out_r, shared_rows, err, st,
                                        pdl);
    if (max_rows <= 8 && wtype == W_Q4_0)
        return launch_stream<W_Q4_0, 3>(maps, items, n_items, n_sms, wtiles, n_ks, glu, out, out_ld, out_r, shared_rows, err, st,
                                        pdl);
    switch (wtype) {
        case W_Q4_0: return launch_t<W_Q4_0>(maps, items, n_items, max_items, wtiles, n_ks, glu, max_rows, out, out_ld, out_r, shared_rows, err, st, pdl);
        case W_Q8_0: return launch_t<W_Q8_0>(maps, items, n_items, max_items, wtiles, n_ks, glu, max_rows, out, out_ld, out_r, shared_rows, err, st, pdl);
        default: return launch_t<W_F16>(maps, items, n_items, max_items, wtiles, n_ks, glu, max_rows, out, out_ld, out_r, shared_rows, err, st, pdl);
    }
}

}  // namespace hymoe
