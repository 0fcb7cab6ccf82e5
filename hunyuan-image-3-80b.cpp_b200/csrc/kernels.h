// kernels.h — host-side launchers of the hymoe CUDA kernels (internal to libhymoe.so).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace hymoe {

// ---- weights.cu
// Re-tiles one GGUF matrix [rows, K] (device bytes, type src_type) into the device tile
// format (dst_type: the same quantised type, or F16 for F32/F16 sources).  glu_I > 0
// selects the gate_up row interleave (rows 0..I-1 gate, I..2I-1 up).
cudaError_t launch_repack(const uint8_t* src, int src_type, uint8_t* dst, int dst_type, int rows,
                          int K, int glu_I, cudaStream_t st);
// Synthetic GGUF tensor of n elements into dst (GGUF bytes of `type`).
cudaError_t launch_synth_gguf(uint8_t* dst, int type, uint64_t n, uint64_t seed, uint64_t stream,
                              float scale, cudaStream_t st);
// Synthetic F32 values.
cudaError_t launch_synth_f32(float* dst, uint64_t n, uint64_t seed, uint64_t stream, float scale,
                             cudaStream_t st);

// Routing variant (FULL mode, topkgating_full, src/hunyuan_moe_full.cpp:119-243, without
// capacity drops).  The default is moe_forward_cpu's routing (src/attention.cpp:224-275).
struct RouteMode {
    int n_group = 0;     // > 0: group-limited greedy over n_group groups of E/n_group experts
    int topk_group = 0;  //      groups kept
    int norm = 1;        // weights = p / sum of the K selected p (else p * scale)
    int clamp = 0;       //      sum clamped below at 1e-8 (FULL mode)
    float scale = 1.f;   // routed_scaling_factor when norm == 0
    int drop = 0;        // capacity-limited routing (one GPU): pairs beyond `capacity` dropped
    float capacity_factor = 1.f;
    int min_capacity = 0;
};

// Top-K entries of a pair dropped by the capacity limit carry this bit (the slot stays in the
// low bits for the debug output); the sort, the GEMMs and the combine skip them.
constexpr int kDroppedPair = 1 << 30;

// Token rows read through the decoder layer's post-attention RMSNorm applied on the fly:
// x[t][j] -> (x[t][j] * rms[t]) * w[j], each product rounded in that order (rms_norm_f32,
// src/rms_norm.cpp:9-33); rms == nullptr reads the rows as they are.
struct RowNorm {
    const float* rms = nullptr;  // [T] 1 / sqrt(sum of squares / H + eps) per token
    const float* w = nullptr;    // [H]
};
#ifdef __CUDACC__
__device__ __forceinline__ float4 norm_row4(float4 v, const RowNorm& n, int t, int j) {
    if (n.rms == nullptr) return v;
    const float s = __ldg(n.rms + t);
    const float4 g = __ldg(reinterpret_cast<const float4*>(n.w + j));
    return make_float4(__fmul_rn(__fmul_rn(v.x, s), g.x), __fmul_rn(__fmul_rn(v.y, s), g.y),
                       __fmul_rn(__fmul_rn(v.z, s), g.z), __fmul_rn(__fmul_rn(v.w, s), g.w));
}
#endif

// ---- router.cu
constexpr int kRouterTok = 16;  // tokens per router CTA (= dispatch chunk)
constexpr int kGemvMaxRows = 64; // token rows per GEMV work item
// Logits, then (topk = true) the top-K kernel with per-chunk slot counts (slot_of: expert ->
// placement slot, nullptr for slot = expert; topk_idx holds slots; mode: routing variant).
cudaError_t launch_router(const float* x, int T, int H, const float* Wr, int E, int K,
                          const float* bias, float* logits, float* probs, float* topk_w,
                          int* topk_idx, int* chunk_counts, const int* slot_of,
                          const RouteMode& mode, bool topk, cudaStream_t st, const RowNorm& nrm = {},
                          bool pdl = false);

// ---- dispatch.cu
constexpr int kMaxSegs = 80;  // >= E + 1 (E <= 64)
struct ItemsArgs {
    const int4* segs;         // {weight group, first row, rows, source rank (expert parallel)}
    const int* n_segs;
    const int* seg_ret;       // fused expert parallel: the source's return row of each
                              // segment's first row (nullptr otherwise)
    int2* aux_gu;             // fused expert parallel: per item {source rank, first return row}
    int2* aux_dn;
    int n_rb_gu, n_rb_dn;     // row blocks per item for gate_up / down
    int tile_n;               // token rows per tensor-core item
    int gemv;                 // 1: items of at most kGemvMaxRows rows for the GEMV path
    int4* items_gu;           // {group, row block, first row, rows}
    int4* items_dn;
    int* n_items;             // [2]: gate_up, down
};
struct PlanArgs {
    const int* chunk_counts;  // [n_chunks][E]
    int n_chunks, T, E, K;
    int* goff;                // [E + 1] routed-row offset of each expert (goff[E] = T*K)
    int* gcnt;                // [E]     routed rows of each expert
    int* chunk_base;          // [n_chunks][E]
    int4* segs;               // single-GPU segments + work items built in the same launch
    int* n_segs;              // (segs == NULL: expert-parallel mode, items built later)
    int shared_apart;         // 1: the shared expert runs as its own launch (no segment here)
    const int* slot_of;       // fused top-K: expert -> placement slot (nullptr: identity)
    RouteMode mode;           // fused top-K: routing variant
    ItemsArgs items;
};
cudaError_t launch_plan(const PlanArgs& a, cudaStream_t st, bool pdl = false);
// T <= kRouterTok (one chunk): top-K of every token and the plan in one launch.
cudaError_t launch_topk_plan(const float* logits, int T, int K, float* probs, float* topk_w,
                             int* topk_idx, const PlanArgs& a, cudaStream_t st, bool pdl = false);

cudaError_t launch_items(const ItemsArgs& a, cudaStream_t st);
// Capacity-limited routing (topkgating_full with drop_tokens, src/hunyuan_moe_full.cpp:205-305):
// every pair's priority among its slot's pairs in k-major order (all tokens' first choices
// before any second choice, tokens in order); pairs at or beyond `capacity` get kDroppedPair in
// topk_idx, weight 0, and leave their chunk's count.  One CTA.
cudaError_t launch_capacity(int* topk_idx, float* topk_w, int* chunk_counts, int T, int K, int E, int capacity,
                            cudaStream_t st);
// The same over an expert-parallel job: recs = every rank's choice record (stride
// ep_choice_rec(E)), this rank's tokens come after those of ranks 0..me-1; the capacity is
// computed on the device from the job's token count (floor(cf * K * T_job / E) in single
// precision, at least K and min_capacity).
cudaError_t launch_capacity_job(int* topk_idx, float* topk_w, int* chunk_counts, int T, int K, int E,
                                const int* recs, int N, int me, float cf, int min_capacity, cudaStream_t st);
// idx[i] = expert_of_slot[idx[i]] for i < n (top-K slots back to expert ids for the caller);
// the dropped-pair bit is cleared; expert_of_slot == nullptr: identity (only the bit is cleared).
cudaError_t launch_unmap_slots(int* idx, const int* expert_of_slot, int n, cudaStream_t st);

// xp_shared == nullptr: the shared expert's rows are written elsewhere (launch_shared_prep).
cudaError_t launch_scatter_gather(const float* x, int T, int H, int E, int K, const int* topk_idx,
                                  const int* chunk_base, int* slot_pos, __half* xp_routed,
                                  __half* xp_shared, cudaStream_t st, const RowNorm& nrm = {},
                                  bool pdl = false);
// The shared expert as its own launch: its fp16 rows xp[0, T) and its work items (one per
// 128-row block, all T rows) for gate_up and down; n_items[2].
cudaError_t launch_shared_prep(const float* x, int T, int H, __half* xp, int group, int n_rb_gu,
                               int n_rb_dn, int4* items_gu, int4* items_dn, int* n_items, cudaStream_t st,
                               const RowNorm& nrm = {});
// C: [N][ld] per-expert counts of every source rank (ld >= E).
cudaError_t launch_ep_segments(const int* C, int ld, int N, int rank, int el, int E, int T, int4* segs,
                               int* n_segs, cudaStream_t st);
// Fused expert parallel: the same receive segments listed local source first, then sources
// rank-1, rank-2, ... (rows stay where they are); seg_ret[i] = the source's position of the
// segment's first row among that source's expert-sorted pairs.
cudaError_t launch_ep_segments_fused(const int* C, int ld, int N, int rank, int el, int T, int4* segs,
                                     int* seg_ret, int* n_segs, cudaStream_t st);

// ---- ep_p2p.cu (expert-parallel dispatch / combine over NVLink peer memory)
constexpr int kEpMaxRanks = 8;
constexpr int kEpMaxK = 8;
// Metadata block of every rank (ints): flags [count | deliver | ready | choice][kEpMaxRanks],
// then the count matrix [kEpMaxRanks][E + 1] (E per-expert pair counts + the source's token
// count), then (capacity-limited routing) the choice-count records [kEpMaxRanks][ep_choice_rec]:
// a rank's pairs per (choice k, slot) [kEpMaxK][E] and its token count.
constexpr int kEpFlagCount = 0, kEpFlagDeliver = kEpMaxRanks, kEpFlagReady = 2 * kEpMaxRanks;
constexpr int kEpFlagChoice = 3 * kEpMaxRanks;
constexpr int kEpCountOff = 4 * kEpMaxRanks;
__host__ __device__ constexpr int ep_choice_off(int E) { return kEpCountOff + kEpMaxRanks * (E + 1); }
__host__ __device__ constexpr int ep_choice_rec(int E) { return kEpMaxK * E + 1; }
__host__ __device__ constexpr int ep_meta_ints(int E) { return ep_choice_off(E) + kEpMaxRanks * ep_choice_rec(E); }
struct EpPeers {  // every rank's buffers as mapped in this process (own entry: local)
    __half* xp[kEpMaxRanks];   // activation matrices
    __half* yr[kEpMaxRanks];   // routed-result matrices (fp16, same rows as xp)
    int* meta[kEpMaxRanks];
    __half* yret[kEpMaxRanks]; // results returned to each source, in its expert-sorted pair order
};
cudaError_t launch_ep_counts(const EpPeers& p, int N, int me, int E, int T, const int* gcnt, uint32_t epoch,
                             uint64_t budget_ns, int* err, cudaStream_t st);
// Capacity-limited routing across ranks: this rank's pairs per (choice, slot) and its token count
// (one ep_choice_rec record) into every rank's choice records, then a bounded wait for every
// rank's (peer memory).  The NCCL transport writes the record with launch_choice_record and
// gathers the records with ncclAllGather.
cudaError_t launch_ep_choice_counts(const EpPeers& p, int N, int me, int E, int K, int T, const int* topk_idx,
                                    uint32_t epoch, uint64_t budget_ns, int* err, cudaStream_t st);
cudaError_t launch_choice_record(const int* topk_idx, int T, int K, int E, int* rec, cudaStream_t st);
// Decode-size calls: every pair's row (fp16) into its owner's xp and the token rows into rows
// [0, T) of this rank's xp; slot_pos = expert-sorted positions; then this rank's delivery flag.
cudaError_t launch_ep_scatter(const EpPeers& p, int N, int me, int E, int el, int T, int H, int K, const float* x,
                              const int* topk_idx, const int* chunk_base, const int* goff, int* slot_pos,
                              unsigned int* done_ctas, uint32_t epoch, cudaStream_t st, const RowNorm& nrm = {});
cudaError_t launch_ep_wait(const EpPeers& p, int N, int me, int flag_off, uint32_t epoch, uint64_t budget_ns,
                           int* err, cudaStream_t st);
cudaError_t launch_ep_raise(const EpPeers& p, int N, int me, int flag_off, uint32_t epoch, cudaStream_t st);
// Decode-size calls: the received segments' result rows back into their sources' yret (at
// seg_ret), then this rank's ready flag on every rank.
cudaError_t launch_ep_push(const EpPeers& p, int N, int me, const int4* segs, const int* seg_ret, const int* n_segs,
                           int H, unsigned int* done_ctas, uint32_t epoch, int n_sms, cudaStream_t st);
// Fused expert parallel, before the GEMMs: slot_pos[t, k] = the pair's expert-sorted position
// (chunk_base + rank in chunk); every token row (fp16) into rows [0, T) of this rank's xp, and
// the pairs this rank owns into their rows of its xp.  The other pairs leave inside the gate_up
// GEMM (EpFuse).
cudaError_t launch_ep_local(const EpPeers& p, int N, int me, int E, int el, int T, int H, int K, const float* x,
                            const int* topk_idx, const int* chunk_base, const int* goff, int* slot_pos,
                            cudaStream_t st, const RowNorm& nrm = {});

// What the grouped GEMM's communication warps need in fused expert-parallel mode.
//   gate_up (mode 1): they store this rank's pairs owned elsewhere (fp16 rows of x) into the
//     owners' xp at their receive rows, then the last CTA raises this rank's delivery flag on
//     every rank; the producer loads an item's token rows from a source only after that
//     source's delivery flag of this call (bounded wait).
//   down (mode 2): after each item's epilogue they copy its routed result rows (this CTA's
//     128 columns) into the source rank's yret at the source's expert-sorted positions; the
//     last CTA then raises this rank's ready flag on every rank.
struct EpFuse {
    EpPeers peers;
    const int2* aux;         // per item {source rank, first return row}
    int N, me, el, E, K, T, H;
    const float* x;          // [T, H] fp32 token rows
    RowNorm nrm;             // the pre-norm applied while reading them (rms == nullptr: none)
    const int* topk_idx;     // [T, K] placement slots
    const int* slot_pos;     // [T, K] expert-sorted positions
    const int* goff;         // [E + 1] expert-sorted offsets of this rank's pairs
    unsigned int* done;      // CTA completion counter (reset to 0 by the last CTA)
    uint32_t epoch;
    uint64_t budget_ns;
};

// ---- gemm_tc.cu (tcgen05 grouped GEMM, 2-SM pairs)
constexpr int kNumBoxes = 3;
constexpr int kMaxBoxRows = 128;
__host__ __device__ constexpr int box_rows(int i) { return i == 0 ? 32 : i == 1 ? 64 : 128; }
struct GemmMaps {
    CUtensorMap b[kNumBoxes];  // token operand, fp16 [rows, K], box {64, box_rows(i)}, SW128
};
struct GemmArgs {
    const int4* items;             // {group, row-block pair, first row, rows}
    const int* n_items;
    const uint8_t* const* wtiles;  // [groups] tile base per group
    int wtype;
    int n_ks;                      // K / 64
    int n_rb;                      // 128-row tiles per group matrix
    int glu;                       // 1: gate_up + SwiGLU epilogue -> fp16; 0: down projection
    void* out;                     // gate_up: fp16 [rows, out_ld]; down: fp32 rows [0, shared_rows)
    __half* out_r;                 // down: fp16 rows [shared_rows, ...) (routed results)
    int shared_rows;
    int out_ld;
    int* err;
    int ep_mode;                   // 0: none; 1: gate_up with the token-row sends; 2: down with
                                   // the result pushes (fused expert parallel, `ep`)
};
cudaError_t launch_gemm_tc(const GemmMaps& maps, const GemmArgs& a, int n_sms, cudaStream_t st,
                           const EpFuse* ep = nullptr);

// ---- gemv.cu (decode path: weight streaming, mma.sync)
constexpr int kGemvBoxes = 4;
__host__ __device__ constexpr int gemv_box_rows(int i) { return 8 << i; }  // 8, 16, 32, 64
struct GemvMaps {
    CUtensorMap x[kGemvBoxes];  // activation operand, fp16 [rows, K], box {64, gemv_box_rows(i)}, SW128
};
// max_rows: the largest item (<= kGemvMaxRows); it sizes the activation stages.  Items of at
// most 8 rows (Q4_0 / Q8_0) run on the persistent streaming variant with n_sms CTAs.
// glu = 0 (down projection): rows below shared_rows go to `out` (fp32), the others to
// `out_r` (fp16, routed results); glu = 1: `out` fp16.
cudaError_t launch_gemv(const GemvMaps& maps, const int4* items, const int* n_items, int max_items,
                        const uint8_t* const* wtiles, int wtype, int n_ks, int glu, int max_rows,
                        void* out, int out_ld, __half* out_r, int shared_rows, int* err, int n_sms,
                        cudaStream_t st, bool pdl = false);

// ---- decode.cu
// The whole block for 1..8 tokens on one GPU (Q4_0 / Q8_0 weights) as one persistent
// cooperative kernel: router chains, top-K and plan, the shared and routed experts' weight
// streams and the combine, with device-side counters in place of kernel boundaries.
constexpr int kDecodeMaxT = 8;
constexpr int kDecodeMaxE = 64;
constexpr int kDecodeMaxRb = 64;  // H / 128
struct DecodeSync {               // zero between calls (the kernel's last CTA resets it)
    uint32_t router_done;         // router CTAs finished
    uint32_t xp_ready;            // the fp16 token rows are written
    uint32_t plan_ready;          // top-K, weights and the active slots are published
    uint32_t n_act;               // routed slots hit by the call
    uint32_t exit_cnt;            // CTAs finished
    uint32_t ticket;              // next list position to hand out
    uint32_t plan_claim;          // who publishes the plan: 0 open, 1 the certified pass, 2 the chains
    uint32_t weights_ready;       // the chains' top-K (weights, rank order) is published
    uint32_t spec_cert;           // tokens the certified pass has decided
    uint32_t spec_fail;           // a token whose selection it could not certify
    uint32_t spec_tok[kDecodeMaxT];     // (token, expert) bounds done, per token
    uint32_t gu_done[kDecodeMaxE + 1];  // gate_up items done, per group (0: shared, 1 + j: routed)
    uint32_t dn_done[kDecodeMaxRb];     // groups done, per down row block
    int32_t act_slot[kDecodeMaxE];      // active routed index j -> placement slot
    int32_t j_of[kDecodeMaxE];          // placement slot -> j (-1: not hit)
    uint64_t spec_mask[kDecodeMaxT];    // certified selection per token (bit = placement slot)
    double spec_lb[kDecodeMaxT * kDecodeMaxE];  // fp64 logit + bias per (token, expert)
    double spec_bd[kDecodeMaxT * kDecodeMaxE];  // bound on the chain's logit - spec_lb
};
struct DecodeMaps {
    CUtensorMap x;  // fp16 token rows (rows 0..7 used), box {64, 8}, SW128
    CUtensorMap h;  // fp16 SwiGLU rows of group g at rows 8g..8g+7, box {64, 8}, SW128
};
struct DecodeArgs {
    const float* x;         // [T, H]
    RowNorm nrm;            // the pre-norm (rms == nullptr: none)
    const float* resid;     // [T, H] or nullptr
    float* out;             // [T, H]
    int T, H, I, E, K, el;  // el: routed slots; the shared expert's tiles are group el
    const float* Wr;        // [E, H] router
    const float* bias;      // [E] or nullptr
    RouteMode mode;
    const int* slot_of;     // expert -> slot, or nullptr
    const uint8_t* const* gu;  // [el + 1] gate_up tiles per slot (shared last)
    const uint8_t* const* dn;  // [el + 1] down tiles
    float* logits;          // [T, E]
    float* probs;           // [T, E] or nullptr
    float* topk_w;          // [T, K]
    int* topk_idx;          // [T, K] (slots)
    __half* xp;             // [>= 8, H] fp16 token rows (DecodeMaps::x)
    __half* hb;             // [(el + 1) * 8, I] (DecodeMaps::h)
    float* ysh;             // [8, H] shared expert's result
    __half* yr;             // [el * 8, H] routed results, group 1 + j at rows 8j..8j+7
    DecodeSync* sync;
    int* err;
};
// Dynamic shared memory of the kernel (0: the shape does not fit it).
size_t decode_smem(int wtype, int T, int H, int E);
// cudaErrorNotSupported when the kernel cannot hold one CTA per SM (cooperative launch).
cudaError_t launch_decode(const DecodeMaps& maps, const DecodeArgs& a, int wtype, int n_sms, cudaStream_t st);

// ---- combine.cu
// out[t] = resid[t] + y_shared[t] + sum_k w[t,k] * y_routed[slot_pos[t,k]] (routed rows fp16)
cudaError_t launch_combine(const float* y_shared, const __half* y_routed, const int* slot_pos,
                           const float* topk_w, const float* resid, float* out, int T, int H,
                           int K, cudaStream_t st, bool pdl = false);

// ---- norm.cu
// rms[t] = 1 / sqrt(sum of squares / H + eps) over T rows of H (H % 64 == 0), the reference's
// rounding (rms_norm_f32's chain); the consumers apply (x * rms) * w while reading x (RowNorm).
cudaError_t launch_rms(const float* x, float eps, int T, int H, float* rms, cudaStream_t st);

}  // namespace hymoe
