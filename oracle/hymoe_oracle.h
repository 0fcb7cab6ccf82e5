/* hymoe_oracle.h — CPU oracle for the MoE block (TEST INFRASTRUCTURE ONLY).
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load this
 * library, and only as the checker.  The product library (libhymoe.so) never links it.
 *
 * Parity pin: the restatement is checked bit-for-bit against the reference's own
 * moe_forward_cpu (src/attention.cpp:191-313), compiled from the reference sources
 * into oracle/_ref/libhyref.so, and against golden fixtures generated from that
 * compiled reference (tests/golden/).  GGUF block (de)quantisation is checked against
 * gguf-py 0.19.0 `gguf.quants` byte-for-byte.
 */
#ifndef HYMOE_ORACLE_H
#define HYMOE_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGUF tensor types used on this path (GGUF spec numbering). */
enum { ORACLE_F32 = 0, ORACLE_F16 = 1, ORACLE_Q4_0 = 2, ORACLE_Q8_0 = 8 };

/* Synthetic-tensor stream ids: stream = layer << 32 | kind << 16 | index. */
enum {
    ORACLE_KIND_ROUTER = 1,  /* index 0 */
    ORACLE_KIND_GATE_UP = 2, /* index = expert, 0xFFFF = shared expert */
    ORACLE_KIND_DOWN = 3,    /* index = expert, 0xFFFF = shared expert */
    ORACLE_KIND_BIAS = 4,    /* index 0 */
    ORACLE_KIND_X = 5,       /* index 0 */
};
#define ORACLE_SHARED_INDEX 0xFFFFu

/* Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as easy as
 * 1, 2, 3", SC'11). */
void oracle_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]);

/* Element i of the synthetic stream: one Philox block with counter
 * {lo(i), hi(i), lo(stream), hi(stream)} and key {lo(seed), hi(seed)}; its 8 16-bit
 * halves u_j sum to S; value = (float)(S - 262140) * c, c = float(stddev*sqrt(1.5)/65536)
 * (Irwin-Hall sum of 8 uniforms: mean 0, standard deviation `stddev`). */
float oracle_synth_scale(float stddev);
void oracle_fill_normal(float* dst, uint64_t n, uint64_t seed, uint64_t stream,
                        float stddev, int nthreads);

/* IEEE binary16 conversions (round to nearest even; subnormals kept). */
uint16_t oracle_f32_to_f16(float f);
float oracle_f16_to_f32(uint16_t h);

/* GGUF blocks: Q4_0 = f16 d + 16 bytes (element j low nibble of byte j, element j+16
 * high nibble), x = (q - 8) * d.  Q8_0 = f16 d + 32 int8, x = q * d.  n % 32 == 0. */
uint64_t oracle_type_nbytes(int type, uint64_t n);
void oracle_quantize(int type, const float* x, uint8_t* dst, uint64_t n);
void oracle_dequantize(int type, const uint8_t* src, float* dst, uint64_t n);

/* Synthetic GGUF tensor of `n` elements: fill_normal -> quantize to `type`. */
void oracle_synth_tensor(int type, uint8_t* dst, uint64_t n, uint64_t seed, uint64_t stream,
                         float stddev, int nthreads);
/* Same tensor as the oracle consumes it: quantize then dequantize to F32. */
void oracle_synth_tensor_f32(int type, float* dst, uint64_t n, uint64_t seed, uint64_t stream,
                             float stddev, int nthreads);

/* RMSNorm, restating src/rms_norm.cpp:9-33. */
void oracle_rms_norm(const float* x, const float* weight, float* out, uint32_t T, uint32_t H,
                     float eps);

/* SwiGLU FFN over n rows, restating src/rms_norm.cpp:39-91. */
void oracle_swiglu_ffn(const float* x, const float* gate_up, const float* down, float* out,
                       uint32_t n, uint32_t H, uint32_t I, int nthreads);

/* Router: logits (+bias), softmax, top-K, renormalise; restating
 * src/attention.cpp:213-276 with an optional per-expert bias added after the dot
 * product.  Any output pointer may be NULL. */
void oracle_router(const float* x, uint32_t T, uint32_t H, uint32_t E, uint32_t K,
                   const float* router_w, const float* bias, float* logits, float* probs,
                   float* topk_w, int32_t* topk_idx, int nthreads);

/* Full MoE block, restating src/attention.cpp:191-313 (+ the caller's residual add,
 * src/decoder_layer.cpp:42, when `resid` is non-NULL).  experts_* hold E pointers;
 * an entry may be NULL when no token selects that expert.  Returns 0, or -1 when a
 * selected expert's weights are NULL. */
int oracle_moe_forward(const float* x, const float* resid, uint32_t T, uint32_t H, uint32_t I,
                       uint32_t E, uint32_t K, const float* router_w, const float* bias,
                       const float* shared_gu, const float* shared_down,
                       const float* const* experts_gu, const float* const* experts_down,
                       float* out, float* dbg_logits, float* dbg_probs, float* dbg_w,
                       int32_t* dbg_idx, int nthreads);

/* FULL-mode routing, topkgating_full (src/hunyuan_moe_full.cpp:119-350), routing part:
 * softmax per token (probs, before any masking); optionally group-limited greedy (groups of
 * E/n_group experts scored by their largest probability, clamped below at 0; the topk_group
 * best groups kept, the others' probabilities zeroed); top-K of the (masked) probabilities;
 * capacity = max(K, (uint32)(capacity_factor*K*T/E)) when drop_tokens, else the largest
 * per-expert pair count, in both cases at least min_capacity; each pair's priority = its
 * position among the pairs of its expert in k-major order (every token's first choice, then
 * every token's second, ...), kept when below capacity; weights renormalised over the K
 * choices (sum clamped at 1e-8) when norm_topk_prob and K > 1, else scaled by
 * routed_scaling_factor.  Ties everywhere go to the lower index.
 * Outputs: probs [T,E], idx/w [T,K] (rank order; w is the combine weight of a kept pair),
 * keep [T,K], exp_counts [E] (all pairs), *capacity.  The auxiliary loss (training only) is
 * not restated.  E and n_group at most 256 (*capacity = 0 otherwise). */
void oracle_topkgating_full(const float* logits, uint32_t T, uint32_t E, uint32_t K,
                            int group_limited, uint32_t n_group, uint32_t topk_group,
                            int drop_tokens, float capacity_factor, uint32_t min_capacity,
                            int norm_topk_prob, float routed_scaling_factor, float* probs,
                            int32_t* idx, float* w, uint8_t* keep, int32_t* exp_counts,
                            uint32_t* capacity);

#ifdef __cplusplus
}
#endif
#endif
