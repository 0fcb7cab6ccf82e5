// C entry points into the reference's own MoE code, compiled from the reference
// sources where they lie (src/attention.cpp, src/rms_norm.cpp, src/hunyuan_model.cpp).
//
// TEST INFRASTRUCTURE ONLY.  This shim is linked into oracle/_ref/libhyref.so, which
// tests, the golden-fixture script and bench.py's CPU-baseline leg use as the checker
// (and, for `bench.py --impl reference`, as the timed reference).  It is never part of
// the product library.
//
// It builds the reference's MoEWeights / HunyuanConfig from plain pointers and calls
//   moe_forward_cpu   (src/attention.cpp:191-313, decl src/hunyuan_model.h:147-156)
//   swiglu_ffn_f32    (src/rms_norm.cpp:39-91)
//   rms_norm_f32      (src/rms_norm.cpp:9-33)
//   topkgating_full   (src/hunyuan_moe_full.cpp:119-350)
// unchanged.
#include "hunyuan_model.h"
#include "hunyuan_moe_full.h"

#include <algorithm>

#include <cstdint>
#include <cstring>

namespace {

void fill(std::vector<float>& v, const float* p, size_t n) {
    if (p) v.assign(p, p + n);
    else v.clear();  // expert never selected by the caller's tokens
}

}  // namespace

extern "C" {

// Weights in PyTorch [out, in] row-major F32, exactly as MoEWeights holds them
// (src/hunyuan_model.h:130-145).  experts_* may hold NULL for experts that no token
// selects; the reference would dereference an empty vector if one were selected.
void* hyref_weights_create(uint32_t H, uint32_t I, uint32_t E,
                           const float* router_w, const float* shared_gu,
                           const float* shared_down, const float* const* experts_gu,
                           const float* const* experts_down) {
    MoEWeights* w = new MoEWeights();
    const size_t gu = (size_t)2 * I * H, dn = (size_t)H * I;
    fill(w->router_weight, router_w, (size_t)E * H);
    fill(w->shared_gate_up, shared_gu, gu);
    fill(w->shared_down, shared_down, dn);
    w->num_experts = E;
    w->experts.resize(E);
    for (uint32_t e = 0; e < E; ++e) {
        fill(w->experts[e].gate_up, experts_gu ? experts_gu[e] : nullptr, gu);
        fill(w->experts[e].down, experts_down ? experts_down[e] : nullptr, dn);
    }
    return w;
}

void hyref_weights_destroy(void* w) { delete static_cast<MoEWeights*>(w); }

// Calls moe_forward_cpu.  `dbg_probs` receives what the reference writes to its
// debug_router_logits argument, which is the softmax output (src/attention.cpp:224-240,278).
void hyref_moe_forward(const float* x, const void* weights, uint32_t T, uint32_t H,
                       uint32_t I, uint32_t K, float* out, float* dbg_probs,
                       float* dbg_w, int32_t* dbg_idx) {
    HunyuanConfig cfg;
    cfg.hidden_size = H;
    cfg.moe_intermediate_size = I;
    cfg.intermediate_size = I;
    cfg.moe_topk = K;
    cfg.compute_derived();
    moe_forward_cpu(x, *static_cast<const MoEWeights*>(weights), T, cfg, out, dbg_probs,
                    dbg_w, dbg_idx);
}

void hyref_swiglu_ffn(const float* x, const float* gate_up, const float* down, float* out,
                      uint32_t n, uint32_t H, uint32_t I) {
    swiglu_ffn_f32(x, gate_up, down, out, n, H, I);
}

void hyref_rms_norm(const float* x, const float* weight, float* out, uint32_t T, uint32_t H,
                    float eps) {
    rms_norm_f32(x, weight, out, T, H, eps);
}

// The largest capacity topkgating_full can compute for these arguments.  It writes its
// dispatch mask with the capacity it computes, so the buffers are sized for this bound
// (moe_forward_full sizes them smaller, which is the heap overflow noted at
// src/hunyuan_moe_full.cpp:296).
uint32_t hyref_full_capacity_bound(uint32_t T, uint32_t E, uint32_t K, int drop_tokens,
                                   float capacity_factor, uint32_t min_capacity) {
    uint32_t c = drop_tokens ? std::max(K, (uint32_t)(capacity_factor * K * T / E)) : T;
    return std::max(c, min_capacity);
}

// Calls topkgating_full; mask / combine receive [T][E][capacity] with the capacity the call
// computed (returned in *capacity; at most hyref_full_capacity_bound).
int hyref_topkgating_full(const float* logits, uint32_t T, uint32_t E, uint32_t K,
                          int group_limited, uint32_t n_group, uint32_t topk_group,
                          int drop_tokens, float capacity_factor, uint32_t min_capacity,
                          int norm_topk_prob, float routed_scaling_factor, float* probs,
                          uint8_t* mask, float* combine, int32_t* exp_counts,
                          uint32_t* capacity, float* capacity_rate) {
    MoERoutingConfig cfg;
    cfg.num_experts = E;
    cfg.moe_topk = K;
    cfg.group_limited_greedy = group_limited != 0;
    cfg.n_group = n_group;
    cfg.topk_group = topk_group;
    cfg.drop_tokens = drop_tokens != 0;
    cfg.capacity_factor = capacity_factor;
    cfg.min_capacity = min_capacity;
    cfg.norm_topk_prob = norm_topk_prob != 0;
    cfg.routed_scaling_factor = routed_scaling_factor;
    const uint32_t bound = hyref_full_capacity_bound(T, E, K, drop_tokens, capacity_factor, min_capacity);
    MoEGateOutput out;
    out.alloc(T, E, K, bound, true);
    topkgating_full(logits, T, cfg, out);
    if (out.expert_capacity > bound) return -1;
    const size_t n = (size_t)T * E * out.expert_capacity;
    for (size_t i = 0; i < n; ++i) mask[i] = out.dispatch_mask[i] ? 1 : 0;
    std::memcpy(combine, out.combine_weights, n * sizeof(float));
    std::memcpy(probs, out.router_probs, (size_t)T * E * sizeof(float));
    std::memcpy(exp_counts, out.exp_counts, E * sizeof(int32_t));
    *capacity = out.expert_capacity;
    *capacity_rate = out.exp_capacity_rate;
    return 0;
}

}  // extern "C"
