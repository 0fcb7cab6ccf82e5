// Integration checker (TEST INFRASTRUCTURE ONLY): the reference's own decoder layer
// (src/decoder_layer.cpp:9-46) compiled twice from its unmodified source —
//   decoder_layer_forward_cpu   : as written, MoE = moe_forward_cpu (src/attention.cpp:191)
//   decoder_layer_forward_hymoe : the same file compiled with
//                                 -Dmoe_forward_cpu=hymoe_moe_forward_cpu
//                                 -Ddecoder_layer_forward_cpu=decoder_layer_forward_hymoe
//                                 so its MoE call (src/decoder_layer.cpp:38) runs on the GPU
//                                 through the C++ adapter and libhymoe.so
// — plus C entry points for tests.  Built into oracle/_ref/libhyref_gpu.so by oracle/Makefile.
#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <vector>

#include "hunyuan_model.h"
#include "hymoe_adapter.h"

void decoder_layer_forward_hymoe(const float* hidden_states, const DecoderLayerWeights& w,
                                 uint32_t n_tokens, const HunyuanConfig& cfg, const int* positions,
                                 float* output);

namespace {

void fill(std::vector<float>& v, const float* p, size_t n) {
    if (p) v.assign(p, p + n);
    else v.clear();
}

HunyuanConfig make_cfg(uint32_t H, uint32_t I, uint32_t K) {
    HunyuanConfig cfg;
    cfg.hidden_size = H;
    cfg.moe_intermediate_size = I;
    cfg.intermediate_size = I;
    cfg.moe_topk = K;
    cfg.compute_derived();
    return cfg;
}

}  // namespace

extern "C" {

// Attention shapes follow the default HunyuanConfig (32 query heads, 8 KV heads, head
// dim 128): qkv [6144, H], o [H, 4096], q/k norm [128].
void* hyref_layer_create(uint32_t H, uint32_t I, uint32_t E, const float* in_ln,
                         const float* post_ln, const float* qkv, const float* o, const float* qn,
                         const float* kn, const float* router_w, const float* shared_gu,
                         const float* shared_down, const float* const* experts_gu,
                         const float* const* experts_down) {
    HunyuanConfig cfg = make_cfg(H, I, 8);
    auto* w = new DecoderLayerWeights();
    fill(w->input_ln_weight, in_ln, H);
    fill(w->post_attn_ln_weight, post_ln, H);
    fill(w->attn.qkv_weight, qkv, static_cast<size_t>(cfg.qkv_total) * H);
    fill(w->attn.o_weight, o, static_cast<size_t>(H) * cfg.hidden_size_q);
    fill(w->attn.q_norm_weight, qn, cfg.attention_head_dim);
    fill(w->attn.k_norm_weight, kn, cfg.attention_head_dim);
    fill(w->moe.router_weight, router_w, static_cast<size_t>(E) * H);
    fill(w->moe.shared_gate_up, shared_gu, static_cast<size_t>(2) * I * H);
    fill(w->moe.shared_down, shared_down, static_cast<size_t>(H) * I);
    w->moe.num_experts = E;
    w->moe.experts.resize(E);
    for (uint32_t e = 0; e < E; ++e) {
        fill(w->moe.experts[e].gate_up, experts_gu[e], static_cast<size_t>(2) * I * H);
        fill(w->moe.experts[e].down, experts_down[e], static_cast<size_t>(H) * I);
    }
    return w;
}

void hyref_layer_destroy(void* w) { delete static_cast<DecoderLayerWeights*>(w); }

// Puts another layer's MoE weights into the same DecoderLayerWeights object.
// in_place = 0: the reference's per-layer streaming on one object
//   (src/hunyuan_full_model.cpp:195-207): release_layer clears and shrinks every vector
//   (:119-130), then the next load fills vectors of the same sizes;
// in_place = 1: the new values are written over the old ones, so every address stays.
// Returns 1 when the router's data sits at its previous address afterwards, else 0.
int hyref_layer_reload_moe(void* wp, uint32_t H, uint32_t I, uint32_t E, const float* router_w,
                           const float* shared_gu, const float* shared_down,
                           const float* const* experts_gu, const float* const* experts_down,
                           int in_place) {
    MoEWeights& m = static_cast<DecoderLayerWeights*>(wp)->moe;
    const void* before = m.router_weight.data();
    const size_t gu = static_cast<size_t>(2) * I * H, dn = static_cast<size_t>(H) * I;
    if (in_place) {
        std::copy(router_w, router_w + static_cast<size_t>(E) * H, m.router_weight.begin());
        std::copy(shared_gu, shared_gu + gu, m.shared_gate_up.begin());
        std::copy(shared_down, shared_down + dn, m.shared_down.begin());
        for (uint32_t e = 0; e < E; ++e) {
            std::copy(experts_gu[e], experts_gu[e] + gu, m.experts[e].gate_up.begin());
            std::copy(experts_down[e], experts_down[e] + dn, m.experts[e].down.begin());
        }
    } else {
        m.shared_gate_up.clear(); m.shared_gate_up.shrink_to_fit();
        m.shared_down.clear(); m.shared_down.shrink_to_fit();
        m.router_weight.clear(); m.router_weight.shrink_to_fit();
        for (auto& e : m.experts) {
            e.gate_up.clear(); e.gate_up.shrink_to_fit();
            e.down.clear(); e.down.shrink_to_fit();
        }
        m.experts.clear();
        fill(m.router_weight, router_w, static_cast<size_t>(E) * H);
        fill(m.shared_gate_up, shared_gu, gu);
        fill(m.shared_down, shared_down, dn);
        m.num_experts = E;
        m.experts.resize(E);
        for (uint32_t e = 0; e < E; ++e) {
            fill(m.experts[e].gate_up, experts_gu[e], gu);
            fill(m.experts[e].down, experts_down[e], dn);
        }
    }
    return m.router_weight.data() == before ? 1 : 0;
}

// which = 0: the reference layer as written; 1: the same source with the GPU MoE.
// Returns 0, or 1 when the GPU path threw (the message goes to stderr).
int hyref_layer_forward(const float* x, const void* w, uint32_t T, uint32_t H, uint32_t I,
                        uint32_t K, int which, float* out) {
    const HunyuanConfig cfg = make_cfg(H, I, K);
    std::vector<int> pos(T);
    for (uint32_t t = 0; t < T; ++t) pos[t] = static_cast<int>(t);
    const auto& lw = *static_cast<const DecoderLayerWeights*>(w);
    try {
        if (which == 0) decoder_layer_forward_cpu(x, lw, T, cfg, pos.data(), out);
        else decoder_layer_forward_hymoe(x, lw, T, cfg, pos.data(), out);
    } catch (const std::exception& e) {
        fprintf(stderr, "%s\n", e.what());
        return 1;
    }
    return 0;
}

// The MoE alone: which = 0 moe_forward_cpu, 1 hymoe_moe_forward_cpu (the adapter).
int hyref_moe_forward(const float* x, const void* w, uint32_t T, uint32_t H, uint32_t I,
                      uint32_t K, int which, float* out, float* dbg_probs, float* dbg_w,
                      int32_t* dbg_idx) {
    const HunyuanConfig cfg = make_cfg(H, I, K);
    const MoEWeights& m = static_cast<const DecoderLayerWeights*>(w)->moe;
    try {
        if (which == 0) moe_forward_cpu(x, m, T, cfg, out, dbg_probs, dbg_w, dbg_idx);
        else hymoe_moe_forward_cpu(x, m, T, cfg, out, dbg_probs, dbg_w, dbg_idx);
    } catch (const std::exception& e) {
        fprintf(stderr, "%s\n", e.what());
        return 1;
    }
    return 0;
}

void hyref_release() { hymoe_adapter::release(); }

}  // extern "C"
