// hymoe_adapter.cpp — see hymoe_adapter.h.  One process-wide GPU context (device from
// HYMOE_DEVICE, default 0) with one layer slot; the weights are re-uploaded when the caller
// passes a different weight set (the reference streams one layer at a time,
// src/hunyuan_full_model.cpp:195-207).
#include "hymoe_adapter.h"

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <stdexcept>
#include <string>

namespace {

struct State {
    hymoe_ctx* ctx = nullptr;
    uint32_t H = 0, I = 0, E = 0, K = 0, max_tokens = 0;
    const void* key[4] = {nullptr, nullptr, nullptr, nullptr};  // identity of the loaded weights
};

std::mutex g_mu;
State g_state;

[[noreturn]] void raise(const char* what, hymoe_ctx* ctx) {
    throw std::runtime_error(std::string("hymoe: ") + what + ": " + hymoe_last_error(ctx));
}

void ensure_context(const HunyuanConfig& cfg, uint32_t E, uint32_t n_tokens) {
    State& s = g_state;
    const uint32_t H = cfg.hidden_size, I = cfg.moe_intermediate_size, K = cfg.moe_topk;
    if (s.ctx && s.H == H && s.I == I && s.E == E && s.K == K && n_tokens <= s.max_tokens) return;
    if (s.ctx) hymoe_destroy(s.ctx);
    s = State{};
    hymoe_config c{};
    c.hidden_size = H;
    c.moe_intermediate_size = I;
    c.num_experts = E;
    c.moe_topk = K;
    c.num_layers = 1;
    c.max_tokens = n_tokens > 4096 ? n_tokens : 4096;
    const char* dev = getenv("HYMOE_DEVICE");
    c.device = dev ? atoi(dev) : 0;
    c.ep_rank = 0;
    c.ep_size = 1;
    if (hymoe_create(&c, &s.ctx) != HYMOE_OK) raise("hymoe_create", nullptr);
    s.H = H;
    s.I = I;
    s.E = E;
    s.K = K;
    s.max_tokens = c.max_tokens;
}

hymoe_tensor view(const std::vector<float>& v, int64_t rows, int64_t cols) {
    hymoe_tensor t{};
    t.data = v.data();
    t.ggml_type = HYMOE_TYPE_F32;
    t.ne[0] = cols;
    t.ne[1] = rows;
    t.nbytes = v.size() * sizeof(float);
    return t;
}

void run(const float* x, uint32_t n_tokens, float* out, float* dbg_logits, float* dbg_w,
         int32_t* dbg_idx) {
    hymoe_debug dbg{};
    dbg.router_probs = dbg_logits;  // the reference's "logits" argument holds probabilities
    dbg.topk_weights = dbg_w;
    dbg.topk_indices = dbg_idx;
    const bool any = dbg_logits || dbg_w || dbg_idx;
    if (hymoe_forward(g_state.ctx, 0, x, nullptr, out, n_tokens, nullptr, any ? &dbg : nullptr,
                      HYMOE_HOST_PTRS) != HYMOE_OK)
        raise("hymoe_forward", g_state.ctx);
}

}  // namespace

namespace hymoe_adapter {
void release() {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_state.ctx) hymoe_destroy(g_state.ctx);
    g_state = State{};
}
}  // namespace hymoe_adapter

void hymoe_moe_forward_cpu(const float* hidden_states, const MoEWeights& w, uint32_t n_tokens,
                           const HunyuanConfig& cfg, float* output, float* debug_router_logits,
                           float* debug_router_weights, int32_t* debug_router_indices) {
    std::lock_guard<std::mutex> lk(g_mu);
    const uint32_t E = w.num_experts, H = cfg.hidden_size, I = cfg.moe_intermediate_size;
    ensure_context(cfg, E, n_tokens);
    State& s = g_state;
    const void* key[4] = {&w, w.router_weight.data(), w.shared_gate_up.data(),
                          E ? w.experts[0].gate_up.data() : nullptr};
    if (std::memcmp(key, s.key, sizeof(key)) != 0) {
        const hymoe_tensor router = view(w.router_weight, E, H);
        const hymoe_tensor sgu = view(w.shared_gate_up, 2 * I, H);
        const hymoe_tensor sdn = view(w.shared_down, H, I);
        std::vector<hymoe_tensor> egu(E), edn(E);
        for (uint32_t e = 0; e < E; ++e) {
            egu[e] = view(w.experts[e].gate_up, 2 * I, H);
            edn[e] = view(w.experts[e].down, H, I);
        }
        if (hymoe_load_layer(s.ctx, 0, &router, &sgu, &sdn, egu.data(), edn.data(),
                             HYMOE_HOST_PTRS) != HYMOE_OK)
            raise("hymoe_load_layer", s.ctx);
        std::memcpy(s.key, key, sizeof(key));
    }
    run(hidden_states, n_tokens, output, debug_router_logits, debug_router_weights,
        debug_router_indices);
}

void hymoe_moe_forward_gguf(const float* hidden_states, const hymoe_adapter::MoEWeightsGGUF& w,
                            uint32_t n_tokens, const HunyuanConfig& cfg, float* output,
                            float* debug_router_logits, float* debug_router_weights,
                            int32_t* debug_router_indices) {
    std::lock_guard<std::mutex> lk(g_mu);
    const uint32_t E = static_cast<uint32_t>(w.experts_gate_up.size());
    ensure_context(cfg, E, n_tokens);
    State& s = g_state;
    const void* key[4] = {&w, w.router.data, w.shared_gate_up.data,
                          E ? w.experts_gate_up[0].data : nullptr};
    if (std::memcmp(key, s.key, sizeof(key)) != 0) {
        if (w.experts_down.size() != E) throw std::runtime_error("hymoe: expert tensor lists differ in length");
        if (hymoe_load_layer(s.ctx, 0, &w.router, &w.shared_gate_up, &w.shared_down,
                             w.experts_gate_up.data(), w.experts_down.data(), HYMOE_HOST_PTRS) != HYMOE_OK)
            raise("hymoe_load_layer", s.ctx);
        std::memcpy(s.key, key, sizeof(key));
    }
    run(hidden_states, n_tokens, output, debug_router_logits, debug_router_weights,
        debug_router_indices);
}
