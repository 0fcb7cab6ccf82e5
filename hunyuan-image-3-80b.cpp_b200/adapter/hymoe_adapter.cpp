// hymoe_adapter.cpp — see hymoe_adapter.h.  One process-wide GPU context (device from
// HYMOE_DEVICE, default 0) with one layer slot; the weights are uploaded again whenever the
// caller passes a different weight set (the reference streams one layer at a time,
// src/hunyuan_full_model.cpp:195-207).
//
// A weight set is recognised by its content, not its addresses: the reference's streaming
// loop keeps one DecoderLayerWeights object for every layer, release_layer frees every vector
// (clear + shrink_to_fit, src/hunyuan_full_model.cpp:119-130) and the next layer's load
// allocates vectors of the same sizes, which the allocator commonly places at the same
// addresses.  Each call therefore fingerprints every tensor (its size and 33 windows of 64
// bytes spread evenly over it, ends included: ~0.3 MB read for a full layer) and re-uploads
// when the fingerprint changes.  Two layers of the model differ in every window.  A caller
// that edits a few weights in place between calls calls hymoe_adapter::invalidate().
#include "hymoe_adapter.h"

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <stdexcept>
#include <string>

namespace {

// hymoe_create's bound on the tokens of one call; longer calls run as chunks of this size
// (every token's result is independent of the others', src/attention.cpp:246-309).
constexpr uint32_t kMaxContextTokens = 8192;

struct State {
    hymoe_ctx* ctx = nullptr;
    uint32_t H = 0, I = 0, E = 0, K = 0, max_tokens = 0;
    bool loaded = false;
    uint64_t fingerprint = 0;  // of the weight set on the device (valid when loaded)
};

std::mutex g_mu;
State g_state;

[[noreturn]] void raise(const char* what, hymoe_ctx* ctx) {
    throw std::runtime_error(std::string("hymoe: ") + what + ": " + hymoe_last_error(ctx));
}

// 64-bit multiply-xorshift mix over the sampled bytes.
struct Fingerprint {
    uint64_t h = 0x243F6A8885A308D3ull;
    void mix(uint64_t v) {
        h ^= v + 0x9E3779B97F4A7C15ull + (h << 6) + (h >> 2);
        h *= 0xBF58476D1CE4E5B9ull;
        h ^= h >> 31;
    }
    void bytes(const uint8_t* p, size_t n) {
        size_t i = 0;
        for (; i + 8 <= n; i += 8) {
            uint64_t w;
            std::memcpy(&w, p + i, 8);
            mix(w);
        }
        uint64_t tail = 0;
        std::memcpy(&tail, p + i, n - i);
        mix(tail ^ (static_cast<uint64_t>(n - i) << 56));
    }
    void tensor(const void* data, size_t nbytes, int64_t tag) {
        constexpr size_t kWin = 64;
        constexpr size_t kWindows = 33;
        mix(static_cast<uint64_t>(nbytes));
        mix(static_cast<uint64_t>(tag));
        if (!data || nbytes == 0) return;
        const uint8_t* p = static_cast<const uint8_t*>(data);
        if (nbytes <= kWin * kWindows) {
            bytes(p, nbytes);
            return;
        }
        for (size_t i = 0; i < kWindows; ++i) bytes(p + (nbytes - kWin) * i / (kWindows - 1), kWin);
    }
};

uint64_t fingerprint_of(const MoEWeights& w, uint32_t E) {
    Fingerprint f;
    f.tensor(w.router_weight.data(), w.router_weight.size() * sizeof(float), -1);
    f.tensor(w.shared_gate_up.data(), w.shared_gate_up.size() * sizeof(float), -2);
    f.tensor(w.shared_down.data(), w.shared_down.size() * sizeof(float), -3);
    for (uint32_t e = 0; e < E; ++e) {
        f.tensor(w.experts[e].gate_up.data(), w.experts[e].gate_up.size() * sizeof(float), 2 * e);
        f.tensor(w.experts[e].down.data(), w.experts[e].down.size() * sizeof(float), 2 * e + 1);
    }
    return f.h;
}

uint64_t fingerprint_of(const hymoe_adapter::MoEWeightsGGUF& w) {
    Fingerprint f;
    auto t = [&](const hymoe_tensor& x, int64_t tag) {
        f.mix(static_cast<uint64_t>(x.ggml_type));
        f.mix(static_cast<uint64_t>(x.ne[0]));
        f.mix(static_cast<uint64_t>(x.ne[1]));
        f.tensor(x.data, x.nbytes, tag);
    };
    t(w.router, -1);
    t(w.shared_gate_up, -2);
    t(w.shared_down, -3);
    for (size_t e = 0; e < w.experts_gate_up.size(); ++e) t(w.experts_gate_up[e], static_cast<int64_t>(2 * e));
    for (size_t e = 0; e < w.experts_down.size(); ++e) t(w.experts_down[e], static_cast<int64_t>(2 * e + 1));
    return f.h;
}

void ensure_context(const HunyuanConfig& cfg, uint32_t E, uint32_t n_tokens) {
    State& s = g_state;
    const uint32_t H = cfg.hidden_size, I = cfg.moe_intermediate_size, K = cfg.moe_topk;
    const uint32_t want = std::min(n_tokens, kMaxContextTokens);
    if (s.ctx && s.H == H && s.I == I && s.E == E && s.K == K && want <= s.max_tokens) return;
    if (s.ctx) hymoe_destroy(s.ctx);
    s = State{};
    hymoe_config c{};
    c.hidden_size = H;
    c.moe_intermediate_size = I;
    c.num_experts = E;
    c.moe_topk = K;
    c.num_layers = 1;
    c.max_tokens = std::max<uint32_t>(want, 4096);
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

// The MoE of n_tokens rows in calls of at most the context's max_tokens rows; each call's
// input, output and debug rows are the matching slices of the caller's arrays.
void run(const float* x, uint32_t n_tokens, float* out, float* dbg_probs, float* dbg_w,
         int32_t* dbg_idx) {
    const State& s = g_state;
    const bool any = dbg_probs || dbg_w || dbg_idx;
    uint32_t t0 = 0;
    do {
        const uint32_t n = std::min(s.max_tokens, n_tokens - t0);
        hymoe_debug dbg{};
        // the reference's "logits" argument holds probabilities (src/attention.cpp:224-240,278)
        dbg.router_probs = dbg_probs ? dbg_probs + static_cast<size_t>(t0) * s.E : nullptr;
        dbg.topk_weights = dbg_w ? dbg_w + static_cast<size_t>(t0) * s.K : nullptr;
        dbg.topk_indices = dbg_idx ? dbg_idx + static_cast<size_t>(t0) * s.K : nullptr;
        const size_t off = static_cast<size_t>(t0) * s.H;
        if (hymoe_forward(s.ctx, 0, x + off, nullptr, out + off, n, nullptr, any ? &dbg : nullptr,
                          HYMOE_HOST_PTRS) != HYMOE_OK)
            raise("hymoe_forward", s.ctx);
        t0 += n;
    } while (t0 < n_tokens);
}

}  // namespace

namespace hymoe_adapter {
void release() {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_state.ctx) hymoe_destroy(g_state.ctx);
    g_state = State{};
}

void invalidate() {
    std::lock_guard<std::mutex> lk(g_mu);
    g_state.loaded = false;
}
}  // namespace hymoe_adapter

void hymoe_moe_forward_cpu(const float* hidden_states, const MoEWeights& w, uint32_t n_tokens,
                           const HunyuanConfig& cfg, float* output, float* debug_router_logits,
                           float* debug_router_weights, int32_t* debug_router_indices) {
    std::lock_guard<std::mutex> lk(g_mu);
    const uint32_t E = w.num_experts, H = cfg.hidden_size, I = cfg.moe_intermediate_size;
    if (w.experts.size() < E) throw std::runtime_error("hymoe: MoEWeights holds fewer experts than num_experts");
    ensure_context(cfg, E, n_tokens);
    State& s = g_state;
    const uint64_t fp = fingerprint_of(w, E);
    if (!s.loaded || fp != s.fingerprint) {
        const hymoe_tensor router = view(w.router_weight, E, H);
        const hymoe_tensor sgu = view(w.shared_gate_up, 2 * I, H);
        const hymoe_tensor sdn = view(w.shared_down, H, I);
        std::vector<hymoe_tensor> egu(E), edn(E);
        for (uint32_t e = 0; e < E; ++e) {
            egu[e] = view(w.experts[e].gate_up, 2 * I, H);
            edn[e] = view(w.experts[e].down, H, I);
        }
        s.loaded = false;
        if (hymoe_load_layer(s.ctx, 0, &router, &sgu, &sdn, egu.data(), edn.data(),
                             HYMOE_HOST_PTRS) != HYMOE_OK)
            raise("hymoe_load_layer", s.ctx);
        s.fingerprint = fp;
        s.loaded = true;
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
    if (w.experts_down.size() != E) throw std::runtime_error("hymoe: expert tensor lists differ in length");
    ensure_context(cfg, E, n_tokens);
    State& s = g_state;
    const uint64_t fp = fingerprint_of(w);
    if (!s.loaded || fp != s.fingerprint) {
        s.loaded = false;
        if (hymoe_load_layer(s.ctx, 0, &w.router, &w.shared_gate_up, &w.shared_down,
                             w.experts_gate_up.data(), w.experts_down.data(), HYMOE_HOST_PTRS) != HYMOE_OK)
            raise("hymoe_load_layer", s.ctx);
        s.fingerprint = fp;
        s.loaded = true;
    }
    run(hidden_states, n_tokens, output, debug_router_logits, debug_router_weights,
        debug_router_indices);
}
