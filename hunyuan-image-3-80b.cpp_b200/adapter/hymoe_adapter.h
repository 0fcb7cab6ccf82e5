// hymoe_adapter.h — drop-in for the reference's moe_forward_cpu, for C++ hosts.
//
// Compiled in the host's own tree, next to its src/hunyuan_model.h (MoEWeights,
// HunyuanConfig).  hymoe_moe_forward_cpu has exactly the parameters and results of
//   moe_forward_cpu (src/hunyuan_model.h:147-156, src/attention.cpp:191-313)
// and computes on the GPU through libhymoe.so.  A host switches by calling it at its call
// site (src/decoder_layer.cpp:38, src/hunyuan_extended.cpp:217) or, without touching the
// source, by compiling that file with -Dmoe_forward_cpu=hymoe_moe_forward_cpu.
#pragma once

#include <cstdint>
#include <vector>

#include "hunyuan_model.h"
#include "hymoe.h"

namespace hymoe_adapter {

// Raw GGUF tensors of one layer's MoE, as HunyuanGGUFLoader reads them before it
// dequantises (src/hunyuan_gguf_loader.cpp:163-223): the quantised sibling of MoEWeights.
// `data` points at host memory the caller keeps alive until the next call.
struct MoEWeightsGGUF {
    hymoe_tensor router{};                 // blk.N.ffn_gate.weight, F32 [E, H]
    hymoe_tensor shared_gate_up{};         // blk.N.ffn_shared_gate_up.weight
    hymoe_tensor shared_down{};            // blk.N.ffn_shared_down.weight
    std::vector<hymoe_tensor> experts_gate_up;  // blk.N.ffn_expert_E_gate_up.weight
    std::vector<hymoe_tensor> experts_down;     // blk.N.ffn_expert_E_down.weight
};

// Releases the adapter's GPU context (device memory, weights).  Optional at exit.
void release();

}  // namespace hymoe_adapter

// Same contract as moe_forward_cpu: output = shared + routed MoE of the (post-attention
// RMS-normalised) hidden states; debug_router_logits receives the softmax probabilities,
// as the reference writes them.  Weights (F32 MoEWeights) are uploaded when a different
// weight set is passed; GPU errors are thrown as std::runtime_error.
void hymoe_moe_forward_cpu(const float* hidden_states, const MoEWeights& w, uint32_t n_tokens,
                           const HunyuanConfig& cfg, float* output,
                           float* debug_router_logits = nullptr,
                           float* debug_router_weights = nullptr,
                           int32_t* debug_router_indices = nullptr);

// The same with quantised (raw GGUF Q4_0 / Q8_0 / F16 / F32) expert weights.
void hymoe_moe_forward_gguf(const float* hidden_states, const hymoe_adapter::MoEWeightsGGUF& w,
                            uint32_t n_tokens, const HunyuanConfig& cfg, float* output,
                            float* debug_router_logits = nullptr,
                            float* debug_router_weights = nullptr,
                            int32_t* debug_router_indices = nullptr);
