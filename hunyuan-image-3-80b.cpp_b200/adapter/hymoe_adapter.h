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

// Makes the next call upload its weights again.  The adapter tells weight sets apart by a
// fingerprint of sampled bytes of every tensor (never by their addresses, which the
// reference's layer-streaming loop reuses from layer to layer); call this after editing a
// few weights of a set in place between two calls.
void invalidate();

}  // namespace hymoe_adapter

// Same contract as moe_forward_cpu: output = shared + routed MoE of the (post-attention
// RMS-normalised) hidden states; debug_router_logits receives the softmax probabilities,
// as the reference writes them.  Weights (F32 MoEWeights) are uploaded whenever their content
// differs from the set on the device (sizes and sampled bytes of every tensor), so one
// MoEWeights object refilled layer after layer is uploaded for each layer.  Any n_tokens is
// accepted: calls above 8192 tokens run as 8192-token chunks.  GPU errors are thrown as
// std::runtime_error.
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
