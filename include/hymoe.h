/* hymoe.h — C ABI of the B200 (sm_100a) MoE block library, libhymoe.so.
 *
 * Drop-in for the MoE step of the reference's decoder layer:
 *   void moe_forward_cpu(const float* hidden_states, const MoEWeights& w, uint32_t n_tokens,
 *                        const HunyuanConfig& cfg, float* output,
 *                        float* debug_router_logits, float* debug_router_weights,
 *                        int32_t* debug_router_indices)
 *   (declared src/hunyuan_model.h:147-156, defined src/attention.cpp:191-313,
 *    called from src/decoder_layer.cpp:38 with the residual added at :42)
 * and of the per-layer weight load it consumes
 *   HunyuanGGUFLoader::load_layer_weights (src/hunyuan_gguf_loader.cpp:229-281,
 *   tensor names blk.N.ffn_gate / ffn_shared_{gate_up,down} / ffn_expert_E_{gate_up,down}).
 *
 * Plain C types only.  Every call returns an hymoe_status; nothing aborts the process.
 * One context per host thread (calls on one context are serialised by the caller).
 */
#ifndef HYMOE_H
#define HYMOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    HYMOE_OK = 0,
    HYMOE_ERR_INVALID_ARG = 1, /* bad pointer, size, type or shape */
    HYMOE_ERR_CUDA = 2,        /* a CUDA runtime/driver call failed */
    HYMOE_ERR_OOM = 3,         /* device allocation failed */
    HYMOE_ERR_UNSUPPORTED = 4, /* configuration this build does not implement */
    HYMOE_ERR_NCCL = 5,        /* NCCL communicator error (expert-parallel mode) */
    HYMOE_ERR_TIMEOUT = 6,     /* a bounded device-side or collective wait expired */
    HYMOE_ERR_STATE = 7        /* call out of order (e.g. layer not loaded) */
} hymoe_status;

/* GGUF tensor types (GGUF numbering, as the reference's ggml_type at
 * src/hunyuan_gguf_loader.cpp:172-177). */
enum {
    HYMOE_TYPE_F32 = 0,
    HYMOE_TYPE_F16 = 1,
    HYMOE_TYPE_Q4_0 = 2, /* 32-element blocks: fp16 d, 16 bytes of nibbles; x = (q-8)*d */
    HYMOE_TYPE_Q8_0 = 8  /* 32-element blocks: fp16 d, 32 int8;            x = q*d     */
};

/* flags for hymoe_load_layer / hymoe_forward */
enum {
    HYMOE_HOST_PTRS = 1, /* pointers are host memory (copied H2D / D2H inside the call) */
    HYMOE_USE_GRAPH = 2, /* hymoe_forward, one GPU, device pointers: capture the call's device
                            work into a CUDA graph keyed by (layer, n_tokens, pointers) on first
                            use and replay it on later calls with the same key (removes launch
                            overhead in decode loops).  Graphs are dropped when a layer is
                            (re)loaded; profiling disables replay. */
    HYMOE_PRE_NORM = 4   /* hymoe_forward: x is the un-normalised hidden state h; the call first
                            applies the layer's post-attention RMSNorm (hymoe_set_norm) with the
                            reference's rounding, rms_norm_f32 (src/rms_norm.cpp:9-33) as
                            src/decoder_layer.cpp:34 applies it, and runs the MoE block on the
                            result.  With residual == x the call is decoder_layer's
                            out = h + moe(rms_norm(h)) (src/decoder_layer.cpp:34-42); with
                            HYMOE_HOST_PTRS, residual == x uploads x once. */
};

typedef struct hymoe_ctx hymoe_ctx;

/* Shapes mirror HunyuanConfig (src/hunyuan_model.h:13-45). */
typedef struct {
    uint32_t hidden_size;           /* H, 4096 (hidden_size, :14); multiple of 128        */
    uint32_t moe_intermediate_size; /* I, 3072 (moe_intermediate_size, :20); multiple of 64 */
    uint32_t num_experts;           /* E, 64 (num_experts, :21); 8..64                    */
    uint32_t moe_topk;              /* K, 8 (moe_topk, :22); 1..8                         */
    uint32_t num_layers;            /* layer slots this context holds                     */
    uint32_t max_tokens;            /* largest n_tokens of one hymoe_forward, <= 8192; with
                                       expert parallelism the same job-wide bound on every rank */
    int32_t device;                 /* CUDA device ordinal                                */
    /* Expert parallelism: ep_size ranks each own num_experts/ep_size consecutive
     * placement slots (consecutive experts unless hymoe_set_placement permutes them).
     * ep_size == 1 runs everything locally.  For ep_size > 1,
     * nccl_unique_id points at the 128-byte id from hymoe_nccl_unique_id() on rank 0;
     * every rank runs in its own process on its own GPU of one node.  Token rows and
     * results move over NVLink peer memory (ep_size <= 8; the ranks map each other's
     * buffers in hymoe_create), or by NCCL send/recv when the environment sets
     * HYMOE_EP_TRANSPORT=nccl.  A peer that stops taking part ends the call with
     * HYMOE_ERR_TIMEOUT after HYMOE_EP_TIMEOUT_S seconds (default 60). */
    int32_t ep_rank;
    int32_t ep_size;
    const void* nccl_unique_id;
} hymoe_config;

/* One GGUF tensor: raw GGUF bytes exactly as stored in the file.
 * ne[0] = input features (contiguous, blocks run along it), ne[1] = output rows,
 * i.e. PyTorch [out, in] row-major (scripts/convert_to_gguf.py:196-200 writes no
 * transpose).  nbytes must equal the GGUF size for (type, ne). */
typedef struct {
    const void* data;
    int32_t ggml_type;
    int64_t ne[2];
    size_t nbytes;
} hymoe_tensor;

/* Optional router outputs, any member may be NULL.  Same memory kind as x. */
typedef struct {
    float* router_logits; /* [T, E] pre-softmax logits (+bias)                          */
    float* router_probs;  /* [T, E] softmax; what moe_forward_cpu writes into its
                             debug_router_logits argument (src/attention.cpp:224-240,278) */
    float* topk_weights;  /* [T, K] renormalised (debug_router_weights)                  */
    int32_t* topk_indices;/* [T, K] rank order (debug_router_indices)                    */
} hymoe_debug;

/* Library version string. */
const char* hymoe_version(void);

/* Writes the 128-byte NCCL unique id that rank 0 hands to every rank. */
hymoe_status hymoe_nccl_unique_id(void* out128);

/* Creates a context on cfg->device; allocates the per-call scratch for max_tokens.
 * Expert-parallel contexts join the NCCL communicator here (collective across ranks). */
hymoe_status hymoe_create(const hymoe_config* cfg, hymoe_ctx** out);

/* Destroys the context and frees all device memory it owns. */
void hymoe_destroy(hymoe_ctx* ctx);

/* Message of the last failing call on this context ("" when none).  With ctx == NULL,
 * the last failure of hymoe_create on this thread. */
const char* hymoe_last_error(const hymoe_ctx* ctx);
/* (With ctx == NULL it also reports the last failure of hymoe_ffn_noalloc on this thread.) */

/* Makes subsequent work run on `stream` (a cudaStream_t; NULL = the context's own). */
hymoe_status hymoe_set_stream(hymoe_ctx* ctx, void* stream);

/* Waits for all work of the context and reports device-side errors (bounded waits that
 * expired, NCCL failures) as a status. */
hymoe_status hymoe_synchronize(hymoe_ctx* ctx);

/* Loads one layer's MoE weights (replaces HunyuanGGUFLoader::load_layer_weights for the
 * MoE tensors, src/hunyuan_gguf_loader.cpp:259-276).
 *   router        blk.N.ffn_gate.weight               [E, H], must be F32
 *   shared_gate_up blk.N.ffn_shared_gate_up.weight    [2I, H]  F32/F16/Q4_0/Q8_0
 *   shared_down    blk.N.ffn_shared_down.weight       [H, I]
 *   experts_gate_up[E] blk.N.ffn_expert_E_gate_up.weight [2I, H]
 *   experts_down[E]    blk.N.ffn_expert_E_down.weight    [H, I]
 * Rows 0..I-1 of gate_up are the gate (SiLU'd), rows I..2I-1 the up projection
 * (src/rms_norm.cpp:70-74).  The bytes are copied to the device and re-tiled there;
 * the caller's buffers may be freed on return.  F32 expert weights are rounded to
 * F16 on the device.  In expert-parallel mode a rank reads only the experts it owns;
 * the other entries may have data == NULL. */
hymoe_status hymoe_load_layer(hymoe_ctx* ctx, uint32_t layer, const hymoe_tensor* router,
                              const hymoe_tensor* shared_gate_up,
                              const hymoe_tensor* shared_down,
                              const hymoe_tensor* experts_gate_up,
                              const hymoe_tensor* experts_down, int flags);

/* Asynchronous hymoe_load_layer (host pointers) for layer streaming: the reference's loop
 * loads a layer, runs it and releases it (src/hunyuan_full_model.cpp:195-207); with this call the
 * next layer's upload runs while the current layer computes.  The tensors are checked and the
 * call returns at once: a loader thread of the context copies them to the device and re-tiles
 * them on its own stream, in the order of the calls.  The host bytes must stay valid and
 * unchanged until hymoe_wait_layer(ctx, layer) returns.  hymoe_forward on this layer may follow
 * immediately: a device-pointer call's work waits for the load on the GPU (no host wait); a
 * host-pointer or graph call waits on the host.  While a load is in flight, do not queue
 * copies from pageable host memory on the stream of a device-pointer call that waits for it
 * (such a copy first synchronises that stream on the host).  The slot is
 * rewritten only after every call already queued on the context's stream, so "load layer l+1
 * into the other slot, then run layer l" overlaps the two.  A failed load makes
 * hymoe_wait_layer and later hymoe_forward calls on that layer fail. */
hymoe_status hymoe_load_layer_async(hymoe_ctx* ctx, uint32_t layer, const hymoe_tensor* router,
                                    const hymoe_tensor* shared_gate_up,
                                    const hymoe_tensor* shared_down,
                                    const hymoe_tensor* experts_gate_up,
                                    const hymoe_tensor* experts_down);

/* Waits until every asynchronous load queued for `layer` has finished (its host buffers may then
 * be freed or reused) and returns the last one's status. */
hymoe_status hymoe_wait_layer(hymoe_ctx* ctx, uint32_t layer);

/* Fills a layer with synthetic weights generated on the device: every tensor ~N(0,std)
 * by the library's Philox4x32-10 / Irwin-Hall generator (one stream per tensor: layer in
 * the high 32 bits, kind 1 router / 2 gate_up / 3 down in bits 16-31, expert index or
 * 0xFFFF for the shared expert in the low 16), quantised to `ggml_type` with the GGUF
 * rule.  The router stays F32.  Bit-identical to the CPU generator of the test oracle.
 * Experts are those of this rank's placement slots.  No reference counterpart: it exists
 * so benchmarks can build 40+ GB of weights without a host round trip. */
hymoe_status hymoe_synth_layer(hymoe_ctx* ctx, uint32_t layer, int32_t ggml_type,
                               uint64_t seed, float stddev);

/* Post-attention RMSNorm weights of one layer for HYMOE_PRE_NORM calls: weight [H] F32
 * (GGUF blk.N.ffn_norm.weight; host memory with HYMOE_HOST_PTRS, else device), eps
 * (HunyuanConfig::rms_norm_eps, GGUF hunyuan.rms_norm_eps).  Copied; weight == NULL removes
 * them.  The first call also allocates a [max_tokens, H] F32 buffer for the normalised rows. */
hymoe_status hymoe_set_norm(hymoe_ctx* ctx, uint32_t layer, const float* weight, float eps, int flags);

/* Routing variant of the FULL-mode router, topkgating_full (MoERoutingConfig,
 * src/hunyuan_moe_full.h:25-47; src/hunyuan_moe_full.cpp:119-243), for every later call of the
 * context (every rank of an expert-parallel job sets the same):
 *   group_limited_greedy: experts in n_group groups of E/n_group (n_group <= 32 dividing E),
 *     each group scored by its largest probability; only the topk_group best groups'
 *     experts can be selected (ties: lower group);
 *   norm_topk_prob: weights = p / sum of the K selected p, the sum clamped below at 1e-8
 *     (with K > 1); otherwise weights = p * routed_scaling_factor;
 *   drop_tokens (capacity_factor, min_capacity): capacity-limited routing (moe_topk <= 8):
 *     capacity = floor(capacity_factor * K * T / E) in single precision, at least K and
 *     min_capacity; each expert keeps its first `capacity` pairs in k-major order (every
 *     token's first choice before any second choice, tokens in order) and the other pairs are
 *     dropped: they take no GEMM rows, add nothing to the output, and their debug weights
 *     read 0 (src/hunyuan_moe_full.cpp:205-305).  With expert parallelism T is the job's token
 *     count and the order runs over the job's tokens in rank order (rank 0's first), as one
 *     call over the concatenated tokens would; every rank must set the same routing.
 *     Without drop_tokens topkgating_full's capacity keeps every pair.
 * The debug probabilities stay the unmasked softmax (the reference's router_probs).
 * NULL restores moe_forward_cpu's routing (the default). */
typedef struct {
    int32_t group_limited_greedy;
    uint32_t n_group;
    uint32_t topk_group;
    int32_t drop_tokens;
    float capacity_factor;
    uint32_t min_capacity;
    int32_t norm_topk_prob;
    float routed_scaling_factor;
} hymoe_routing;
hymoe_status hymoe_set_routing(hymoe_ctx* ctx, const hymoe_routing* routing);

/* Expert placement of one layer for expert parallelism.  slot_of_expert[e] (a
 * permutation of 0..E-1; NULL = identity, the default) puts expert e in slot s, held by
 * rank s / (E/ep_size) as its local expert s % (E/ep_size).  Every rank must set the same
 * placement.  The layer's weights are marked unloaded: call hymoe_load_layer (or
 * hymoe_synth_layer) afterwards, which then loads the experts of this rank's slots.
 * Routing, outputs and the debug indices (expert ids) do not depend on the placement; it
 * only decides which rank computes which expert, so a placement that evens out the
 * ranks' expected rows shortens the slowest rank's GEMMs.  No reference counterpart (the
 * reference runs on one CPU). */
hymoe_status hymoe_set_placement(hymoe_ctx* ctx, uint32_t layer, const int32_t* slot_of_expert);

/* Host helper (no context, no device): a placement for hymoe_set_placement that balances
 * per-expert loads `load[n_experts]` (e.g. routed rows observed on a calibration batch)
 * over ep_size ranks of n_experts/ep_size experts each — greedy, heaviest expert first
 * (ties: lower expert), to the least-loaded rank with a free slot (ties: lower rank).
 * HYMOE_ERR_INVALID_ARG unless n_experts % ep_size == 0 and every load is >= 0. */
hymoe_status hymoe_balance_placement(uint32_t n_experts, uint32_t ep_size, const double* load,
                                     int32_t* slot_of_expert);

/* The MoE block of one decoder layer for n_tokens tokens:
 *   out[t] = residual[t] + shared(x[t]) + sum_k w[t,k] * expert_{idx[t,k]}(x[t])
 * (src/attention.cpp:191-313; residual add of src/decoder_layer.cpp:42 when residual
 * is non-NULL; out may alias residual).  x, residual and out are [n_tokens, H] F32
 * row-major.  router_bias [E] (nullable) is added to the router logits before the
 * softmax (no reference counterpart; 0 reproduces the reference).  In expert-parallel
 * mode every rank calls this with its own tokens (n_tokens may differ per rank).
 * With HYMOE_HOST_PTRS the call copies in, computes and copies out before returning;
 * otherwise it is asynchronous on the context's stream.  Host-pointer calls run as token
 * chunks whose copies overlap the compute: on one GPU calls of >= 2048 tokens without debug
 * outputs (up to 4 chunks of >= 2048 tokens); with expert parallelism every host-pointer call
 * of a context whose max_tokens is >= 4096 (max_tokens / 2048 chunks, at most 4, each rank
 * splitting its own tokens; every rank must pass HYMOE_HOST_PTRS on the same calls).  The
 * results equal one call's: every token's output is independent of the others'. */
hymoe_status hymoe_forward(hymoe_ctx* ctx, uint32_t layer, const float* x,
                           const float* residual, float* out, uint32_t n_tokens,
                           const float* router_bias, hymoe_debug* dbg, int flags);

/* Per-phase device timing for benchmarks and tracing: while enabled, hymoe_forward
 * brackets each phase with CUDA events on the context's stream.  No reference
 * counterpart (the reference has no timers). */
enum {
    HYMOE_PHASE_ROUTER = 0,   /* router GEMV (+ softmax + top-K when T > 16) */
    HYMOE_PHASE_PLAN = 1,     /* prefix scan + work lists (+ top-K, T <= 16) */
    HYMOE_PHASE_DISPATCH = 2, /* scatter / gather of token rows              */
    HYMOE_PHASE_GATE_UP = 3,  /* grouped gate_up GEMM + SwiGLU               */
    HYMOE_PHASE_DOWN = 4,     /* grouped down GEMM                           */
    HYMOE_PHASE_COMBINE = 5,  /* weighted combine + residual                 */
    HYMOE_PHASE_EP_DISPATCH = 6, /* expert-parallel token exchange           */
    HYMOE_PHASE_EP_COMBINE = 7,  /* expert-parallel result exchange          */
    HYMOE_PHASE_COPY_IN = 8,     /* HYMOE_HOST_PTRS: host -> device copies (summed over the
                                    copies; on pipelined calls they overlap the compute)  */
    HYMOE_PHASE_COPY_OUT = 9,    /* HYMOE_HOST_PTRS: device -> host copies                */
    HYMOE_NUM_PHASES = 10
};

/* enable != 0 clears the accumulators and starts recording; 0 stops. */
hymoe_status hymoe_profile(hymoe_ctx* ctx, int enable);

/* Waits for the context's stream, then writes for each of the first n phases the total
 * device milliseconds and the number of kernel launches (copies, for the copy phases)
 * recorded since recording began. */
hymoe_status hymoe_profile_read(hymoe_ctx* ctx, float* total_ms, int32_t* launches, int n);

/* Limits of hymoe_ffn_noalloc: its scratch is one fixed array per device. */
#define HYMOE_NOALLOC_MAX_TOKENS 8
#define HYMOE_NOALLOC_MAX_INTERMEDIATE 16384

/* One SwiGLU expert FFN for up to 8 tokens that allocates no device memory.
 * No counterpart in the reference: it exists for callers that cannot call cudaMalloc,
 * e.g. code running inside CUDA stream capture (allocation calls are not permitted
 * there), engines whose device memory belongs to another allocator or pool, or decode
 * loops that must not allocate per step.  Needs no context.
 *   y[t] = down( silu(gate_up[0:I] x[t]) * gate_up[I:2I] x[t] )   (src/rms_norm.cpp:39-91)
 * gate_up [2I, H] and down [H, I] are standard GGUF tensors (F32/F16/Q4_0/Q8_0, one
 * type) whose data, like x [n_tokens, H] and y [n_tokens, H] (F32), are DEVICE pointers
 * owned by the caller, 16-byte aligned.  n_tokens <= HYMOE_NOALLOC_MAX_TOKENS,
 * I <= HYMOE_NOALLOC_MAX_INTERMEDIATE; larger sizes are rejected with
 * HYMOE_ERR_INVALID_ARG.  The intermediate activation lives in a 512 KiB static device
 * array that every GPU loading the library holds until process exit.  The first call on
 * a device looks up that array's device address (cudaGetSymbolAddress) with the device
 * current; make that first call before any stream capture.  Asynchronous on `stream`
 * (a cudaStream_t, NULL = legacy default stream).  All calls share the array: calls
 * that overlap on the GPU (unordered streams) race and give wrong results. */
hymoe_status hymoe_ffn_noalloc(const hymoe_tensor* gate_up, const hymoe_tensor* down,
                               const float* x, float* y, uint32_t n_tokens, void* stream);

/* ---- GGUF weight files (replaces HunyuanGGUFLoader, src/hunyuan_gguf_loader.h:20-71, for
 * the MoE tensors).  A file (GGUF version 2 or 3) is parsed by the library and mapped
 * read-only; tensors are views of their raw GGUF blocks in the mapping, valid until
 * hymoe_gguf_close.  Every count, length and extent in the file is checked against its
 * size: a malformed file gives HYMOE_ERR_INVALID_ARG (HYMOE_ERR_UNSUPPORTED for another
 * version), never a read outside the mapping.  Host-only: no context, no device. */
typedef struct hymoe_gguf hymoe_gguf;

/* Opens and parses `path` (HunyuanGGUFLoader::open_layer, src/hunyuan_gguf_loader.cpp:125). */
hymoe_status hymoe_gguf_open(const char* path, hymoe_gguf** out);
void hymoe_gguf_close(hymoe_gguf* file);
/* Message of this thread's last failing hymoe_gguf_* call. */
const char* hymoe_gguf_last_error(void);

/* Tensor `name` as a host view: data in the mapping, ggml_type, ne[0] innermost (GGUF
 * order: columns), ne[1] rows, nbytes of its blocks.  F32/F16/Q4_0/Q8_0 tensors of 1 or 2
 * dimensions; other types or ranks give HYMOE_ERR_UNSUPPORTED
 * (HunyuanGGUFLoader::load_tensor, src/hunyuan_gguf_loader.cpp:150-161, without the
 * dequantisation). */
hymoe_status hymoe_gguf_tensor(const hymoe_gguf* file, const char* name, hymoe_tensor* out);

/* A u32 metadata value, e.g. "hunyuan.num_experts" (HunyuanGGUFLoader::get_metadata_u32,
 * src/hunyuan_gguf_loader.cpp:286-291). */
hymoe_status hymoe_gguf_get_u32(const hymoe_gguf* file, const char* key, uint32_t* out);

/* The MoE tensors of decoder layer `layer_idx` under the reference converter's names
 * (scripts/convert_to_gguf.py:70-137; read at src/hunyuan_gguf_loader.cpp:260-277):
 * blk.N.ffn_gate (router), blk.N.ffn_shared_gate_up / _down, and
 * blk.N.ffn_expert_E_gate_up / _down for E < n_experts (arrays of n_experts). */
hymoe_status hymoe_gguf_moe_tensors(const hymoe_gguf* file, uint32_t layer_idx, uint32_t n_experts,
                                    hymoe_tensor* router, hymoe_tensor* shared_gate_up,
                                    hymoe_tensor* shared_down, hymoe_tensor* experts_gate_up,
                                    hymoe_tensor* experts_down);

/* hymoe_gguf_moe_tensors for the context's E experts, then hymoe_load_layer from the
 * mapping (HYMOE_HOST_PTRS) into layer slot `layer` (HunyuanGGUFLoader::load_layer_weights,
 * src/hunyuan_gguf_loader.cpp:229-281, for the MoE part).  Expert blocks are read as
 * standard GGUF Q4_0/Q8_0 (not the reference loader's Q4_0 decode,
 * src/hunyuan_gguf_loader.cpp:41-72).  A router stored as F16/Q8_0/Q4_0 (the reference's
 * converter gives every tensor of a layer one type) is decoded to F32 on the host first. */
hymoe_status hymoe_load_layer_gguf(hymoe_ctx* ctx, uint32_t layer, const hymoe_gguf* file,
                                   uint32_t layer_idx);

/* hymoe_load_layer_gguf through hymoe_load_layer_async: the file must stay open until
 * hymoe_wait_layer(ctx, layer) returns. */
hymoe_status hymoe_load_layer_gguf_async(hymoe_ctx* ctx, uint32_t layer, const hymoe_gguf* file,
                                         uint32_t layer_idx);

#ifdef __cplusplus
}
#endif
#endif /* HYMOE_H */
