// hymoe_api.cu — the C ABI (include/hymoe.h): context, device weight store, and the
// per-call orchestration of the MoE block on one GPU or expert-parallel over several.
//
// Forward pipeline for one layer call (on the context's stream):
//   [H2D x, residual]        (HYMOE_HOST_PTRS; >= 2048 tokens: pipelined token chunks with
//                            the copies on two copy streams)
//   router                   logits (+ softmax / top-K / renorm + per-chunk expert counts)
//   plan_kernel              per-expert counts, offsets and chunk bases of the pair sort and
//                            the work items (topk_plan_kernel: top-K + plan, <= 16 tokens)
//   scatter_gather_kernel    stable counting sort of (token, rank) pairs into fp16 rows;
//                            shared-expert rows go to rows [0, T) of the GEMM input
//   [expert parallel]        peer memory: counts to every rank, rows stored straight into
//                            the owners' matrices (ep_p2p.cu; tensor-core calls send them from
//                            inside the gate_up GEMM, overlapped with its MMAs); or NCCL:
//                            all-gather of counts and grouped ncclSend/ncclRecv of the rows
//   items_kernel             GEMM work items from the row segments (expert parallel)
//   gate_up GEMM             tcgen05 grouped GEMM + SwiGLU epilogue -> h (fp16); decode
//                            sizes (groups <= 64 rows): weight-streaming kernels, the shared
//                            expert on a forked stream for 4-8 tokens
//   down GEMM                -> y (shared expert, fp32) and yr (routed, fp16)
//   [expert parallel]        peer memory: results pushed back into each source's return
//                            matrix (tensor-core calls: from inside the down GEMM, item by
//                            item), ready flags; or NCCL: routed results back to their sources
//   combine_kernel           out = residual + shared + sum_k w_k y_k
//   [D2H out, debug]         (HYMOE_HOST_PTRS only)
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <nccl.h>

#include <chrono>
#include <cmath>
#include <cstdlib>
#include <thread>

#include <algorithm>
#include <condition_variable>
#include <cstdarg>
#include <deque>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/hymoe.h"
#include "common.cuh"
#include "kernels.h"

using namespace hymoe;

namespace {

thread_local std::string g_create_error;

struct LayerStore {
    bool loaded = false;
    int wtype = -1;                    // device tile type (Q4_0 / Q8_0 / F16)
    float* router = nullptr;           // [E, H] f32
    uint8_t* gu = nullptr;             // groups x gate_up tiles
    uint8_t* dn = nullptr;             // groups x down tiles
    const uint8_t** d_gu_ptrs = nullptr;  // device [groups] tile bases
    const uint8_t** d_dn_ptrs = nullptr;
};

size_t gguf_nbytes(int type, int64_t n) {
    switch (type) {
        case HYMOE_TYPE_F32: return static_cast<size_t>(n) * 4;
        case HYMOE_TYPE_F16: return static_cast<size_t>(n) * 2;
        case HYMOE_TYPE_Q4_0: return static_cast<size_t>(n / 32) * 18;
        case HYMOE_TYPE_Q8_0: return static_cast<size_t>(n / 32) * 34;
        default: return 0;
    }
}

int tile_type_for(int ggml_type) {
    return ggml_type == HYMOE_TYPE_Q4_0 ? W_Q4_0 : ggml_type == HYMOE_TYPE_Q8_0 ? W_Q8_0 : W_F16;
}

using EncodeTiledFn = PFN_cuTensorMapEncodeTiled_v12000;

EncodeTiledFn get_encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

using WaitValueFn = PFN_cuStreamWaitValue32_v11070;
using WriteValueFn = PFN_cuStreamWriteValue32_v11070;

// Stream memory operations (the wait happens in the GPU's front end: no kernel, no SM).
struct StreamMemOps {
    WaitValueFn wait = nullptr;
    WriteValueFn write = nullptr;
};
const StreamMemOps& stream_mem_ops() {
    static StreamMemOps ops;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuStreamWaitValue32", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            ops.wait = reinterpret_cast<WaitValueFn>(p);
        p = nullptr;
        if (cudaGetDriverEntryPoint("cuStreamWriteValue32", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            ops.write = reinterpret_cast<WriteValueFn>(p);
    });
    return ops;
}

using AddressRangeFn = PFN_cuMemGetAddressRange_v3020;

// Base of the allocation holding `p` (an IPC handle maps the whole allocation).
bool allocation_base(const void* p, uintptr_t* base) {
    static AddressRangeFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<AddressRangeFn>(f);
    });
    if (!fn) return false;
    CUdeviceptr b = 0;
    size_t sz = 0;
    if (fn(&b, &sz, reinterpret_cast<CUdeviceptr>(p)) != CUDA_SUCCESS) return false;
    *base = static_cast<uintptr_t>(b);
    return true;
}

}  // namespace

namespace hymoe {
void set_thread_error(const char* msg) { g_create_error = msg ? msg : ""; }
}  // namespace hymoe

struct GraphKey {
    uint32_t layer, n_tokens;
    const void* p[8];
    GraphKey(uint32_t l, uint32_t n, const void* a, const void* b, const void* c, const void* d,
             const void* e, const void* f, const void* g, const void* h)
        : layer(l), n_tokens(n), p{a, b, c, d, e, f, g, h} {}
    bool operator<(const GraphKey& o) const {
        if (layer != o.layer) return layer < o.layer;
        if (n_tokens != o.n_tokens) return n_tokens < o.n_tokens;
        for (int i = 0; i < 8; ++i)
            if (p[i] != o.p[i]) return p[i] < o.p[i];
        return false;
    }
};

constexpr int kChunkMinTokens = 2048;  // host-pointer calls of at least this size are pipelined

struct hymoe_ctx {
    hymoe_config cfg{};
    std::string err;
    cudaStream_t own_stream = nullptr;
    cudaStream_t copy_stream = nullptr;  // host-pointer calls: chunk uploads beside the compute
    cudaStream_t down_stream = nullptr;  // ... and chunk downloads
    cudaStream_t side_stream = nullptr;  // decode calls: the shared expert beside the router
    cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
    bool pdl = true;  // decode chains with programmatic dependent launch (HYMOE_PDL=0 at create: off)
    int4 *items_sh_gu = nullptr, *items_sh_dn = nullptr;
    int* n_items_sh = nullptr;
    cudaStream_t stream = nullptr;
    int n_sms = 148;
    int H = 0, I = 0, E = 0, K = 0;
    int groups = 0;           // local routed experts + shared
    int e_local = 0, e_first = 0;
    size_t gu_group_bytes = 0, dn_group_bytes = 0;
    std::vector<LayerStore> layers;
    // Expert placement per layer: empty = identity (slot s holds expert s).  Otherwise
    // expert_of_slot[l][s] is the expert in slot s, and place_dev[l] holds [E] slot_of then
    // [E] expert_of_slot on the device.  Slot s lives on rank s / e_local as local expert
    // s % e_local.
    std::vector<std::vector<int>> expert_of_slot;
    std::vector<int*> place_dev;
    // Post-attention RMSNorm per layer (hymoe_set_norm): [H] weights on the device (nullptr:
    // none) and eps; rms_buf holds a HYMOE_PRE_NORM call's per-token factors (the kernels that
    // read the token rows normalise them on the fly).
    std::vector<float*> norm_w;
    std::vector<float> norm_eps;
    float* rms_buf = nullptr;
    RouteMode route;  // routing variant (hymoe_set_routing); default: moe_forward_cpu's
    int expert_at(uint32_t layer, int slot) const {
        return expert_of_slot[layer].empty() ? slot : expert_of_slot[layer][slot];
    }

    // scratch (sized for max_tokens at create; expert-parallel receive side included)
    size_t rows_cap = 0;
    int max_items = 0;
    float *x_dev = nullptr, *resid_dev = nullptr, *out_dev = nullptr;
    float *logits = nullptr, *probs = nullptr, *topk_w = nullptr;
    int *topk_idx = nullptr, *chunk_counts = nullptr, *chunk_base = nullptr, *goff = nullptr;
    int *slot_pos = nullptr, *n_items = nullptr, *err_word = nullptr;
    int4 *items_gu = nullptr, *items_dn = nullptr;
    __half *xp = nullptr, *hbuf = nullptr;
    float* y = nullptr;        // shared expert's results [T, H] fp32
    __half* yr = nullptr;      // routed results, fp16, same row numbers as xp
    uint8_t* tmp = nullptr;   // load / synthesis staging of one GGUF tensor
    size_t tmp_bytes = 0;
    GemmMaps maps_xp{}, maps_h{};
    GemvMaps gmaps_xp{}, gmaps_h{};
    // One-kernel decode path (1..8 tokens on one GPU): its scratch, counters and maps.
    bool dec_ok = false;
    __half* dec_h = nullptr;   // [(el + 1) * 8, I]
    __half* dec_yr = nullptr;  // [el * 8, H]
    float* dec_ysh = nullptr;  // [8, H]
    DecodeSync* dec_sync = nullptr;
    DecodeMaps dec_maps{};

    float* bias_dev = nullptr;
    int4* segs = nullptr;
    int* n_segs = nullptr;
    int* seg_ret = nullptr;     // expert parallel (peer memory): return row of each segment
    int2 *aux_gu = nullptr, *aux_dn = nullptr;  // ... and per item {source, return row}
    float* dbg_w = nullptr;     // pipelined expert-parallel host calls: debug top-K weights
    int* dbg_idx = nullptr;     // and indices of every chunk (allocated on first use)
    int* gcnt = nullptr;

    // expert parallelism
    ncclComm_t comm = nullptr;
    bool comm_broken = false;
    __half* xp_send = nullptr;   // [T*K, H] routed rows in destination order
    __half* y_ret = nullptr;     // [T*K, H] routed results back from their ranks (fp16), in this
                                 // rank's expert-sorted pair order (peers write it directly)
    int* C_dev = nullptr;        // [N][E] gathered per-expert counts
    int* choice_dev = nullptr;   // [N][ep_choice_rec(E)] gathered choice records (NCCL transport)
    int* C_host = nullptr;       // pinned copy
    cudaEvent_t ev_counts = nullptr;
    double ep_timeout_s = 60.0;
    bool joining = false;  // communicator setup: connection establishment gets a longer budget
    double host_wait_s() const { return joining ? std::max(ep_timeout_s, 120.0) : ep_timeout_s; }

    // expert parallelism over NVLink peer memory (the default transport; HYMOE_EP_TRANSPORT=nccl
    // selects the NCCL send/recv exchange instead)
    bool p2p = false;
    EpPeers peers{};
    int* ep_meta = nullptr;             // this rank's flags + count matrix
    unsigned int* done_ctas = nullptr;  // dispatch completion counter
    uint32_t epoch = 0;                 // calls made; flags carry it
    std::vector<void*> ipc_opened;

    // Asynchronous layer loads (hymoe_load_layer_async): the caller's thread validates and queues
    // a job; the loader thread issues the job's copies and re-tiling on load_stream (pageable
    // host copies block only that thread), then writes ready[layer] = the job's epoch with a
    // stream memory operation; a forward of that layer makes its stream wait (in the GPU's front
    // end) for ready[layer] >= the last epoch issued for it.
    struct LoadJob {
        uint32_t layer = 0, epoch = 0;
        int wt = 0;
        float* d_router = nullptr;
        uint8_t *d_gu = nullptr, *d_dn = nullptr;
        size_t gu_bytes = 0, dn_bytes = 0;
        hymoe_tensor router{};
        std::vector<hymoe_tensor> gu, dn;  // per weight group (local experts, then shared)
        std::vector<float> router_f32;     // a router decoded on the host (GGUF)
        cudaEvent_t prior = nullptr;       // the caller's stream at the time of the call
    };
    std::thread loader;
    std::mutex lmu;
    std::condition_variable lcv, ldone;
    std::deque<LoadJob> jobs;
    bool lstop = false;
    cudaStream_t load_stream = nullptr;
    uint8_t* load_tmp = nullptr;        // one GGUF tensor in flight (the job's stream orders reuse)
    uint32_t* ready = nullptr;          // device [num_layers]: last completed load epoch per layer
    std::vector<uint32_t> issued, done;  // per layer: last epoch queued / finished (host)
    std::vector<hymoe_status> lstatus;  // per layer: status of the last finished load
    std::string lerr;                   // message of the last failed load

    std::map<GraphKey, cudaGraphExec_t> graphs;  // HYMOE_USE_GRAPH replays
    void clear_graphs() {
        for (auto& kv : graphs) cudaGraphExecDestroy(kv.second);
        graphs.clear();
    }

    // per-phase profiling (hymoe_profile)
    bool prof = false;
    std::vector<std::pair<cudaEvent_t, cudaEvent_t>> prof_ev[HYMOE_NUM_PHASES];
    int prof_launches[HYMOE_NUM_PHASES] = {};
    std::vector<cudaEvent_t> ev_pool;
    cudaEvent_t prof_open = nullptr;
    cudaEvent_t take_event() {
        cudaEvent_t e = nullptr;
        if (!ev_pool.empty()) {
            e = ev_pool.back();
            ev_pool.pop_back();
        } else {
            cudaEventCreate(&e);
        }
        return e;
    }
    void phase_begin() {
        if (!prof) return;
        prof_open = take_event();
        cudaEventRecord(prof_open, stream);
    }
    void phase_end(int phase, int launches = 1) {
        if (!prof || !prof_open) return;
        cudaEvent_t e = take_event();
        cudaEventRecord(e, stream);
        prof_ev[phase].emplace_back(prof_open, e);
        prof_launches[phase] += launches;
        prof_open = nullptr;
    }
    // An asynchronous copy on `s`, bracketed by profile events (phase COPY_IN / COPY_OUT) while
    // profiling is on.
    cudaError_t timed_copy(int phase, void* dst, const void* src, size_t bytes, cudaMemcpyKind kind,
                           cudaStream_t s) {
        if (bytes == 0) return cudaSuccess;
        cudaEvent_t a = nullptr;
        if (prof) {
            a = take_event();
            cudaEventRecord(a, s);
        }
        const cudaError_t e = cudaMemcpyAsync(dst, src, bytes, kind, s);
        if (prof) {
            cudaEvent_t b = take_event();
            cudaEventRecord(b, s);
            prof_ev[phase].emplace_back(a, b);
            prof_launches[phase] += 1;
        }
        return e;
    }
    void prof_clear() {
        for (auto& v : prof_ev) {
            for (auto& pr : v) {
                ev_pool.push_back(pr.first);
                ev_pool.push_back(pr.second);
            }
            v.clear();
        }
        for (int& n : prof_launches) n = 0;
    }

    hymoe_status fail(hymoe_status st, const char* fmt, ...) {
        char buf[512];
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(buf, sizeof(buf), fmt, ap);
        va_end(ap);
        err = buf;
        return st;
    }
    hymoe_status cuda_fail(cudaError_t e, const char* what) {
        return fail(e == cudaErrorMemoryAllocation ? HYMOE_ERR_OOM : HYMOE_ERR_CUDA,
                    "%s: %s", what, cudaGetErrorString(e));
    }
};

hymoe_status ep_poll(hymoe_ctx* c, const char* what);
hymoe_status ep_wait_event(hymoe_ctx* c, cudaEvent_t ev, const char* what);

#define HY_CUDA(ctx, call)                                          \
    do {                                                            \
        cudaError_t _e = (call);                                    \
        if (_e != cudaSuccess) return (ctx)->cuda_fail(_e, #call);  \
    } while (0)

namespace {

template <typename T>
cudaError_t dalloc(T** p, size_t count) {
    return cudaMalloc(reinterpret_cast<void**>(p), sizeof(T) * (count ? count : 1));
}

hymoe_status make_tmap(hymoe_ctx* c, CUtensorMap* map, void* base, uint64_t K, uint64_t rows,
                       uint32_t box_rows_) {
    EncodeTiledFn enc = get_encode_fn();
    if (!enc) return c->fail(HYMOE_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[2] = {K, rows};
    cuuint64_t strides[1] = {K * 2};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(kTileK), box_rows_};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return c->fail(HYMOE_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", r);
    return HYMOE_OK;
}

hymoe_status make_maps(hymoe_ctx* c, GemmMaps* m, GemvMaps* gm, void* base, uint64_t K, uint64_t rows) {
    for (int i = 0; i < kNumBoxes; ++i) {
        hymoe_status st = make_tmap(c, &m->b[i], base, K, rows, static_cast<uint32_t>(box_rows(i)));
        if (st != HYMOE_OK) return st;
    }
    for (int i = 0; i < kGemvBoxes; ++i) {
        hymoe_status st = make_tmap(c, &gm->x[i], base, K, rows, static_cast<uint32_t>(gemv_box_rows(i)));
        if (st != HYMOE_OK) return st;
    }
    return HYMOE_OK;
}

void free_layer(LayerStore& L) {
    cudaFree(L.router);
    cudaFree(L.gu);
    cudaFree(L.dn);
    cudaFree(L.d_gu_ptrs);
    cudaFree(L.d_dn_ptrs);
    L = LayerStore{};
}

hymoe_status ensure_layer(hymoe_ctx* c, uint32_t layer, int wtype) {
    LayerStore& L = c->layers[layer];
    const int TB = tile_bytes(wtype);
    const size_t gu_bytes = static_cast<size_t>(2 * c->I / kTileRows) * (c->H / kTileK) * TB;
    const size_t dn_bytes = static_cast<size_t>(c->H / kTileRows) * (c->I / kTileK) * TB;
    if (L.gu && L.wtype == wtype) return HYMOE_OK;
    free_layer(L);
    L.wtype = wtype;
    c->gu_group_bytes = gu_bytes;
    c->dn_group_bytes = dn_bytes;
    HY_CUDA(c, dalloc(&L.router, static_cast<size_t>(c->E) * c->H));
    HY_CUDA(c, dalloc(&L.gu, gu_bytes * c->groups));
    HY_CUDA(c, dalloc(&L.dn, dn_bytes * c->groups));
    HY_CUDA(c, dalloc(&L.d_gu_ptrs, c->groups));
    HY_CUDA(c, dalloc(&L.d_dn_ptrs, c->groups));
    std::vector<const uint8_t*> gp(c->groups), dp(c->groups);
    for (int g = 0; g < c->groups; ++g) {
        gp[g] = L.gu + gu_bytes * g;
        dp[g] = L.dn + dn_bytes * g;
    }
    HY_CUDA(c, cudaMemcpy(L.d_gu_ptrs, gp.data(), sizeof(void*) * c->groups, cudaMemcpyHostToDevice));
    HY_CUDA(c, cudaMemcpy(L.d_dn_ptrs, dp.data(), sizeof(void*) * c->groups, cudaMemcpyHostToDevice));
    return HYMOE_OK;
}

bool tensor_ok(const hymoe_tensor* t, int64_t rows, int64_t cols, int want_type) {
    if (!t || !t->data) return false;
    if (t->ne[0] != cols || t->ne[1] != rows) return false;
    if (want_type >= 0 && t->ggml_type != want_type) return false;
    const size_t nb = gguf_nbytes(t->ggml_type, rows * cols);
    return nb != 0 && t->nbytes == nb;
}

// Copies (if on host) and re-tiles one expert matrix into `dst`.
hymoe_status load_matrix(hymoe_ctx* c, const hymoe_tensor* t, uint8_t* dst, int dst_type,
                         int rows, int K, int glu_I, bool host) {
    const uint8_t* src = static_cast<const uint8_t*>(t->data);
    if (host) {
        HY_CUDA(c, cudaMemcpyAsync(c->tmp, t->data, t->nbytes, cudaMemcpyHostToDevice, c->stream));
        src = c->tmp;
    }
    HY_CUDA(c, launch_repack(src, t->ggml_type, dst, dst_type, rows, K, glu_I, c->stream));
    if (host) HY_CUDA(c, cudaStreamSynchronize(c->stream));  // tmp is reused by the next tensor
    return HYMOE_OK;
}

// Validates one layer's tensors for this rank (hymoe_load_layer's rules); *wt = the device tile
// type.
hymoe_status check_layer_tensors(hymoe_ctx* c, uint32_t layer, const hymoe_tensor* router,
                                 const hymoe_tensor* shared_gate_up, const hymoe_tensor* shared_down,
                                 const hymoe_tensor* experts_gate_up, const hymoe_tensor* experts_down, int* wt) {
    const int H = c->H, I = c->I, E = c->E;
    if (!tensor_ok(router, E, H, HYMOE_TYPE_F32))
        return c->fail(HYMOE_ERR_INVALID_ARG, "router must be F32 [E=%d, H=%d]", E, H);
    if (!shared_gate_up || !shared_down || !experts_gate_up || !experts_down)
        return c->fail(HYMOE_ERR_INVALID_ARG, "null tensor array");
    const int gt = shared_gate_up->ggml_type;
    if (gt != HYMOE_TYPE_F32 && gt != HYMOE_TYPE_F16 && gt != HYMOE_TYPE_Q4_0 && gt != HYMOE_TYPE_Q8_0)
        return c->fail(HYMOE_ERR_INVALID_ARG, "unsupported GGUF type %d", gt);
    if (!tensor_ok(shared_gate_up, 2 * I, H, gt) || !tensor_ok(shared_down, H, I, gt))
        return c->fail(HYMOE_ERR_INVALID_ARG, "shared expert tensors: bad shape/type/size");
    for (int le = 0; le < c->e_local; ++le) {
        const int ge = c->expert_at(layer, c->e_first + le);
        if (!tensor_ok(&experts_gate_up[ge], 2 * I, H, gt) || !tensor_ok(&experts_down[ge], H, I, gt))
            return c->fail(HYMOE_ERR_INVALID_ARG,
                           "expert %d tensors: bad shape/size or type differs from the shared expert", ge);
    }
    *wt = tile_type_for(gt);
    return HYMOE_OK;
}

// Loader thread: one job at a time, in queue order.  Every step is issued on load_stream; the
// ready flag is written even after a failure (the waiting forward must not wait forever), and
// the failure is kept for hymoe_wait_layer / hymoe_forward / hymoe_synchronize.
hymoe_status run_load_job(hymoe_ctx* c, hymoe_ctx::LoadJob& j, std::string* msg) {
    cudaStream_t s = c->load_stream;
    const int H = c->H, I = c->I;
    cudaError_t e = cudaStreamWaitEvent(s, j.prior, 0);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(j.d_router, j.router.data, j.router.nbytes, cudaMemcpyHostToDevice, s);
    for (size_t g = 0; g < j.gu.size() && e == cudaSuccess; ++g) {
        e = cudaMemcpyAsync(c->load_tmp, j.gu[g].data, j.gu[g].nbytes, cudaMemcpyHostToDevice, s);
        if (e == cudaSuccess)
            e = launch_repack(c->load_tmp, j.gu[g].ggml_type, j.d_gu + j.gu_bytes * g, j.wt, 2 * I, H, I, s);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(c->load_tmp, j.dn[g].data, j.dn[g].nbytes, cudaMemcpyHostToDevice, s);
        if (e == cudaSuccess)
            e = launch_repack(c->load_tmp, j.dn[g].ggml_type, j.d_dn + j.dn_bytes * g, j.wt, H, I, 0, s);
    }
    const CUresult w = stream_mem_ops().write(reinterpret_cast<CUstream>(s),
                                              reinterpret_cast<CUdeviceptr>(c->ready + j.layer), j.epoch,
                                              CU_STREAM_WRITE_VALUE_DEFAULT);
    const cudaError_t sync = cudaStreamSynchronize(s);  // the caller's host buffers are free after this
    if (e != cudaSuccess || sync != cudaSuccess || w != CUDA_SUCCESS) {
        cudaGetLastError();
        *msg = std::string("asynchronous load of layer ") + std::to_string(j.layer) + ": " +
               (w != CUDA_SUCCESS && e == cudaSuccess && sync == cudaSuccess
                    ? "cuStreamWriteValue32 failed"
                    : cudaGetErrorString(e != cudaSuccess ? e : sync));
        return HYMOE_ERR_CUDA;
    }
    return HYMOE_OK;
}

void loader_main(hymoe_ctx* c) {
    cudaSetDevice(c->cfg.device);
    while (true) {
        hymoe_ctx::LoadJob job;
        {
            std::unique_lock<std::mutex> lk(c->lmu);
            c->lcv.wait(lk, [&] { return c->lstop || !c->jobs.empty(); });
            if (c->jobs.empty()) return;
            job = std::move(c->jobs.front());
            c->jobs.pop_front();
        }
        std::string msg;
        const hymoe_status st = run_load_job(c, job, &msg);
        cudaEventDestroy(job.prior);
        {
            std::lock_guard<std::mutex> lk(c->lmu);
            c->done[job.layer] = job.epoch;
            c->lstatus[job.layer] = st;
            if (st != HYMOE_OK) c->lerr = msg;
        }
        c->ldone.notify_all();
    }
}

// Starts the loader thread and its stream, staging buffer and ready flags (first use).
hymoe_status ensure_loader(hymoe_ctx* c) {
    if (c->loader.joinable()) return HYMOE_OK;
    const StreamMemOps& ops = stream_mem_ops();
    if (!ops.wait || !ops.write)
        return c->fail(HYMOE_ERR_UNSUPPORTED, "stream memory operations (cuStreamWaitValue32) are unavailable");
    const size_t n = c->layers.size();
    if (!c->load_stream) HY_CUDA(c, cudaStreamCreateWithFlags(&c->load_stream, cudaStreamNonBlocking));
    if (!c->load_tmp) HY_CUDA(c, dalloc(&c->load_tmp, c->tmp_bytes));
    if (!c->ready) {
        HY_CUDA(c, dalloc(&c->ready, n));
        HY_CUDA(c, cudaMemset(c->ready, 0, sizeof(uint32_t) * n));
    }
    c->issued.assign(n, 0);
    c->done.assign(n, 0);
    c->lstatus.assign(n, HYMOE_OK);
    c->lstop = false;
    c->loader = std::thread(loader_main, c);
    return HYMOE_OK;
}

// Waits until every queued load of `layer` (every layer: layer == UINT32_MAX) has finished;
// returns the status of the last finished load of that layer (HYMOE_OK for all layers unless
// one failed).
hymoe_status wait_loads(hymoe_ctx* c, uint32_t layer) {
    if (!c->loader.joinable()) return HYMOE_OK;
    std::unique_lock<std::mutex> lk(c->lmu);
    auto finished = [&](uint32_t l) { return c->done[l] >= c->issued[l]; };
    c->ldone.wait(lk, [&] {
        if (layer != UINT32_MAX) return finished(layer);
        for (uint32_t l = 0; l < c->issued.size(); ++l)
            if (!finished(l)) return false;
        return true;
    });
    if (layer != UINT32_MAX) return c->lstatus[layer];
    for (hymoe_status st : c->lstatus)
        if (st != HYMOE_OK) return st;
    return HYMOE_OK;
}

}  // namespace

namespace {

double now_s() {
    return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

}  // namespace

// Polls the non-blocking communicator until its pending operation is enqueued (or fails);
// on the deadline the communicator is aborted and marked broken.
hymoe_status ep_poll(hymoe_ctx* c, const char* what) {
    const double t0 = now_s();
    while (true) {
        ncclResult_t st = ncclSuccess;
        ncclResult_t r = ncclCommGetAsyncError(c->comm, &st);
        if (r != ncclSuccess || (st != ncclSuccess && st != ncclInProgress)) {
            c->comm_broken = true;
            return c->fail(HYMOE_ERR_NCCL, "%s: %s", what,
                           ncclGetErrorString(r != ncclSuccess ? r : st));
        }
        if (st == ncclSuccess) return HYMOE_OK;
        if (now_s() - t0 > c->host_wait_s()) {
            c->comm_broken = true;
            ncclCommAbort(c->comm);
            c->comm = nullptr;
            return c->fail(HYMOE_ERR_TIMEOUT, "%s: no progress within %.0f s", what, c->host_wait_s());
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

// Waits for `ev` with a deadline while watching the communicator for asynchronous errors.
hymoe_status ep_wait_event(hymoe_ctx* c, cudaEvent_t ev, const char* what) {
    const double t0 = now_s();
    while (true) {
        const cudaError_t q = cudaEventQuery(ev);
        if (q == cudaSuccess) return HYMOE_OK;
        if (q != cudaErrorNotReady) return c->cuda_fail(q, what);
        if (c->comm) {
            ncclResult_t st = ncclSuccess;
            ncclCommGetAsyncError(c->comm, &st);
            if (st != ncclSuccess && st != ncclInProgress) {
                c->comm_broken = true;
                return c->fail(HYMOE_ERR_NCCL, "%s: %s", what, ncclGetErrorString(st));
            }
        }
        if (now_s() - t0 > c->host_wait_s()) {
            c->comm_broken = true;
            if (c->comm) ncclCommAbort(c->comm);
            c->comm = nullptr;
            return c->fail(HYMOE_ERR_TIMEOUT, "%s: no completion within %.0f s", what, c->host_wait_s());
        }
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}

// ============================================================================ C ABI

extern "C" {

const char* hymoe_version(void) { return "hymoe 0.1 (sm_100a)"; }

hymoe_status hymoe_nccl_unique_id(void* out128) {
    if (!out128) return HYMOE_ERR_INVALID_ARG;
    static_assert(sizeof(ncclUniqueId) == 128, "NCCL unique id is 128 bytes");
    return ncclGetUniqueId(static_cast<ncclUniqueId*>(out128)) == ncclSuccess ? HYMOE_OK
                                                                              : HYMOE_ERR_NCCL;
}

const char* hymoe_last_error(const hymoe_ctx* ctx) {
    return ctx ? ctx->err.c_str() : g_create_error.c_str();
}

// Maps every rank's xp, y and metadata block into this process (CUDA IPC; the handles travel
// through the communicator).  Every rank must own a distinct GPU and the same max_tokens.  The
// ranks agree on the outcome: either all use peer memory or all keep the NCCL exchange.
hymoe_status ep_p2p_setup(hymoe_ctx* c) {
    const int N = c->cfg.ep_size, me = c->cfg.ep_rank;
    const size_t meta_ints = static_cast<size_t>(ep_meta_ints(c->E));
    HY_CUDA(c, dalloc(&c->ep_meta, meta_ints));
    HY_CUDA(c, cudaMemset(c->ep_meta, 0, meta_ints * sizeof(int)));
    HY_CUDA(c, dalloc(&c->done_ctas, 1));
    HY_CUDA(c, cudaMemset(c->done_ctas, 0, sizeof(unsigned int)));
    constexpr int kBufs = 4;     // xp, yr, metadata, y_ret
    constexpr size_t kRec = 512;  // bytes per rank in the gathered buffer
    struct Rec {
        unsigned char uuid[16];
        uint32_t max_tokens, ok, pad[2];
        uint64_t off[kBufs];  // offset of each buffer inside the allocation its handle maps
        cudaIpcMemHandle_t h[kBufs];
    };
    static_assert(sizeof(Rec) <= kRec, "record");
    Rec mine{};
    cudaDeviceProp prop{};
    HY_CUDA(c, cudaGetDeviceProperties(&prop, c->cfg.device));
    memcpy(mine.uuid, &prop.uuid, 16);
    mine.max_tokens = c->cfg.max_tokens;
    mine.ok = 1;
    const void* bufs[kBufs] = {c->xp, c->yr, c->ep_meta, c->y_ret};
    for (int i = 0; i < kBufs; ++i) {
        uintptr_t base = 0;
        if (!allocation_base(bufs[i], &base) || cudaIpcGetMemHandle(&mine.h[i], reinterpret_cast<void*>(base)) != cudaSuccess) {
            cudaGetLastError();
            mine.ok = 0;
            break;
        }
        mine.off[i] = reinterpret_cast<uintptr_t>(bufs[i]) - base;
    }
    char* dbuf = nullptr;
    HY_CUDA(c, dalloc(&dbuf, kRec * (N + 1)));
    std::vector<Rec> recs(N);
    auto gather = [&]() -> hymoe_status {
        HY_CUDA(c, cudaMemcpy(dbuf, &mine, sizeof(Rec), cudaMemcpyHostToDevice));
        ncclResult_t r = ncclAllGather(dbuf, dbuf + kRec, kRec, ncclChar, c->comm, c->stream);
        if (r != ncclSuccess && r != ncclInProgress)
            return c->fail(HYMOE_ERR_NCCL, "ncclAllGather(peer handles): %s", ncclGetErrorString(r));
        hymoe_status s2 = ep_poll(c, "peer handle exchange");
        if (s2 != HYMOE_OK) return s2;
        cudaEvent_t ev = c->take_event();
        HY_CUDA(c, cudaEventRecord(ev, c->stream));
        s2 = ep_wait_event(c, ev, "peer handle exchange");
        c->ev_pool.push_back(ev);
        if (s2 != HYMOE_OK) return s2;
        for (int s = 0; s < N; ++s)
            HY_CUDA(c, cudaMemcpy(&recs[s], dbuf + kRec * (s + 1), sizeof(Rec), cudaMemcpyDeviceToHost));
        return HYMOE_OK;
    };
    hymoe_status st = gather();
    if (st != HYMOE_OK) {
        cudaFree(dbuf);
        return st;
    }
    for (int s = 0; s < N; ++s) {
        if (recs[s].max_tokens != c->cfg.max_tokens) {
            cudaFree(dbuf);
            return c->fail(HYMOE_ERR_INVALID_ARG, "rank %d has max_tokens %u, rank %d has %u (must be one job-wide bound)",
                           s, recs[s].max_tokens, me, c->cfg.max_tokens);
        }
        for (int u = 0; u < s; ++u)
            if (memcmp(recs[s].uuid, recs[u].uuid, 16) == 0) {
                cudaFree(dbuf);
                return c->fail(HYMOE_ERR_UNSUPPORTED, "ranks %d and %d run on the same GPU; expert parallelism "
                               "needs one GPU per rank", u, s);
            }
    }
    bool all_ok = true;
    for (int s = 0; s < N; ++s) all_ok = all_ok && recs[s].ok;
    EpPeers P{};
    P.xp[me] = c->xp;
    P.yr[me] = c->yr;
    P.meta[me] = c->ep_meta;
    P.yret[me] = c->y_ret;
    for (int s = 0; s < N && all_ok && mine.ok; ++s) {
        if (s == me) continue;
        void* ptr[kBufs] = {nullptr, nullptr, nullptr, nullptr};
        for (int i = 0; i < kBufs; ++i) {
            if (cudaIpcOpenMemHandle(&ptr[i], recs[s].h[i], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
                cudaGetLastError();
                mine.ok = 0;
                break;
            }
            c->ipc_opened.push_back(ptr[i]);
        }
        if (!mine.ok) break;
        P.xp[s] = reinterpret_cast<__half*>(static_cast<char*>(ptr[0]) + recs[s].off[0]);
        P.yr[s] = reinterpret_cast<__half*>(static_cast<char*>(ptr[1]) + recs[s].off[1]);
        P.meta[s] = reinterpret_cast<int*>(static_cast<char*>(ptr[2]) + recs[s].off[2]);
        P.yret[s] = reinterpret_cast<__half*>(static_cast<char*>(ptr[3]) + recs[s].off[3]);
    }
    // second round: every rank learns whether every rank mapped every peer
    if (all_ok) {
        st = gather();
        if (st != HYMOE_OK) {
            cudaFree(dbuf);
            return st;
        }
        for (int s = 0; s < N; ++s) all_ok = all_ok && recs[s].ok;
    }
    cudaFree(dbuf);
    if (!all_ok) {  // keep the NCCL exchange
        for (void* p : c->ipc_opened) cudaIpcCloseMemHandle(p);
        c->ipc_opened.clear();
        return HYMOE_OK;
    }
    c->peers = P;
    c->p2p = true;
    return HYMOE_OK;
}

hymoe_status hymoe_create(const hymoe_config* cfg, hymoe_ctx** out) {
    g_create_error.clear();
    if (!cfg || !out) {
        g_create_error = "null argument";
        return HYMOE_ERR_INVALID_ARG;
    }
    *out = nullptr;
    const uint32_t H = cfg->hidden_size, I = cfg->moe_intermediate_size, E = cfg->num_experts,
                   K = cfg->moe_topk;
    if (H == 0 || H % 128 || I == 0 || I % 64 || E < 1 || E > 64 || K < 1 || K > 8 || K > E ||
        cfg->max_tokens == 0 || cfg->max_tokens > 8192 || cfg->num_layers == 0 || cfg->ep_size < 1 ||
        cfg->ep_rank < 0 || cfg->ep_rank >= cfg->ep_size || E % cfg->ep_size) {
        g_create_error =
            "unsupported shape: need H%128==0, I%64==0, 1<=E<=64, 1<=K<=8, K<=E, E%ep_size==0, "
            "1<=max_tokens<=8192";
        return HYMOE_ERR_INVALID_ARG;
    }
    if (cudaSetDevice(cfg->device) != cudaSuccess) {
        g_create_error = "cudaSetDevice failed";
        return HYMOE_ERR_CUDA;
    }
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, cfg->device);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, cfg->device);
    if (major != 10 || minor != 0) {
        g_create_error = "this build targets sm_100a (B200); device is not compute capability 10.0";
        return HYMOE_ERR_UNSUPPORTED;
    }
    hymoe_ctx* c = new hymoe_ctx();
    c->cfg = *cfg;
    c->H = H;
    c->I = I;
    c->E = E;
    c->K = K;
    c->e_local = E / cfg->ep_size;
    c->e_first = cfg->ep_rank * c->e_local;
    c->groups = c->e_local + 1;
    c->layers.resize(cfg->num_layers);
    c->expert_of_slot.resize(cfg->num_layers);
    c->place_dev.assign(cfg->num_layers, nullptr);
    c->norm_w.assign(cfg->num_layers, nullptr);
    c->norm_eps.assign(cfg->num_layers, 0.f);
    cudaDeviceGetAttribute(&c->n_sms, cudaDevAttrMultiProcessorCount, cfg->device);

    auto bail = [&](hymoe_status st) {
        g_create_error = c->err;
        hymoe_destroy(c);
        return st;
    };
    if (cudaStreamCreateWithFlags(&c->own_stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&c->copy_stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&c->down_stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&c->side_stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&c->ev_fork, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&c->ev_join, cudaEventDisableTiming) != cudaSuccess)
        return bail(c->fail(HYMOE_ERR_CUDA, "cudaStreamCreate failed"));
    c->stream = c->own_stream;

    const size_t T = cfg->max_tokens;
    // Rows of the expert-sorted activation matrix: local pairs + shared rows, plus (for
    // expert parallelism) rows received from other ranks.
    const int N = cfg->ep_size, el = c->e_local;
    // GEMM input rows: T shared rows, then routed rows (all local pairs on one GPU; with
    // expert parallelism at most min(K, E/N) rows per token of each of the N ranks).
    const size_t routed_cap = N == 1 ? T * K : static_cast<size_t>(N) * T * std::min<uint32_t>(K, el);
    const size_t rows = T + routed_cap;
    c->rows_cap = rows;
    const size_t n_chunks = (T + kRouterTok - 1) / kRouterTok;
    const int n_rb = std::max<int>(2 * I / kTileRows, H / kTileRows);
    c->max_items = n_rb * static_cast<int>(rows / kGemvMaxRows + kMaxSegs + 1);
    cudaError_t e = cudaSuccess;
    auto A = [&](cudaError_t r) {
        if (e == cudaSuccess) e = r;
    };
    A(dalloc(&c->x_dev, T * H));
    A(dalloc(&c->resid_dev, T * H));
    A(dalloc(&c->out_dev, T * H));
    A(dalloc(&c->logits, T * E));
    A(dalloc(&c->probs, T * E));
    A(dalloc(&c->topk_w, T * K));
    A(dalloc(&c->topk_idx, T * K));
    A(dalloc(&c->chunk_counts, n_chunks * E));
    A(dalloc(&c->chunk_base, n_chunks * E));
    A(dalloc(&c->goff, E + 2));
    A(dalloc(&c->gcnt, E));
    A(dalloc(&c->segs, kMaxSegs));
    A(dalloc(&c->n_segs, 1));
    A(dalloc(&c->seg_ret, kMaxSegs));
    A(dalloc(&c->bias_dev, E));
    A(dalloc(&c->slot_pos, T * K));
    A(dalloc(&c->n_items, 2));
    A(dalloc(&c->err_word, 1));
    A(dalloc(&c->items_gu, c->max_items));
    A(dalloc(&c->items_dn, c->max_items));
    if (N > 1) {
        A(dalloc(&c->aux_gu, c->max_items));
        A(dalloc(&c->aux_dn, c->max_items));
    }
    A(dalloc(&c->items_sh_gu, n_rb));
    A(dalloc(&c->items_sh_dn, n_rb));
    A(dalloc(&c->n_items_sh, 2));
    A(dalloc(&c->xp, rows * H));
    A(dalloc(&c->hbuf, rows * I));
    A(dalloc(&c->y, T * H));
    A(dalloc(&c->yr, rows * H));
    if (N > 1) {
        A(dalloc(&c->xp_send, T * K * H));
        A(dalloc(&c->y_ret, T * K * H));
        A(dalloc(&c->C_dev, static_cast<size_t>(N) * E));
        A(dalloc(&c->choice_dev, static_cast<size_t>(N) * ep_choice_rec(E)));
        A(cudaMallocHost(reinterpret_cast<void**>(&c->C_host), sizeof(int) * N * E));
        A(cudaEventCreateWithFlags(&c->ev_counts, cudaEventDisableTiming));
    }
    c->tmp_bytes = static_cast<size_t>(2 * I) * H * 4;  // largest GGUF tensor (F32 gate_up)
    A(dalloc(&c->tmp, c->tmp_bytes));
    if (e != cudaSuccess) return bail(c->cuda_fail(e, "scratch allocation"));
    if (cudaMemset(c->err_word, 0, sizeof(int)) != cudaSuccess)
        return bail(c->fail(HYMOE_ERR_CUDA, "cudaMemset failed"));
    hymoe_status st = make_maps(c, &c->maps_xp, &c->gmaps_xp, c->xp, H, rows);
    if (st == HYMOE_OK) st = make_maps(c, &c->maps_h, &c->gmaps_h, c->hbuf, I, rows);
    if (st != HYMOE_OK) return bail(st);
    {
        // The one-kernel decode path: one GPU, a device that launches cooperative grids, and
        // switched on by HYMOE_DECODE_FUSED=1 (default: off, the multi-kernel path serves every
        // size; it is faster on the measured B200s until the one-kernel path's front end is
        // hidden).
        int coop = 0;
        cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, cfg->device);
        const char* pd = getenv("HYMOE_PDL");
        c->pdl = !(pd && strcmp(pd, "0") == 0);
        const char* df = getenv("HYMOE_DECODE_FUSED");
        const bool fused_on = df && strcmp(df, "1") == 0;
        if (N == 1 && coop && fused_on && E <= kDecodeMaxE && H / kTileRows <= kDecodeMaxRb) {
            const size_t hrows = static_cast<size_t>(el + 1) * 8;
            A(dalloc(&c->dec_h, hrows * I));
            A(dalloc(&c->dec_yr, static_cast<size_t>(el) * 8 * H));
            A(dalloc(&c->dec_ysh, static_cast<size_t>(8) * H));
            A(dalloc(&c->dec_sync, 1));
            if (e == cudaSuccess) A(cudaMemset(c->dec_sync, 0, sizeof(DecodeSync)));
            if (e == cudaSuccess) A(cudaMemset(c->dec_h, 0, sizeof(__half) * hrows * I));
            if (e == cudaSuccess) A(cudaMemset(c->xp, 0, sizeof(__half) * 8 * H));
            if (e != cudaSuccess) return bail(c->cuda_fail(e, "decode scratch allocation"));
            c->dec_maps.x = c->gmaps_xp.x[0];  // rows 0..7 of xp, box {64, 8}
            st = make_tmap(c, &c->dec_maps.h, c->dec_h, I, hrows, 8);
            if (st != HYMOE_OK) return bail(st);
            c->dec_ok = true;
        }
    }
    if (N > 1) {
        if (!cfg->nccl_unique_id) return bail(c->fail(HYMOE_ERR_INVALID_ARG, "ep_size > 1 needs nccl_unique_id"));
        if (const char* v = getenv("HYMOE_EP_TIMEOUT_S")) c->ep_timeout_s = atof(v);
        c->joining = true;
        // Non-blocking communicator: joining is polled against a deadline so that a rank
        // that never arrives ends this call with an error instead of a hang.
        ncclConfig_t ncfg = NCCL_CONFIG_INITIALIZER;
        ncfg.blocking = 0;
        ncclUniqueId id;
        memcpy(&id, cfg->nccl_unique_id, sizeof(id));
        ncclResult_t r = ncclCommInitRankConfig(&c->comm, N, id, cfg->ep_rank, &ncfg);
        if (r != ncclSuccess && r != ncclInProgress)
            return bail(c->fail(HYMOE_ERR_NCCL, "ncclCommInitRankConfig: %s", ncclGetErrorString(r)));
        st = ep_poll(c, "joining the expert-parallel communicator");
        if (st != HYMOE_OK) return bail(st);
        const char* tr = getenv("HYMOE_EP_TRANSPORT");
        if (N <= kEpMaxRanks && !(tr && strcmp(tr, "nccl") == 0)) {
            st = ep_p2p_setup(c);
            if (st != HYMOE_OK) return bail(st);
        }
        c->joining = false;
    }
    *out = c;
    return HYMOE_OK;
}

void hymoe_destroy(hymoe_ctx* c) {
    if (!c) return;
    cudaSetDevice(c->cfg.device);
    if (c->loader.joinable()) {  // queued loads finish first
        {
            std::lock_guard<std::mutex> lk(c->lmu);
            c->lstop = true;
        }
        c->lcv.notify_all();
        c->loader.join();
    }
    if (c->p2p && c->comm && !c->comm_broken) {
        // Peers may still read this rank's y (their combine) or write its xp: a bounded barrier
        // over the communicator orders the frees after every rank's last call.
        const ncclResult_t r = ncclAllReduce(c->gcnt, c->gcnt, 1, ncclInt32, ncclSum, c->comm, c->stream);
        if ((r == ncclSuccess || r == ncclInProgress) && ep_poll(c, "destroy barrier") == HYMOE_OK) {
            cudaEvent_t ev = c->take_event();
            cudaEventRecord(ev, c->stream);
            if (ep_wait_event(c, ev, "destroy barrier") != HYMOE_OK) c->comm_broken = true;
            c->ev_pool.push_back(ev);
        } else {
            c->comm_broken = true;
        }
    }
    if (c->own_stream) cudaStreamSynchronize(c->own_stream);
    if (c->copy_stream) cudaStreamSynchronize(c->copy_stream);
    if (c->down_stream) cudaStreamSynchronize(c->down_stream);
    if (c->side_stream) cudaStreamSynchronize(c->side_stream);
    for (auto& L : c->layers) free_layer(L);
    for (int* p : c->place_dev) cudaFree(p);
    for (float* p : c->norm_w) cudaFree(p);
    cudaFree(c->rms_buf);
    cudaFree(c->x_dev);
    cudaFree(c->resid_dev);
    cudaFree(c->out_dev);
    cudaFree(c->logits);
    cudaFree(c->probs);
    cudaFree(c->topk_w);
    cudaFree(c->topk_idx);
    cudaFree(c->chunk_counts);
    cudaFree(c->chunk_base);
    cudaFree(c->goff);
    cudaFree(c->bias_dev);
    cudaFree(c->slot_pos);
    cudaFree(c->n_items);
    cudaFree(c->err_word);
    cudaFree(c->items_gu);
    cudaFree(c->items_dn);
    cudaFree(c->xp);
    cudaFree(c->hbuf);
    cudaFree(c->dec_h);
    cudaFree(c->dec_yr);
    cudaFree(c->dec_ysh);
    cudaFree(c->dec_sync);
    cudaFree(c->y);
    cudaFree(c->yr);
    cudaFree(c->tmp);
    if (c->comm) {
        if (c->comm_broken) ncclCommAbort(c->comm);
        else ncclCommDestroy(c->comm);
    }
    for (void* p : c->ipc_opened) cudaIpcCloseMemHandle(p);
    cudaFree(c->ep_meta);
    cudaFree(c->done_ctas);
    cudaFree(c->xp_send);
    cudaFree(c->y_ret);
    cudaFree(c->C_dev);
    cudaFree(c->choice_dev);
    if (c->C_host) cudaFreeHost(c->C_host);
    if (c->ev_counts) cudaEventDestroy(c->ev_counts);
    cudaFree(c->gcnt);
    cudaFree(c->segs);
    cudaFree(c->n_segs);
    cudaFree(c->seg_ret);
    cudaFree(c->aux_gu);
    cudaFree(c->aux_dn);
    cudaFree(c->dbg_w);
    cudaFree(c->dbg_idx);
    c->clear_graphs();
    c->prof_clear();
    for (cudaEvent_t e : c->ev_pool) cudaEventDestroy(e);
    if (c->own_stream) cudaStreamDestroy(c->own_stream);
    if (c->copy_stream) cudaStreamDestroy(c->copy_stream);
    if (c->down_stream) cudaStreamDestroy(c->down_stream);
    if (c->side_stream) cudaStreamDestroy(c->side_stream);
    if (c->load_stream) cudaStreamDestroy(c->load_stream);
    cudaFree(c->load_tmp);
    cudaFree(c->ready);
    if (c->ev_fork) cudaEventDestroy(c->ev_fork);
    if (c->ev_join) cudaEventDestroy(c->ev_join);
    cudaFree(c->items_sh_gu);
    cudaFree(c->items_sh_dn);
    cudaFree(c->n_items_sh);
    delete c;
}

hymoe_status hymoe_set_stream(hymoe_ctx* c, void* stream) {
    if (!c) return HYMOE_ERR_INVALID_ARG;
    c->stream = stream ? static_cast<cudaStream_t>(stream) : c->own_stream;
    return HYMOE_OK;
}

hymoe_status hymoe_synchronize(hymoe_ctx* c) {
    if (!c) return HYMOE_ERR_INVALID_ARG;
    HY_CUDA(c, cudaSetDevice(c->cfg.device));
    if (c->cfg.ep_size > 1 && c->comm) {
        // Bounded: a peer that stopped taking part ends the wait with an error.
        cudaEvent_t ev = c->take_event();
        HY_CUDA(c, cudaEventRecord(ev, c->stream));
        hymoe_status s2 = ep_wait_event(c, ev, "synchronize");
        c->ev_pool.push_back(ev);
        if (s2 != HYMOE_OK) return s2;
    }
    HY_CUDA(c, cudaStreamSynchronize(c->stream));
    int word = 0;
    HY_CUDA(c, cudaMemcpy(&word, c->err_word, sizeof(int), cudaMemcpyDeviceToHost));
    if (word != 0) {
        cudaMemset(c->err_word, 0, sizeof(int));
        if (word & DEVERR_TIMEOUT_PEER) c->comm_broken = true;
        if (word & DEVERR_SPEC_MISMATCH)
            return c->fail(HYMOE_ERR_CUDA, "decode kernel: certified routing disagreed with the router (code 0x%x)", word);
        return c->fail(HYMOE_ERR_TIMEOUT, "device-side bounded wait expired (code 0x%x)", word);
    }
    return HYMOE_OK;
}

hymoe_status hymoe_load_layer(hymoe_ctx* c, uint32_t layer, const hymoe_tensor* router,
                              const hymoe_tensor* shared_gate_up, const hymoe_tensor* shared_down,
                              const hymoe_tensor* experts_gate_up,
                              const hymoe_tensor* experts_down, int flags) {
    if (!c) return HYMOE_ERR_INVALID_ARG;
    if (layer >= c->layers.size()) return c->fail(HYMOE_ERR_INVALID_ARG, "layer %u out of range", layer);
    HY_CUDA(c, cudaSetDevice(c->cfg.device));
    const int H = c->H, I = c->I;
    int wt = 0;
    hymoe_status st = check_layer_tensors(c, layer, router, shared_gate_up, shared_down, experts_gate_up,
                                          experts_down, &wt);
    if (st != HYMOE_OK) return st;
    wait_loads(c, layer);  // an asynchronous load of this slot finishes first
    c->clear_graphs();
    st = ensure_layer(c, layer, wt);
    if (st != HYMOE_OK) return st;
    LayerStore& L = c->layers[layer];
    L.loaded = false;
    const bool host = (flags & HYMOE_HOST_PTRS) != 0;
    HY_CUDA(c, cudaMemcpyAsync(L.router, router->data, router->nbytes,
                               host ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice, c->stream));
    for (int g = 0; g < c->groups; ++g) {
        const bool shared = g == c->e_local;
        const int ge = shared ? 0 : c->expert_at(layer, c->e_first + g);
        const hymoe_tensor* tg = shared ? shared_gate_up : &experts_gate_up[ge];
        const hymoe_tensor* td = shared ? shared_down : &experts_down[ge];
        st = load_matrix(c, tg, L.gu + c->gu_group_bytes * g, wt, 2 * I, H, I, host);
        if (st == HYMOE_OK) st = load_matrix(c, td, L.dn + c->dn_group_bytes * g, wt, H, I, 0, host);
        if (st != HYMOE_OK) return st;
    }
    HY_CUDA(c, cudaStreamSynchronize(c->stream));
    L.loaded = true;
    return HYMOE_OK;
}

hymoe_status hymoe_synth_layer(hymoe_ctx* c, uint32_t layer, int32_t ggml_type, uint64_t seed,
                               float stddev) {
    if (!c) return HYMOE_ERR_INVALID_ARG;
    if (layer >= c->layers.size()) return c->fail(HYMOE_ERR_INVALID_ARG, "layer %u out of range", layer);
    if (ggml_type != HYMOE_TYPE_F32 && ggml_type != HYMOE_TYPE_F16 && ggml_type != HYMOE_TYPE_Q4_0 &&
        ggml_type != HYMOE_TYPE_Q8_0)
        return c->fail(HYMOE_ERR_INVALID_ARG, "unsupported GGUF type %d", ggml_type);
    HY_CUDA(c, cudaSetDevice(c->cfg.device));
    const int H = c->H, I = c->I, E = c->E;
    const int wt = tile_type_for(ggml_type);
    wait_loads(c, layer);  // an asynchronous load of this slot finishes first
    c->clear_graphs();
    hymoe_status st = ensure_layer(c, layer, wt);
    if (st != HYMOE_OK) return st;
    LayerStore& L = c->layers[layer];
    L.loaded = false;
    // c = float(stddev * sqrt(1.5) / 65536), computed in double as the CPU generator does.
    const float scale = static_cast<float>(static_cast<double>(stddev) * 1.2247448713915890491 / 65536.0);
    auto sid = [&](int kind, int index) {
        return (static_cast<uint64_t>(layer) << 32) | (static_cast<uint64_t>(kind) << 16) |
               static_cast<uint64_t>(index);
    };
    HY_CUDA(c, launch_synth_f32(L.router, static_cast<uint64_t>(E) * H, seed, sid(1, 0), scale, c->stream));
    for (int g = 0; g < c->groups; ++g) {
        const bool shared = g == c->e_local;
        const int idx = shared ? 0xFFFF : c->expert_at(layer, c->e_first + g);
        HY_CUDA(c, launch_synth_gguf(c->tmp, ggml_type, static_cast<uint64_t>(2 * I) * H, seed,
                                     sid(2, idx), scale, c->stream));
        HY_CUDA(c, launch_repack(c->tmp, ggml_type, L.gu + c->gu_group_bytes * g, wt, 2 * I, H, I,
                                 c->stream));
        HY_CUDA(c, launch_synth_gguf(c->tmp, ggml_type, static_cast<uint64_t>(H) * I, seed,
                                     sid(3, idx), scale, c->stream));
        HY_CUDA(c, launch_repack(c->tmp, ggml_type, L.dn + c->dn_group_bytes * g, wt, H, I, 0,
                                 c->stream));
    }
    HY_CUDA(c, cudaStreamSynchronize(c->stream));
    L.loaded = true;
    return HYMOE_OK;
}

// GGUF block decode of a router stored quantised (the reference's converter labels every
// tensor of a layer with one type, scripts/convert_to_gguf.py:196-200): standard blocks,
// F16 exact, Q8_0 q*d, Q4_0 (q-8)*d with element j in the low nibble of byte j and j+16 in
// the high nibble; products in f32.
static float half_to_float(uint16_t h) {
    const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu, mant = h & 0x3FFu, bits;
    if (exp == 0x1F) {
        bits = sign | 0x7F800000u | (mant << 13);
    } else if (exp != 0) {
        bits = sign | ((exp + 112u) << 23) | (mant << 13);
    } else if (mant == 0) {
        bits = sign;
    } else {  // subnormal: normalise
        int e = -1;
        do {
            mant <<= 1;
            ++e;
        } while (!(mant & 0x400u));
        bits = sign | ((112u - static_cast<uint32_t>(e)) << 23) | ((mant & 0x3FFu) << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

static bool dequant_router(const hymoe_tensor* t, std::vector<float>* out) {
    const size_t n = static_cast<size_t>(t->ne[0]) * static_cast<size_t>(t->ne[1]);
    out->resize(n);
    const uint8_t* p = static_cast<const uint8_t*>(t->data);
    switch (t->ggml_type) {
        case HYMOE_TYPE_F16:
            for (size_t i = 0; i < n; ++i) {
                uint16_t h;
                std::memcpy(&h, p + 2 * i, 2);
                (*out)[i] = half_to_float(h);
            }
            return true;
        case HYMOE_TYPE_Q8_0:
        case HYMOE_TYPE_Q4_0: {
            const bool q8 = t->ggml_type == HYMOE_TYPE_Q8_0;
            const size_t bs = q8 ? 34 : 18;
            for (size_t b = 0; b < n / 32; ++b) {
                const uint8_t* blk = p + b * bs;
                uint16_t h;
                std::memcpy(&h, blk, 2);
                const float d = half_to_float(h);
                for (int j = 0; j < 32; ++j) {
                    const int q = q8 ? static_cast<int>(static_cast<int8_t>(blk[2 + j]))
                                     : static_cast<int>(j < 16 ? (blk[2 + j] & 0xF) : (blk[2 + j - 16] >> 4)) - 8;
                    (*out)[b * 32 + j] = static_cast<float>(q) * d;
                }
            }
            return true;
        }
        default:
            return false;
    }
}

hymoe_status hymoe_load_layer_gguf(hymoe_ctx* c, uint32_t layer, const hymoe_gguf* file, uint32_t layer_idx) {
    if (!c || !file) return HYMOE_ERR_INVALID_ARG;
    const int E = c->E;
    std::vector<hymoe_tensor> egu(E), edn(E);
    hymoe_tensor router{}, sgu{}, sdn{};
    const hymoe_status st = hymoe_gguf_moe_tensors(file, layer_idx, E, &router, &sgu, &sdn, egu.data(), edn.data());
    if (st != HYMOE_OK) return c->fail(st, "GGUF layer %u: %s", layer_idx, hymoe_gguf_last_error());
    std::vector<float> rf;
    if (router.ggml_type != HYMOE_TYPE_F32) {
        if (router.ne[0] != c->H || router.ne[1] != E || router.nbytes != gguf_nbytes(router.ggml_type, static_cast<int64_t>(E) * c->H) ||
            !dequant_router(&router, &rf))
            return c->fail(HYMOE_ERR_INVALID_ARG, "GGUF layer %u: router [%lld, %lld] of type %d", layer_idx,
                           static_cast<long long>(router.ne[1]), static_cast<long long>(router.ne[0]), router.ggml_type);
        router.data = rf.data();
        router.ggml_type = HYMOE_TYPE_F32;
        router.nbytes = rf.size() * sizeof(float);
    }
    return hymoe_load_layer(c, layer, &router, &sgu, &sdn, egu.data(), edn.data(), HYMOE_HOST_PTRS);
}

// Queues an asynchronous load (the tensors are validated already; router_f32 holds a router
// decoded on the host, kept alive by the job).
static hymoe_status queue_load(hymoe_ctx* c, uint32_t layer, const hymoe_tensor* router,
                               const hymoe_tensor* shared_gate_up, const hymoe_tensor* shared_down,
                               const hymoe_tensor* experts_gate_up, const hymoe_tensor* experts_down, int wt,
                               std::vector<float>&& router_f32) {
    hymoe_status st = ensure_loader(c);
    if (st != HYMOE_OK) return st;
    c->clear_graphs();
    LayerStore& L0 = c->layers[layer];
    if (L0.gu && L0.wtype != wt) {  // the slot is reallocated for another type: nothing may use it
        wait_loads(c, layer);
        HY_CUDA(c, cudaStreamSynchronize(c->stream));
    }
    st = ensure_layer(c, layer, wt);
    if (st != HYMOE_OK) return st;
    LayerStore& L = c->layers[layer];
    hymoe_ctx::LoadJob j;
    j.layer = layer;
    j.wt = wt;
    j.d_router = L.router;
    j.d_gu = L.gu;
    j.d_dn = L.dn;
    j.gu_bytes = c->gu_group_bytes;
    j.dn_bytes = c->dn_group_bytes;
    j.router = *router;
    j.router_f32 = std::move(router_f32);
    if (!j.router_f32.empty()) j.router.data = j.router_f32.data();
    for (int g = 0; g < c->groups; ++g) {
        const bool shared = g == c->e_local;
        const int ge = shared ? 0 : c->expert_at(layer, c->e_first + g);
        j.gu.push_back(shared ? *shared_gate_up : experts_gate_up[ge]);
        j.dn.push_back(shared ? *shared_down : experts_down[ge]);
    }
    // the slot is rewritten only after every call queued so far on the context's stream
    HY_CUDA(c, cudaEventCreateWithFlags(&j.prior, cudaEventDisableTiming));
    const cudaError_t e = cudaEventRecord(j.prior, c->stream);
    if (e != cudaSuccess) {
        cudaEventDestroy(j.prior);
        return c->cuda_fail(e, "cudaEventRecord");
    }
    {
        std::lock_guard<std::mutex> lk(c->lmu);
        j.epoch = ++c->issued[layer];
        c->jobs.push_back(std::move(j));
    }
    c->lcv.notify_one();
    L.loaded = true;
    return HYMOE_OK;
}

hymoe_status hymoe_load_layer_async(hymoe_ctx* c, uint32_t layer, const hymoe_tensor* router,
                                    const hymoe_tensor* shared_gate_up, const hymoe_tensor* shared_down,
                                    const hymoe_tensor* experts_gate_up, const hymoe_tensor* experts_down) {
    if (!c) return HYMOE_ERR_INVALID_ARG;
    if (layer >= c->layers.size()) return c->fail(HYMOE_ERR_INVALID_ARG, "layer %u out of range", layer);
    HY_CUDA(c, cudaSetDevice(c->cfg.device));
    int wt = 0;
    const hymoe_status st = check_layer_tensors(c, layer, router, shared_gate_up, shared_down, experts_gate_up,
                                                experts_down, &wt);
    if (st != HYMOE_OK) return st;
    return queue_load(c, layer, router, shared_gate_up, shared_down, experts_gate_up, experts_down, wt, {});
}

hymoe_status hymoe_load_layer_gguf_async(hymoe_ctx* c, uint32_t layer, const hymoe_gguf* file, uint32_t layer_idx) {
    if (!c || !file) return HYMOE_ERR_INVALID_ARG;
    if (layer >= c->layers.size()) return c->fail(HYMOE_ERR_INVALID_ARG, "layer %u out of range", layer);
    HY_CUDA(c, cudaSetDevice(c->cfg.device));
    const int E = c->E;
    std::vector<hymoe_tensor> egu(E), edn(E);
    hymoe_tensor router{}, sgu{}, sdn{};
    hymoe_status st = hymoe_gguf_moe_tensors(file, layer_idx, E, &router, &sgu, &sdn, egu.data(), edn.data());
    if (st != HYMOE_OK) return c->fail(st, "GGUF layer %u: %s", layer_idx, hymoe_gguf_last_error());
    std::vector<float> rf;
    if (router.ggml_type != HYMOE_TYPE_F32) {
        if (router.ne[0] != c->H || router.ne[1] != E ||
            router.nbytes != gguf_nbytes(router.ggml_type, static_cast<int64_t>(E) * c->H) || !dequant_router(&router, &rf))
            return c->fail(HYMOE_ERR_INVALID_ARG, "GGUF layer %u: router [%lld, %lld] of type %d", layer_idx,
                           static_cast<long long>(router.ne[1]), static_cast<long long>(router.ne[0]), router.ggml_type);
        router.data = rf.data();
        router.ggml_type = HYMOE_TYPE_F32;
        router.nbytes = rf.size() * sizeof(float);
    }
    int wt = 0;
    st = check_layer_tensors(c, layer, &router, &sgu, &sdn, egu.data(), edn.data(), &wt);
    if (st != HYMOE_OK) return st;
    return queue_load(c, layer, &router, &sgu, &sdn, egu.data(), edn.data(), wt, std::move(rf));
}

hymoe_status hymoe_wait_layer(hymoe_ctx* c, uint32_t layer) {
    if (!c) return HYMOE_ERR_INVALID_ARG;
    if (layer >= c->layers.size()) return c->fail(HYMOE_ERR_INVALID_ARG, "layer %u out of range", layer);
    const hymoe_status st = wait_loads(c, layer);
    if (st != HYMOE_OK) {
        std::lock_guard<std::mutex> lk(c->lmu);
        return c->fail(st, "%s", c->lerr.c_str());
    }
    return HYMOE_OK;
}

hymoe_status hymoe_set_norm(hymoe_ctx* c, uint32_t layer, const float* weight, float eps, int flags) {
    if (!c) return HYMOE_ERR_INVALID_ARG;
    if (layer >= c->layers.size()) return c->fail(HYMOE_ERR_INVALID_ARG, "layer %u out of range", layer);
    if (!(eps >= 0.f) || eps == INFINITY) return c->fail(HYMOE_ERR_INVALID_ARG, "eps %g", static_cast<double>(eps));
    HY_CUDA(c, cudaSetDevice(c->cfg.device));
    HY_CUDA(c, cudaStreamSynchronize(c->stream));  // no call still reads the old weights
    c->clear_graphs();                             // eps is baked into captured launches
    if (!weight) {
        cudaFree(c->norm_w[layer]);
        c->norm_w[layer] = nullptr;
        return HYMOE_OK;
    }
    if (!c->rms_buf) HY_CUDA(c, dalloc(&c->rms_buf, static_cast<size_t>(c->cfg.max_tokens)));
    if (!c->norm_w[layer]) HY_CUDA(c, dalloc(&c->norm_w[layer], static_cast<size_t>(c->H)));
    const bool host = (flags & HYMOE_HOST_PTRS) != 0;
    HY_CUDA(c, cudaMemcpy(c->norm_w[layer], weight, sizeof(float) * c->H,
                          host ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice));
    c->norm_eps[layer] = eps;
    return HYMOE_OK;
}

hymoe_status hymoe_set_routing(hymoe_ctx* c, const hymoe_routing* r) {
    if (!c) return HYMOE_ERR_INVALID_ARG;
    RouteMode m;  // NULL: moe_forward_cpu's routing
    if (r) {
        if (r->drop_tokens) {
            if (c->K > kEpMaxK)
                return c->fail(HYMOE_ERR_UNSUPPORTED, "capacity drops need moe_topk <= %d", kEpMaxK);
            if (!(r->capacity_factor >= 0.f) || !std::isfinite(r->capacity_factor))
                return c->fail(HYMOE_ERR_INVALID_ARG, "capacity_factor %g", static_cast<double>(r->capacity_factor));
            m.drop = 1;
            m.capacity_factor = r->capacity_factor;
            m.min_capacity = static_cast<int>(std::min<uint32_t>(r->min_capacity, 1u << 30));
        }
        if (r->group_limited_greedy) {
            if (r->n_group == 0 || r->n_group > 32 || c->E % static_cast<int>(r->n_group) != 0 ||
                r->topk_group == 0 || r->topk_group > r->n_group)
                return c->fail(HYMOE_ERR_INVALID_ARG, "group-limited routing: n_group %u (1..32, dividing E=%d), "
                               "topk_group %u (1..n_group)", r->n_group, c->E, r->topk_group);
            m.n_group = static_cast<int>(r->n_group);
            m.topk_group = static_cast<int>(r->topk_group);
        }
        if (!std::isfinite(r->routed_scaling_factor))
            return c->fail(HYMOE_ERR_INVALID_ARG, "routed_scaling_factor is not finite");
        // topkgating_full renormalises only when K > 1 (src/hunyuan_moe_full.cpp:229-243)
        m.norm = r->norm_topk_prob && c->K > 1 ? 1 : 0;
        m.clamp = 1;
        m.scale = r->routed_scaling_factor;
    }
    HY_CUDA(c, cudaSetDevice(c->cfg.device));
    HY_CUDA(c, cudaStreamSynchronize(c->stream));
    c->clear_graphs();  // the mode is baked into captured launches
    c->route = m;
    return HYMOE_OK;
}

hymoe_status hymoe_set_placement(hymoe_ctx* c, uint32_t layer, const int32_t* slot_of_expert) {
    if (!c) return HYMOE_ERR_INVALID_ARG;
    if (layer >= c->layers.size()) return c->fail(HYMOE_ERR_INVALID_ARG, "layer %u out of range", layer);
    const int E = c->E;
    std::vector<int> expert_of(E, -1);
    bool identity = true;
    if (slot_of_expert) {
        for (int e = 0; e < E; ++e) {
            const int s = slot_of_expert[e];
            if (s < 0 || s >= E || expert_of[s] >= 0)
                return c->fail(HYMOE_ERR_INVALID_ARG, "placement is not a permutation of 0..%d (expert %d -> %d)",
                                E - 1, e, s);
            expert_of[s] = e;
            identity = identity && s == e;
        }
    }
    HY_CUDA(c, cudaSetDevice(c->cfg.device));
    wait_loads(c, layer);
    HY_CUDA(c, cudaStreamSynchronize(c->stream));  // no call of this layer still reads the old map
    c->clear_graphs();
    c->layers[layer].loaded = false;  // the experts of this rank's slots change: load again
    if (identity) {
        cudaFree(c->place_dev[layer]);
        c->place_dev[layer] = nullptr;
        c->expert_of_slot[layer].clear();
        return HYMOE_OK;
    }
    if (!c->place_dev[layer]) HY_CUDA(c, dalloc(&c->place_dev[layer], 2 * static_cast<size_t>(E)));
    std::vector<int> both(slot_of_expert, slot_of_expert + E);
    both.insert(both.end(), expert_of.begin(), expert_of.end());
    HY_CUDA(c, cudaMemcpy(c->place_dev[layer], both.data(), sizeof(int) * 2 * E, cudaMemcpyHostToDevice));
    c->expert_of_slot[layer] = expert_of;
    return HYMOE_OK;
}

// Greedy longest-processing-time placement with exactly E/ep_size experts per rank: experts in
// decreasing load (ties: lower expert first) each go to the least-loaded rank that still has a
// free slot (ties: lower rank), taking that rank's next slot.
hymoe_status hymoe_balance_placement(uint32_t n_experts, uint32_t ep_size, const double* load,
                                     int32_t* slot_of_expert) {
    if (!load || !slot_of_expert || n_experts == 0 || ep_size == 0 || n_experts % ep_size != 0)
        return HYMOE_ERR_INVALID_ARG;
    const int E = static_cast<int>(n_experts), N = static_cast<int>(ep_size), el = E / N;
    std::vector<int> order(E);
    for (int e = 0; e < E; ++e) {
        if (!(load[e] >= 0.0)) return HYMOE_ERR_INVALID_ARG;  // negative or NaN
        order[e] = e;
    }
    std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return load[a] > load[b]; });
    std::vector<double> sum(N, 0.0);
    std::vector<int> used(N, 0);
    for (int e : order) {
        int best = -1;
        for (int r = 0; r < N; ++r)
            if (used[r] < el && (best < 0 || sum[r] < sum[best])) best = r;
        slot_of_expert[e] = best * el + used[best]++;
        sum[best] += load[e];
    }
    return HYMOE_OK;
}

hymoe_status hymoe_forward(hymoe_ctx* c, uint32_t layer, const float* x, const float* residual,
                           float* out, uint32_t n_tokens, const float* router_bias,
                           hymoe_debug* dbg, int flags) {
    if (!c) return HYMOE_ERR_INVALID_ARG;
    if (layer >= c->layers.size() || !c->layers[layer].loaded)
        return c->fail(HYMOE_ERR_STATE, "layer %u not loaded", layer);
    if (n_tokens > c->cfg.max_tokens)
        return c->fail(HYMOE_ERR_INVALID_ARG, "n_tokens %u exceeds max_tokens %u", n_tokens,
                       c->cfg.max_tokens);
    if ((!x || !out) && n_tokens > 0) return c->fail(HYMOE_ERR_INVALID_ARG, "null x/out");
    const bool pre_norm = (flags & HYMOE_PRE_NORM) != 0;
    if (pre_norm && !c->norm_w[layer])
        return c->fail(HYMOE_ERR_STATE, "layer %u has no RMSNorm weights (hymoe_set_norm)", layer);
    const bool ep = c->cfg.ep_size > 1;
    if (ep && (c->comm_broken || !c->comm))
        return c->fail(HYMOE_ERR_STATE, "expert-parallel communicator is unusable after an earlier failure");
    HY_CUDA(c, cudaSetDevice(c->cfg.device));
    if (c->loader.joinable()) {
        // An asynchronous load of this layer still in flight: the call's device work waits for it
        // (a wait in the stream's front end, no host wait); a finished load that failed fails the
        // call.  Captured graphs are not given such a wait, and neither are host-pointer calls:
        // their copies from pageable memory synchronise the stream on the host first, which
        // must not depend on the loader thread making progress (its own pageable copies): the
        // host waits for the load instead.
        uint32_t want = 0;
        bool finished = true;
        hymoe_status lst = HYMOE_OK;
        {
            std::lock_guard<std::mutex> lk(c->lmu);
            want = c->issued[layer];
            finished = c->done[layer] >= want;
            if (finished) lst = c->lstatus[layer];
        }
        if (!finished && (flags & (HYMOE_USE_GRAPH | HYMOE_HOST_PTRS))) {
            lst = wait_loads(c, layer);
            finished = true;
        }
        if (lst != HYMOE_OK) {
            std::lock_guard<std::mutex> lk(c->lmu);
            return c->fail(lst, "%s", c->lerr.c_str());
        }
        if (!finished) {
            const CUresult r = stream_mem_ops().wait(reinterpret_cast<CUstream>(c->stream),
                                                     reinterpret_cast<CUdeviceptr>(c->ready + layer), want,
                                                     CU_STREAM_WAIT_VALUE_GEQ);
            if (r != CUDA_SUCCESS) return c->fail(HYMOE_ERR_CUDA, "cuStreamWaitValue32 failed (%d)", static_cast<int>(r));
        }
    }
    const LayerStore& L = c->layers[layer];
    const int* slot_of = c->place_dev[layer];  // nullptr: identity placement
    const int T = static_cast<int>(n_tokens), H = c->H, I = c->I, E = c->E, K = c->K;
    const int N = c->cfg.ep_size, rank = c->cfg.ep_rank, el = c->e_local;
    const bool host = (flags & HYMOE_HOST_PTRS) != 0;
    cudaStream_t st = c->stream;
    const size_t xbytes = static_cast<size_t>(T) * H * sizeof(float);

    // Host-pointer calls in token chunks, so that the copies overlap the compute: every upload
    // is queued at once on one copy stream, each chunk computes when its upload has landed, and
    // its download (second copy stream) starts when it is done.  Every token's result is
    // independent of the others', so the output is the same as one call's.
    //   One GPU: calls of >= 2048 tokens without debug outputs, ~2048-token chunks (smaller ones
    //   lose more GEMM efficiency than the overlap gains).
    //   Expert parallel: every rank must run the same number of exchanges, so the chunk count
    //   comes from the job-wide max_tokens (>= 4096: max_tokens / 2048 chunks, at most 4), each
    //   rank splitting its own tokens (a chunk may have none); debug outputs go through device
    //   scratch.
    const int max_tok = static_cast<int>(c->cfg.max_tokens);
    const bool chunk_one = host && !ep && !dbg && T >= kChunkMinTokens && !(flags & HYMOE_USE_GRAPH);
    const bool chunk_ep = host && ep && max_tok >= 2 * kChunkMinTokens && !(flags & HYMOE_USE_GRAPH);
    if (chunk_one || chunk_ep) {
        const int n_ch = chunk_ep ? std::min(4, max_tok / kChunkMinTokens) : std::min(4, T / kChunkMinTokens);
        const int per = (T + n_ch - 1) / n_ch;
        cudaStream_t up = c->copy_stream, down = c->down_stream;
        const float* dbias = nullptr;
        if (router_bias) {
            HY_CUDA(c, cudaMemcpyAsync(c->bias_dev, router_bias, sizeof(float) * E, cudaMemcpyHostToDevice, st));
            dbias = c->bias_dev;
        }
        if (dbg && (dbg->topk_weights || dbg->topk_indices) && !c->dbg_w) {
            HY_CUDA(c, dalloc(&c->dbg_w, static_cast<size_t>(max_tok) * K));
            HY_CUDA(c, dalloc(&c->dbg_idx, static_cast<size_t>(max_tok) * K));
        }
        // both copy streams follow earlier work on the compute stream (they rewrite x_dev / out_dev)
        std::vector<cudaEvent_t> evs;
        auto ev = [&]() {
            evs.push_back(c->take_event());
            return evs.back();
        };
        cudaEvent_t ev0 = ev();
        HY_CUDA(c, cudaEventRecord(ev0, st));
        HY_CUDA(c, cudaStreamWaitEvent(up, ev0, 0));
        HY_CUDA(c, cudaStreamWaitEvent(down, ev0, 0));
        std::vector<cudaEvent_t> in(n_ch, nullptr);
        for (int ch = 0; ch < n_ch; ++ch) {
            const int t0 = std::min(T, ch * per), n = std::min(per, T - t0);
            const size_t off = static_cast<size_t>(t0) * H, bytes = static_cast<size_t>(n) * H * sizeof(float);
            HY_CUDA(c, c->timed_copy(HYMOE_PHASE_COPY_IN, c->x_dev + off, x + off, bytes, cudaMemcpyHostToDevice, up));
            if (residual && residual != x)
                HY_CUDA(c, c->timed_copy(HYMOE_PHASE_COPY_IN, c->resid_dev + off, residual + off, bytes,
                                         cudaMemcpyHostToDevice, up));
            in[ch] = ev();
            HY_CUDA(c, cudaEventRecord(in[ch], up));
        }
        hymoe_status result = HYMOE_OK;
        for (int ch = 0; ch < n_ch && result == HYMOE_OK; ++ch) {
            const int t0 = std::min(T, ch * per), n = std::min(per, T - t0);
            const size_t off = static_cast<size_t>(t0) * H, bytes = static_cast<size_t>(n) * H * sizeof(float);
            HY_CUDA(c, cudaStreamWaitEvent(st, in[ch], 0));
            const float* r = !residual ? nullptr : residual == x ? c->x_dev + off : c->resid_dev + off;
            hymoe_debug d2{};
            if (dbg) {
                d2.router_logits = dbg->router_logits ? c->logits + static_cast<size_t>(t0) * E : nullptr;
                d2.router_probs = dbg->router_probs ? c->probs + static_cast<size_t>(t0) * E : nullptr;
                d2.topk_weights = dbg->topk_weights ? c->dbg_w + static_cast<size_t>(t0) * K : nullptr;
                d2.topk_indices = dbg->topk_indices ? c->dbg_idx + static_cast<size_t>(t0) * K : nullptr;
            }
            result = hymoe_forward(c, layer, c->x_dev + off, r, c->out_dev + off, static_cast<uint32_t>(n), dbias,
                                   dbg ? &d2 : nullptr, flags & ~HYMOE_HOST_PTRS);
            cudaEvent_t done = ev();
            HY_CUDA(c, cudaEventRecord(done, st));
            HY_CUDA(c, cudaStreamWaitEvent(down, done, 0));
            HY_CUDA(c, c->timed_copy(HYMOE_PHASE_COPY_OUT, out + off, c->out_dev + off, bytes, cudaMemcpyDeviceToHost,
                                     down));
        }
        if (dbg && result == HYMOE_OK && T > 0) {
            const size_t te = static_cast<size_t>(T) * E, tk = static_cast<size_t>(T) * K;
            if (dbg->router_logits)
                HY_CUDA(c, cudaMemcpyAsync(dbg->router_logits, c->logits, te * sizeof(float), cudaMemcpyDeviceToHost, down));
            if (dbg->router_probs)
                HY_CUDA(c, cudaMemcpyAsync(dbg->router_probs, c->probs, te * sizeof(float), cudaMemcpyDeviceToHost, down));
            if (dbg->topk_weights)
                HY_CUDA(c, cudaMemcpyAsync(dbg->topk_weights, c->dbg_w, tk * sizeof(float), cudaMemcpyDeviceToHost, down));
            if (dbg->topk_indices)
                HY_CUDA(c, cudaMemcpyAsync(dbg->topk_indices, c->dbg_idx, tk * sizeof(int), cudaMemcpyDeviceToHost, down));
        }
        cudaEvent_t fin = ev();
        HY_CUDA(c, cudaEventRecord(fin, down));
        HY_CUDA(c, cudaStreamWaitEvent(st, fin, 0));  // synchronising the stream covers the copies
        hymoe_status sync = hymoe_synchronize(c);
        for (cudaEvent_t e : evs) c->ev_pool.push_back(e);
        return result != HYMOE_OK ? result : sync;
    }

    const float* dx = x;
    const float* dres = residual;
    float* dout = out;
    const float* dbias = router_bias;
    float* dlog = dbg ? dbg->router_logits : nullptr;
    float* dprob = dbg ? dbg->router_probs : nullptr;
    if (host) {
        if (T > 0) HY_CUDA(c, c->timed_copy(HYMOE_PHASE_COPY_IN, c->x_dev, x, xbytes, cudaMemcpyHostToDevice, st));
        dx = c->x_dev;
        if (residual && residual == x) {
            dres = c->x_dev;  // decoder_layer form out = h + moe(...): one upload
        } else if (residual && T > 0) {
            HY_CUDA(c, c->timed_copy(HYMOE_PHASE_COPY_IN, c->resid_dev, residual, xbytes, cudaMemcpyHostToDevice, st));
            dres = c->resid_dev;
        }
        dout = c->out_dev;
        if (router_bias) {
            HY_CUDA(c, cudaMemcpyAsync(c->bias_dev, router_bias, sizeof(float) * E,
                                       cudaMemcpyHostToDevice, st));
            dbias = c->bias_dev;
        }
        if (dlog) dlog = c->logits;
        if (dprob) dprob = c->probs;
    }
    // A rank with no tokens still takes part in every collective of the exchange.
    if (T == 0 && !ep) return host ? hymoe_synchronize(c) : HYMOE_OK;

    const bool p2p = ep && c->p2p;
    const uint32_t epoch = p2p ? ++c->epoch : 0;
    const uint64_t budget_ns = static_cast<uint64_t>(c->ep_timeout_s * 1e9);
    // Capacity-limited routing over an expert-parallel job: every rank's choice record (pairs per
    // (choice, slot) and its token count), by peer memory or an NCCL all-gather.
    auto choice_recs = [&]() -> const int* {
        return p2p ? c->ep_meta + ep_choice_off(E) : c->choice_dev;
    };
    auto exchange_choices = [&]() -> hymoe_status {
        if (p2p) {
            HY_CUDA(c, launch_ep_choice_counts(c->peers, N, rank, E, K, T, c->topk_idx, epoch, budget_ns, c->err_word, st));
            return HYMOE_OK;
        }
        const int rl = ep_choice_rec(E);
        HY_CUDA(c, launch_choice_record(c->topk_idx, T, K, E, c->choice_dev + static_cast<size_t>(rank) * rl, st));
        ncclResult_t r = ncclAllGather(c->choice_dev + static_cast<size_t>(rank) * rl, c->choice_dev, rl, ncclInt32,
                                       c->comm, st);
        if (r != ncclSuccess && r != ncclInProgress)
            return c->fail(HYMOE_ERR_NCCL, "ncclAllGather(choice counts): %s", ncclGetErrorString(r));
        return ep_poll(c, "choice-count exchange");
    };
    auto device_part = [&]() -> hymoe_status {
        // HYMOE_PRE_NORM: the layer's RMSNorm first; everything below reads the normalised rows
        // (the residual stays the caller's).  Timed with the router phase.
        // HYMOE_PRE_NORM: the layer's RMSNorm.  One kernel computes each token's factor
        // 1 / rms (the reference's chain); every kernel that reads the token rows (router,
        // dispatch, expert-parallel sends) applies (x * rms) * w as it loads them, so the
        // normalised rows are never written out.  The residual stays the caller's x.  Timed with
        // the router phase.
        const float* dxn = dx;
        RowNorm nrm{};
        if (pre_norm && T > 0) {
            c->phase_begin();
            HY_CUDA(c, launch_rms(dx, c->norm_eps[layer], T, H, c->rms_buf, st));
            c->phase_end(HYMOE_PHASE_ROUTER);
            nrm.rms = c->rms_buf;
            nrm.w = c->norm_w[layer];
        }
        // Debug outputs (the multi-kernel and the one-kernel paths alike).
        auto debug_out = [&]() -> hymoe_status {
            if (!dbg || T <= 0) return HYMOE_OK;
            const cudaMemcpyKind kd = host ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice;
            if (dbg->topk_weights)
                HY_CUDA(c, cudaMemcpyAsync(dbg->topk_weights, c->topk_w, sizeof(float) * T * K, kd, st));
            if (dbg->topk_indices) {
                // slots back to expert ids, dropped-pair marks cleared (topk_idx is not read
                // again in this call)
                if (slot_of || c->route.drop)
                    HY_CUDA(c, launch_unmap_slots(c->topk_idx, slot_of ? slot_of + E : nullptr,
                                                  static_cast<int>(T * K), st));
                HY_CUDA(c, cudaMemcpyAsync(dbg->topk_indices, c->topk_idx, sizeof(int) * T * K, kd, st));
            }
            if (host && dlog)
                HY_CUDA(c, cudaMemcpyAsync(dbg->router_logits, dlog, sizeof(float) * T * E, kd, st));
            if (host && dprob)
                HY_CUDA(c, cudaMemcpyAsync(dbg->router_probs, dprob, sizeof(float) * T * E, kd, st));
            return HYMOE_OK;
        };
        // 1..8 tokens on one GPU (Q4_0 / Q8_0, no capacity drops): the whole block is one
        // cooperative kernel (decode.cu), timed as the gate_up phase.
        if (c->dec_ok && !ep && T >= 1 && T <= kDecodeMaxT && !c->route.drop &&
            (L.wtype == W_Q4_0 || L.wtype == W_Q8_0) && K <= 8 && decode_smem(L.wtype, T, H, E) != 0) {
            DecodeArgs da{};
            da.x = dx;
            da.nrm = nrm;
            da.resid = dres;
            da.out = dout;
            da.T = T;
            da.H = H;
            da.I = I;
            da.E = E;
            da.K = K;
            da.el = el;
            da.Wr = L.router;
            da.bias = dbias;
            da.mode = c->route;
            da.slot_of = slot_of;
            da.gu = L.d_gu_ptrs;
            da.dn = L.d_dn_ptrs;
            da.logits = dlog ? dlog : c->logits;
            da.probs = dprob;
            da.topk_w = c->topk_w;
            da.topk_idx = c->topk_idx;
            da.xp = c->xp;
            da.hb = c->dec_h;
            da.ysh = c->dec_ysh;
            da.yr = c->dec_yr;
            da.sync = c->dec_sync;
            da.err = c->err_word;
            c->phase_begin();
            HY_CUDA(c, launch_decode(c->dec_maps, da, L.wtype, c->n_sms, st));
            c->phase_end(HYMOE_PHASE_GATE_UP);
            return debug_out();
        }
        // Decode regime: every group has at most kGemvMaxRows rows (on one GPU a group has
        // at most T rows: the shared expert T, a routed expert at most one row per token).
        bool gemv = T <= kGemvMaxRows;
        size_t gemv_rows = static_cast<size_t>(T);
        const int tiles_gu = 2 * I / kTileRows, tiles_dn = H / kTileRows;
        auto items_args = [&](bool gv) {
            ItemsArgs ia{};
            ia.segs = c->segs;
            ia.n_segs = c->n_segs;
            ia.n_rb_gu = gv ? tiles_gu : (tiles_gu + 1) / 2;  // GEMV: one tile; tensor core: tile pairs
            ia.n_rb_dn = gv ? tiles_dn : (tiles_dn + 1) / 2;
            ia.tile_n = 256;
            ia.gemv = gv ? 1 : 0;
            ia.items_gu = c->items_gu;
            ia.items_dn = c->items_dn;
            ia.n_items = c->n_items;
            if (p2p) {  // segments carry their sources and return rows; tensor-core items too
                ia.seg_ret = c->seg_ret;
                if (!gv) {
                    ia.aux_gu = c->aux_gu;
                    ia.aux_dn = c->aux_dn;
                }
            }
            return ia;
        };
        // Decode sizes on one GPU: the shared expert needs no routing, so it streams its weights
        // on a forked stream while the router, the plan and the dispatch run (on <= 48 CTAs,
        // leaving SMs to them); the combine joins both streams.  From 4 tokens on the router's
        // chains last long enough to hide it (measured: T=8 0.357 -> 0.351 ms; at T=1 the fork
        // outlasted the front end and delayed the routed launch, 0.105 -> 0.119 ms).
        const bool shared_apart = !ep && gemv && T >= 4 && T <= 8 && (L.wtype == W_Q4_0 || L.wtype == W_Q8_0);
        // Decode-size chains on one GPU (1..64 tokens, weight-streaming kernels): router (and
        // top-K), plan, scatter, gate_up, down and combine are launched with programmatic
        // dependent launch, so each is scheduled while its predecessor finishes (every one of
        // these kernels waits for its predecessor's completion before it reads anything).
        const bool pdl = c->pdl && !ep && gemv && T >= 1 && T <= kGemvMaxRows && !c->route.drop &&
                         (L.wtype == W_Q4_0 || L.wtype == W_Q8_0);
        if (shared_apart) {
            cudaStream_t side = c->side_stream;
            HY_CUDA(c, cudaEventRecord(c->ev_fork, st));
            HY_CUDA(c, cudaStreamWaitEvent(side, c->ev_fork, 0));
            HY_CUDA(c, launch_shared_prep(dxn, T, H, c->xp, el, tiles_gu, tiles_dn, c->items_sh_gu, c->items_sh_dn,
                                          c->n_items_sh, side, nrm));
            HY_CUDA(c, launch_gemv(c->gmaps_xp, c->items_sh_gu, c->n_items_sh, tiles_gu, L.d_gu_ptrs, L.wtype,
                                   H / kTileK, 1, T, c->hbuf, I, nullptr, 0, c->err_word, std::min(c->n_sms, tiles_gu), side));
            HY_CUDA(c, launch_gemv(c->gmaps_h, c->items_sh_dn, c->n_items_sh + 1, tiles_dn, L.d_dn_ptrs, L.wtype,
                                   I / kTileK, 0, T, c->y, H, c->yr, T, c->err_word, std::min(c->n_sms, tiles_dn), side));
            HY_CUDA(c, cudaEventRecord(c->ev_join, side));
        }
        if (T > 0) {
            const int n_chunks = (T + kRouterTok - 1) / kRouterTok;
            // T <= 16 (one router chunk): the top-K runs inside the plan launch (not with
            // capacity drops, which need every token's choices before the plan).
            const bool fused = n_chunks == 1 && !c->route.drop;
            c->phase_begin();
            HY_CUDA(c, launch_router(dxn, T, H, L.router, E, K, dbias, dlog ? dlog : c->logits, dprob,
                                     c->topk_w, c->topk_idx, c->chunk_counts, slot_of, c->route, !fused, st,
                                     nrm, pdl));
            c->phase_end(HYMOE_PHASE_ROUTER, fused ? 1 : 2);
            if (c->route.drop) {
                // topkgating_full's capacity with drop_tokens (src/hunyuan_moe_full.cpp:205-224):
                // floor(capacity_factor * K * T / E) in single precision, at least K and
                // min_capacity; pairs beyond it in k-major order are dropped.  Expert parallel:
                // over the job's tokens (rank 0's first), from every rank's choice counts.
                c->phase_begin();
                if (ep) {
                    hymoe_status sx = exchange_choices();
                    if (sx != HYMOE_OK) return sx;
                    HY_CUDA(c, launch_capacity_job(c->topk_idx, c->topk_w, c->chunk_counts, T, K, E, choice_recs(), N,
                                                   rank, c->route.capacity_factor, c->route.min_capacity, st));
                } else {
                    const uint32_t f = static_cast<uint32_t>(c->route.capacity_factor * static_cast<float>(K) *
                                                             static_cast<float>(T) / static_cast<float>(E));
                    const int cap = std::max(std::max<int>(static_cast<int>(std::min<uint32_t>(f, 1u << 30)), K),
                                             c->route.min_capacity);
                    HY_CUDA(c, launch_capacity(c->topk_idx, c->topk_w, c->chunk_counts, T, K, E, cap, st));
                }
                c->phase_end(HYMOE_PHASE_ROUTER);
            }
            PlanArgs pa{};
            pa.chunk_counts = c->chunk_counts;
            pa.n_chunks = n_chunks;
            pa.T = T;
            pa.E = E;
            pa.K = K;
            pa.goff = c->goff;
            pa.gcnt = c->gcnt;
            pa.chunk_base = c->chunk_base;
            pa.segs = ep ? nullptr : c->segs;
            pa.n_segs = c->n_segs;
            pa.shared_apart = shared_apart ? 1 : 0;
            pa.slot_of = slot_of;
            pa.mode = c->route;
            pa.items = items_args(gemv);
            c->phase_begin();
            if (fused)
                HY_CUDA(c, launch_topk_plan(dlog ? dlog : c->logits, T, K, dprob, c->topk_w, c->topk_idx, pa, st, pdl));
            else
                HY_CUDA(c, launch_plan(pa, st, pdl));
            c->phase_end(HYMOE_PHASE_PLAN);
            if (!p2p) {  // peer-memory dispatch writes the rows straight to their owners
                c->phase_begin();
                HY_CUDA(c, launch_scatter_gather(dxn, T, H, E, K, c->topk_idx, c->chunk_base, c->slot_pos,
                                                 ep ? c->xp_send : c->xp + static_cast<size_t>(T) * H,
                                                 shared_apart ? nullptr : c->xp, st, nrm, pdl));
                c->phase_end(HYMOE_PHASE_DISPATCH);
            }
        } else {
            HY_CUDA(c, cudaMemsetAsync(c->gcnt, 0, sizeof(int) * E, st));
            if (c->route.drop && ep) {  // a rank without tokens still takes part in the exchange
                hymoe_status sx = exchange_choices();
                if (sx != HYMOE_OK) return sx;
            }
        }

        std::vector<size_t> send_cnt(N, 0), send_off(N, 0), recv_cnt(N, 0), recv_off(N, 0);
        if (p2p) {
            // Counts to every rank (bounded wait for theirs).  Tensor-core calls: this rank's
            // token rows and the pairs it owns into its own xp now; the pairs other ranks own
            // leave from inside the gate_up GEMM.  Decode-size calls: every row to its owner now,
            // then wait until every rank's rows have landed here.  Either way the receive
            // segments come from the count matrix on the device.
            c->phase_begin();
            HY_CUDA(c, launch_ep_counts(c->peers, N, rank, E, T, c->gcnt, epoch, budget_ns, c->err_word, st));
            if (!gemv) {
                HY_CUDA(c, launch_ep_local(c->peers, N, rank, E, el, T, H, K, dxn, c->topk_idx, c->chunk_base,
                                           c->goff, c->slot_pos, st, nrm));
            } else {
                if (T > 0)
                    HY_CUDA(c, launch_ep_scatter(c->peers, N, rank, E, el, T, H, K, dxn, c->topk_idx, c->chunk_base,
                                                 c->goff, c->slot_pos, c->done_ctas, epoch, st, nrm));
                else
                    HY_CUDA(c, launch_ep_raise(c->peers, N, rank, kEpFlagDeliver, epoch, st));
                HY_CUDA(c, launch_ep_wait(c->peers, N, rank, kEpFlagDeliver, epoch, budget_ns, c->err_word, st));
            }
            HY_CUDA(c, launch_ep_segments_fused(c->ep_meta + kEpCountOff, E + 1, N, rank, el, T, c->segs,
                                                c->seg_ret, c->n_segs, st));
            c->phase_end(HYMOE_PHASE_EP_DISPATCH, gemv ? 4 : 3);
            // Received counts stay on the device: size the decode kernel for full 64-row items.
            gemv_rows = kGemvMaxRows;
        } else if (ep) {
            // Count exchange: every rank learns how many rows each rank sends to each expert.
            c->phase_begin();
            ncclResult_t r = ncclAllGather(c->gcnt, c->C_dev, E, ncclInt32, c->comm, st);
            if (r != ncclSuccess && r != ncclInProgress)
                return c->fail(HYMOE_ERR_NCCL, "ncclAllGather(counts): %s", ncclGetErrorString(r));
            hymoe_status s2 = ep_poll(c, "count exchange");
            if (s2 != HYMOE_OK) return s2;
            HY_CUDA(c, cudaMemcpyAsync(c->C_host, c->C_dev, sizeof(int) * N * E, cudaMemcpyDeviceToHost, st));
            HY_CUDA(c, cudaEventRecord(c->ev_counts, st));
            s2 = ep_wait_event(c, c->ev_counts, "count exchange");
            if (s2 != HYMOE_OK) return s2;
            size_t so = 0, ro = T, total_sent = 0;
            for (int d = 0; d < N; ++d) {
                size_t sc = 0, rc = 0;
                for (int le = 0; le < el; ++le) {
                    sc += static_cast<size_t>(c->C_host[rank * E + d * el + le]);
                    rc += static_cast<size_t>(c->C_host[d * E + rank * el + le]);
                }
                send_cnt[d] = sc;
                send_off[d] = so;
                so += sc;
                recv_cnt[d] = rc;
                recv_off[d] = ro;
                ro += rc;
                total_sent += sc;
            }
            size_t max_rows = static_cast<size_t>(T);
            for (int le = 0; le < el; ++le) {
                size_t rows_le = 0;
                for (int src = 0; src < N; ++src) rows_le += static_cast<size_t>(c->C_host[src * E + rank * el + le]);
                max_rows = std::max(max_rows, rows_le);
            }
            gemv = max_rows <= static_cast<size_t>(kGemvMaxRows);
            gemv_rows = max_rows;
            // every pair is sent once, except those a capacity dropped
            if (c->route.drop ? total_sent > static_cast<size_t>(T) * K : total_sent != static_cast<size_t>(T) * K)
                return c->fail(HYMOE_ERR_STATE, "count exchange inconsistent: %zu rows for %d pairs", total_sent, T * K);
            // Every rank checks every rank's receive size (all hold the full count matrix), so
            // either all ranks proceed to the exchange or all return this error.
            for (int d = 0; d < N; ++d) {
                size_t rd = 0, td = 0;
                for (int src = 0; src < N; ++src)
                    for (int le = 0; le < el; ++le) rd += static_cast<size_t>(c->C_host[src * E + d * el + le]);
                for (int e2 = 0; e2 < E; ++e2) td += static_cast<size_t>(c->C_host[d * E + e2]);
                if (td / K + rd > c->rows_cap)
                    return c->fail(HYMOE_ERR_INVALID_ARG,
                                   "rank %d would receive %zu rows, above capacity %zu (max_tokens must be the "
                                   "same job-wide bound on every rank)", d, rd, c->rows_cap);
            }
            // Token rows to the ranks that own their experts (fp16, H per row).
            ncclGroupStart();
            for (int d = 0; d < N; ++d) {
                if (send_cnt[d])
                    ncclSend(c->xp_send + send_off[d] * H, send_cnt[d] * H, ncclFloat16, d, c->comm, st);
                if (recv_cnt[d])
                    ncclRecv(c->xp + recv_off[d] * H, recv_cnt[d] * H, ncclFloat16, d, c->comm, st);
            }
            r = ncclGroupEnd();
            if (r != ncclSuccess && r != ncclInProgress)
                return c->fail(HYMOE_ERR_NCCL, "token exchange: %s", ncclGetErrorString(r));
            s2 = ep_poll(c, "token exchange");
            if (s2 != HYMOE_OK) return s2;
            HY_CUDA(c, launch_ep_segments(c->C_dev, E, N, rank, el, E, T, c->segs, c->n_segs, st));
            c->phase_end(HYMOE_PHASE_EP_DISPATCH, 2);
        }

        if (ep) {  // single GPU: the plan kernel built the work items already
            c->phase_begin();
            HY_CUDA(c, launch_items(items_args(gemv), st));
            c->phase_end(HYMOE_PHASE_PLAN);
        }
        const size_t rows_in_use = p2p ? c->rows_cap
                                   : ep ? recv_off[N - 1] + recv_cnt[N - 1] : static_cast<size_t>(T) * (K + 1);
        EpFuse fuse{};
        if (p2p && !gemv) {
            fuse.peers = c->peers;
            fuse.N = N;
            fuse.me = rank;
            fuse.el = el;
            fuse.E = E;
            fuse.K = K;
            fuse.T = T;
            fuse.H = H;
            fuse.x = dxn;
            fuse.nrm = nrm;
            fuse.topk_idx = c->topk_idx;
            fuse.slot_pos = c->slot_pos;
            fuse.goff = c->goff;
            fuse.done = c->done_ctas;
            fuse.epoch = epoch;
            fuse.budget_ns = budget_ns;
        }
        if (gemv) {
            const int max_it = static_cast<int>(std::min<size_t>(
                c->max_items, static_cast<size_t>(tiles_gu) * ((rows_in_use + kGemvMaxRows - 1) / kGemvMaxRows + kMaxSegs)));
            c->phase_begin();
            const int mr = static_cast<int>(std::max<size_t>(1, gemv_rows));
            HY_CUDA(c, launch_gemv(c->gmaps_xp, c->items_gu, c->n_items, max_it, L.d_gu_ptrs, L.wtype, H / kTileK,
                                   1, mr, c->hbuf, I, nullptr, 0, c->err_word, c->n_sms, st, pdl));
            c->phase_end(HYMOE_PHASE_GATE_UP);
            c->phase_begin();
            HY_CUDA(c, launch_gemv(c->gmaps_h, c->items_dn, c->n_items + 1, max_it, L.d_dn_ptrs, L.wtype,
                                   I / kTileK, 0, mr, c->y, H, c->yr, T, c->err_word, c->n_sms, st, pdl));
            c->phase_end(HYMOE_PHASE_DOWN);
            if (p2p) {  // routed results back into their sources' return matrices, ready flags
                c->phase_begin();
                HY_CUDA(c, launch_ep_push(c->peers, N, rank, c->segs, c->seg_ret, c->n_segs, H, c->done_ctas, epoch,
                                          c->n_sms, st));
                c->phase_end(HYMOE_PHASE_EP_COMBINE);
            }
        } else {
            GemmArgs ga{};
            ga.items = c->items_gu;
            ga.n_items = c->n_items;
            ga.wtiles = L.d_gu_ptrs;
            ga.wtype = L.wtype;
            ga.n_ks = H / kTileK;
            ga.n_rb = tiles_gu;
            ga.glu = 1;
            ga.out = c->hbuf;
            ga.out_ld = I;
            ga.err = c->err_word;
            ga.ep_mode = p2p ? 1 : 0;  // fused: the remote rows leave and arrive during the GEMM
            fuse.aux = c->aux_gu;
            c->phase_begin();
            HY_CUDA(c, launch_gemm_tc(c->maps_xp, ga, c->n_sms, st, p2p ? &fuse : nullptr));
            c->phase_end(HYMOE_PHASE_GATE_UP);
            ga.items = c->items_dn;
            ga.n_items = c->n_items + 1;
            ga.wtiles = L.d_dn_ptrs;
            ga.n_ks = I / kTileK;
            ga.n_rb = tiles_dn;
            ga.glu = 0;
            ga.out = c->y;
            ga.out_r = c->yr;
            ga.shared_rows = T;
            ga.out_ld = H;
            ga.ep_mode = p2p ? 2 : 0;  // fused: results go back to their sources item by item
            fuse.aux = c->aux_dn;
            c->phase_begin();
            HY_CUDA(c, launch_gemm_tc(c->maps_h, ga, c->n_sms, st, p2p ? &fuse : nullptr));
            c->phase_end(HYMOE_PHASE_DOWN);
        }

        const __half* y_routed = c->yr + static_cast<size_t>(T) * H;
        if (p2p) {
            // Every owner has pushed this rank's results into y_ret: wait for their ready flags
            // (a rank without tokens waits too, so the next call's writes follow every owner's
            // GEMMs).
            c->phase_begin();
            HY_CUDA(c, launch_ep_wait(c->peers, N, rank, kEpFlagReady, epoch, budget_ns, c->err_word, st));
            c->phase_end(HYMOE_PHASE_EP_COMBINE);
            y_routed = c->y_ret;
        } else if (ep) {
            // Routed results back to the ranks their tokens came from (fp16, H per row).
            c->phase_begin();
            ncclGroupStart();
            for (int d = 0; d < N; ++d) {
                if (recv_cnt[d])
                    ncclSend(c->yr + recv_off[d] * H, recv_cnt[d] * H, ncclFloat16, d, c->comm, st);
                if (send_cnt[d])
                    ncclRecv(c->y_ret + send_off[d] * H, send_cnt[d] * H, ncclFloat16, d, c->comm, st);
            }
            ncclResult_t r = ncclGroupEnd();
            if (r != ncclSuccess && r != ncclInProgress)
                return c->fail(HYMOE_ERR_NCCL, "result exchange: %s", ncclGetErrorString(r));
            hymoe_status s2 = ep_poll(c, "result exchange");
            if (s2 != HYMOE_OK) return s2;
            c->phase_end(HYMOE_PHASE_EP_COMBINE);
            y_routed = c->y_ret;
        }
        if (shared_apart) HY_CUDA(c, cudaStreamWaitEvent(st, c->ev_join, 0));  // the shared expert's rows of y
        if (T > 0) {
            c->phase_begin();
            HY_CUDA(c, launch_combine(c->y, y_routed, c->slot_pos, c->topk_w, dres, dout, T, H, K, st,
                                      pdl && !shared_apart));
            c->phase_end(HYMOE_PHASE_COMBINE);
            hymoe_status sd = debug_out();
            if (sd != HYMOE_OK) return sd;
        }
        return HYMOE_OK;
    };

    const bool graph = (flags & HYMOE_USE_GRAPH) && !ep && !host && !c->prof && T > 0;
    if (!graph) {
        hymoe_status s2 = device_part();
        if (s2 != HYMOE_OK) return s2;
    } else {
        // One captured graph per (layer, token count, buffers); replayed while they repeat.
        const GraphKey key{layer | (pre_norm ? 0x80000000u : 0u), n_tokens, dx, dres, dout, dbias, dlog, dprob,
                           dbg ? dbg->topk_weights : nullptr, dbg ? dbg->topk_indices : nullptr};
        auto hit = c->graphs.find(key);
        if (hit == c->graphs.end()) {
            if (c->graphs.size() >= 64) c->clear_graphs();
            HY_CUDA(c, cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
            hymoe_status s2 = device_part();
            cudaGraph_t g = nullptr;
            const cudaError_t ec = cudaStreamEndCapture(st, &g);
            if (s2 != HYMOE_OK) {
                if (g) cudaGraphDestroy(g);
                return s2;
            }
            if (ec != cudaSuccess) return c->cuda_fail(ec, "cudaStreamEndCapture");
            cudaGraphExec_t ex = nullptr;
            const cudaError_t ei = cudaGraphInstantiate(&ex, g, 0);
            cudaGraphDestroy(g);
            if (ei != cudaSuccess) return c->cuda_fail(ei, "cudaGraphInstantiate");
            hit = c->graphs.emplace(key, ex).first;
        }
        HY_CUDA(c, cudaGraphLaunch(hit->second, st));
    }
    if (host) {
        if (T > 0) HY_CUDA(c, c->timed_copy(HYMOE_PHASE_COPY_OUT, out, dout, xbytes, cudaMemcpyDeviceToHost, st));
        return hymoe_synchronize(c);
    }
    return HYMOE_OK;
}

hymoe_status hymoe_profile(hymoe_ctx* c, int enable) {
    if (!c) return HYMOE_ERR_INVALID_ARG;
    if (enable) c->prof_clear();
    c->prof = enable != 0;
    return HYMOE_OK;
}

hymoe_status hymoe_profile_read(hymoe_ctx* c, float* total_ms, int32_t* launches, int n) {
    if (!c || n < 0 || n > HYMOE_NUM_PHASES) return HYMOE_ERR_INVALID_ARG;
    HY_CUDA(c, cudaSetDevice(c->cfg.device));
    HY_CUDA(c, cudaStreamSynchronize(c->stream));
    for (int p = 0; p < n; ++p) {
        float tot = 0.f;
        for (auto& pr : c->prof_ev[p]) {
            float ms = 0.f;
            HY_CUDA(c, cudaEventElapsedTime(&ms, pr.first, pr.second));
            tot += ms;
        }
        if (total_ms) total_ms[p] = tot;
        if (launches) launches[p] = c->prof_launches[p];
    }
    return HYMOE_OK;
}

}  // extern "C"
