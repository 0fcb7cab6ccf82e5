// ffn_noalloc.cu — hymoe_ffn_noalloc: one SwiGLU expert FFN for a few tokens that
// allocates no device memory.
//
// For callers that cannot call cudaMalloc (code running inside CUDA stream capture, where
// allocation calls are not permitted; engines whose device memory is owned by another
// allocator or pool and forbid raw driver allocations after start-up; real-time decode
// loops that must not allocate per step).  Such a caller owns every buffer it passes:
// the GGUF weights and the activations already live in device memory.  The only
// intermediate this computation needs, the SwiGLU activation h[n_tokens, I], lives in
// the fixed array below, which every GPU that loads the library holds until the process
// exits.
//
// Maximum sizes: n_tokens <= HYMOE_NOALLOC_MAX_TOKENS (8), I <= HYMOE_NOALLOC_MAX_INTERMEDIATE
// (16384): 8 x 16384 floats = 512 KiB per device.
//
// The computation is src/rms_norm.cpp:39-91 (swiglu_ffn_f32): h = silu(x Wg^T) * (x Wu^T),
// y = h Wd^T, with the weights read straight from standard GGUF blocks (fp32 accumulate).
#include <cstdio>
#include <mutex>

#include "../../include/hymoe.h"
#include "common.cuh"

namespace hymoe {
namespace {

constexpr int kNaTokens = HYMOE_NOALLOC_MAX_TOKENS;
constexpr int kNaInter = HYMOE_NOALLOC_MAX_INTERMEDIATE;

// Shared by every call on a device; each call overwrites the rows it reads
// (h[n][j] for n < n_tokens, j < I) before reading them, so nothing needs clearing.
// Calls that overlap on the GPU (different streams, no ordering) race on it.
static __device__ __align__(256) float g_noalloc_h[kNaTokens * kNaInter];

// Value j (0..31) of one standard GGUF block.
template <int WT>
__device__ __forceinline__ void gguf_block(const uint8_t* blk, float (&v)[32]) {
    if constexpr (WT == W_Q4_0) {
        const float d = __half2float(*reinterpret_cast<const __half*>(blk));
        const uint16_t* q = reinterpret_cast<const uint16_t*>(blk + 2);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t two = q[i];  // bytes 2i, 2i+1
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const uint32_t byte = (two >> (8 * k)) & 0xFFu;
                v[2 * i + k] = static_cast<float>(static_cast<int>(byte & 0xFu) - 8) * d;
                v[2 * i + k + 16] = static_cast<float>(static_cast<int>(byte >> 4) - 8) * d;
            }
        }
    } else if constexpr (WT == W_Q8_0) {
        const float d = __half2float(*reinterpret_cast<const __half*>(blk));
        const uint16_t* q = reinterpret_cast<const uint16_t*>(blk + 2);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const uint32_t two = q[i];
            v[2 * i] = static_cast<float>(static_cast<int8_t>(two & 0xFFu)) * d;
            v[2 * i + 1] = static_cast<float>(static_cast<int8_t>(two >> 8)) * d;
        }
    } else if constexpr (WT == W_F16) {
        const __half2* h = reinterpret_cast<const __half2*>(blk);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const float2 f = __half22float2(h[i]);
            v[2 * i] = f.x;
            v[2 * i + 1] = f.y;
        }
    } else {
        const float* f = reinterpret_cast<const float*>(blk);
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = f[i];
    }
}

template <int WT>
constexpr int block_bytes() {
    return WT == W_Q4_0 ? 18 : WT == W_Q8_0 ? 34 : WT == W_F16 ? 64 : 128;
}

// Warp-wide dot products of one GGUF row (K values) with n activation rows.
template <int WT>
__device__ __forceinline__ void row_dots(const uint8_t* row, const float* act, int act_ld, int K,
                                         int n, float (&acc)[kNaTokens]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int t = 0; t < kNaTokens; ++t) acc[t] = 0.f;
    for (int b = lane; b < K / 32; b += 32) {
        float v[32];
        gguf_block<WT>(row + static_cast<size_t>(b) * block_bytes<WT>(), v);
#pragma unroll
        for (int t = 0; t < kNaTokens; ++t) {
            if (t >= n) break;
            const float4* a = reinterpret_cast<const float4*>(act + static_cast<size_t>(t) * act_ld + 32 * b);
            float s = 0.f;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const float4 x = a[c];
                s = fmaf(v[4 * c], x.x, s);
                s = fmaf(v[4 * c + 1], x.y, s);
                s = fmaf(v[4 * c + 2], x.z, s);
                s = fmaf(v[4 * c + 3], x.w, s);
            }
            acc[t] += s;
        }
    }
#pragma unroll
    for (int t = 0; t < kNaTokens; ++t)
#pragma unroll
        for (int o = 16; o; o >>= 1) acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], o);
}

// One warp per intermediate column j: gate row j and up row I + j -> h[t][j].
template <int WT>
__global__ __launch_bounds__(256) void ffn_gate_up_kernel(const uint8_t* __restrict__ gu,
                                                          const float* __restrict__ x, int H,
                                                          int I, int n, float* __restrict__ h) {
    const int j = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (j >= I) return;
    const size_t row_bytes = static_cast<size_t>(H / 32) * block_bytes<WT>();
    float g[kNaTokens], u[kNaTokens];
    row_dots<WT>(gu + static_cast<size_t>(j) * row_bytes, x, H, H, n, g);
    row_dots<WT>(gu + static_cast<size_t>(I + j) * row_bytes, x, H, H, n, u);
    if ((threadIdx.x & 31) == 0)
        for (int t = 0; t < n; ++t) h[static_cast<size_t>(t) * kNaInter + j] = silu_mul(g[t], u[t]);
}

// One warp per output feature i: y[t][i] = h[t] . Wd[i].
template <int WT>
__global__ __launch_bounds__(256) void ffn_down_kernel(const uint8_t* __restrict__ dn,
                                                       const float* __restrict__ h, int H, int I,
                                                       int n, float* __restrict__ y) {
    const int i = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (i >= H) return;
    const size_t row_bytes = static_cast<size_t>(I / 32) * block_bytes<WT>();
    float acc[kNaTokens];
    row_dots<WT>(dn + static_cast<size_t>(i) * row_bytes, h, kNaInter, I, n, acc);
    if ((threadIdx.x & 31) == 0)
        for (int t = 0; t < n; ++t) y[static_cast<size_t>(t) * H + i] = acc[t];
}

template <int WT>
cudaError_t launch_ffn(const uint8_t* gu, const uint8_t* dn, const float* x, float* y, int H,
                       int I, int n, float* h, cudaStream_t st) {
    ffn_gate_up_kernel<WT><<<(I + 7) / 8, 256, 0, st>>>(gu, x, H, I, n, h);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    ffn_down_kernel<WT><<<(H + 7) / 8, 256, 0, st>>>(dn, h, H, I, n, y);
    return cudaGetLastError();
}

// Device address of g_noalloc_h, looked up once per device with that device current.
// The host-side name of the array is only a stand-in, never a device address.
std::mutex g_mu;
float* g_scratch[128] = {};

cudaError_t scratch_for_current_device(float** out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 128) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_scratch[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_h);
        if (e != cudaSuccess) return e;
        g_scratch[dev] = static_cast<float*>(p);
    }
    *out = g_scratch[dev];
    return cudaSuccess;
}

// Memory the kernels, which run on the current device `dev`, may read and write directly:
// device memory of that device, or managed memory.  Another GPU's memory is refused (it would
// turn into peer traffic, or an illegal access without a peer mapping).
bool on_device(const void* p, int dev) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    if (a.type == cudaMemoryTypeManaged) return true;
    return a.type == cudaMemoryTypeDevice && a.device == dev;
}

size_t gguf_bytes(int type, int64_t n) {
    switch (type) {
        case HYMOE_TYPE_F32: return static_cast<size_t>(n) * 4;
        case HYMOE_TYPE_F16: return static_cast<size_t>(n) * 2;
        case HYMOE_TYPE_Q4_0: return static_cast<size_t>(n / 32) * 18;
        case HYMOE_TYPE_Q8_0: return static_cast<size_t>(n / 32) * 34;
        default: return 0;
    }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

// Thread-local message slot read by hymoe_last_error(NULL) (hymoe_api.cu).
void set_thread_error(const char* msg);

}  // namespace hymoe

using namespace hymoe;

extern "C" hymoe_status hymoe_ffn_noalloc(const hymoe_tensor* gate_up, const hymoe_tensor* down,
                                          const float* x, float* y, uint32_t n_tokens,
                                          void* stream) {
    auto bad = [](hymoe_status st, const char* msg) {
        set_thread_error(msg);
        return st;
    };
    set_thread_error("");
    if (!gate_up || !down || !gate_up->data || !down->data || !x || !y)
        return bad(HYMOE_ERR_INVALID_ARG, "hymoe_ffn_noalloc: null argument");
    if (n_tokens == 0) return HYMOE_OK;
    if (n_tokens > HYMOE_NOALLOC_MAX_TOKENS)
        return bad(HYMOE_ERR_INVALID_ARG,
                   "hymoe_ffn_noalloc: n_tokens exceeds HYMOE_NOALLOC_MAX_TOKENS (8)");
    const int t = gate_up->ggml_type;
    const int64_t H = gate_up->ne[0], I2 = gate_up->ne[1];
    if (t != down->ggml_type || (t != HYMOE_TYPE_F32 && t != HYMOE_TYPE_F16 &&
                                 t != HYMOE_TYPE_Q4_0 && t != HYMOE_TYPE_Q8_0))
        return bad(HYMOE_ERR_INVALID_ARG, "hymoe_ffn_noalloc: both tensors must share one GGUF type "
                                          "of F32/F16/Q4_0/Q8_0");
    if (H <= 0 || I2 <= 0 || I2 % 2 || H % 32 || (I2 / 2) % 32 || down->ne[0] != I2 / 2 ||
        down->ne[1] != H)
        return bad(HYMOE_ERR_INVALID_ARG, "hymoe_ffn_noalloc: need gate_up [2I, H], down [H, I], "
                                          "H and I multiples of 32");
    if (I2 / 2 > HYMOE_NOALLOC_MAX_INTERMEDIATE)
        return bad(HYMOE_ERR_INVALID_ARG,
                   "hymoe_ffn_noalloc: intermediate size exceeds HYMOE_NOALLOC_MAX_INTERMEDIATE (16384)");
    if (gate_up->nbytes != gguf_bytes(t, H * I2) || down->nbytes != gguf_bytes(t, H * I2 / 2))
        return bad(HYMOE_ERR_INVALID_ARG, "hymoe_ffn_noalloc: nbytes does not match the GGUF size");
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) return bad(HYMOE_ERR_CUDA, "hymoe_ffn_noalloc: cudaGetDevice failed");
    if (!on_device(gate_up->data, dev) || !on_device(down->data, dev) || !on_device(x, dev) || !on_device(y, dev))
        return bad(HYMOE_ERR_INVALID_ARG, "hymoe_ffn_noalloc: every pointer must be device memory of the "
                                          "current device (or managed memory)");
    if (!aligned16(gate_up->data) || !aligned16(down->data) || !aligned16(x) || !aligned16(y))
        return bad(HYMOE_ERR_INVALID_ARG, "hymoe_ffn_noalloc: pointers must be 16-byte aligned");
    float* h = nullptr;
    cudaError_t e = scratch_for_current_device(&h);
    if (e != cudaSuccess)
        return bad(HYMOE_ERR_CUDA, "hymoe_ffn_noalloc: cudaGetSymbolAddress failed");
    const uint8_t* gu = static_cast<const uint8_t*>(gate_up->data);
    const uint8_t* dn = static_cast<const uint8_t*>(down->data);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int Hi = static_cast<int>(H), Ii = static_cast<int>(I2 / 2), n = static_cast<int>(n_tokens);
    switch (t) {
        case HYMOE_TYPE_Q4_0: e = launch_ffn<W_Q4_0>(gu, dn, x, y, Hi, Ii, n, h, st); break;
        case HYMOE_TYPE_Q8_0: e = launch_ffn<W_Q8_0>(gu, dn, x, y, Hi, Ii, n, h, st); break;
        case HYMOE_TYPE_F16: e = launch_ffn<W_F16>(gu, dn, x, y, Hi, Ii, n, h, st); break;
        default: e = launch_ffn<W_F32>(gu, dn, x, y, Hi, Ii, n, h, st); break;
    }
    if (e != cudaSuccess) return bad(HYMOE_ERR_CUDA, "hymoe_ffn_noalloc: kernel launch failed");
    return HYMOE_OK;
}
