// weights.cu — GGUF -> device tile re-tiling, and the on-device synthetic generator.
//
// Re-tiling keeps every GGUF block's information unchanged, so the device holds exactly the
// GGUF Q4_0 / Q8_0 bytes (hunyuan_gguf_loader.cpp:172-177 sizes): the fp16 d and the Q4_0
// nibbles verbatim, the Q8_0 int8 quants stored excess-128 (q ^ 0x80 = q + 128 as an
// unsigned byte), which lets the kernels turn a byte into the fp16 value 1024 + q + 128
// with a single byte permute.  F32 and F16 matrices become F16 tiles.
//
// The generator restates the test oracle's published algorithm on the device:
// Philox4x32-10 (Salmon et al., SC'11) per element, Irwin-Hall sum of its 8 16-bit
// halves, then the GGUF quantisation rule of gguf-py 0.19.0 (gguf/quants.py).  Every
// float operation is an explicitly rounded IEEE operation (no contraction), so the
// bytes equal the CPU generator's.
#include "common.cuh"
#include "kernels.h"

namespace hymoe {

namespace {

__device__ __forceinline__ int gguf_block_bytes(int t) {
    return t == W_Q4_0 ? 18 : t == W_Q8_0 ? 34 : t == W_F16 ? 64 : 128;
}

// One thread per (row block, k tile, tile row r, block b).
__global__ void repack_kernel(const uint8_t* __restrict__ src, int src_type,
                              uint8_t* __restrict__ dst, int dst_type, int rows, int K,
                              int glu_I) {
    const int n_ks = K / kTileK;
    const int n_rb = rows / kTileRows;
    const int64_t total = static_cast<int64_t>(n_rb) * n_ks * 256;
    const int64_t item = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (item >= total) return;
    const int rb_ks = static_cast<int>(item >> 8);
    const int e = static_cast<int>(item & 255);
    const int r = e >> 1, b = e & 1;
    const int rb = rb_ks / n_ks, ks = rb_ks % n_ks;
    int srow;
    if (glu_I > 0) {  // gate_up tile: groups of 16 gate rows and their 16 up rows
        const int j = 16 * (r >> 5) + (r & 15);
        srow = (r & 16) ? glu_I + kGluHalf * rb + j : kGluHalf * rb + j;
    }
    else
        srow = kTileRows * rb + r;
    const int bsz = gguf_block_bytes(src_type);
    const uint8_t* sb = src + static_cast<int64_t>(srow) * (K / 32) * bsz +
                        static_cast<int64_t>(2 * ks + b) * bsz;
    uint8_t* tile = dst + static_cast<int64_t>(rb_ks) * tile_bytes(dst_type);
    if (dst_type == W_Q4_0 || dst_type == W_Q8_0) {
        const int qn = dst_type == W_Q4_0 ? 16 : 32;
        tile[2 * e] = sb[0];
        tile[2 * e + 1] = sb[1];
        uint8_t* q = tile + 512 + e * qn;
        const uint8_t flip = dst_type == W_Q8_0 ? 0x80 : 0x00;
        for (int j = 0; j < qn; ++j) q[j] = sb[2 + j] ^ flip;
    } else {  // F16 tile row r, halves [32 b, 32 b + 32)
        __half* row = reinterpret_cast<__half*>(tile) + r * kTileK + 32 * b;
        if (src_type == W_F16) {
            const __half* s = reinterpret_cast<const __half*>(sb);
            for (int j = 0; j < 32; ++j) row[j] = s[j];
        } else {
            const float* s = reinterpret_cast<const float*>(sb);
            for (int j = 0; j < 32; ++j) row[j] = __float2half_rn(s[j]);
        }
    }
}

__device__ __forceinline__ void philox4x32_10(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3,
                                              uint32_t k0, uint32_t k1, uint32_t (&o)[4]) {
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        if (r) {
            k0 += 0x9E3779B9u;
            k1 += 0xBB67AE85u;
        }
        const uint32_t hi0 = __umulhi(0xD2511F53u, c0), lo0 = 0xD2511F53u * c0;
        const uint32_t hi1 = __umulhi(0xCD9E8D57u, c2), lo1 = 0xCD9E8D57u * c2;
        const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
        c1 = lo1;
        c3 = lo0;
        c0 = n0;
        c2 = n2;
    }
    o[0] = c0;
    o[1] = c1;
    o[2] = c2;
    o[3] = c3;
}

__device__ __forceinline__ float synth_value(uint64_t i, uint64_t seed, uint64_t stream,
                                             float c) {
    uint32_t r[4];
    philox4x32_10(static_cast<uint32_t>(i), static_cast<uint32_t>(i >> 32),
                  static_cast<uint32_t>(stream), static_cast<uint32_t>(stream >> 32),
                  static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32), r);
    int s = 0;
#pragma unroll
    for (int w = 0; w < 4; ++w) s += static_cast<int>(r[w] & 0xFFFFu) + static_cast<int>(r[w] >> 16);
    return __fmul_rn(static_cast<float>(s - 262140), c);
}

// One 16-bit store: every GGUF block (18 / 34 / 64 bytes) starts on an even offset of a
// cudaMalloc'd buffer, so the fp16 field is 2-byte aligned.
__device__ __forceinline__ void put_half(uint8_t* p, float v) {
    *reinterpret_cast<__half*>(p) = __float2half_rn(v);
}

// One thread per 32-element GGUF block.
__global__ void synth_gguf_kernel(uint8_t* __restrict__ dst, int type, uint64_t nblocks,
                                  uint64_t seed, uint64_t stream, float c) {
    const uint64_t blk = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (blk >= nblocks) return;
    float x[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) x[j] = synth_value(32 * blk + j, seed, stream, c);
    if (type == W_F32) {
        float* o = reinterpret_cast<float*>(dst) + 32 * blk;
        for (int j = 0; j < 32; ++j) o[j] = x[j];
        return;
    }
    if (type == W_F16) {
        uint8_t* o = dst + 64 * blk;
        for (int j = 0; j < 32; ++j) put_half(o + 2 * j, x[j]);
        return;
    }
    if (type == W_Q4_0) {
        uint8_t* o = dst + 18 * blk;
        float amax = 0.0f, vmax = 0.0f;
        for (int j = 0; j < 32; ++j) {
            const float a = fabsf(x[j]);
            if (a > amax) {
                amax = a;
                vmax = x[j];
            }
        }
        const float d = __fdiv_rn(vmax, -8.0f);
        const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        uint8_t q[32];
        for (int j = 0; j < 32; ++j) {
            const float t = truncf(__fadd_rn(__fmul_rn(x[j], id), 8.5f));
            const int v = t < 0.0f ? 0 : static_cast<int>(t);
            q[j] = static_cast<uint8_t>(v > 15 ? 15 : v);
        }
        put_half(o, d);
        for (int j = 0; j < 16; ++j) o[2 + j] = static_cast<uint8_t>(q[j] | (q[j + 16] << 4));
        return;
    }
    // Q8_0
    uint8_t* o = dst + 34 * blk;
    float amax = 0.0f;
    for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(x[j]));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    put_half(o, d);
    for (int j = 0; j < 32; ++j)
        o[2 + j] = static_cast<uint8_t>(static_cast<int8_t>(roundf(__fmul_rn(x[j], id))));
}

__global__ void synth_f32_kernel(float* __restrict__ dst, uint64_t n, uint64_t seed,
                                 uint64_t stream, float c) {
    const uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) dst[i] = synth_value(i, seed, stream, c);
}

}  // namespace

cudaError_t launch_repack(const uint8_t* src, int src_type, uint8_t* dst, int dst_type, int rows,
                          int K, int glu_I, cudaStream_t st) {
    const int64_t total = static_cast<int64_t>(rows / kTileRows) * (K / kTileK) * 256;
    const int threads = 256;
    const int64_t blocks = (total + threads - 1) / threads;
    repack_kernel<<<static_cast<unsigned>(blocks), threads, 0, st>>>(src, src_type, dst, dst_type,
                                                                     rows, K, glu_I);
    return cudaGetLastError();
}

cudaError_t launch_synth_gguf(uint8_t* dst, int type, uint64_t n, uint64_t seed, uint64_t stream,
                              float scale, cudaStream_t st) {
    const uint64_t nb = n / 32;
    const int threads = 128;
    synth_gguf_kernel<<<static_cast<unsigned>((nb + threads - 1) / threads), threads, 0, st>>>(
        dst, type, nb, seed, stream, scale);
    return cudaGetLastError();
}

cudaError_t launch_synth_f32(float* dst, uint64_t n, uint64_t seed, uint64_t stream, float scale,
                             cudaStream_t st) {
    const int threads = 256;
    synth_f32_kernel<<<static_cast<unsigned>((n + threads - 1) / threads), threads, 0, st>>>(
        dst, n, seed, stream, scale);
    return cudaGetLastError();
}

}  // namespace hymoe
