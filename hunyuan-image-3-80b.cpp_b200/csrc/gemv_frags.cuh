// gemv_frags.cuh — register fragments of the weight-streaming kernels (gemv.cu, decode.cu):
// GGUF Q4_0 / Q8_0 / F16 tiles and fp16 activation boxes as mma.sync m16n8k16 operands.
//
// The quants become exact fp16 integers (q - 8 or q, via the 0x6400 magic-number trick).  A
// k-permutation shared by A and B (each thread's MMA k positions 2c, 2c+1, 2c+8, 2c+9,
// c = lane % 4, hold four CONSECUTIVE quants of a GGUF block) lets each thread build its A
// fragments from wide shared-memory loads of raw quants; B columns are token rows permuted so
// that the swizzled activation loads are free of bank conflicts too.
#pragma once

#include <type_traits>

#include "common.cuh"

namespace hymoe {
namespace gemvf {

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// Four consecutive excess-128 Q8_0 bytes (one 32-bit word) -> two half2 {q0,q1}, {q2,q3}.
__device__ __forceinline__ void q8x4_to_h2(uint32_t w, uint32_t& lo, uint32_t& hi) {
    const __half2 off = __float2half2_rn(1152.0f);  // 1024 magic + 128 excess
    lo = h2u(__hsub2(u2h(__byte_perm(w, 0x64u, 0x4140)), off));
    hi = h2u(__hsub2(u2h(__byte_perm(w, 0x64u, 0x4342)), off));
}

// Nibbles of four consecutive Q4_0 bytes -> (q - 8) as half2: low nibbles (first half of the
// block) and high nibbles (second half).
__device__ __forceinline__ void q4x4_to_h2(uint32_t w, uint32_t (&low)[2], uint32_t (&high)[2]) {
    const __half2 off = __float2half2_rn(1032.0f);  // 1024 magic + 8 offset
    const uint32_t p0 = __byte_perm(w, 0, 0x4140), p1 = __byte_perm(w, 0, 0x4342);
    low[0] = h2u(__hsub2(u2h((p0 & 0x000F000Fu) | 0x64006400u), off));
    low[1] = h2u(__hsub2(u2h((p1 & 0x000F000Fu) | 0x64006400u), off));
    high[0] = h2u(__hsub2(u2h(((p0 >> 4) & 0x000F000Fu) | 0x64006400u), off));
    high[1] = h2u(__hsub2(u2h(((p1 >> 4) & 0x000F000Fu) | 0x64006400u), off));
}

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Token row of the n-tile held by B column m (m = lane / 4 for the B fragment, 2c and 2c + 1
// for the accumulator): a permutation chosen so that each shared-memory phase of the
// activation loads touches distinct banks under the 128-byte swizzle.
template <int WT>
__device__ __forceinline__ int col_token(int m) {
    if constexpr (WT == W_Q4_0) return ((m & 3) << 1) | (m >> 2);  // half-warps: rows 0,2,4,6 / 1,3,5,7
    else return ((m & 1) << 2) | (m >> 1);                          // quarter-warps: rows n, n + 4
}

// A fragments of one 16-row group (MMA rows g and g + 8 = tile rows r0 and r0 + 8) for both
// GGUF blocks b and both k-steps s of each: a[b][s][0..3].  Element order inside a
// 32-element block (the k-permutation; x uses the same one):
//   Q8_0, F16: thread c holds elements 8c + 4s + {0..3}
//   Q4_0:      thread c holds elements 16s + 4c + {0..3} (low nibbles s = 0, high s = 1)
// PRE: the fragments are multiplied by the block scales in fp16 (the tensor-core path's
// rounding of each weight); otherwise they hold the exact integers q (Q8_0) or q - 8 (Q4_0)
// and d[b][row] returns the scales, applied to each block's fp32 partial sums.
template <int WT, bool PRE>
__device__ __forceinline__ void tile_frags(const uint8_t* tile, int r0, int c, uint32_t (&a)[2][2][4],
                                           float (&d)[2][2]) {
    if constexpr (WT == W_F16) {  // tile [128 rows][64 halves]
#pragma unroll
        for (int b = 0; b < 2; ++b) {
            const uint4 v0 = *reinterpret_cast<const uint4*>(tile + (r0 * 64 + 32 * b + 8 * c) * 2);
            const uint4 v1 = *reinterpret_cast<const uint4*>(tile + ((r0 + 8) * 64 + 32 * b + 8 * c) * 2);
            a[b][0][0] = v0.x; a[b][0][2] = v0.y; a[b][1][0] = v0.z; a[b][1][2] = v0.w;
            a[b][0][1] = v1.x; a[b][0][3] = v1.y; a[b][1][1] = v1.z; a[b][1][3] = v1.w;
            d[b][0] = d[b][1] = 1.0f;
        }
    } else {
        // scales: entries 2r, 2r + 1 (blocks 0, 1 of row r) are one 32-bit word
        const __half2 s0 = *reinterpret_cast<const __half2*>(tile + 4 * r0);
        const __half2 s1 = *reinterpret_cast<const __half2*>(tile + 4 * (r0 + 8));
        const uint8_t* q = tile + 512;
#pragma unroll
        for (int b = 0; b < 2; ++b) {
            if constexpr (WT == W_Q8_0) {
                const uint2 v0 = *reinterpret_cast<const uint2*>(q + 32 * (2 * r0 + b) + 8 * c);
                const uint2 v1 = *reinterpret_cast<const uint2*>(q + 32 * (2 * (r0 + 8) + b) + 8 * c);
                q8x4_to_h2(v0.x, a[b][0][0], a[b][0][2]);
                q8x4_to_h2(v0.y, a[b][1][0], a[b][1][2]);
                q8x4_to_h2(v1.x, a[b][0][1], a[b][0][3]);
                q8x4_to_h2(v1.y, a[b][1][1], a[b][1][3]);
            } else {  // Q4_0
                uint32_t l0[2], h0[2], l1[2], h1[2];
                q4x4_to_h2(*reinterpret_cast<const uint32_t*>(q + 16 * (2 * r0 + b) + 4 * c), l0, h0);
                q4x4_to_h2(*reinterpret_cast<const uint32_t*>(q + 16 * (2 * (r0 + 8) + b) + 4 * c), l1, h1);
                a[b][0][0] = l0[0]; a[b][0][2] = l0[1]; a[b][0][1] = l1[0]; a[b][0][3] = l1[1];
                a[b][1][0] = h0[0]; a[b][1][2] = h0[1]; a[b][1][1] = h1[0]; a[b][1][3] = h1[1];
            }
        }
        if constexpr (PRE) {
#pragma unroll
            for (int b = 0; b < 2; ++b) {
                const __half2 d0 = b ? __high2half2(s0) : __low2half2(s0);  // row r0
                const __half2 d1 = b ? __high2half2(s1) : __low2half2(s1);  // row r0 + 8
#pragma unroll
                for (int s = 0; s < 2; ++s) {
                    a[b][s][0] = h2u(__hmul2(u2h(a[b][s][0]), d0));
                    a[b][s][2] = h2u(__hmul2(u2h(a[b][s][2]), d0));
                    a[b][s][1] = h2u(__hmul2(u2h(a[b][s][1]), d1));
                    a[b][s][3] = h2u(__hmul2(u2h(a[b][s][3]), d1));
                }
            }
        } else {
            d[0][0] = __low2float(s0); d[1][0] = __high2float(s0);
            d[0][1] = __low2float(s1); d[1][1] = __high2float(s1);
        }
    }
}

// The raw shared-memory words of one 16-row group of a Q4_0 / Q8_0 tile that tile_frags<WT, false>
// reads (scales of rows r0 and r0 + 8, quants of both blocks), loaded first so that a caller can
// hand the tile's buffer back to its copy engine before the conversion and the MMAs.
template <int WT>
struct RawGroup {
    uint32_t s0, s1;                                            // block scales, rows r0 / r0 + 8
    typename std::conditional<WT == W_Q8_0, uint2, uint32_t>::type v[2][2];  // [block][row r0 / r0 + 8]
};

template <int WT>
__device__ __forceinline__ void tile_raw(const uint8_t* tile, int r0, int c, RawGroup<WT>& g) {
    g.s0 = *reinterpret_cast<const uint32_t*>(tile + 4 * r0);
    g.s1 = *reinterpret_cast<const uint32_t*>(tile + 4 * (r0 + 8));
    const uint8_t* q = tile + 512;
#pragma unroll
    for (int b = 0; b < 2; ++b) {
        if constexpr (WT == W_Q8_0) {
            g.v[b][0] = *reinterpret_cast<const uint2*>(q + 32 * (2 * r0 + b) + 8 * c);
            g.v[b][1] = *reinterpret_cast<const uint2*>(q + 32 * (2 * (r0 + 8) + b) + 8 * c);
        } else {
            g.v[b][0] = *reinterpret_cast<const uint32_t*>(q + 16 * (2 * r0 + b) + 4 * c);
            g.v[b][1] = *reinterpret_cast<const uint32_t*>(q + 16 * (2 * (r0 + 8) + b) + 4 * c);
        }
    }
}

// tile_frags<WT, false> from the raw words (the same fragments and scales).
template <int WT>
__device__ __forceinline__ void raw_frags(const RawGroup<WT>& g, uint32_t (&a)[2][2][4], float (&d)[2][2]) {
#pragma unroll
    for (int b = 0; b < 2; ++b) {
        if constexpr (WT == W_Q8_0) {
            q8x4_to_h2(g.v[b][0].x, a[b][0][0], a[b][0][2]);
            q8x4_to_h2(g.v[b][0].y, a[b][1][0], a[b][1][2]);
            q8x4_to_h2(g.v[b][1].x, a[b][0][1], a[b][0][3]);
            q8x4_to_h2(g.v[b][1].y, a[b][1][1], a[b][1][3]);
        } else {
            uint32_t l0[2], h0[2], l1[2], h1[2];
            q4x4_to_h2(g.v[b][0], l0, h0);
            q4x4_to_h2(g.v[b][1], l1, h1);
            a[b][0][0] = l0[0]; a[b][0][2] = l0[1]; a[b][0][1] = l1[0]; a[b][0][3] = l1[1];
            a[b][1][0] = h0[0]; a[b][1][2] = h0[1]; a[b][1][1] = h1[0]; a[b][1][3] = h1[1];
        }
    }
    const __half2 s0 = u2h(g.s0), s1 = u2h(g.s1);
    d[0][0] = __low2float(s0); d[1][0] = __high2float(s0);
    d[0][1] = __low2float(s1); d[1][1] = __high2float(s1);
}

// B fragments of one token row (128 bytes = 64 halves, 16-byte chunks swizzled by XOR with
// row & 7) for both blocks and k-steps, in the element order of tile_frags.
template <int WT>
__device__ __forceinline__ void x_frags(const uint8_t* xrow, int sw, int c, uint32_t (&bx)[2][2][2]) {
#pragma unroll
    for (int b = 0; b < 2; ++b) {
        if constexpr (WT == W_Q4_0) {
#pragma unroll
            for (int s = 0; s < 2; ++s) {  // halves 32b + 16s + 4c .. +3
                const int chunk = 4 * b + 2 * s + (c >> 1);
                const uint2 v = *reinterpret_cast<const uint2*>(xrow + 16 * (chunk ^ sw) + 8 * (c & 1));
                bx[b][s][0] = v.x;
                bx[b][s][1] = v.y;
            }
        } else {  // halves 32b + 8c .. +7
            const uint4 v = *reinterpret_cast<const uint4*>(xrow + 16 * ((4 * b + c) ^ sw));
            bx[b][0][0] = v.x; bx[b][0][1] = v.y;
            bx[b][1][0] = v.z; bx[b][1][1] = v.w;
        }
    }
}

}  // namespace gemvf
}  // namespace hymoe
