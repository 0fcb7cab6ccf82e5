// common.cuh — shared definitions for the hymoe sm_100a kernels.
//
// Device weight format ("tiles").  The C ABI accepts standard GGUF blocks; on load each
// expert matrix is re-tiled on the device (same bytes per block, different order) so a
// (128-row x 64-column) slab is one contiguous, 16-byte aligned run that a single bulk
// copy moves into shared memory:
//
//   tile(rb, ks) = rows [128 rb, 128 rb + 128) x columns [64 ks, 64 ks + 64)
//   Q4_0 : [ d   : 256 x f16 ][ qs : 256 x 16 B ]          4608 B
//   Q8_0 : [ d   : 256 x f16 ][ qs : 256 x 32 B ]          8704 B
//   F16  : [ 128 rows x 64 halves, row-major ]           16384 B
// where entry (r, b) = 2 r + b is row r's GGUF block b (b = 0, 1) of the slab.  Tiles of a
// row block are consecutive along ks.  For a gate_up matrix ([2I, H]) tile rows 0..63
// are gate rows 64 rb + r and rows 64..127 are the matching up rows I + 64 rb + r, so a
// tile yields both halves of the SwiGLU for 64 output columns.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace hymoe {

constexpr int kTileRows = 128;  // weight rows per tile
constexpr int kTileK = 64;      // K elements per tile (two GGUF blocks)
constexpr int kGluHalf = 64;    // gate (or up) rows per gate_up tile
// Row order inside a gate_up tile: four groups of 32 rows, each 16 gate rows followed by the
// matching 16 up rows, so one TMEM lane quarter (one warp) holds both SwiGLU halves of its 16
// output columns.  Output column j (0..63) of the tile:
__host__ __device__ constexpr int glu_gate_row(int j) { return 32 * (j >> 4) + (j & 15); }
__host__ __device__ constexpr int glu_up_row(int j) { return 32 * (j >> 4) + 16 + (j & 15); }

enum WType : int { W_F32 = 0, W_F16 = 1, W_Q4_0 = 2, W_Q8_0 = 8 };

__host__ __device__ constexpr int tile_bytes(int wt) {
    return wt == W_Q4_0 ? 4608 : wt == W_Q8_0 ? 8704 : 16384;
}

// Device-side error word codes (bit flags), read back by hymoe_synchronize.
enum DevErr : int {
    DEVERR_TIMEOUT_PRODUCER = 1,
    DEVERR_TIMEOUT_DEQUANT = 2,
    DEVERR_TIMEOUT_MMA = 4,
    DEVERR_TIMEOUT_EPILOGUE = 8,
    DEVERR_BAD_ITEM = 16,
    DEVERR_TIMEOUT_PEER = 32,  // a peer GPU's flag did not arrive in time
    DEVERR_TIMEOUT_DECODE = 64,  // the one-kernel decode path: a counter did not arrive in time
    DEVERR_SPEC_MISMATCH = 128,  // the certified routing pass disagreed with the chains (a defect)
};

// ------------------------------------------------------------------ PTX wrappers

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte asynchronous global -> shared copies (cp.async, L2 only) and their groups.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Programmatic dependent launch.  A kernel launched with the programmatic-serialisation
// attribute (launch_kernel(pdl = true)) may be scheduled while its predecessor in the stream is
// still running: griddep_wait blocks until that predecessor has completed and its writes are
// visible (a no-op for a kernel launched without the attribute), and griddep_launch_dependents
// lets the next such kernel be scheduled.  Every kernel a launcher may launch with the
// attribute calls griddep_wait before it touches global memory.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_kernel(bool pdl, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                 cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wall-clock budget of one barrier wait.  Every wait in these kernels is bounded: on
// expiry (or when another warp already reported an error) the waiter records `code` in
// the device error word and returns false, and the caller unwinds.
constexpr uint64_t kWaitBudgetNs = 2000000000ull;  // 2 s

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    uint32_t spins = 0;
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((++spins & 63u) == 0) {
            if (*(volatile int*)err != 0) return false;
            if (globaltimer_ns() - t0 > kWaitBudgetNs) {
                atomicOr(err, code);
                return false;
            }
        }
    }
}

// Time-bounded wait that ignores the error word: used only to let copies already in
// flight land before a CTA exits.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(bar, parity))
        if (globaltimer_ns() - t0 > kWaitBudgetNs) return;
}

// Non-suspending test of a barrier phase.
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded busy-poll wait, for a latency-critical single thread (the MMA issuer): it never
// suspends, so it observes a phase completion without a wake-up delay.
__device__ __forceinline__ bool mbar_wait_poll(uint64_t* bar, uint32_t parity, int* err, int code) {
    if (mbar_test_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    uint32_t spins = 0;
    while (true) {
        if (mbar_test_wait(bar, parity)) return true;
        if ((++spins & 255u) == 0) {
            if (*(volatile int*)err != 0) return false;
            if (globaltimer_ns() - t0 > kWaitBudgetNs) {
                atomicOr(err, code);
                return false;
            }
        }
    }
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Orders this thread's earlier generic-proxy observations of global memory (e.g. data that
// another GPU stored, published by a flag this thread acquired) before its later
// async-proxy (TMA) reads of global memory.
__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// System-scope flag accesses (flags that other GPUs write or read over NVLink).
__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys_u32(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// CTA-scope counter in shared memory: release-add by producers, acquire-load by a poller.
__device__ __forceinline__ void red_release_cta_add(uint32_t* p, uint32_t v) {
    asm volatile("red.release.cta.shared::cta.add.u32 [%0], %1;" ::"r"(smem_u32(p)), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_cta_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)) : "memory");
    return v;
}

// Named barrier over `n` threads (a multiple of 32) of this CTA.
__device__ __forceinline__ void named_bar_sync(int id, int n) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// 2-D tiled TMA load (no multicast) completing on `bar`.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}

// 2-D tiled TMA load into this CTA's shared memory whose completion is counted on a
// barrier of either CTA of the 2-SM pair (`bar_cluster`: shared::cluster address).  No
// multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map,
                                                 uint32_t bar_cluster, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1)
        : "memory");
}

// 1-D bulk copy global -> shared (16-byte aligned, size multiple of 16), no multicast.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// ---- tcgen05 (5th-generation tensor core, tensor memory)

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (fp16 in, fp32 accumulate).
__device__ __forceinline__ void mma_f16_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                           uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrives once on `bar` when every tcgen05.mma this thread issued before it completes.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns; thread i of the warp gets lane (base + i).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, "
        "[%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor for a K-major operand in the 128-byte swizzle layout:
// 8-row x 128-byte atoms, atoms of consecutive row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);  // start address
    d |= static_cast<uint64_t>(1) << 16;                  // leading byte offset (16 B)
    d |= static_cast<uint64_t>(1024 >> 4) << 32;          // stride byte offset
    d |= static_cast<uint64_t>(1) << 46;                  // descriptor version (sm_100)
    d |= static_cast<uint64_t>(2) << 61;                  // SWIZZLE_128B
    return d;
}

// Instruction descriptor, kind::f16: fp16 A and B (both K-major), fp32 D, M x N.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N) {
    return (1u << 4)                                  // D format f32
           | (0u << 7) | (0u << 10)                   // A, B format f16
           | (static_cast<uint32_t>(N >> 3) << 17)    // N / 8
           | (static_cast<uint32_t>(M >> 4) << 24);   // M / 16
}

// Byte offset of 16-byte chunk `c` (0..7) of row `r` inside a 128B-swizzled K-major tile.
__device__ __forceinline__ uint32_t sw128_offset(uint32_t r, uint32_t c) {
    return r * 128u + ((c ^ (r & 7u)) << 4);
}


// ---- cluster / 2-SM (cta_group::2) helpers

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// All threads of both CTAs of the cluster: release this CTA's prior shared-memory writes
// (barrier initialisation) to the peer and wait for the peer.
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// shared::cluster address of `p` (a shared::cta variable) in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}

// Arrive on a barrier of a (possibly remote) CTA of the cluster, given its shared::cluster
// address.  Default (CTA-scope release) semantics, as CUTLASS's cluster barriers use: the
// consumer of the data is the tensor core, ordered by fence.proxy.async on the writer and
// tcgen05.fence::after_thread_sync on the issuer.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait with cluster-scope acquire (arrivals come from the peer CTA too).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int* err, int code) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    uint32_t spins = 0;
    while (true) {
        if (mbar_try_wait_cluster(bar, parity)) return true;
        if ((++spins & 63u) == 0) {
            if (*(volatile int*)err != 0) return false;
            if (globaltimer_ns() - t0 > kWaitBudgetNs) {
                atomicOr(err, code);
                return false;
            }
        }
    }
}

__device__ __forceinline__ void tmem_alloc_2sm(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish_2sm() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_2sm(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

// Pair MMA issued by the leader CTA: A rows 0..M/2-1 and B rows 0..N/2-1 from this CTA's
// shared memory, the other halves from the peer at the same offsets; each CTA's tensor
// memory receives its M/2 accumulator rows.
__device__ __forceinline__ void mma_f16_ss_2sm(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                               uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrives on `bar` (same offset) in every CTA of `cta_mask` once the pair MMAs this thread
// issued complete.
__device__ __forceinline__ void mma_commit_2sm_mc(uint64_t* bar, uint16_t cta_mask) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
        " [%0], %1;" ::"r"(smem_u32(bar)),
        "h"(cta_mask)
        : "memory");
}

__device__ __forceinline__ void mma_commit_2sm(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

// ------------------------------------------------------------------ small helpers

__device__ __forceinline__ float silu_mul(float g, float u) {
    // silu(g) * u with silu(g) = g * (1 / (1 + e^-g)), as src/rms_norm.cpp:73-74.
    const float s = g * (1.0f / (1.0f + expf(-g)));
    return s * u;
}

}  // namespace hymoe
