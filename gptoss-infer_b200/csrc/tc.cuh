// sm_100a tensor-core plumbing: mbarriers with bounded waits, TMA and bulk copies (no multicast anywhere), TMEM
// allocation, tcgen05 block-scaled MMA (kind::mxf4, e2m1 x e2m1 with E8M0 scales per 32 elements), tcgen05.cp of
// scale factors and tcgen05.ld of accumulators.
//
// Shared-memory operand layout (both A = weights and B = activations, K-major): the 128-byte swizzled canonical
// layout. A tile of R rows and 128 bytes of K (256 e2m1 values) is R*128 bytes; row r starts at r*128 and its 16-byte
// chunk j sits at chunk position j ^ (r % 8). Tiles start on 1024-byte boundaries. One MMA consumes K = 64 values
// (32 bytes) per row, so the descriptor of MMA j of a tile starts 32*j bytes in.
//
// Scale-factor chunk layout (one per 128 rows x 128 K, i.e. 4 scale bytes per row): 512 bytes, byte
// (r % 32) * 16 + (r / 32) * 4 + kb for row r and k-block kb. tcgen05.cp 32x128b.warpx4 copies it to 4 TMEM columns
// (every lane quadrant gets the same 32 x 16 bytes); MMA j of the chunk reads scale bytes 2j and 2j+1 (sf_id 2j).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

namespace gpt {
namespace tc {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// One lane of a converged warp (the warp must be converged at the call).
__device__ __forceinline__ bool elect_one() {
    uint32_t pred;
    asm volatile("{\n\t.reg .pred p;\n\telect.sync _|p, 0xffffffff;\n\tselp.u32 %0, 1, 0, p;\n\t}" : "=r"(pred));
    return pred != 0;
}

// ---------------------------------------------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                     smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
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

// Non-suspending probe of a phase (mbarrier.test_wait): cheaper than try_wait when the phase has already completed.
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

// Every wait is bounded: mbarrier.try_wait suspends the thread in hardware until the phase completes or a short
// system-defined window passes, so the loop needs no sleep of its own (one would only delay the wake-up); after
// kSpinLimit unsuccessful tries (well over a second) the wait gives up, records `where` in *err (first error wins)
// and returns false; callers then skip the dependent work, drain and exit. A phase that has already completed is
// caught by one test_wait first.
constexpr uint32_t kSpinLimit = 1u << 24;

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int where) {
    if (mbar_test_wait(bar, parity)) return true;
    for (uint32_t i = 0; i < kSpinLimit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    if (err) atomicCAS(err, 0, where);
    return false;
}

// Bounded wait with a sleep between tries, for threads whose wake-up latency does not matter (they would otherwise
// take issue slots from the producer and MMA threads of their own and co-resident CTAs while they wait).
__device__ __forceinline__ bool mbar_wait_sleepy(uint64_t* bar, uint32_t parity, int* err, int where, uint32_t ns) {
    for (uint32_t i = 0; i < kSpinLimit / 16; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        __nanosleep(ns);
    }
    if (err) atomicCAS(err, 0, where);
    return false;
}

// ---------------------------------------------------------------------------------------------------- copies
// 1-D bulk copy global -> shared completing on an mbarrier (both addresses 16-byte aligned, size a multiple of 16).
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(smem_dst)),
        "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// 2-D tiled TMA load (no multicast); x is the innermost coordinate in elements, y the row.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const void* tmap, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(smem_dst)),
        "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// 3-D tiled TMA load (no multicast): x innermost (elements), y row, z matrix.
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const void* tmap, int x, int y, int z, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(smem_u32(smem_dst)),
        "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

// L2 prefetches (no shared memory, no completion): a 3-D tensor box, and a contiguous range (16-byte aligned, size a
// multiple of 16).
__device__ __forceinline__ void tma_prefetch_l2_3d(const void* tmap, int x, int y, int z) {
    asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(tmap), "r"(x), "r"(y),
                 "r"(z)
                 : "memory");
}
__device__ __forceinline__ void bulk_prefetch_l2(const void* gsrc, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(gsrc), "r"(bytes) : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// 16-byte asynchronous global -> shared copy through L2 (generic proxy; both addresses 16-byte aligned). Many can be
// in flight per thread without holding registers; cp_async_wait_all waits for all of this thread's copies.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Generic-proxy shared-memory writes -> visible to the async proxy (tensor core, tcgen05.cp).
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ---------------------------------------------------------------------------------------------------- TMEM
// Allocation is warp-wide; the base address is written to shared memory.
__device__ __forceinline__ void tmem_alloc(uint32_t* holder, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(holder)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// ---------------------------------------------------------------------------------------------------- descriptors
// Shared-memory matrix descriptor (sm_100 format, version 1): start, leading and stride byte offsets in 16-byte
// units, layout type in bits 61-63 (0 = no swizzle, 2 = 128-byte swizzle).
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                              uint32_t layout) {
    uint64_t d = 0;
    d |= uint64_t((saddr >> 4) & 0x3FFFu);
    d |= uint64_t((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= uint64_t((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= uint64_t(1) << 46;                                   // descriptor version for sm_100
    d |= uint64_t(layout & 7u) << 61;
    return d;
}

// K-major operand in the 128-byte swizzled layout: 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) { return smem_desc(saddr, 16, 1024, 2); }

// K-major operand in the 64-byte swizzled layout (64-byte rows: 64 bytes of K per row, 8-row atoms of 512 bytes; 16-byte
// chunk j of row r at chunk position j ^ ((r / 2) % 4)), as a TMA box of 64-byte rows with the 64-byte swizzle writes
// it. One MMA reads 32 bytes of K per row, so MMA j of a 64-byte row starts 32*j bytes in.
__device__ __forceinline__ uint64_t desc_sw64(uint32_t saddr) { return smem_desc(saddr, 16, 512, 4); }

// The same layout with all 8-row groups at one address (stride 0): an 8-row operand (1 KB per 128 bytes of K) read as
// M = 128 rows, rows r and r + 8 identical; the accumulator rows repeat with period 8.
__device__ __forceinline__ uint64_t desc_sw128_rows8(uint32_t saddr) { return smem_desc(saddr, 16, 0, 2); }

// Scale-factor chunk source for tcgen05.cp 32x128b: 32 rows of 16 bytes, contiguous (core matrices of 8 rows x 16
// bytes, 128 bytes apart), no swizzle.
__device__ __forceinline__ uint64_t desc_sf_chunk(uint32_t saddr) { return smem_desc(saddr, 0, 128, 0); }

// The same copy from an 8-row chunk (128 bytes, rows 0-7): all four 8-row groups read the same 128 bytes, so TMEM lanes
// l and l + 8 receive the same scales (the scales of an 8-row operand read as 128 rows).
__device__ __forceinline__ uint64_t desc_sf_chunk8(uint32_t saddr) { return smem_desc(saddr, 0, 0, 0); }

// Instruction descriptor of tcgen05.mma kind::mxf4 (block 32, E8M0 scales, K = 64, both operands K-major e2m1):
// b_sf_id bits 4-5, a/b format (E2M1 = 1) bits 7-9 / 10-12, N >> 3 bits 17-22, scale format E8M0 bit 23,
// M >> 4 bits 24-28, a_sf_id bits 29-30.
__host__ __device__ constexpr uint32_t idesc_mxf4(int M, int N, uint32_t a_sf_id, uint32_t b_sf_id) {
    return (b_sf_id << 4) | (1u << 7) | (1u << 10) | (uint32_t(N >> 3) << 17) | (1u << 23) |
           (uint32_t(M >> 4) << 24) | (a_sf_id << 29);
}

// D[tmem] (+)= A[smem] x B[smem]^T with per-32 scales from TMEM. Issued by one thread.
__device__ __forceinline__ void mma_mxf4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t sfa_tmem, uint32_t sfb_tmem, bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(uint32_t(accumulate)), "r"(sfa_tmem), "r"(sfb_tmem)
        : "memory");
}

// Copy one 512-byte scale chunk (32 rows x 16 bytes) to 4 TMEM columns, replicated into all 4 lane quadrants.
__device__ __forceinline__ void tmem_cp_sf(uint32_t tmem_col, uint64_t sdesc) {
    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(tmem_col), "l"(sdesc) : "memory");
}

// Arrive on an mbarrier once every previously issued tcgen05 operation of this thread has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// Warp reads 32 lanes (its quadrant) x 8 consecutive fp32 columns: thread t gets lane (quadrant*32 + t).
__device__ __forceinline__ void tmem_ld_32x32b_x8(uint32_t taddr, float* v) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
// Warp reads 32 lanes (its quadrant) x 16 / 32 consecutive fp32 columns: thread t gets lane (quadrant*32 + t).
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Byte offset of (row, byte-in-128) inside a 128-byte-swizzled K-major tile.
__host__ __device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t kbyte) {
    return row * 128u + ((((kbyte >> 4) ^ (row & 7u)) << 4) | (kbyte & 15u));
}

// Byte offset of (row, k-block) inside a 512-byte scale chunk covering 128 rows x 4 k-blocks.
__host__ __device__ __forceinline__ uint32_t sf_offset(uint32_t row, uint32_t kb) {
    return (row & 31u) * 16u + (row >> 5) * 4u + kb;
}

}  // namespace tc
}  // namespace gpt
