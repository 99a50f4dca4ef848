// xm_umma.cuh -- thin inline-PTX layer over the sm_100a 5th-generation tensor
// core (tcgen05): shared-memory matrix descriptors, instruction descriptors,
// TMEM allocation, MMA issue / commit and TMEM loads, bounded mbarrier waits
// and TMA tensor loads. Written from the PTX ISA (tcgen05, mbarrier and
// cp.async.bulk.tensor) and the descriptor bit layouts documented in
// CUTLASS's cute/arch/mma_sm100_desc.hpp.
//
// Operand tiles use the SWIZZLE_NONE canonical layouts, built from "core
// matrices" of 8 rows x 16 bytes stored contiguously (128 B):
//   K-major  (rows = M or N, K contiguous): core (r, c) covers rows 8r..8r+7 and
//            K elements [c*16B, c*16B+16B); its byte offset is r*SBO + c*LBO.
//   MN-major (rows = K, M/N contiguous):    core (r, c) covers K rows 8r..8r+7
//            and M/N elements [c*16B, ...); its byte offset is c*SBO + r*LBO.
// In both, SBO steps along M/N and LBO steps along K (descriptor fields
// stride_byte_offset / leading_byte_offset).
#pragma once

#include <cstdint>

namespace xm {
namespace umma {

// ---------------------------------------------------------------- descriptors

__device__ __forceinline__ uint64_t smem_desc(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1u) << 46;  // descriptor version for sm_100
    // base_offset = 0, lbo_mode = 0, layout_type = SWIZZLE_NONE (0)
    return d;
}

// As smem_desc, for the 128-byte-swizzled canonical layouts (layout type 2):
// K-major: rows of 64 bf16 (128 bytes), 16-byte chunk j of row r at j ^ (r & 7),
// 8-row groups `sbo` bytes apart, `lbo` unused; a K step inside the 128-byte
// row advances the start address. MN-major: 64-element MN atoms `lbo` bytes
// apart, 8-row K groups `sbo` bytes apart. Atoms 1024-byte aligned.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    return smem_desc(smem_addr, lbo_bytes, sbo_bytes) | (static_cast<uint64_t>(2u) << 61);
}

// kind::f16 instruction descriptor: D f32, A/B bf16, dense.
// a_mn / b_mn: operand stored MN-major (else K-major).
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N, bool a_mn, bool b_mn) {
    return (1u << 4)                           // c_format = F32
           | (1u << 7)                         // a_format = BF16
           | (1u << 10)                        // b_format = BF16
           | ((a_mn ? 1u : 0u) << 15)          // a_major
           | ((b_mn ? 1u : 0u) << 16)          // b_major
           | (static_cast<uint32_t>(N >> 3) << 17)  // n_dim
           | (static_cast<uint32_t>(M >> 4) << 24); // m_dim
}

// ---------------------------------------------------------------- TMEM

// Allocate `ncols` TMEM columns (power of two >= 32); executed by one full warp.
__device__ __forceinline__ void tmem_alloc(uint32_t *smem_dst, uint32_t ncols) {
    const uint32_t dst = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(dst), "r"(ncols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols));
}

__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

// Generic-proxy shared-memory writes -> visible to the tensor core (async proxy).
__device__ __forceinline__ void fence_smem_to_async() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }

// ---------------------------------------------------------------- MMA

// D[tmem] (+)= A[smem] * B[smem], issued by a single thread.
__device__ __forceinline__ void mma_bf16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            bool accumulate) {
    asm volatile(
        "{\n\t"
        ".reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t"
        "}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate ? 1u : 0u), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}

// Arrive on `mbar` once every MMA previously issued by this thread has completed.
__device__ __forceinline__ void mma_commit(uint64_t *mbar) {
    const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(mbar));
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(a)
                 : "memory");
}

// ---------------------------------------------------------------- mbarrier

__device__ __forceinline__ void mbar_init(uint64_t *mbar, uint32_t count) {
    const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(mbar));
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(a), "r"(count));
}

// Wait for the phase with parity `parity` to complete. Bounded: after
// `max_polls` unsuccessful polls the wait gives up and returns false, so a
// missing arrival can never hang the GPU; the caller records the failure.
__device__ __forceinline__ bool mbar_wait(uint64_t *mbar, uint32_t parity, uint32_t max_polls = (1u << 22)) {
    const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(mbar));
    for (uint32_t i = 0; i < max_polls; ++i) {
        uint32_t done;
        asm volatile(
            "{\n\t"
            ".reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t"
            "}\n"
            : "=r"(done)
            : "r"(a), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}

// As mbar_wait, but each poll suspends the thread in hardware until the phase
// completes or `suspend_ns` nanoseconds pass (a waiter that does not compete
// for issue slots with the warps doing the work); at most `max_polls` polls.
__device__ __forceinline__ bool mbar_wait_suspend(uint64_t *mbar, uint32_t parity, uint32_t suspend_ns,
                                                  uint32_t max_polls) {
    const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(mbar));
    for (uint32_t i = 0; i < max_polls; ++i) {
        uint32_t done;
        asm volatile(
            "{\n\t"
            ".reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t"
            "}\n"
            : "=r"(done)
            : "r"(a), "r"(parity), "r"(suspend_ns)
            : "memory");
        if (done) return true;
    }
    return false;
}

// Expect `bytes` more transaction bytes on `mbar` and arrive once (the phase
// completes when the arrival count and the bytes have both been reached).
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *mbar, uint32_t bytes) {
    const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(mbar));
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(a), "r"(bytes) : "memory");
}

// ---------------------------------------------------------------- TMA

// Tiled 3-D tensor copy global -> this CTA's shared memory (no multicast),
// completing `bytes` of transactions on `mbar`. `tmap` is the address of a
// CUtensorMap in kernel-parameter (grid-constant) memory; c0 is the innermost
// coordinate, in elements (c0 * element size must be a multiple of 16 bytes).
__device__ __forceinline__ void tma_load_3d(void *smem_dst, const void *tmap, int c0, int c1, int c2,
                                            uint64_t *mbar) {
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
    const uint32_t b = static_cast<uint32_t>(__cvta_generic_to_shared(mbar));
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];\n" ::"r"(d),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(c2), "r"(b)
        : "memory");
}

// As tma_load_3d, for a 4-dimensional tensor map.
__device__ __forceinline__ void tma_load_4d(void *smem_dst, const void *tmap, int c0, int c1, int c2, int c3,
                                            uint64_t *mbar) {
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
    const uint32_t b = static_cast<uint32_t>(__cvta_generic_to_shared(mbar));
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
        "%5}], [%6];\n" ::"r"(d),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(b)
        : "memory");
}

// Untiled bulk copy global -> this CTA's shared memory (no multicast),
// completing `bytes` of transactions on `mbar`. Both addresses 16-byte aligned,
// `bytes` a multiple of 16.
__device__ __forceinline__ void bulk_load(void *smem_dst, const void *gmem_src, uint32_t bytes, uint64_t *mbar) {
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
    const uint32_t b = static_cast<uint32_t>(__cvta_generic_to_shared(mbar));
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(d),
        "l"(reinterpret_cast<uint64_t>(gmem_src)), "r"(bytes), "r"(b)
        : "memory");
}

// Plain arrival on `mbar` (count 1).
__device__ __forceinline__ void mbar_arrive(uint64_t *mbar) {
    const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(mbar));
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(a) : "memory");
}

// ---------------------------------------------------------------- TMEM -> registers

// Each thread of warp w reads TMEM lane 32*(w%4) + lane, 16 consecutive 32-bit
// columns starting at the column of `taddr` (lane field must be 32*(w%4)).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
        "%14, %15}, [%16];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// As tmem_ld16, 8 consecutive columns.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }

// Registers -> TMEM: the inverse of tmem_ld16 (same lane rule); complete with tmem_wait_st.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16};\n" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
        "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
        "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
        "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
        "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
        : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }

}  // namespace umma
}  // namespace xm
