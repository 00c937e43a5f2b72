// pd_tcgen05.cuh — 5th-generation tensor-core (tcgen05) primitives for sm_100a.
//
// Inline PTX for the MQA decode engine (pd_decode_mqa.cuh): tensor-memory
// allocation, single-thread MMAs with shared-memory operand descriptors and
// FP32 accumulators in tensor memory, commits onto mbarriers, and warp-wide
// tensor-memory loads and stores.  Bit layouts follow the PTX ISA's
// "shared memory descriptor" and "instruction descriptor" tables for
// tcgen05.mma (the same fields CUTLASS names in cute/arch/mma_sm100_desc.hpp).
#pragma once

#include <stdint.h>

namespace pd {
namespace tc {

// ---------------------------------------------------------------- descriptors
// Layout field of a shared-memory descriptor (bits 61-63).
constexpr uint64_t kNoSwizzle = 0;    // 8-row x 16-byte core matrices
constexpr uint64_t kSwizzle128 = 2;   // 8-row x 128-byte atoms, 16-byte chunks XORed by row

// Shared-memory matrix descriptor: start address >> 4 (bits 0-13), leading
// byte offset >> 4 (16-29), stride byte offset >> 4 (32-45), descriptor
// version 1 (46-47), base offset 0 (49-51: every swizzle atom we use is
// 1024-byte aligned), layout (61-63).
//   K-major, 128-byte swizzle: rows of 128 B, 8-row groups `sbo` apart; the
//     K step inside an atom advances the start address (lbo unused).
//   K-major, no swizzle: 8x8 core matrices of 128 contiguous bytes; `lbo` =
//     distance between K-adjacent core matrices, `sbo` = between 8-row groups.
//   MN-major, 128-byte swizzle: 64-element (128 B) MN rows, one per K index;
//     `lbo` = distance between 64-wide MN blocks, `sbo` = between 8-row K groups.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo, uint64_t layout) {
    return uint64_t((addr >> 4) & 0x3fffu) | (uint64_t((lbo >> 4) & 0x3fffu) << 16) |
           (uint64_t((sbo >> 4) & 0x3fffu) << 32) | (1ull << 46) | (layout << 61);
}

// Instruction descriptor of kind::f16 with FP16 A and B and an FP32
// accumulator: D format F32 (bits 4-5 = 1), A and B format F16 (7-9, 10-12 =
// 0), A / B major (15 / 16: 0 K-major, 1 MN-major), N >> 3 (17-22), M >> 4 (24-28).
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N, bool a_mn_major, bool b_mn_major) {
    return (1u << 4) | (uint32_t(a_mn_major) << 15) | (uint32_t(b_mn_major) << 16) |
           (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}

// ---------------------------------------------------------------- tensor memory
// Warp-wide: allocate `cols` columns (a power of two >= 32) of this CTA's
// tensor memory; the address lands in shared memory at `dst`.
__device__ __forceinline__ void alloc(uint32_t dst, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst), "r"(cols)
                 : "memory");
}

__device__ __forceinline__ void relinquish_alloc_permit() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void dealloc(uint32_t taddr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}

// Ordering of tcgen05 operations around thread synchronisation (mbarrier
// waits, bar.sync): `before` ahead of the signalling side, `after` behind the
// waiting side.
__device__ __forceinline__ void fence_before_sync() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void fence_after_sync() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Generic-proxy shared-memory writes (st.shared) made visible to the async
// proxy that tcgen05.mma reads its operands through.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- MMA
// D[tmem] (+)= A[smem] * B[smem], issued by one thread; accumulate = 0
// overwrites D.
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// One arrive on the mbarrier once every MMA this thread issued so far has
// completed (and its operands may be overwritten).
__device__ __forceinline__ void commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

// ---------------------------------------------------------------- loads / stores
// Warp-wide, 16 lanes x 32 columns: thread t gets lane (t % 16) of the
// warp's 32-lane sub-partition, columns col + 16 * (t / 16) + [0, 16).
__device__ __forceinline__ void ld_16x32bx2_x16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.16x32bx2.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16], 16;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}

__device__ __forceinline__ void st_16x32bx2_x16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.16x32bx2.x16.b32 [%0], 16, "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

__device__ __forceinline__ void wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

}  // namespace tc
}  // namespace pd
