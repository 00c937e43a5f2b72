// pd_device.cuh — sm_100a device primitives used by the decode kernels.
//
// Thin inline-PTX wrappers: shared-memory mbarriers (with bounded waits),
// tiled TMA loads (cp.async.bulk.tensor, no multicast), ldmatrix / movmatrix
// and the m16n8k16 FP16 tensor-core MMA with FP32 accumulation.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace pd {

constexpr unsigned kFullMask = 0xffffffffu;
// A barrier that has not completed after this long means the pipeline is
// broken; the kernel records PD_DEVERR_TIMEOUT and unwinds instead of hanging.
constexpr unsigned long long kWaitTimeoutNs = 2000000000ull;
// A CTA waiting at a plain launch's grid barrier leaves after this long if a
// CTA of the launch has not started (grid_arrive).
constexpr uint32_t kBarrierLeaveNs = 50000u;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_init_fence() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}

// Non-blocking test of the same (never suspends the thread).
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}

// Wait for the phase with the given parity to complete; false after the timeout.
// A phase that has completed already is seen by the non-blocking test.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity,
                                          unsigned long long timeout_ns = kWaitTimeoutNs) {
    if (mbar_test_wait(bar, parity)) return true;
    const unsigned long long start = global_ns();
    for (;;) {
#pragma unroll 1
        for (int i = 0; i < 32; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (global_ns() - start > timeout_ns) return false;
    }
}

// ---------------------------------------------------------------- clusters
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Every thread of every CTA of the cluster arrives (releasing its earlier
// writes, distributed shared memory included) and waits for all the others.
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

// Generic address of the same shared-memory location in CTA `rank` of this
// cluster (ordinary loads and stores reach it).
template <typename P>
__device__ __forceinline__ P *cluster_map(P *p, uint32_t rank) {
    uint64_t r;
    asm volatile("mapa.u64 %0, %1, %2;" : "=l"(r) : "l"(reinterpret_cast<uint64_t>(p)), "r"(rank));
    return reinterpret_cast<P *>(r);
}

// ---------------------------------------------------------------- TMA
// 5-D tiled load into CTA shared memory, completion counted on `bar`.
__device__ __forceinline__ void tma_load_5d(uint32_t dst, const CUtensorMap *map, int c0, int c1, int c2,
                                            int c3, int c4, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void tma_prefetch_descriptor(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ int4 shfl_int4(int4 v, int src) {
    return make_int4(__shfl_sync(kFullMask, v.x, src), __shfl_sync(kFullMask, v.y, src),
                     __shfl_sync(kFullMask, v.z, src), __shfl_sync(kFullMask, v.w, src));
}

// ---------------------------------------------------------------- grid barrier
__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Grid-wide barrier on counters that only ever grow (no reset between
// launches, so CUDA-graph replays work).  `count` holds the arrivals in its
// low 54 bits: each of the `ctas` CTAs adds one per launch, and this launch's
// barrier is complete once they reach the next multiple of `ctas` above the
// CTA's own ticket.  `started` gets one per CTA per launch as the CTA starts.
//
// Under a cooperative launch (leave_mode 0) every CTA is resident and a CTA
// simply waits.  A plain launch does not promise that: an SM partition or a
// kernel in another stream can hold back some CTAs until others exit.  So with
// leave_mode 1 a CTA that has waited leave_ns while `started` shows a CTA of
// this launch not yet started leaves instead: it sets its bit in `left` and
// adds 2^54 to `count`.  The CTA whose arrival completes the barrier reads the
// number that left in the high bits of its ticket and merges their shares as
// well as its own; a CTA whose leave comes after that arrival takes it back
// and stays.  leave_mode 2 leaves at the first wait (tests the path).
enum : int { kBarrierGo = 0, kBarrierGoMergeLeft = 1, kBarrierLeft = 2, kBarrierTimeout = 3 };
constexpr int kArrivalBits = 54;
constexpr unsigned long long kArrivalMask = (1ull << kArrivalBits) - 1;
constexpr unsigned long long kLeftUnit = 1ull << kArrivalBits;

struct GridBarrier {
    unsigned long long *count;     // arrivals (low 54 bits), CTAs that left (high 10 bits)
    unsigned long long *started;   // CTAs started, over all launches
    unsigned long long *left;      // one bit per CTA that left this launch's barrier (1024 bits)
    uint32_t leave_mode;           // 0 wait, 1 leave after leave_ns if a CTA has not started, 2 leave at once
    uint32_t leave_ns;
};

// Called by one thread per CTA after the CTA's own barrier; its writes before
// the call are visible to every CTA that returns kBarrierGo*.  `*left_count`
// gets the number of CTAs that left (kBarrierGoMergeLeft only).
__device__ __forceinline__ int grid_arrive(const GridBarrier &gb, unsigned ctas, unsigned cta,
                                           unsigned *left_count,
                                           unsigned long long timeout_ns = kWaitTimeoutNs) {
    __threadfence();
    const unsigned long long old = atomicAdd(gb.count, 1ull);
    const unsigned long long target = ((old & kArrivalMask) / ctas + 1) * ctas;
    if ((old & kArrivalMask) + 1 == target) {
        __threadfence();
        *left_count = unsigned(old >> kArrivalBits);
        return *left_count ? kBarrierGoMergeLeft : kBarrierGo;
    }
    const unsigned long long start = global_ns();
    for (;;) {
        if ((ld_acquire_u64(gb.count) & kArrivalMask) >= target) break;
        const unsigned long long t = global_ns() - start;
        if (gb.leave_mode == 2 ||
            (gb.leave_mode == 1 && t > gb.leave_ns && ld_acquire_u64(gb.started) < target)) {
            const unsigned long long bit = 1ull << (cta & 63);
            atomicOr(gb.left + cta / 64, bit);
            __threadfence();
            const unsigned long long o = atomicAdd(gb.count, kLeftUnit);
            if ((o & kArrivalMask) < target) return kBarrierLeft;
            // the barrier completed first: take the leave back and stay
            atomicAdd(gb.count, 0ull - kLeftUnit);
            atomicAnd(gb.left + cta / 64, ~bit);
            break;
        }
        if (t > timeout_ns) return kBarrierTimeout;
    }
    __threadfence();
    return kBarrierGo;
}

// Release at system scope: the caller's earlier writes (and those it has
// synchronised with) become visible to other GPUs before its later stores.
__device__ __forceinline__ void fence_release_sys() {
    asm volatile("fence.acq_rel.sys;" ::: "memory");
}

// ---------------------------------------------------------------- named barrier
__device__ __forceinline__ void named_barrier_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---------------------------------------------------------------- tensor-core fragments
__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

// Transpose an 8x8 b16 matrix held one row-pair per thread (ldmatrix fragment layout).
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t a) {
    uint32_t d;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
    return d;
}

// D += A(16x16, row) * B(16x8, col); FP16 inputs, FP32 accumulators.
__device__ __forceinline__ void mma_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
}

__device__ __forceinline__ float2 unpack_half2(uint32_t v) {
    __half2 h = *reinterpret_cast<__half2 *>(&v);
    return __half22float2(h);
}

__device__ __forceinline__ float4 lds_f4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr));
    return v;
}

__device__ __forceinline__ float2 lds_f2(uint32_t addr) {
    float2 v;
    asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr));
    return v;
}

// Offset of the 16-byte chunk `chunk` (counted along the row) of row `row`
// inside a block written by TMA with CU_TENSOR_MAP_SWIZZLE_128B: each 128-byte
// box of the row is ROWS rows x 128 B, and inside every 8-row / 1024-byte atom
// the chunk index is XORed with (row % 8).  Blocks are 1024-byte aligned.
template <int ROWS>
__device__ __forceinline__ uint32_t swz128(int row, int chunk) {
    const int box = chunk >> 3;
    const int c = (chunk & 7) ^ (row & 7);
    return static_cast<uint32_t>(box * ROWS * 128 + row * 128 + (c << 4));
}

}  // namespace pd
