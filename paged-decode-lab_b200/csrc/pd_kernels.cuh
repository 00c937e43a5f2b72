// pd_kernels.cuh — launch shapes of the decode kernel and the per-shape entry tables.
//
// Each pd_kernels_<dtype>_d<D>_t<T>.cu instantiates the kernels of one
// (dtype, head_dim, page_size) triple, so the library's ~120 kernels compile
// in parallel translation units.
#pragma once

#include "pd_decode_kernel.cuh"
#include "pd_decode_mqa.cuh"
#include "pd_kernels_select.hpp"

namespace pd {

using KernelFn = void (*)(const CUtensorMap, const CUtensorMap, const DecodeArgs);

struct KernelEntry {
    KernelFn fn;
    int threads;
    size_t smem;
    int consumers;
    int slots;
    int nsub;       // sub-pipelines: partial slots each segment's warps write (1 when folded)
};

// Shape of one kernel: HG KV heads per page tile and NSUB sub-pipelines of
// HG consumer warps each.  NSUB starts at max_sub_pipelines() and halves
// until at least NSUB page tiles fit in shared memory; the ring then takes as
// many slots as fit, rounded down to a multiple of NSUB.
template <typename Elt, int D, int T, int GT, int HG, int NSUB>
struct RingFit {
    using Probe = KernelShape<Elt, D, T, GT, HG, NSUB, NSUB>;
    static constexpr size_t FIXED = Probe::SMEM - Probe::RING - Probe::BARS - Probe::FLAGS;
    static constexpr size_t AVAIL = FIXED + 1024 < 232448 ? 232448 - FIXED - 1024 : 0;
    static constexpr int FIT = int(AVAIL / (Probe::TILE_BYTES + 20));
    static constexpr int CAP = FIT > 32 ? 32 : FIT;
    static constexpr int SLOTS = CAP / NSUB * NSUB;
};

template <typename Elt, int D, int T, int GT, int HG, int NSUB>
struct PickSub {
    static constexpr int value =
        (NSUB == 1 || RingFit<Elt, D, T, GT, HG, NSUB>::SLOTS >= NSUB)
            ? NSUB
            : PickSub<Elt, D, T, GT, HG, (NSUB > 1 ? NSUB / 2 : 1)>::value;
};
template <typename Elt, int D, int T, int GT, int HG>
struct PickSub<Elt, D, T, GT, HG, 1> {
    static constexpr int value = 1;
};

template <typename Elt, int D, int T, int GT, int HG>
struct LaunchShape {
    static constexpr int NSUB = PickSub<Elt, D, T, GT, HG, max_sub_pipelines(sizeof(Elt), HG, GT, D, T)>::value;
    static constexpr int SLOTS = RingFit<Elt, D, T, GT, HG, NSUB>::SLOTS;
    static_assert(SLOTS >= NSUB && SLOTS >= 1, "a page tile does not fit in shared memory");
};

template <typename Elt, int D, int T, int GT, int HG, int MODE>
KernelEntry make_entry() {
    using L = LaunchShape<Elt, D, T, GT, HG>;
    using S = KernelShape<Elt, D, T, GT, HG, L::NSUB, L::SLOTS>;
    return {&paged_decode_kernel<Elt, D, T, GT, HG, L::NSUB, L::SLOTS, MODE>, S::THREADS, S::SMEM, S::NC,
            L::SLOTS, S::FOLD ? 1 : L::NSUB};
}

// KV heads per tile are instantiated while an FP16 page tile (K + V of HG
// heads) stays within 64 KiB, so the FP32 tile (twice as large) still fits
// in shared memory, and while a tile has at most 8 consumer warps; the
// planner never asks for more (choose_heads_per_tile).
constexpr bool heads_per_tile_allowed(int D, int T, int GT, int hg) {
    return 4 * D * T * hg <= 65536 && tile_consumers(hg, GT) <= 8;
}

template <typename Elt, int D, int T, int GT, int HG, int MODE>
KernelEntry entry_clamped() {
    if constexpr (HG > 1 && !heads_per_tile_allowed(D, T, GT, HG))
        return entry_clamped<Elt, D, T, GT, HG / 2, MODE>();
    else
        return make_entry<Elt, D, T, GT, HG, MODE>();
}

template <typename Elt, int D, int T, int GT, int MODE>
KernelEntry entry_for_hg(int hg) {
    switch (hg) {
        case 8: return entry_clamped<Elt, D, T, GT, 8, MODE>();
        case 4: return entry_clamped<Elt, D, T, GT, 4, MODE>();
        case 2: return entry_clamped<Elt, D, T, GT, 2, MODE>();
        default: return entry_clamped<Elt, D, T, GT, 1, MODE>();
    }
}

// The tcgen05 kernel (decode only; the gather debug mode keeps the warp-level kernel).
template <int D, int T>
KernelEntry make_mqa_entry() {
    using S = MqaShape<D, T>;
    return {&paged_decode_mqa_kernel<D, T>, S::THREADS, S::SMEM, S::NC, S::VSS * S::NP, 1};
}

template <typename Elt, int D, int T, int MODE>
KernelEntry entry_for(int gt, int hg, int engine) {
    if constexpr (MODE == kModeDecode && std::is_same<Elt, __half>::value) {
        if (engine == kEngineTensorMemory && mqa_tensor_memory_shape(2, hg, gt, D, T)) return make_mqa_entry<D, T>();
    }
    if (MODE == kModeGather || gt == 8) return entry_for_hg<Elt, D, T, 8, MODE>(hg);
    if (gt == 16) return entry_for_hg<Elt, D, T, 16, MODE>(hg);
    return entry_for_hg<Elt, D, T, 32, MODE>(hg);
}

// Merge of the decode kernel's partials, launched programmatically dependent
// on it (PDL) on the same stream (pd_merge.cu).
cudaError_t launch_merge_partials(const DecodeArgs &args, int hg, int gt, int nsub, int D,
                                  cudaStream_t stream);

// Max-corrected merge of [shards, rows, D] shard outputs (pd_merge.cu).
cudaError_t launch_merge_shards(const float *shard_out, const float *shard_stats, int shards, int64_t stride,
                                int64_t rows, int D, float *out, cudaStream_t stream);

// Defined in the per-shape translation units.
KernelEntry kernel_entry_f16_d64_t16(int gt, int hg, int mode, int engine);
KernelEntry kernel_entry_f16_d64_t32(int gt, int hg, int mode, int engine);
KernelEntry kernel_entry_f16_d128_t16(int gt, int hg, int mode, int engine);
KernelEntry kernel_entry_f16_d128_t32(int gt, int hg, int mode, int engine);
KernelEntry kernel_entry_f32_d64_t16(int gt, int hg, int mode, int engine);
KernelEntry kernel_entry_f32_d64_t32(int gt, int hg, int mode, int engine);
KernelEntry kernel_entry_f32_d128_t16(int gt, int hg, int mode, int engine);
KernelEntry kernel_entry_f32_d128_t32(int gt, int hg, int mode, int engine);

}  // namespace pd

#define PD_DEFINE_ENTRY(NAME, ELT, D, T)                                                        \
    namespace pd {                                                                             \
    KernelEntry NAME(int gt, int hg, int mode, int engine) {                                   \
        return mode == kModeDecode ? entry_for<ELT, D, T, kModeDecode>(gt, hg, engine)         \
                                   : entry_for<ELT, D, T, kModeGather>(gt, hg, engine);        \
    }                                                                                          \
    }
