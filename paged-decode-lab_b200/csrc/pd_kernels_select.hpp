// pd_kernels_select.hpp — host-side choice of the KV heads gathered per page tile.
#pragma once

namespace pd {

// Consumer engines of the decode kernels: warp-level (m16n8k16 MMAs or FP32
// FMAs in every consumer warp) or tcgen05 (one thread issues the MMAs into
// tensor memory; pd_decode_mqa.cuh).
enum : int { kEngineWarp = 0, kEngineTensorMemory = 1 };

// Shapes the tcgen05 kernel serves: FP16 group tiles of 32 query heads (groups
// of 17..32 query heads per KV head, MQA-like) over one KV head per page tile.
inline constexpr bool mqa_tensor_memory_shape(int elt, int hg, int gt, int D, int T) {
    return elt == 2 && hg == 1 && gt == 32 && (D == 64 || D == 128) && (T == 16 || T == 32);
}

// Consumer warps reading one page tile: HG KV heads x GT/8 query-head
// slices each.  At most 8.
inline constexpr int tile_consumers(int hg, int gt) { return hg * (gt / 8); }

// Largest KV-head group (1, 2, 4 or 8; dividing kv_heads; at most 8 consumer
// warps per tile) whose page tile (K + V of elt-byte elements) stays within
// `target_bytes`, which is capped at 64 KiB.
inline int choose_heads_per_tile(int elt, int D, int T, int GT, int kv_heads, int target_bytes) {
    const int per_head = 2 * D * elt * T;
    if (target_bytes > 65536) target_bytes = 65536;
    int best = 1;
    for (int hg = 2; hg <= 8; hg *= 2)
        if (kv_heads % hg == 0 && hg * per_head <= target_bytes && tile_consumers(hg, GT) <= 8) best = hg;
    return best;
}

// Sub-pipelines a kernel shape starts from (it may use fewer when its page
// tiles leave room for fewer ring slots); consumer warps are
// tile_consumers * NSUB <= 8.  An FP16 warp folds a 16-token slice of a tile
// in ~450 cycles, so 32 KiB or larger tiles keep up with HBM with one warp per
// (head, query slice) and need no sub-pipelines (a group on one CTA then
// writes its output without a merge); smaller tiles add up to four
// sub-pipelines, within the 8 warps (one per (head, slice) measured 20 %
// slower on 16 KiB tiles, four 2 % faster than two for two heads).  FP32
// plans use 32 KiB tiles and two sub-pipelines, so each sub-pipeline keeps
// several slots in flight.
inline constexpr int max_sub_pipelines(int elt, int hg, int gt, int D, int T) {
    return (8 / tile_consumers(hg, gt) < 1)
               ? 1
               : (elt == 2 ? ((2 * D * 2 * T * hg >= 32768) ? 1
                              : (8 / tile_consumers(hg, gt) < 4 ? 8 / tile_consumers(hg, gt) : 4))
                           : (8 / tile_consumers(hg, gt) < 2 ? 8 / tile_consumers(hg, gt) : 2));
}

// Whether a kernel with sub-pipelines folds their states together inside the
// CTA at each segment end, so that a segment writes one partial (and a group
// that one CTA sees whole writes its output directly).  Measured against one
// partial per sub-pipeline: the one-KV-head rank shape of config 4 on 8 GPUs
// (8 KiB tiles, four sub-pipelines) 106.1 -> 103.2 us, FP32 config 3a 324.4 ->
// 318.6; config 3b (two sub-pipelines of four warps, latency-bound, and two
// fewer ring slots for the hand-off buffer) 25.4 -> 26.2, so it does not fold.
inline constexpr bool fold_sub_pipelines(int elt, int hg, int gt, int D, int T) {
    return max_sub_pipelines(elt, hg, gt, D, T) > 1 && (elt == 4 || max_sub_pipelines(elt, hg, gt, D, T) >= 4);
}

}  // namespace pd
