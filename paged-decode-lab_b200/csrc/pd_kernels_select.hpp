// pd_kernels_select.hpp — host-side choice of the KV heads gathered per page tile.
#pragma once

namespace pd {

// Largest KV-head group (1, 2, 4 or 8; at most the consumer warps per CTA,
// which is 4 when 32 query heads share a KV head and 8 otherwise; dividing
// kv_heads) whose page tile (K + V of elt-byte elements) stays within
// `target_bytes`, which is capped at 64 KiB.
inline int choose_heads_per_tile(int elt, int D, int T, int GT, int kv_heads, int target_bytes) {
    const int nc0 = GT == 32 ? 4 : 8;
    const int per_head = 2 * D * elt * T;
    if (target_bytes > 65536) target_bytes = 65536;
    int best = 1;
    for (int hg = 2; hg <= nc0; hg *= 2)
        if (kv_heads % hg == 0 && hg * per_head <= target_bytes) best = hg;
    return best;
}

// Sub-pipelines a kernel shape starts from (it may use fewer when its page
// tiles leave room for fewer ring slots): consumer warps are HG * NSUB.  FP16
// tiles with at least 4 KV heads keep 4-8 warps busy with NSUB = 1 (one warp
// per head sees the whole group, so unsplit groups need no merge); otherwise
// NC0 / HG sub-pipelines fill NC0 warps (8, or 4 when 32 query heads share a
// KV head).
inline constexpr int max_sub_pipelines(int elt, int hg, int gt) {
    return (elt == 2 && hg >= 4) ? 1 : ((gt == 32 ? 4 : 8) / hg > 0 ? (gt == 32 ? 4 : 8) / hg : 1);
}

}  // namespace pd
