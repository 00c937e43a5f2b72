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

}  // namespace pd
