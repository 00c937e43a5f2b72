// pd_plan.cpp — plan builder: validation, balanced page partition, device image.
//
// The reference plans a rectangular grid [Hq, B, splits] sized by the longest
// sequence (runtime.py:49, decode.cu:176).  Here the unit of work is a page
// tile of one group = (sequence, group of HG KV heads, query-head tile): all
// G query heads of a KV head share every K/V byte they read, and one TMA box
// brings a page's rows for HG heads at once.  The total page-tile count over
// all groups is cut into num_ctas equal contiguous ranges, so each persistent
// CTA (one per SM) streams the same number of bytes, ragged batches included.
// A group cut by range boundaries is seen in pieces; each piece's warps
// write (m, l, o) partials that a small dependent kernel merges with the
// max-corrected merge.
#include "pd_plan.hpp"

#include "pd_kernels_select.hpp"

#include <algorithm>
#include <climits>
#include <cstdlib>
#include <cstring>

namespace pd {

namespace {
thread_local std::string g_last_error;
// FP16 page tiles (K + V of HG heads) aim at this size: four TMA boxes of up
// to 16 KiB each keep the single issuing thread far ahead of HBM (a TMA
// instruction costs about the same to issue whatever its size).  FP32 tiles
// aim at half of it: FP32 warps fold tiles more slowly, so more ring slots
// per sub-pipeline matter more than fewer TMA instructions.
constexpr int kTileTargetBytes = 64 * 1024;

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }
}  // namespace

void set_error(const std::string &msg) { g_last_error = msg; }

pd_status fail(pd_status status, const std::string &msg) {
    g_last_error = msg;
    return status;
}

const std::string &last_error() { return g_last_error; }

pd_status build_plan(const pd_layout *layout, const int32_t *table, int64_t width,
                     const int32_t *lengths, const int32_t *max_lengths, int32_t split_tokens,
                     int32_t merge_mode, pd_dtype dtype, int32_t num_ctas, int32_t sm_count,
                     pd_plan &p, bool allow_pair) {
    if (!layout) return fail(PD_ERR_VALUE, "layout must not be NULL");
    const pd_layout L = *layout;
    // Layout.__post_init__ (oracle.py:24-27)
    if (L.batch <= 0 || L.query_heads <= 0 || L.kv_heads <= 0 || L.head_dim <= 0 ||
        L.page_size <= 0 || L.physical_pages <= 0)
        return fail(PD_ERR_VALUE, "layout dimensions must be positive");
    if (L.query_heads % L.kv_heads)
        return fail(PD_ERR_VALUE, "query_heads must be divisible by kv_heads");
    // DecodePlan limits (runtime.py:33-42)
    if (merge_mode != 0 && merge_mode != 1)
        return fail(PD_ERR_VALUE, "merge must be 'serial' or 'shared'");
    if (L.head_dim != 64 && L.head_dim != 128)
        return fail(PD_ERR_VALUE, "head_dim must be 64 or 128");
    if (L.page_size != 16 && L.page_size != 32)
        return fail(PD_ERR_VALUE, "page_size must be 16 or 32");
    if (L.batch > 65535 || L.query_heads > 65535)
        return fail(PD_ERR_VALUE, "batch/head count exceeds CUDA grid limits");
    if (split_tokens < 1 || split_tokens > 1048576)
        return fail(PD_ERR_VALUE, "split_tokens must be an integer in [1,1048576]");
    if (dtype != PD_FLOAT16 && dtype != PD_FLOAT32)
        return fail(PD_ERR_TYPE, "q/k/v must share float16 or float32 dtype");
    // validate_metadata (oracle.py:30-47)
    if (width < 0) return fail(PD_ERR_VALUE, "page table must have shape [batch, logical_pages]");
    if (!lengths || (width > 0 && !table))
        return fail(PD_ERR_VALUE, "table and lengths must not be NULL");
    const int64_t capacity = width * L.page_size;
    for (int b = 0; b < L.batch; ++b)
        if (lengths[b] < 0 || lengths[b] > capacity)
            return fail(PD_ERR_VALUE, "sequence length exceeds page table capacity");
    if (std::max<int64_t>(width, L.physical_pages) > INT32_MAX)
        return fail(PD_ERR_VALUE, "metadata exceeds int32 addressing limits");
    for (int b = 0; b < L.batch; ++b) {
        const int64_t live = (int64_t(lengths[b]) + L.page_size - 1) / L.page_size;
        for (int64_t i = 0; i < live; ++i) {
            const int32_t page = table[b * width + i];
            if (page < 0 || page >= L.physical_pages)
                return fail(PD_ERR_VALUE, "live logical page maps outside physical cache");
        }
    }
    if (width > 65536) return fail(PD_ERR_VALUE, "page table width must not exceed 65536");
    // A dynamic plan's work covers each sequence up to its capacity.
    if (max_lengths)
        for (int b = 0; b < L.batch; ++b)
            if (max_lengths[b] < lengths[b] || max_lengths[b] > capacity)
                return fail(PD_ERR_VALUE, "max_lengths must lie between lengths and the page table capacity");
    const int32_t *span = max_lengths ? max_lengths : lengths;
    int32_t max_context = 0, max_span = 0;
    for (int b = 0; b < L.batch; ++b) {
        max_context = std::max(max_context, lengths[b]);
        max_span = std::max(max_span, span[b]);
    }
    if (max_span > 1048576)
        return fail(PD_ERR_VALUE, "this implementation supports at most 1M context tokens");
    const int64_t splits = std::max<int64_t>(1, (int64_t(max_context) + split_tokens - 1) / split_tokens);
    if (splits > 65535) return fail(PD_ERR_VALUE, "too many context splits");
    // TMA row coordinates are int32: page * page_size must fit.
    if (L.physical_pages * L.page_size > INT32_MAX)
        return fail(PD_ERR_VALUE, "physical_pages * page_size exceeds int32 TMA coordinates");

    p.layout = L;
    p.width = width;
    p.split_tokens = split_tokens;
    p.merge_mode = merge_mode;
    p.dtype = dtype;
    p.splits = int32_t(splits);
    p.max_context = max_context;
    p.max_span = max_span;
    p.dynamic = max_lengths != nullptr;
    p.group = L.query_heads / L.kv_heads;
    p.group_tile = p.group <= 8 ? 8 : (p.group <= 16 ? 16 : 32);
    p.group_splits = (p.group + p.group_tile - 1) / p.group_tile;
    if (table)
        p.table.assign(table, table + size_t(L.batch) * width);
    else
        p.table.clear();
    p.lengths.assign(lengths, lengths + L.batch);

    // ---------------------------------------------------------------- groups
    // A group is (sequence b, KV-head group of HG heads, query-head tile gs):
    // its page tiles carry HG heads' K and V for one page.
    const int T = L.page_size;
    // PD_TILE_KIB overrides the tile target (tuning; capped at 64 KiB).
    int target = dtype == PD_FLOAT16 ? kTileTargetBytes : kTileTargetBytes / 2;
    if (const char *env = std::getenv("PD_TILE_KIB")) {
        const int kib = std::atoi(env);
        if (kib >= 1) target = kib * 1024;
    }
    // FP16 group tiles of 32 query heads: the tcgen05 kernel (one KV head per
    // page tile), measured faster than the warp-level kernel (m16n8k16 MMAs,
    // up to two KV heads per tile) for head_dim 64 and 128 with pages of 16
    // and 32 tokens (B64 x 2048 tokens, 32:1: 15.1 / 20.4 us against 19.1 /
    // 22.0 at head_dim 64, 17.5 / 21.1 against 25.3 / 30.3 at head_dim 128,
    // pages 32 / 16; eight sequences of 8k tokens: 18.9 against 18.1).
    // PD_MQA_ENGINE=tcgen05 or warp forces either kernel for every such plan.
    const char *engine_env = std::getenv("PD_MQA_ENGINE");
    const bool force_warp = engine_env && std::strcmp(engine_env, "warp") == 0;
    const bool tensor_memory = dtype == PD_FLOAT16 && p.group_tile == 32 && !force_warp;
    const int hg = tensor_memory ? 1
                                 : choose_heads_per_tile(dtype == PD_FLOAT16 ? 2 : 4, L.head_dim, T, p.group_tile,
                                                         L.kv_heads, target);
    p.heads_per_tile = hg;
    p.engine = tensor_memory && mqa_tensor_memory_shape(2, hg, p.group_tile, L.head_dim, T) ? kEngineTensorMemory
                                                                                          : kEngineWarp;
    const int kv_groups = L.kv_heads / hg;
    const int64_t ngroups = int64_t(L.batch) * kv_groups * p.group_splits;
    if (ngroups > INT32_MAX / 2) return fail(PD_ERR_VALUE, "too many (sequence, KV head) groups");
    std::vector<int64_t> gpages(ngroups);
    p.groups.assign(size_t(ngroups) * 8, 0);
    int64_t total = 0;
    for (int b = 0, gi = 0; b < L.batch; ++b)
        for (int kg = 0; kg < kv_groups; ++kg)
            for (int gs = 0; gs < p.group_splits; ++gs, ++gi) {
                int32_t *g = &p.groups[size_t(gi) * 8];
                g[0] = b;
                g[1] = kg * hg;                        // first KV head of the group
                g[2] = gs * p.group_tile;              // query-head offset inside each KV head's group
                g[3] = std::min(p.group_tile, p.group - gs * p.group_tile);
                g[4] = span[b];                        // tokens the group's work covers
                g[5] = -1;
                g[6] = 0;
                gpages[gi] = (int64_t(span[b]) + T - 1) / T;
                total += gpages[gi];
            }
    if (total > INT32_MAX) return fail(PD_ERR_VALUE, "too many page tiles per decode step");
    p.total_pages = total;

    // ---------------------------------------------------------------- balance
    // The warp-level kernels cost about the same per page tile: CTAs get equal
    // page counts.  The tcgen05 kernel works in steps of 128 tokens of one
    // segment and a step costs about the same whether full or not: CTAs get
    // equal step counts, and cuts fall on step boundaries of the group, unless
    // there are fewer than 4 steps per CTA (then more CTAs streaming part steps
    // beat fewer streaming whole ones).
    int64_t C = num_ctas > 0 ? num_ctas : std::max(1, sm_count);
    int64_t unit = p.engine == kEngineTensorMemory ? std::max(1, 128 / T) : 1;   // pages per unit
    // Pair plans (tcgen05 engine, automatic CTA count): when the groups are
    // about equally long and two CTAs per group fill most of the SMs, CTAs
    // 2g and 2g + 1 form a cluster that streams the two halves of group g (cut
    // on a step boundary) and merges them through distributed shared memory:
    // no partials, no grid barrier, no merge kernel.  PD_PAIR=0 / 1 turns
    // the choice off / on wherever the groups fit.
    p.cluster = 1;
    if (allow_pair && p.engine == kEngineTensorMemory && num_ctas <= 0 && sm_count > 0 && ngroups >= 1 &&
        2 * ngroups <= std::min(sm_count, 1024)) {
        int64_t longest = 0;
        for (int64_t gi = 0; gi < ngroups; ++gi) longest = std::max(longest, gpages[gi]);
        bool pair = longest * ngroups * 8 <= total * 9 && 2 * ngroups * 4 >= int64_t(sm_count) * 3;
        if (const char *env = std::getenv("PD_PAIR")) {
            if (std::strcmp(env, "0") == 0) pair = false;
            if (std::strcmp(env, "1") == 0) pair = true;
        }
        if (pair) p.cluster = 2;
    }
    int64_t total_units = 0;
    for (int64_t gi = 0; gi < ngroups; ++gi) total_units += (gpages[gi] + unit - 1) / unit;
    if (unit > 1 && total_units < 4 * C && p.cluster == 1) {
        unit = 1;
        total_units = total;
    }
    C = p.cluster == 2 ? 2 * ngroups : std::max<int64_t>(1, std::min<int64_t>(C, std::max<int64_t>(1, total_units)));
    p.num_ctas = int32_t(C);
    auto bound = [&](int64_t c) { return c * total_units / C; };   // start of CTA c's range, in units
    std::vector<std::vector<int32_t>> per(C);
    std::vector<int32_t> seg_count(ngroups, 0);
    int64_t cursor = 0, c = 0, empty = 0;
    for (int64_t gi = 0; gi < ngroups && p.cluster == 2; ++gi) {
        // the first CTA takes the first half of the group's steps (rounded up)
        const int64_t np = gpages[gi];
        const int64_t cut = std::min(np, ((np + unit - 1) / unit + 1) / 2 * unit);
        per[2 * gi] = {int32_t(gi), 0, int32_t(cut), 0};
        per[2 * gi + 1] = {int32_t(gi), int32_t(cut), int32_t(np), 0};
        seg_count[gi] = 2;
    }
    for (int64_t gi = 0; gi < ngroups && p.cluster == 1; ++gi) {
        const int64_t np = gpages[gi];
        if (np == 0) {
            // empty sequence: a zero-page segment writes its zero rows
            auto &v = per[empty++ % C];
            v.insert(v.end(), {int32_t(gi), 0, 0, -1});
            seg_count[gi] = 1;
            continue;
        }
        const int64_t nu = (np + unit - 1) / unit;
        int64_t start = cursor;
        const int64_t end = cursor + nu;
        while (start < end) {
            while (bound(c + 1) <= start) ++c;
            const int64_t stop = std::min(end, bound(c + 1));
            per[c].insert(per[c].end(), {int32_t(gi), int32_t((start - cursor) * unit),
                                         int32_t(std::min(np, (stop - cursor) * unit)), 0});
            ++seg_count[gi];
            start = stop;
        }
        cursor = end;
    }
    // Partial slots.  A segment's consumer warps may run as several
    // sub-pipelines (alternate page tiles).  Kernel shapes that fold their
    // states inside the CTA (fold_sub_pipelines) write one partial slot per
    // segment; the others write one per sub-pipeline, and slot_stride =
    // max_sub_pipelines() slots are reserved per segment.  A group with one
    // segment and slot_stride == 1 is seen whole by one CTA, which writes the
    // final output itself.
    {
        const int elt = dtype == PD_FLOAT16 ? 2 : 4;
        p.slot_stride = (p.engine == kEngineTensorMemory || fold_sub_pipelines(elt, hg, p.group_tile, L.head_dim, T))
                            ? 1
                            : max_sub_pipelines(elt, hg, p.group_tile, L.head_dim, T);
    }
    std::vector<int32_t> next_slot(ngroups, -1);
    int64_t slots = 0;
    for (int64_t gi = 0; gi < ngroups; ++gi) {
        int32_t *g = &p.groups[size_t(gi) * 8];
        g[6] = seg_count[gi];
        if (p.cluster == 2 || (seg_count[gi] == 1 && p.slot_stride == 1)) {
            g[5] = -1;
        } else {
            g[5] = int32_t(slots);
            next_slot[gi] = int32_t(slots);
            slots += int64_t(seg_count[gi]) * p.slot_stride;
        }
    }
    if (slots > INT32_MAX / 64) return fail(PD_ERR_VALUE, "too many partial slots");
    p.num_pieces = int32_t(slots);
    // Output rows of the split groups, merged after the decode.  With no more
    // CTAs than SMs the decode CTAs can all be resident at once (one CTA per
    // SM by construction), so they merge them in-kernel after a grid barrier.
    // Each row: {output row b * Hq + query head, first slot, segments, column
    // hh * GT + q of the [slot][HG][GT] partial layout}.
    p.merge_rows.clear();
    if (int64_t(L.batch) * L.query_heads > INT32_MAX) return fail(PD_ERR_VALUE, "too many output rows");
    for (int64_t gi = 0; gi < ngroups; ++gi) {
        const int32_t *g = &p.groups[size_t(gi) * 8];
        if (g[5] < 0) continue;
        for (int hh = 0; hh < hg; ++hh)
            for (int q = 0; q < g[3]; ++q) {
                const int64_t row = int64_t(g[0]) * L.query_heads + int64_t(g[1] + hh) * p.group + g[2] + q;
                p.merge_rows.insert(p.merge_rows.end(),
                                    {int32_t(row), g[5], g[6], hh * p.group_tile + q});
            }
    }
    p.sm_count = sm_count;
    p.merge_in_kernel = !p.merge_rows.empty() && sm_count > 0 && C <= sm_count && C <= 1024;
    p.cta_off.assign(size_t(C) + 1, 0);
    p.segs.clear();
    for (int64_t i = 0; i < C; ++i) {
        for (size_t k = 0; k < per[i].size(); k += 4) {
            int32_t *sv = &per[i][k];
            const int32_t gi = sv[0];
            if (next_slot[gi] < 0) {
                sv[3] = -1;
            } else {
                sv[3] = next_slot[gi];
                next_slot[gi] += p.slot_stride;
            }
        }
        p.segs.insert(p.segs.end(), per[i].begin(), per[i].end());
        p.cta_off[i + 1] = int32_t(p.segs.size() / 4);
    }

    // Per-CTA header (64 words): [0] first segment index, [1] end index,
    // [4..7] the first segment, [8..15] its group's 8 words, [16..47] the page
    // ids of its first 32 pages (0 past its end).  The kernel starts streaming
    // after reading these 256 bytes, with no further dependent loads.
    p.head.assign(size_t(C) * 64, 0);
    for (int64_t i = 0; i < C; ++i) {
        int32_t *h = &p.head[size_t(i) * 64];
        h[0] = p.cta_off[i];
        h[1] = p.cta_off[i + 1];
        if (h[0] == h[1]) continue;
        const int32_t *sv = &p.segs[size_t(h[0]) * 4];
        std::copy(sv, sv + 4, h + 4);
        const int32_t *g = &p.groups[size_t(sv[0]) * 8];
        std::copy(g, g + 8, h + 8);
        for (int k = 0; k < 32 && sv[1] + k < sv[2]; ++k)
            h[16 + k] = p.table[size_t(g[0]) * p.width + sv[1] + k];
    }

    // ---------------------------------------------------------------- device image
    DeviceImage &im = p.image;
    size_t off = 0;
    im.off_error = off;    off = align256(off + 192);
    im.off_head = off;     off = align256(off + p.head.size() * 4);
    im.off_segs = off;     off = align256(off + p.segs.size() * 4);
    im.off_groups = off;   off = align256(off + p.groups.size() * 4);
    im.off_merge = off;    off = align256(off + p.merge_rows.size() * 4);
    im.off_lengths = off;  off = align256(off + p.lengths.size() * 4);
    im.off_table = off;    off = align256(off + p.table.size() * 4);
    im.off_part_o = off;   off = align256(off + size_t(slots) * hg * p.group_tile * L.head_dim * 4);
    im.off_part_ml = off;  off = align256(off + size_t(slots) * hg * p.group_tile * 8);
    im.bytes = off;
    p.host_image.assign(im.off_part_o, 0);
    std::memcpy(p.host_image.data() + im.off_head, p.head.data(), p.head.size() * 4);
    std::memcpy(p.host_image.data() + im.off_segs, p.segs.data(), p.segs.size() * 4);
    std::memcpy(p.host_image.data() + im.off_groups, p.groups.data(), p.groups.size() * 4);
    if (!p.merge_rows.empty())
        std::memcpy(p.host_image.data() + im.off_merge, p.merge_rows.data(), p.merge_rows.size() * 4);
    std::memcpy(p.host_image.data() + im.off_lengths, p.lengths.data(), p.lengths.size() * 4);
    if (!p.table.empty())
        std::memcpy(p.host_image.data() + im.off_table, p.table.data(), p.table.size() * 4);
    return PD_OK;
}

}  // namespace pd
