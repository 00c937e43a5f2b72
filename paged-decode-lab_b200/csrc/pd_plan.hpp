// pd_plan.hpp — host-side plan: metadata validation, work balancing, device image.
#pragma once

#include <cuda.h>

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

#include "paged_decode.h"

namespace pd {

// Message of the last failing call on this thread (pd_last_error).
void set_error(const std::string &msg);
pd_status fail(pd_status status, const std::string &msg);
const std::string &last_error();

struct DeviceImage {
    // off_error is always 0 (pd_static_read_errors relies on it).  256 bytes:  +0 the error word (u32), +4 the count of launches whose
    // grid barrier fell back to merging for CTAs that left (u32), +8 the barrier's
    // arrival count (u64), +16 its started count (u64), +64 its left-CTA bits (16 x u64)
    size_t off_error = 0, off_head = 0, off_segs = 0, off_groups = 0, off_merge = 0, off_lengths = 0;
    size_t off_table = 0, off_part_o = 0, off_part_ml = 0, bytes = 0;
};

struct TensorMapCache {
    const void *k = nullptr;
    const void *v = nullptr;
    int dtype = -1;
    int token_groups = -1;   // map_k lands pages as [8-token group][box][8 tokens] (the tcgen05 kernel's decode)
    alignas(64) CUtensorMap map_k;
    alignas(64) CUtensorMap map_v;
};

}  // namespace pd

struct pd_plan {
    pd_layout layout{};
    int64_t width = 0;             // logical pages per table row
    int32_t split_tokens = 0;
    int32_t merge_mode = 0;
    int32_t device = -1;
    pd_dtype dtype = PD_FLOAT16;
    int32_t group = 0;             // G = Hq / Hkv
    int32_t group_tile = 8;        // GT: query heads processed together (8, 16, 32)
    int32_t group_splits = 1;      // ceil(G / GT)
    int32_t heads_per_tile = 1;    // HG: KV heads gathered per page tile
    int32_t engine = 0;            // consumer engine of the decode kernel (kEngine*)
    int32_t num_ctas = 0;
    int32_t cluster = 1;           // CTAs per cluster: 2 for a pair plan (two halves of each group)
    int32_t splits = 1;
    int32_t max_context = 0;
    int32_t num_pieces = 0;        // partial slots (segments that write partials x slot_stride)
    int32_t slot_stride = 1;       // partial slots per segment (1: sub-pipelines are folded in the CTA)
    int64_t total_pages = 0;
    int32_t sm_count = 0;          // SMs of the plan's device
    bool merge_in_kernel = false;  // split groups merged by the decode CTAs after a grid barrier
    bool dynamic = false;          // work covers max_lengths; live lengths / table read at launch
    int32_t max_span = 0;          // longest sequence the work list covers (max_lengths or lengths)
    int32_t barrier_mode = 0;      // PD_BARRIER_*: how the grid barrier before the merge is launched
    const void *occ_fn = nullptr;  // kernel whose co-resident CTA count is cached in occ_ctas
    int32_t occ_ctas = 0;
    std::vector<int32_t> table;    // [B * W]
    std::vector<int32_t> lengths;  // [B]
    std::vector<int32_t> cta_off;  // [C + 1]
    std::vector<int32_t> segs;     // 4 per segment
    std::vector<int32_t> groups;   // 8 per group: b, kv0, qoff, nh, length, slot0 (-1: direct), segments, 0
    std::vector<int32_t> head;        // [C][64] per-CTA header (kernel args: `head`)
    std::vector<int32_t> merge_rows;  // 4 per merged row: out row, first slot, segments, column
    pd::DeviceImage image;
    std::vector<uint8_t> host_image;  // metadata part of the device buffer
    uint8_t *dev = nullptr;           // bound device buffer (caller-owned)
    size_t dev_bytes = 0;
    uint8_t *ws = nullptr;            // split-K workspace bound apart from `dev` (pd_plan_bind_split)
    pd::TensorMapCache tmaps;
};

namespace pd {

// Validate metadata and build the balanced work list; `sm_count` is used when
// num_ctas <= 0.  Mirrors the checks of runtime.py:33-51 and oracle.py:20-47.
// `max_lengths` (nullable) makes a dynamic plan: its work list covers
// sequence b up to max_lengths[b] tokens, and launches may pass live lengths
// <= max_lengths and a page table updated on the device.
// `allow_pair` = false never builds a pair plan (clusters of two CTAs).
pd_status build_plan(const pd_layout *layout, const int32_t *table, int64_t width,
                     const int32_t *lengths, const int32_t *max_lengths, int32_t split_tokens,
                     int32_t merge_mode, pd_dtype dtype, int32_t num_ctas, int32_t sm_count,
                     pd_plan &plan, bool allow_pair = true);

}  // namespace pd
