// pd_api.cu — C ABI of the decode operator: plans, TMA descriptors, launches.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <new>
#include <set>
#include <string>
#include <type_traits>
#include <utility>

#include "pd_kernels.cuh"
#include "pd_plan.hpp"

#define PD_API extern "C" __attribute__((visibility("default")))

namespace pd {
const std::string &last_error();

namespace {

KernelEntry kernel_for(pd_dtype dtype, int D, int T, int gt, int hg, int mode, int engine) {
    if (dtype == PD_FLOAT16) {
        if (D == 64)
            return T == 16 ? kernel_entry_f16_d64_t16(gt, hg, mode, engine)
                           : kernel_entry_f16_d64_t32(gt, hg, mode, engine);
        return T == 16 ? kernel_entry_f16_d128_t16(gt, hg, mode, engine)
                       : kernel_entry_f16_d128_t32(gt, hg, mode, engine);
    }
    if (D == 64)
        return T == 16 ? kernel_entry_f32_d64_t16(gt, hg, mode, engine) : kernel_entry_f32_d64_t32(gt, hg, mode, engine);
    return T == 16 ? kernel_entry_f32_d128_t16(gt, hg, mode, engine) : kernel_entry_f32_d128_t32(gt, hg, mode, engine);
}

std::mutex g_attr_mutex;
std::set<std::pair<int, KernelFn>> g_attr_done;

pd_status ensure_smem_attribute(int device, const KernelEntry &e) {
    std::lock_guard<std::mutex> lock(g_attr_mutex);
    if (g_attr_done.count({device, e.fn})) return PD_OK;
    const cudaError_t err = cudaFuncSetAttribute(reinterpret_cast<const void *>(e.fn),
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 int(e.smem));
    if (err != cudaSuccess)
        return fail(PD_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(err));
    g_attr_done.insert({device, e.fn});
    return PD_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult query;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &query) ==
                cudaSuccess &&
            query == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    });
    return fn;
}

// K or V cache [P, T, Hkv, D] viewed as 5-D {128/elt, T, D*elt/128, Hkv, P}
// (strides in bytes: elt, Hkv*D*elt, 128, D*elt, T*Hkv*D*elt).  One box = all
// of a page's rows for HG KV heads, landing in shared memory as
// [head][128-byte box of the row][token] rows of 128 bytes, so the 128-byte
// swizzle XORs by token and one instruction moves the whole K (or V) page.
// With token_groups (the tcgen05 kernel's K) the view splits the token into
// 8-token groups, so that one box per page lands the rows of each 128-byte
// column of a whole step at one fixed stride per 8 rows.
pd_status encode_cache_map(const pd_plan &p, const void *base, pd_dtype dtype, int hg, CUtensorMap *map,
                           bool token_groups = false) {
    auto encode = tensor_map_encoder();
    if (!encode) return fail(PD_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    const cuuint64_t elt = dtype == PD_FLOAT16 ? 2 : 4;
    const pd_layout &L = p.layout;
    const cuuint64_t row = cuuint64_t(L.head_dim) * elt;
    const cuuint64_t nbox = row / 128;
    const cuuint64_t hkv = cuuint64_t(L.kv_heads), T = cuuint64_t(L.page_size);
    // {128 bytes of a row, token, 128-byte box of the row, KV head, page}: one
    // box {all, T, all, hg, 1} lands as [head][box][token] 128-byte rows.
    cuuint64_t dims[5] = {128 / elt, T, nbox, hkv, cuuint64_t(L.physical_pages)};
    cuuint64_t strides[4] = {row * hkv, 128, row, row * hkv * T};
    cuuint32_t box[5] = {cuuint32_t(128 / elt), cuuint32_t(T), cuuint32_t(nbox), cuuint32_t(hg), 1};
    if (token_groups) {
        // The tcgen05 kernel's K: {128 bytes, token within 8, 128-byte box of
        // any KV head's row (box b of head h is h * nbox + b), 8-token group,
        // page}; one box {all, 8, nbox, T / 8, 1} per page and head lands as
        // [group][box][8 tokens] 128-byte rows, so the 8-row groups of one box
        // column sit nbox * 1024 bytes apart across all pages of a step.
        dims[1] = 8;
        dims[2] = nbox * hkv;
        dims[3] = T / 8;
        strides[0] = row * hkv;
        strides[1] = 128;
        strides[2] = 8 * row * hkv;
        box[1] = 8;
        box[3] = cuuint32_t(T / 8);
        box[4] = 1;
    }
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    const CUresult r = encode(map,
                              dtype == PD_FLOAT16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                  : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                              5, const_cast<void *>(base), dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(PD_ERR_CUDA, "cuTensorMapEncodeTiled failed with code " + std::to_string(int(r)));
    return PD_OK;
}

struct DeviceGuard {
    int prev = -1;
    cudaError_t err = cudaSuccess;
    explicit DeviceGuard(int device) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != device) err = cudaSetDevice(device);
    }
    ~DeviceGuard() {
        if (prev >= 0 && err == cudaSuccess) cudaSetDevice(prev);
    }
};

pd_status check_bound(const pd_plan *p) {
    if (!p) return fail(PD_ERR_VALUE, "plan must not be NULL");
    if (p->device < 0) return fail(PD_ERR_VALUE, "host-only plan (device < 0) cannot launch");
    if (!p->dev) return fail(PD_ERR_UNBOUND, "plan has no device buffer: call pd_plan_bind first");
    return PD_OK;
}

pd_status check_dtype(const pd_plan *p, pd_dtype dtype) {
    if (dtype != PD_FLOAT16 && dtype != PD_FLOAT32)
        return fail(PD_ERR_TYPE, "q/k/v must share float16 or float32 dtype");
    if (dtype != p->dtype) return fail(PD_ERR_TYPE, "input dtype differs from the plan's dtype");
    return PD_OK;
}

DecodeArgs make_args_at(pd_plan *p, uint8_t *dev, const void *q, float *out, float *stats) {
    DecodeArgs a{};
    const DeviceImage &im = p->image;
    a.q = q;
    a.table = reinterpret_cast<const int32_t *>(dev + im.off_table);
    a.head = reinterpret_cast<const int4 *>(dev + im.off_head);
    a.segs = reinterpret_cast<const int4 *>(dev + im.off_segs);
    a.groups = reinterpret_cast<const int4 *>(dev + im.off_groups);
    // the split-K partials: in the plan's own buffer, or in a workspace bound
    // apart from the metadata (pd_plan_bind_split, shareable between plans)
    uint8_t *ws = (p->ws && dev == p->dev) ? p->ws : dev + im.off_part_o;
    a.part_o = reinterpret_cast<float *>(ws);
    a.part_ml = reinterpret_cast<float2 *>(ws + (im.off_part_ml - im.off_part_o));
    a.out = out;
    a.stats = stats;
    a.error = reinterpret_cast<uint32_t *>(dev + im.off_error);
    a.Hq = p->layout.query_heads;
    a.Hkv = p->layout.kv_heads;
    a.W = int32_t(p->width);
    a.max_len = p->max_span;
    a.group = p->group;
    a.slot_stride = p->slot_stride;
    a.num_groups = int32_t(p->groups.size() / 8);
    a.gb.count = reinterpret_cast<unsigned long long *>(dev + im.off_error + 8);
    a.gb.started = reinterpret_cast<unsigned long long *>(dev + im.off_error + 16);
    a.gb.left = reinterpret_cast<unsigned long long *>(dev + im.off_error + 64);
    a.gb.leave_mode = 0;
    a.gb.leave_ns = kBarrierLeaveNs;
    a.fallbacks = reinterpret_cast<uint32_t *>(dev + im.off_error + 4);
    a.merge_rows = reinterpret_cast<const int4 *>(dev + im.off_merge);
    a.num_merge_rows = int32_t(p->merge_rows.size() / 4);
    a.fused_merge = p->merge_in_kernel ? 1 : 0;
    a.lengths = reinterpret_cast<const int32_t *>(dev + im.off_lengths);
    a.dynamic = p->dynamic ? 1 : 0;
    a.xworld = 0;
    a.rows = p->layout.batch * p->layout.query_heads;
    a.P = p->layout.physical_pages;
    a.scale_log2 = float(1.4426950408889634 / std::sqrt(double(p->layout.head_dim)));
    return a;
}

DecodeArgs make_args(pd_plan *p, const void *q, float *out, float *stats) {
    return make_args_at(p, p->dev, q, out, stats);
}

pd_status launch(pd_plan *p, const void *k, const void *v, pd_dtype dtype, int mode,
                 const DecodeArgs &args, void *stream) {
    if (!k || !v) return fail(PD_ERR_VALUE, "k and v must not be NULL");
    if ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) & 15)
        return fail(PD_ERR_VALUE, "k and v must be 16-byte aligned");
    TensorMapCache &tc = p->tmaps;
    const int token_groups = p->engine == kEngineTensorMemory && mode == kModeDecode ? 1 : 0;
    if (tc.k != k || tc.v != v || tc.dtype != int(dtype) || tc.token_groups != token_groups) {
        pd_status s = encode_cache_map(*p, k, dtype, p->heads_per_tile, &tc.map_k, token_groups != 0);
        if (s != PD_OK) return s;
        s = encode_cache_map(*p, v, dtype, p->heads_per_tile, &tc.map_v);
        if (s != PD_OK) return s;
        tc.k = k;
        tc.v = v;
        tc.dtype = int(dtype);
        tc.token_groups = token_groups;
    }
    const KernelEntry e =
        kernel_for(dtype, p->layout.head_dim, p->layout.page_size, p->group_tile, p->heads_per_tile, mode,
                   p->engine);
    pd_status s = ensure_smem_attribute(p->device, e);
    if (s != PD_OK) return s;
    const auto st = static_cast<cudaStream_t>(stream);
    DecodeArgs la = args;
    if (mode != kModeDecode) la.fused_merge = 0;
    la.pair = mode == kModeDecode && p->cluster == 2 ? 1 : 0;
    // Every decode launch is programmatically dependent on the kernel before
    // it (the kernel waits with griddepcontrol.wait before touching q, the
    // caches or its outputs), so its launch and set-up overlap that kernel.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(p->num_ctas));
    cfg.blockDim = dim3(unsigned(e.threads));
    cfg.dynamicSmemBytes = e.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeCooperative;
    attr[1].val.cooperative = 1;
    cfg.attrs = attr;
    cudaError_t err;
    if (la.pair) {
        // clusters of two CTAs (one group each); they wait only for each other
        if (la.xworld || la.fused_merge) return fail(PD_ERR_VALUE, "a pair plan cannot take part in an exchange");
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = 2;
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = 1;
        cfg.numAttrs = 2;
        err = cudaLaunchKernelEx(&cfg, e.fn, tc.map_k, tc.map_v, la);
        if (err != cudaSuccess)
            return fail(PD_ERR_CUDA, std::string("decode launch: ") + cudaGetErrorString(err));
        return PD_OK;
    }
    if (la.fused_merge && !la.xworld && p->barrier_mode != PD_BARRIER_COOPERATIVE) {
        // A plain launch starts on SMs as the previous kernel's CTAs leave
        // them (measured 2-3 us a step ahead of a cooperative launch).  The
        // grid barrier then lets a CTA leave when another has not started, so
        // residency is not required; the CTAs must merely fit the GPU at once.
        if (p->occ_fn != reinterpret_cast<const void *>(e.fn)) {
            int per_sm = 0;
            err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, e.fn, e.threads, e.smem);
            if (err != cudaSuccess)
                return fail(PD_ERR_CUDA, std::string("occupancy query: ") + cudaGetErrorString(err));
            p->occ_fn = reinterpret_cast<const void *>(e.fn);
            p->occ_ctas = per_sm * p->sm_count;
        }
        if (p->num_ctas <= p->occ_ctas) {
            la.gb.leave_mode = p->barrier_mode == PD_BARRIER_LEAVE_AT_ONCE ? 2u : 1u;
        } else {
            la.fused_merge = 0;
        }
    } else if (la.fused_merge || la.xworld) {
        // The CTAs wait for each other at a grid barrier before merging, and
        // in exchange mode for every CTA of every rank; a cooperative launch
        // guarantees they are all resident, or refuses.
        cfg.numAttrs = 2;
        err = cudaLaunchKernelEx(&cfg, e.fn, tc.map_k, tc.map_v, la);
        if (err == cudaSuccess) return PD_OK;
        if (err != cudaErrorCooperativeLaunchTooLarge || la.xworld)
            return fail(PD_ERR_CUDA, std::string("decode launch: ") + cudaGetErrorString(err));
        (void)cudaGetLastError();   // not all CTAs fit at once: merge with the separate kernel
        la.fused_merge = 0;
    }
    cfg.numAttrs = 1;
    err = cudaLaunchKernelEx(&cfg, e.fn, tc.map_k, tc.map_v, la);
    if (err != cudaSuccess)
        return fail(PD_ERR_CUDA, std::string("decode launch: ") + cudaGetErrorString(err));
    if (mode == kModeDecode && p->num_pieces > 0 && !la.fused_merge) {
        err = launch_merge_partials(la, p->heads_per_tile, p->group_tile, e.nsub, p->layout.head_dim, st);
        if (err != cudaSuccess)
            return fail(PD_ERR_CUDA, std::string("merge launch: ") + cudaGetErrorString(err));
    }
    return PD_OK;
}

pd_status decode_impl(pd_plan *p, const void *q, const void *k, const void *v, pd_dtype dtype,
                      float *out, float *stats, void *stream, const int32_t *table = nullptr,
                      const int32_t *lengths = nullptr, const DecodeArgs *exchange = nullptr) {
    pd_status s = check_bound(p);
    if (s != PD_OK) return s;
    if ((s = check_dtype(p, dtype)) != PD_OK) return s;
    if (!q || !out) return fail(PD_ERR_VALUE, "q and out must not be NULL");
    if ((reinterpret_cast<uintptr_t>(q) & 15) || (reinterpret_cast<uintptr_t>(out) & 15))
        return fail(PD_ERR_VALUE, "q and out must be 16-byte aligned");
    if (stats && (reinterpret_cast<uintptr_t>(stats) & 7))
        return fail(PD_ERR_VALUE, "stats must be 8-byte aligned");
    DeviceGuard guard(p->device);
    if (guard.err != cudaSuccess)
        return fail(PD_ERR_CUDA, std::string("cudaSetDevice: ") + cudaGetErrorString(guard.err));
    DecodeArgs args = make_args(p, q, out, stats);
    if (table) args.table = table;
    if (lengths) args.lengths = lengths;
    if (exchange) {
        std::copy(exchange->xpeer, exchange->xpeer + kMaxRanks, args.xpeer);
        args.xslot = exchange->xslot;
        args.xrank = exchange->xrank;
        args.xworld = exchange->xworld;
    }
    return launch(p, k, v, dtype, kModeDecode, args, stream);
}

// One rank's slot: rows * D o floats, then {m, l, tag, 0} per row.
int64_t exchange_slot_bytes(const pd_plan *p) {
    const int64_t rows = int64_t(p->layout.batch) * p->layout.query_heads;
    return (rows * (p->layout.head_dim + 4) * 4 + 255) / 256 * 256;
}

}  // namespace
}  // namespace pd

using namespace pd;

namespace {
// Clusters of two CTAs of a pair plan's decode kernel that can be resident at once on `device`.
pd_status max_active_pair_clusters(const pd_plan &p, int device, int *clusters) {
    const KernelEntry e = kernel_for(p.dtype, p.layout.head_dim, p.layout.page_size, p.group_tile,
                                     p.heads_per_tile, kModeDecode, p.engine);
    DeviceGuard guard(device);
    if (guard.err != cudaSuccess)
        return fail(PD_ERR_CUDA, std::string("cudaSetDevice: ") + cudaGetErrorString(guard.err));
    pd_status s = ensure_smem_attribute(device, e);
    if (s != PD_OK) return s;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(p.num_ctas));
    cfg.blockDim = dim3(unsigned(e.threads));
    cfg.dynamicSmemBytes = e.smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t err = cudaOccupancyMaxActiveClusters(clusters, e.fn, &cfg);
    if (err != cudaSuccess)
        return fail(PD_ERR_CUDA, std::string("cluster occupancy query: ") + cudaGetErrorString(err));
    return PD_OK;
}

pd_status create_impl(const pd_layout *layout, const int32_t *table, int64_t table_width,
                      const int32_t *lengths, const int32_t *max_lengths, int32_t split_tokens,
                      int32_t merge_mode, pd_dtype dtype, int32_t device, int32_t num_ctas,
                      pd_plan **out_plan) {
    if (!out_plan) return fail(PD_ERR_VALUE, "out_plan must not be NULL");
    *out_plan = nullptr;
    int sm_count = 148;
    if (device >= 0) {
        const cudaError_t err = cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, device);
        if (err != cudaSuccess)
            return fail(PD_ERR_CUDA, std::string("device query: ") + cudaGetErrorString(err));
    }
    pd_plan *p = new (std::nothrow) pd_plan();
    if (!p) return fail(PD_ERR_VALUE, "out of host memory");
    pd_status s = build_plan(layout, table, table_width, lengths, max_lengths, split_tokens, merge_mode,
                             dtype, num_ctas, sm_count, *p);
    if (s == PD_OK && p->cluster == 2 && device >= 0) {
        // A pair plan only where all its clusters of two CTAs fit on the device
        // at once (shared memory, GPC boundaries); otherwise one CTA per SM.
        int clusters = 0;
        s = max_active_pair_clusters(*p, device, &clusters);
        if (s == PD_OK && 2 * int64_t(clusters) < p->num_ctas) {
            *p = pd_plan();
            s = build_plan(layout, table, table_width, lengths, max_lengths, split_tokens, merge_mode, dtype,
                           num_ctas, sm_count, *p, false);
        }
    }
    if (s != PD_OK) {
        delete p;
        return s;
    }
    p->device = device;
    *out_plan = p;
    return PD_OK;
}
}  // namespace

PD_API pd_status pd_plan_create(const pd_layout *layout, const int32_t *table, int64_t table_width,
                                const int32_t *lengths, int32_t split_tokens, int32_t merge_mode,
                                pd_dtype dtype, int32_t device, int32_t num_ctas, pd_plan **out_plan) {
    return create_impl(layout, table, table_width, lengths, nullptr, split_tokens, merge_mode, dtype, device,
                       num_ctas, out_plan);
}

PD_API pd_status pd_plan_create_dynamic(const pd_layout *layout, const int32_t *table, int64_t table_width,
                                        const int32_t *lengths, const int32_t *max_lengths,
                                        int32_t split_tokens, int32_t merge_mode, pd_dtype dtype,
                                        int32_t device, int32_t num_ctas, pd_plan **out_plan) {
    if (!max_lengths) return fail(PD_ERR_VALUE, "max_lengths must not be NULL");
    return create_impl(layout, table, table_width, lengths, max_lengths, split_tokens, merge_mode, dtype,
                       device, num_ctas, out_plan);
}

PD_API void pd_plan_destroy(pd_plan *plan) { delete plan; }

PD_API pd_status pd_plan_get_info(const pd_plan *p, pd_plan_info *info) {
    if (!p || !info) return fail(PD_ERR_VALUE, "plan and info must not be NULL");
    info->splits = p->splits;
    info->max_context = p->max_context;
    info->num_ctas = p->num_ctas;
    info->num_segments = int32_t(p->segs.size() / 4);
    info->num_groups = int32_t(p->groups.size() / 8);
    info->num_pieces = p->num_pieces;
    info->group_tile = p->group_tile;
    info->heads_per_tile = p->heads_per_tile;
    info->slot_stride = p->slot_stride;
    info->engine = p->engine;
    info->cluster_ctas = p->cluster;
    info->total_pages = int32_t(p->total_pages);
    info->merge_rows = int32_t(p->merge_rows.size() / 4);
    info->merge_in_kernel = p->merge_in_kernel ? 1 : 0;
    info->dynamic = p->dynamic ? 1 : 0;
    info->max_span = p->max_span;
    info->workspace_bytes = int64_t(p->image.bytes - p->image.off_part_o);
    info->device_bytes = int64_t(p->image.bytes);
    return PD_OK;
}

PD_API pd_status pd_plan_copy_worklist(const pd_plan *p, int32_t *segments, int32_t *groups,
                                       int32_t *cta_offsets) {
    if (!p) return fail(PD_ERR_VALUE, "plan must not be NULL");
    if (segments) std::copy(p->segs.begin(), p->segs.end(), segments);
    if (groups) std::copy(p->groups.begin(), p->groups.end(), groups);
    if (cta_offsets) std::copy(p->cta_off.begin(), p->cta_off.end(), cta_offsets);
    return PD_OK;
}

PD_API size_t pd_plan_device_bytes(const pd_plan *p) { return p ? p->image.bytes : 0; }

namespace {
// Upload the plan's metadata into `buffer` (>= `need` bytes) and bind it.
pd_status bind_impl(pd_plan *p, void *buffer, size_t bytes, size_t need, void *stream) {
    if (!p) return fail(PD_ERR_VALUE, "plan must not be NULL");
    if (p->device < 0) return fail(PD_ERR_VALUE, "host-only plan (device < 0) cannot be bound");
    if (!buffer || bytes < need)
        return fail(PD_ERR_VALUE, "device buffer is NULL or smaller than the plan needs");
    if (reinterpret_cast<uintptr_t>(buffer) & 255)
        return fail(PD_ERR_VALUE, "device buffer must be 256-byte aligned");
    DeviceGuard guard(p->device);
    if (guard.err != cudaSuccess)
        return fail(PD_ERR_CUDA, std::string("cudaSetDevice: ") + cudaGetErrorString(guard.err));
    auto st = static_cast<cudaStream_t>(stream);
    cudaError_t err = cudaMemcpyAsync(buffer, p->host_image.data(), p->host_image.size(),
                                      cudaMemcpyHostToDevice, st);
    if (err == cudaSuccess) err = cudaStreamSynchronize(st);
    if (err != cudaSuccess)
        return fail(PD_ERR_CUDA, std::string("plan upload: ") + cudaGetErrorString(err));
    p->dev = static_cast<uint8_t *>(buffer);
    p->dev_bytes = bytes;
    p->ws = nullptr;
    return PD_OK;
}
}  // namespace

PD_API pd_status pd_plan_bind(pd_plan *p, void *buffer, size_t bytes, void *stream) {
    return bind_impl(p, buffer, bytes, p ? p->image.bytes : 0, stream);
}

PD_API size_t pd_plan_metadata_bytes(const pd_plan *p) { return p ? p->image.off_part_o : 0; }

PD_API size_t pd_plan_workspace_bytes(const pd_plan *p) {
    return p ? p->image.bytes - p->image.off_part_o : 0;
}

PD_API pd_status pd_plan_bind_split(pd_plan *p, void *metadata, size_t metadata_bytes, void *workspace,
                                    size_t workspace_bytes, void *stream) {
    if (!p) return fail(PD_ERR_VALUE, "plan must not be NULL");
    const size_t ws_need = p->image.bytes - p->image.off_part_o;
    if (ws_need > 0 && (!workspace || workspace_bytes < ws_need))
        return fail(PD_ERR_VALUE, "workspace is NULL or smaller than pd_plan_workspace_bytes()");
    if (reinterpret_cast<uintptr_t>(workspace) & 255)
        return fail(PD_ERR_VALUE, "workspace must be 256-byte aligned");
    const pd_status s = bind_impl(p, metadata, metadata_bytes, p->image.off_part_o, stream);
    if (s != PD_OK) return s;
    p->ws = ws_need > 0 ? static_cast<uint8_t *>(workspace) : nullptr;
    return PD_OK;
}

PD_API pd_status pd_decode(pd_plan *p, const void *q, const void *k, const void *v, pd_dtype dtype,
                           float *out, void *stream) {
    return decode_impl(p, q, k, v, dtype, out, nullptr, stream);
}

PD_API pd_status pd_decode_dynamic(pd_plan *p, const void *q, const void *k, const void *v, pd_dtype dtype,
                                   const int32_t *table, const int32_t *lengths, float *out, float *stats,
                                   void *stream) {
    if (p && !p->dynamic) return fail(PD_ERR_VALUE, "plan was not built by pd_plan_create_dynamic");
    if (!table || !lengths) return fail(PD_ERR_VALUE, "table and lengths must not be NULL");
    if ((reinterpret_cast<uintptr_t>(table) | reinterpret_cast<uintptr_t>(lengths)) & 3)
        return fail(PD_ERR_VALUE, "table and lengths must be 4-byte aligned");
    return decode_impl(p, q, k, v, dtype, out, stats, stream, table, lengths);
}

PD_API pd_status pd_decode_with_stats(pd_plan *p, const void *q, const void *k, const void *v,
                                      pd_dtype dtype, float *out, float *stats, void *stream) {
    if (!stats) return fail(PD_ERR_VALUE, "stats must not be NULL");
    return decode_impl(p, q, k, v, dtype, out, stats, stream);
}

PD_API pd_status pd_merge_shards(const float *shard_out, const float *shard_stats, int32_t shards,
                                 int64_t shard_stride, int64_t rows, int32_t head_dim, float *out,
                                 void *stream) {
    if (!shard_out || !shard_stats || !out) return fail(PD_ERR_VALUE, "pointers must not be NULL");
    if (shards < 1 || rows < 0 || head_dim <= 0 || (head_dim & 31))
        return fail(PD_ERR_VALUE, "shards >= 1, rows >= 0 and head_dim a positive multiple of 32 required");
    if (shards > 1 && shard_stride < rows * head_dim)
        return fail(PD_ERR_VALUE, "shard_stride must cover a shard's rows * head_dim outputs");
    if (reinterpret_cast<uintptr_t>(shard_stats) & 7)
        return fail(PD_ERR_VALUE, "shard_stats must be 8-byte aligned");
    if (rows == 0) return PD_OK;
    if ((rows + 7) / 8 > INT32_MAX) return fail(PD_ERR_VALUE, "too many rows");
    const cudaError_t err =
        launch_merge_shards(shard_out, shard_stats, shards, shard_stride, rows, head_dim, out,
                            static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess)
        return fail(PD_ERR_CUDA, std::string("merge launch: ") + cudaGetErrorString(err));
    return PD_OK;
}

// ---------------------------------------------------------------------------
// Decode without any device allocation by the caller or the library.
//
// Callers that cannot call cudaMalloc (a host program whose device memory is
// owned and pooled by another framework, a plugin that may only touch the
// buffers it is handed, code running where allocation is forbidden) still
// need somewhere to put a plan's metadata and split-K partials.  This entry
// point uses one file-scope device array instead: every GPU that loads this
// library holds it (kStaticScratchBytes) until the process exits.
namespace pd {
namespace {
constexpr size_t kStaticScratchBytes = size_t(16) << 20;
static __device__ __align__(256) uint8_t g_static_scratch[kStaticScratchBytes];

std::mutex g_static_mutex;
constexpr int kMaxDevices = 256;
uint8_t *g_static_address[kMaxDevices] = {};

// The symbol names a host-side stand-in; the device address must come from
// cudaGetSymbolAddress, taken once per device with that device current.
pd_status static_scratch(int device, uint8_t **out) {
    if (device < 0 || device >= kMaxDevices) return fail(PD_ERR_VALUE, "device index out of range");
    std::lock_guard<std::mutex> lock(g_static_mutex);
    if (!g_static_address[device]) {
        void *ptr = nullptr;
        const cudaError_t err = cudaGetSymbolAddress(&ptr, g_static_scratch);
        if (err != cudaSuccess || !ptr)
            return fail(PD_ERR_CUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(err));
        g_static_address[device] = static_cast<uint8_t *>(ptr);
    }
    *out = g_static_address[device];
    return PD_OK;
}
}  // namespace
}  // namespace pd

PD_API size_t pd_static_scratch_capacity(void) { return kStaticScratchBytes; }

PD_API pd_status pd_decode_static(pd_plan *p, const void *q, const void *k, const void *v, pd_dtype dtype,
                                  float *out, void *stream) {
    if (!p) return fail(PD_ERR_VALUE, "plan must not be NULL");
    if (p->device < 0) return fail(PD_ERR_VALUE, "host-only plan (device < 0) cannot launch");
    // A dynamic plan decodes live metadata that only pd_decode_dynamic takes.
    if (p->dynamic)
        return fail(PD_ERR_VALUE, "pd_decode_static takes plans from pd_plan_create; "
                                  "a dynamic plan needs pd_decode_dynamic");
    pd_status s = check_dtype(p, dtype);
    if (s != PD_OK) return s;
    if (!q || !out) return fail(PD_ERR_VALUE, "q and out must not be NULL");
    if ((reinterpret_cast<uintptr_t>(q) & 15) || (reinterpret_cast<uintptr_t>(out) & 15))
        return fail(PD_ERR_VALUE, "q and out must be 16-byte aligned");
    if (p->image.bytes > kStaticScratchBytes)
        return fail(PD_ERR_VALUE, "plan needs " + std::to_string(p->image.bytes) +
                                      " bytes of scratch; pd_decode_static has " +
                                      std::to_string(kStaticScratchBytes));
    DeviceGuard guard(p->device);
    if (guard.err != cudaSuccess)
        return fail(PD_ERR_CUDA, std::string("cudaSetDevice: ") + cudaGetErrorString(guard.err));
    uint8_t *scratch = nullptr;
    if ((s = static_scratch(p->device, &scratch)) != PD_OK) return s;
    // This call's metadata (and a zeroed error word) replace whatever the last
    // call left in the shared array; partial slots are always written before
    // they are read, so they need no clearing.
    const auto st = static_cast<cudaStream_t>(stream);
    const cudaError_t err =
        cudaMemcpyAsync(scratch, p->host_image.data(), p->host_image.size(), cudaMemcpyHostToDevice, st);
    if (err != cudaSuccess)
        return fail(PD_ERR_CUDA, std::string("scratch upload: ") + cudaGetErrorString(err));
    const DecodeArgs args = make_args_at(p, scratch, q, out, nullptr);
    return launch(p, k, v, dtype, kModeDecode, args, stream);
}

PD_API pd_status pd_static_read_errors(int32_t device, uint32_t *error_word, void *stream) {
    if (!error_word) return fail(PD_ERR_VALUE, "error_word must not be NULL");
    DeviceGuard guard(device);
    if (guard.err != cudaSuccess)
        return fail(PD_ERR_CUDA, std::string("cudaSetDevice: ") + cudaGetErrorString(guard.err));
    uint8_t *scratch = nullptr;
    pd_status s = static_scratch(device, &scratch);
    if (s != PD_OK) return s;
    // Every plan image starts with its error word (offset 0), so the last
    // static call's word sits at the start of the array.
    auto st = static_cast<cudaStream_t>(stream);
    uint32_t word = 0;
    cudaError_t err = cudaMemcpyAsync(&word, scratch, 4, cudaMemcpyDeviceToHost, st);
    if (err == cudaSuccess) err = cudaMemsetAsync(scratch, 0, 4, st);
    if (err == cudaSuccess) err = cudaStreamSynchronize(st);
    if (err != cudaSuccess)
        return fail(PD_ERR_CUDA, std::string("static error word read: ") + cudaGetErrorString(err));
    *error_word = word;
    return PD_OK;
}

PD_API pd_status pd_gather_debug(pd_plan *p, const void *k, const void *v, pd_dtype dtype,
                                 void *dense_k, void *dense_v, void *stream) {
    pd_status s = check_bound(p);
    if (s != PD_OK) return s;
    if ((s = check_dtype(p, dtype)) != PD_OK) return s;
    if (!dense_k || !dense_v) return fail(PD_ERR_VALUE, "dense outputs must not be NULL");
    if ((reinterpret_cast<uintptr_t>(dense_k) | reinterpret_cast<uintptr_t>(dense_v)) & 15)
        return fail(PD_ERR_VALUE, "dense outputs must be 16-byte aligned");
    DeviceGuard guard(p->device);
    if (guard.err != cudaSuccess)
        return fail(PD_ERR_CUDA, std::string("cudaSetDevice: ") + cudaGetErrorString(guard.err));
    DecodeArgs args = make_args(p, nullptr, nullptr, nullptr);
    args.dense_k = dense_k;
    args.dense_v = dense_v;
    return launch(p, k, v, dtype, kModeGather, args, stream);
}

PD_API pd_status pd_plan_set_barrier(pd_plan *p, int32_t mode) {
    if (!p) return fail(PD_ERR_VALUE, "plan must not be NULL");
    if (mode != PD_BARRIER_PLAIN && mode != PD_BARRIER_COOPERATIVE && mode != PD_BARRIER_LEAVE_AT_ONCE)
        return fail(PD_ERR_VALUE, "barrier mode must be PD_BARRIER_PLAIN, _COOPERATIVE or _LEAVE_AT_ONCE");
    p->barrier_mode = mode;
    return PD_OK;
}

PD_API pd_status pd_plan_read_barrier_fallbacks(pd_plan *p, uint32_t *count, void *stream) {
    pd_status s = check_bound(p);
    if (s != PD_OK) return s;
    if (!count) return fail(PD_ERR_VALUE, "count must not be NULL");
    DeviceGuard guard(p->device);
    auto st = static_cast<cudaStream_t>(stream);
    uint32_t word = 0;
    cudaError_t err = cudaMemcpyAsync(&word, p->dev + p->image.off_error + 4, 4, cudaMemcpyDeviceToHost, st);
    if (err == cudaSuccess) err = cudaMemsetAsync(p->dev + p->image.off_error + 4, 0, 4, st);
    if (err == cudaSuccess) err = cudaStreamSynchronize(st);
    if (err != cudaSuccess)
        return fail(PD_ERR_CUDA, std::string("fallback count read: ") + cudaGetErrorString(err));
    *count = word;
    return PD_OK;
}

PD_API pd_status pd_plan_read_errors(pd_plan *p, uint32_t *error_word, void *stream) {
    pd_status s = check_bound(p);
    if (s != PD_OK) return s;
    if (!error_word) return fail(PD_ERR_VALUE, "error_word must not be NULL");
    DeviceGuard guard(p->device);
    auto st = static_cast<cudaStream_t>(stream);
    uint32_t word = 0;
    cudaError_t err = cudaMemcpyAsync(&word, p->dev + p->image.off_error, 4, cudaMemcpyDeviceToHost, st);
    if (err == cudaSuccess) err = cudaMemsetAsync(p->dev + p->image.off_error, 0, 4, st);
    if (err == cudaSuccess) err = cudaStreamSynchronize(st);
    if (err != cudaSuccess)
        return fail(PD_ERR_CUDA, std::string("error word read: ") + cudaGetErrorString(err));
    *error_word = word;
    return PD_OK;
}

PD_API const char *pd_status_string(pd_status status) {
    switch (status) {
        case PD_OK: return "ok";
        case PD_ERR_VALUE: return "invalid value";
        case PD_ERR_TYPE: return "invalid dtype";
        case PD_ERR_CUDA: return "CUDA error";
        case PD_ERR_DEVICE: return "device error word set";
        case PD_ERR_UNBOUND: return "plan not bound to a device buffer";
    }
    return "unknown status";
}

PD_API const char *pd_last_error(void) { return pd::last_error().c_str(); }

PD_API int32_t pd_abi_version(void) { return PD_ABI_VERSION; }

// ------------------------------------------------------------------ peer exchange (sequence sharding)
PD_API size_t pd_exchange_bytes(const pd_plan *p, int32_t world) {
    if (!p || world < 1 || world > kMaxRanks) return 0;
    return size_t(kXRecv + 2 * int64_t(world) * exchange_slot_bytes(p));
}

PD_API pd_status pd_exchange_alloc(int32_t device, size_t bytes, void **buffer, void *ipc_handle) {
    if (!buffer || !ipc_handle || bytes == 0) return fail(PD_ERR_VALUE, "buffer, ipc_handle and bytes are required");
    *buffer = nullptr;
    DeviceGuard guard(device);
    if (guard.err != cudaSuccess)
        return fail(PD_ERR_CUDA, std::string("cudaSetDevice: ") + cudaGetErrorString(guard.err));
    void *ptr = nullptr;
    cudaError_t err = cudaMalloc(&ptr, bytes);
    if (err == cudaSuccess) err = cudaMemset(ptr, 0, bytes);   // arrival counter and launch counts start at 0
    cudaIpcMemHandle_t h;
    if (err == cudaSuccess) err = cudaIpcGetMemHandle(&h, ptr);
    if (err != cudaSuccess) {
        if (ptr) cudaFree(ptr);
        return fail(PD_ERR_CUDA, std::string("exchange buffer: ") + cudaGetErrorString(err));
    }
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handles are 64 bytes");
    std::memcpy(ipc_handle, &h, sizeof(h));
    *buffer = ptr;
    return PD_OK;
}

PD_API pd_status pd_exchange_open(int32_t device, const void *ipc_handle, void **peer_buffer) {
    if (!ipc_handle || !peer_buffer) return fail(PD_ERR_VALUE, "ipc_handle and peer_buffer are required");
    *peer_buffer = nullptr;
    DeviceGuard guard(device);
    if (guard.err != cudaSuccess)
        return fail(PD_ERR_CUDA, std::string("cudaSetDevice: ") + cudaGetErrorString(guard.err));
    cudaIpcMemHandle_t h;
    std::memcpy(&h, ipc_handle, sizeof(h));
    const cudaError_t err = cudaIpcOpenMemHandle(peer_buffer, h, cudaIpcMemLazyEnablePeerAccess);
    if (err != cudaSuccess) return fail(PD_ERR_CUDA, std::string("peer buffer: ") + cudaGetErrorString(err));
    return PD_OK;
}

PD_API pd_status pd_exchange_close(int32_t device, void *peer_buffer) {
    DeviceGuard guard(device);
    const cudaError_t err = cudaIpcCloseMemHandle(peer_buffer);
    if (err != cudaSuccess) return fail(PD_ERR_CUDA, std::string("close peer buffer: ") + cudaGetErrorString(err));
    return PD_OK;
}

PD_API pd_status pd_exchange_free(int32_t device, void *buffer) {
    DeviceGuard guard(device);
    const cudaError_t err = cudaFree(buffer);
    if (err != cudaSuccess) return fail(PD_ERR_CUDA, std::string("free exchange buffer: ") + cudaGetErrorString(err));
    return PD_OK;
}

PD_API pd_status pd_decode_exchange(pd_plan *p, const void *q, const void *k, const void *v, pd_dtype dtype,
                                    void *const *buffers, int32_t rank, int32_t world, float *out,
                                    float *stats, void *stream) {
    if (!p) return fail(PD_ERR_VALUE, "plan must not be NULL");
    if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world)
        return fail(PD_ERR_VALUE, "world must be in [1, 8] and rank in [0, world)");
    if (!buffers) return fail(PD_ERR_VALUE, "buffers must not be NULL");
    for (int s = 0; s < world; ++s)
        if (!buffers[s] || (reinterpret_cast<uintptr_t>(buffers[s]) & 255))
            return fail(PD_ERR_VALUE, "exchange buffers must be non-NULL and 256-byte aligned");
    if (p->num_ctas > 1024) return fail(PD_ERR_VALUE, "exchange mode supports at most 1024 CTAs per rank");
    if (p->cluster != 1)
        return fail(PD_ERR_VALUE, "exchange mode needs a plan without CTA pairs (create it with num_ctas > 0)");
    DecodeArgs x{};
    for (int s = 0; s < world; ++s) x.xpeer[s] = static_cast<uint8_t *>(buffers[s]);
    x.xslot = exchange_slot_bytes(p);
    x.xrank = rank;
    x.xworld = world;
    return decode_impl(p, q, k, v, dtype, out, stats, stream, nullptr, nullptr, &x);
}
