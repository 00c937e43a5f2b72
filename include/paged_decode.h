/* paged_decode.h — C ABI of the B200 (sm_100a) paged split-K GQA decode operator.
 *
 * Drop-in boundary for ensigncode/paged-decode-lab.  The reference binds one
 * pybind entry, ext.decode(q, k, v, table, lengths, numerator, stats, out,
 * split_tokens, merge_mode) (src/paged_decode/csrc/bindings.cpp:9 ->
 * decode_cuda, src/paged_decode/csrc/decode.cu:197-246), behind the Python
 * DecodePlan (src/paged_decode/runtime.py:23-90).  This header splits that
 * into a host-side plan (built once from CPU metadata, like DecodePlan.__init__)
 * and an allocation-free decode call (like DecodePlan.run).  Only plain C
 * types cross it: no torch types, no exceptions; every call returns a
 * pd_status and pd_last_error() gives the message.
 *
 * Layouts (as in the reference, decode.cu:59-60):
 *   q      [batch, query_heads, head_dim]                 float16 | float32
 *   k, v   [physical_pages, page_size, kv_heads, head_dim] same dtype as q
 *   table  [batch, table_width] int32, -1 allowed past each row's live pages
 *   lengths[batch] int32
 *   out    [batch, query_heads, head_dim] float32
 * Query head h reads KV head h / (query_heads / kv_heads); scores are scaled
 * by 1/sqrt(head_dim); an empty sequence yields a zero row.
 *
 * Device memory is owned by the caller: pd_plan_device_bytes() says how many
 * bytes one plan needs (metadata + split-K workspace), the caller allocates
 * them (cudaMalloc, a torch tensor, ...) and hands them to pd_plan_bind().
 * pd_decode() allocates nothing, never synchronises and may be captured in a
 * CUDA graph.  A plan may be used on one stream at a time.
 */
#ifndef PAGED_DECODE_B200_H
#define PAGED_DECODE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PD_ABI_VERSION 8

typedef enum pd_status {
    PD_OK = 0,
    PD_ERR_VALUE = 1,        /* bad shape, limit, pointer or state (Python: ValueError)  */
    PD_ERR_TYPE = 2,         /* unsupported dtype (Python: TypeError)                    */
    PD_ERR_CUDA = 3,         /* a CUDA runtime/driver call failed (Python: RuntimeError) */
    PD_ERR_DEVICE = 4,       /* a kernel raised its error word (Python: RuntimeError)    */
    PD_ERR_UNBOUND = 5       /* plan has no device buffer yet (Python: RuntimeError)     */
} pd_status;

typedef enum pd_dtype { PD_FLOAT16 = 0, PD_FLOAT32 = 1 } pd_dtype;

/* Error-word bits a kernel can raise (read with pd_plan_read_errors). */
#define PD_DEVERR_TIMEOUT 1u      /* a bounded wait on a shared-memory barrier ran out */
#define PD_DEVERR_BAD_PAGE 2u     /* a live page id outside [0, physical_pages): tokens skipped */
#define PD_DEVERR_LENGTH 8u       /* a dynamic launch's length exceeded the plan's max_lengths: clamped */

/* Replaces oracle.Layout (src/paged_decode/oracle.py:11-27). */
typedef struct pd_layout {
    int32_t batch;
    int32_t query_heads;
    int32_t kv_heads;
    int32_t head_dim;        /* 64 or 128 */
    int32_t page_size;       /* 16 or 32  */
    int64_t physical_pages;
} pd_layout;

typedef struct pd_plan pd_plan;

typedef struct pd_plan_info {
    int32_t splits;          /* max(1, ceil(max_context / split_tokens)), runtime.py:49 */
    int32_t max_context;     /* max(lengths) */
    int32_t num_ctas;        /* persistent CTAs the decode kernel launches */
    int32_t num_segments;    /* (group, page range) work segments over all CTAs */
    int32_t num_groups;      /* (sequence, KV-head group, query-head tile) groups */
    int32_t num_pieces;      /* partial slots written by the decode kernel and merged after it */
    int32_t slot_stride;     /* partial slots per segment (1: a CTA folds its sub-pipelines first) */
    int32_t group_tile;      /* query heads per group tile (8, 16 or 32) */
    int32_t heads_per_tile;  /* KV heads gathered per page tile (1, 2, 4 or 8) */
    int32_t total_pages;     /* page tiles streamed per decode (all groups) */
    int32_t merge_rows;      /* output rows merged from partials after the decode */
    int32_t merge_in_kernel; /* 1: the decode CTAs merge them after a grid barrier
                                (num_ctas <= SMs; see pd_plan_set_barrier), 0: a dependent
                                merge kernel does */
    int32_t dynamic;         /* 1: built by pd_plan_create_dynamic */
    int32_t max_span;        /* longest sequence the work list covers (max_lengths, else lengths) */
    int64_t workspace_bytes; /* split-K partials, o and (m, l) (pd_plan_workspace_bytes) */
    int64_t device_bytes;    /* everything pd_plan_bind needs (metadata + workspace) */
    int32_t engine;          /* consumer engine of the decode kernel: PD_ENGINE_WARP (every
                                consumer warp runs m16n8k16 MMAs or FP32 FMAs) or
                                PD_ENGINE_TCGEN05 (FP16 group tiles of 32 query heads, head_dim
                                128, 32-token pages; any FP16 32-head tile when the environment
                                has PD_MQA_ENGINE=tcgen05 at plan creation, none with
                                PD_MQA_ENGINE=warp: single threads issue the MMAs into tensor
                                memory) */
    int32_t cluster_ctas;    /* CTAs per thread-block cluster of the decode launch: 1, or 2 for a
                                pair plan (tcgen05 engine, num_ctas <= 0 at creation, groups of
                                near-equal length that fill at least 3/4 of the SMs two CTAs
                                each, and on a device only if all its clusters fit at once;
                                PD_PAIR=0 / 1 in the environment at plan creation turns
                                it off / on wherever the groups fit): the two CTAs of a cluster
                                stream the two halves of one group and merge them through
                                distributed shared memory, with no partials, grid barrier or
                                merge kernel.  pd_decode_exchange rejects pair plans. */
} pd_plan_info;

#define PD_ENGINE_WARP 0
#define PD_ENGINE_TCGEN05 1

/* Build a plan from host metadata.  Replaces DecodePlan.__init__'s checks and
 * split planning (runtime.py:32-69) and decode_cuda's validation
 * (decode.cu:201-237).  Copies table and lengths.  merge_mode 0 = "serial",
 * 1 = "shared" is accepted for API compatibility (runtime.py:33-34); the
 * decode always merges split partials the same way (the decode CTAs after a
 * grid barrier when num_ctas <= SMs, else a dependent merge kernel launched
 * right behind the decode kernel).  A plan serves one input dtype:
 * the page tiles it gathers are sized for it (the Python DecodePlan keeps one
 * plan per dtype behind its dtype-agnostic run()).  device < 0 builds a
 * host-only plan (inspection, no decode).  num_ctas <= 0 picks one CTA per SM
 * of device, or two CTAs per group in clusters of two (a pair plan, see
 * pd_plan_info.cluster_ctas).
 */
pd_status pd_plan_create(const pd_layout *layout, const int32_t *table, int64_t table_width,
                         const int32_t *lengths, int32_t split_tokens, int32_t merge_mode,
                         pd_dtype dtype, int32_t device, int32_t num_ctas, pd_plan **out_plan);

/* A dynamic plan: as pd_plan_create, but the work list covers sequence b up
 * to max_lengths[b] tokens (lengths[b] <= max_lengths[b] <= table_width *
 * page_size), so that a decode loop can grow its sequences without a new
 * plan: pd_decode_dynamic takes the live page table and lengths from device
 * memory at every launch.  Page ids past lengths[b] may be -1 here.  No
 * reference counterpart: the reference needs a new plan whenever a length
 * changes (runtime.py:25-30).
 */
pd_status pd_plan_create_dynamic(const pd_layout *layout, const int32_t *table, int64_t table_width,
                                 const int32_t *lengths, const int32_t *max_lengths, int32_t split_tokens,
                                 int32_t merge_mode, pd_dtype dtype, int32_t device, int32_t num_ctas,
                                 pd_plan **out_plan);

void pd_plan_destroy(pd_plan *plan);

pd_status pd_plan_get_info(const pd_plan *plan, pd_plan_info *info);

/* Work list, for inspection and tests: segments as int32 quadruples
 * (group, first_page, end_page, first partial slot or -1), groups as int32
 * octuples (batch, first_kv_head, query_head_offset, query_heads, length,
 * first partial slot or -1, segments, 0): the group covers heads_per_tile KV
 * heads from first_kv_head and, of each one's G query heads, query_heads of
 * them from query_head_offset; slot -1 means the output is written directly;
 * cta_offsets receives the per-CTA segment offsets [num_ctas + 1].  Any
 * pointer may be NULL.
 */
pd_status pd_plan_copy_worklist(const pd_plan *plan, int32_t *segments, int32_t *groups,
                                int32_t *cta_offsets);

size_t pd_plan_device_bytes(const pd_plan *plan);

/* Give the plan its device buffer (>= pd_plan_device_bytes, 256-byte aligned,
 * on the plan's device) and upload metadata on `stream` (a cudaStream_t; NULL
 * = legacy default stream).  Synchronises that stream.  May be called again
 * to move the plan to a new buffer or to clear its error word and counters.
 */
pd_status pd_plan_bind(pd_plan *plan, void *device_buffer, size_t bytes, void *stream);

/* The two parts of pd_plan_device_bytes(): the plan's metadata (page table,
 * work list, error word and barrier counters; uploaded by the bind) and its
 * split-K workspace (partial outputs, written and read within each launch).
 * Replace DecodePlan.workspace_bytes (runtime.py:71-73), which counts the
 * reference's numerator and stats tensors. */
size_t pd_plan_metadata_bytes(const pd_plan *plan);
size_t pd_plan_workspace_bytes(const pd_plan *plan);

/* As pd_plan_bind, with the metadata and the workspace in separate buffers
 * (each >= its size above, 256-byte aligned; the workspace may be NULL when
 * its size is 0).  A workspace carries nothing from one launch to the next,
 * so plans whose launches stay in one stream order may share one (the Python
 * DecodePlan binds its FP16 and FP32 plans to one workspace of the larger
 * size).  No reference counterpart. */
pd_status pd_plan_bind_split(pd_plan *plan, void *metadata, size_t metadata_bytes, void *workspace,
                             size_t workspace_bytes, void *stream);

/* One decode step.  Replaces ext.decode / decode_cuda (bindings.cpp:9,
 * decode.cu:197-246).  out receives FP32 [batch, query_heads, head_dim].
 * k and v must be 16-byte aligned (TMA); dtype must be the plan's.
 * Asynchronous on `stream`: one decode kernel (which also merges the
 * partials after a grid barrier when the plan has some and num_ctas <= SMs;
 * see pd_plan_set_barrier), or the decode kernel and a dependent merge
 * kernel.  Launches of one plan must stay in one stream order: they share the
 * plan's partial slots and barrier counters.
 */
pd_status pd_decode(pd_plan *plan, const void *q, const void *k, const void *v, pd_dtype dtype,
                    float *out, void *stream);

/* As pd_decode, and also writes stats[batch, query_heads, 2] = (m, l): the
 * running maximum of score*log2(e)/sqrt(head_dim) and the softmax denominator
 * relative to it (m = -inf, l = 0 for an empty sequence).  Used by sequence
 * sharding: each GPU decodes its page range, then pd_merge_shards combines.
 * No reference counterpart (the reference never ran on more than one GPU).
 */
pd_status pd_decode_with_stats(pd_plan *plan, const void *q, const void *k, const void *v,
                               pd_dtype dtype, float *out, float *stats, void *stream);

/* One decode step of a dynamic plan with live metadata in device memory:
 * table int32 [batch, table_width] (the plan's width) and lengths int32
 * [batch], read when the kernel runs, so a CUDA graph of "update metadata,
 * decode" replays without host work.  Pages at or past lengths[b] are
 * skipped; a length above max_lengths[b] is clamped to it and flags
 * PD_DEVERR_LENGTH; a live page id outside [0, physical_pages) is skipped and
 * flags PD_DEVERR_BAD_PAGE.  stats may be NULL.
 */
pd_status pd_decode_dynamic(pd_plan *plan, const void *q, const void *k, const void *v, pd_dtype dtype,
                            const int32_t *table, const int32_t *lengths, float *out, float *stats,
                            void *stream);

/* Max-corrected merge of per-shard results (the merge algebra of
 * oracle.py:88-96 applied across shards), as written by pd_decode_with_stats.
 * Shard s's normalised outputs (rows x head_dim floats) start at
 * shard_out + s * shard_stride and its (m, l) pairs (rows x 2 floats) at
 * shard_stats + s * shard_stride; shard_stride counts floats.  For one packed
 * buffer per shard ([rows * head_dim outputs][rows * 2 stats], the layout the
 * sequence-sharded all-gather produces) pass shard_stats = shard_out +
 * rows * head_dim and shard_stride = rows * (head_dim + 2).  Writes
 * out [rows, head_dim].  Device pointers on the current device.
 */
pd_status pd_merge_shards(const float *shard_out, const float *shard_stats, int32_t shards,
                          int64_t shard_stride, int64_t rows, int32_t head_dim, float *out,
                          void *stream);

/* Debug gather through the decode kernel's own TMA page path: writes the
 * live K and V rows of every (sequence, KV head) as dense
 * [batch, kv_heads, max_context, head_dim] arrays in the input dtype
 * (rows past a sequence's length are left untouched).  Bit-exact with
 * oracle.gather_cache (oracle.py:50-56) by construction; used by the tests.
 */
pd_status pd_gather_debug(pd_plan *plan, const void *k, const void *v, pd_dtype dtype,
                          void *dense_k, void *dense_v, void *stream);

/* As pd_decode, but with no device memory from the caller or the library.
 * No counterpart in the reference: it exists for callers that cannot call
 * cudaMalloc (their device memory is owned by another framework's pool, or
 * they may only touch the buffers they are handed).  The plan needs no
 * pd_plan_bind; its metadata and split-K partials go to one file-scope
 * device array of pd_static_scratch_capacity() bytes (16 MiB) that every
 * GPU loading this library holds until exit.  A plan needing more
 * (pd_plan_device_bytes) is rejected with PD_ERR_VALUE, and so is a dynamic
 * plan (its live metadata goes through pd_decode_dynamic).  Each call
 * uploads the plan's metadata from host memory into the array on `stream`
 * (overwriting the previous call's contents and zeroing its error word),
 * then launches.  All calls share the array: calls that overlap on the GPU
 * (other streams; each device has its own array) race.  The first call on a
 * device looks up the array's device address (cudaGetSymbolAddress, with
 * that device current) and keeps it for the life of the process; make that
 * first call before any stream capture, and none after a cudaDeviceReset.
 * Read the kernel's error word with pd_static_read_errors.  Allocates
 * nothing: no cudaMalloc, cudaFree or allocating library routine.
 */
pd_status pd_decode_static(pd_plan *plan, const void *q, const void *k, const void *v,
                           pd_dtype dtype, float *out, void *stream);

/* Size of the device array pd_decode_static uses (bytes). */
size_t pd_static_scratch_capacity(void);

/* The error word (PD_DEVERR_* bits) that the last pd_decode_static call on
 * `device` left in the array: copied to *error_word and cleared
 * (synchronises `stream`).  No counterpart in the reference; allocates
 * nothing. */
pd_status pd_static_read_errors(int32_t device, uint32_t *error_word, void *stream);

/* Copy the device error word to *error_word and clear it (synchronises `stream`). */
pd_status pd_plan_read_errors(pd_plan *plan, uint32_t *error_word, void *stream);

/* How a plan whose split rows are merged inside the decode kernel (pd_plan_info
 * merge_in_kernel) launches the grid barrier before the merge.  No reference
 * counterpart (the reference always merges with a second kernel).
 *   PD_BARRIER_PLAIN (default): a plain launch, so that it can start on SMs as
 *     the previous kernel's CTAs leave them.  Nothing then promises that all
 *     CTAs are resident together (an SM partition, a kernel in another stream),
 *     so a CTA that has waited at the barrier for 50 us while some CTA of the
 *     launch has not yet started leaves, and the CTA that completes the barrier
 *     merges the rows of those that left.  Same results, bit for bit.
 *   PD_BARRIER_COOPERATIVE: a cooperative launch: all CTAs resident, or it is
 *     refused and the separate merge kernel runs instead.
 *   PD_BARRIER_LEAVE_AT_ONCE: a plain launch in which every CTA that has to
 *     wait leaves at once (exercises the fallback; for tests).
 * Exchange launches (pd_decode_exchange) are always cooperative. */
#define PD_BARRIER_PLAIN 0
#define PD_BARRIER_COOPERATIVE 1
#define PD_BARRIER_LEAVE_AT_ONCE 2
pd_status pd_plan_set_barrier(pd_plan *plan, int32_t mode);

/* Launches since the last call whose barrier fell back to merging the rows of
 * CTAs that left; copies the count to *count and clears it (synchronises
 * `stream`). */
pd_status pd_plan_read_barrier_fallbacks(pd_plan *plan, uint32_t *count, void *stream);

const char *pd_status_string(pd_status status);
const char *pd_last_error(void);     /* message of this thread's last failing call */
int32_t pd_abi_version(void);

/* ------------------------------------------------------------------------
 * Sequence sharding over NVLink peer memory, one kernel per rank per step.
 * No reference counterpart (the reference never ran on more than one GPU).
 *
 * Each rank holds one exchange buffer of pd_exchange_bytes() bytes, made by
 * pd_exchange_alloc (cudaMalloc + a CUDA IPC handle) and opened by every
 * other rank of the node with pd_exchange_open.  pd_decode_exchange decodes
 * this rank's pages (its plan covers its share of every sequence) and stores
 * each finished row (normalised o, m, l) into this rank's slot of every
 * rank's buffer over NVLink, tagging it with the launch number after a
 * system-scope release fence.  Each output row is merged from the ranks'
 * copies (max-corrected merge) into out (and stats when not NULL) as soon as
 * all of them carry this launch's tag (bounded wait, PD_DEVERR_TIMEOUT).
 * Every rank must call it once per step, in the same order, with buffers[s] =
 * rank s's buffer as seen from this GPU (buffers[rank] = its own); at most
 * 1024 CTAs per rank.  No multicast and no library kernel touches peer
 * memory.  A pair plan (pd_plan_info.cluster_ctas == 2) is rejected with
 * PD_ERR_VALUE: create exchange plans with num_ctas > 0.
 */
size_t pd_exchange_bytes(const pd_plan *plan, int32_t world);
pd_status pd_exchange_alloc(int32_t device, size_t bytes, void **buffer, void *ipc_handle /* 64 bytes */);
pd_status pd_exchange_open(int32_t device, const void *ipc_handle, void **peer_buffer);
pd_status pd_exchange_close(int32_t device, void *peer_buffer);
pd_status pd_exchange_free(int32_t device, void *buffer);
pd_status pd_decode_exchange(pd_plan *plan, const void *q, const void *k, const void *v, pd_dtype dtype,
                             void *const *buffers, int32_t rank, int32_t world, float *out, float *stats,
                             void *stream);

/* Diagnostics, no reference counterpart: runs the decode kernel's two kinds
 * of bounded wait against events that never happen -- an mbarrier phase that
 * no thread completes (words[0]) and a grid barrier for two CTAs that only one
 * reaches (words[1]) -- each giving up after timeout_us (1 .. 1e6) and
 * recording PD_DEVERR_TIMEOUT in its word.  Proves the timeout path on a GPU
 * without a fault or a hang; synchronous on the default stream of `device`.
 */
pd_status pd_selftest_wait_timeouts(int32_t device, uint32_t timeout_us, uint32_t *words);

/* Diagnostics, no reference counterpart: one CTA reaches a grid barrier for two
 * CTAs in PD_BARRIER_PLAIN's leave mode, with leave_us (1 .. 1e5) as the wait
 * before leaving.  outcomes[0]: the partner has not started -- the CTA leaves
 * (2); outcomes[1]: the number of CTAs that left, as recorded in the barrier's
 * count (1); outcomes[2]: the CTA's left bit (1); outcomes[3]: the partner has
 * started but never arrives -- the CTA must stay, and times out after
 * 4 * leave_us (3).  Synchronous on the default stream of `device`. */
pd_status pd_selftest_barrier_leave(int32_t device, uint32_t leave_us, uint32_t *outcomes);

#ifdef __cplusplus
}
#endif

#endif /* PAGED_DECODE_B200_H */
