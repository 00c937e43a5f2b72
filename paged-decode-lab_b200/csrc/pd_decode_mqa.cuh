// pd_decode_mqa.cuh — the decode kernel for wide query groups (MQA-like:
// 17..32 query heads per KV head, FP16) on the 5th-generation tensor cores.
//
// Same work list, partials and merges as paged_decode_kernel
// (pd_decode_kernel.cuh; the reference's partial_decode + merge in
// src/paged_decode/csrc/decode.cu:26-168), with the streaming and consumer
// sides rebuilt around tcgen05.  A step is NP consecutive pages of one
// segment (NS = NP * T = 128 score columns):
//
//   * warp 7 (producer): lane 0 streams K a step at a time into step slots
//     laid out [page][8-token group][128-byte column][8 tokens][128 B] (one
//     8 KiB box per page: a column's 8-row groups sit a fixed stride apart over
//     the whole step), lane 1 a step's V pages into V step slots; the lanes
//     walk the work list independently;
//   * warp 2 stages each segment's 32 query rows in shared memory (128-byte
//     swizzled, K-major) two segments ahead;
//   * one thread of warp 3 issues S = Q K^T for a whole step once its K has
//     landed (M = 64 rows of which the 32 query heads are 0..31, N = NS, K =
//     16 head dims per MMA) into one of two score blocks in tensor memory;
//     one thread of warp 6, once a step's weights P are in shared memory and
//     its V pages have landed, issues O += P V page by page (N = head dim)
//     into one of two output blocks (consecutive segments alternate).  Two
//     issuing threads, so that neither kind waits for the other's inputs;
//   * warps 0 and 4 own query heads 0..15, warps 1 and 5 heads 16..31
//     (tensor-memory lanes 0..15 of sub-partitions 0 and 1); of each step's
//     columns a warp takes one half, two threads per head.  Online softmax in
//     base 2 with a lazily moved reference maximum: the two warps of a head
//     trade their row maxima each step, and only a maximum that passes the
//     reference by more than 2^8 moves it (and rescales the output block), so
//     weights stay <= 256 in FP16.  A segment's output block is read back
//     once the next segment's first weights are out and written exactly as
//     the warp-level kernel writes it (final row, exchange row or (m, l, o)
//     partial, m the true maximum).
//
// Pair plans launch clusters of two CTAs that stream the two halves of one
// group: each sends the partial (m, l, o) rows of the partner's 16 query heads
// into the partner's shared memory (its unused second query buffer) and
// keeps its own in weight buffer 0; after a cluster barrier each merges its
// 16 heads and writes the final rows, with no partials in global memory, no
// grid barrier and no merge kernel.
//
// mbarriers order the roles: K and V slot full/empty (TMA -> score / PV
// MMAs), q_full/q_empty (query rows), s_full (scores ready), p_full (weights
// written), p_free (the step's PV products done: its weights and V pages are
// free), o_free (an output block read back), pair (the two softmax warps of
// the same heads).  Every wait is bounded; on a timeout the CTA records
// PD_DEVERR_TIMEOUT, unwinds, waits for its own MMAs and frees its tensor
// memory.
#pragma once

#include "pd_decode_kernel.cuh"
#include "pd_tcgen05.cuh"

namespace pd {

template <int D, int T>
struct MqaShape {
    static constexpr int GT = 32;                       // query heads of a group tile: MMA rows 0..31
    // warps 0..6 (all merge at the end), warp 7 produces: eight warps, two per
    // SM sub-partition, so each thread may hold up to 255 registers
    static constexpr int NC = 7;
    static constexpr int THREADS = (NC + 1) * 32;
    static constexpr int W_Q = 2, W_MMA = 3, W_PV = 6;  // softmax: warps 0, 1, 4, 5
    static constexpr int M = 64;                        // MMA rows (the smallest cta_group::1 shape)
    static constexpr int ROW_BYTES = D * 2;
    static constexpr int NBOX = ROW_BYTES / 128;        // 128-byte boxes per token row
    static constexpr int HALF_BYTES = NBOX * T * 128;   // K (or V) rows of one page: [box][token]
    static constexpr int NS = 128;                      // score columns per step
    static constexpr int NP = NS / T;                   // pages per step
    static constexpr int KSTEPS = D / 16;               // K = 16 MMAs of S = Q K^T
    static constexpr int PSTEPS = T / 16;               // K = 16 MMAs of O += P V per page
    static constexpr int OCW = D / 64;                  // 32-column output blocks per softmax warp
    static constexpr int CW = NS / 64;                  // 32-column score blocks per softmax warp and step
    static constexpr int Q_BOX = GT * 128;              // one 128-byte box of the 32 query rows
    static constexpr int Q_BYTES = NBOX * Q_BOX;
    static constexpr int P_SBO = NS * 16;               // 8 rows of NS FP16 weights (8x8 core matrices)
    static constexpr int P_BYTES = (GT / 8) * P_SBO;
    // An M = 64 MMA reads 64 rows of A; rows 32..63 (never read back from
    // tensor memory) come from whatever follows the 32 written rows, which
    // must be allocated shared memory: shared memory holds [P0][P1][Q0][Q1]
    // [rings], so P buffer 1 reads on into the Q buffers and Q buffer 1 into
    // the rings.
    static constexpr int P_READ = (M / 8) * P_SBO;                      // from a P buffer's start
    static constexpr int Q_READ = (NBOX - 1) * Q_BOX + (M / 8) * 1024;  // from a Q buffer's start
    // tensor-memory columns: output blocks [0, D) and [D, 2 D) (alternate segments),
    // score blocks [2 D, 2 D + NS), [2 D + NS, 2 D + 2 NS)
    static constexpr int S_COL = 2 * D;
    static constexpr int TMEM_COLS = (S_COL + 2 * NS) <= 256 ? 256 : 512;
    static constexpr int NBARS = 20;   // s_full, p_full, p_free, q_full, q_empty, o_free, mma_done: 2 each; pair: 4
    static constexpr int XMAX_BYTES = 2 * 2 * 2 * 16 * 4;   // [pair phase][heads half][warp][row] row maxima
    static constexpr int XL_BYTES = 2 * 2 * 16 * 4;         // [heads half][warp][row] denominators
    static constexpr int PAIR_ML_BYTES = 2 * 16 * 8;        // pair plans: (m, l) of 16 rows, own and received
    // K arrives a step at a time into KSS step slots laid out [page][8-token
    // group][box][8 tokens][128 B], so one MMA takes a whole step's scores per
    // 16 head dims (its 8-row groups NBOX * 1024 bytes apart); a step
    // slot is free once those scores are done.  V also arrives a step at a time
    // (its NP pages on one mbarrier, [page][box][T tokens][128 B]) into VSS
    // step slots, each free once its PV products are done; the V ring holds two
    // steps and streams ahead with the rest.  A TMA stream refilled one 8 KiB
    // page per mbarrier reached about 19 GB/s per SM, four pages per mbarrier
    // 45 GB/s.  Per slot: full and empty mbarriers and a valid-page mask (20 bytes).
    static constexpr int KSTEP_BYTES = NBOX * NS * 128;
    static constexpr int VSTEP_BYTES = NP * HALF_BYTES;
    static constexpr int KSS = 2;
    static constexpr size_t FIXED = 1024 + 2 * size_t(P_BYTES) + 2 * size_t(Q_BYTES) + NBARS * 8 +
                                    PAIR_ML_BYTES + XMAX_BYTES + XL_BYTES + 16 + 16 + 16 + size_t(KSS) * (KSTEP_BYTES + 20);
    static constexpr int VFIT = int((232448 - FIXED) / (VSTEP_BYTES + 20));
    static constexpr int VSS = VFIT * NP > 48 ? 48 / NP : VFIT;   // V step slots (at most 48 pages)
    static constexpr size_t RING = size_t(KSS) * KSTEP_BYTES + size_t(VSS) * VSTEP_BYTES;   // [K steps][V steps]
    static constexpr size_t SMEM = FIXED + size_t(VSS) * (VSTEP_BYTES + 20);

    static_assert(D == 64 || D == 128, "head_dim 64 or 128");
    static_assert(T == 16 || T == 32, "page_size 16 or 32");
    static_assert(NS == 64 || NS == 128, "a step is 64 or 128 score columns");
    static_assert(P_READ <= P_BYTES + 2 * Q_BYTES, "P buffer 1's unread rows must stay inside the Q buffers");
    static_assert(Q_READ <= Q_BYTES + size_t(KSS) * KSTEP_BYTES, "Q buffer 1's unread rows must stay inside the rings");
    static_assert(S_COL + 2 * NS <= TMEM_COLS, "tensor memory budget");
    static_assert(NP * (T * 128) % 1024 == 0 && (T * 128) % 1024 == 0, "pages keep 1024-byte swizzle atoms");
    // a step's V pages are released after its PV products: the V ring must
    // hold two steps at once, and then some to stream ahead
    static_assert(VSS >= 3, "V ring too small for the steps in flight");
    // pair plans: 16 rows of D FP32 outputs in weight buffer 0 (own) and query buffer 1 (received)
    static_assert(16 * D * 4 <= P_BYTES && 16 * D * 4 <= Q_BYTES, "pair rows must fit their buffers");
    static_assert(SMEM <= 232448 && SMEM > 116 * 1024,
                  "one CTA per SM: its tensor memory is never contended by a second CTA of the grid");
};

// One thread's share of an output row: columns c0 + 32c + 16 half + [0, 16)
// (c < OCW) of the tensor-memory output block, scaled, as float4 stores.
template <int OCW>
__device__ __forceinline__ void store_o_part(float *dst, const uint32_t (&ov)[OCW][16], int c0, int half,
                                             float scale) {
#pragma unroll
    for (int c = 0; c < OCW; ++c)
#pragma unroll
        for (int e = 0; e < 16; e += 4)
            *reinterpret_cast<float4 *>(dst + c0 + 32 * c + 16 * half + e) =
                make_float4(__uint_as_float(ov[c][e]) * scale, __uint_as_float(ov[c][e + 1]) * scale,
                            __uint_as_float(ov[c][e + 2]) * scale, __uint_as_float(ov[c][e + 3]) * scale);
}

// Pair plans: the same share of row r (< 16) of a 16-row block, with row r's
// 16-byte chunk k stored at chunk k ^ r, so that the sixteen rows' threads
// storing (or, in the merge, loading) the same columns reach distinct banks.
template <int OCW>
__device__ __forceinline__ void store_pair_row(float *row, int r, const uint32_t (&ov)[OCW][16], int c0, int half,
                                               float scale) {
#pragma unroll
    for (int c = 0; c < OCW; ++c)
#pragma unroll
        for (int e = 0; e < 16; e += 4)
            *reinterpret_cast<float4 *>(row + 4 * (((c0 + 32 * c + 16 * half + e) >> 2) ^ r)) =
                make_float4(__uint_as_float(ov[c][e]) * scale, __uint_as_float(ov[c][e + 1]) * scale,
                            __uint_as_float(ov[c][e + 2]) * scale, __uint_as_float(ov[c][e + 3]) * scale);
}

__device__ __forceinline__ float max3f(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

// 2^x (hardware approximation; results below 2^-126 flush to 0, which FP16
// weights could not hold anyway).
__device__ __forceinline__ float ex2_ftz(float x) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

// Producer warp of the tcgen05 kernel: two lanes, each walking the CTA's work
// list on its own, so that neither kind of load waits for the other's slots.
//   lane 0, K by steps (NP consecutive pages of one segment): step s into step
//     slot s % KSS, one TMA load per page (the token-group view: page p at
//     p * HALF_BYTES), once the scores of step s - KSS are done;
//   lane 1, V by steps: step s into V step slot s % VSS, one TMA load per
//     page ([column][token], page p at p * HALF_BYTES), once the PV products
//     of step s - VSS are done.
// Pages past a dynamic plan's live length, or with an id outside the cache,
// land nothing and are marked invalid (a bit per page of the step).  Waits
// poll without suspending: the two lanes share one warp.
template <int T, int NP, int NS, int NBOX, int HALF_BYTES, int KSTEP_BYTES, int KSS, int VSS>
__device__ __forceinline__ void stream_mqa_pages(const CUtensorMap *tm_k, const CUtensorMap *tm_v,
                                                 const DecodeArgs &a, uint8_t *kring, uint8_t *vring,
                                                 uint64_t *kfull, uint64_t *kempty, uint64_t *vfull,
                                                 uint64_t *vempty, unsigned *kvalid, unsigned *vvalid,
                                                 SmemFlags *flags, int seg_begin, int seg_end, int lane) {
    if (lane > 1) return;
    tma_prefetch_descriptor(lane == 0 ? tm_k : tm_v);
    const auto claim = [&](uint64_t *empty, int use) -> bool {
        if (use == 0) return !flags->abort;
        const uint32_t bar = smem_u32(empty), par = (use - 1) & 1;
        const unsigned long long t0 = global_ns();
        while (!mbar_test_wait(bar, par)) {
            if (flags->abort) return false;
            if (global_ns() - t0 > kWaitTimeoutNs) {
                atomicOr(a.error, kErrTimeout);
                flags->abort = 1;
                return false;
            }
        }
        return true;
    };
    // 0: stream it; 1: not live yet; 2: id outside the cache (the reference
    // skips those tokens, decode.cu:58; plans validate ids, so this is defence only)
    const auto page_state = [&](int id, int64_t first_token, int live_end) {
        return first_token >= live_end ? 1 : (id >= 0 && int64_t(id) < a.P) ? 0 : 2;
    };
    int gs = 0;
    for (int si = seg_begin; si < seg_end; ++si) {
        const int4 sg = __ldg(a.segs + si);
        const int npg = sg.z - sg.y;
        if (npg == 0) continue;
        const int4 g0 = __ldg(a.groups + 2 * sg.x);
        const int32_t *trow = a.table + int64_t(g0.x) * a.W + sg.y;
        const int live_end = a.dynamic ? max(0, a.lengths[g0.x]) : INT_MAX;
        for (int p0 = 0; p0 < npg; p0 += NP) {
            const int n = min(NP, npg - p0);
            int ids[NP];
            unsigned mask = 0;
#pragma unroll
            for (int p = 0; p < NP; ++p) {
                ids[p] = p < n ? __ldg(trow + p0 + p) : 0;
                const int st = p < n ? page_state(ids[p], int64_t(sg.y + p0 + p) * T, live_end) : 1;
                if (st == 2 && lane == 0) atomicOr(a.error, kErrBadPage);
                if (st == 0) mask |= 1u << p;
            }
            if (lane == 0) {
                const int ks = gs % KSS;
                if (!claim(kempty + ks, gs / KSS)) return;
                const uint32_t fb = smem_u32(kfull + ks);
                kvalid[ks] = mask;
                if (mask) mbar_arrive_expect_tx(fb, uint32_t(__popc(mask)) * HALF_BYTES);
                else mbar_arrive(fb);
#pragma unroll
                for (int p = 0; p < NP; ++p)
                    if ((mask >> p) & 1u)
                        tma_load_5d(smem_u32(kring + size_t(ks) * KSTEP_BYTES + p * HALF_BYTES), tm_k, 0, 0,
                                    g0.y * NBOX, 0, ids[p], fb);
            } else {
                const int vs = gs % VSS;
                if (!claim(vempty + vs, gs / VSS)) return;
                const uint32_t fb = smem_u32(vfull + vs);
                vvalid[vs] = mask;
                if (mask) mbar_arrive_expect_tx(fb, uint32_t(__popc(mask)) * HALF_BYTES);
                else mbar_arrive(fb);
#pragma unroll
                for (int p = 0; p < NP; ++p)
                    if ((mask >> p) & 1u)
                        tma_load_5d(smem_u32(vring + (size_t(vs) * NP + p) * HALF_BYTES), tm_v, 0, 0, 0, g0.y, ids[p],
                                    fb);
            }
            ++gs;
        }
    }
}

template <int D, int T>
__global__ void __launch_bounds__(MqaShape<D, T>::THREADS, 1)
    paged_decode_mqa_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                            const DecodeArgs a) {
    using S = MqaShape<D, T>;
    constexpr int NC = S::NC, NS = S::NS, NP = S::NP, KSS = S::KSS, VSS = S::VSS, GT = S::GT, OCW = S::OCW,
                  CW = S::CW, HALF = S::HALF_BYTES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *pbuf = smem;                                   // [2][P_BYTES]
    uint8_t *qbuf = pbuf + 2 * S::P_BYTES;                  // [2][Q_BYTES]
    uint8_t *ring = qbuf + 2 * S::Q_BYTES;
    uint8_t *kring = ring;                                  // [KSS][box][NS tokens][128 B]
    uint8_t *vring = ring + size_t(KSS) * S::KSTEP_BYTES;   // [VSS][NP pages][box][T tokens][128 B]
    uint64_t *kfull = reinterpret_cast<uint64_t *>(ring + S::RING);
    uint64_t *kempty = kfull + KSS;
    uint64_t *vfull = kempty + KSS;
    uint64_t *vempty = vfull + VSS;
    uint64_t *s_full = vempty + VSS;        // [2] per score block
    uint64_t *p_full = s_full + 2;          // [2] per weight buffer
    uint64_t *p_free = p_full + 2;          // [2]
    uint64_t *q_full = p_free + 2;          // [2] per query buffer
    uint64_t *q_empty = q_full + 2;         // [2]
    uint64_t *pair_bar = q_empty + 2;       // [2 heads halves][2 phases]
    uint64_t *o_free = pair_bar + 4;        // [2] per output block
    uint64_t *mma_done = o_free + 2;        // [2] score MMAs, PV MMAs
    float2 *pair_ml = reinterpret_cast<float2 *>(mma_done + 2);   // pair plans: [own, received][16 rows]
    float *xmax = reinterpret_cast<float *>(pair_ml + 32);
    float *xl = xmax + S::XMAX_BYTES / 4;
    unsigned *svalid = reinterpret_cast<unsigned *>(xl + S::XL_BYTES / 4);   // [2]: pages streamed, per score block
    unsigned *kvalid = svalid + 4;                                           // [KSS]: pages streamed, per K step
    unsigned *vvalid = kvalid + KSS;                                         // [VSS]: pages streamed, per V step
    SmemFlags *flags = reinterpret_cast<SmemFlags *>(vvalid + VSS);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(flags + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int4 hv = lane < 12 ? __ldg(a.head + int64_t(blockIdx.x) * 16 + lane) : make_int4(0, 0, 0, 0);
    const int seg_begin = __shfl_sync(kFullMask, hv.x, 0);
    const int seg_end = __shfl_sync(kFullMask, hv.y, 0);

    if (threadIdx.x == 0) {
        for (int s = 0; s < KSS; ++s) {
            mbar_init(smem_u32(kfull + s), 1);
            mbar_init(smem_u32(kempty + s), 1);   // one commit of the score thread
        }
        for (int s = 0; s < VSS; ++s) {
            mbar_init(smem_u32(vfull + s), 1);
            mbar_init(smem_u32(vempty + s), 1);   // one commit of the PV thread
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(smem_u32(s_full + b), 2);      // the scores' commit and the MMA thread (svalid)
            mbar_init(smem_u32(p_full + b), 4);      // the four softmax warps
            mbar_init(smem_u32(p_free + b), 1);
            mbar_init(smem_u32(q_full + b), 1);
            mbar_init(smem_u32(q_empty + b), 1);
        }
        for (int i = 0; i < 4; ++i) mbar_init(smem_u32(pair_bar + i), 2);
        mbar_init(smem_u32(o_free), 4);
        mbar_init(smem_u32(o_free + 1), 4);
        mbar_init(smem_u32(mma_done), 1);
        mbar_init(smem_u32(mma_done + 1), 1);
        flags->abort = 0;
        mbar_init_fence();
    }
    if (warp == S::W_MMA) {
        tc::alloc(smem_u32(tmem_slot), S::TMEM_COLS);
        tc::relinquish_alloc_permit();
        tc::fence_before_sync();
    }
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    // pair plans: this CTA's rank in its cluster; both CTAs have started (their
    // shared memory may be written by the partner) once the barrier passes
    const uint32_t prank = a.pair ? cluster_ctarank() : 0u;
    if (a.pair) cluster_sync_all();

    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (a.fused_merge && threadIdx.x == 0) atomicAdd(a.gb.started, 1ull);
    const uint32_t xe = a.xworld
        ? __ldcv(reinterpret_cast<const unsigned int *>(a.xpeer[a.xrank] + kXEpochs) + blockIdx.x) + 1u : 0u;
    const int xpar = int(xe & 1u);

    if (warp == NC) {
        stream_mqa_pages<T, NP, NS, S::NBOX, HALF, S::KSTEP_BYTES, KSS, VSS>(
            &tm_k, &tm_v, a, kring, vring, kfull, kempty, vfull, vempty, kvalid, vvalid, flags, seg_begin, seg_end,
            lane);
        if (a.pair) cluster_sync_all();   // the partner's merge waits for every thread of both CTAs
        return;
    }

    const auto fail_wait = [&]() {
        if (!flags->abort) atomicOr(a.error, kErrTimeout);
        flags->abort = 1;
    };
    // A whole warp waits and decides together (a timed-out lane must not
    // leave its warp diverged at the next warp-wide instruction).
    const auto warp_wait = [&](uint64_t *bar, int parity) {
        return __all_sync(kFullMask, mbar_wait(smem_u32(bar), uint32_t(parity)));
    };
    const auto warp_abort = [&]() { return __any_sync(kFullMask, flags->abort != 0); };
    const int4 sg_h = shfl_int4(hv, 1), g0_h = shfl_int4(hv, 2), g1_h = shfl_int4(hv, 3);

    if (warp == S::W_Q) {
        // ------------------------------------------------------------ query rows
        // Segment sc (counting segments with pages) goes to buffer sc % 2 once
        // the score MMAs of segment sc - 2 are done: row g of the tile at
        // [box][row][128 B], 16-byte chunks XORed by row % 8 (the layout the
        // 128-byte-swizzle descriptor reads); rows past the group's heads are zero.
        int sc = 0;
        for (int si = seg_begin; si < seg_end && !warp_abort(); ++si) {
            const int4 sg = si == seg_begin ? sg_h : a.segs[si];
            if (sg.z == sg.y) continue;
            const int4 g0 = si == seg_begin ? g0_h : a.groups[2 * sg.x];
            const int qb = sc & 1;
            if (sc >= 2 && !warp_wait(q_empty + qb, ((sc >> 1) - 1) & 1)) {
                if (lane == 0) fail_wait();
                break;
            }
            const int nh = g0.w;
            const __half *qrow = static_cast<const __half *>(a.q) +
                                 (int64_t(g0.x) * a.Hq + int64_t(g0.y) * a.group + g0.z) * D;
            uint8_t *qs = qbuf + qb * S::Q_BYTES;
            constexpr int CPR = D / 8;   // 16-byte chunks per row
#pragma unroll 4
            for (int e = lane; e < GT * CPR; e += 32) {
                const int row = e / CPR, c = e % CPR;
                uint4 v = make_uint4(0u, 0u, 0u, 0u);
                if (row < nh) v = __ldg(reinterpret_cast<const uint4 *>(qrow + int64_t(row) * D) + c);
                *reinterpret_cast<uint4 *>(qs + swz128<GT>(row, c)) = v;
            }
            tc::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(q_full + qb));
            ++sc;
        }
    } else if (warp == S::W_MMA) {
        // ------------------------------------------------------------ score MMAs (one thread)
        // S = Q K^T for a step once its K has landed (one MMA per 16 head dims
        // over all NS tokens of the step), into score block gs % 2 once the
        // weights of step gs - 2 (which read that block) are written.
        if (lane == 0) {
            constexpr uint32_t ID_S = tc::idesc_f16_f32(S::M, NS, false, false);   // Q, K: K-major
            bool stop = false;
            int gs = 0, sc = 0;
            for (int si = seg_begin; si < seg_end && !stop; ++si) {
                const int4 sg = si == seg_begin ? sg_h : a.segs[si];
                const int npg = sg.z - sg.y;
                if (npg == 0) continue;
                const int qb = sc & 1;
                if (!mbar_wait(smem_u32(q_full + qb), (sc >> 1) & 1)) {
                    stop = true;
                    break;
                }
                const uint32_t qa = smem_u32(qbuf + qb * S::Q_BYTES);
                for (int p0 = 0; p0 < npg; p0 += NP) {
                    const int n = min(NP, npg - p0);
                    const int b = gs & 1;
                    if (flags->abort || (gs >= 2 && !mbar_wait(smem_u32(p_full + b), ((gs >> 1) - 1) & 1))) {
                        stop = true;
                        break;
                    }
                    const int ks = gs % KSS;
                    if (!mbar_wait(smem_u32(kfull + ks), (gs / KSS) & 1)) {
                        stop = true;
                        break;
                    }
                    tc::fence_after_sync();
                    // pages past the step's n, or not streamed, leave stale rows: their
                    // score columns are masked by the softmax
                    const unsigned valid = kvalid[ks] & ((1u << n) - 1u);
                    if (valid) {
                        const uint32_t kb = smem_u32(kring + size_t(ks) * S::KSTEP_BYTES);
#pragma unroll
                        for (int kk = 0; kk < S::KSTEPS; ++kk) {
                            const uint32_t koff = (kk >> 2) * 1024 + (kk & 3) * 32;
                            const uint64_t ad = tc::smem_desc(qa + (kk >> 2) * S::Q_BOX + (kk & 3) * 32, 16, 1024,
                                                              tc::kSwizzle128);
                            const uint64_t bd = tc::smem_desc(kb + koff, 16, S::NBOX * 1024, tc::kSwizzle128);
                            tc::mma_f16(tmem + S::S_COL + b * NS, ad, bd, ID_S, kk > 0 ? 1u : 0u);
                        }
                    }
                    tc::commit(smem_u32(kempty + ks));   // the step's K, once these scores are done
                    tc::commit(smem_u32(s_full + b));
                    svalid[b] = valid;
                    mbar_arrive(smem_u32(s_full + b));
                    if (p0 + NP >= npg) tc::commit(smem_u32(q_empty + qb));   // the segment's query rows
                    ++gs;
                }
                ++sc;
            }
            if (stop) fail_wait();
            // every score MMA has finished before the ring is reused or freed
            tc::commit(smem_u32(mma_done));
            if (!mbar_wait(smem_u32(mma_done), 0)) fail_wait();
        }
        __syncwarp();
    } else if (warp == S::W_PV) {
        // ------------------------------------------------------------ PV MMAs (one thread)
        // Once a step's weights are written and its V step has landed: O += P V
        // for each streamed page (a segment's first product overwrites, after
        // the previous segment's output block was read back), then commits that
        // free the weight buffer and the V step slot.
        if (lane == 0) {
            constexpr uint32_t ID_O = tc::idesc_f16_f32(S::M, D, false, true);    // P K-major, V MN-major
            bool stop = false;
            int gs = 0, sc = 0;
            for (int si = seg_begin; si < seg_end && !stop; ++si) {
                const int4 sg = si == seg_begin ? sg_h : a.segs[si];
                const int npg = sg.z - sg.y;
                if (npg == 0) continue;
                uint32_t accumulate = 0;
                for (int p0 = 0; p0 < npg; p0 += NP) {
                    const int n = min(NP, npg - p0);
                    const int b = gs & 1;
                    // output block sc % 2 was read back for segment sc - 2
                    if (!mbar_wait(smem_u32(p_full + b), (gs >> 1) & 1) ||
                        (p0 == 0 && sc >= 2 && !mbar_wait(smem_u32(o_free + (sc & 1)), ((sc >> 1) - 1) & 1))) {
                        stop = true;
                        break;
                    }
                    const int vs = gs % VSS;
                    if (!mbar_wait(smem_u32(vfull + vs), (gs / VSS) & 1)) {
                        stop = true;
                        break;
                    }
                    tc::fence_after_sync();
                    const uint32_t pb = smem_u32(pbuf + b * S::P_BYTES);
                    const unsigned vmask = vvalid[vs];
                    for (int p = 0; p < n; ++p) {
                        if (!((vmask >> p) & 1u)) continue;
                        const uint32_t vb = smem_u32(vring + (size_t(vs) * NP + p) * HALF);
#pragma unroll
                        for (int kk = 0; kk < S::PSTEPS; ++kk) {
                            const uint64_t ad =
                                tc::smem_desc(pb + (p * S::PSTEPS + kk) * 256, 128, S::P_SBO, tc::kNoSwizzle);
                            const uint64_t bd = tc::smem_desc(vb + kk * 16 * 128, T * 128, 1024, tc::kSwizzle128);
                            tc::mma_f16(tmem + (sc & 1) * D, ad, bd, ID_O, accumulate);
                            accumulate = 1;
                        }
                    }
                    tc::commit(smem_u32(p_free + b));
                    tc::commit(smem_u32(vempty + vs));
                    ++gs;
                }
                ++sc;
            }
            if (stop) fail_wait();
            tc::commit(smem_u32(mma_done + 1));
            if (!mbar_wait(smem_u32(mma_done + 1), 0)) fail_wait();
        }
        __syncwarp();
    } else if (warp == 0 || warp == 1 || warp == 4 || warp == 5) {
        // ------------------------------------------------------------ softmax
        const int quad = warp & 3;                  // heads 16 quad .. + 15: TMEM lanes of sub-partition quad
        const int cs = warp >> 2;                   // which half of a step's score columns (and of O)
        const int hrow = 16 * quad + (lane & 15);   // query head of the tile (MMA row)
        const int half = lane >> 4;                 // which 16 of each 32 columns
        const uint32_t tl = tmem + (uint32_t(32 * quad) << 16);   // this warp's lane sub-partition
        const int c0 = cs * (NS / 2);               // first score column of this warp
        const int oc0 = cs * (D / 2);               // first output column of this warp
        // The two warps of the same heads meet through pair_bar[quad][n % 2]
        // (n counts their meetings); row maxima travel through
        // xmax[n % 2][quad][cs][row].
        int npair = 0;
        const auto pair_sync = [&]() -> bool {
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(pair_bar + quad * 2 + (npair & 1)));
            const bool ok = warp_wait(pair_bar + quad * 2 + (npair & 1), (npair >> 1) & 1);
            ++npair;
            return ok;
        };
        // A segment's output is read back and written once the next segment's
        // first weights are out (or after the last segment), so the softmax does
        // not wait for the segment's last PV products; the output blocks of
        // consecutive segments alternate (sc % 2).
        struct Seg {
            int4 sg, g0;
            int nh, last_gs, ob;
            float m_ref, m_top, l;   // l: this thread's share of the denominator
            bool o_live;             // a PV product was issued into output block ob
            bool tmem;               // the segment had pages (its output block is released)
        };
        const auto finish = [&](const Seg &q) -> bool {
            uint32_t ov[OCW][16];    // this warp's part of the output row
            float l = q.l;
            if (q.o_live) {
                if (!warp_wait(p_free + (q.last_gs & 1), (q.last_gs >> 1) & 1)) return false;
                tc::fence_after_sync();
#pragma unroll
                for (int c = 0; c < OCW; ++c) tc::ld_16x32bx2_x16(tl + q.ob * D + oc0 + 32 * c, ov[c]);
                tc::wait_ld();
            }
            if (q.tmem) {
                tc::fence_before_sync();
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(o_free + q.ob));
            }
            if (!q.o_live) {
                l = 0.f;
#pragma unroll
                for (int c = 0; c < OCW; ++c)
#pragma unroll
                    for (int e = 0; e < 16; ++e) ov[c][e] = 0u;
            } else {
                // the row's denominator: this warp's two halves, then both warps, added
                // in warp order so that both hold the same bits
                const float lw = l + __shfl_xor_sync(kFullMask, l, 16);
                float *xr = xl + quad * 32;
                if (half == 0) xr[cs * 16 + (lane & 15)] = lw;
                if (!pair_sync()) return false;
                l = xr[lane & 15] + xr[16 + (lane & 15)];
            }
            // (m, l, o) against the true maximum, as the warp-level kernel writes them
            const float f = q.m_top == -INFINITY ? 0.f : ex2_ftz(q.m_ref - q.m_top);
            l *= f;
            const bool mine = hrow < q.nh;
            if (a.pair) {
                // heads 16 prank .. + 15 stay in weight buffer 0 (free: the last PV
                // products are done), the others go to the partner's query buffer 1
                const bool own = quad == int(prank);
                float *rows = reinterpret_cast<float *>(own ? pbuf : qbuf + S::Q_BYTES);
                float2 *ml = pair_ml + (own ? 0 : 16);
                if (!own) {
                    rows = cluster_map(rows, prank ^ 1u);
                    ml = cluster_map(ml, prank ^ 1u);
                }
                if (mine) store_pair_row<OCW>(rows + (lane & 15) * D, lane & 15, ov, oc0, half, f);
                if (mine && cs == 0 && half == 0) ml[lane & 15] = make_float2(q.m_top, l);
                return true;
            }
            const int64_t qhead = int64_t(q.g0.x) * a.Hq + int64_t(q.g0.y) * a.group + q.g0.z + hrow;
            const float inv = l > 0.f ? 1.f / l : 0.f;
            if (q.sg.w < 0 && a.xworld) {
                // the final row of this rank: to its slot in every rank's exchange buffer
                for (int x = 0; x < a.xworld; ++x) {
                    float *slot = xslot_of(a, x, xpar);
                    if (mine) {
                        store_o_part<OCW>(slot + qhead * D, ov, oc0, half, f * inv);
                        if (cs == 0 && half == 0)
                            *reinterpret_cast<float2 *>(xmeta_of<D>(slot, a, qhead)) = make_float2(q.m_top, l);
                    }
                }
                // both warps' parts of these rows are stored: tag them
                if (!pair_sync()) return false;
                if (cs == 0)
                    publish_rows<D>(a, qhead - (lane & 15), max(0, min(16, q.nh - 16 * quad)), xpar, xe, lane);
            } else {
                // the group's only segment, seen whole by this CTA: final output;
                // else the segment's (m, l, o) partial in slot sg.w
                const int64_t pr = int64_t(q.sg.w) * GT + hrow;
                if (mine) store_o_part<OCW>(q.sg.w < 0 ? a.out + qhead * D : a.part_o + pr * D, ov, oc0, half,
                                            q.sg.w < 0 ? f * inv : f);
                if (mine && cs == 0 && half == 0) {
                    if (q.sg.w >= 0) a.part_ml[pr] = make_float2(q.m_top, l);
                    else if (a.stats) reinterpret_cast<float2 *>(a.stats)[qhead] = make_float2(q.m_top, l);
                }
            }
            return true;
        };
        Seg pend{};
        bool has_pend = false;
        int sc = 0;   // segments with pages so far: this one's output block is sc % 2
        int gs = 0;
        bool stop = false;
        for (int si = seg_begin; si < seg_end; ++si) {
            const int4 sg = si == seg_begin ? sg_h : a.segs[si];
            const int4 g0 = si == seg_begin ? g0_h : a.groups[2 * sg.x];
            const int4 g1 = si == seg_begin ? g1_h : a.groups[2 * sg.x + 1];
            const int nh = g0.w;
            int length = g1.x;
            if (a.dynamic) {
                const int live = a.lengths[g0.x];
                if (live > length && warp == 0 && lane == 0) atomicOr(a.error, kErrLength);
                length = min(max(live, 0), length);
            }
            const int npg = sg.z - sg.y;
            float m_ref = -INFINITY;   // the maximum the weights are taken against
            float m_top = -INFINITY;   // the true running maximum
            bool o_live = false;       // a PV product has been issued in this segment
            float l = 0.f;
            if (npg > 0 && !stop) {
                for (int p0 = 0; p0 < npg; p0 += NP) {
                    const int n = min(NP, npg - p0);
                    const int b = gs & 1;
                    if (warp_abort() || !warp_wait(s_full + b, (gs >> 1) & 1)) {
                        stop = true;
                        break;
                    }
                    tc::fence_after_sync();
                    uint32_t sv[CW][16];
#pragma unroll
                    for (int c = 0; c < CW; ++c) tc::ld_16x32bx2_x16(tl + S::S_COL + b * NS + c0 + 32 * c, sv[c]);
                    const unsigned valid = svalid[b];   // written before the MMA thread's arrive
                    tc::wait_ld();
                    // mask pages not streamed and tokens past the end (raw scores: the scale is > 0)
                    const int tok0 = (sg.y + p0) * T;
                    if (!(n == NP && valid == (1u << NP) - 1u && tok0 + NS <= length)) {
#pragma unroll
                        for (int c = 0; c < CW; ++c)
#pragma unroll
                            for (int e = 0; e < 16; ++e) {
                                const int col = c0 + 32 * c + 16 * half + e;
                                if (!(col < n * T && ((valid >> (col / T)) & 1u) && tok0 + col < length))
                                    sv[c][e] = __float_as_uint(-INFINITY);
                            }
                    }
                    // this thread's maximum (a tree of 3-input maxima), then the row's over both warps
                    float t4[4 * CW];
#pragma unroll
                    for (int i = 0; i < 4 * CW; ++i) {
                        const uint32_t *x = &sv[i >> 2][(i & 3) * 4];
                        t4[i] = max3f(__uint_as_float(x[0]), __uint_as_float(x[1]),
                                      fmaxf(__uint_as_float(x[2]), __uint_as_float(x[3])));
                    }
                    float mloc = fmaxf(max3f(t4[0], t4[1], t4[2]), t4[3]);
                    if constexpr (CW == 2) mloc = fmaxf(mloc, fmaxf(max3f(t4[4], t4[5], t4[6]), t4[7]));
                    mloc = fmaxf(mloc, __shfl_xor_sync(kFullMask, mloc, 16));
                    float *xm = xmax + (npair & 1) * 64 + quad * 32;
                    if (half == 0) xm[cs * 16 + (lane & 15)] = mloc;
                    if (!pair_sync()) {
                        stop = true;
                        break;
                    }
                    const float mx = fmaxf(mloc, xm[(cs ^ 1) * 16 + (lane & 15)]) * a.scale_log2;
                    m_top = fmaxf(m_top, mx);
                    const bool grow = mx > m_ref + 8.f;
                    float alpha = 1.f;
                    if (grow) {
                        alpha = ex2_ftz(m_ref - mx);   // 0 while nothing was seen
                        m_ref = mx;
                    }
                    const float nu = m_ref == -INFINITY ? 0.f : -m_ref;
                    // weight buffer b is free once the PV products of step gs - 2 are done
                    if (gs >= 2 && !warp_wait(p_free + b, ((gs >> 1) - 1) & 1)) {
                        stop = true;
                        break;
                    }
                    // row hrow, tokens c0 + 32c + 16 half + [0, 16): two 8x8 core matrices
                    const uint32_t prow = smem_u32(pbuf + b * S::P_BYTES) + (hrow & 7) * 16 + (hrow >> 3) * S::P_SBO;
                    float lstep = 0.f;
#pragma unroll
                    for (int c = 0; c < CW; ++c) {
                        float pw[16];
#pragma unroll
                        for (int e = 0; e < 16; ++e) pw[e] = ex2_ftz(fmaf(__uint_as_float(sv[c][e]), a.scale_log2, nu));
                        uint32_t w[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e) w[e] = pack_half2(pw[2 * e], pw[2 * e + 1]);
                        // this thread's share of the denominator, summed as a tree
#pragma unroll
                        for (int e = 0; e < 8; ++e) pw[e] = pw[2 * e] + pw[2 * e + 1];
#pragma unroll
                        for (int e = 0; e < 4; ++e) pw[e] = pw[2 * e] + pw[2 * e + 1];
                        lstep += (pw[0] + pw[1]) + (pw[2] + pw[3]);
                        const uint32_t at = prow + ((c0 + 32 * c + 16 * half) >> 3) * 128;
                        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(at), "r"(w[0]), "r"(w[1]),
                                     "r"(w[2]), "r"(w[3]) : "memory");
                        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(at + 128), "r"(w[4]),
                                     "r"(w[5]), "r"(w[6]), "r"(w[7]) : "memory");
                    }
                    l = fmaf(l, alpha, lstep);
                    // V rows past the sequence end in its last page may hold anything,
                    // NaN included; their weight 0 must not meet them in the MMA.
                    if (quad == 0) {
                        const int pz = (length - tok0) / T;
                        const int vt = (length - tok0) - pz * T;
                        if (length > tok0 && pz < n && vt > 0 && ((valid >> pz) & 1u)) {
                            // the page's load landed (seen here too, before writing over it)
                            if (!warp_wait(vfull + gs % VSS, (gs / VSS) & 1)) {
                                stop = true;
                                break;
                            }
                            uint8_t *vrows = vring + (size_t(gs % VSS) * NP + pz) * HALF;
                            constexpr int UPR = S::NBOX * 8;   // 16-byte units per token row
                            for (int e = cs * 32 + lane; e < (T - vt) * UPR; e += 64) {
                                const int row = vt + e / UPR, u16 = e % UPR;
                                *reinterpret_cast<uint4 *>(vrows + (u16 >> 3) * (T * 128) + row * 128 + (u16 & 7) * 16) =
                                    make_uint4(0u, 0u, 0u, 0u);
                            }
                        }
                    }
                    // A moved reference rescales what the earlier steps built: the two
                    // warps of these heads see the same maxima, so both take this branch
                    // (each its part of the output block).
                    if (__any_sync(kFullMask, grow && o_live)) {
                        if (!warp_wait(p_free + ((gs - 1) & 1), ((gs - 1) >> 1) & 1)) {
                            stop = true;
                            break;
                        }
                        tc::fence_after_sync();
#pragma unroll
                        for (int c = 0; c < OCW; ++c) {
                            const uint32_t col = (sc & 1) * D + oc0 + 32 * c;
                            uint32_t r[16];
                            tc::ld_16x32bx2_x16(tl + col, r);
                            tc::wait_ld();
#pragma unroll
                            for (int e = 0; e < 16; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * alpha);
                            tc::st_16x32bx2_x16(tl + col, r);
                        }
                        tc::wait_st();
                    }
                    o_live = o_live || valid != 0u;
                    tc::fence_proxy_async_smem();
                    tc::fence_before_sync();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(smem_u32(p_full + b));
                    if (has_pend) {   // the previous segment's output, now that these weights are out
                        has_pend = false;
                        if (!finish(pend)) {
                            stop = true;
                            break;
                        }
                    }
                    ++gs;
                }
                if (!stop) {
                    pend = Seg{sg, g0, nh, gs - 1, sc & 1, m_ref, m_top, l, o_live, true};
                    has_pend = true;
                }
                ++sc;
            } else if (npg == 0) {
                // an empty sequence: zero rows, (m, l) = (-inf, 0)
                if (!finish(Seg{sg, g0, nh, 0, 0, -INFINITY, -INFINITY, 0.f, false, false})) stop = true;
            }
            if (stop) {
                if (lane == 0) fail_wait();
                break;
            }
        }
        if (has_pend && !stop && !finish(pend) && lane == 0) fail_wait();
        tc::fence_before_sync();
    }

    // every tensor-memory access and MMA of this CTA is done: free the columns
    named_barrier_sync(2, NC * 32);
    if (warp == S::W_MMA) {
        tc::fence_after_sync();
        tc::dealloc(tmem, S::TMEM_COLS);
    }
    if (a.pair) {
        // both halves' rows are in place once every thread of the pair is here
        cluster_sync_all();
        if ((warp == 0 || warp == 1 || warp == 4 || warp == 5) && (warp & 3) == int(prank)) {
            const int cs = warp >> 2, half = lane >> 4, r = lane & 15;
            const int hrow = 16 * int(prank) + r;
            if (hrow < g0_h.w) {
                const float2 mo = pair_ml[r], mp = pair_ml[16 + r];
                const float mx = fmaxf(mo.x, mp.x);
                const float wo = mo.x == -INFINITY ? 0.f : ex2_ftz(mo.x - mx);
                const float wp = mp.x == -INFINITY ? 0.f : ex2_ftz(mp.x - mx);
                const float l = fmaf(mo.y, wo, mp.y * wp);
                const float inv = l > 0.f ? 1.f / l : 0.f;
                const float so = wo * inv, sp = wp * inv;
                const float *ro = reinterpret_cast<const float *>(pbuf) + r * D;
                const float *rp = reinterpret_cast<const float *>(qbuf + S::Q_BYTES) + r * D;
                const int64_t qhead = int64_t(g0_h.x) * a.Hq + int64_t(g0_h.y) * a.group + g0_h.z + hrow;
                float *dst = a.out + qhead * D;
#pragma unroll
                for (int c = 0; c < OCW; ++c)
#pragma unroll
                    for (int e = 0; e < 16; e += 4) {
                        const int col = cs * (D / 2) + 32 * c + 16 * half + e;
                        const int sw = 4 * ((col >> 2) ^ r);   // store_pair_row's chunk order
                        const float4 x = *reinterpret_cast<const float4 *>(ro + sw);
                        const float4 y = *reinterpret_cast<const float4 *>(rp + sw);
                        *reinterpret_cast<float4 *>(dst + col) =
                            make_float4(fmaf(x.x, so, y.x * sp), fmaf(x.y, so, y.y * sp), fmaf(x.z, so, y.z * sp),
                                        fmaf(x.w, so, y.w * sp));
                    }
                if (a.stats && cs == 0 && half == 0) reinterpret_cast<float2 *>(a.stats)[qhead] = make_float2(mx, l);
            }
        }
        asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
        return;
    }
    finish_decode<D, 1, GT, 1, NC, S::RING>(a, ring, flags, warp, lane, xpar, xe);
    if (a.fused_merge || a.xworld) return;
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

}  // namespace pd
