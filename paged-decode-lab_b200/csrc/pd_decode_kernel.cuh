// pd_decode_kernel.cuh — persistent paged split-K GQA decode kernel for sm_100a.
//
// Replaces the reference's partial_decode + merge_decode/merge_shared
// (src/paged_decode/csrc/decode.cu:26-168) with one persistent kernel:
//
//   * one CTA per SM walks a host-built list of segments; a segment is a run
//     of logical pages of one group = (sequence, KV-head group of HG heads,
//     query-head tile); the host balances page tiles across CTAs, so every SM
//     streams the same number of bytes, ragged batches included;
//   * warp NC (producer) looks up each page in the page table and gathers the
//     page's K rows, then its V rows, for all HG KV heads of the group with
//     one 5-D tiled TMA load each ({128 B of a row, T, D*elt/128, Hkv, P}
//     view, 128-byte swizzle, no multicast) into a ring of shared-memory
//     slots, completion tracked by mbarriers.  One instruction moves a whole
//     K or V page of HG heads because a TMA instruction costs the same ~75
//     issue cycles whatever its size; many bytes per instruction keep one
//     thread ahead of HBM;
//   * a consumer warp owns one KV head of the group and a slice of 8 of its
//     query heads (QT = GT / 8 slices; wide groups such as MQA split their
//     query heads over warps that read the same tile) and takes every NSUB-th
//     tile; it folds its tiles into an online softmax (running max m,
//     denominator l, unnormalised output o) for its 8 query heads: FP16
//     inputs use m16n8k16 tensor-core MMAs (S^T = K Q^T, O^T += V^T P^T, FP32
//     accumulators), FP32 inputs use FP32 FMAs;
//   * consumer warps never wait for each other: at the end of its share of
//     a segment a warp writes its heads' normalised output directly when it
//     alone saw the whole group (one segment, NSUB == 1), else an (m, l, o)
//     partial; a small merge kernel, launched programmatically dependent on
//     this one (PDL), combines the partials with the max-corrected merge.
//
// All exponentials are base 2 on scores pre-multiplied by log2(e)/sqrt(D);
// this is the reference's exp(s - m) rewritten, not a different softmax.
#pragma once

#include <climits>
#include <type_traits>

#include "pd_device.cuh"
#include "pd_kernels_select.hpp"

namespace pd {

struct DecodeArgs {
    const void *q;            // [B, Hq, D] in the input dtype
    const int32_t *table;     // [B, W]
    const int4 *head;         // [C][16] per-CTA header: {seg_begin, seg_end}, first segment,
                              // its group (2 int4), page ids of its first 32 pages
    const int4 *segs;         // {group, first_page, end_page, slot (-1: write output directly)}
    const int4 *groups;       // 2 per group: {b, kv_head0, q_head_offset, nh}, {length, slot0, segments, 0}
    float *part_o;            // [slots, HG, GT, D] unnormalised partial outputs
    float2 *part_ml;          // [slots, HG, GT] (m, l) of each partial
    float *out;               // [B, Hq, D]
    float *stats;             // [B, Hq, 2] (m, l) or nullptr
    uint32_t *error;          // error word (PD_DEVERR_* bits)
    void *dense_k;            // gather mode: [B, Hkv, max_len, D]
    void *dense_v;
    int32_t Hq, Hkv, W, max_len, group;   // group = G = Hq / Hkv
    int32_t slot_stride;      // partial slots reserved per segment (>= NSUB)
    int32_t num_groups;
    // in-kernel merge: the grid barrier (its counters live in the plan) and the rows to merge
    GridBarrier gb;
    uint32_t *fallbacks;         // launches whose last CTA merged the shares of CTAs that left
    const int4 *merge_rows;      // split groups' rows: {out row, slot0, segments, head * GT + query head}
    int32_t num_merge_rows;
    int32_t fused_merge;         // 1: the CTAs merge the partials after a grid barrier
    int32_t pair;                // 1: clusters of two CTAs split each group and merge it themselves
    // Dynamic plans: groups cover each sequence up to its capacity (group word
    // 4); the live length of sequence b is min(lengths[b], capacity), pages at
    // or past it are skipped, and page ids always come from `table`.
    const int32_t *lengths;
    int32_t dynamic;
    // Sequence-sharded exchange (xworld > 0).  Every final row of this rank
    // (normalised o, then (m, l)) goes to this rank's slot in every rank's
    // exchange buffer over NVLink, followed (after a system-scope release
    // fence) by the row's tag: this launch's number.  A row of `out` is merged
    // from the ranks' rows once all of their tags show this launch.  Buffer
    // layout: u32 launch count per CTA at +256, then two parities (alternate
    // launches) of xworld slots of xslot bytes: [B*Hq*D o floats][B*Hq x
    // {m, l, tag, 0}].
    uint8_t *xpeer[8];
    int64_t xslot;
    int32_t xrank, xworld;
    int32_t rows;                 // B * Hq
    int64_t P;
    float scale_log2;         // log2(e) / sqrt(D)
};

constexpr uint32_t kErrTimeout = 1u;
constexpr uint32_t kErrBadPage = 2u;
constexpr uint32_t kErrLength = 8u;
constexpr int kMaxRanks = 8;
constexpr int64_t kXEpochs = 256;     // u32 launch counts, one per CTA (up to 1024 CTAs)
constexpr int64_t kXRecv = 256 + 4096;

// Where this rank's rows go: slot `rank` of rank s's buffer, parity p.
__device__ __forceinline__ float *xslot_of(const DecodeArgs &a, int s, int parity) {
    return reinterpret_cast<float *>(a.xpeer[s] + kXRecv + (int64_t(parity) * a.xworld + a.xrank) * a.xslot);
}

// {m, l, tag, 0} of `row` in a slot (after the slot's rows * D o floats).
template <int D>
__device__ __forceinline__ float4 *xmeta_of(float *slot, const DecodeArgs &a, int64_t row) {
    return reinterpret_cast<float4 *>(slot + int64_t(a.rows) * D) + row;
}

__device__ __forceinline__ void st_relaxed_sys_u32(unsigned *p, unsigned v) {
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_sys_u32(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// After a warp stored rows rows0 .. rows0 + n - 1 (o and (m, l)) into every
// rank's slot: release them, then tag each with this launch's number.
template <int D>
__device__ __forceinline__ void publish_rows(const DecodeArgs &a, int64_t row0, int n, int xpar, unsigned xe,
                                             int lane) {
    __syncwarp();
    if (lane == 0 && n > 0) {
        fence_release_sys();
        for (int s = 0; s < a.xworld; ++s) {
            float *slot = xslot_of(a, s, xpar);
            for (int i = 0; i < n; ++i)
                st_relaxed_sys_u32(reinterpret_cast<unsigned *>(&xmeta_of<D>(slot, a, row0 + i)->z), xe);
        }
    }
    __syncwarp();
}

template <typename Elt, int D, int T, int GT, int HG, int NSUB, int SLOTS>
struct KernelShape {
    static constexpr int ELT = sizeof(Elt);
    static constexpr int QT = GT / 8;                  // 8-query-head slices per KV head
    static constexpr int CPT = HG * QT;                // consumer warps reading each tile
    static constexpr int NC = CPT * NSUB;              // consumer warps
    static constexpr int ROW_BYTES = D * ELT;
    static constexpr int NBOX = ROW_BYTES / 128;       // 128-byte TMA boxes per token row
    static constexpr int BOX_ELEMS = 128 / ELT;
    static constexpr int HEAD_BYTES = NBOX * T * 128;  // one head's K (or V) rows: [box][token]
    static constexpr int HALF_BYTES = HG * HEAD_BYTES; // K (or V) part of one page tile: [head][box][token]
    static constexpr int TILE_BYTES = 2 * HALF_BYTES;
    static constexpr int THREADS = (NC + 1) * 32;
    static constexpr size_t RING = size_t(SLOTS) * TILE_BYTES;
    // FP16 keeps each warp's 8 query heads in registers; FP32 stages them in
    // the warp's own shared-memory slice (no swizzle: lanes read whole rows).
    static constexpr bool Q_SMEM = ELT != 2;
    static constexpr size_t QS = Q_SMEM ? size_t(NC) * 8 * D * ELT : 0;
    // With sub-pipelines, the warps of sub-pipelines 1.. hand their state for
    // each segment to sub-pipeline 0 through shared memory: one entry each of
    // 8 query heads' o [8][D] and (m, l) [8], and a full / free mbarrier per
    // (head, slice) of a tile.
    static constexpr bool FOLD = NSUB > 1 && fold_sub_pipelines(ELT, HG, GT, D, T);
    static constexpr int CSTATES = FOLD ? NC - CPT : 0;
    static constexpr size_t COMB_ENTRY = size_t(8) * D * 4 + 8 * 8;
    static constexpr size_t COMB = size_t(CSTATES) * COMB_ENTRY;
    static constexpr size_t BARS = size_t(SLOTS) * 16 + (FOLD ? size_t(CPT) * 16 : 0);
    static constexpr size_t FLAGS = size_t(SLOTS) * 4 + 16;
    static constexpr size_t SMEM = 1024 + RING + QS + COMB + BARS + FLAGS;
};

struct SmemFlags {
    volatile int abort;
    int barrier;        // grid_arrive's outcome (kBarrier*)
    int pad[2];
};

// ------------------------------------------------------------------ FP16 tensor-core engine
// One warp's online-softmax state for the GT query heads of one KV head.
// S^T[t][g] = K[t][:] . Q[g][:]  with A = K tile (ldmatrix), B = Q^T fragments;
// O^T[d][g] += V^T[d][t] P^T[t][g] with A = V tile (ldmatrix.trans), B = P^T,
// where P^T comes from the S^T accumulators by movmatrix.trans (no shared memory).
// A head's K (or V) rows sit in NBOX boxes of T 128-byte rows each: byte
// box*T*128 + t*128 of the head's block, 16-byte chunks XORed by t % 8.
template <int D, int T, int GT>
struct HalfEngine {
    static constexpr int NT = GT / 8;    // n-tiles of 8 query heads
    static constexpr int KS = D / 16;    // k-steps of the QK^T product
    static constexpr int DT = D / 16;    // m-tiles of the PV product (head dims)
    static constexpr int MT = T / 16;    // 16-token m-tiles per page
    static_assert(NT == 1, "a warp computes 8 query heads: one MMA n-tile");

    uint32_t qf[KS][NT][2];   // Q^T fragments of the warp's 8 query heads, in registers
    float acc[DT][NT][4];
    float m[NT][2], l[NT][2];
    int lane;

    // Q^T fragment: b0 = Q[g][d0..d0+1], b1 = Q[g][d0+8..d0+9], g = nt*8 + lane/4.
    __device__ __forceinline__ void begin(const __half *qrow, int nh, int lane_) {
        lane = lane_;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int g = nt * 8 + (lane >> 2);
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
                const int d0 = ks * 16 + 2 * (lane & 3);
                uint32_t lo = 0, hi = 0;
                if (g < nh) {
                    const uint32_t *src = reinterpret_cast<const uint32_t *>(qrow + g * D + d0);
                    lo = src[0];
                    hi = src[4];
                }
                qf[ks][nt][0] = lo;
                qf[ks][nt][1] = hi;
            }
        }
#pragma unroll
        for (int dt = 0; dt < DT; ++dt)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[dt][nt][i] = 0.f;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            m[nt][0] = m[nt][1] = -INFINITY;
            l[nt][0] = l[nt][1] = 0.f;
        }
    }

    __device__ __forceinline__ void q_frag(int ks, int nt, uint32_t &b0, uint32_t &b1) const {
        b0 = qf[ks][nt][0];
        b1 = qf[ks][nt][1];
    }

    __device__ __forceinline__ void tile(uint32_t kbase, uint32_t vbase, int valid, float scale_log2) {
        const int mi = lane >> 3, r8 = lane & 7;
        float x[MT][NT][4];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int i = 0; i < 4; ++i) x[mt][nt][i] = 0.f;
            const int row = mt * 16 + r8 + (mi & 1) * 8;
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
                uint32_t a[4];
                ldmatrix_x4(a, kbase + swz128<T>(row, ks * 2 + (mi >> 1)));
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    uint32_t b0, b1;
                    q_frag(ks, nt, b0, b1);
                    mma_16816(x[mt][nt], a, b0, b1);
                }
            }
        }
        // scale into log2 units and mask tokens past the sequence end
        const bool full = valid >= T;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int tok = mt * 16 + (lane >> 2) + ((i & 2) ? 8 : 0);
                    float v = x[mt][nt][i] * scale_log2;
                    if (!full && tok >= valid) v = -INFINITY;
                    x[mt][nt][i] = v;
                }
        uint32_t pb[MT][NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                mx0 = fmaxf(mx0, fmaxf(x[mt][nt][0], x[mt][nt][2]));
                mx1 = fmaxf(mx1, fmaxf(x[mt][nt][1], x[mt][nt][3]));
            }
#pragma unroll
            for (int s = 4; s < 32; s <<= 1) {
                mx0 = fmaxf(mx0, __shfl_xor_sync(kFullMask, mx0, s));
                mx1 = fmaxf(mx1, __shfl_xor_sync(kFullMask, mx1, s));
            }
            const float n0 = fmaxf(m[nt][0], mx0), n1 = fmaxf(m[nt][1], mx1);
            const float u0 = n0 == -INFINITY ? 0.f : n0, u1 = n1 == -INFINITY ? 0.f : n1;
            const float a0 = exp2f(m[nt][0] - u0), a1 = exp2f(m[nt][1] - u1);
            m[nt][0] = n0;
            m[nt][1] = n1;
            l[nt][0] *= a0;
            l[nt][1] *= a1;
#pragma unroll
            for (int dt = 0; dt < DT; ++dt) {
                acc[dt][nt][0] *= a0;
                acc[dt][nt][1] *= a1;
                acc[dt][nt][2] *= a0;
                acc[dt][nt][3] *= a1;
            }
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                // The weights enter the MMA as FP16; l sums the same rounded
                // weights so that o / l stays an exact convex combination.
                const uint32_t p01 = pack_half2(exp2f(x[mt][nt][0] - u0), exp2f(x[mt][nt][1] - u1));
                const uint32_t p23 = pack_half2(exp2f(x[mt][nt][2] - u0), exp2f(x[mt][nt][3] - u1));
                const float2 f01 = unpack_half2(p01), f23 = unpack_half2(p23);
                l[nt][0] += f01.x + f23.x;
                l[nt][1] += f01.y + f23.y;
                pb[mt][nt][0] = movmatrix_trans(p01);
                pb[mt][nt][1] = movmatrix_trans(p23);
            }
        }
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            const int row = mt * 16 + r8 + (mi >> 1) * 8;
            // tokens of this lane's V^T fragment halves: a0/a1 hold c0, c0 + 1; a2/a3 c0 + 8, c0 + 9
            const int c0 = mt * 16 + 2 * (lane & 3);
#pragma unroll
            for (int dt = 0; dt < DT; ++dt) {
                uint32_t a[4];
                ldmatrix_x4_trans(a, vbase + swz128<T>(row, dt * 2 + (mi & 1)));
                if (!full) {
                    // Rows past the sequence end (the rest of its last page) may hold
                    // anything, NaN included; their weight 0 must not meet them in the MMA.
                    a[0] = mask_tokens(a[0], c0, valid);
                    a[1] = mask_tokens(a[1], c0, valid);
                    a[2] = mask_tokens(a[2], c0 + 8, valid);
                    a[3] = mask_tokens(a[3], c0 + 8, valid);
                }
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) mma_16816(acc[dt][nt], a, pb[mt][nt][0], pb[mt][nt][1]);
            }
        }
    }

    // Zero the FP16 halves of `v` (tokens tok, tok + 1) at or past `valid`.
    static __device__ __forceinline__ uint32_t mask_tokens(uint32_t v, int tok, int valid) {
        return tok >= valid ? 0u : (tok + 1 >= valid ? (v & 0xffffu) : v);
    }

    // Sum l over the 8 lanes that share each query head (lane & 3 picks the head pair).
    __device__ __forceinline__ void reduce() {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int i = 0; i < 2; ++i)
#pragma unroll
                for (int s = 4; s < 32; s <<= 1) l[nt][i] += __shfl_xor_sync(kFullMask, l[nt][i], s);
    }

    // After reduce(): fold in another warp's reduced state for the same query heads,
    // o_s [heads][D] unnormalised and ml_s [heads] = (m, l), with the max-corrected
    // merge (oracle.py:88-96); an empty state (l = 0) changes nothing.
    __device__ __forceinline__ void absorb(const float *o_s, const float2 *ml_s) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const int g = nt * 8 + 2 * (lane & 3) + i;
                const float2 st = ml_s[g];
                if (st.y > 0.f) {
                    const float M = fmaxf(m[nt][i], st.x);
                    const float a = exp2f(m[nt][i] - M), b = exp2f(st.x - M);   // a = 0 for an empty state
                    m[nt][i] = M;
                    l[nt][i] = fmaf(l[nt][i], a, st.y * b);
#pragma unroll
                    for (int dt = 0; dt < DT; ++dt) {
                        const int d = dt * 16 + (lane >> 2);
                        acc[dt][nt][i] = fmaf(acc[dt][nt][i], a, o_s[g * D + d] * b);
                        acc[dt][nt][i + 2] = fmaf(acc[dt][nt][i + 2], a, o_s[g * D + d + 8] * b);
                    }
                }
            }
    }

    // f(g, d, o, m, l) for every accumulator element this lane holds.
    template <typename F>
    __device__ __forceinline__ void for_each_o(F &&f) const {
#pragma unroll
        for (int dt = 0; dt < DT; ++dt)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const int g = nt * 8 + 2 * (lane & 3);
                const int d = dt * 16 + (lane >> 2);
                f(g, d, acc[dt][nt][0], m[nt][0], l[nt][0]);
                f(g + 1, d, acc[dt][nt][1], m[nt][1], l[nt][1]);
                f(g, d + 8, acc[dt][nt][2], m[nt][0], l[nt][0]);
                f(g + 1, d + 8, acc[dt][nt][3], m[nt][1], l[nt][1]);
            }
    }

    // f(g, m, l) once per query head (lanes 0-3).
    template <typename F>
    __device__ __forceinline__ void for_each_ml(F &&f) const {
        if (lane < 4) {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int i = 0; i < 2; ++i) f(nt * 8 + 2 * lane + i, m[nt][i], l[nt][i]);
        }
    }
};

// ------------------------------------------------------------------ FP32 engine
// Lanes own tokens for the scores (one row of K per lane, Q broadcast from
// shared memory) and own head dims for the value sum.
template <int D, int T, int GT>
struct FloatEngine {
    static constexpr int DPL = D / 32;             // value dims per lane
    static constexpr int HALVES = 32 / T;          // lanes per token in the score phase
    static constexpr int CHUNKS = D / 4 / HALVES;  // float4 chunks of K per lane

    float acc[GT][DPL];
    float m[GT], l[GT];
    uint32_t qs;
    int nh, lane;

    __device__ __forceinline__ void begin(int nh_, int lane_, uint32_t qs_) {
        nh = nh_;
        lane = lane_;
        qs = qs_;
#pragma unroll
        for (int g = 0; g < GT; ++g) {
            m[g] = -INFINITY;
            l[g] = 0.f;
#pragma unroll
            for (int i = 0; i < DPL; ++i) acc[g][i] = 0.f;
        }
    }

    // The head count is dispatched to a compile-time bound so that an MHA
    // warp (one query head) runs no code for the seven unused head slots.
    __device__ __forceinline__ void tile(uint32_t kbase, uint32_t vbase, int valid, float scale_log2) {
        switch (nh) {
            case 1: tile_n<1>(kbase, vbase, valid, scale_log2); break;
            case 2: tile_n<2>(kbase, vbase, valid, scale_log2); break;
            case 3: tile_n<3>(kbase, vbase, valid, scale_log2); break;
            case 4: tile_n<4>(kbase, vbase, valid, scale_log2); break;
            case 5: tile_n<5>(kbase, vbase, valid, scale_log2); break;
            case 6: tile_n<6>(kbase, vbase, valid, scale_log2); break;
            case 7: tile_n<7>(kbase, vbase, valid, scale_log2); break;
            default: if (nh > 0) tile_n<GT>(kbase, vbase, valid, scale_log2); break;
        }
    }

    template <int NH>
    __device__ __forceinline__ void tile_n(uint32_t kbase, uint32_t vbase, int valid, float scale_log2) {
        const int t = lane % T;
        const int half = lane / T;
        float x[NH];
#pragma unroll
        for (int g = 0; g < NH; ++g) x[g] = 0.f;
#pragma unroll 4
        for (int c = 0; c < CHUNKS; ++c) {
            const int chunk = half * CHUNKS + c;
            const float4 kv = lds_f4(kbase + swz128<T>(t, chunk));
#pragma unroll
            for (int g = 0; g < NH; ++g) {
                const float4 qv = lds_f4(qs + (g * D + chunk * 4) * 4);
                x[g] = fmaf(qv.x, kv.x, x[g]);
                x[g] = fmaf(qv.y, kv.y, x[g]);
                x[g] = fmaf(qv.z, kv.z, x[g]);
                x[g] = fmaf(qv.w, kv.w, x[g]);
            }
        }
#pragma unroll
        for (int g = 0; g < NH; ++g) {
            float s = x[g];
            if (HALVES == 2) s += __shfl_xor_sync(kFullMask, s, 16);
            s = t < valid ? s * scale_log2 : -INFINITY;
            float mx = s;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(kFullMask, mx, o));
            const float nm = fmaxf(m[g], mx);
            const float u = nm == -INFINITY ? 0.f : nm;
            const float alpha = exp2f(m[g] - u);
            m[g] = nm;
            const float p = exp2f(s - u);
            l[g] = l[g] * alpha + (half == 0 ? p : 0.f);
#pragma unroll
            for (int i = 0; i < DPL; ++i) acc[g][i] *= alpha;
            x[g] = p;
        }
        // Only the valid rows: the rest of a sequence's last page may hold anything
        // (NaN included), and a zero weight times NaN is NaN.
        if (valid >= T) {
#pragma unroll 8
            for (int tt = 0; tt < T; ++tt) value_row<NH>(vbase, x, tt);
        } else {
            for (int tt = 0; tt < valid; ++tt) value_row<NH>(vbase, x, tt);
        }
    }

    // acc[g] += p[g][tt] * V[tt] for the NH live heads (p[g] lives in lane tt of x[g]).
    template <int NH>
    __device__ __forceinline__ void value_row(uint32_t vbase, const float (&x)[NH], int tt) {
        float vv[DPL];
        if constexpr (DPL == 2) {
            const float2 v2 = lds_f2(vbase + swz128<T>(tt, lane >> 1) + (lane & 1) * 8);
            vv[0] = v2.x;
            vv[1] = v2.y;
        } else {
            const float4 v4 = lds_f4(vbase + swz128<T>(tt, lane));
            vv[0] = v4.x;
            vv[1] = v4.y;
            vv[2] = v4.z;
            vv[3] = v4.w;
        }
#pragma unroll
        for (int g = 0; g < NH; ++g) {
            const float p = __shfl_sync(kFullMask, x[g], tt);
#pragma unroll
            for (int i = 0; i < DPL; ++i) acc[g][i] = fmaf(p, vv[i], acc[g][i]);
        }
    }

    __device__ __forceinline__ void reduce() {
#pragma unroll
        for (int g = 0; g < GT; ++g) {
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) l[g] += __shfl_xor_sync(kFullMask, l[g], o);
        }
    }

    // After reduce(): fold in another warp's reduced state (see HalfEngine::absorb).
    __device__ __forceinline__ void absorb(const float *o_s, const float2 *ml_s) {
#pragma unroll
        for (int g = 0; g < GT; ++g) {
            const float2 st = ml_s[g];
            if (st.y > 0.f) {
                const float M = fmaxf(m[g], st.x);
                const float a = exp2f(m[g] - M), b = exp2f(st.x - M);
                m[g] = M;
                l[g] = fmaf(l[g], a, st.y * b);
#pragma unroll
                for (int i = 0; i < DPL; ++i) acc[g][i] = fmaf(acc[g][i], a, o_s[g * D + lane * DPL + i] * b);
            }
        }
    }

    template <typename F>
    __device__ __forceinline__ void for_each_o(F &&f) const {
#pragma unroll
        for (int g = 0; g < GT; ++g)
#pragma unroll
            for (int i = 0; i < DPL; ++i) f(g, lane * DPL + i, acc[g][i], m[g], l[g]);
    }

    template <typename F>
    __device__ __forceinline__ void for_each_ml(F &&f) const {
        if (lane == 0) {
#pragma unroll
            for (int g = 0; g < GT; ++g) f(g, m[g], l[g]);
        }
    }
};

template <typename Elt, int D, int T, int GT>
struct EngineFor;
template <int D, int T, int GT>
struct EngineFor<__half, D, T, GT> {
    using type = HalfEngine<D, T, GT>;
};
template <int D, int T, int GT>
struct EngineFor<float, D, T, GT> {
    using type = FloatEngine<D, T, GT>;
};

// ------------------------------------------------------------------ kernel
enum : int { kModeDecode = 0, kModeGather = 1 };

// ------------------------------------------------------------------ producer warp
// Streams the CTA's page tiles into the ring: for each page of each segment,
// the page's K rows, then its V rows, for the HG KV heads of the group
// (TILE_BYTES per tile, V at +HALF_BYTES), one 5-D TMA load each, completion
// counted on the slot's full barrier.  Slot j % SLOTS is refilled once its
// empty barrier shows use j / SLOTS - 1 released.  Pages past a dynamic
// plan's live length, or with an id outside the cache, land nothing and mark
// the slot invalid.
template <int T, int TILE_BYTES, int HALF_BYTES, int SLOTS>
__device__ __forceinline__ void stream_page_tiles(const CUtensorMap *tm_k, const CUtensorMap *tm_v,
                                                  const DecodeArgs &a, uint8_t *ring, uint64_t *full_bar,
                                                  uint64_t *empty_bar, int *slot_valid, SmemFlags *flags,
                                                  const int4 hv, int seg_begin, int seg_end, int lane) {
    // Tiles of 8 KiB or less (one KV head, page 16) need more than one
    // thread issuing; larger ones keep a single issuing lane (measured).
    constexpr int PL = (TILE_BYTES <= 8192 && SLOTS >= 8) ? 4 : 1;
    if (lane == 0) {
        tma_prefetch_descriptor(tm_k);
        tma_prefetch_descriptor(tm_v);
    }
    bool stop = false;
    int j = 0;
    int4 sg = shfl_int4(hv, 1), g0 = shfl_int4(hv, 2);
    // lane i: page id of the first segment's page i (header words 16..47)
    const int4 hp = shfl_int4(hv, 4 + (lane >> 2));
    const int first_pages = (lane & 3) == 0 ? hp.x : (lane & 3) == 1 ? hp.y : (lane & 3) == 2 ? hp.z : hp.w;
    for (int si = seg_begin; si < seg_end; ++si) {
        // the next segment and its group load while this one streams
        const bool more = si + 1 < seg_end;
        const int4 nsg = more ? __ldg(a.segs + si + 1) : sg;
        int4 ng0 = g0;
        bool ng0_loaded = !more;
        const int32_t *trow = a.table + int64_t(g0.x) * a.W;
        const int kv0 = g0.y;
        // dynamic plans: pages at or past the live length are skipped
        const int live_end = a.dynamic ? max(0, a.lengths[g0.x]) : INT_MAX;
        for (int pg = sg.y; pg < sg.z; pg += 32) {
            const int n = min(32, sg.z - pg);
            const int mine = (!a.dynamic && si == seg_begin && pg == sg.y)
                                 ? first_pages
                                 : (lane < n ? __ldg(trow + pg + lane) : 0);
            // PL lanes issue PL consecutive tiles side by side, so one
            // TMA instruction carries PL tiles.
            for (int i = 0; i < n; i += PL) {
                const int cnt = min(PL, n - i);
                const int page = __shfl_sync(kFullMask, mine, (i + lane) & 31);
                if (lane < cnt && !stop) {
                    const int jj = j + lane;
                    const int slot = jj % SLOTS;
                    const int use = jj / SLOTS;
                    const uint32_t fb = smem_u32(full_bar + slot);
                    if (flags->abort ||
                        (use > 0 && !mbar_wait(smem_u32(empty_bar + slot), (use - 1) & 1))) {
                        if (!flags->abort) atomicOr(a.error, kErrTimeout);
                        flags->abort = 1;
                        stop = true;
                    } else if (int64_t(pg + i + lane) * T >= live_end) {
                        slot_valid[slot] = 0;   // not live yet: nothing to stream
                        mbar_arrive(fb);
                    } else if (page >= 0 && int64_t(page) < a.P) {
                        slot_valid[slot] = 1;
                        mbar_arrive_expect_tx(fb, TILE_BYTES);
                        const uint32_t dst = smem_u32(ring + size_t(slot) * TILE_BYTES);
                        // one instruction each for all of the page's K and V rows
                        tma_load_5d(dst, tm_k, 0, 0, 0, kv0, page, fb);
                        tma_load_5d(dst + HALF_BYTES, tm_v, 0, 0, 0, kv0, page, fb);
                    } else {
                        // The reference skips tokens whose page id is out of range
                        // (decode.cu:58); plans validate ids, so this is defence only.
                        atomicOr(a.error, kErrBadPage);
                        slot_valid[slot] = 0;
                        mbar_arrive(fb);
                    }
                }
                j += cnt;
            }
            if (!ng0_loaded) {
                ng0 = __ldg(a.groups + 2 * nsg.x);
                ng0_loaded = true;
            }
        }
        if (!ng0_loaded) ng0 = __ldg(a.groups + 2 * nsg.x);
        sg = nsg;
        g0 = ng0;
    }
}

// ------------------------------------------------------------------ in-kernel merge
// Runs in every CTA after the grid barrier (grid_arrive), in place
// of the separate merge kernel.  The split groups' output rows (merge_rows,
// {out row, first slot, segments, column}) are cut into gridDim.x contiguous
// shares.  With at least NC rows a warp takes every NC-th row of its CTA's
// share and merges it alone; with fewer, each row gets a team of NC / rows
// warps whose states meet in shared memory (`scratch`, the idle ring) and are
// combined by the row's first warp in member order.  A warp folds its
// partials into a running (m, l, o) with the max-corrected merge (the
// oracle.py:88-96 algebra), U partials in flight per lane, so a row costs one
// or two L2 round trips.  Every launch adds the same numbers in the same
// order.  Partials are read at L2 (ld.global.cg): other SMs wrote them during
// this launch.
template <int D, int HG, int GT, int NSUB>
struct RowMerge {
    static constexpr int CH = D / 4;                  // float4 chunks of a row
    static constexpr int LP = CH < 32 ? 32 / CH : 1;  // lane groups, each on its own partials
    static constexpr int CPL = CH > 32 ? CH / 32 : 1; // chunks per lane
    static constexpr int U = 8;
    float m, l;
    float4 o[CPL];

    __device__ __forceinline__ void add(float om, float ol, const float4 (&oo)[CPL]) {
        if (!(ol > 0.f)) return;
        const float nm = fmaxf(m, om);
        const float al = exp2f(m - nm), be = exp2f(om - nm);
        l = fmaf(l, al, be * ol);
#pragma unroll
        for (int cc = 0; cc < CPL; ++cc) {
            o[cc].x = fmaf(o[cc].x, al, be * oo[cc].x);
            o[cc].y = fmaf(o[cc].y, al, be * oo[cc].y);
            o[cc].z = fmaf(o[cc].z, al, be * oo[cc].z);
            o[cc].w = fmaf(o[cc].w, al, be * oo[cc].w);
        }
        m = nm;
    }

    // Partials first, first + step, ... of the row `meta`; every lane ends with
    // the merged state of its chunks.
    __device__ __forceinline__ void fold(const DecodeArgs &a, int4 meta, int first, int step, int lane) {
        m = -INFINITY;
        l = 0.f;
#pragma unroll
        for (int cc = 0; cc < CPL; ++cc) o[cc] = make_float4(0.f, 0.f, 0.f, 0.f);
        const int lg = LP > 1 ? lane / CH : 0;
        const int c0 = LP > 1 ? lane % CH : lane;
        const int parts = meta.z * NSUB;
        const int st = step * LP;
        for (int p0 = first + step * lg; p0 < parts; p0 += st * U) {
            float2 ml[U];
            float4 ov[U][CPL];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int p = p0 + u * st;
                ml[u] = make_float2(-INFINITY, 0.f);
                if (p < parts) {
                    const int64_t slot = int64_t(meta.y) + int64_t(p / NSUB) * a.slot_stride + p % NSUB;
                    const int64_t pr = slot * (HG * GT) + meta.w;
                    ml[u] = __ldcg(a.part_ml + pr);
                    const float4 *src = reinterpret_cast<const float4 *>(a.part_o + pr * D);
#pragma unroll
                    for (int cc = 0; cc < CPL; ++cc) ov[u][cc] = __ldcg(src + c0 + cc * 32);
                }
            }
#pragma unroll
            for (int u = 0; u < U; ++u) add(ml[u].x, ml[u].y, ov[u]);
        }
#pragma unroll
        for (int off = CH; off < 32; off *= 2) {   // fold the lane groups (D < 128)
            const float om = __shfl_xor_sync(kFullMask, m, off);
            const float ol = __shfl_xor_sync(kFullMask, l, off);
            float4 oo[CPL];
#pragma unroll
            for (int cc = 0; cc < CPL; ++cc) {
                oo[cc].x = __shfl_xor_sync(kFullMask, o[cc].x, off);
                oo[cc].y = __shfl_xor_sync(kFullMask, o[cc].y, off);
                oo[cc].z = __shfl_xor_sync(kFullMask, o[cc].z, off);
                oo[cc].w = __shfl_xor_sync(kFullMask, o[cc].w, off);
            }
            add(om, ol, oo);
        }
    }

    // Normalised output (zero for an empty row) and, if asked, the (m, l) stats.
    // Exchange mode (a.xworld > 0): the row goes to this rank's slot of every
    // rank's exchange buffer (parity xpar) instead, with its (m, l).
    __device__ __forceinline__ void write(const DecodeArgs &a, int4 meta, int lane, int xpar) const {
        const int c0 = LP > 1 ? lane % CH : lane;
        if (LP > 1 && lane >= CH) return;
        const float inv = l > 0.f ? 1.f / l : 0.f;
        float4 v[CPL];
#pragma unroll
        for (int cc = 0; cc < CPL; ++cc)
            v[cc] = make_float4(o[cc].x * inv, o[cc].y * inv, o[cc].z * inv, o[cc].w * inv);
        if (a.xworld) {
            for (int s = 0; s < a.xworld; ++s) {
                float *slot = xslot_of(a, s, xpar);
#pragma unroll
                for (int cc = 0; cc < CPL; ++cc)
                    reinterpret_cast<float4 *>(slot + int64_t(meta.x) * D)[c0 + cc * 32] = v[cc];
                if (lane == 0) *reinterpret_cast<float2 *>(xmeta_of<D>(slot, a, meta.x)) = make_float2(m, l);
            }
            return;
        }
        float4 *dst = reinterpret_cast<float4 *>(a.out + int64_t(meta.x) * D);
#pragma unroll
        for (int cc = 0; cc < CPL; ++cc) dst[c0 + cc * 32] = v[cc];
        if (a.stats && lane == 0) reinterpret_cast<float2 *>(a.stats)[meta.x] = make_float2(m, l);
    }
};

template <int D, int HG, int GT, int NSUB, int NC>
__device__ __forceinline__ void merge_in_kernel(const DecodeArgs &a, uint8_t *scratch, int warp, int lane,
                                                int64_t lo, int rows, int team, int4 meta0, int xpar,
                                                unsigned xe) {
    using M = RowMerge<D, HG, GT, NSUB>;
    M rm;
    if constexpr ((NC <= 4 || HG == 8) && M::LP == 1) {
        if (team == 1) {
            // Four or fewer consumer warps, or tiles of eight KV heads: each warp
            // merges many rows (config 3c: ~7 of ~3 partials each; config 4: ~8
            // of 2-3).  The partials of a warp's rows form one stream, U loads in
            // flight across row boundaries, so the warp waits for one L2 round
            // trip per U partials, not one per row.  Each row still adds its
            // partials in slot order, as fold() does.  (Measured: config 4 679.4
            // -> 673.5 us, config 2 80.3 -> 81.2; the single-head eight-warp
            // kernel of config 3b lost 1.2 us and keeps one row at a time.)
            const int K = rows > warp ? (rows - warp + NC - 1) / NC : 0;
            for (int k0 = 0; k0 < K; k0 += 32) {
                const int kn = min(32, K - k0);
                // lane i: descriptor of row k0 + i (merge rows have >= 1 segment)
                const int4 mine = (k0 == 0 && lane == 0) ? meta0
                                  : lane < kn ? __ldg(a.merge_rows + lo + warp + int64_t(k0 + lane) * NC)
                                              : make_int4(0, 0, 0, 0);
                int k = 0, p = 0, cur = 0;
                int4 mk = shfl_int4(mine, 0);
                int pk = mk.z * NSUB;
                rm.m = -INFINITY;
                rm.l = 0.f;
#pragma unroll
                for (int cc = 0; cc < M::CPL; ++cc) rm.o[cc] = make_float4(0.f, 0.f, 0.f, 0.f);
                while (k < kn) {
                    float2 ml[M::U];
                    float4 ov[M::U][M::CPL];
                    int rowof[M::U];
#pragma unroll
                    for (int u = 0; u < M::U; ++u) {
                        rowof[u] = -1;
                        if (k < kn) {
                            const int64_t slot = int64_t(mk.y) + int64_t(p / NSUB) * a.slot_stride + p % NSUB;
                            const int64_t pr = slot * (HG * GT) + mk.w;
                            ml[u] = __ldcg(a.part_ml + pr);
                            const float4 *src = reinterpret_cast<const float4 *>(a.part_o + pr * D);
#pragma unroll
                            for (int cc = 0; cc < M::CPL; ++cc) ov[u][cc] = __ldcg(src + lane + cc * 32);
                            rowof[u] = k;
                            if (++p == pk) {
                                p = 0;
                                if (++k < kn) {
                                    mk = shfl_int4(mine, k);
                                    pk = mk.z * NSUB;
                                }
                            }
                        }
                    }
#pragma unroll
                    for (int u = 0; u < M::U; ++u) {
                        if (rowof[u] < 0) break;
                        if (rowof[u] != cur) {   // row `cur` is complete
                            const int4 mc = shfl_int4(mine, cur);
                            rm.write(a, mc, lane, xpar);
                            if (a.xworld) publish_rows<D>(a, mc.x, 1, xpar, xe, lane);
                            rm.m = -INFINITY;
                            rm.l = 0.f;
#pragma unroll
                            for (int cc = 0; cc < M::CPL; ++cc) rm.o[cc] = make_float4(0.f, 0.f, 0.f, 0.f);
                            cur = rowof[u];
                        }
                        rm.add(ml[u].x, ml[u].y, ov[u]);
                    }
                }
                if (kn > 0) {
                    const int4 mc = shfl_int4(mine, cur);
                    rm.write(a, mc, lane, xpar);
                    if (a.xworld) publish_rows<D>(a, mc.x, 1, xpar, xe, lane);
                }
            }
            return;
        }
    }
    if (team == 1) {
        int4 meta = meta0;
        for (int r = warp; r < rows; r += NC) {
            const int4 next = r + NC < rows ? __ldg(a.merge_rows + lo + r + NC) : meta;
            rm.fold(a, meta, 0, 1, lane);
            rm.write(a, meta, lane, xpar);
            if (a.xworld) publish_rows<D>(a, meta.x, 1, xpar, xe, lane);
            meta = next;
        }
        return;
    }
    float4 *res_o = reinterpret_cast<float4 *>(scratch);                         // [NC][D / 4]
    float2 *res_ml = reinterpret_cast<float2 *>(scratch + size_t(NC) * D * 4);   // [NC]
    if (warp < rows * team) {
        rm.fold(a, meta0, warp / rows, team, lane);
        const int c0 = M::LP > 1 ? lane % M::CH : lane;
        if (M::LP == 1 || lane < M::CH) {
#pragma unroll
            for (int cc = 0; cc < M::CPL; ++cc) res_o[warp * M::CH + c0 + cc * 32] = rm.o[cc];
        }
        if (lane == 0) res_ml[warp] = make_float2(rm.m, rm.l);
    }
    named_barrier_sync(1, NC * 32);
    if (warp < rows) {
        // member 0 of row `warp` combines members k = 1 .. team - 1 (warps warp + k * rows)
        const int c0 = M::LP > 1 ? lane % M::CH : lane;
        for (int k = 1; k < team; ++k) {
            const float2 ml = res_ml[warp + k * rows];
            float4 oo[M::CPL];
#pragma unroll
            for (int cc = 0; cc < M::CPL; ++cc)
                oo[cc] = (M::LP == 1 || lane < M::CH) ? res_o[(warp + k * rows) * M::CH + c0 + cc * 32]
                                                      : make_float4(0.f, 0.f, 0.f, 0.f);
            rm.add(ml.x, ml.y, oo);
        }
        rm.write(a, meta0, lane, xpar);
        if (a.xworld) publish_rows<D>(a, meta0.x, 1, xpar, xe, lane);
    }
}

// Exchange mode: this CTA's share of the output rows, each merged as soon as
// every rank's copy of it carries this launch's tag: the max-corrected merge
// (oracle.py:88-96) of the ranks' normalised rows o_s with weights
// 2^(m_s - M) l_s; zero when all are empty.  One warp per row: lane s polls
// rank s's tag, then every (m, l) and every lane's o chunk of all ranks load
// together; `stats` gets the merged (M, L).
template <int D, int NC>
__device__ __forceinline__ void merge_ranks(const DecodeArgs &a, int warp, int lane, int xpar, unsigned xe) {
    constexpr int CH = D / 4;
    const int64_t R = a.rows;
    const int64_t lo = R * blockIdx.x / gridDim.x, hi = R * (blockIdx.x + 1) / gridDim.x;
    float *slot0 = reinterpret_cast<float *>(a.xpeer[a.xrank] + kXRecv + int64_t(xpar) * a.xworld * a.xslot);
    const int64_t step = a.xslot / 4;   // floats from one rank's slot to the next
    for (int64_t row = lo + warp; row < hi; row += NC) {
        bool ok = true;
        if (lane < a.xworld) {
            const unsigned *tag =
                reinterpret_cast<const unsigned *>(&xmeta_of<D>(slot0 + lane * step, a, row)->z);
            if (ld_acquire_sys_u32(tag) < xe) {
                const unsigned long long start = global_ns();
                while (ld_acquire_sys_u32(tag) < xe)
                    if (global_ns() - start > kWaitTimeoutNs) {
                        ok = false;
                        break;
                    }
            }
        }
        ok = __all_sync(kFullMask, ok);
        __syncwarp();
        if (!ok) {
            if (lane == 0) atomicOr(a.error, kErrTimeout);
            continue;
        }
        float2 ml[kMaxRanks];
        float4 v[kMaxRanks];
#pragma unroll
        for (int s = 0; s < kMaxRanks; ++s) {
            ml[s] = make_float2(-INFINITY, 0.f);
            v[s] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (s < a.xworld) {
                ml[s] = __ldcv(reinterpret_cast<const float2 *>(xmeta_of<D>(slot0 + s * step, a, row)));
                if (lane < CH) v[s] = __ldcv(reinterpret_cast<const float4 *>(slot0 + s * step + row * D) + lane);
            }
        }
        float top = -INFINITY;
#pragma unroll
        for (int s = 0; s < kMaxRanks; ++s)
            if (ml[s].y > 0.f) top = fmaxf(top, ml[s].x);
        float den = 0.f;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int s = 0; s < kMaxRanks; ++s)
            if (ml[s].y > 0.f) {
                const float w = exp2f(ml[s].x - top) * ml[s].y;
                den += w;
                acc.x = fmaf(w, v[s].x, acc.x);
                acc.y = fmaf(w, v[s].y, acc.y);
                acc.z = fmaf(w, v[s].z, acc.z);
                acc.w = fmaf(w, v[s].w, acc.w);
            }
        const float inv = den > 0.f ? 1.f / den : 0.f;
        if (lane < CH)
            reinterpret_cast<float4 *>(a.out + row * D)[lane] =
                make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
        if (a.stats && lane == 0) reinterpret_cast<float2 *>(a.stats)[row] = make_float2(top, den);
    }
}

// ------------------------------------------------------------------ end of a decode launch
// After the CTA's consumer warps (0 .. NC - 1) have written every row and
// partial of their segments: the in-kernel merge (grid barrier, then this
// CTA's share of the split rows, with `ring` as scratch) and, in exchange
// mode, the merge of this CTA's output rows from every rank's copies.
// Partials were written with NSUB slots per segment.
template <int D, int HG, int GT, int NSUB, int NC, size_t RING>
__device__ __forceinline__ void finish_decode(const DecodeArgs &a, uint8_t *ring, SmemFlags *flags, int warp,
                                              int lane, int xpar, uint32_t xe) {
    if (a.fused_merge) {
        // merge scratch, then a snapshot of the left-CTA bits (1024 bits)
        static_assert(size_t(NC) * (D * 4 + 8) + 128 <= RING, "merge scratch must fit in the ring");
        unsigned long long *left_snap =
            reinterpret_cast<unsigned long long *>(ring + size_t(NC) * (D * 4 + 8));
        // CTA c's share of the merge rows: rows [lo, lo + rows), a team of
        // `team` warps per row when there are fewer rows than warps, and
        // this warp's first row descriptor
        const int64_t R = a.num_merge_rows;
        const auto share = [&](unsigned c, int64_t &lo, int &rows, int &team) {
            lo = R * c / gridDim.x;
            rows = int(R * (c + 1) / gridDim.x - lo);
            team = (rows >= NC || rows == 0) ? 1 : NC / rows;
            const bool has = team == 1 ? warp < rows : warp < rows * team;
            return has ? __ldg(a.merge_rows + lo + (team == 1 ? warp : warp % rows)) : make_int4(0, 0, 0, 0);
        };
        int64_t mlo;
        int mrows, team;
        const int4 meta0 = share(blockIdx.x, mlo, mrows, team);   // loads while the CTAs gather
        named_barrier_sync(1, NC * 32);   // this CTA's partials are written
        unsigned nleft = 0;
        if (warp == 0 && lane == 0) {
            const int r = grid_arrive(a.gb, gridDim.x, blockIdx.x, &nleft);
            if (r == kBarrierTimeout) {
                atomicOr(a.error, kErrTimeout);
                flags->abort = 1;
            }
            if (r == kBarrierGoMergeLeft)
                for (unsigned w = 0; w < (gridDim.x + 63) / 64; ++w) left_snap[w] = __ldcg(a.gb.left + w);
            flags->barrier = r;
        }
        named_barrier_sync(1, NC * 32);
        const int verdict = flags->barrier;
        // After an abort a TMA load may still be landing in the ring: no merge.
        if (!flags->abort && verdict != kBarrierLeft) {
            merge_in_kernel<D, HG, GT, NSUB, NC>(a, ring, warp, lane, mlo, mrows, team, meta0, xpar, xe);
            if (verdict == kBarrierGoMergeLeft) {
                // this CTA completed the barrier after others left: merge their shares too
                for (unsigned c = 0; c < gridDim.x; ++c) {
                    if (c == blockIdx.x || !((left_snap[c / 64] >> (c % 64)) & 1ull)) continue;
                    int64_t clo;
                    int crows, cteam;
                    const int4 cmeta0 = share(c, clo, crows, cteam);
                    named_barrier_sync(1, NC * 32);   // the scratch is free again
                    merge_in_kernel<D, HG, GT, NSUB, NC>(a, ring, warp, lane, clo, crows, cteam, cmeta0,
                                                         xpar, xe);
                }
                named_barrier_sync(1, NC * 32);
                if (warp == 0 && lane == 0) {   // clear the leaves for the next launch
                    for (unsigned w = 0; w < (gridDim.x + 63) / 64; ++w) atomicAnd(a.gb.left + w, ~left_snap[w]);
                    atomicAdd(a.gb.count, 0ull - (unsigned long long)nleft * kLeftUnit);
                    atomicAdd(a.fallbacks, 1u);
                }
            }
        }
    }
    if (a.xworld) {
        // This CTA's rows are published (tagged) as they are written; merge
        // this CTA's share of the output rows as the ranks' copies arrive.
        if (warp == 0 && lane == 0)   // this CTA's launch count, read back by the next launch
            reinterpret_cast<uint32_t *>(a.xpeer[a.xrank] + kXEpochs)[blockIdx.x] = xe;
        if (!flags->abort) merge_ranks<D, NC>(a, warp, lane, xpar, xe);
    }
}

template <typename Elt, int D, int T, int GT, int HG, int NSUB, int SLOTS, int MODE>
__global__ void __launch_bounds__((HG * (GT / 8) * NSUB + 1) * 32, 1)
    paged_decode_kernel(const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const DecodeArgs a) {
    using S = KernelShape<Elt, D, T, GT, HG, NSUB, SLOTS>;
    constexpr int NC = S::NC;
    static_assert(S::ROW_BYTES % 128 == 0, "token rows must be whole 128-byte boxes");
    static_assert(T % 8 == 0, "boxes of T rows must keep 1024-byte swizzle alignment");
    static_assert(S::SMEM <= 232448, "shared memory budget exceeded");
    // Tile j goes to slot j % SLOTS and to the warps of sub-pipeline j % NSUB;
    // with SLOTS a multiple of NSUB every slot is consumed by one fixed set of
    // warps, which keeps every mbarrier parity wait within one phase of the
    // last phase those warps consumed (parity cannot tell phase u from u - 2).
    static_assert(SLOTS % NSUB == 0, "ring slots must be a multiple of the sub-pipelines");
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *ring = smem;
    uint8_t *qsm = ring + S::RING;
    float *comb = reinterpret_cast<float *>(qsm + S::QS);
    uint64_t *full_bar = reinterpret_cast<uint64_t *>(qsm + S::QS + S::COMB);
    uint64_t *empty_bar = full_bar + SLOTS;
    uint64_t *comb_full = empty_bar + SLOTS;            // S::FOLD: [CPT]
    uint64_t *comb_free = comb_full + (S::FOLD ? S::CPT : 0);
    int *slot_valid = reinterpret_cast<int *>(comb_free + (S::FOLD ? S::CPT : 0));
    SmemFlags *flags = reinterpret_cast<SmemFlags *>(slot_valid + SLOTS);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // Every warp reads the CTA header (12 int4, one per lane): the first page
    // tile then needs one dependent load before its TMA instead of four.
    const int4 hv = lane < 12 ? __ldg(a.head + int64_t(blockIdx.x) * 16 + lane) : make_int4(0, 0, 0, 0);
    const int seg_begin = __shfl_sync(kFullMask, hv.x, 0);
    const int seg_end = __shfl_sync(kFullMask, hv.y, 0);

    if (threadIdx.x == 0) {
        for (int s = 0; s < SLOTS; ++s) {
            mbar_init(smem_u32(full_bar + s), 1);
            mbar_init(smem_u32(empty_bar + s), S::CPT);   // released by the warps that read it
        }
        if constexpr (S::FOLD) {
            for (int c = 0; c < S::CPT; ++c) {
                mbar_init(smem_u32(comb_full + c), NSUB - 1);   // sub-pipelines 1.. posted their state
                mbar_init(smem_u32(comb_free + c), 1);          // sub-pipeline 0 has read them
            }
        }
        flags->abort = 0;
        mbar_init_fence();
    }
    __syncthreads();
    // Launched programmatically dependent on the previous kernel in the
    // stream: everything above (plan metadata, shared-memory set-up) may
    // overlap its tail; q, the caches and every output wait for it to finish.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (MODE == kModeDecode && a.fused_merge && threadIdx.x == 0) atomicAdd(a.gb.started, 1ull);
    // Exchange mode: this launch's number (1, 2, ...) and the buffer parity it writes.
    const uint32_t xe = a.xworld
        ? __ldcv(reinterpret_cast<const unsigned int *>(a.xpeer[a.xrank] + kXEpochs) + blockIdx.x) + 1u : 0u;
    const int xpar = int(xe & 1u);

    if (warp == NC) {
        stream_page_tiles<T, S::TILE_BYTES, S::HALF_BYTES, SLOTS>(&tm_k, &tm_v, a, ring, full_bar, empty_bar,
                                                                slot_valid, flags, hv, seg_begin, seg_end, lane);
        return;
    }

    // ---------------------------------------------------------------- consumers
    const int hh = warp % S::CPT / S::QT;   // KV head of the group this warp owns
    const int qt = warp % S::QT;            // its 8-query-head slice of that head
    const int sub = warp / S::CPT;          // it takes tiles j with j % NSUB == sub
    const int hoff = hh * S::HEAD_BYTES;   // its head's block in each half of a tile
    bool stop = false;
    int j = 0;
    int seg_ends = 0;                       // segments this warp has finished (handoff phases)
    const int4 sg_h = shfl_int4(hv, 1), g0_h = shfl_int4(hv, 2), g1_h = shfl_int4(hv, 3);
    for (int si = seg_begin; si < seg_end; ++si) {
        const int4 sg = si == seg_begin ? sg_h : a.segs[si];
        const int4 g0 = si == seg_begin ? g0_h : a.groups[2 * sg.x];
        const int4 g1 = si == seg_begin ? g1_h : a.groups[2 * sg.x + 1];
        const int b = g0.x, kv0 = g0.y, qoff = g0.z, nh = g0.w;
        int length = g1.x;
        if (a.dynamic) {
            const int live = a.lengths[b];
            if (live > length && warp == 0 && lane == 0) atomicOr(a.error, kErrLength);
            length = min(max(live, 0), length);
        }
        const int npg = sg.z - sg.y;
        const int first = ((sub - j) % NSUB + NSUB) % NSUB;

        if constexpr (MODE == kModeGather) {
            constexpr int CPR = S::ROW_BYTES / 16;   // 16-byte chunks per token row
            for (int t = first; t < npg; t += NSUB) {
                const int jj = j + t;
                const int slot = jj % SLOTS;
                if (stop || flags->abort) break;
                if (!mbar_wait(smem_u32(full_bar + slot), (jj / SLOTS) & 1)) {
                    if (lane == 0) atomicOr(a.error, kErrTimeout);
                    flags->abort = 1;
                    stop = true;
                    break;
                }
                const int lp = sg.y + t;
                const int valid = min(T, length - lp * T);
                if (slot_valid[slot]) {
                    const uint32_t kb = smem_u32(ring + size_t(slot) * S::TILE_BYTES) + hoff;
                    const int64_t base = (int64_t(b) * a.Hkv + kv0 + hh) * a.max_len + int64_t(lp) * T;
                    for (int idx = lane; idx < valid * CPR; idx += 32) {
                        const int r = idx / CPR, c = idx % CPR;
                        const float4 kv = lds_f4(kb + swz128<T>(r, c));
                        const float4 vv = lds_f4(kb + S::HALF_BYTES + swz128<T>(r, c));
                        const int64_t off = (base + r) * S::ROW_BYTES + c * 16;
                        *reinterpret_cast<float4 *>(static_cast<uint8_t *>(a.dense_k) + off) = kv;
                        *reinterpret_cast<float4 *>(static_cast<uint8_t *>(a.dense_v) + off) = vv;
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(empty_bar + slot));
            }
            j += npg;
        } else {
            using Engine = typename EngineFor<Elt, D, T, 8>::type;
            Engine eng;
            // this warp's query heads: (kv0 + hh) * G + qoff + qt * 8 + g, g < nw
            const int nw = min(8, nh - qt * 8);     // may be <= 0: the warp then idles on its tiles
            const int64_t qhead0 = int64_t(b) * a.Hq + int64_t(kv0 + hh) * a.group + qoff + qt * 8;
            const Elt *qrow = static_cast<const Elt *>(a.q) + qhead0 * D;
            uint8_t *qmine = qsm + size_t(warp) * 8 * D * sizeof(Elt);
            const uint32_t qs = smem_u32(qmine);
            if constexpr (S::Q_SMEM) {
                // FP32: this warp's Q rows (zero rows for heads past nh) into its own slice
                constexpr int CPR = D * int(sizeof(Elt)) / 16;
                for (int e = lane; e < 8 * CPR; e += 32) {
                    const int g = e / CPR, c = e % CPR;
                    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (g < nw) v = __ldg(reinterpret_cast<const float4 *>(qrow + int64_t(g) * D) + c);
                    reinterpret_cast<float4 *>(qmine + size_t(g) * D * sizeof(Elt))[c] = v;
                }
                __syncwarp();
            }
            if constexpr (std::is_same<Elt, __half>::value)
                eng.begin(reinterpret_cast<const __half *>(qrow), nw, lane);
            else
                eng.begin(nw, lane, qs);

            for (int t = first; t < npg; t += NSUB) {
                const int jj = j + t;
                const int slot = jj % SLOTS;
                if (stop || flags->abort) break;
                if (!mbar_wait(smem_u32(full_bar + slot), (jj / SLOTS) & 1)) {
                    if (lane == 0) atomicOr(a.error, kErrTimeout);
                    flags->abort = 1;
                    stop = true;
                    break;
                }
                if (slot_valid[slot]) {
                    const int lp = sg.y + t;
                    const uint32_t kb = smem_u32(ring + size_t(slot) * S::TILE_BYTES) + hoff;
                    eng.tile(kb, kb + S::HALF_BYTES, min(T, length - lp * T),
                             a.scale_log2);
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(empty_bar + slot));
            }
            j += npg;

            // ---------------------------------------------------- publish this warp's state
            eng.reduce();
            if constexpr (S::FOLD) {
                // Sub-pipelines 1.. post their state for this (head, slice) and go on;
                // sub-pipeline 0 folds them in, in sub-pipeline order (so results repeat
                // bit for bit), and writes the segment's one result.
                const int ci = warp % S::CPT;
                const uint32_t cf = smem_u32(comb_full + ci), cr = smem_u32(comb_free + ci);
                bool ok = true;
                if (sub > 0) {
                    float *o_s = comb + size_t((sub - 1) * S::CPT + ci) * (S::COMB_ENTRY / 4);
                    float2 *ml_s = reinterpret_cast<float2 *>(o_s + 8 * D);
                    if (seg_ends > 0) ok = mbar_wait(cr, (seg_ends - 1) & 1);   // the last state was read
                    if (ok) {
                        eng.for_each_o([&](int g, int d, float o, float, float) { o_s[g * D + d] = o; });
                        eng.for_each_ml([&](int g, float m, float l) { ml_s[g] = make_float2(m, l); });
                    }
                    __threadfence_block();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(cf);
                } else {
                    ok = mbar_wait(cf, seg_ends & 1);
                    if (ok) {
#pragma unroll 1
                        for (int sp = 1; sp < NSUB; ++sp) {
                            const float *o_s = comb + size_t((sp - 1) * S::CPT + ci) * (S::COMB_ENTRY / 4);
                            eng.absorb(o_s, reinterpret_cast<const float2 *>(o_s + 8 * D));
                        }
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(cr);
                }
                if (!ok) {
                    if (lane == 0) atomicOr(a.error, kErrTimeout);
                    flags->abort = 1;
                    stop = true;
                }
                ++seg_ends;
            }
            if (S::FOLD && sub > 0) {
                // its state went to sub-pipeline 0
            } else if (sg.w < 0 && a.xworld) {
                // the final row of this rank: to its slot in every rank's exchange buffer
                for (int x = 0; x < a.xworld; ++x) {
                    float *slot = xslot_of(a, x, xpar);
                    eng.for_each_o([&](int g, int d, float o, float, float l) {
                        if (g < nw) slot[(qhead0 + g) * D + d] = l > 0.f ? o / l : 0.f;
                    });
                    eng.for_each_ml([&](int g, float m, float l) {
                        if (g < nw) *reinterpret_cast<float2 *>(xmeta_of<D>(slot, a, qhead0 + g)) = make_float2(m, l);
                    });
                }
                publish_rows<D>(a, qhead0, max(nw, 0), xpar, xe, lane);
            } else if (sg.w < 0) {
                // the group's only segment, seen whole by this CTA: final output
                eng.for_each_o([&](int g, int d, float o, float, float l) {
                    if (g < nw) a.out[(qhead0 + g) * D + d] = l > 0.f ? o / l : 0.f;
                });
                if (a.stats)
                    eng.for_each_ml([&](int g, float m, float l) {
                        if (g < nw) reinterpret_cast<float2 *>(a.stats)[qhead0 + g] = make_float2(m, l);
                    });
            } else {
                // [slot][head] partial row: one slot per segment when folded, else one per sub-pipeline
                const int64_t ps = (int64_t(sg.w) + (S::FOLD ? 0 : sub)) * HG + hh;
                eng.for_each_o([&](int g, int d, float o, float, float) {
                    if (g < nw) a.part_o[(ps * GT + qt * 8 + g) * D + d] = o;
                });
                eng.for_each_ml([&](int g, float m, float l) {
                    if (g < nw) a.part_ml[ps * GT + qt * 8 + g] = make_float2(m, l);
                });
            }
        }
    }
    if constexpr (MODE == kModeDecode) {
        finish_decode<D, HG, GT, (S::FOLD ? 1 : NSUB), NC, S::RING>(a, ring, flags, warp, lane, xpar, xe);
        if (a.fused_merge || a.xworld) return;
    }
    // Let the dependent merge kernel launch; it still waits for this grid to finish.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ------------------------------------------------------------------ partial merge
// One CTA per output row (group, KV head hh of the group, query head g):
// max-corrected merge (the oracle.py:88-96 algebra) of the partials that
// `nsub` sub-pipelines wrote for each of the group's segments.  Warp 0 finds
// the maximum M and denominator L; then each thread owns one float4 of head
// dims and every R-th partial (R = 256 / (D/4)), and the R partial sums are
// added in shared memory.  Launched programmatically dependent on the decode
// kernel: griddepcontrol.wait returns once that grid has finished and its
// writes are visible.
constexpr int kMergeThreads = 256;

template <int HG, int GT>
__global__ void __launch_bounds__(kMergeThreads) merge_partials_kernel(const DecodeArgs a, int nsub, int D) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    __shared__ float4 sums[kMergeThreads];
    __shared__ float2 top_den;
    const int64_t rowid = blockIdx.x;
    const int gi = int(rowid / (HG * GT));
    const int hh = int(rowid / GT % HG);
    const int g = int(rowid % GT);
    const int4 g0 = a.groups[2 * gi];
    const int4 g1 = a.groups[2 * gi + 1];
    if (g1.y < 0 || g >= g0.w) return;         // written directly, or a padding head
    const int parts = g1.z * nsub;
    auto slot_row = [&](int p) {
        return (int64_t(g1.y) + int64_t(p / nsub) * a.slot_stride + p % nsub) * HG + hh;
    };
    const int tid = threadIdx.x, lane = tid & 31;
    if (tid < 32) {
        float top = -INFINITY;
        for (int p = lane; p < parts; p += 32) {
            const float2 ml = a.part_ml[slot_row(p) * GT + g];
            if (ml.y > 0.f) top = fmaxf(top, ml.x);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) top = fmaxf(top, __shfl_xor_sync(kFullMask, top, o));
        float den = 0.f;
        for (int p = lane; p < parts; p += 32) {
            const float2 ml = a.part_ml[slot_row(p) * GT + g];
            if (ml.y > 0.f) den = fmaf(exp2f(ml.x - top), ml.y, den);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) den += __shfl_xor_sync(kFullMask, den, o);
        if (lane == 0) top_den = make_float2(top, den);
    }
    __syncthreads();
    const float top = top_den.x, den = top_den.y;
    const int chunks = D / 4;                   // float4 chunks per row
    const int lanes_p = kMergeThreads / chunks; // partials summed in parallel
    const int c = tid % chunks, r = tid / chunks;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
    for (int p = r; p < parts; p += lanes_p) {
        const int64_t pr = slot_row(p);
        const float2 ml = a.part_ml[pr * GT + g];
        if (ml.y > 0.f) {
            const float w = exp2f(ml.x - top);
            const float4 o = reinterpret_cast<const float4 *>(a.part_o + (pr * GT + g) * D)[c];
            acc.x = fmaf(w, o.x, acc.x);
            acc.y = fmaf(w, o.y, acc.y);
            acc.z = fmaf(w, o.z, acc.z);
            acc.w = fmaf(w, o.w, acc.w);
        }
    }
    sums[tid] = acc;
    __syncthreads();
    if (r == 0) {
        for (int k = 1; k < lanes_p; ++k) {
            const float4 v = sums[k * chunks + c];
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        const int64_t row = int64_t(g0.x) * a.Hq + int64_t(g0.y + hh) * a.group + g0.z + g;
        reinterpret_cast<float4 *>(a.out + row * D)[c] =
            den > 0.f ? make_float4(acc.x / den, acc.y / den, acc.z / den, acc.w / den)
                      : make_float4(0.f, 0.f, 0.f, 0.f);
        if (a.stats && c == 0) reinterpret_cast<float2 *>(a.stats)[row] = make_float2(top, den);
    }
}

}  // namespace pd
