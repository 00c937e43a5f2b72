// pd_merge.cu — merge of per-shard decode results (sequence sharding across GPUs).
#include "pd_kernels.cuh"

namespace pd {

// ------------------------------------------------------------------ cross-shard merge
// out[row] = sum_s exp2(m_s - M) * l_s * o_s / sum_s exp2(m_s - M) * l_s over shards
// with l_s > 0 (o_s is each shard's normalised output); zero when all are empty.
// Shard s's rows start at shard_out + s * stride and shard_stats + s * stride.
static __global__ void merge_shards_kernel(const float *__restrict__ shard_out,
                                    const float *__restrict__ shard_stats, int shards, int64_t stride,
                                    int64_t rows, int D, float *__restrict__ out) {
    const int64_t row = int64_t(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    float top = -INFINITY;
    for (int s = 0; s < shards; ++s) {
        const float2 ml = *reinterpret_cast<const float2 *>(shard_stats + int64_t(s) * stride + 2 * row);
        if (ml.y > 0.f) top = fmaxf(top, ml.x);
    }
    float den = 0.f;
    for (int s = 0; s < shards; ++s) {
        const float2 ml = *reinterpret_cast<const float2 *>(shard_stats + int64_t(s) * stride + 2 * row);
        if (ml.y > 0.f) den = fmaf(exp2f(ml.x - top), ml.y, den);
    }
    for (int d = lane; d < D; d += 32) {
        float num = 0.f;
        for (int s = 0; s < shards; ++s) {
            const float2 ml = *reinterpret_cast<const float2 *>(shard_stats + int64_t(s) * stride + 2 * row);
            if (ml.y > 0.f)
                num = fmaf(exp2f(ml.x - top) * ml.y, shard_out[int64_t(s) * stride + row * D + d], num);
        }
        out[row * D + d] = den > 0.f ? num / den : 0.f;
    }
}


template <int HG, int GT>
static cudaError_t launch_merge(const DecodeArgs &args, int nsub, int D, cudaStream_t stream) {
    const int64_t rows = int64_t(args.num_groups) * HG * GT;
    if (rows > INT32_MAX) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(rows));
    cfg.blockDim = dim3(kMergeThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, merge_partials_kernel<HG, GT>, args, nsub, D);
}

cudaError_t launch_merge_partials(const DecodeArgs &args, int hg, int gt, int nsub, int D,
                                  cudaStream_t stream) {
    switch (gt * 16 + hg) {
        case 8 * 16 + 1: return launch_merge<1, 8>(args, nsub, D, stream);
        case 8 * 16 + 2: return launch_merge<2, 8>(args, nsub, D, stream);
        case 8 * 16 + 4: return launch_merge<4, 8>(args, nsub, D, stream);
        case 8 * 16 + 8: return launch_merge<8, 8>(args, nsub, D, stream);
        case 16 * 16 + 1: return launch_merge<1, 16>(args, nsub, D, stream);
        case 16 * 16 + 2: return launch_merge<2, 16>(args, nsub, D, stream);
        case 16 * 16 + 4: return launch_merge<4, 16>(args, nsub, D, stream);
        case 16 * 16 + 8: return launch_merge<8, 16>(args, nsub, D, stream);
        case 32 * 16 + 1: return launch_merge<1, 32>(args, nsub, D, stream);
        case 32 * 16 + 2: return launch_merge<2, 32>(args, nsub, D, stream);
        case 32 * 16 + 4: return launch_merge<4, 32>(args, nsub, D, stream);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_merge_shards(const float *shard_out, const float *shard_stats, int shards, int64_t stride,
                                int64_t rows, int D, float *out, cudaStream_t stream) {
    constexpr int kRowsPerBlock = 8;
    const int64_t blocks = (rows + kRowsPerBlock - 1) / kRowsPerBlock;
    merge_shards_kernel<<<unsigned(blocks), kRowsPerBlock * 32, 0, stream>>>(shard_out, shard_stats, shards,
                                                                             stride, rows, D, out);
    return cudaGetLastError();
}

}  // namespace pd
