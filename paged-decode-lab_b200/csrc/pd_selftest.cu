// pd_selftest.cu — the decode kernel's bounded waits, run against events that
// never happen, so that their timeout path can be tested without a GPU fault.
#include <string>

#include "paged_decode.h"
#include "pd_device.cuh"
#include "pd_plan.hpp"

#define PD_API extern "C" __attribute__((visibility("default")))

namespace pd {
namespace {

// words[0]: an mbarrier phase that no thread completes (the wait a consumer
// makes for a page tile that never lands); words[1]: a grid barrier for two
// CTAs that only this one reaches (the wait before the in-kernel merge).
// Each wait gives up after `timeout_ns` and records PD_DEVERR_TIMEOUT.
__global__ void wait_timeout_kernel(unsigned long long *ticket, uint32_t *words,
                                    unsigned long long timeout_ns) {
    __shared__ uint64_t bar;
    if (threadIdx.x != 0) return;
    mbar_init(smem_u32(&bar), 1);
    mbar_init_fence();
    if (!mbar_wait(smem_u32(&bar), 0, timeout_ns)) atomicOr(words + 0, PD_DEVERR_TIMEOUT);
    if (!grid_barrier(ticket, 2u, timeout_ns)) atomicOr(words + 1, PD_DEVERR_TIMEOUT);
}

}  // namespace
}  // namespace pd

using namespace pd;

PD_API pd_status pd_selftest_wait_timeouts(int32_t device, uint32_t timeout_us, uint32_t *words) {
    if (!words) return fail(PD_ERR_VALUE, "words must not be NULL");
    if (timeout_us == 0 || timeout_us > 1000000u) return fail(PD_ERR_VALUE, "timeout_us must be in [1, 1e6]");
    int prev = -1;
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    cudaError_t err = cudaSetDevice(device);
    void *buf = nullptr;
    if (err == cudaSuccess) err = cudaMalloc(&buf, 16);
    if (err == cudaSuccess) err = cudaMemset(buf, 0, 16);
    if (err == cudaSuccess) {
        auto *ticket = static_cast<unsigned long long *>(buf);
        auto *w = reinterpret_cast<uint32_t *>(static_cast<uint8_t *>(buf) + 8);
        wait_timeout_kernel<<<1, 32>>>(ticket, w, 1000ull * timeout_us);
        err = cudaGetLastError();
        if (err == cudaSuccess) err = cudaMemcpy(words, w, 8, cudaMemcpyDeviceToHost);
    }
    if (buf) cudaFree(buf);
    if (prev >= 0 && prev != device) cudaSetDevice(prev);
    if (err != cudaSuccess) return fail(PD_ERR_CUDA, std::string("self-test: ") + cudaGetErrorString(err));
    return PD_OK;
}
