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
// CTAs that only this one reaches, in the mode that never leaves (the wait
// before the in-kernel merge of a cooperative launch).
// Each wait gives up after `timeout_ns` and records PD_DEVERR_TIMEOUT.
__global__ void wait_timeout_kernel(unsigned long long *ticket, uint32_t *words,
                                    unsigned long long timeout_ns) {
    __shared__ uint64_t bar;
    if (threadIdx.x != 0) return;
    mbar_init(smem_u32(&bar), 1);
    mbar_init_fence();
    if (!mbar_wait(smem_u32(&bar), 0, timeout_ns)) atomicOr(words + 0, PD_DEVERR_TIMEOUT);
    GridBarrier gb{ticket, ticket + 1, ticket + 2, 0u, 0u};   // cooperative mode: never leaves
    unsigned left = 0;
    if (grid_arrive(gb, 2u, 0u, &left, timeout_ns) == kBarrierTimeout) atomicOr(words + 1, PD_DEVERR_TIMEOUT);
}

// One CTA at a grid barrier for two in leave mode 1.  counters: [0] arrivals,
// [1] started, [2] left bits; the caller sets `started`.
__global__ void barrier_leave_kernel(unsigned long long *counters, uint32_t *outcomes, int slot,
                                     unsigned leave_ns, unsigned long long timeout_ns) {
    if (threadIdx.x != 0) return;
    GridBarrier gb{counters, counters + 1, counters + 2, 1u, leave_ns};
    unsigned left = 0;
    outcomes[slot] = uint32_t(grid_arrive(gb, 2u, 0u, &left, timeout_ns));
    if (slot == 0) {
        outcomes[1] = uint32_t(__ldcg(counters) >> kArrivalBits);
        outcomes[2] = uint32_t(__ldcg(counters + 2) & 1ull);
    }
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
    if (err == cudaSuccess) err = cudaMalloc(&buf, 64);
    if (err == cudaSuccess) err = cudaMemset(buf, 0, 64);
    if (err == cudaSuccess) {
        auto *ticket = static_cast<unsigned long long *>(buf);     // + started, left bits
        auto *w = reinterpret_cast<uint32_t *>(static_cast<uint8_t *>(buf) + 32);
        wait_timeout_kernel<<<1, 32>>>(ticket, w, 1000ull * timeout_us);
        err = cudaGetLastError();
        if (err == cudaSuccess) err = cudaMemcpy(words, w, 8, cudaMemcpyDeviceToHost);
    }
    if (buf) cudaFree(buf);
    if (prev >= 0 && prev != device) cudaSetDevice(prev);
    if (err != cudaSuccess) return fail(PD_ERR_CUDA, std::string("self-test: ") + cudaGetErrorString(err));
    return PD_OK;
}

PD_API pd_status pd_selftest_barrier_leave(int32_t device, uint32_t leave_us, uint32_t *outcomes) {
    if (!outcomes) return fail(PD_ERR_VALUE, "outcomes must not be NULL");
    if (leave_us == 0 || leave_us > 100000u) return fail(PD_ERR_VALUE, "leave_us must be in [1, 1e5]");
    int prev = -1;
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    cudaError_t err = cudaSetDevice(device);
    void *buf = nullptr;
    if (err == cudaSuccess) err = cudaMalloc(&buf, 256);
    if (err == cudaSuccess) err = cudaMemset(buf, 0, 256);
    if (err == cudaSuccess) {
        auto *a = static_cast<unsigned long long *>(buf);          // partner never started
        auto *b = a + 8;                                            // partner started, never arrives
        auto *w = reinterpret_cast<uint32_t *>(a + 16);
        const unsigned long long one = 1, ns = 1000ull * leave_us;
        err = cudaMemcpy(a + 1, &one, 8, cudaMemcpyHostToDevice);   // only this CTA started
        const unsigned long long two = 2;
        if (err == cudaSuccess) err = cudaMemcpy(b + 1, &two, 8, cudaMemcpyHostToDevice);
        if (err == cudaSuccess) {
            barrier_leave_kernel<<<1, 32>>>(a, w, 0, unsigned(ns), 4 * ns);
            barrier_leave_kernel<<<1, 32>>>(b, w, 3, unsigned(ns), 4 * ns);
            err = cudaGetLastError();
        }
        if (err == cudaSuccess) err = cudaMemcpy(outcomes, w, 16, cudaMemcpyDeviceToHost);
    }
    if (buf) cudaFree(buf);
    if (prev >= 0 && prev != device) cudaSetDevice(prev);
    if (err != cudaSuccess) return fail(PD_ERR_CUDA, std::string("self-test: ") + cudaGetErrorString(err));
    return PD_OK;
}
