// Decode and gather kernels for FP32 inputs, head_dim 128, page_size 16.
#include "pd_kernels.cuh"

PD_DEFINE_ENTRY(kernel_entry_f32_d128_t16, float, 128, 16)
