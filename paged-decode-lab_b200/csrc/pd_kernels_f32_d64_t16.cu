// Decode and gather kernels for FP32 inputs, head_dim 64, page_size 16.
#include "pd_kernels.cuh"

PD_DEFINE_ENTRY(kernel_entry_f32_d64_t16, float, 64, 16)
