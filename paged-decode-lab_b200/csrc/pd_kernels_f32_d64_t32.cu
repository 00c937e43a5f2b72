// Decode and gather kernels for FP32 inputs, head_dim 64, page_size 32.
#include "pd_kernels.cuh"

PD_DEFINE_ENTRY(kernel_entry_f32_d64_t32, float, 64, 32)
