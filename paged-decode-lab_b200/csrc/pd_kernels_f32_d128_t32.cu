// Decode and gather kernels for FP32 inputs, head_dim 128, page_size 32.
#include "pd_kernels.cuh"

PD_DEFINE_ENTRY(kernel_entry_f32_d128_t32, float, 128, 32)
