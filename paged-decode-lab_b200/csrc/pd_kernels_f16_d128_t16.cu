// Decode and gather kernels for FP16 inputs, head_dim 128, page_size 16.
#include "pd_kernels.cuh"

PD_DEFINE_ENTRY(kernel_entry_f16_d128_t16, __half, 128, 16)
