// Decode and gather kernels for FP16 inputs, head_dim 64, page_size 32.
#include "pd_kernels.cuh"

PD_DEFINE_ENTRY(kernel_entry_f16_d64_t32, __half, 64, 32)
