// Kernel instantiations for bf16 inputs with e4m3 quantised output (see farq_kernel.cuh).
#include "farq_kernel.cuh"

FARQ_KERNEL_TABLE(kernel_bf16_e4m3, __nv_bfloat16, true)
