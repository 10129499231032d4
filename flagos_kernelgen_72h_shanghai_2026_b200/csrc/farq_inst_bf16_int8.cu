// Kernel instantiations for bf16 inputs with int8 quantised output (see farq_kernel.cuh).
#include "farq_kernel.cuh"

FARQ_KERNEL_TABLE(kernel_bf16_int8, __nv_bfloat16, false)
