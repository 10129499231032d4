// Kernel instantiations for fp16 inputs with int8 quantised output (see farq_kernel.cuh).
#include "farq_kernel.cuh"

FARQ_KERNEL_TABLE(kernel_fp16_int8, __half, false)
