// Kernel instantiations for fp16 inputs with e4m3 quantised output (see farq_kernel.cuh).
#include "farq_kernel.cuh"

FARQ_KERNEL_TABLE(kernel_fp16_e4m3, __half, true)
