// Tensor-parallel kernel instantiations for fp16 inputs with int8 output (see farq_ar_kernel.cuh); compiled once per -DFARQ_AR_WMAX in {1, 2, 4, 8}.
#include "farq_ar_kernel.cuh"

FARQ_AR_KERNEL_TABLE(ar_kernel_fp16_int8, __half, false)
