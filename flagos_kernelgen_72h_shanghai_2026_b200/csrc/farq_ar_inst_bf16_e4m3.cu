// Tensor-parallel kernel instantiations for bf16 inputs with e4m3 output (see farq_ar_kernel.cuh); compiled once per -DFARQ_AR_WMAX in {1, 2, 4, 8}.
#include "farq_ar_kernel.cuh"

FARQ_AR_KERNEL_TABLE(ar_kernel_bf16_e4m3, __nv_bfloat16, true)
