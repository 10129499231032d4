// dsa_topk.cu — host side of libdsa_topk.so: argument validation, launch
// planning and the C ABI declared in include/dsa_topk.h. Device code:
// dsa_topk_kernel.cuh.
//
// The reference routes each (B, H, Q, NB, top_k, block_size) to one of a
// dozen Triton pipelines (single-program sort, chunk-local select + merge,
// radix threshold; src/task02_dsa_topk_page_table_transform.py:1666-1726).
// Here one kernel covers every shape; the host only picks the CTA width T
// and the four-score vectors per thread J (a row holds at most 4 * J * T
// scores) and sizes a persistent grid from the occupancy of that kernel.
#include <cuda_runtime.h>
#include <stdint.h>
#include <atomic>

#include "dsa_topk.h"
#include "dsa_topk_kernel.cuh"

namespace dsa {

constexpr int kMaxJ = 8;
constexpr int kMaxDevices = 64;
constexpr int kSlots = 3 * kMaxJ * 3;  // dtype x J x T
std::atomic<int> g_sm_count[kMaxDevices];
std::atomic<int> g_occ[kMaxDevices][kSlots];        // resident CTAs per SM (0 = unknown)
std::atomic<int> g_occ_smem[kMaxDevices][kSlots];   // dynamic smem the occupancy was taken at
std::atomic<int> g_smem_set[kMaxDevices][kSlots];   // dynamic smem granted to the kernel

// Instantiated shapes: 128 threads with J = 1..8 (NB <= 4096); 256 and 512
// threads with J = 5..8 (4096 < NB <= 16384).
template <typename S, int NT>
KernelFn pick_j(int J) {
  switch (J) {
    case 1: return NT == 128 ? dsa_topk_kernel<S, 1, 128> : nullptr;
    case 2: return NT == 128 ? dsa_topk_kernel<S, 2, 128> : nullptr;
    case 3: return NT == 128 ? dsa_topk_kernel<S, 3, 128> : nullptr;
    case 4: return NT == 128 ? dsa_topk_kernel<S, 4, 128> : nullptr;
    case 5: return dsa_topk_kernel<S, 5, NT>;
    case 6: return dsa_topk_kernel<S, 6, NT>;
    case 7: return dsa_topk_kernel<S, 7, NT>;
    case 8: return dsa_topk_kernel<S, 8, NT>;
    default: return nullptr;
  }
}

template <typename S>
KernelFn pick_t(int J, int T) {
  switch (T) {
    case 128: return pick_j<S, 128>(J);
    case 256: return pick_j<S, 256>(J);
    case 512: return pick_j<S, 512>(J);
    default: return nullptr;
  }
}

KernelFn topk_kernel(int scores_dtype, int J, int T) {
  switch (scores_dtype) {
    case DSA_DTYPE_FP32: return pick_t<float>(J, T);
    case DSA_DTYPE_BF16: return pick_t<__nv_bfloat16>(J, T);
    case DSA_DTYPE_FP16: return pick_t<__half>(J, T);
    default: return nullptr;
  }
}

int index_size(int dt) {
  return dt == DSA_DTYPE_INT32 ? 4 : dt == DSA_DTYPE_INT64 ? 8 : 0;
}
int score_size(int dt) {
  return dt == DSA_DTYPE_FP32 ? 4 : (dt == DSA_DTYPE_BF16 || dt == DSA_DTYPE_FP16) ? 2 : 0;
}
bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// CTA width and vectors per thread for a row of NB scores (nvec = NB / 4
// four-score vectors, each thread holds J <= 8 of them, i.e. at most 32
// keys in registers): 128 threads up to NB = 4096, then 256 and 512.
void pick_shape(int64_t NB, int* T, int* J) {
  const int64_t nvec = NB / 4;
  *T = nvec <= 128 * 8 ? 128 : nvec <= 256 * 8 ? 256 : 512;
  *J = (int)((nvec + *T - 1) / *T);
}

// Lower-bound groups: a thread vouches for its vouch_of(J) largest vector
// maxima (4, 2 or 1 distinct keys), and so does a group of g threads (the
// merged lists). g = the largest power of two <= 32 that leaves
// vouch * T / g >= K (group 0 when even g = 1 falls short: no bound). A
// thread whose vectors are masked vouches for keys 0, which turns the bound
// off for that row (the kernel then takes every selectable key).
int pick_group(int T, int J, int K) {
  const int vouch = vouch_of(J);
  if (K > vouch * T) return 0;
  int g = 1;
  while (g < 32 && vouch * T / (2 * g) >= K) g *= 2;
  return g;
}

int validate(const dsa_topk_args_t* a) {
  if (!a) return DSA_ERR_NULL_POINTER;
  if (a->struct_size != sizeof(dsa_topk_args_t) || a->reserved0 != 0) return DSA_ERR_BAD_ARGS_SIZE;
  if (a->B < 0 || a->H < 0 || a->Q < 0 || a->NB < 1 || a->NB % 4 != 0 || a->block_size < 1)
    return DSA_ERR_BAD_SHAPE;
  if (a->top_k < 1 || a->top_k > kMaxTopK) return DSA_ERR_BAD_TOPK;
  if (!score_size(a->scores_dtype) || !index_size(a->index_dtype) || !index_size(a->page_dtype) ||
      !index_size(a->blocks_dtype))
    return DSA_ERR_BAD_DTYPE;
  if (a->NB > kMaxBlocks) return DSA_ERR_UNSUPPORTED;
  // rows * NB and rows * K must not overflow (a shape beyond any memory).
  const int64_t lim = (int64_t)1 << 40;
  if (a->B > lim || a->H > lim || a->Q > lim) return DSA_ERR_BAD_SHAPE;
  const double rows = (double)a->B * (double)a->H * (double)a->Q;
  if (rows * (double)a->NB > 9.0e18 || rows * (double)a->top_k > 9.0e18) return DSA_ERR_BAD_SHAPE;
  // rows are indexed in 32 bits on the device (B*H*Q < 2^31)
  if (rows >= 2147483648.0) return DSA_ERR_UNSUPPORTED;
  return DSA_OK;
}

}  // namespace dsa

using namespace dsa;

extern "C" {

int dsa_topk_abi_version(void) { return DSA_TOPK_ABI_VERSION; }

const char* dsa_topk_strerror(int status) {
  switch (status) {
    case DSA_OK: return "ok";
    case DSA_ERR_NULL_POINTER: return "a required pointer is NULL";
    case DSA_ERR_BAD_SHAPE:
      return "bad shape: need B, H, Q >= 0, NB >= 1, NB % 4 == 0 and block_size >= 1";
    case DSA_ERR_BAD_TOPK: return "top_k must be in [1, 2048]";
    case DSA_ERR_BAD_DTYPE: return "unsupported dtype (scores fp32/bf16/fp16, indices int32/int64)";
    case DSA_ERR_ALIGNMENT:
      return "misaligned pointer (scores 16-byte aligned, index tensors aligned to their element size)";
    case DSA_ERR_UNSUPPORTED: return "NB > 16384 or B*H*Q >= 2^31 is not supported";
    case DSA_ERR_CUDA: return "a CUDA runtime call failed";
    case DSA_ERR_BAD_ARGS_SIZE:
      return "argument struct size mismatch (header and library differ) or reserved field not 0";
    default: return "unknown dsa_topk status";
  }
}

int dsa_topk_launch(const dsa_topk_args_t* a, void* stream) {
  int st = validate(a);
  if (st != DSA_OK) return st;
  const int64_t rows = a->B * a->H * a->Q;
  if (rows == 0) return DSA_OK;
  if (!a->scores || !a->page_table || !a->q_pos || !a->kv_lens || !a->out_blocks || !a->out_pages)
    return DSA_ERR_NULL_POINTER;
  const int ib = index_size(a->index_dtype), pb = index_size(a->page_dtype),
            bb = index_size(a->blocks_dtype);
  if (!aligned(a->scores, 16) || !aligned(a->page_table, pb) || !aligned(a->out_pages, pb) ||
      !aligned(a->q_pos, ib) || !aligned(a->kv_lens, ib) || !aligned(a->out_blocks, bb))
    return DSA_ERR_ALIGNMENT;

  int T, J;
  pick_shape(a->NB, &T, &J);
  KernelFn fn = topk_kernel(a->scores_dtype, J, T);
  if (!fn) return DSA_ERR_UNSUPPORTED;
  const int slot = (a->scores_dtype * kMaxJ + (J - 1)) * 3 + (T == 128 ? 0 : T == 256 ? 1 : 2);

  int dev;
  if (cudaGetDevice(&dev) != cudaSuccess) return DSA_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return DSA_ERR_CUDA;
  int sms = g_sm_count[dev].load(std::memory_order_relaxed);
  if (sms <= 0) {
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return DSA_ERR_CUDA;
    g_sm_count[dev].store(sms, std::memory_order_relaxed);
  }
  const int cap = candidate_cap(a->top_k);
  const int vec_bytes = score_size(a->scores_dtype) * 4;
  const int smem = (int)smem_layout(T, J, vec_bytes, a->top_k, cap).total;
  if (smem > g_smem_set[dev][slot].load(std::memory_order_relaxed)) {
    if (cudaFuncSetAttribute(reinterpret_cast<const void*>(fn),
                             cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return DSA_ERR_CUDA;
    g_smem_set[dev][slot].store(smem, std::memory_order_relaxed);
  }
  int occ = g_occ[dev][slot].load(std::memory_order_relaxed);
  if (occ <= 0 || g_occ_smem[dev][slot].load(std::memory_order_relaxed) != smem) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, T, smem) != cudaSuccess)
      return DSA_ERR_CUDA;
    if (occ < 1) return DSA_ERR_UNSUPPORTED;
    g_occ[dev][slot].store(occ, std::memory_order_relaxed);
    g_occ_smem[dev][slot].store(smem, std::memory_order_relaxed);
  }
  int64_t grid = (int64_t)sms * occ;
  if (grid > rows) grid = rows;

  Params p;
  p.scores = a->scores;
  p.page_table = a->page_table;
  p.q_pos = a->q_pos;
  p.kv_lens = a->kv_lens;
  p.out_blocks = a->out_blocks;
  p.out_pages = a->out_pages;
  p.rows = rows;
  p.HQ = a->H * a->Q;
  p.Q = a->Q;
  p.NB = (int32_t)a->NB;
  p.K = a->top_k;
  p.block_size = a->block_size;
  p.index_bytes = ib;
  p.page_bytes = pb;
  p.blocks_bytes = bb;
  p.cap = cap;
  p.group = pick_group(T, J, a->top_k);
  fast_div_init((uint32_t)p.HQ, &p.hq_mul, &p.hq_shift);
  fast_div_init((uint32_t)p.Q, &p.q_mul, &p.q_shift);

  // Programmatic stream serialisation: this launch may start while the
  // previous kernel in the stream drains; the kernel waits for it
  // (griddepcontrol.wait) before its first global-memory access.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(T);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, fn, p) != cudaSuccess) return DSA_ERR_CUDA;
  return DSA_OK;
}

}  // extern "C"
