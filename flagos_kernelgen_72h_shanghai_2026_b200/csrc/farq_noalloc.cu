// farq_noalloc.cu — host-buffer entry point that allocates no memory.
//
// Who needs it: code that holds its tensors in host memory and is not allowed
// to allocate on the GPU — for example a plugin living inside a process whose
// device allocator belongs to another framework (a second allocator would
// fragment or exceed that framework's memory budget), or foreign-language
// callers (C, FFI bindings) that only ever see host buffers and have no device
// allocator at all. Such callers cannot call cudaMalloc, so the device memory
// this path needs to stage a call is a fixed array compiled into the library.
//
// The array (kNoAllocScratchBytes, 64 MiB) is a file-scope __device__ variable:
// every GPU that loads libfarq.so holds it until the process exits. In host
// code its name is only a host-side stand-in, never a device address; the
// device address is obtained once per device with cudaGetSymbolAddress, on
// the first call made on that device (make that first call before any stream
// capture). Every call on a device shares the array, so calls that overlap on
// the GPU (different streams, or different host threads) race on it; calls
// on one stream are ordered. Nothing in the array has to start at zero: every
// byte a call reads there was written earlier in the same call.
#include <cuda_runtime.h>
#include <stdint.h>
#include <mutex>

#include "farq.h"

namespace {

constexpr size_t kNoAllocScratchBytes = 64ull << 20;
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
uint8_t* g_noalloc_ptr[kNoAllocMaxDevices];  // device address of the array, per device

size_t up256(size_t n) { return (n + 255) / 256 * 256; }

int elem_size(int dt) {
  switch (dt) {
    case FARQ_DTYPE_BF16:
    case FARQ_DTYPE_FP16: return 2;
    case FARQ_DTYPE_FP32: return 4;
    case FARQ_DTYPE_INT8:
    case FARQ_DTYPE_E4M3: return 1;
    default: return 0;
  }
}

// Device address of the scratch array on the current device (set-up on the
// first call per device).
int scratch_address(uint8_t** out) {
  int dev;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices)
    return FARQ_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return FARQ_ERR_CUDA;
    g_noalloc_ptr[dev] = static_cast<uint8_t*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return FARQ_OK;
}

// Bytes of the array reserved at its start for the status word.
constexpr size_t kStatusBytes = 256;

// Staging bytes one call needs, for a shape that already passed
// farq::validate_args (D <= 16384, G in [8, 256]) and M <= the row limit
// below, so no term can overflow.
size_t noalloc_bytes(int64_t M, int64_t D, int32_t group_size, int32_t x_dtype,
                     int32_t gamma_dtype, int32_t residual_out_dtype, int32_t norm_out_dtype,
                     bool write_norm) {
  const size_t N = (size_t)M * (size_t)D;
  return kStatusBytes + up256(N * elem_size(x_dtype)) * 2 +
         up256((size_t)D * elem_size(gamma_dtype)) + up256(N * elem_size(residual_out_dtype)) +
         (write_norm ? up256(N * elem_size(norm_out_dtype)) : 0) + up256(N) +
         up256((size_t)M * (size_t)(D / group_size) * 4);
}

}  // namespace

namespace farq {
int validate_args(const farq_args_t* a);  // farq.cu
}

extern "C" {

int farq_launch_host_noalloc(const farq_args_t* a, void* stream) {
  // Every check comes before the first copy is queued, so a rejected call
  // leaves nothing in flight that still reads or writes the caller's buffers.
  int st = farq::validate_args(a);
  if (st != FARQ_OK) return st;
  const int64_t M = a->M, D = a->D;
  const int G = a->group_size;
  // Host tensors must be contiguous: row strides 0 or the natural ones.
  if ((a->x_row_stride && a->x_row_stride != D) ||
      (a->residual_row_stride && a->residual_row_stride != D) ||
      (a->residual_out_row_stride && a->residual_out_row_stride != D) ||
      (a->norm_out_row_stride && a->norm_out_row_stride != D) ||
      (a->x_q_row_stride && a->x_q_row_stride != D) ||
      (a->x_scale_row_stride && a->x_scale_row_stride != D / G) ||
      (a->flags & FARQ_FLAG_SCALE_COLUMN_MAJOR))
    return FARQ_ERR_BAD_SHAPE;
  if (M == 0) return FARQ_OK;
  if (!a->x || !a->residual || !a->gamma || !a->residual_out || !a->x_q || !a->x_scale)
    return FARQ_ERR_NULL_POINTER;
  // Every row stages at least its D quantised bytes, so more rows than
  // this can never fit; checking it first keeps the size sum below from
  // wrapping around for absurd M.
  if (M > (int64_t)(kNoAllocScratchBytes / (size_t)D)) return FARQ_ERR_NOALLOC_TOO_LARGE;
  const size_t need = noalloc_bytes(M, D, G, a->x_dtype, a->gamma_dtype, a->residual_out_dtype,
                                    a->norm_out_dtype, a->norm_out != nullptr);
  if (need > kNoAllocScratchBytes) return FARQ_ERR_NOALLOC_TOO_LARGE;

  uint8_t* base = nullptr;
  st = scratch_address(&base);
  if (st != FARQ_OK) return st;
  const int xs = elem_size(a->x_dtype), gs = elem_size(a->gamma_dtype),
            ros = elem_size(a->residual_out_dtype), nos = elem_size(a->norm_out_dtype);
  const size_t N = (size_t)M * (size_t)D;
  int32_t* dstatus = reinterpret_cast<int32_t*>(base);
  uint8_t* dx = base + kStatusBytes;
  uint8_t* dr = dx + up256(N * xs);
  uint8_t* dg = dr + up256(N * xs);
  uint8_t* dro = dg + up256((size_t)D * gs);
  uint8_t* dno = dro + up256(N * ros);
  uint8_t* dq = dno + (a->norm_out ? up256(N * nos) : 0);
  uint8_t* ds = dq + up256(N);
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  // The status word, when given, is a host int here: it is carried to the
  // device with the inputs and back with the outputs, keeping its contract
  // (set on a device timeout, never cleared by the library).
  if ((a->status &&
       cudaMemcpyAsync(dstatus, a->status, sizeof(int32_t), cudaMemcpyHostToDevice, s) !=
           cudaSuccess) ||
      cudaMemcpyAsync(dx, a->x, N * xs, cudaMemcpyHostToDevice, s) != cudaSuccess ||
      cudaMemcpyAsync(dr, a->residual, N * xs, cudaMemcpyHostToDevice, s) != cudaSuccess ||
      cudaMemcpyAsync(dg, a->gamma, (size_t)D * gs, cudaMemcpyHostToDevice, s) != cudaSuccess)
    return FARQ_ERR_CUDA;
  farq_args_t d = *a;
  d.x = dx;
  d.residual = dr;
  d.gamma = dg;
  d.residual_out = dro;
  d.norm_out = a->norm_out ? dno : nullptr;
  d.x_q = dq;
  d.x_scale = reinterpret_cast<float*>(ds);
  d.status = a->status ? dstatus : nullptr;
  d.x_row_stride = d.residual_row_stride = d.residual_out_row_stride = 0;
  d.norm_out_row_stride = d.x_q_row_stride = d.x_scale_row_stride = 0;
  // Everything farq_launch checks beyond validate_args concerns the staged
  // device pointers, which are 256-byte aligned and contiguous.
  st = farq_launch(&d, stream);
  if (st != FARQ_OK) return st;
  if (cudaMemcpyAsync(a->residual_out, dro, N * ros, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      (a->norm_out &&
       cudaMemcpyAsync(a->norm_out, dno, N * nos, cudaMemcpyDeviceToHost, s) != cudaSuccess) ||
      cudaMemcpyAsync(a->x_q, dq, N, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaMemcpyAsync(a->x_scale, ds, (size_t)M * (D / G) * 4, cudaMemcpyDeviceToHost, s) !=
          cudaSuccess ||
      (a->status &&
       cudaMemcpyAsync(a->status, dstatus, sizeof(int32_t), cudaMemcpyDeviceToHost, s) !=
           cudaSuccess))
    return FARQ_ERR_CUDA;
  return FARQ_OK;
}

}  // extern "C"
