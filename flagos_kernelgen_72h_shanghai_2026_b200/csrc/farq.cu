// farq.cu — B200 (sm_100a) fused residual-add + RMSNorm + per-token group
// quantisation, exported through the C ABI declared in include/farq.h.
//
// Reference behaviour (sinpeyw/flagos-kernelgen-72h-shanghai-2026,
// src/task01_fused_add_rmsnorm_group_quant.py):
//   per-row math ............ :65-121 (full row), :1127-1348 (segmented),
//                             :1401-1546 (two rows per program)
//   quantisation ............ :1089-1104  scale = max(gmax*(inv/127), 1e-12),
//                                         q = trunc(clamp(norm*(1/scale), ±127))
//   reduction ............... :1274-1278  inv = rsqrt(sum(r*r)/D + eps), fp32
//   entry / routing ......... :1731-1851
//
// Design (one kernel for every shape the reference routes separately):
//   * Persistent CTAs; CTA b owns rows b, b+grid, b+2*grid, ...
//   * Each row of x and residual is brought into a shared-memory pipeline
//     stage by two cp.async.bulk copies (the TMA engine, no multicast) that
//     complete on an mbarrier; `stages` rows per CTA are in flight.
//   * Thread t of an NT-thread CTA owns the 16-byte vectors v = k*NT + t,
//     k < K, of every row. gamma for those columns lives in registers for
//     the life of the CTA, so shared memory holds only x and residual.
//   * Phase 1 (per row): r = x + residual in fp32, residual_out written once
//     (streaming store), sum of r*r, w = r*gamma kept in registers, group
//     absmax by xor-shuffles across the G/8 lanes that share a group.
//   * sum(r*r) is accumulated in fp64 (exact squares of fp32 values, error
//     ~1e-16 relative) and rounded to fp32 once, so inv_rms does not depend
//     on the summation order. With fp32 accumulation every ulp of inv_rms
//     flips the group-maximum element between 126 and 127 (it sits on
//     exactly ±QMAX mathematically), which alone would cost ~0.4% of q at
//     G=64.
//   * One CTA barrier reduces sum(r*r); right after it the stage is free and
//     the next row is queued into it, so the copy overlaps phase 2.
//   * Phase 2: norm = w*inv_rms, scale, q (int8 truncation or e4m3
//     round-to-nearest-even with saturation), streaming stores.
//   * Every wait on the device is bounded; a wait that runs out sets the
//     caller's status word and the CTA drains its copies and returns.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <atomic>

#include "farq.h"

namespace farq {

constexpr int kMaxK = 4;              // 16-byte vectors per thread per row
constexpr int kMaxThreads = 512;      // threads per CTA
constexpr int64_t kMaxHidden = (int64_t)kMaxK * kMaxThreads * 8;  // 16384
constexpr int kMaxStages = 8;
constexpr uint32_t kSpinLimit = 1u << 26;  // bounded mbarrier polls

struct Params {
  const uint8_t* x;
  const uint8_t* res;
  const void* gamma;
  uint8_t* rout;
  uint8_t* nout;     // may be null
  uint8_t* q;
  float* scale;
  int32_t* status;   // may be null
  int64_t M;
  int64_t sx, sr, sro, sno, sq, ss;  // row strides in bytes (scale: floats)
  int32_t D;
  int32_t nvec;      // D / 8
  int32_t G;
  int32_t glanes;    // G / 8
  int32_t gamma_dtype, rout_dtype, nout_dtype;
  int32_t ue8m0;
  int32_t stages;
  uint32_t row_bytes;  // D * sizeof(x element)
  float eps;
};

// ---------------------------------------------------------------- PTX helpers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: true when the phase completed, false when the poll limit ran out.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
  for (uint32_t i = 0; i < kSpinLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
// Global -> shared bulk copy through the TMA engine, completion counted in
// bytes on `bar`. Destination is this CTA's own shared memory.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(pol)
      : "memory");
}
__device__ __forceinline__ void st_cs_v4(void* p, uint4 v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void st_cs_v2(void* p, uint32_t a, uint32_t b) {
  asm volatile("st.global.cs.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(a), "r"(b) : "memory");
}
__device__ __forceinline__ void st_cs_f32(float* p, float v) {
  asm volatile("st.global.cs.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}

// ------------------------------------------------------------ element formats
__device__ __forceinline__ void unpack8(const uint4 v, float f[8], __nv_bfloat16*) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
__device__ __forceinline__ void unpack8(const uint4 v, float f[8], __half*) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
    float2 t = __half22float2(h);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
__device__ __forceinline__ uint32_t pack2(float a, float b, int dtype) {
  if (dtype == FARQ_DTYPE_BF16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
// Store 8 fp32 values as `dtype` (BF16/FP16 round-to-nearest-even, or FP32)
// at element offset 8*v of row pointer `row`.
__device__ __forceinline__ void store8(uint8_t* row, int v, const float f[8], int dtype) {
  if (dtype == FARQ_DTYPE_FP32) {
    float* p = reinterpret_cast<float*>(row) + 8 * (int64_t)v;
    st_cs_v4(p, make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                           __float_as_uint(f[3])));
    st_cs_v4(p + 4, make_uint4(__float_as_uint(f[4]), __float_as_uint(f[5]),
                               __float_as_uint(f[6]), __float_as_uint(f[7])));
  } else {
    uint4 o;
    o.x = pack2(f[0], f[1], dtype);
    o.y = pack2(f[2], f[3], dtype);
    o.z = pack2(f[4], f[5], dtype);
    o.w = pack2(f[6], f[7], dtype);
    st_cs_v4(row + 16 * (int64_t)v, o);
  }
}
__device__ __forceinline__ void load_gamma8(const void* g, int v, int dtype, float f[8]) {
  if (dtype == FARQ_DTYPE_FP32) {
    const float4* p = reinterpret_cast<const float4*>(g) + 2 * (int64_t)v;
    float4 a = __ldg(p), b = __ldg(p + 1);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
    f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  } else {
    uint4 raw = __ldg(reinterpret_cast<const uint4*>(g) + v);
    if (dtype == FARQ_DTYPE_BF16)
      unpack8(raw, f, (__nv_bfloat16*)nullptr);
    else
      unpack8(raw, f, (__half*)nullptr);
  }
}
// Two fp32 -> two e4m3 bytes, round-to-nearest-even, saturating to ±448.
// Result low byte = lo, high byte = hi.
__device__ __forceinline__ uint32_t e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint32_t i8(float v) {
  v = fminf(fmaxf(v, -127.0f), 127.0f);
  return static_cast<uint32_t>(__float2int_rz(v)) & 0xffu;
}
// Round a positive normal fp32 up to the next power of two (identity on
// powers of two): clear the mantissa, bump the exponent if it was non-zero.
__device__ __forceinline__ float pow2_ceil(float s) {
  uint32_t b = __float_as_uint(s);
  if (b & 0x007fffffu) b = (b & 0xff800000u) + 0x00800000u;
  return __uint_as_float(b);
}

// -------------------------------------------------------------------- kernel
template <typename Tin, int K, bool E4M3>
__global__ void __launch_bounds__(kMaxThreads, 1) farq_rows_kernel(const Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x;
  const int NT = blockDim.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int nwarps = NT >> 5;
  const int S = p.stages;
  const uint32_t stage_bytes = 2u * p.row_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)S * stage_bytes);
  double* red = reinterpret_cast<double*>(bars + kMaxStages);
  __shared__ int s_abort;

  const int64_t nrows = (p.M - blockIdx.x + gridDim.x - 1) / gridDim.x;  // rows of this CTA
  if (nrows <= 0) return;

  uint64_t pol = 0;
  if (tid == 0) {
    pol = policy_evict_first();
    for (int s = 0; s < S; ++s) mbar_init(smem_u32(&bars[s]), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    s_abort = 0;
  }
  __syncthreads();
  int64_t issued = 0;  // rows queued (thread 0 only)
  if (tid == 0) {
    for (; issued < nrows && issued < S; ++issued) {
      const int64_t row = blockIdx.x + issued * gridDim.x;
      const uint32_t bar = smem_u32(&bars[issued]);
      const uint32_t dst = smem_u32(smem + (size_t)issued * stage_bytes);
      mbar_arrive_expect_tx(bar, stage_bytes);
      bulk_load(dst, p.x + row * p.sx, p.row_bytes, bar, pol);
      bulk_load(dst + p.row_bytes, p.res + row * p.sr, p.row_bytes, bar, pol);
    }
  }

  // gamma for this thread's columns, fp32, for the life of the CTA.
  float gam[K][8];
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const int v = k * NT + tid;
    if (v < p.nvec) {
      load_gamma8(p.gamma, v, p.gamma_dtype, gam[k]);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) gam[k][e] = 0.f;
    }
  }

  const float qmax = E4M3 ? 448.0f : 127.0f;
  int64_t consumed = nrows;  // rows whose copy was waited for

  for (int64_t i = 0; i < nrows; ++i) {
    const int s = (int)(i % S);
    const uint32_t parity = (uint32_t)((i / S) & 1);
    const bool ok = mbar_wait_bounded(smem_u32(&bars[s]), parity);
    if (__syncthreads_or(!ok)) {
      if (tid == 0 && p.status) atomicExch(p.status, (int)FARQ_ERR_DEVICE_TIMEOUT);
      if (tid == 0) s_abort = 1;
      consumed = i;
      break;
    }
    const int64_t row = blockIdx.x + i * gridDim.x;
    const uint8_t* sx = smem + (size_t)s * stage_bytes;
    const uint8_t* sr = sx + p.row_bytes;
    uint8_t* rout_row = p.rout + row * p.sro;

    // ---- phase 1
    float w[K][8];
    float gmax[K];
    double ss = 0.0;  // sum of r*r, accumulated in fp64 (see header)
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int v = k * NT + tid;
      float m = 0.f;
      if (v < p.nvec) {
        const uint4 xv = reinterpret_cast<const uint4*>(sx)[v];
        const uint4 rv = reinterpret_cast<const uint4*>(sr)[v];
        float a[8], b[8];
        unpack8(xv, a, (Tin*)nullptr);
        unpack8(rv, b, (Tin*)nullptr);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          a[e] = a[e] + b[e];
          ss = fma((double)a[e], (double)a[e], ss);
          w[k][e] = a[e] * gam[k][e];
          m = fmaxf(m, fabsf(w[k][e]));
        }
        store8(rout_row, v, a, p.rout_dtype);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) w[k][e] = 0.f;
      }
      for (int o = 1; o < p.glanes; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      gmax[k] = m;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) red[warp] = ss;
    __syncthreads();

    // Stage s is no longer read: queue the row that will use it next.
    if (tid == 0 && issued < nrows) {
      const int64_t nrow = blockIdx.x + issued * gridDim.x;
      const int ns = (int)(issued % S);  // == s
      const uint32_t bar = smem_u32(&bars[ns]);
      const uint32_t dst = smem_u32(smem + (size_t)ns * stage_bytes);
      mbar_arrive_expect_tx(bar, stage_bytes);
      bulk_load(dst, p.x + nrow * p.sx, p.row_bytes, bar, pol);
      bulk_load(dst + p.row_bytes, p.res + nrow * p.sr, p.row_bytes, bar, pol);
      ++issued;
    }

    double total = 0.0;
    for (int j = 0; j < nwarps; ++j) total += red[j];
    const float inv_rms =
        __frcp_rn(__fsqrt_rn(__fadd_rn(__fdiv_rn(__double2float_rn(total), (float)p.D), p.eps)));
    const float step = __fdiv_rn(inv_rms, qmax);

    // ---- phase 2
    uint8_t* nout_row = p.nout ? p.nout + row * p.sno : nullptr;
    uint8_t* q_row = p.q + row * p.sq;
    float* sc_row = p.scale + row * p.ss;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int v = k * NT + tid;
      if (v < p.nvec) {
        float sc = fmaxf(gmax[k] * step, 1.0e-12f);
        if (p.ue8m0) sc = pow2_ceil(sc);
        const float isc = __frcp_rn(sc);
        float nrm[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) nrm[e] = w[k][e] * inv_rms;
        if (nout_row) store8(nout_row, v, nrm, p.nout_dtype);
        uint32_t lo, hi;
        if (E4M3) {
          lo = e4m3x2(nrm[0] * isc, nrm[1] * isc) | (e4m3x2(nrm[2] * isc, nrm[3] * isc) << 16);
          hi = e4m3x2(nrm[4] * isc, nrm[5] * isc) | (e4m3x2(nrm[6] * isc, nrm[7] * isc) << 16);
        } else {
          lo = i8(nrm[0] * isc) | (i8(nrm[1] * isc) << 8) | (i8(nrm[2] * isc) << 16) |
               (i8(nrm[3] * isc) << 24);
          hi = i8(nrm[4] * isc) | (i8(nrm[5] * isc) << 8) | (i8(nrm[6] * isc) << 16) |
               (i8(nrm[7] * isc) << 24);
        }
        st_cs_v2(q_row + 8 * (int64_t)v, lo, hi);
        if ((lane & (p.glanes - 1)) == 0) st_cs_f32(sc_row + (v / p.glanes), sc);
      }
    }
  }

  // Abort path: make sure no bulk copy still targets this CTA's shared memory.
  __syncthreads();
  if (s_abort && tid == 0) {
    // Copies for rows [consumed, issued) may still be in flight.
    for (int64_t j = consumed; j < issued; ++j) {
      const int s = (int)(j % S);
      const uint32_t parity = (uint32_t)((j / S) & 1);
      (void)mbar_wait_bounded(smem_u32(&bars[s]), parity);
    }
  }
}

// ---------------------------------------------------------------- host side
using KernelFn = void (*)(const Params);

template <typename Tin, bool E4M3>
KernelFn pick_k(int K) {
  switch (K) {
    case 1: return farq_rows_kernel<Tin, 1, E4M3>;
    case 2: return farq_rows_kernel<Tin, 2, E4M3>;
    case 3: return farq_rows_kernel<Tin, 3, E4M3>;
    default: return farq_rows_kernel<Tin, 4, E4M3>;
  }
}
KernelFn pick_kernel(int x_dtype, bool e4m3, int K) {
  if (x_dtype == FARQ_DTYPE_BF16)
    return e4m3 ? pick_k<__nv_bfloat16, true>(K) : pick_k<__nv_bfloat16, false>(K);
  return e4m3 ? pick_k<__half, true>(K) : pick_k<__half, false>(K);
}

constexpr int kMaxDevices = 64;
std::atomic<int> g_sm_count[kMaxDevices];
std::atomic<int> g_smem_optin[kMaxDevices];
// Largest dynamic shared memory already granted, per device and kernel slot.
constexpr int kSlots = 2 * 2 * kMaxK;
std::atomic<int> g_smem_set[kMaxDevices][kSlots];

int kernel_slot(int x_dtype, bool e4m3, int K) {
  return ((x_dtype == FARQ_DTYPE_BF16 ? 0 : 1) * 2 + (e4m3 ? 1 : 0)) * kMaxK + (K - 1);
}

cudaError_t device_info(int* dev, int* sms, int* smem_optin) {
  cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return e;
  if (*dev < 0 || *dev >= kMaxDevices) return cudaErrorInvalidDevice;
  int s = g_sm_count[*dev].load(std::memory_order_relaxed);
  int o = g_smem_optin[*dev].load(std::memory_order_relaxed);
  if (s <= 0 || o <= 0) {
    e = cudaDeviceGetAttribute(&s, cudaDevAttrMultiProcessorCount, *dev);
    if (e != cudaSuccess) return e;
    e = cudaDeviceGetAttribute(&o, cudaDevAttrMaxSharedMemoryPerBlockOptin, *dev);
    if (e != cudaSuccess) return e;
    g_sm_count[*dev].store(s, std::memory_order_relaxed);
    g_smem_optin[*dev].store(o, std::memory_order_relaxed);
  }
  *sms = s;
  *smem_optin = o;
  return cudaSuccess;
}

int dtype_size(int dt) {
  switch (dt) {
    case FARQ_DTYPE_BF16:
    case FARQ_DTYPE_FP16: return 2;
    case FARQ_DTYPE_FP32: return 4;
    case FARQ_DTYPE_INT8:
    case FARQ_DTYPE_E4M3: return 1;
    default: return 0;
  }
}
bool is_float_out(int dt) {
  return dt == FARQ_DTYPE_BF16 || dt == FARQ_DTYPE_FP16 || dt == FARQ_DTYPE_FP32;
}

struct Plan {
  int threads, K, grid, stages;
  size_t smem;
};

// Shared memory per SM usable by resident CTAs (B200: 228 KB, 1 KB of it
// reserved by the system per CTA).
constexpr int kSmemPerSm = 228 * 1024;
constexpr int kSmemReservedPerCta = 1024;

int make_plan(int64_t M, int64_t D, int x_dtype, int sms, int smem_optin, int tune_ctas,
              int tune_stages, Plan* pl) {
  const int64_t nvec = D / 8;
  int K = (int)((nvec + 255) / 256);
  if (K < 1) K = 1;
  if (K > kMaxK) K = kMaxK;
  int64_t per = (nvec + K - 1) / K;
  int threads = (int)((per + 31) / 32) * 32;
  if (threads > kMaxThreads) return FARQ_ERR_UNSUPPORTED;
  const size_t row_bytes = (size_t)D * dtype_size(x_dtype);
  const size_t stage = 2 * row_bytes;
  const size_t fixed = sizeof(uint64_t) * kMaxStages + sizeof(double) * 32;
  // Default: two CTAs per SM when each can keep >= 2 rows in flight,
  // otherwise one CTA per SM with as many stages as fit.
  int ctas = tune_ctas > 0 ? tune_ctas : 0;
  int stages = tune_stages > 0 ? tune_stages : 0;
  auto max_stages_for = [&](int c) -> int {
    int64_t budget = kSmemPerSm / c - kSmemReservedPerCta - 64;
    if (budget > smem_optin) budget = smem_optin;
    budget -= (int64_t)fixed;
    if (budget <= 0) return 0;
    int64_t s = budget / (int64_t)stage;
    return (int)(s > kMaxStages ? kMaxStages : s);
  };
  if (ctas == 0) {
    ctas = (max_stages_for(2) >= 2 && threads * 2 <= 1024) ? 2 : 1;
  }
  int smax = max_stages_for(ctas);
  if (smax < 1) return FARQ_ERR_UNSUPPORTED;
  if (stages == 0) stages = smax < 4 ? smax : 4;
  if (stages > smax) stages = smax;
  int64_t grid = (int64_t)sms * ctas;
  if (grid > M) grid = M;
  if (grid < 1) grid = 1;
  pl->threads = threads;
  pl->K = K;
  pl->grid = (int)grid;
  pl->stages = stages;
  pl->smem = stage * stages + fixed;
  return FARQ_OK;
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

}  // namespace farq

using namespace farq;

extern "C" {

int farq_abi_version(void) { return FARQ_ABI_VERSION; }

int64_t farq_max_hidden(void) { return kMaxHidden; }

const char* farq_strerror(int status) {
  switch (status) {
    case FARQ_OK: return "ok";
    case FARQ_ERR_NULL_POINTER: return "a required pointer is NULL";
    case FARQ_ERR_BAD_SHAPE: return "bad shape: need M >= 0, D > 0, D % 8 == 0 and D % group_size == 0";
    case FARQ_ERR_BAD_GROUP: return "group_size must be a power of two in [8, 256]";
    case FARQ_ERR_BAD_DTYPE: return "unsupported dtype combination";
    case FARQ_ERR_ALIGNMENT: return "misaligned pointer or row stride (16-byte rows required)";
    case FARQ_ERR_UNSUPPORTED: return "hidden size above the supported maximum (16384)";
    case FARQ_ERR_CUDA: return "a CUDA runtime call failed";
    case FARQ_ERR_BAD_ARGS_SIZE: return "farq_args_t size mismatch (header and library differ)";
    case FARQ_ERR_DEVICE_TIMEOUT: return "a bounded device-side wait ran out";
    default: return "unknown farq status";
  }
}

int farq_plan(int64_t M, int64_t D, int32_t group_size, int32_t x_dtype, int32_t tune_ctas_per_sm,
              int32_t tune_stages, int64_t out[5]) {
  if (!out) return FARQ_ERR_NULL_POINTER;
  if (M < 0 || D <= 0 || D % 8 != 0 || group_size <= 0 || D % group_size != 0)
    return FARQ_ERR_BAD_SHAPE;
  if (D > kMaxHidden) return FARQ_ERR_UNSUPPORTED;
  if (x_dtype != FARQ_DTYPE_BF16 && x_dtype != FARQ_DTYPE_FP16) return FARQ_ERR_BAD_DTYPE;
  int dev, sms, optin;
  if (device_info(&dev, &sms, &optin) != cudaSuccess) return FARQ_ERR_CUDA;
  Plan pl;
  int st = make_plan(M > 0 ? M : 1, D, x_dtype, sms, optin, tune_ctas_per_sm, tune_stages, &pl);
  if (st != FARQ_OK) return st;
  out[0] = pl.threads;
  out[1] = pl.K;
  out[2] = pl.grid;
  out[3] = pl.stages;
  out[4] = (int64_t)pl.smem;
  return FARQ_OK;
}

int farq_launch(const farq_args_t* a, void* stream) {
  if (!a) return FARQ_ERR_NULL_POINTER;
  if (a->struct_size != sizeof(farq_args_t)) return FARQ_ERR_BAD_ARGS_SIZE;
  const int64_t M = a->M, D = a->D;
  const int G = a->group_size;
  if (M < 0 || D <= 0 || D % 8 != 0) return FARQ_ERR_BAD_SHAPE;
  if (G < 8 || G > 256 || (G & (G - 1)) != 0) return FARQ_ERR_BAD_GROUP;
  if (D % G != 0) return FARQ_ERR_BAD_SHAPE;
  if (D > kMaxHidden) return FARQ_ERR_UNSUPPORTED;
  if (a->x_dtype != FARQ_DTYPE_BF16 && a->x_dtype != FARQ_DTYPE_FP16) return FARQ_ERR_BAD_DTYPE;
  if (!is_float_out(a->gamma_dtype) || !is_float_out(a->residual_out_dtype))
    return FARQ_ERR_BAD_DTYPE;
  if (a->norm_out && !is_float_out(a->norm_out_dtype)) return FARQ_ERR_BAD_DTYPE;
  if (a->q_dtype != FARQ_DTYPE_INT8 && a->q_dtype != FARQ_DTYPE_E4M3) return FARQ_ERR_BAD_DTYPE;
  if (M == 0) return FARQ_OK;
  if (!a->x || !a->residual || !a->gamma || !a->residual_out || !a->x_q || !a->x_scale)
    return FARQ_ERR_NULL_POINTER;

  const int xs = dtype_size(a->x_dtype);
  const int ros = dtype_size(a->residual_out_dtype);
  const int nos = a->norm_out ? dtype_size(a->norm_out_dtype) : 0;
  const int64_t sx = a->x_row_stride ? a->x_row_stride : D;
  const int64_t sr = a->residual_row_stride ? a->residual_row_stride : D;
  const int64_t sro = a->residual_out_row_stride ? a->residual_out_row_stride : D;
  const int64_t sno = a->norm_out_row_stride ? a->norm_out_row_stride : D;
  const int64_t sq = a->x_q_row_stride ? a->x_q_row_stride : D;
  const int64_t ss = a->x_scale_row_stride ? a->x_scale_row_stride : D / G;
  if (sx < D || sr < D || sro < D || sq < D || ss < D / G || (a->norm_out && sno < D))
    return FARQ_ERR_BAD_SHAPE;
  // 16-byte rows for the bulk copies and vector stores; 8-byte q rows.
  if (!aligned(a->x, 16) || !aligned(a->residual, 16) || !aligned(a->residual_out, 16) ||
      !aligned(a->gamma, 16) || (a->norm_out && !aligned(a->norm_out, 16)) ||
      !aligned(a->x_q, 8) || !aligned(a->x_scale, 4))
    return FARQ_ERR_ALIGNMENT;
  if ((sx * xs) % 16 || (sr * xs) % 16 || (sro * ros) % 16 || (a->norm_out && (sno * nos) % 16) ||
      sq % 8)
    return FARQ_ERR_ALIGNMENT;

  int dev, sms, optin;
  if (device_info(&dev, &sms, &optin) != cudaSuccess) return FARQ_ERR_CUDA;
  Plan pl;
  int st = make_plan(M, D, a->x_dtype, sms, optin, a->tune_ctas_per_sm, a->tune_stages, &pl);
  if (st != FARQ_OK) return st;

  const bool e4m3 = a->q_dtype == FARQ_DTYPE_E4M3;
  KernelFn fn = pick_kernel(a->x_dtype, e4m3, pl.K);
  const int slot = kernel_slot(a->x_dtype, e4m3, pl.K);
  if ((int)pl.smem > g_smem_set[dev][slot].load(std::memory_order_relaxed)) {
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem) !=
        cudaSuccess)
      return FARQ_ERR_CUDA;
    g_smem_set[dev][slot].store((int)pl.smem, std::memory_order_relaxed);
  }

  Params p;
  p.x = static_cast<const uint8_t*>(a->x);
  p.res = static_cast<const uint8_t*>(a->residual);
  p.gamma = a->gamma;
  p.rout = static_cast<uint8_t*>(a->residual_out);
  p.nout = static_cast<uint8_t*>(a->norm_out);
  p.q = static_cast<uint8_t*>(a->x_q);
  p.scale = a->x_scale;
  p.status = a->status;
  p.M = M;
  p.sx = sx * xs;
  p.sr = sr * xs;
  p.sro = sro * ros;
  p.sno = a->norm_out ? sno * nos : 0;
  p.sq = sq;
  p.ss = ss;
  p.D = (int32_t)D;
  p.nvec = (int32_t)(D / 8);
  p.G = G;
  p.glanes = G / 8;
  p.gamma_dtype = a->gamma_dtype;
  p.rout_dtype = a->residual_out_dtype;
  p.nout_dtype = a->norm_out_dtype;
  p.ue8m0 = (a->flags & FARQ_FLAG_UE8M0) ? 1 : 0;
  p.stages = pl.stages;
  p.row_bytes = (uint32_t)(D * xs);
  p.eps = a->eps;

  void* kargs[] = {&p};
  if (cudaLaunchKernel(reinterpret_cast<const void*>(fn), dim3(pl.grid), dim3(pl.threads), kargs,
                       pl.smem, static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return FARQ_ERR_CUDA;
  return FARQ_OK;
}

}  // extern "C"
