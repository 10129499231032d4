// farq_kernel.cuh — device code of the B200 (sm_100a) fused residual-add +
// RMSNorm + per-token group quantisation kernel (C ABI: include/farq.h).
//
// Reference behaviour (sinpeyw/flagos-kernelgen-72h-shanghai-2026,
// src/task01_fused_add_rmsnorm_group_quant.py):
//   per-row math ............ :65-121 (full row), :1127-1348 (segmented),
//                             :1401-1546 (two rows per program)
//   quantisation ............ :1089-1104  scale = max(gmax*(inv/127), 1e-12),
//                                         q = trunc(clamp(norm*(1/scale), ±127))
//   reduction ............... :1274-1278  inv = rsqrt(sum(r*r)/D + eps)
//
// Execution model (one kernel for every shape the reference routes separately):
//   * A CTA holds `teams` independent row teams of T threads (T a multiple of
//     32) and a ring of S >= teams shared-memory slots. CTA-local row n
//     (global row blockIdx.x + n*grid) goes to slot n % S and team n % teams.
//     A row of x and one of residual enter a slot by two cp.async.bulk copies
//     (TMA engine, no multicast) that complete on the slot's mbarrier.
//   * Teams synchronise only among themselves, on named barrier 1 + team, so
//     one team's reduction never stalls another. When a team has read its
//     slot it refills it with CTA row n + S and publishes n + S in the slot's
//     sequence word (release store); the team that processes that row
//     acquires the word before it waits on the mbarrier phase, which rules
//     out waiting on a stale phase of a slot it did not drain itself. With
//     S > teams, S - teams rows stay in flight while every team computes.
//   * gamma is converted to fp32 once per CTA into shared memory.
//   * Thread t of a team owns the 16-byte vectors v = k*T + t, k < K, of a
//     row. Phase 1: r = x + residual (fp32), residual_out written once,
//     sum(r*r) in fp64, w = r*gamma kept in registers, per-group absmax by
//     xor-shuffles over the GL = G/8 lanes of a group. One team barrier
//     reduces sum(r*r) and frees the slot. Phase 2: norm = w*inv_rms,
//     scale, q (int8 truncation or e4m3 RNE with saturation).
//   * sum(r*r) is accumulated in fp64 (exact squares of fp32 values, error
//     ~1e-16 relative) and rounded to fp32 once, so inv_rms does not depend
//     on the summation order. With fp32 accumulation every ulp of inv_rms
//     flips a group-maximum element (which sits on ±QMAX mathematically)
//     between two codes, on ~1/(2G) of all elements.
//   * Launched with programmatic stream serialisation: the next call's CTAs
//     launch, set up and prefetch their first rows into L2 while this one
//     drains, and wait (griddepcontrol) before their first global-memory read.
//   * Every device-side wait is bounded; a wait that runs out sets the
//     caller's status word, and the CTA drains its copies and returns.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "farq.h"

namespace farq {

constexpr int kMaxK = 8;              // 16-byte vectors per thread per row
constexpr int kMaxCtaThreads = 512;   // threads per CTA (launch bound)
constexpr int kMaxTeamThreads = 512;  // threads per row team
constexpr int kMaxTeamWarps = kMaxTeamThreads / 32;
// Largest D: gamma (4D bytes) and one slot (4D bytes for 2-byte inputs) must
// fit the 227 KB of shared memory a CTA may use.
constexpr int64_t kMaxHidden = 16384;
constexpr int kMaxStages = 8;           // ring slots per CTA
constexpr int kMaxTeams = 15;         // named barriers 1..15
constexpr uint64_t kWaitLimitNs = 2000000000ull;   // default bound of device waits (2 s)
constexpr uint64_t kTestWaitLimitNs = 1000000ull;  // bound under the test-only forced timeout

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
  int64_t sx, sr, sro, sno, sq, ss;  // row strides in bytes (ss: in floats)
  int64_t sgs;                       // x_scale group stride in floats (1: row-major)
  int32_t D;
  int32_t nvec;      // D / 8
  int32_t team_threads;
  int32_t teams;
  int32_t stages;
  uint32_t row_bytes;  // D * sizeof(x element)
  int32_t gamma_dtype, rout_dtype, nout_dtype;
  int32_t ue8m0;
  int32_t force_timeout;  // test only: team 0 waits for a sequence value nobody writes
  float eps;
  uint64_t wait_limit_ns; // bound of every device-side wait
};

// Shared-memory carve-up, identical on host and device.
struct SmemLayout {
  size_t gamma, stages, bars, seq, red, total;
};
__host__ __device__ inline SmemLayout smem_layout(int D, uint32_t row_bytes, int teams,
                                                  int stages) {
  SmemLayout L;
  L.gamma = 0;
  L.stages = (size_t)D * sizeof(float);                       // multiple of 32
  L.bars = L.stages + (size_t)stages * 2 * row_bytes;         // multiple of 32
  L.seq = L.bars + (size_t)stages * sizeof(uint64_t);
  L.red = L.seq + (size_t)kMaxStages * sizeof(uint32_t);      // 8-byte aligned
  L.total = L.red + (size_t)teams * kMaxTeamWarps * sizeof(double);
  return L;
}

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
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait: true when the phase completed, false after limit_ns.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0 && globaltimer_ns() - t0 > limit_ns) return false;
  }
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
// Global -> shared bulk copy through the TMA engine into this CTA's own
// shared memory, completion counted in bytes on `bar`.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(pol)
      : "memory");
}
// Prefetch `bytes` (multiple of 16, 16-byte aligned) of global memory into L2.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
// Release store / acquire load of a shared-memory word (slot sequence numbers).
__device__ __forceinline__ void seq_release(uint32_t* p, uint32_t v) {
  asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(smem_u32(p)), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)) : "memory");
  return v;
}
// Bounded wait for a slot's sequence word to reach `want`.
__device__ __forceinline__ bool seq_wait_bounded(const uint32_t* p, uint32_t want, uint64_t limit_ns) {
  if (ld_acquire(p) == want) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (ld_acquire(p) == want) return true;
    __nanosleep(64);
    if ((i & 63u) == 0 && globaltimer_ns() - t0 > limit_ns) return false;
  }
}
// Named barrier over `count` threads.
__device__ __forceinline__ void team_sync(uint32_t id, uint32_t count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
// Named barrier that also ORs a predicate over the participating threads.
__device__ __forceinline__ bool team_sync_or(uint32_t id, uint32_t count, bool flag) {
  uint32_t any;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "bar.red.or.pred p, %2, %3, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(any)
      : "r"((uint32_t)flag), "r"(id), "r"(count)
      : "memory");
  return any != 0;
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
template <typename T>
struct Unpack;
template <>
struct Unpack<__nv_bfloat16> {
  // 8 bf16 -> 8 fp32: a bf16 is the top half of the fp32 with the same value.
  __device__ __forceinline__ static void run(const uint4 v, float f[8]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
};
template <>
struct Unpack<__half> {
  __device__ __forceinline__ static void run(const uint4 v, float f[8]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
};

__device__ __forceinline__ uint32_t pack2(float a, float b, int dtype) {
  if (dtype == FARQ_DTYPE_BF16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
// Store 8 fp32 values as `dtype` (BF16/FP16 round-to-nearest-even, or FP32)
// at element offset 8*v of the row that starts at `row`.
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
    const float4 a = __ldg(p), b = __ldg(p + 1);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
    f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  } else {
    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(g) + v);
    if (dtype == FARQ_DTYPE_BF16)
      Unpack<__nv_bfloat16>::run(raw, f);
    else
      Unpack<__half>::run(raw, f);
  }
}
// Two fp32 -> two e4m3 bytes (low byte = lo), round-to-nearest-even,
// saturating to ±448.
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
  const uint32_t b = __float_as_uint(s);
  const uint32_t up = (b + 0x007fffffu) & 0xff800000u;  // carries into the exponent iff mantissa != 0
  return __uint_as_float(up);
}

// -------------------------------------------------------------------- kernel
template <typename Tin, int K, int GL, bool E4M3>
__global__ void __launch_bounds__(kMaxCtaThreads, 1) farq_rows_kernel(const Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const SmemLayout L = smem_layout(p.D, p.row_bytes, p.teams, p.stages);
  const int T = p.team_threads;
  const int TEAMS = p.teams;
  const int team = threadIdx.x / T;
  const int tt = threadIdx.x - team * T;
  const int lane = threadIdx.x & 31;
  const int twarp = tt >> 5;
  const int S = p.stages;  // ring slots of the CTA, S >= TEAMS
  const uint32_t stage_bytes = 2u * p.row_bytes;
  const uint32_t bar_id = 1u + (uint32_t)team;

  const float4* sg = reinterpret_cast<const float4*>(smem + L.gamma);
  uint8_t* ring = smem + L.stages;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint32_t* seq = reinterpret_cast<uint32_t*>(smem + L.seq);
  double* my_red = reinterpret_cast<double*>(smem + L.red) + team * kMaxTeamWarps;

  // CTA-local row n is global row blockIdx.x + n*gridDim.x; it sits in ring
  // slot n % S and is processed by team n % TEAMS.
  const int64_t G = gridDim.x;
  const int64_t nrows = blockIdx.x < p.M ? (p.M - 1 - blockIdx.x) / G + 1 : 0;
  const uint64_t pol = policy_evict_first();
  // Programmatic dependent launch: this grid may have been started while the
  // previous kernel in the stream was still draining. Wait for it to finish
  // (and its writes to be visible) before touching global memory, and let the
  // next launch begin its own set-up as early as possible.
  // While the previous kernel drains, warm L2 with this CTA's first rows and
  // gamma. A bulk L2 prefetch only moves lines into the device's L2, the point
  // of coherence for every writer, so data the previous kernel still writes
  // lands there too and the reads after the wait below see it.
  if (threadIdx.x == 0) {
    for (int s = 0; s < S && s < nrows; ++s) {
      const int64_t row = blockIdx.x + (int64_t)s * G;
      bulk_prefetch_l2(p.x + row * p.sx, p.row_bytes);
      bulk_prefetch_l2(p.res + row * p.sr, p.row_bytes);
    }
    bulk_prefetch_l2(p.gamma, (uint32_t)p.nvec * (p.gamma_dtype == FARQ_DTYPE_FP32 ? 32u : 16u));
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  // gamma -> fp32 shared memory, once per CTA, in two planes (elements 0-3,
  // then 4-7 of every vector) so that a warp's 16-byte reads of one plane are
  // contiguous (no bank conflicts). The first round of gamma loads is issued
  // before the row copies: queued behind the copies of all CTAs it would
  // arrive microseconds after the rows and hold back the first row.
  float4* gs = reinterpret_cast<float4*>(smem + L.gamma);
  float g_first[8];
  const bool has_first = threadIdx.x < p.nvec;
  if (has_first) load_gamma8(p.gamma, threadIdx.x, p.gamma_dtype, g_first);
  __syncthreads();  // every thread's first gamma load is issued (not yet complete)

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) mbar_init(smem_u32(&bars[s]), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    for (int s = 0; s < S; ++s) {
      seq[s] = (uint32_t)s;
      if (s < nrows) {
        const int64_t row = blockIdx.x + (int64_t)s * G;
        const uint32_t bar = smem_u32(&bars[s]);
        const uint32_t dst = smem_u32(ring + (size_t)s * stage_bytes);
        mbar_arrive_expect_tx(bar, stage_bytes);
        bulk_load(dst, p.x + row * p.sx, p.row_bytes, bar, pol);
        bulk_load(dst + p.row_bytes, p.res + row * p.sr, p.row_bytes, bar, pol);
      }
    }
  }
  if (has_first) {
    gs[threadIdx.x] = make_float4(g_first[0], g_first[1], g_first[2], g_first[3]);
    gs[p.nvec + threadIdx.x] = make_float4(g_first[4], g_first[5], g_first[6], g_first[7]);
  }
  for (int v = threadIdx.x + blockDim.x; v < p.nvec; v += blockDim.x) {
    float g[8];
    load_gamma8(p.gamma, v, p.gamma_dtype, g);
    gs[v] = make_float4(g[0], g[1], g[2], g[3]);
    gs[p.nvec + v] = make_float4(g[4], g[5], g[6], g[7]);
  }
  __syncthreads();

  const float qmax = E4M3 ? 448.0f : 127.0f;
  const int nvec = p.nvec;
  const int tw = T >> 5;
  bool failed = false;

  // This team's rows n = team, team + TEAMS, ...: slot s = n % S and the
  // slot's fill count j = n / S are advanced incrementally.
  int64_t n = team;
  int s = team % S;
  uint32_t j = (uint32_t)(team / S);
  const int64_t step_rows = (int64_t)TEAMS * G;
  uint8_t* rout_row = p.rout + (blockIdx.x + n * G) * p.sro;
  uint8_t* nout_row = p.nout ? p.nout + (blockIdx.x + n * G) * p.sno : nullptr;
  uint8_t* q_row = p.q + (blockIdx.x + n * G) * p.sq;
  float* sc_row = p.scale + (blockIdx.x + n * G) * p.ss;
  const int64_t d_ro = step_rows * p.sro, d_no = step_rows * p.sno;
  const int64_t d_q = step_rows * p.sq, d_s = step_rows * p.ss;

  for (; n < nrows; n += TEAMS) {
    // Wait until the slot holds row n: first its sequence word (written
    // with release semantics by the team that armed the slot, so the
    // mbarrier phase below cannot be a stale one), then the copy itself.
    const uint32_t want = (p.force_timeout && team == 0) ? 0xffffffffu : (uint32_t)n;
    bool ok = seq_wait_bounded(&seq[s], want, p.wait_limit_ns);
    ok = ok && mbar_wait_bounded(smem_u32(&bars[s]), j & 1u, p.wait_limit_ns);
    if (team_sync_or(bar_id, T, !ok)) {
      if (tt == 0 && p.status) atomicExch(p.status, (int)FARQ_ERR_DEVICE_TIMEOUT);
      failed = true;
      break;
    }
    const uint8_t* sx = ring + (size_t)s * stage_bytes;
    const uint8_t* sr = sx + p.row_bytes;

    // ---- phase 1
    float w[K][8];
    float gmax[K];
    double ss0 = 0.0, ss1 = 0.0;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int v = k * T + tt;
      float m = 0.f;
      if (v < nvec) {
        float a[8], b[8];
        Unpack<Tin>::run(reinterpret_cast<const uint4*>(sx)[v], a);
        Unpack<Tin>::run(reinterpret_cast<const uint4*>(sr)[v], b);
        const float4 g0 = sg[v], g1 = sg[nvec + v];
        const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          a[e] = a[e] + b[e];
          if (e & 1)
            ss1 = fma((double)a[e], (double)a[e], ss1);
          else
            ss0 = fma((double)a[e], (double)a[e], ss0);
          w[k][e] = a[e] * g[e];
          m = fmaxf(m, fabsf(w[k][e]));
        }
        store8(rout_row, v, a, p.rout_dtype);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) w[k][e] = 0.f;
      }
#pragma unroll
      for (int o = 1; o < GL; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      gmax[k] = m;
    }
    double ss = ss0 + ss1;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) my_red[twarp] = ss;
    team_sync(bar_id, T);

    // The slot is no longer read: refill it with CTA row n + S.
    if (tt == 0 && n + S < nrows) {
      const int64_t row = blockIdx.x + (n + S) * G;
      const uint32_t bar = smem_u32(&bars[s]);
      const uint32_t dst = smem_u32(ring + (size_t)s * stage_bytes);
      mbar_arrive_expect_tx(bar, stage_bytes);
      bulk_load(dst, p.x + row * p.sx, p.row_bytes, bar, pol);
      bulk_load(dst + p.row_bytes, p.res + row * p.sr, p.row_bytes, bar, pol);
      seq_release(&seq[s], (uint32_t)(n + S));
    }

    double total = 0.0;
    for (int q = 0; q < tw; ++q) total += my_red[q];
    const float inv_rms =
        __frcp_rn(__fsqrt_rn(__fadd_rn(__fdiv_rn(__double2float_rn(total), (float)p.D), p.eps)));
    const float step = __fdiv_rn(inv_rms, qmax);

    // ---- phase 2
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int v = k * T + tt;
      if (v < nvec) {
        float sc = fmaxf(gmax[k] * step, 1.0e-12f);
        sc = p.ue8m0 ? pow2_ceil(sc) : sc;
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
        if ((lane & (GL - 1)) == 0) st_cs_f32(sc_row + (v / GL) * p.sgs, sc);
      }
    }
    rout_row += d_ro;
    if (nout_row) nout_row += d_no;
    q_row += d_q;
    sc_row += d_s;
    s += TEAMS;
    if (s >= S) {
      s -= S;
      ++j;
    }
  }

  // No bulk copy may still target this CTA's shared memory when it exits:
  // after a failed wait, drain every slot's last armed fill (bounded).
  if (__syncthreads_or(failed) && threadIdx.x == 0) {
    for (int t = 0; t < S; ++t) {
      const uint32_t last = ld_acquire(&seq[t]);
      if ((int64_t)last < nrows)
        (void)mbar_wait_bounded(smem_u32(&bars[t]), (last / (uint32_t)S) & 1u, p.wait_limit_ns);
    }
  }
}

using KernelFn = void (*)(const Params);

// Kernel table of one (input dtype, quantised dtype) pair, indexed by
// K (1..kMaxK) and log2(GL) (0..5). Defined in farq_inst_*.cu.
KernelFn kernel_bf16_int8(int K, int gl_log2);
KernelFn kernel_bf16_e4m3(int K, int gl_log2);
KernelFn kernel_fp16_int8(int K, int gl_log2);
KernelFn kernel_fp16_e4m3(int K, int gl_log2);

}  // namespace farq

// Instantiates the kernel table of one (Tin, E4M3) pair.
#define FARQ_KERNEL_TABLE(NAME, TIN, E4M3)                                              \
  namespace farq {                                                                      \
  template <int K>                                                                      \
  static KernelFn NAME##_k(int gl_log2) {                                               \
    switch (gl_log2) {                                                                  \
      case 0: return farq_rows_kernel<TIN, K, 1, E4M3>;                                 \
      case 1: return farq_rows_kernel<TIN, K, 2, E4M3>;                                 \
      case 2: return farq_rows_kernel<TIN, K, 4, E4M3>;                                 \
      case 3: return farq_rows_kernel<TIN, K, 8, E4M3>;                                 \
      case 4: return farq_rows_kernel<TIN, K, 16, E4M3>;                                \
      default: return farq_rows_kernel<TIN, K, 32, E4M3>;                               \
    }                                                                                   \
  }                                                                                     \
  KernelFn NAME(int K, int gl_log2) {                                                   \
    switch (K) {                                                                        \
      case 1: return NAME##_k<1>(gl_log2);                                              \
      case 2: return NAME##_k<2>(gl_log2);                                              \
      case 3: return NAME##_k<3>(gl_log2);                                              \
      case 4: return NAME##_k<4>(gl_log2);                                              \
      case 5: return NAME##_k<5>(gl_log2);                                              \
      case 6: return NAME##_k<6>(gl_log2);                                              \
      case 7: return NAME##_k<7>(gl_log2);                                              \
      default: return NAME##_k<8>(gl_log2);                                             \
    }                                                                                   \
  }                                                                                     \
  }
