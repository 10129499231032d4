// farq_ar_kernel.cuh — tensor-parallel variant: all-reduce of W partial
// activations fused with residual add + RMSNorm + per-token group
// quantisation, over NVLink peer memory (C ABI: farq_ar_launch, include/farq.h).
//
// Where it sits: in tensor-parallel inference the layer before the norm is a
// row-parallel GEMM, so every rank holds a partial sum P_k [M, D] of x. The
// reference operator (src/task01_fused_add_rmsnorm_group_quant.py:1731) runs
// after an all-reduce has produced x on every rank; this kernel does both:
//
//   x        = round_to_input_dtype( sum_k fp32(P_k) )   (ranks k = 0..W-1 in order)
//   then the reference per-row math on x and residual, with every output row
//   written to all W ranks (the outputs are replicated, as after an all-reduce).
//
// Execution (the single-GPU kernel's structure, farq_kernel.cuh, with wider slots):
//   * Rank r owns the contiguous row slab [row_begin, row_end). A CTA holds
//     `teams` row teams (named barriers) and a ring of S >= teams slots; CTA-
//     local slab row n goes to slot n % S and team n % teams, with the slot's
//     sequence word (release/acquire) guarding against stale mbarrier phases.
//   * A slot holds a row's W partial rows — read from every rank's memory by
//     cp.async.bulk (unicast TMA copies, never multicast) — and its local
//     residual row, completing on the slot's mbarrier. Phase 1 sums the
//     partials in rank order. At W <= 2 four teams fit (as on one GPU); at
//     W = 8 a slot is 9 rows and one team fits.
//   * Outputs are written with plain stores to each rank's buffer (peer
//     pointers over NVLink, including this rank's own).
//   * Two cross-rank barriers per CTA, on epoch flags in every rank's signal
//     buffer: at the start (every rank's partial is complete and every rank has
//     finished with the previous contents of its output buffers) and at the end
//     (every peer's writes into this rank's outputs are visible before this
//     kernel completes). CTA b of rank r meets CTA b of every other rank; the
//     launch shape is identical on all ranks. Every wait is bounded in time; a
//     wait that runs out sets the status word and the CTA returns.
#pragma once

#include <type_traits>

#include "farq_kernel.cuh"

namespace farq {

constexpr int kMaxWorld = 8;
constexpr int kMaxArCtas = 1024;  // signal-buffer slots per phase

struct ArParams {
  const uint8_t* part[kMaxWorld];  // partial activations, one per rank
  uint8_t* rout[kMaxWorld];
  uint8_t* nout[kMaxWorld];        // all null when norm_out is not written
  uint8_t* q[kMaxWorld];
  float* scale[kMaxWorld];
  uint32_t* signal[kMaxWorld];     // each rank's signal buffer
  const uint8_t* res;              // local residual
  const void* gamma;
  int32_t* status;
  int64_t row_begin, row_end;      // this rank's slab
  int32_t D, nvec, team_threads, teams, stages, world, rank;  // stages: ring slots of the CTA
  uint32_t row_bytes;              // D * sizeof(x element)
  int32_t gamma_dtype, nout_dtype, ue8m0;
  uint32_t epoch;
  int32_t force_timeout;
  float eps;
  uint64_t wait_limit_ns;
};

// Shared memory: gamma (fp32, two planes) | S slots of (W + 1) rows |
// S mbarriers | S sequence words | per team reduction words.
struct ArLayout {
  size_t gamma, slots, bars, seq, red, total;
};
__host__ __device__ inline ArLayout ar_layout(int D, uint32_t row_bytes, int world, int teams,
                                              int stages) {
  ArLayout L;
  L.gamma = 0;
  L.slots = (size_t)D * sizeof(float);
  L.bars = L.slots + (size_t)stages * (world + 1) * row_bytes;
  L.seq = L.bars + (size_t)stages * sizeof(uint64_t);
  L.red = L.seq + (size_t)kMaxStages * sizeof(uint32_t);
  L.total = L.red + (size_t)teams * kMaxTeamWarps * sizeof(double);
  return L;
}

__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_relaxed_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_acq_rel_sys() {
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}

// Cross-rank barrier of CTA blockIdx.x for `phase`, run by one thread: signal
// every rank, then wait (bounded) until every rank has signalled this CTA.
// The caller orders what must precede the signal (every thread's
// fence_acq_rel_sys and a CTA barrier, before the end barrier); the fence after the wait
// orders the peers' earlier writes before this CTA's later accesses.
// Returns false when the wait ran out.
__device__ __forceinline__ bool ar_barrier(const ArParams& p, int phase, uint32_t want) {
  const size_t base = ((size_t)phase * kMaxArCtas + blockIdx.x) * kMaxWorld;
  for (int k = 0; k < p.world; ++k) st_relaxed_sys(p.signal[k] + base + p.rank, p.epoch);
  const uint32_t* mine = p.signal[p.rank] + base;
  const uint64_t t0 = globaltimer_ns();
  for (int k = 0; k < p.world; ++k) {
    for (uint32_t i = 0;; ++i) {
      if ((int32_t)(ld_relaxed_sys(mine + k) - want) >= 0) break;
      __nanosleep(20);
      if ((i & 255u) == 255u && globaltimer_ns() - t0 > p.wait_limit_ns) return false;
    }
  }
  fence_acq_rel_sys();
  return true;
}

// WMAX (1, 2, 4 or 8) bounds the world size W at compile time: the loops
// over ranks unroll to WMAX with a guard for W < WMAX, so a world of one or
// two ranks carries no code for eight.
template <typename Tin, int K, int GL, bool E4M3, int WMAX>
__global__ void __launch_bounds__(kMaxCtaThreads, 1) farq_ar_kernel(const ArParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const ArLayout L = ar_layout(p.D, p.row_bytes, p.world, p.teams, p.stages);
  const int T = p.team_threads;
  const int TEAMS = p.teams;
  const int team = threadIdx.x / T;
  const int tt = threadIdx.x - team * T;
  const int lane = threadIdx.x & 31;
  const int twarp = tt >> 5;
  const int S = p.stages;  // ring slots of the CTA, S >= TEAMS
  const int W = p.world;
  const uint32_t rb = p.row_bytes;
  const uint32_t slot_bytes = (uint32_t)(W + 1) * rb;  // W partial rows, then the residual row
  const uint32_t bar_id = 1u + (uint32_t)team;
  const float4* sg = reinterpret_cast<const float4*>(smem + L.gamma);
  uint8_t* ring = smem + L.slots;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint32_t* seq = reinterpret_cast<uint32_t*>(smem + L.seq);
  double* my_red = reinterpret_cast<double*>(smem + L.red) + team * kMaxTeamWarps;
  __shared__ int s_fail;

  // CTA-local slab row n (global row row_begin + blockIdx.x + n*grid) sits in
  // ring slot n % S and is processed by team n % TEAMS.
  const int64_t G = gridDim.x;
  const int64_t slab = p.row_end - p.row_begin;
  const int64_t nrows = blockIdx.x < slab ? (slab - 1 - blockIdx.x) / G + 1 : 0;
  const uint64_t pol = policy_evict_first();
  asm volatile("griddepcontrol.wait;" ::: "memory");

  auto fill = [&](int slot, int64_t row) {
    const uint32_t bar = smem_u32(&bars[slot]);
    const uint32_t dst = smem_u32(ring + (size_t)slot * slot_bytes);
    mbar_arrive_expect_tx(bar, slot_bytes);
#pragma unroll
    for (int k = 0; k < WMAX; ++k)  // constant indices keep the peer pointers out of memory
      if (k < W) bulk_load(dst + (uint32_t)k * rb, p.part[k] + row * rb, rb, bar, pol);
    bulk_load(dst + (uint32_t)W * rb, p.res + row * rb, rb, bar, pol);
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) mbar_init(smem_u32(&bars[s]), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    // Start barrier: every rank's partial is complete and every rank has
    // finished with the previous contents of its output buffers.
    // (test-only flag: wait for an epoch no rank signals)
    s_fail = ar_barrier(p, 0, p.force_timeout ? p.epoch + 0x40000000u : p.epoch) ? 0 : 1;
    // The barrier's acquire is a generic-proxy operation; the peer rows are
    // read by bulk copies (async proxy), which it orders only after this
    // proxy fence.
    asm volatile("fence.proxy.async.global;" ::: "memory");
    for (int s = 0; s < S; ++s) {
      seq[s] = (uint32_t)s;
      if (!s_fail && s < nrows) fill(s, p.row_begin + blockIdx.x + (int64_t)s * G);
    }
  }
  for (int v = threadIdx.x; v < p.nvec; v += blockDim.x) {
    float g[8];
    load_gamma8(p.gamma, v, p.gamma_dtype, g);
    float4* d = reinterpret_cast<float4*>(smem + L.gamma);
    d[v] = make_float4(g[0], g[1], g[2], g[3]);
    d[p.nvec + v] = make_float4(g[4], g[5], g[6], g[7]);
  }
  __syncthreads();
  if (s_fail) {
    if (threadIdx.x == 0 && p.status) atomicExch(p.status, (int)FARQ_ERR_DEVICE_TIMEOUT);
    return;
  }
  // Each team's first thread issues the later refills: it too orders them
  // (async proxy) after the barrier it observed through __syncthreads.
  if (tt == 0) asm volatile("fence.proxy.async.global;" ::: "memory");

  const float qmax = E4M3 ? 448.0f : 127.0f;
  const int nvec = p.nvec;
  const int tw = T >> 5;
  const int xdt = std::is_same<Tin, __nv_bfloat16>::value ? FARQ_DTYPE_BF16 : FARQ_DTYPE_FP16;
  const int groups = p.D / (GL * 8);
  bool failed = false;
  int64_t n = team;
  int s = team % S;
  uint32_t jf = (uint32_t)(team / S);  // fill count of the slot

  for (; n < nrows; n += TEAMS) {
    const int64_t row = p.row_begin + blockIdx.x + n * G;
    bool ok = seq_wait_bounded(&seq[s], (uint32_t)n, p.wait_limit_ns);
    ok = ok && mbar_wait_bounded(smem_u32(&bars[s]), jf & 1u, p.wait_limit_ns);
    if (team_sync_or(bar_id, T, !ok)) {
      if (tt == 0 && p.status) atomicExch(p.status, (int)FARQ_ERR_DEVICE_TIMEOUT);
      failed = true;
      break;
    }
    const uint8_t* slot = ring + (size_t)s * slot_bytes;
    const uint8_t* sr = slot + (size_t)W * rb;

    // ---- phase 1: x = sum of the partials in rank order, rounded to the
    // input dtype (the all-reduced activation); r = x + residual
    float w[K][8];
    float gmax[K];
    double ss0 = 0.0, ss1 = 0.0;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int v = k * T + tt;
      float m = 0.f;
      if (v < nvec) {
        float a[8], b[8];
        Unpack<Tin>::run(reinterpret_cast<const uint4*>(slot)[v], a);
#pragma unroll
        for (int rk = 1; rk < WMAX; ++rk) {
          if (rk < W) {
            Unpack<Tin>::run(reinterpret_cast<const uint4*>(slot + (size_t)rk * rb)[v], b);
#pragma unroll
            for (int e = 0; e < 8; ++e) a[e] += b[e];
          }
        }
        const uint4 xr = make_uint4(pack2(a[0], a[1], xdt), pack2(a[2], a[3], xdt),
                                    pack2(a[4], a[5], xdt), pack2(a[6], a[7], xdt));
        Unpack<Tin>::run(xr, a);
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
#pragma unroll
        for (int rk = 0; rk < WMAX; ++rk)
          if (rk < W) store8(p.rout[rk] + row * rb, v, a, xdt);
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
      fill(s, row + (int64_t)S * G);
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
        if (p.nout[0]) {
#pragma unroll
          for (int rk = 0; rk < WMAX; ++rk)
            if (rk < W)
              store8(p.nout[rk] + row * (int64_t)p.D * (p.nout_dtype == FARQ_DTYPE_FP32 ? 4 : 2),
                     v, nrm, p.nout_dtype);
        }
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
#pragma unroll
        for (int rk = 0; rk < WMAX; ++rk) {
          if (rk < W) {
            st_cs_v2(p.q[rk] + row * (int64_t)p.D + 8 * (int64_t)v, lo, hi);
            if ((lane & (GL - 1)) == 0) st_cs_f32(p.scale[rk] + row * groups + v / GL, sc);
          }
        }
      }
    }
    s += TEAMS;
    if (s >= S) {
      s -= S;
      ++jf;
    }
  }

  // After a failed wait: drain every slot's last armed fill (bounded) and
  // skip the end barrier (a peer did not deliver).
  if (__syncthreads_or(failed)) {
    if (threadIdx.x == 0)
      for (int t = 0; t < S; ++t) {
        const uint32_t last = ld_acquire(&seq[t]);
        if ((int64_t)last < nrows)
          (void)mbar_wait_bounded(smem_u32(&bars[t]), (last / (uint32_t)S) & 1u, p.wait_limit_ns);
      }
    return;
  }
  // End barrier: every thread's stores to every rank are ordered before the
  // signal; the kernel completes only after every rank's CTA of the same
  // index has signalled, i.e. after all writes into this rank landed.
  fence_acq_rel_sys();
  __syncthreads();
  if (threadIdx.x == 0) {
    if (!ar_barrier(p, 1, p.epoch) && p.status) atomicExch(p.status, (int)FARQ_ERR_DEVICE_TIMEOUT);
  }
}

using ArKernelFn = void (*)(const ArParams);
// Kernel tables by (K, log2 GL), one per input/output type and WMAX; the
// farq_ar_inst_*.cu sources are compiled once per WMAX (-DFARQ_AR_WMAX=w).
#define FARQ_AR_DECLARE(NAME)            \
  ArKernelFn NAME##_w1(int K, int gl_log2); \
  ArKernelFn NAME##_w2(int K, int gl_log2); \
  ArKernelFn NAME##_w4(int K, int gl_log2); \
  ArKernelFn NAME##_w8(int K, int gl_log2);
FARQ_AR_DECLARE(ar_kernel_bf16_int8)
FARQ_AR_DECLARE(ar_kernel_bf16_e4m3)
FARQ_AR_DECLARE(ar_kernel_fp16_int8)
FARQ_AR_DECLARE(ar_kernel_fp16_e4m3)
#undef FARQ_AR_DECLARE

}  // namespace farq

#define FARQ_AR_CAT2(a, b) a##b
#define FARQ_AR_CAT(a, b) FARQ_AR_CAT2(a, b)
#define FARQ_AR_KERNEL_TABLE(NAME, TIN, E4M3)                                           \
  namespace farq {                                                                      \
  template <int K>                                                                      \
  static ArKernelFn NAME##_k(int gl_log2) {                                             \
    constexpr int W = FARQ_AR_WMAX;                                                     \
    switch (gl_log2) {                                                                  \
      case 0: return farq_ar_kernel<TIN, K, 1, E4M3, W>;                                \
      case 1: return farq_ar_kernel<TIN, K, 2, E4M3, W>;                                \
      case 2: return farq_ar_kernel<TIN, K, 4, E4M3, W>;                                \
      case 3: return farq_ar_kernel<TIN, K, 8, E4M3, W>;                                \
      case 4: return farq_ar_kernel<TIN, K, 16, E4M3, W>;                               \
      default: return farq_ar_kernel<TIN, K, 32, E4M3, W>;                              \
    }                                                                                   \
  }                                                                                     \
  ArKernelFn FARQ_AR_CAT(NAME##_w, FARQ_AR_WMAX)(int K, int gl_log2) {                  \
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
