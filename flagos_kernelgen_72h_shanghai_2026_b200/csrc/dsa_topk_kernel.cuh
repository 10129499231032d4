// dsa_topk_kernel.cuh — device code of the B200 (sm_100a) DSA top-k
// page-table transform (C ABI: include/dsa_topk.h).
//
// Reference behaviour (sinpeyw/flagos-kernelgen-72h-shanghai-2026,
// src/task02_dsa_topk_page_table_transform.py):
//   causal prefix ........... :161-166  last = min(pos // bs, min(cdiv(kv, bs), NB) - 1)
//   selectable .............. :166-167  candidate and score != -inf
//   order ................... :489-505  ordered fp32 key (-0 -> +0), then block id ascending
//   outputs ................. :170-175  ids (-1 when missing), pages = page_table[b*NB + id]
//
// Execution model: a persistent grid of CTAs of T threads (128 for NB <=
// 4096); a CTA takes rows blockIdx.x, blockIdx.x + grid, ... one at a time.
// Thread t owns the four-score vectors v = j*T + t (j < J) of a row, i.e.
// block ids 4v..4v+3. The next row's vectors are copied global -> shared by
// cp.async while the current row is processed (each thread copies and later
// reads only its own vectors, so no CTA barrier guards the staging buffer).
//
// Per row, exactly:
//  1. keys: every score becomes an order-preserving 32-bit key, 0 for a block
//     that is not selectable. Per-thread max and count of selectable keys.
//  2. lower bound: threads are grouped so that there are at least K groups;
//     every group max is a distinct key, so at least K keys are >= the
//     smallest group max (t0). One block reduction gives the selectable
//     count, the row max `hi` and t0.
//  3. compaction: the keys >= t0 (about 470 of 4096 at K = 128 for Gaussian
//     scores) are appended to a shared candidate list as 64-bit codes
//     (key << 32 | ~id), one shared atomic per warp. Codes are unique, so
//     their order is the exact output order. If more than `cap` keys pass
//     (heavy ties, K > T), a radix refinement over the register keys raises
//     the bound first (512-bin digits of key - lo, narrowing by 9 bits per
//     level); when it reaches a single key value that still has too many
//     copies, the copies are taken in block-id order by block scans.
//  4. exact top-K of the candidates: a 512-bin histogram of (key - lo) over
//     the adaptive range [lo, hi] locates the bin of the K-th code; the
//     candidates in it and above are scattered into bin segments (descending
//     bins), and each is ranked inside its own segment (typically 1-3 codes)
//     by comparing codes. Output slot = segment start + rank.
//  5. outputs: ids, and pages gathered from page_table, -1 beyond the
//     selectable count; coalesced stores.
//
// No scratch memory in global memory; no device-side waits.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "dsa_topk.h"

namespace dsa {

constexpr int kMaxThreads = 512;
constexpr int kBins = 512;      // histogram digits of 9 bits
constexpr int kBinBits = 9;
constexpr int kMaxTopK = 2048;
constexpr int kMinCap = 1024;   // candidate list capacity (at least K)
constexpr int64_t kMaxBlocks = 16384;

struct Params {
  const void* scores;
  const void* page_table;
  const void* q_pos;
  const void* kv_lens;
  void* out_blocks;
  void* out_pages;
  int64_t rows;        // B*H*Q
  int64_t HQ;          // H*Q
  int64_t Q;
  int32_t NB;
  int32_t K;
  int32_t block_size;
  int32_t index_bytes;   // q_pos / kv_lens element size (4 or 8)
  int32_t page_bytes;    // page_table / out_pages element size (4 or 8)
  int32_t blocks_bytes;  // out_blocks element size (4 or 8)
  int32_t cap;           // candidate list capacity (>= K)
  int32_t group;         // threads per lower-bound group (power of two <= 32), 0 = no bound
};

// Shared-memory carve-up (dynamic part), identical on host and device.
struct Smem {
  size_t stage, cand, ord, hist, F, outid, total;
};
__host__ __device__ inline size_t align16(size_t v) { return (v + 15) / 16 * 16; }
__host__ __device__ inline Smem smem_layout(int T, int J, int vec_bytes, int K, int cap) {
  Smem L;
  L.stage = 0;
  L.cand = align16((size_t)T * J * vec_bytes);
  L.ord = L.cand + (size_t)cap * sizeof(uint64_t);
  L.hist = L.ord + (size_t)cap * sizeof(uint64_t);
  L.F = L.hist + align16((kBins + 1) * sizeof(uint32_t));
  L.outid = L.F + align16((kBins + 1) * sizeof(uint32_t));
  L.total = L.outid + align16((size_t)K * sizeof(int32_t));
  return L;
}
__host__ __device__ inline int candidate_cap(int K) { return K > kMinCap ? K : kMinCap; }

// ------------------------------------------------------------------ loads
template <typename T>
struct Vec4;  // raw storage of 4 scores
template <>
struct Vec4<float> {
  using raw = uint4;
  static constexpr int kBytes = 16;
  __device__ __forceinline__ static void to_f32(const raw& v, float f[4]) {
    f[0] = __uint_as_float(v.x);
    f[1] = __uint_as_float(v.y);
    f[2] = __uint_as_float(v.z);
    f[3] = __uint_as_float(v.w);
  }
};
template <>
struct Vec4<__nv_bfloat16> {
  using raw = uint2;
  static constexpr int kBytes = 8;
  __device__ __forceinline__ static void to_f32(const raw& v, float f[4]) {
    f[0] = __uint_as_float(v.x << 16);
    f[1] = __uint_as_float(v.x & 0xffff0000u);
    f[2] = __uint_as_float(v.y << 16);
    f[3] = __uint_as_float(v.y & 0xffff0000u);
  }
};
template <>
struct Vec4<__half> {
  using raw = uint2;
  static constexpr int kBytes = 8;
  __device__ __forceinline__ static void to_f32(const raw& v, float f[4]) {
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
    f[0] = a.x;
    f[1] = a.y;
    f[2] = b.x;
    f[3] = b.y;
  }
};

// Asynchronous global -> shared copy of one vector (16 bytes: L2 only; 8
// bytes: the .ca form, the only one for that size).
template <int BYTES>
__device__ __forceinline__ void cp_async(void* smem_dst, const void* gsrc) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(smem_dst);
  if (BYTES == 16)
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(gsrc) : "memory");
  else
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(d), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Order-preserving key of an fp32 score (T2:489-494): -0.0 is folded to
// +0.0, negative values are bit-inverted, the others get the sign bit. The
// key of an unselectable element is 0 (and the all-ones NaN pattern, whose
// key is 0, ranks below every other element, exactly where an unselectable
// one would end up).
__device__ __forceinline__ uint32_t score_key(float f) {
  uint32_t b = __float_as_uint(f);
  b = (f == 0.0f) ? 0u : b;                                       // -0.0 -> +0.0
  const uint32_t k = b ^ ((uint32_t)((int32_t)b >> 31) | 0x80000000u);
  return b == 0xff800000u ? 0u : k;                               // -inf is not selectable
}

__device__ __forceinline__ int64_t load_index(const void* p, int64_t i, int bytes) {
  // The reference casts q_pos and kv_lens to int32 after loading (T2:161-162).
  return bytes == 8 ? (int64_t)(int32_t)__ldg(reinterpret_cast<const long long*>(p) + i)
                    : (int64_t)__ldg(reinterpret_cast<const int*>(p) + i);
}

// Candidates of a row: block ids 0..n-1 (T2:161-166).
__device__ __forceinline__ int row_candidates(const Params& p, int64_t row) {
  const int64_t b = row / p.HQ;
  const int64_t q = row - (row / p.Q) * p.Q;
  const int64_t pos = load_index(p.q_pos, b * p.Q + q, p.index_bytes);
  const int64_t kv = load_index(p.kv_lens, b, p.index_bytes);
  if (pos < 0 || kv <= 0) return 0;
  int64_t valid = (kv + p.block_size - 1) / p.block_size;
  if (valid > p.NB) valid = p.NB;
  int64_t last = pos / p.block_size;
  if (last > valid - 1) last = valid - 1;
  return (int)(last + 1);
}

__device__ __forceinline__ uint32_t bitlen(uint32_t v) { return v ? 32u - __clz(v) : 0u; }
// Digit width for the range [lo, hi]: the smallest s with (hi - lo) >> s < 512.
__device__ __forceinline__ uint32_t digit_shift(uint32_t lo, uint32_t hi) {
  const uint32_t l = bitlen(hi - lo);
  return l > (uint32_t)kBinBits ? l - kBinBits : 0u;
}

// Inclusive prefix sum of `v` over the CTA in thread order; `tot` gets the
// CTA total. Uses buf[0..31] between two barriers.
__device__ __forceinline__ uint32_t block_incl_scan(uint32_t v, uint32_t* buf, uint32_t* tot) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t u = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += u;
  }
  if (lane == 31) buf[warp] = v;
  __syncthreads();
  uint32_t before = 0, all = 0;
  for (int w = 0; w < nw; ++w) {
    const uint32_t x = buf[w];
    before += w < warp ? x : 0u;
    all += x;
  }
  *tot = all;
  __syncthreads();
  return v + before;
}

// Suffix counts of a 512-bin histogram plus an overflow count `ov` (keys
// above every bin): F[b] = ov + sum of hist[b..511], F[512] = ov. Returns the
// bin b with F[b+1] < need <= F[b] (1 <= need <= F[0]). Thread t owns
// 512 / T consecutive bins, thread 0 the highest ones. Ends with a barrier.
__device__ __forceinline__ uint32_t suffix_find(const uint32_t* hist, uint32_t ov, uint32_t need,
                                                uint32_t* F, uint32_t* buf, uint32_t* s_bin) {
  const int T = blockDim.x;
  const int bpt = kBins / T;
  const int lo = kBins - (threadIdx.x + 1) * bpt;  // lowest bin of this thread
  uint32_t local = 0;
  for (int i = 0; i < bpt; ++i) local += hist[lo + i];
  uint32_t tot;
  const uint32_t incl = block_incl_scan(local, buf, &tot);
  uint32_t acc = ov + incl - local;  // keys in bins above this thread's range
  for (int b = lo + bpt - 1; b >= lo; --b) {
    const uint32_t c = hist[b];
    if (acc < need && need <= acc + c) *s_bin = (uint32_t)b;
    acc += c;
    F[b] = acc;
  }
  if (threadIdx.x == 0) F[kBins] = ov;
  __syncthreads();
  return *s_bin;
}

// --------------------------------------------------------------- kernel
// NT threads per CTA (128, 256 or 512), J vectors per thread. The register
// budget leaves room for 5 CTAs of 128 threads per SM (2 of 256).
template <typename Tin, int J, int NT>
__global__ void __launch_bounds__(NT, NT == 128 ? 5 : NT == 256 ? 2 : 1)
    dsa_topk_kernel(const Params p) {
  using V = Vec4<Tin>;
  using raw = typename V::raw;
  extern __shared__ __align__(16) uint8_t smem[];
  constexpr int T = NT;
  const int t = threadIdx.x;
  const int lane = t & 31, warp = t >> 5, nw = T >> 5;
  const int NB = p.NB;
  const int nvec = NB >> 2;
  const int K = p.K;
  const int cap = p.cap;
  const Smem L = smem_layout(T, J, V::kBytes, K, cap);
  raw* stage = reinterpret_cast<raw*>(smem + L.stage);
  uint64_t* cand = reinterpret_cast<uint64_t*>(smem + L.cand);
  uint64_t* ord = reinterpret_cast<uint64_t*>(smem + L.ord);
  uint32_t* hist = reinterpret_cast<uint32_t*>(smem + L.hist);
  uint32_t* F = reinterpret_cast<uint32_t*>(smem + L.F);
  int32_t* outid = reinterpret_cast<int32_t*>(smem + L.outid);
  __shared__ uint32_t s_red[2][3][32];
  __shared__ uint32_t s_buf[32];
  __shared__ uint32_t s_C;
  __shared__ uint32_t s_bin;
  const Tin* scores = static_cast<const Tin*>(p.scores);

  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  auto issue = [&](int64_t r, int n) {
    const Tin* base = scores + r * (int64_t)NB;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int v = j * T + t;
      if (v < nvec && 4 * v < n) cp_async<V::kBytes>(stage + v, base + 4 * (int64_t)v);
    }
    cp_async_commit();
  };

  int64_t row = blockIdx.x;
  const int64_t G = gridDim.x;
  int n_cur = 0, n_next = 0;
  if (row < p.rows) {
    n_cur = row_candidates(p, row);
    issue(row, n_cur);
    if (row + G < p.rows) n_next = row_candidates(p, row + G);
  }
  int rb = 0;  // reduction buffer parity

  for (; row < p.rows; row += G, rb ^= 1) {
    const int n = n_cur;
    // ---- 1. keys of this row (own staged vectors)
    cp_async_wait_all();
    uint32_t key[J][4];
    uint32_t mx = 0, nz = 0;
    const bool full = n == NB;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int v = j * T + t;
      float f[4] = {0.f, 0.f, 0.f, 0.f};
      const bool in = v < nvec && 4 * v < n;
      if (in) V::to_f32(stage[v], f);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t k = score_key(f[c]);
        if (!full) k = (in && 4 * v + c < n) ? k : 0u;
        else if (!(v < nvec)) k = 0u;
        key[j][c] = k;
        mx = max(mx, k);
        nz += k != 0u ? 1u : 0u;
      }
    }
    // the staged vectors are in registers (mx depends on every one of them,
    // and the empty asm orders that before the copies below): start the next
    // row's copies into the same buffer
    asm volatile("" ::"r"(mx), "r"(nz));
    if (row + G < p.rows) {
      issue(row + G, n_next);
      n_cur = n_next;
      if (row + 2 * G < p.rows) n_next = row_candidates(p, row + 2 * G);
    }

    // ---- 2. block reduction: selectable count, max key, lower bound
    uint32_t gm = mx;
    for (int o = 1; o < p.group; o <<= 1) gm = max(gm, __shfl_xor_sync(0xffffffffu, gm, o));
    uint32_t t0 = p.group > 0 ? gm : 0u;
    uint32_t wnz = nz, wmx = mx;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      wnz += __shfl_xor_sync(0xffffffffu, wnz, o);
      wmx = max(wmx, __shfl_xor_sync(0xffffffffu, wmx, o));
      t0 = min(t0, __shfl_xor_sync(0xffffffffu, t0, o));
    }
    if (lane == 0) {
      s_red[rb][0][warp] = wnz;
      s_red[rb][1][warp] = wmx;
      s_red[rb][2][warp] = t0;
    }
    if (t == 0) s_C = 0;
    for (int i = t; i < kBins + 1; i += T) hist[i] = 0;
    __syncthreads();
    uint32_t total = 0, hi = 0, lo = 0xffffffffu;
    for (int w = 0; w < nw; ++w) {
      total += s_red[rb][0][w];
      hi = max(hi, s_red[rb][1][w]);
      lo = min(lo, s_red[rb][2][w]);
    }
    const uint32_t need = total < (uint32_t)K ? total : (uint32_t)K;
    if (total <= (uint32_t)K) lo = 1u;   // every selectable key is an output
    lo = max(lo, 1u);

    if (need > 0) {
      // ---- 3. compaction of the keys >= lo (refined first if too many)
      uint32_t C = 0;
      bool tie_path = false;
      uint32_t kth = 0, above = 0;
      for (;;) {
        uint32_t cnt = 0;
#pragma unroll
        for (int j = 0; j < J; ++j)
#pragma unroll
          for (int c = 0; c < 4; ++c) cnt += key[j][c] >= lo ? 1u : 0u;
        uint32_t incl = cnt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const uint32_t u = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += u;
        }
        uint32_t base = 0;
        if (lane == 31) base = atomicAdd(&s_C, incl);
        base = __shfl_sync(0xffffffffu, base, 31);
        uint32_t o = base + incl - cnt;
        if (o + cnt <= (uint32_t)cap) {
#pragma unroll
          for (int j = 0; j < J; ++j)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const uint32_t k = key[j][c];
              if (k >= lo) {
                cand[o++] = ((uint64_t)k << 32) | (uint64_t)(0xffffffffu - (uint32_t)(4 * (j * T + t) + c));
              }
            }
        }
        __syncthreads();
        C = s_C;
        if (C <= (uint32_t)cap) break;

        // Too many: radix refinement of the bound over the register keys.
        // Level 0 spans [lo, hi]; each level splits the K-th key's bin of
        // the previous level into 512 (keys above it counted as overflow).
        uint32_t s = digit_shift(lo, hi);
        uint32_t lvl_lo = lo;
        bool first = true;
        for (;;) {
          if (!first)
            for (int i = t; i < kBins + 1; i += T) hist[i] = 0;
          if (!first) __syncthreads();
          first = false;
#pragma unroll
          for (int j = 0; j < J; ++j)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const uint32_t k = key[j][c];
              if (k >= lvl_lo) {
                const uint32_t d = (k - lvl_lo) >> s;
                atomicAdd(&hist[d < (uint32_t)kBins ? d : (uint32_t)kBins], 1u);
              }
            }
          __syncthreads();
          const uint32_t ov = hist[kBins];
          const uint32_t b = suffix_find(hist, ov, need, F, s_buf, &s_bin);
          const uint32_t cnt_ge = F[b];
          above = F[b + 1];
          lvl_lo += b << s;
          if (cnt_ge <= (uint32_t)cap) {
            lo = lvl_lo;
            break;
          }
          if (s == 0) {  // one key value, too many copies of it
            tie_path = true;
            kth = lvl_lo;
            break;
          }
          s = s > (uint32_t)kBinBits ? s - kBinBits : 0u;
          __syncthreads();  // F and s_bin are read above before the next level rewrites them
        }
        __syncthreads();
        if (t == 0) s_C = 0;
        for (int i = t; i < kBins + 1; i += T) hist[i] = 0;
        __syncthreads();
        if (tie_path) break;
      }

      if (tie_path) {
        // keys above the K-th key (fewer than need), then the first
        // need - above copies of it in block-id order (ids 4(jT + t) + c)
        const uint32_t r = need - above;
#pragma unroll
        for (int j = 0; j < J; ++j)
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint32_t k = key[j][c];
            if (k > kth) cand[atomicAdd(&s_C, 1u)] =
                ((uint64_t)k << 32) | (uint64_t)(0xffffffffu - (uint32_t)(4 * (j * T + t) + c));
          }
        uint32_t eq_base = 0;
#pragma unroll
        for (int j = 0; j < J; ++j) {
          uint32_t e = 0;
#pragma unroll
          for (int c = 0; c < 4; ++c) e += key[j][c] == kth ? 1u : 0u;
          uint32_t tot;
          const uint32_t incl = block_incl_scan(e, s_buf, &tot);
          uint32_t pos = eq_base + incl - e;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            if (key[j][c] == kth) {
              if (pos < r)
                cand[atomicAdd(&s_C, 1u)] =
                    ((uint64_t)kth << 32) | (uint64_t)(0xffffffffu - (uint32_t)(4 * (j * T + t) + c));
              ++pos;
            }
          }
          eq_base += tot;
        }
        __syncthreads();
        C = s_C;
        lo = kth;
      }

      // ---- 4. exact order of the top `need` candidates
      const uint32_t s = digit_shift(lo, hi);
      for (uint32_t i = t; i < C; i += T)
        atomicAdd(&hist[((uint32_t)(cand[i] >> 32) - lo) >> s], 1u);
      __syncthreads();
      const uint32_t bstar = suffix_find(hist, 0u, need, F, s_buf, &s_bin);
      for (uint32_t i = t; i < C; i += T) {
        const uint64_t code = cand[i];
        const uint32_t d = ((uint32_t)(code >> 32) - lo) >> s;
        if (d >= bstar) ord[F[d + 1] + atomicSub(&hist[d], 1u) - 1u] = code;
      }
      __syncthreads();
      const uint32_t E = F[bstar];
      for (uint32_t i = t; i < E; i += T) {
        const uint64_t code = ord[i];
        const uint32_t d = ((uint32_t)(code >> 32) - lo) >> s;
        const uint32_t s0 = F[d + 1], s1 = F[d];
        uint32_t rank = 0;
        for (uint32_t q = s0; q < s1; ++q) rank += ord[q] > code ? 1u : 0u;
        const uint32_t slot = s0 + rank;
        if (slot < need) outid[slot] = (int32_t)(0xffffffffu - (uint32_t)code);
      }
      __syncthreads();
    }

    // ---- 5. outputs: ids and their pages, -1 beyond the winners
    const int64_t b = row / p.HQ;
    for (int k = t; k < K; k += T) {
      const int32_t id = k < (int)need ? outid[k] : -1;
      const int64_t o = row * (int64_t)K + k;
      int64_t page = -1;
      if (id >= 0) {
        const int64_t pi = b * (int64_t)NB + id;
        page = p.page_bytes == 8 ? (int64_t)__ldg(reinterpret_cast<const long long*>(p.page_table) + pi)
                                 : (int64_t)__ldg(reinterpret_cast<const int*>(p.page_table) + pi);
      }
      if (p.blocks_bytes == 8)
        reinterpret_cast<long long*>(p.out_blocks)[o] = id;
      else
        reinterpret_cast<int*>(p.out_blocks)[o] = id;
      if (p.page_bytes == 8)
        reinterpret_cast<long long*>(p.out_pages)[o] = page;
      else
        reinterpret_cast<int*>(p.out_pages)[o] = (int)page;
    }
  }
  cp_async_wait_all();
}

using KernelFn = void (*)(const Params);
KernelFn topk_kernel(int scores_dtype, int J, int T);  // dsa_topk.cu

}  // namespace dsa
