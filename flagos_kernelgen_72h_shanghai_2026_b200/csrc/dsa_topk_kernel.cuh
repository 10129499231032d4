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
//  1. keys: every score becomes an order-preserving 32-bit key (a raw key
//     first: the sign handling only), 0 for a masked block; per-thread max.
//  2. lower bound: every thread keeps its four (or two) largest vector
//     maxima, so it holds that many distinct keys >= the last one; threads
//     are grouped (lists merged by shuffles) so that the groups vouch for at
//     least K keys, and the smallest group bound t0 has at least K keys >= it. One block reduction gives
//     the row max `hi` and t0. When t0 is above the raw key of -inf, every key >= t0 is
//     selectable and K of them exist; otherwise (short or -inf-heavy rows)
//     the keys are made exact and all selectable keys are candidates.
//  3. compaction: the keys >= t0 (about 300 of 4096 at K = 128 for Gaussian
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

#include <type_traits>

#include "dsa_topk.h"

namespace dsa {

constexpr int kMaxThreads = 512;
constexpr int kBins = 512;      // histogram digits of 9 bits
constexpr int kBinBits = 9;
constexpr int kMaxTopK = 2048;
constexpr int kMinCap = 768;    // candidate list capacity (at least K)
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
  int32_t group;         // threads per lower-bound group (power of two <= 32), 0 = no bound;
                         // T / group * vouch_of(J) >= K
  uint32_t hq_mul, hq_shift;  // row / (H*Q) = fast_div(row, ...)  (rows < 2^31)
  uint32_t q_mul, q_shift;    // row / Q
};

// Division of n < 2^31 by a constant d >= 1 with a precomputed multiplier
// (the round-up method of Granlund and Montgomery, "Division by invariant
// integers using multiplication", 1994): l = ceil(log2 d),
// m = floor(2^32 (2^l - d) / d) + 1, n / d = (umulhi(n, m) + n) >> l.
__host__ inline void fast_div_init(uint32_t d, uint32_t* mul, uint32_t* shift) {
  uint32_t l = 0;
  while (l < 32 && (1ull << l) < d) ++l;
  *mul = (uint32_t)(((1ull << 32) * ((1ull << l) - d)) / d + 1);
  *shift = l;
}
__device__ __forceinline__ uint32_t fast_div(uint32_t n, uint32_t mul, uint32_t shift) {
  return (__umulhi(n, mul) + n) >> shift;
}

// Shared-memory carve-up (dynamic part), identical on host and device: the
// staging buffer for a row's scores, the candidate list and its bin-ordered
// copy, histogram and suffix counts.
struct Smem {
  size_t stage, cand, ord, hist, F, total;
};
__host__ __device__ inline size_t align16(size_t v) { return (v + 15) / 16 * 16; }
__host__ __device__ inline Smem smem_layout(int T, int J, int vec_bytes, int K, int cap) {
  Smem L;
  L.stage = 0;
  L.cand = align16((size_t)T * J * vec_bytes);
  L.ord = L.cand + (size_t)cap * sizeof(uint64_t);
  L.hist = L.ord + (size_t)cap * sizeof(uint64_t);
  L.F = L.hist + align16((kBins + 1) * sizeof(uint32_t));
  L.total = L.F + align16((kBins + 1) * sizeof(uint32_t));
  return L;
}
// Keys a thread (and a group of threads) vouches for in the lower bound:
// its 4, 2 or 1 largest vector maxima, as its J vectors allow.
__host__ __device__ constexpr int vouch_of(int J) { return J >= 4 ? 4 : J >= 2 ? 2 : 1; }
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

__device__ __forceinline__ float to_float(float v) { return v; }
__device__ __forceinline__ float to_float(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_float(__half v) { return __half2float(v); }

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
// exact key of an unselectable element (masked, or -inf) is 0; the all-ones
// NaN pattern also has key 0 and ranks below every other element, exactly
// where an unselectable one would end up.
//
// The kernel first works on raw keys (sign handling only): they order like
// the exact keys except that -0.0 sits one below +0.0 and -inf (raw
// 0x007fffff) is still nonzero. exact_key() maps a raw key to the exact one.
constexpr uint32_t kRawNegZero = 0x7fffffffu;  // raw key of -0.0
constexpr uint32_t kPosZero = 0x80000000u;     // key of +0.0
constexpr uint32_t kRawNegInf = 0x007fffffu;   // raw key of -inf
__device__ __forceinline__ uint32_t raw_key(float f) {
  const uint32_t b = __float_as_uint(f);
  return b ^ ((uint32_t)((int32_t)b >> 31) | 0x80000000u);
}
__device__ __forceinline__ uint32_t fold_zero(uint32_t r) { return r == kRawNegZero ? kPosZero : r; }
__device__ __forceinline__ uint32_t exact_key(uint32_t r) {
  return r == kRawNegInf ? 0u : fold_zero(r);
}

__device__ __forceinline__ int64_t load_index(const void* p, int64_t i, int bytes) {
  // The reference casts q_pos and kv_lens to int32 after loading (T2:161-162).
  return bytes == 8 ? (int64_t)(int32_t)__ldg(reinterpret_cast<const long long*>(p) + i)
                    : (int64_t)__ldg(reinterpret_cast<const int*>(p) + i);
}

// Candidates of a row: block ids 0..n-1 (T2:161-166).
__device__ __forceinline__ int row_candidates(const Params& p, uint32_t row) {
  const int64_t b = fast_div(row, p.hq_mul, p.hq_shift);
  const int64_t q = row - fast_div(row, p.q_mul, p.q_shift) * (uint32_t)p.Q;
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
// above every bin): F[b] = ov + sum of hist[b..511], F[512] = ov, and the bin
// b with F[b+1] < need <= F[b] (1 <= need <= F[0]) into *s_bin. Run by one
// warp: lane l owns the 16 bins 496 - 16 l .. 511 - 16 l (lane 0 the highest).
// The caller brackets it with CTA barriers.
__device__ __forceinline__ void suffix_scan_warp(const uint32_t* hist, uint32_t ov, uint32_t need,
                                                 uint32_t* F, uint32_t* s_bin) {
  const int lane = threadIdx.x & 31;
  const int lo = kBins - 16 * (lane + 1);
  uint32_t h[16];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint4 v = reinterpret_cast<const uint4*>(hist + lo)[q];
    h[4 * q] = v.x;
    h[4 * q + 1] = v.y;
    h[4 * q + 2] = v.z;
    h[4 * q + 3] = v.w;
  }
  uint32_t local = 0;
#pragma unroll
  for (int i = 0; i < 16; ++i) local += h[i];
  uint32_t incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t u = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += u;
  }
  uint32_t acc = ov + incl - local;  // keys in bins above this lane's range
  uint32_t f[16];
#pragma unroll
  for (int i = 15; i >= 0; --i) {
    if (acc < need && need <= acc + h[i]) *s_bin = (uint32_t)(lo + i);
    acc += h[i];
    f[i] = acc;
  }
#pragma unroll
  for (int q = 0; q < 4; ++q)
    reinterpret_cast<uint4*>(F + lo)[q] = make_uint4(f[4 * q], f[4 * q + 1], f[4 * q + 2], f[4 * q + 3]);
  if (lane == 0) F[kBins] = ov;
}

// out_blocks[row, slot] = id and out_pages[row, slot] = page_table[b, id]
// (-1 for both when id < 0), T2:170-175.
__device__ __forceinline__ void write_out(const Params& p, int64_t row, uint32_t slot, int32_t id) {
  const int64_t o = row * (int64_t)p.K + slot;
  int64_t page = -1;
  if (id >= 0) {
    const int64_t b = fast_div((uint32_t)row, p.hq_mul, p.hq_shift);
    const int64_t pi = b * (int64_t)p.NB + id;
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

// --------------------------------------------------------------- kernel
// NT threads per CTA (128, 256 or 512), J vectors per thread. The register
// budget leaves room for 7 CTAs of 128 threads per SM (6 when J >= 7,
// 2 of 256 threads).
template <typename Tin, int J, int NT>
__global__ void __launch_bounds__(NT, NT == 128 ? (J >= 7 ? 6 : 7) : NT == 256 ? 2 : 1)
    dsa_topk_kernel(const Params p) {
  using V = Vec4<Tin>;
  using raw = typename V::raw;
  extern __shared__ __align__(16) uint8_t smem[];
  constexpr int T = NT;
  // keys a thread vouches for in the lower bound: its VOUCH largest vector maxima
  constexpr int VOUCH = vouch_of(J);
  const int t = threadIdx.x;
  const int lane = t & 31, warp = t >> 5, nw = T >> 5;
  const int NB = p.NB;
  const int nvec = NB >> 2;
  const int K = p.K;
  const int cap = p.cap;
  const Smem L = smem_layout(T, J, V::kBytes, K, cap);
  uint64_t* cand = reinterpret_cast<uint64_t*>(smem + L.cand);
  uint32_t* hist = reinterpret_cast<uint32_t*>(smem + L.hist);
  uint32_t* F = reinterpret_cast<uint32_t*>(smem + L.F);
  __shared__ uint32_t s_red[2][4][32];
  __shared__ uint32_t s_buf[32];
  __shared__ uint32_t s_C;
  __shared__ uint32_t s_bin;
  const Tin* scores = static_cast<const Tin*>(p.scores);

  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  raw* const stage = reinterpret_cast<raw*>(smem + L.stage);
  uint64_t* const ord = reinterpret_cast<uint64_t*>(smem + L.ord);
  auto issue = [&](int64_t r, int n) {
    const Tin* base = scores + r * (int64_t)NB + 4 * t;
    raw* st = stage + t;
    const int nv = (n + 3) >> 2;  // vectors holding candidates (nv <= nvec)
#pragma unroll
    for (int j = 0; j < J; ++j)
      if (j * T + t < nv) cp_async<V::kBytes>(st + j * T, base + 4 * j * T);
    cp_async_commit();
  };

  int64_t row = blockIdx.x;
  const int64_t G = gridDim.x;
  int n_cur = 0, n_next = 0;
  if (row < p.rows) {
    n_cur = row_candidates(p, (uint32_t)row);
    issue(row, n_cur);
    if (row + G < p.rows) n_next = row_candidates(p, (uint32_t)(row + G));
  }
  int rb = 0;  // parity of the reduction buffer
  // The next row's copies go into the staging buffer once this row is done
  // with it: after the compaction (every thread has passed its barrier).
  auto issue_next = [&]() {
    if (row + G < p.rows) {
      issue(row + G, n_next);
      n_cur = n_next;
      if (row + 2 * G < p.rows) n_next = row_candidates(p, (uint32_t)(row + 2 * G));
    }
  };

  for (; row < p.rows; row += G, rb ^= 1) {
    const int n = n_cur;
    // ---- 1. raw keys of this row (own staged vectors), 0 when masked
    cp_async_wait_all();
    uint32_t key[J][4];
    // the VOUCH largest vector maxima of this thread, descending (a[0] = max)
    uint32_t a[VOUCH];
#pragma unroll
    for (int i = 0; i < VOUCH; ++i) a[i] = 0;
    {
      const int nfv = n >> 2;  // vectors whose four blocks are all candidates
#pragma unroll
      for (int j = 0; j < J; ++j) {
        const int v = j * T + t;
        if (v < nfv) {  // warp-uniform except in the warp holding the row's end
          float f[4];
          V::to_f32(stage[v], f);
#pragma unroll
          for (int c = 0; c < 4; ++c) key[j][c] = raw_key(f[c]);
        } else {
          float f[4] = {0.f, 0.f, 0.f, 0.f};
          if (v == nfv && 4 * v < n) V::to_f32(stage[v], f);
#pragma unroll
          for (int c = 0; c < 4; ++c) key[j][c] = 4 * v + c < n ? raw_key(f[c]) : 0u;
        }
        uint32_t vm = max(max(key[j][0], key[j][1]), max(key[j][2], key[j][3]));
#pragma unroll
        for (int i = 0; i < VOUCH; ++i) {  // insert into the sorted list
          const uint32_t hi_i = max(a[i], vm);
          vm = min(a[i], vm);
          a[i] = hi_i;
        }
      }
    }
    // ---- 2. block reduction: max raw key and the lower bound t0. A thread
    // holds VOUCH distinct keys >= a[VOUCH-1] (the maxima of VOUCH of its
    // vectors); a group of threads holds VOUCH distinct keys >= the VOUCH-th
    // largest of its members' lists (merged by xor shuffles). With
    // T / group * VOUCH >= K, at least K keys are >= t0 = the smallest
    // group's VOUCH-th largest.
    const uint32_t mx = a[0];
    for (int o = 1; o < p.group; o <<= 1) {
      uint32_t b[VOUCH];
#pragma unroll
      for (int i = 0; i < VOUCH; ++i) b[i] = __shfl_xor_sync(0xffffffffu, a[i], o);
      // top VOUCH of two descending lists: pairwise max against the reversed
      // partner list gives them as a bitonic sequence, then sort it
#pragma unroll
      for (int i = 0; i < VOUCH; ++i) a[i] = max(a[i], b[VOUCH - 1 - i]);
#pragma unroll
      for (int w = VOUCH / 2; w > 0; w /= 2)
#pragma unroll
        for (int i = 0; i < VOUCH; ++i)
          if ((i & w) == 0) {
            const uint32_t x = a[i], y = a[i + w];
            a[i] = max(x, y);
            a[i + w] = min(x, y);
          }
    }
    uint32_t t0 = p.group > 0 ? a[VOUCH - 1] : 0u;
    uint32_t wmx = mx;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      wmx = max(wmx, __shfl_xor_sync(0xffffffffu, wmx, o));
      t0 = min(t0, __shfl_xor_sync(0xffffffffu, t0, o));
    }
    if (lane == 0) {
      s_red[rb][1][warp] = wmx;
      s_red[rb][2][warp] = t0;
    }
    if (t == 0) s_C = 0;
    for (int i = t; i < kBins + 1; i += T) hist[i] = 0;
    __syncthreads();
    uint32_t hi = 0, lo = 0xffffffffu;
    for (int w = 0; w < nw; ++w) {
      hi = max(hi, s_red[rb][1][w]);
      lo = min(lo, s_red[rb][2][w]);
    }
    uint32_t need;
    bool exact = false;  // keys in registers are exact keys
    if (lo > kRawNegInf) {
      // Fast path: every group max is a selectable key, so at least K
      // selectable keys are >= lo, and every raw key >= lo is selectable.
      need = (uint32_t)K;
      if (lo == kPosZero) lo = kRawNegZero;  // -0.0 ranks with +0.0
      hi = fold_zero(hi);
    } else {
      // No usable bound (a group holds no selectable key): exact keys, the
      // selectable count and the exact max, then every selectable key is a
      // candidate.
      uint32_t nz = 0, ex = 0;
#pragma unroll
      for (int j = 0; j < J; ++j)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          key[j][c] = exact_key(key[j][c]);
          nz += key[j][c] != 0u ? 1u : 0u;
          ex = max(ex, key[j][c]);
        }
      exact = true;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        nz += __shfl_xor_sync(0xffffffffu, nz, o);
        ex = max(ex, __shfl_xor_sync(0xffffffffu, ex, o));
      }
      if (lane == 0) {
        s_red[rb][0][warp] = nz;
        s_red[rb][3][warp] = ex;
      }
      __syncthreads();
      uint32_t total = 0;
      hi = 0;
      for (int w = 0; w < nw; ++w) {
        total += s_red[rb][0][w];
        hi = max(hi, s_red[rb][3][w]);
      }
      need = total < (uint32_t)K ? total : (uint32_t)K;
      lo = 1u;
      // s_red[rb] is rewritten two rows from now, after this row's barriers
    }

    if (need > 0) {
      // ---- 3. compaction of the keys >= lo (refined first if too many);
      // codes carry the exact key (the only raw key >= lo that differs from
      // its exact key is -0.0)
      uint32_t C = 0;
      bool tie_path = false;
      uint32_t kth = 0, above = 0;
      uint32_t s = 0;  // digit shift of the exact stage: (key - lo) >> s < 512
      for (;;) {
        s = digit_shift(lo, hi);
        // bit 4j + c of `mask`: key[j][c] >= lo (J * 4 <= 32 keys)
        // (per-vector nibbles first, then combined pairwise: no 32-long
        // dependency chain through one register)
        uint32_t nib[J];
#pragma unroll
        for (int j = 0; j < J; ++j)
          nib[j] = (key[j][0] >= lo ? 1u : 0u) | (key[j][1] >= lo ? 2u : 0u) |
                   (key[j][2] >= lo ? 4u : 0u) | (key[j][3] >= lo ? 8u : 0u);
#pragma unroll
        for (int w = 1; w < J; w *= 2)
#pragma unroll
          for (int j = 0; j + w < J; j += 2 * w) nib[j] |= nib[j + w] << (4 * w);
        uint32_t mask = nib[0];
        const uint32_t cnt = __popc(mask);
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
          // the candidate's score is re-read from the staging buffer; its
          // exact key is the raw key with -0.0 folded (the mask holds no
          // masked, -inf or key-0 element)
          const Tin* sv = reinterpret_cast<const Tin*>(stage) + 4 * t;
          const uint32_t nid = 0xffffffffu - 4u * (uint32_t)t;  // ~id of this thread's block 0
          auto append = [&](auto fold) {
            // two candidates per trip: independent loads and stores overlap
            while (mask) {
              const int i0 = __ffs(mask) - 1;
              mask &= mask - 1;
              const bool two = mask != 0;
              const int i1 = two ? __ffs(mask) - 1 : i0;
              mask &= two ? mask - 1 : mask;
              const int off0 = (i0 >> 2) * (4 * T) + (i0 & 3);  // id - 4t
              const int off1 = (i1 >> 2) * (4 * T) + (i1 & 3);
              uint32_t k0 = raw_key(to_float(sv[off0]));
              uint32_t k1 = raw_key(to_float(sv[off1]));
              if (decltype(fold)::value) {
                k0 = fold_zero(k0);
                k1 = fold_zero(k1);
              }
              cand[o] = ((uint64_t)k0 << 32) | (uint64_t)(nid - (uint32_t)off0);
              atomicAdd(&hist[(k0 - lo) >> s], 1u);
              if (two) {
                cand[o + 1] = ((uint64_t)k1 << 32) | (uint64_t)(nid - (uint32_t)off1);
                atomicAdd(&hist[(k1 - lo) >> s], 1u);
              }
              o += two ? 2 : 1;
            }
          };
          if (lo <= kPosZero)
            append(std::true_type{});
          else
            append(std::false_type{});
        }
        __syncthreads();
        C = s_C;
        if (C <= (uint32_t)cap) break;

        // Too many: radix refinement of the bound over the register keys
        // (made exact first, so that -0.0 and +0.0 are one value). Level 0
        // spans [lo, hi]; each level splits the K-th key's bin of the
        // previous level into 512 (keys above it counted as overflow).
        if (!exact) {
#pragma unroll
          for (int j = 0; j < J; ++j)
#pragma unroll
            for (int c = 0; c < 4; ++c) key[j][c] = exact_key(key[j][c]);
          exact = true;
          lo = fold_zero(lo);
        }
        uint32_t sr = digit_shift(lo, hi);
        uint32_t lvl_lo = lo;
        for (;;) {
          // (the failed compaction above, or the previous level, counted
          // into hist; every thread has read it since the last barrier)
          for (int i = t; i < kBins + 1; i += T) hist[i] = 0;
          __syncthreads();
#pragma unroll
          for (int j = 0; j < J; ++j)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const uint32_t k = key[j][c];
              if (k >= lvl_lo) {
                const uint32_t d = (k - lvl_lo) >> sr;
                atomicAdd(&hist[d < (uint32_t)kBins ? d : (uint32_t)kBins], 1u);
              }
            }
          __syncthreads();
          if (warp == 0) suffix_scan_warp(hist, hist[kBins], need, F, &s_bin);
          __syncthreads();
          const uint32_t b = s_bin;
          const uint32_t cnt_ge = F[b];
          above = F[b + 1];
          lvl_lo += b << sr;
          if (cnt_ge <= (uint32_t)cap) {
            lo = lvl_lo;
            break;
          }
          if (sr == 0) {  // one key value, too many copies of it
            tie_path = true;
            kth = lvl_lo;
            break;
          }
          sr = sr > (uint32_t)kBinBits ? sr - kBinBits : 0u;
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
        lo = kth;
        s = digit_shift(lo, hi);
#pragma unroll
        for (int j = 0; j < J; ++j)
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint32_t k = key[j][c];
            if (k > kth) {
              cand[atomicAdd(&s_C, 1u)] =
                  ((uint64_t)k << 32) | (uint64_t)(0xffffffffu - (uint32_t)(4 * (j * T + t) + c));
              atomicAdd(&hist[(k - lo) >> s], 1u);
            }
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
              if (pos < r) {
                cand[atomicAdd(&s_C, 1u)] =
                    ((uint64_t)kth << 32) | (uint64_t)(0xffffffffu - (uint32_t)(4 * (j * T + t) + c));
                atomicAdd(&hist[0], 1u);
              }
              ++pos;
            }
          }
          eq_base += tot;
        }
        __syncthreads();
        C = s_C;
      }

      issue_next();
      // ---- 4. exact order of the top `need` candidates (their digit
      // histogram was counted during the compaction)
      if (warp == 0) suffix_scan_warp(hist, 0u, need, F, &s_bin);
      __syncthreads();
      const uint32_t bstar = s_bin;
      for (uint32_t i = t; i < C; i += T) {
        const uint64_t code = cand[i];
        const uint32_t d = ((uint32_t)(code >> 32) - lo) >> s;
        if (d >= bstar) ord[F[d + 1] + atomicSub(&hist[d], 1u) - 1u] = code;
      }
      __syncthreads();
      // ---- 5. each winner's slot = its segment start + its rank inside the
      // segment; the thread that finds it writes the id and the page
      const uint32_t E = F[bstar];
      for (uint32_t i = t; i < E; i += T) {
        const uint64_t code = ord[i];
        const uint32_t d = ((uint32_t)(code >> 32) - lo) >> s;
        const uint32_t s0 = F[d + 1], s1 = F[d];
        uint32_t rank = 0;
        for (uint32_t q = s0; q < s1; ++q) rank += ord[q] > code ? 1u : 0u;
        const uint32_t slot = s0 + rank;
        if (slot < need) write_out(p, row, slot, (int32_t)(0xffffffffu - (uint32_t)code));
      }
    }
    if (need == 0) issue_next();
    // slots beyond the selectable count
    for (int k = (int)need + t; k < K; k += T) write_out(p, row, (uint32_t)k, -1);
  }
  cp_async_wait_all();
}

using KernelFn = void (*)(const Params);
KernelFn topk_kernel(int scores_dtype, int J, int T);  // dsa_topk.cu

}  // namespace dsa
