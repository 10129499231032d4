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
// Execution model: one CTA of T threads per row at a time (persistent grid,
// rows blockIdx.x, blockIdx.x + grid, ...). Thread t owns the 4-element
// vectors v = j*T + t, j < J, of a row, i.e. block ids 4v..4v+3; it loads
// them (only those inside the row's causal prefix) one row ahead into
// registers, so the next row's HBM reads overlap this row's selection.
//
// Selection is exact: scores become order-preserving 32-bit keys (0 = not
// selectable), and the K-th largest key is found by a radix select over the
// keys held in registers — digit 1 = bits 31..20 (4096-bin shared-memory
// histogram), then, only for keys in the K-th key's bin, bits 19..10 and
// bits 9..0 (1024 bins each). A pass stops early once the K-th key's bin can
// be taken whole. If the K-th key itself occurs several times, the equal
// keys are taken in block-id order by a block-wide scan (the reference's id
// tie-break). The `need` = min(K, selectable) winners are then ranked by
// their 64-bit (key, ~id) codes, and ids and page-table entries are written
// with coalesced stores.
//
// No scratch memory: all intermediate state is in registers and shared
// memory. No device-side waits.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "dsa_topk.h"

namespace dsa {

constexpr int kMaxThreads = 512;
constexpr int kBins1 = 4096;   // digit 1: key bits 31..20
constexpr int kBins2 = 1024;   // digits 2 and 3: key bits 19..10, 9..0
constexpr int kMaxTopK = 2048;
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
};

// Shared-memory carve-up (dynamic part), identical on host and device.
struct Smem {
  size_t hist, list, outid, total;
};
__host__ __device__ inline Smem smem_layout(int K) {
  Smem L;
  L.hist = 0;
  L.list = L.hist + kBins1 * sizeof(uint32_t);
  L.outid = L.list + (size_t)K * sizeof(uint64_t);
  L.total = L.outid + ((size_t)K * sizeof(int32_t) + 15) / 16 * 16;
  return L;
}

// ------------------------------------------------------------------ loads
template <typename T>
struct Vec4;  // raw storage of 4 scores
template <>
struct Vec4<float> {
  using raw = uint4;
  __device__ __forceinline__ static raw load(const float* p) {
    raw v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
  }
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
  __device__ __forceinline__ static raw load(const __nv_bfloat16* p) {
    raw v;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];"
                 : "=r"(v.x), "=r"(v.y)
                 : "l"(p));
    return v;
  }
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
  __device__ __forceinline__ static raw load(const __half* p) {
    raw v;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];"
                 : "=r"(v.x), "=r"(v.y)
                 : "l"(p));
    return v;
  }
  __device__ __forceinline__ static void to_f32(const raw& v, float f[4]) {
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
    f[0] = a.x;
    f[1] = a.y;
    f[2] = b.x;
    f[3] = b.y;
  }
};

// Order-preserving key of an fp32 score (T2:489-494): -0.0 is folded to
// +0.0, negative values are bit-inverted, the others get the sign bit. The
// key of an unselectable element is 0 (and the all-ones NaN pattern, whose
// key is 0, ranks below every other element, exactly where an unselectable
// one would end up).
__device__ __forceinline__ uint32_t score_key(float f, bool candidate) {
  uint32_t b = __float_as_uint(f);
  if ((b << 1) == 0u) b = 0u;                       // +-0.0 -> +0.0
  const uint32_t k = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return (candidate && b != 0xff800000u) ? k : 0u;  // -inf is not selectable
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

// ------------------------------------------------------------ block scans
// Inclusive prefix sum of `v` over the threads of the CTA in thread order;
// `tot` receives the CTA total. Uses warp_buf[0..31]; starts and ends with
// __syncthreads-free warp work around one barrier pair.
__device__ __forceinline__ uint32_t block_incl_scan(uint32_t v, uint32_t* warp_buf,
                                                    uint32_t* tot) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t u = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += u;
  }
  if (lane == 31) warp_buf[warp] = v;
  __syncthreads();
  uint32_t before = 0, all = 0;
  for (int w = 0; w < nw; ++w) {
    const uint32_t x = warp_buf[w];
    before += w < warp ? x : 0u;
    all += x;
  }
  *tot = all;
  __syncthreads();  // warp_buf may be reused right after
  return v + before;
}

// Result of a threshold search: the bin holding the `need`-th largest key
// among the histogram's keys, the number of keys in higher bins and in it.
struct BinHit {
  uint32_t bin, above, count;
};

// Every thread owns nbins / T consecutive bins, thread 0 the highest ones.
// Exactly one thread finds need inside its range (1 <= need <= total).
__device__ __forceinline__ BinHit find_bin(const uint32_t* hist, int nbins, uint32_t need,
                                           uint32_t* warp_buf, BinHit* s_hit) {
  const int T = blockDim.x;
  const int bpt = nbins / T;
  const int lo = nbins - (threadIdx.x + 1) * bpt;  // lowest bin of this thread
  uint32_t local = 0;
  for (int i = 0; i < bpt; ++i) local += hist[lo + i];
  uint32_t tot;
  const uint32_t incl = block_incl_scan(local, warp_buf, &tot);
  const uint32_t excl = incl - local;
  if (excl < need && need <= incl) {
    uint32_t acc = excl;
    for (int b = lo + bpt - 1; b >= lo; --b) {
      const uint32_t c = hist[b];
      if (acc + c >= need) {
        *s_hit = BinHit{(uint32_t)b, acc, c};
        break;
      }
      acc += c;
    }
  }
  __syncthreads();
  return *s_hit;
}

// --------------------------------------------------------------- kernel
template <typename Tin, int J>
__global__ void __launch_bounds__(kMaxThreads) dsa_topk_kernel(const Params p) {
  extern __shared__ __align__(16) uint8_t smem[];
  const Smem L = smem_layout(p.K);
  uint32_t* hist = reinterpret_cast<uint32_t*>(smem + L.hist);
  uint64_t* list = reinterpret_cast<uint64_t*>(smem + L.list);
  int32_t* outid = reinterpret_cast<int32_t*>(smem + L.outid);
  __shared__ uint32_t s_warp[32];
  __shared__ uint32_t s_count;
  __shared__ BinHit s_hit;

  using V = Vec4<Tin>;
  using raw = typename V::raw;
  const int T = blockDim.x;
  const int t = threadIdx.x;
  const int NB = p.NB;
  const int K = p.K;
  const Tin* scores = static_cast<const Tin*>(p.scores);

  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  int64_t row = blockIdx.x;
  raw nxt[J];
  int n_nxt = 0;
  auto prefetch = [&](int64_t r) {
    n_nxt = row_candidates(p, r);
    const Tin* base = scores + r * (int64_t)NB;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int v = j * T + t;
      if (4 * v < n_nxt) nxt[j] = V::load(base + 4 * (int64_t)v);
    }
  };
  if (row < p.rows) prefetch(row);

  for (; row < p.rows; row += gridDim.x) {
    // ---- keys of this row (registers), next row's loads in flight
    const int n = n_nxt;
    uint32_t key[J][4];
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int v = j * T + t;
      float f[4] = {0.f, 0.f, 0.f, 0.f};
      if (4 * v < n) V::to_f32(nxt[j], f);
#pragma unroll
      for (int c = 0; c < 4; ++c) key[j][c] = score_key(f[c], 4 * v + c < n);
    }
    if (row + gridDim.x < p.rows) prefetch(row + gridDim.x);

    // ---- pass 1: histogram of bits 31..20
    for (int i = t; i < kBins1 / 4; i += T) reinterpret_cast<uint4*>(hist)[i] = make_uint4(0, 0, 0, 0);
    __syncthreads();
    uint32_t mine = 0;
#pragma unroll
    for (int j = 0; j < J; ++j)
#pragma unroll
      for (int c = 0; c < 4; ++c)
        if (key[j][c]) {
          atomicAdd(&hist[key[j][c] >> 20], 1u);
          ++mine;
        }
    __syncthreads();
    uint32_t total;
    (void)block_incl_scan(mine, s_warp, &total);
    const uint32_t need = total < (uint32_t)K ? total : (uint32_t)K;

    // Selection rule: keys k != 0 with (k >> shift) > prefix, and with
    // (k >> shift) == prefix either all of them (take_all) or, after the
    // last digit, the first `ties` of them in block-id order.
    uint32_t prefix = 0, above = 0;
    int shift = 32;
    bool take_all = true;
    if (need > 0 && need < total) {
      BinHit h = find_bin(hist, kBins1, need, s_warp, &s_hit);
      prefix = h.bin;
      shift = 20;
      above = h.above;
      take_all = h.above + h.count == need;
      for (int pass = 0; pass < 2 && !take_all; ++pass) {
        const int s2 = 10 - 10 * pass;  // digit bits s2+9 .. s2
        for (int i = t; i < kBins2 / 4; i += T) reinterpret_cast<uint4*>(hist)[i] = make_uint4(0, 0, 0, 0);
        __syncthreads();
#pragma unroll
        for (int j = 0; j < J; ++j)
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint32_t k = key[j][c];
            if (k && (k >> shift) == prefix) atomicAdd(&hist[(k >> s2) & (kBins2 - 1)], 1u);
          }
        __syncthreads();
        h = find_bin(hist, kBins2, need - above, s_warp, &s_hit);
        prefix = (prefix << 10) | h.bin;
        shift = s2;
        above += h.above;
        take_all = above + h.count == need;
      }
    }
    // shift == 32 means "every selectable key" (need == total)
    const uint32_t ties = need - above;  // keys equal to the full key to take

    // ---- gather the winners into `list` as 64-bit (key, ~id) codes
    if (t == 0) s_count = 0;
    __syncthreads();
    if (need > 0) {
      uint32_t tie_base = 0;
#pragma unroll
      for (int j = 0; j < J; ++j) {
        const int v = j * T + t;
        bool sel[4];
        uint32_t eq = 0;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint32_t k = key[j][c];
          const uint32_t hi = shift == 32 ? 0u : (k >> shift);
          sel[c] = k != 0 && (shift == 32 || hi > prefix || (hi == prefix && take_all));
          eq += (k != 0 && !take_all && hi == prefix) ? 1u : 0u;
        }
        if (!take_all) {
          // Keys equal to the K-th key: the first `ties` in block-id order
          // (ids 4v+c, v = j*T + t: thread order within one j, j ascending).
          uint32_t tot;
          const uint32_t incl = block_incl_scan(eq, s_warp, &tot);
          uint32_t pos = tie_base + incl - eq;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint32_t k = key[j][c];
            if (k != 0 && (k >> shift) == prefix) {
              sel[c] = pos < ties;
              ++pos;
            }
          }
          tie_base += tot;
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          if (sel[c]) {
            const uint32_t slot = atomicAdd(&s_count, 1u);
            list[slot] = ((uint64_t)key[j][c] << 32) | (uint64_t)(0xffffffffu - (uint32_t)(4 * v + c));
          }
        }
      }
    }
    __syncthreads();

    // ---- rank the winners (codes are unique) and place their ids. Each
    // winner is compared with all the others by `sub` neighbouring lanes
    // (need <= T/sub), whose partial counts are summed by shuffles.
    {
      uint32_t np2 = 1;
      while (np2 < need) np2 <<= 1;
      int sub = (uint32_t)T >= np2 ? T / (int)np2 : 1;
      if (sub > 32) sub = 32;
      const int per_round = T / sub;
      for (uint32_t base = 0; base < need; base += per_round) {
        const uint32_t i = base + t / sub;
        const int part = t & (sub - 1);
        uint32_t rank = 0;
        uint64_t me = 0;
        if (i < need) {
          me = list[i];
          for (uint32_t q = part; q < need; q += sub) rank += list[q] > me ? 1u : 0u;
        }
        for (int o = sub >> 1; o > 0; o >>= 1) rank += __shfl_xor_sync(0xffffffffu, rank, o);
        if (i < need && part == 0) outid[rank] = (int32_t)(0xffffffffu - (uint32_t)me);
      }
    }
    __syncthreads();

    // ---- outputs: ids and their pages, -1 beyond the winners
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
    // the next row's first histogram write must not overtake this row's reads
    __syncthreads();
  }
}

using KernelFn = void (*)(const Params);
KernelFn topk_kernel(int scores_dtype, int J);  // dsa_topk.cu

}  // namespace dsa
