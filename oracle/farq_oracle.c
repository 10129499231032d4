/*
 * farq_oracle.c — plain-C CPU restatement of fused residual-add + RMSNorm +
 * per-token group quantisation.
 *
 * TEST INFRASTRUCTURE / CPU BASELINE ONLY. Built by oracle/c_oracle.py (gcc)
 * into oracle/_build/libfarq_oracle.so; used by the tests (cross-check of
 * oracle/farq_oracle.py, bit for bit) and by bench.py's CPU-baseline legs.
 * Nothing in the product path calls it.
 *
 * The arithmetic follows the reference, sinpeyw/flagos-kernelgen-72h-shanghai-2026
 * src/task01_fused_add_rmsnorm_group_quant.py, exactly as oracle/farq_oracle.py
 * restates it (same operation order, same rounding):
 *   r        = f32(x) + f32(residual)                      :1151-1157
 *   residual_out = RNE(r) in the input format              :1160
 *   inv_rms  = 1 / sqrt(fl32(sum r*r (double)) / D + eps)  :1274-1278
 *   w        = r * f32(gamma)                              :1163-1164
 *   gmax     = max |w| over the group                      :1165-1167
 *   norm     = w * inv_rms                                 :1089
 *   scale    = max(gmax * (inv_rms / QMAX), 1e-12)         :1090  (UE8M0: next power of two)
 *   q        = int8: trunc(clamp(norm * (1/scale), +-127)) :1091-1104
 *              e4m3: round-to-nearest-even onto the e4m3fn grid, saturating at +-448
 * Compile without floating-point contraction (-ffp-contract=off): every
 * product and sum is rounded on its own, as in the CUDA kernel.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static inline float bits_f32(uint32_t b) {
  float f;
  memcpy(&f, &b, 4);
  return f;
}
static inline uint32_t f32_bits(float f) {
  uint32_t b;
  memcpy(&b, &f, 4);
  return b;
}

/* 16-bit formats: 0 = bfloat16, 1 = float16. */
static inline float load16(uint16_t h, int fmt) {
  if (fmt == 0) return bits_f32((uint32_t)h << 16);
  /* IEEE half -> float, exact */
  const uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 0x1f, m = h & 0x3ff;
  if (e == 0) {
    if (m == 0) return bits_f32(s);
    return (s ? -1.0f : 1.0f) * ldexpf((float)m, -24); /* subnormal: m * 2^-24, exact */
  }
  if (e == 31) return bits_f32(s | 0x7f800000u | (m << 13));
  return bits_f32(s | ((e + 112) << 23) | (m << 13));
}

/* float -> bfloat16 / float16, round to nearest even (NaN kept quiet). */
static inline uint16_t store16(float f, int fmt) {
  uint32_t b = f32_bits(f);
  if (fmt == 0) {
    if ((b & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((b >> 16) | 0x40);
    b += 0x7fffu + ((b >> 16) & 1u);
    return (uint16_t)(b >> 16);
  }
  const uint32_t s = (b >> 16) & 0x8000u;
  const float a = fabsf(f);
  if (a != a) return (uint16_t)(s | 0x7e00u);
  if (a >= 65520.0f) return (uint16_t)(s | 0x7c00u); /* rounds to inf */
  if (a < ldexpf(1.0f, -14)) {                      /* subnormal: multiple of 2^-24 */
    const float q = rintf(a * ldexpf(1.0f, 24));    /* exact scaling, RNE */
    return (uint16_t)(s | (uint32_t)q);
  }
  int e;
  frexpf(a, &e); /* a = m * 2^e, m in [0.5, 1) */
  const float q = rintf(ldexpf(a, 11 - e)); /* 11 significant bits, RNE */
  /* q in [1024, 2048]; 2048 carries into the next binade */
  uint32_t mant = (uint32_t)q, ex = (uint32_t)(e - 1 + 15);
  if (mant == 2048) {
    mant = 1024;
    ex += 1;
  }
  if (ex >= 31) return (uint16_t)(s | 0x7c00u);
  return (uint16_t)(s | (ex << 10) | (mant - 1024));
}

/* fp32 -> float8_e4m3fn bits, round to nearest even, saturating finite values at +-448.
 * Normal range (|v| >= 2^-6): round the fp32 mantissa to 3 bits in integer
 * arithmetic (add half an ulp minus one, plus the kept lsb, then truncate:
 * ties go to even; a carry moves into the exponent). Below 2^-6 the e4m3
 * grid is uniform in steps of 2^-9, so v * 2^9 (exact) is rounded to an
 * integer. */
static inline uint8_t e4m3(float v) {
  if (v != v) return 0x7f;
  uint32_t b = f32_bits(v);
  const uint8_t s = (b >> 31) ? 0x80 : 0;
  b &= 0x7fffffffu;
  if (b >= 0x43e00000u) return s | 0x7e; /* |v| >= 448 */
  if (b < 0x3c800000u) {                 /* |v| < 2^-6: subnormal grid */
    const float q = rintf(bits_f32(b) * 512.0f);
    return s | (uint8_t)q;               /* q = 8 is the smallest normal, 0x08 */
  }
  b += 0x7ffffu + ((b >> 20) & 1u);
  b &= 0xfff00000u;
  if (b > 0x43e00000u) return s | 0x7e;  /* rounded above 448 */
  const uint32_t ex = (b >> 23) - 127 + 7, mant = (b >> 20) & 7u;
  return s | (uint8_t)((ex << 3) | mant);
}

static inline float pow2_ceil(float s) {
  uint32_t b = f32_bits(s);
  if (b & 0x007fffffu) b = (b & 0xff800000u) + 0x00800000u;
  return bits_f32(b);
}

/*
 * x, residual: [M, D] 16-bit (fmt); gamma: [D] fp32 (already converted);
 * residual_out: [M, D] 16-bit (fmt); norm_out: [M, D] bf16 or NULL;
 * q: [M, D] bytes; scale: [M, D/G] fp32. q_mode 0 = int8, 1 = e4m3.
 * Rows are independent and split over `threads` OpenMP threads (0 = default).
 */
void farq_oracle_rows(const uint16_t* x, const uint16_t* residual, const float* gamma,
                      uint16_t* residual_out, uint16_t* norm_out, uint8_t* q, float* scale,
                      int64_t M, int64_t D, int G, int fmt, int q_mode, int ue8m0, float eps,
                      int threads) {
  const float qmax = q_mode ? 448.0f : 127.0f;
  const int64_t groups = D / G;
#pragma omp parallel num_threads(threads > 0 ? threads : 1) if (threads != 1)
  {
    float r[16384];
#pragma omp for schedule(static)
    for (int64_t m = 0; m < M; ++m) {
      const uint16_t* xr = x + m * D;
      const uint16_t* rr = residual + m * D;
      double ss = 0.0;
      for (int64_t d = 0; d < D; ++d) {
        const float v = load16(xr[d], fmt) + load16(rr[d], fmt);
        r[d] = v;
        residual_out[m * D + d] = store16(v, fmt);
        ss += (double)v * (double)v;
      }
      const float mean = (float)ss / (float)D;
      const float inv = 1.0f / sqrtf(mean + eps);
      const float step = inv / qmax;
      for (int64_t g = 0; g < groups; ++g) {
        float gmax = 0.0f;
        for (int64_t d = g * G; d < (g + 1) * G; ++d) {
          const float w = r[d] * gamma[d];
          const float a = fabsf(w);
          if (a > gmax) gmax = a;
        }
        float sc = gmax * step;
        if (!(sc >= 1.0e-12f)) sc = 1.0e-12f;
        if (ue8m0) sc = pow2_ceil(sc);
        const float isc = 1.0f / sc;
        scale[m * groups + g] = sc;
        for (int64_t d = g * G; d < (g + 1) * G; ++d) {
          const float nrm = (r[d] * gamma[d]) * inv;
          if (norm_out) norm_out[m * D + d] = store16(nrm, 0);
          const float v = nrm * isc;
          if (q_mode) {
            q[m * D + d] = e4m3(v);
          } else {
            float c = v < -127.0f ? -127.0f : (v > 127.0f ? 127.0f : v);
            q[m * D + d] = (uint8_t)(int8_t)(int)truncf(c);
          }
        }
      }
    }
  }
}
