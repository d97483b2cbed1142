/*
 * ta_math.h -- portable binary32 arithmetic primitives shared by the sm_100a
 * kernels and by the host-side C restatement used to check them.
 *
 * Every function here is written with IEEE-754 basic operations only
 * (+, -, *, /, sqrt, explicit fmaf) plus exact integer bit manipulation, so a
 * compliant host compiler (gcc -ffp-contract=off) and nvcc (--fmad=false,
 * -prec-div=true, -prec-sqrt=true, no -ftz) produce bit-identical results.
 * Nothing here reproduces a vendor math library: the log/exp kernels are our
 * own Chebyshev fits (coefficients from gen_math_coeffs.py), Philox4x32-10 is
 * the counter-based generator of Salmon, Moraes, Dror and Shaw, "Parallel
 * random numbers: as easy as 1, 2, 3" (SC'11), and the fp16 conversion is the
 * IEEE round-to-nearest-even rule written out on the bit fields.
 *
 * Accuracy (checked exhaustively over all positive binary32 inputs by the
 * test-suite): ta_logf and ta_expf are faithfully rounded (max error < 1 ulp).
 */
#ifndef TA_MATH_H
#define TA_MATH_H

#include <stdint.h>
#include <math.h>

#if defined(__CUDACC__)
#define TA_HD __host__ __device__ __forceinline__
#else
#define TA_HD static inline
#endif

/* ---- bit casts --------------------------------------------------------- */
TA_HD uint32_t ta_f2u(float f) {
#if defined(__CUDA_ARCH__)
  return __float_as_uint(f);
#else
  union { float f; uint32_t u; } c; c.f = f; return c.u;
#endif
}
TA_HD float ta_u2f(uint32_t u) {
#if defined(__CUDA_ARCH__)
  return __uint_as_float(u);
#else
  union { float f; uint32_t u; } c; c.u = u; return c.f;
#endif
}

/* ---- IEEE basic operations (explicitly rounded, never contracted) ------- */
TA_HD float ta_fma(float a, float b, float c) {
#if defined(__CUDA_ARCH__)
  return __fmaf_rn(a, b, c);
#else
  return fmaf(a, b, c);
#endif
}
TA_HD float ta_mul(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fmul_rn(a, b);
#else
  return a * b;
#endif
}
TA_HD float ta_add(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fadd_rn(a, b);
#else
  return a + b;
#endif
}
TA_HD float ta_sub(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fsub_rn(a, b);
#else
  return a - b;
#endif
}
TA_HD float ta_div(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fdiv_rn(a, b);
#else
  return a / b;
#endif
}
TA_HD float ta_sqrt(float a) {
#if defined(__CUDA_ARCH__)
  return __fsqrt_rn(a);
#else
  return sqrtf(a);
#endif
}

/* Polynomial coefficients, highest degree first (gen_math_coeffs.py). */
/* log1p kernel Q(f) = (log1p(f) - f) / f^2 on [-1/3, 1/3], degree 9. */
#define TA_LOG_Q0 0x1.dba26p-4f
#define TA_LOG_Q1 (-0x1.04a268p-3f)
#define TA_LOG_Q2 0x1.bc8cf8p-4f
#define TA_LOG_Q3 (-0x1.f4963ep-4f)
#define TA_LOG_Q4 0x1.24c926p-3f
#define TA_LOG_Q5 (-0x1.55909ep-3f)
#define TA_LOG_Q6 0x1.9998d4p-3f
#define TA_LOG_Q7 (-0x1.ffff2cp-3f)
#define TA_LOG_Q8 0x1.555556p-2f
#define TA_LOG_Q9 (-0x1p-1f)
/* exp kernel P(r) = (e^r - 1 - r) / r^2 on |r| <= ln2/2, degree 5. */
#define TA_EXP_P0 0x1.a127fcp-13f
#define TA_EXP_P1 0x1.6d469p-10f
#define TA_EXP_P2 0x1.1110ep-7f
#define TA_EXP_P3 0x1.5554e6p-5f
#define TA_EXP_P4 0x1.555556p-3f
#define TA_EXP_P5 0x1p-1f

/* ln2 split: TA_LN2_HI has 15 significant bits so e*TA_LN2_HI is exact for
 * |e| < 512. */
#define TA_LN2_HI 0x1.62e4p-1f
#define TA_LN2_LO 0x1.7f7d1cp-20f
#define TA_LOG2E 0x1.715476p+0f

/*
 * Natural logarithm, binary32, faithfully rounded.
 * x = 2^e * m with m in [2/3, 4/3); f = m - 1 (exact);
 * log(x) = e*ln2 + f + f^2 Q(f), with e*ln2_hi + f summed by Fast2Sum so the
 * only large rounding is the final one.
 * Special inputs: NaN -> the same NaN, +inf -> +inf, 0 -> -inf, negative -> NaN.
 */
/* The polynomial core of ta_logf for a normal positive finite x, with the
 * exponent offset ex of a prior exact scaling. Called with ex = 0 on any
 * finite x it is the fast-path log of the kernels (no special cases). */
TA_HD float ta_logf_core(float x, int32_t ex) {
  uint32_t ix = ta_f2u(x);
  int32_t e = ((int32_t)(ix - 0x3f2aaaabu)) >> 23;
  float m = ta_u2f(ix - ((uint32_t)e << 23));
  float f = ta_sub(m, 1.0f); /* exact: m in [2/3, 4/3) */
  float ef = (float)(e + ex);
  float q = TA_LOG_Q0;
  q = ta_fma(q, f, TA_LOG_Q1);
  q = ta_fma(q, f, TA_LOG_Q2);
  q = ta_fma(q, f, TA_LOG_Q3);
  q = ta_fma(q, f, TA_LOG_Q4);
  q = ta_fma(q, f, TA_LOG_Q5);
  q = ta_fma(q, f, TA_LOG_Q6);
  q = ta_fma(q, f, TA_LOG_Q7);
  q = ta_fma(q, f, TA_LOG_Q8);
  q = ta_fma(q, f, TA_LOG_Q9);
  float f2 = ta_mul(f, f);
  float hi = ta_mul(ef, TA_LN2_HI);          /* exact */
  float s = ta_add(hi, f);
  float err = ta_add(ta_sub(hi, s), f);      /* Fast2Sum: exact, |hi| >= |f| or hi == 0 */
  float lo = ta_fma(f2, q, ta_fma(ef, TA_LN2_LO, err));
  return ta_add(s, lo);
}

TA_HD float ta_logf(float x) {
  if (x != x) return x; /* NaN propagates unchanged */
  if (!(x > 0.0f)) {
    if (x == 0.0f) return -INFINITY;
    return ta_u2f(0x7fc00000u); /* negative */
  }
  if (x == INFINITY) return x;
  int32_t ex = 0;
  if (x < 0x1p-126f) { /* subnormal: scale into the normal range (exact) */
    x = ta_mul(x, 0x1p23f);
    ex = -23;
  }
  return ta_logf_core(x, ex);
}

/*
 * Exponential, binary32, faithfully rounded (incl. gradual underflow).
 * k = rint(x*log2e), r = x - k*ln2 (two-step Cody-Waite, first step exact),
 * e^r = 1 + r + r^2 P(r) with 1 + r summed by Fast2Sum, then scaled by
 * 2^k as two exact-or-once-rounded power-of-two multiplications.
 */
TA_HD float ta_expf(float x) {
  if (x != x) return x;
  if (x > 100.0f) return INFINITY;
  if (x < -110.0f) return 0.0f;
  float kf = rintf(ta_mul(x, TA_LOG2E));
  float r = ta_fma(kf, -TA_LN2_HI, x);
  r = ta_fma(kf, -TA_LN2_LO, r);
  float p = TA_EXP_P0;
  p = ta_fma(p, r, TA_EXP_P1);
  p = ta_fma(p, r, TA_EXP_P2);
  p = ta_fma(p, r, TA_EXP_P3);
  p = ta_fma(p, r, TA_EXP_P4);
  p = ta_fma(p, r, TA_EXP_P5);
  float r2 = ta_mul(r, r);
  float s = ta_add(1.0f, r);
  float err = ta_add(ta_sub(1.0f, s), r);    /* Fast2Sum, |1| >= |r| */
  float y = ta_add(s, ta_fma(r2, p, err));
  int32_t k = (int32_t)kf;
  int32_t k1 = k / 2;
  int32_t k2 = k - k1;
  y = ta_mul(y, ta_u2f((uint32_t)(k1 + 127) << 23));
  return ta_mul(y, ta_u2f((uint32_t)(k2 + 127) << 23));
}

/* ---- binary16 conversions (IEEE round-to-nearest-even) ----------------- */
TA_HD uint16_t ta_f32_to_f16(float f) {
  uint32_t x = ta_f2u(f);
  uint32_t sign = (x >> 16) & 0x8000u;
  x &= 0x7fffffffu;
  if (x >= 0x7f800000u) /* inf / NaN (quiet) */
    return (uint16_t)(sign | (x > 0x7f800000u ? 0x7e00u : 0x7c00u));
  if (x >= 0x47800000u) return (uint16_t)(sign | 0x7c00u); /* >= 65536 */
  if (x < 0x38800000u) { /* result is subnormal or zero */
    if (x < 0x33000000u) return (uint16_t)sign; /* < 2^-25 */
    uint32_t e = x >> 23;
    uint32_t m = (x & 0x7fffffu) | 0x800000u;
    uint32_t shift = 126u - e;
    uint32_t q = m >> shift;
    uint32_t rem = m & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1u);
    if (rem > half || (rem == half && (q & 1u))) q++;
    return (uint16_t)(sign | q);
  }
  uint32_t base = x - 0x38000000u;
  uint32_t q = base >> 13;
  uint32_t rem = base & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
  return (uint16_t)(sign | q);
}

TA_HD float ta_f16_to_f32(uint16_t h) {
  uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
  uint32_t e = ((uint32_t)h >> 10) & 0x1fu;
  uint32_t m = (uint32_t)h & 0x3ffu;
  if (e == 0) {
    float v = ta_mul((float)m, 0x1p-24f); /* exact */
    return ta_u2f(ta_f2u(v) | sign);
  }
  if (e == 31) return ta_u2f(sign | 0x7f800000u | (m << 13));
  return ta_u2f(sign | ((e + 112u) << 23) | (m << 13));
}

/* ---- bfloat16 conversions (round-to-nearest-even, NaN kept quiet) ------ */
TA_HD uint16_t ta_f32_to_bf16(float f) {
  uint32_t x = ta_f2u(f);
  if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40u);
  uint32_t lsb = (x >> 16) & 1u;
  x += 0x7fffu + lsb;
  return (uint16_t)(x >> 16);
}
TA_HD float ta_bf16_to_f32(uint16_t h) { return ta_u2f((uint32_t)h << 16); }

/* ---- Philox4x32-10 (Salmon et al., SC'11) ------------------------------ */
#define TA_PHILOX_M0 0xD2511F53u
#define TA_PHILOX_M1 0xCD9E8D57u
#define TA_PHILOX_W0 0x9E3779B9u
#define TA_PHILOX_W1 0xBB67AE85u

TA_HD void ta_philox4x32_10(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3,
                            uint32_t k0, uint32_t k1, uint32_t out[4]) {
#if defined(__CUDA_ARCH__)
#pragma unroll
#endif
  for (int r = 0; r < 10; ++r) {
    uint64_t p0 = (uint64_t)TA_PHILOX_M0 * (uint64_t)c0;
    uint64_t p1 = (uint64_t)TA_PHILOX_M1 * (uint64_t)c2;
    uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
    uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
    c0 = hi1 ^ c1 ^ k0;
    c1 = lo1;
    c2 = hi0 ^ c3 ^ k1;
    c3 = lo0;
    k0 += TA_PHILOX_W0;
    k1 += TA_PHILOX_W1;
  }
  out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

/*
 * Stochastic-rounding draws (shared by kernel and checker).
 * Every element takes a uniform u = (lead * 2^8 + trail) * 2^-24 on the
 * 24-bit grid of torch.rand, with lead (16 bits) and trail (8 bits) from two
 * separate Philox4x32-10 streams keyed by (seed_lo, seed_hi). Element
 * t = 4Q + i of block b (quad Q = j + 8k: lane j of the block's 8-lane
 * group, the lane's quad k, element i of the quad) reads
 *   lead  = 16-bit half (h & 1) of word h >> 1, h = 4(k & 1) + i, of
 *           Philox(b*16 + 2j + (k >> 1), tensor_id, step, b >> 28),
 *   trail = byte i of word k of Philox(b*8 + j, tensor_id, step, (b >> 29) | 2^31).
 * The lead bits alone decide all but about 2^-16 of the roundings (the
 * kernel tests whether u's remaining 2^-16 uncertainty can matter) and the
 * trail stream is drawn only where it can. The draw depends only on (seed,
 * tensor, step, element), so it is the same however the tensor is split
 * across GPUs.
 */
TA_HD void ta_sr_lead_counter(uint64_t block, uint32_t lane, uint32_t pair, uint32_t tensor_id,
                              uint32_t step, uint32_t c[4]) {
  c[0] = (uint32_t)(block * 16u + 2u * lane + pair);
  c[1] = tensor_id;
  c[2] = step;
  c[3] = (uint32_t)(block >> 28);
}
TA_HD void ta_sr_trail_counter(uint64_t block, uint32_t lane, uint32_t tensor_id, uint32_t step,
                               uint32_t c[4]) {
  c[0] = (uint32_t)(block * 8u + lane);
  c[1] = tensor_id;
  c[2] = step;
  c[3] = (uint32_t)(block >> 29) | 0x80000000u;
}
/* lead half of element (k, i) from the lead words of quad pair k >> 1; trail
 * byte from the lane's trail words */
TA_HD uint32_t ta_sr_lead(const uint32_t w[4], int k, int i) {
  const int h = 4 * (k & 1) + i;
  return (w[h >> 1] >> (16 * (h & 1))) & 0xffffu;
}
TA_HD uint32_t ta_sr_trail(const uint32_t t[4], int k, int i) { return (t[k] >> (8 * i)) & 0xffu; }
/* u from its two parts (exact: a 24-bit integer times a power of two) */
TA_HD float ta_sr_u(uint32_t lead, uint32_t trail) {
  return ta_mul((float)((lead << 8) | trail), 0x1p-24f);
}

#endif /* TA_MATH_H */
