// Q16 fixed-point integer primitives shared by the CPU oracle and the sm_100a
// kernels.  Every function here is a bit-exact restatement of the integer
// semantics of the reference engine:
//   crates/arc-inference/src/integer_lut.rs:7-147   (LUT exp, softmax, argmax, isqrt)
//   crates/arc-inference/src/cached_integer_model.rs:985-1027 (RMSNorm, RoPE, SiLU)
//
// The reference is Rust compiled without overflow checks, so i64 `+ - *`
// wrap modulo 2^64.  Signed overflow is undefined in C++/CUDA, so every
// wrapping operation goes through uint64_t and is reinterpreted.  `/` on i64
// truncates toward zero in both languages and `>>` on a signed value is an
// arithmetic shift (guaranteed since C++20, and what nvcc/gcc emit anyway).
#pragma once
#include <stdint.h>

#if defined(__CUDACC__)
#define Q16_HD __host__ __device__ __forceinline__
#else
#define Q16_HD inline
#endif

namespace q16 {

constexpr int FRAC_BITS = 16;
constexpr int64_t ONE = int64_t(1) << FRAC_BITS;  // 65536
constexpr int64_t EXP_RANGE = 8 * ONE;            // LUT covers [-8*ONE, 0]
constexpr int64_t EXP_STEP = ONE / 32;            // 2048 per LUT entry
constexpr int64_t EXP_DECAY = 63521;              // exp(-1/32) in Q16
constexpr int EXP_LUT_N = 257;

// Wrapping i64 arithmetic (two's complement, modulo 2^64).
Q16_HD int64_t wadd(int64_t a, int64_t b) { return (int64_t)((uint64_t)a + (uint64_t)b); }
Q16_HD int64_t wsub(int64_t a, int64_t b) { return (int64_t)((uint64_t)a - (uint64_t)b); }
Q16_HD int64_t wmul(int64_t a, int64_t b) { return (int64_t)((uint64_t)a * (uint64_t)b); }
// (a*b) >> 16 with a wrapping product, as `(a * b) >> FRAC_BITS` in Rust.
Q16_HD int64_t mulshr(int64_t a, int64_t b) { return wmul(a, b) >> FRAC_BITS; }
// Truncating division; i64::MIN / -1 wraps in Rust's release build only via
// an explicit panic path, which cannot be reached with a positive divisor.
Q16_HD int64_t tdiv(int64_t a, int64_t b) { return a / b; }

// floor(num / den) for 0 <= num < 2^34 and den >= 1 whose quotient is below
// 2^20 (the sigmoid and softmax weight divisions: quotients <= ONE).  On the
// device: an estimate from single-precision operands and the correctly
// rounded reciprocal (relative error below 2^-21, so within 1 of the true
// quotient at these sizes), then the exact remainder decides a final +-1
// (the last step of schoolbook long division).  The host divides directly.
Q16_HD int64_t udiv_small(int64_t num, int64_t den) {
#if defined(__CUDA_ARCH__)
  uint64_t q = (uint64_t)((float)num * __frcp_rn((float)den));
  const int64_t r = (int64_t)((uint64_t)num - q * (uint64_t)den);
  if (r < 0) --q;
  else if (r >= den) ++q;
  return (int64_t)q;
#else
  return num / den;
#endif
}

// exp LUT: T[256] = ONE, T[i] = (T[i+1] * 63521) >> 16 (integer_lut.rs:24-51).
// The table is built by the recurrence so it has no float dependency.
inline void build_exp_lut(int64_t* t) {
  t[256] = ONE;
  for (int i = 255; i >= 0; --i) t[i] = (t[i + 1] * EXP_DECAY) >> FRAC_BITS;
}

// integer_exp (integer_lut.rs:56-74) given a prebuilt LUT.
Q16_HD int64_t integer_exp(int64_t x, const int64_t* lut) {
  if (x >= 0) return ONE;
  if (x <= -EXP_RANGE) return 0;
  int64_t off = x + EXP_RANGE;  // (0, 8*ONE)
  int64_t idx = off / EXP_STEP;
  int64_t frac = off % EXP_STEP;
  if (idx >= 256) return ONE;
  int64_t lo = lut[idx];
  int64_t hi = lut[idx + 1];
  return lo + ((hi - lo) * frac) / EXP_STEP;
}

// integer_isqrt (integer_lut.rs:123-147): 3 Newton-Raphson steps in Q16.
Q16_HD int64_t integer_isqrt(int64_t x) {
  if (x <= 0) return ONE * 100;
  uint64_t ux = (uint64_t)x;
#if defined(__CUDA_ARCH__)
  const int lz = __clzll((long long)ux);  // leading zeros (x > 0)
#else
  int lz = 0;
  for (int b = 63; b >= 0; --b) {
    if ((ux >> b) & 1) break;
    ++lz;
  }
#endif
  int64_t bits = 63 - lz;
  // ONE * 256 / 2^k with k <= 32: a positive dividend over a power of two,
  // so the truncating division is the right shift
  int64_t y = (ONE * 256) >> ((bits + 1) / 2);
  if (y <= 0) y = 1;
  for (int it = 0; it < 3; ++it) {
    int64_t y2 = wmul(y, y) >> FRAC_BITS;
    int64_t xy2 = wmul(x, y2) >> FRAC_BITS;
    int64_t three_minus = wsub(3 * ONE, xy2);
    y = wmul(y, three_minus) / (2 * ONE);
    if (y <= 0) y = 1;
  }
  return y;
}

// silu_i64 (cached_integer_model.rs:1016-1027).
Q16_HD int64_t silu(int64_t x, const int64_t* lut) {
  int64_t sig;
  if (x >= 0) {
    int64_t e = integer_exp(wsub(0, x), lut);
    int64_t den = ONE + e;
    if (den < 1) den = 1;
    sig = udiv_small(ONE * ONE, den);  // e in [0, ONE]: den in [ONE, 2 ONE]
  } else {
    int64_t e = integer_exp(x, lut);
    int64_t den = ONE + e;
    if (den < 1) den = 1;
    sig = udiv_small(e * ONE, den);
  }
  return mulshr(x, sig);
}

// Gated FFN element: (silu(g) * u) >> 16 (cached_integer_model.rs:1496-1498).
Q16_HD int64_t swiglu(int64_t g, int64_t u, const int64_t* lut) {
  return mulshr(silu(g, lut), u);
}

// Half-split RoPE of one pair (cached_integer_model.rs:1002-1012).
Q16_HD void rope_pair(int64_t& x0, int64_t& x1, int64_t c, int64_t s) {
  int64_t a = wsub(mulshr(x0, c), mulshr(x1, s));
  int64_t b = wadd(mulshr(x0, s), mulshr(x1, c));
  x0 = a;
  x1 = b;
}

// Repetition penalty of one logit (cached_integer_model.rs:1537-1546).
Q16_HD int64_t penalize(int64_t v) {
  return v > 0 ? wmul(v, 5) / 6 : wmul(v, 6) / 5;
}

// Attention score of one key (cached_integer_model.rs:1460-1463):
// ((dot >> 16) * attn_scale) >> 16, with `dot` the wrapping Q32 dot product.
Q16_HD int64_t attn_score(int64_t dot, int64_t attn_scale) {
  return mulshr(dot >> FRAC_BITS, attn_scale);
}

// RMSNorm scale: isqrt(ss / n + 1) where ss = sum((x*x) >> 16) (985-1000).
Q16_HD int64_t rms_inv(int64_t ss, int64_t n) {
  return integer_isqrt(wadd(ss / n, 1));
}
// RMSNorm output element given inv_rms and gamma.
Q16_HD int64_t rms_apply(int64_t x, int64_t inv_rms, int64_t g) {
  return mulshr(mulshr(x, inv_rms), g);
}

// Signed-digit (radix 256, digits in [-128,127]) limb decomposition used by
// the tensor-core GEMM.  sum_l d_l * 256^l == x (mod 2^64) for 8 digits, and
// `limbs_needed` is the smallest count whose digit sum equals x exactly.
Q16_HD int limbs_needed(int64_t x) {
  int n = 0;
  while (x != 0 && n < 8) {
    int64_t d = (int64_t)(int8_t)(uint8_t)((uint64_t)x & 0xFF);
    x = wsub(x, d) >> 8;
    ++n;
  }
  return n;
}

}  // namespace q16
