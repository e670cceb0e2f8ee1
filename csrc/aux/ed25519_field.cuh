// A2 building blocks: GF(2^255 - 19) arithmetic in ten signed 32-bit limbs
// of alternating 26 and 25 bits (radix 2^25.5), SHA-512 (FIPS 180-4) and the
// reduction of 512-bit integers modulo the group order L (Barrett, HAC
// algorithm 14.42, base 2^64).
//
// Limb k sits at bit e_k = 0, 26, 51, 77, 102, 128, 153, 179, 204, 230.  A
// product f_i g_j lands at e_i + e_j, which is e_{i+j} + 1 when i and j are
// both odd (hence the factor 2), and a position e_{k+10} = e_k + 255 folds
// back with 2^255 = 19 (mod p).  Each f_i g_j is one 32 x 32 -> 64-bit
// multiply-add; the terms that fold are summed apart and multiplied by 19
// once, so a product of limbs up to 2^27 stays below 2^63.  Outputs of
// mul / sq are carried to |limb| <= 2^25 (+ a few units); add / sub do not
// carry, and callers carry any sum of more than two carried values before it
// feeds a multiplication.
//
// Every constant (d, 2d, sqrt(-1), SHA-512 round constants and initial
// words, L, floor(2^512 / L), the base-point table) is computed on the host
// from its definition (arc_chain_b200/crypto/ed25519_ref.py) and uploaded
// into the symbols below by arcb_ed25519_init.
#pragma once
#include <stdint.h>

namespace ed {

__constant__ int32_t c_d[10], c_d2[10], c_sqrtm1[10];
__constant__ uint64_t c_K[80], c_H0[8];
__constant__ uint64_t c_L[4], c_mu[5];

struct fe {
  int32_t v[10];
};

__device__ __forceinline__ int lbits(int k) { return (k & 1) ? 25 : 26; }
__device__ __forceinline__ int lpos(int k) { return 26 * ((k + 1) >> 1) + 25 * (k >> 1); }

__device__ __forceinline__ fe fe_zero() {
  fe r;
#pragma unroll
  for (int i = 0; i < 10; ++i) r.v[i] = 0;
  return r;
}
__device__ __forceinline__ fe fe_one() {
  fe r = fe_zero();
  r.v[0] = 1;
  return r;
}
__device__ __forceinline__ fe fe_const(const int32_t* c) {
  fe r;
#pragma unroll
  for (int i = 0; i < 10; ++i) r.v[i] = c[i];
  return r;
}
__device__ __forceinline__ fe fe_add(const fe& a, const fe& b) {
  fe r;
#pragma unroll
  for (int i = 0; i < 10; ++i) r.v[i] = a.v[i] + b.v[i];
  return r;
}
__device__ __forceinline__ fe fe_sub(const fe& a, const fe& b) {
  fe r;
#pragma unroll
  for (int i = 0; i < 10; ++i) r.v[i] = a.v[i] - b.v[i];
  return r;
}
__device__ __forceinline__ fe fe_neg(const fe& a) {
  fe r;
#pragma unroll
  for (int i = 0; i < 10; ++i) r.v[i] = -a.v[i];
  return r;
}

// Rounding carry chain 0 -> 1 -> ... -> 9 -> 0 -> 1 over 64-bit limbs.
__device__ __forceinline__ fe carry64(int64_t h[10]) {
#pragma unroll
  for (int k = 0; k < 10; ++k) {
    const int b = lbits(k);
    const int64_t c = (h[k] + ((int64_t)1 << (b - 1))) >> b;
    h[k] -= c << b;
    if (k < 9) h[k + 1] += c;
    else h[0] += 19 * c;
  }
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int b = lbits(k);
    const int64_t c = (h[k] + ((int64_t)1 << (b - 1))) >> b;
    h[k] -= c << b;
    h[k + 1] += c;
  }
  fe r;
#pragma unroll
  for (int i = 0; i < 10; ++i) r.v[i] = (int32_t)h[i];
  return r;
}

__device__ __forceinline__ fe fe_carry(const fe& a) {
  int64_t h[10];
#pragma unroll
  for (int i = 0; i < 10; ++i) h[i] = a.v[i];
  return carry64(h);
}

__device__ __forceinline__ fe fe_mul(const fe& f, const fe& g) {
  int64_t lo[10], hi[10];
#pragma unroll
  for (int k = 0; k < 10; ++k) lo[k] = hi[k] = 0;
#pragma unroll
  for (int i = 0; i < 10; ++i) {
    const int32_t fi = f.v[i], fi2 = 2 * f.v[i];
#pragma unroll
    for (int j = 0; j < 10; ++j) {
      const int64_t p = (int64_t)(((i & 1) && (j & 1)) ? fi2 : fi) * (int64_t)g.v[j];
      if (i + j < 10) lo[i + j] += p;
      else hi[i + j - 10] += p;
    }
  }
  int64_t h[10];
#pragma unroll
  for (int k = 0; k < 10; ++k) h[k] = lo[k] + 19 * hi[k];
  return carry64(h);
}

__device__ __forceinline__ fe fe_sq(const fe& f) {
  int64_t lo[10], hi[10];
#pragma unroll
  for (int k = 0; k < 10; ++k) lo[k] = hi[k] = 0;
#pragma unroll
  for (int i = 0; i < 10; ++i) {
#pragma unroll
    for (int j = i; j < 10; ++j) {
      const int c = (i == j ? 1 : 2) * (((i & 1) && (j & 1)) ? 2 : 1);
      const int64_t p = (int64_t)(c * f.v[i]) * (int64_t)f.v[j];
      if (i + j < 10) lo[i + j] += p;
      else hi[i + j - 10] += p;
    }
  }
  int64_t h[10];
#pragma unroll
  for (int k = 0; k < 10; ++k) h[k] = lo[k] + 19 * hi[k];
  return carry64(h);
}

__device__ __forceinline__ fe fe_sqn(fe f, int n) {
  for (int i = 0; i < n; ++i) f = fe_sq(f);
  return f;
}

// Canonical value (0 <= x < p) as limbs in [0, 2^b): floor carries until
// the limbs settle, then subtract p when x + 19 reaches 2^255.
__device__ __forceinline__ void fe_canon(const fe& a, int64_t h[10]) {
#pragma unroll
  for (int i = 0; i < 10; ++i) h[i] = a.v[i];
#pragma unroll
  for (int pass = 0; pass < 4; ++pass) {
#pragma unroll
    for (int k = 0; k < 10; ++k) {
      const int b = lbits(k);
      const int64_t c = h[k] >> b;
      h[k] -= c << b;
      if (k < 9) h[k + 1] += c;
      else h[0] += 19 * c;
    }
  }
  int64_t t[10];
  int64_t c = 19;
#pragma unroll
  for (int k = 0; k < 10; ++k) {
    const int b = lbits(k);
    t[k] = h[k] + c;
    c = t[k] >> b;
    t[k] &= ((int64_t)1 << b) - 1;
  }
  if (c) {
#pragma unroll
    for (int k = 0; k < 10; ++k) h[k] = t[k];
  }
}

// 32 little-endian bytes as four 64-bit words.
__device__ __forceinline__ void fe_to_words(const fe& a, uint64_t w[4]) {
  int64_t h[10];
  fe_canon(a, h);
  w[0] = w[1] = w[2] = w[3] = 0;
#pragma unroll
  for (int k = 0; k < 10; ++k) {
    const int p = lpos(k), q = p >> 6, s = p & 63;
    const uint64_t v = (uint64_t)h[k];
    w[q] |= v << s;
    if (s + lbits(k) > 64) w[q + 1] |= v >> (64 - s);
  }
}

// From four little-endian 64-bit words; bit 255 is ignored and values in
// [p, 2^255) are kept unreduced (they are equal mod p).
__device__ __forceinline__ fe fe_from_words(const uint64_t w[4]) {
  fe r;
#pragma unroll
  for (int k = 0; k < 10; ++k) {
    const int p = lpos(k), q = p >> 6, s = p & 63, b = lbits(k);
    uint64_t v = w[q] >> s;
    if (s + b > 64) v |= w[q + 1] << (64 - s);
    r.v[k] = (int32_t)(v & ((1ull << b) - 1));
  }
  return r;
}

__device__ __forceinline__ bool fe_iszero(const fe& a) {
  uint64_t w[4];
  fe_to_words(a, w);
  return (w[0] | w[1] | w[2] | w[3]) == 0;
}
__device__ __forceinline__ int fe_isneg(const fe& a) {
  uint64_t w[4];
  fe_to_words(a, w);
  return (int)(w[0] & 1);
}

// z^(2^k - 1) for the chain k = 1, 2, 4, 5, 10, 20, 40, 50, 100, 200, 250;
// a(m + n) = a(m)^(2^n) * a(n).
__device__ __forceinline__ fe fe_pow2_250m1(const fe& z) {
  const fe a1 = z;
  const fe a2 = fe_mul(fe_sq(a1), a1);
  const fe a4 = fe_mul(fe_sqn(a2, 2), a2);
  const fe a5 = fe_mul(fe_sq(a4), a1);
  const fe a10 = fe_mul(fe_sqn(a5, 5), a5);
  const fe a20 = fe_mul(fe_sqn(a10, 10), a10);
  const fe a40 = fe_mul(fe_sqn(a20, 20), a20);
  const fe a50 = fe_mul(fe_sqn(a40, 10), a10);
  const fe a100 = fe_mul(fe_sqn(a50, 50), a50);
  const fe a200 = fe_mul(fe_sqn(a100, 100), a100);
  return fe_mul(fe_sqn(a200, 50), a50);
}

// z^(p - 2) = z^((2^250 - 1) * 2^5 + 11)
__device__ __forceinline__ fe fe_invert(const fe& z) {
  const fe z2 = fe_sq(z);
  const fe z11 = fe_mul(fe_mul(fe_sqn(z2, 2), z2), z);
  return fe_mul(fe_sqn(fe_pow2_250m1(z), 5), z11);
}

// z^((p - 5) / 8) = z^((2^250 - 1) * 4 + 1)
__device__ __forceinline__ fe fe_pow22523(const fe& z) { return fe_mul(fe_sqn(fe_pow2_250m1(z), 2), z); }

// ---------------------------------------------------------------- SHA-512
__device__ __forceinline__ uint64_t rotr64(uint64_t x, int n) { return (x >> n) | (x << (64 - n)); }

// Streams bytes into 128-byte blocks; call absorb() per byte run, then
// finish(total_len) and read h.
struct Sha512 {
  uint64_t h[8];
  uint64_t w[16];
  int fill;  // bytes in the current block

  __device__ void init() {
#pragma unroll
    for (int i = 0; i < 8; ++i) h[i] = c_H0[i];
#pragma unroll
    for (int i = 0; i < 16; ++i) w[i] = 0;
    fill = 0;
  }
  __device__ void block() {
    uint64_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
    uint64_t s[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) s[i] = w[i];
#pragma unroll 16
    for (int t = 0; t < 80; ++t) {
      uint64_t wt;
      if (t < 16) {
        wt = s[t & 15];
      } else {
        const uint64_t x15 = s[(t - 15) & 15], x2 = s[(t - 2) & 15];
        const uint64_t s0 = rotr64(x15, 1) ^ rotr64(x15, 8) ^ (x15 >> 7);
        const uint64_t s1 = rotr64(x2, 19) ^ rotr64(x2, 61) ^ (x2 >> 6);
        wt = s[t & 15] + s0 + s[(t - 7) & 15] + s1;
        s[t & 15] = wt;
      }
      const uint64_t S1 = rotr64(e, 14) ^ rotr64(e, 18) ^ rotr64(e, 41);
      const uint64_t ch = (e & f) ^ (~e & g);
      const uint64_t t1 = hh + S1 + ch + c_K[t] + wt;
      const uint64_t S0 = rotr64(a, 28) ^ rotr64(a, 34) ^ rotr64(a, 39);
      const uint64_t mj = (a & b) ^ (a & c) ^ (b & c);
      const uint64_t t2 = S0 + mj;
      hh = g;
      g = f;
      f = e;
      e = d + t1;
      d = c;
      c = b;
      b = a;
      a = t1 + t2;
    }
    h[0] += a;
    h[1] += b;
    h[2] += c;
    h[3] += d;
    h[4] += e;
    h[5] += f;
    h[6] += g;
    h[7] += hh;
#pragma unroll
    for (int i = 0; i < 16; ++i) w[i] = 0;
    fill = 0;
  }
  __device__ __forceinline__ void byte(uint32_t v) {
    const int i = fill >> 3, sh = 56 - 8 * (fill & 7);
    w[i] |= (uint64_t)(v & 0xFF) << sh;
    if (++fill == 128) block();
  }
  __device__ void finish(uint64_t total_len) {
    byte(0x80);
    if (fill > 112) {
      while (fill != 0) byte(0);
    }
    w[14] = 0;
    w[15] = total_len << 3;
    block();
  }
};

// ---------------------------------------------------------------- mod L
typedef unsigned __int128 u128;

// r = x mod L for x < 2^512 (8 little-endian limbs), Barrett with b = 2^64,
// k = 4: q3 = ((x >> 192) * mu) >> 320; r = (x - q3 L) mod 2^320; then at
// most two subtractions of L.
__device__ __forceinline__ void mod_l(const uint64_t x[8], uint64_t r[4]) {
  uint64_t q2[10];
#pragma unroll
  for (int i = 0; i < 10; ++i) q2[i] = 0;
#pragma unroll
  for (int i = 0; i < 5; ++i) {
    u128 c = 0;
#pragma unroll
    for (int j = 0; j < 5; ++j) {
      c += (u128)x[3 + i] * c_mu[j] + q2[i + j];
      q2[i + j] = (uint64_t)c;
      c >>= 64;
    }
    q2[i + 5] = (uint64_t)c;
  }
  const uint64_t* q3 = q2 + 5;
  uint64_t r2[5] = {0, 0, 0, 0, 0};
#pragma unroll
  for (int i = 0; i < 5; ++i) {
    u128 c = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (i + j >= 5) break;
      c += (u128)q3[i] * c_L[j] + r2[i + j];
      r2[i + j] = (uint64_t)c;
      c >>= 64;
    }
    if (i + 4 < 5) r2[i + 4] += (uint64_t)c;
  }
  uint64_t t[5];
  uint64_t borrow = 0;
#pragma unroll
  for (int i = 0; i < 5; ++i) {
    const u128 d = (u128)x[i] - r2[i] - borrow;
    t[i] = (uint64_t)d;
    borrow = (uint64_t)(d >> 64) & 1;
  }
  for (int rep = 0; rep < 3; ++rep) {
    // t >= L ?
    bool ge = t[4] != 0;
    if (!ge) {
      ge = true;
      for (int i = 3; i >= 0; --i) {
        if (t[i] != c_L[i]) {
          ge = t[i] > c_L[i];
          break;
        }
      }
    }
    if (!ge) break;
    uint64_t bw = 0;
#pragma unroll
    for (int i = 0; i < 5; ++i) {
      const u128 d = (u128)t[i] - (i < 4 ? c_L[i] : 0) - bw;
      t[i] = (uint64_t)d;
      bw = (uint64_t)(d >> 64) & 1;
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) r[i] = t[i];
}

__device__ __forceinline__ bool scalar_lt_l(const uint64_t s[4]) {
  for (int i = 3; i >= 0; --i)
    if (s[i] != c_L[i]) return s[i] < c_L[i];
  return false;
}

}  // namespace ed
