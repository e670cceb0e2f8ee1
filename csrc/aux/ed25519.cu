// A2: Ed25519 batch signature verification on sm_100a, one thread per
// signature (reference: crates/arc-gpu/src/cuda/ed25519_verify.cu:432-494,
// host crates/arc-gpu/src/lib.rs:470-495 verify_strict).  Rule, per
// signature (R, S) on message M under public key A:
//   S < L; A and R decompress (y mod p, square root exists) and are not of
//   small order; k = SHA-512(R || A || M) mod L;
//   valid iff encode([S]B - [k]A) == R.
// Points use extended twisted-Edwards coordinates (X : Y : Z : T), a = -1,
// with the complete unified addition (d is not a square mod p).  [S]B sums
// 64 entries of a fixed table j * 16^i * B (signed radix-16 digits, no
// doublings); [k]A runs 4-bit signed windows over a per-thread table of
// j * A, j = 1..8.  Field arithmetic: ed25519_field.cuh.
#include <cuda_runtime.h>
#include <stdint.h>

#include "../kernels/common.cuh"
#include "ed25519_field.cuh"

namespace ed {

__device__ int32_t g_base[64 * 8 * 30];  // (y+x, y-x, 2d x y) of j 16^i B

struct ge {
  fe X, Y, Z, T;
};
struct gc {  // cached: (Y + X, Y - X, 2Z, 2d T)
  fe ypx, ymx, z2, t2d;
};
struct gn {  // affine table entry: (y + x, y - x, 2d x y)
  fe ypx, ymx, xy2d;
};

__device__ __forceinline__ ge ge_ident() { return ge{fe_zero(), fe_one(), fe_one(), fe_zero()}; }

__device__ __forceinline__ gc ge_cached(const ge& p) {
  return gc{fe_carry(fe_add(p.Y, p.X)), fe_carry(fe_sub(p.Y, p.X)), fe_carry(fe_add(p.Z, p.Z)),
            fe_mul(p.T, fe_const(c_d2))};
}
__device__ __forceinline__ gc gc_neg(const gc& q) { return gc{q.ymx, q.ypx, q.z2, fe_neg(q.t2d)}; }

// p + q (q cached): A = (Y1-X1)(Y2-X2), B = (Y1+X1)(Y2+X2), C = T1 2d T2,
// D = Z1 2Z2, E = B-A, F = D-C, G = D+C, H = B+A -> (EF, GH, FG, EH).
__device__ __forceinline__ ge ge_add(const ge& p, const gc& q) {
  const fe a = fe_mul(fe_sub(p.Y, p.X), q.ymx);
  const fe b = fe_mul(fe_add(p.Y, p.X), q.ypx);
  const fe c = fe_mul(p.T, q.t2d);
  const fe d = fe_mul(p.Z, q.z2);
  const fe e = fe_sub(b, a), f = fe_sub(d, c), g = fe_add(d, c), h = fe_add(b, a);
  return ge{fe_mul(e, f), fe_mul(g, h), fe_mul(f, g), fe_mul(e, h)};
}

// p + q (q affine table entry, Z2 = 1): D = 2 Z1.
__device__ __forceinline__ ge ge_madd(const ge& p, const gn& q) {
  const fe a = fe_mul(fe_sub(p.Y, p.X), q.ymx);
  const fe b = fe_mul(fe_add(p.Y, p.X), q.ypx);
  const fe c = fe_mul(p.T, q.xy2d);
  const fe d = fe_add(p.Z, p.Z);
  const fe e = fe_sub(b, a), f = fe_sub(d, c), g = fe_add(d, c), h = fe_add(b, a);
  return ge{fe_mul(e, f), fe_mul(g, h), fe_mul(f, g), fe_mul(e, h)};
}

// 2p for a = -1: A = X^2, B = Y^2, C = 2 Z^2, E = (X+Y)^2 - A - B,
// G = B - A, F = G - C, H = -A - B -> (EF, GH, FG, EH).  T of the input is
// not used; with_t = false skips the output T.
__device__ __forceinline__ ge ge_dbl(const ge& p, bool with_t) {
  const fe a = fe_sq(p.X), b = fe_sq(p.Y);
  const fe zz = fe_sq(p.Z);
  const fe c = fe_add(zz, zz);
  const fe e = fe_carry(fe_sub(fe_sub(fe_sq(fe_add(p.X, p.Y)), a), b));
  const fe g = fe_sub(b, a);
  const fe f = fe_carry(fe_sub(g, c));
  const fe h = fe_neg(fe_add(a, b));
  ge r;
  r.X = fe_mul(e, f);
  r.Y = fe_mul(g, h);
  r.Z = fe_mul(f, g);
  r.T = with_t ? fe_mul(e, h) : fe_zero();
  return r;
}

__device__ __forceinline__ bool ge_small_order(const ge& p) {
  const ge q = ge_dbl(ge_dbl(ge_dbl(p, false), false), false);
  return fe_iszero(q.X) && fe_iszero(fe_sub(q.Y, q.Z));
}

// Decompression: y from the low 255 bits, x = u v^3 (u v^7)^((p-5)/8) with
// u = y^2 - 1, v = d y^2 + 1; x *= sqrt(-1) when v x^2 = -u; fails when
// neither v x^2 = u nor -u; x negated to the sign bit (x = 0 stays 0).
__device__ bool ge_decompress(const uint64_t w[4], ge& out) {
  const fe y = fe_from_words(w);
  const int sign = (int)(w[3] >> 63);
  const fe yy = fe_sq(y);
  const fe u = fe_sub(yy, fe_one());
  const fe v = fe_add(fe_mul(yy, fe_const(c_d)), fe_one());
  const fe v3 = fe_mul(fe_sq(v), v);
  const fe v7 = fe_mul(fe_sq(v3), v);
  fe x = fe_mul(fe_mul(u, v3), fe_pow22523(fe_mul(u, v7)));
  const fe vxx = fe_mul(v, fe_sq(x));
  if (!fe_iszero(fe_sub(vxx, u))) {
    if (!fe_iszero(fe_add(vxx, u))) return false;
    x = fe_mul(x, fe_const(c_sqrtm1));
  }
  if (fe_isneg(x) != sign) x = fe_neg(x);
  out.X = fe_carry(x);
  out.Y = y;
  out.Z = fe_one();
  out.T = fe_mul(out.X, y);
  return true;
}

__device__ void ge_encode(const ge& p, uint64_t w[4]) {
  const fe zi = fe_invert(p.Z);
  const fe x = fe_mul(p.X, zi), y = fe_mul(p.Y, zi);
  fe_to_words(y, w);
  w[3] |= (uint64_t)fe_isneg(x) << 63;
}

// Signed radix-16 digits e[i] in [-8, 8] with s = sum e[i] 16^i (s < 2^253).
__device__ __forceinline__ void radix16(const uint64_t s[4], int8_t e[64]) {
  int c = 0;
#pragma unroll
  for (int i = 0; i < 64; ++i) {
    int v = (int)((s[i >> 4] >> (4 * (i & 15))) & 15) + c;
    c = (v + 8) >> 4;
    v -= c << 4;
    e[i] = (int8_t)v;
  }
  e[63] = (int8_t)(e[63] + (c << 4));
}

__device__ __forceinline__ gn base_entry(int i, int e) {
  gn r;
  if (e == 0) {
    r.ypx = fe_one();
    r.ymx = fe_one();
    r.xy2d = fe_zero();
    return r;
  }
  const int a = e < 0 ? -e : e;
  const int32_t* t = g_base + ((size_t)i * 8 + (a - 1)) * 30;
#pragma unroll
  for (int k = 0; k < 10; ++k) {
    r.ypx.v[k] = __ldg(t + k);
    r.ymx.v[k] = __ldg(t + 10 + k);
    r.xy2d.v[k] = __ldg(t + 20 + k);
  }
  if (e < 0) {
    const fe tmp = r.ypx;
    r.ypx = r.ymx;
    r.ymx = tmp;
    r.xy2d = fe_neg(r.xy2d);
  }
  return r;
}

__device__ ge mul_base(const uint64_t s[4]) {
  int8_t e[64];
  radix16(s, e);
  ge p = ge_ident();
  for (int i = 0; i < 64; ++i) p = ge_madd(p, base_entry(i, e[i]));
  return p;
}

__device__ ge mul_var(const uint64_t s[4], const ge& a) {
  int8_t e[64];
  radix16(s, e);
  gc tab[8];
  tab[0] = ge_cached(a);
  ge acc = a;
  for (int j = 1; j < 8; ++j) {
    acc = ge_add(acc, tab[0]);
    tab[j] = ge_cached(acc);
  }
  ge q = ge_ident();
  for (int i = 63; i >= 0; --i) {
    if (i != 63) {
      q = ge_dbl(q, false);
      q = ge_dbl(q, false);
      q = ge_dbl(q, false);
      q = ge_dbl(q, true);
    }
    const int v = e[i];
    if (v != 0) {
      const gc t = tab[(v < 0 ? -v : v) - 1];
      q = ge_add(q, v < 0 ? gc_neg(t) : t);
    }
  }
  return q;
}

__device__ __forceinline__ void load32(const uint8_t* p, uint64_t w[4]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint64_t v = 0;
#pragma unroll
    for (int b = 0; b < 8; ++b) v |= (uint64_t)p[8 * i + b] << (8 * b);
    w[i] = v;
  }
}

// Result codes (0 = valid).
enum : int { OK = 0, BAD_S = 1, BAD_A = 2, BAD_R = 3, SMALL_A = 4, SMALL_R = 5, MISMATCH = 6 };

__device__ int verify_one(const uint8_t* sig, const uint8_t* pk, const uint64_t k[4]) {
  uint64_t S[4], Aw[4], Rw[4];
  load32(sig + 32, S);
  if (!scalar_lt_l(S)) return BAD_S;
  load32(pk, Aw);
  load32(sig, Rw);
  ge A, R;
  if (!ge_decompress(Aw, A)) return BAD_A;
  if (!ge_decompress(Rw, R)) return BAD_R;
  if (ge_small_order(A)) return SMALL_A;
  if (ge_small_order(R)) return SMALL_R;
  const ge sb = mul_base(S);
  const ge ka = mul_var(k, A);
  const ge rp = ge_add(sb, gc_neg(ge_cached(ka)));
  uint64_t enc[4];
  ge_encode(rp, enc);
  return (enc[0] == Rw[0] && enc[1] == Rw[1] && enc[2] == Rw[2] && enc[3] == Rw[3]) ? OK : MISMATCH;
}

__device__ void hash_k(const uint8_t* sig, const uint8_t* pk, const uint8_t* msg, int64_t mlen, uint64_t k[4]) {
  Sha512 h;
  h.init();
  for (int i = 0; i < 32; ++i) h.byte(sig[i]);
  for (int i = 0; i < 32; ++i) h.byte(pk[i]);
  for (int64_t i = 0; i < mlen; ++i) h.byte(msg[i]);
  h.finish(64 + (uint64_t)mlen);
  uint64_t x[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    // digest bytes 8i..8i+7 (big-endian word) read as a little-endian integer
    const uint64_t v = h.h[i];
    uint64_t r = 0;
#pragma unroll
    for (int b = 0; b < 8; ++b) r |= ((v >> (8 * b)) & 0xFF) << (8 * (7 - b));
    x[i] = r;
  }
  mod_l(x, k);
}

__global__ void __launch_bounds__(128) k_verify(const uint8_t* __restrict__ sigs, const uint8_t* __restrict__ pks,
                                                const uint8_t* __restrict__ msgs, const int64_t* __restrict__ offs,
                                                int64_t n, int* __restrict__ out) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint8_t* sig = sigs + 64 * i;
  const uint8_t* pk = pks + 32 * i;
  uint64_t k[4];
  hash_k(sig, pk, msgs + offs[i], offs[i + 1] - offs[i], k);
  out[i] = verify_one(sig, pk, k);
}

// Records of 128 bytes [R | S | k | A] with k = H(R || A || M) computed by
// the caller (reduced mod L here), the reference kernel's input layout.
__global__ void __launch_bounds__(128) k_verify_prehashed(const uint8_t* __restrict__ rec, int64_t n,
                                                          int* __restrict__ out) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint8_t* r = rec + 128 * i;
  uint64_t x[8] = {0, 0, 0, 0, 0, 0, 0, 0}, k[4];
  load32(r + 64, x);
  mod_l(x, k);
  out[i] = verify_one(r, r + 96, k);
}

// Test entry: op 0 mul, 1 sq, 2 invert, 3 pow22523 (a, b: field elements as
// 32 bytes), 4 a mod L (a: 64 bytes), 5 [a]B, 6 [a]P (b: point encoding),
// 7 decompress + encode of a; out: 32 bytes, code: 0 ok / 1 failed decode.
__global__ void k_selftest(int op, const uint8_t* __restrict__ in, int64_t n, uint8_t* __restrict__ out,
                           int* __restrict__ code) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint8_t* a = in + 64 * i;
  uint64_t wa[4], wb[4], res[4] = {0, 0, 0, 0};
  load32(a, wa);
  load32(a + 32, wb);
  int c = 0;
  if (op <= 3) {
    const fe fa = fe_from_words(wa), fb = fe_from_words(wb);
    fe r = op == 0 ? fe_mul(fa, fb) : op == 1 ? fe_sq(fa) : op == 2 ? fe_invert(fa) : fe_pow22523(fa);
    fe_to_words(r, res);
  } else if (op == 4) {
    uint64_t x[8];
    for (int j = 0; j < 8; ++j) x[j] = j < 4 ? wa[j] : wb[j - 4];
    mod_l(x, res);
  } else if (op == 5) {
    ge_encode(mul_base(wa), res);
  } else if (op == 6) {
    ge p;
    if (ge_decompress(wb, p)) ge_encode(mul_var(wa, p), res);
    else c = 1;
  } else if (op == 7) {
    ge p;
    if (ge_decompress(wa, p)) ge_encode(p, res);
    else c = 1;
  }
  for (int j = 0; j < 32; ++j) out[32 * i + j] = (uint8_t)(res[j >> 3] >> (8 * (j & 7)));
  code[i] = c;
}

}  // namespace ed

extern "C" {

// Uploads the host-computed constants to the current device: curve (30
// int32: d, 2d, sqrt(-1) limbs), SHA-512 K[80] and H0[8], L (4 words),
// floor(2^512 / L) (5 words), base table (64 * 8 * 30 int32).
int arcb_ed25519_init(const int32_t* curve, const uint64_t* K, const uint64_t* H0, const uint64_t* Lw,
                      const uint64_t* mu, const int32_t* table) {
  cudaError_t e;
  if ((e = cudaMemcpyToSymbol(ed::c_d, curve, 40))) return (int)e;
  if ((e = cudaMemcpyToSymbol(ed::c_d2, curve + 10, 40))) return (int)e;
  if ((e = cudaMemcpyToSymbol(ed::c_sqrtm1, curve + 20, 40))) return (int)e;
  if ((e = cudaMemcpyToSymbol(ed::c_K, K, 80 * 8))) return (int)e;
  if ((e = cudaMemcpyToSymbol(ed::c_H0, H0, 8 * 8))) return (int)e;
  if ((e = cudaMemcpyToSymbol(ed::c_L, Lw, 4 * 8))) return (int)e;
  if ((e = cudaMemcpyToSymbol(ed::c_mu, mu, 5 * 8))) return (int)e;
  if ((e = cudaMemcpyToSymbol(ed::g_base, table, sizeof(int32_t) * 64 * 8 * 30))) return (int)e;
  return 0;
}

// n signatures sigs [n, 64] (R | S), keys pks [n, 32], messages packed in
// msgs with offsets offs [n + 1]; out [n] result codes (0 = valid).
int arcb_ed25519_verify(const uint8_t* sigs, const uint8_t* pks, const uint8_t* msgs, const int64_t* offs, int64_t n,
                        int* out, void* stream) {
  if (n <= 0) return 0;
  const int64_t blocks = (n + 127) / 128;
  return launch_k(ed::k_verify, dim3((unsigned)blocks), dim3(128), 0, (cudaStream_t)stream, sigs, pks, msgs, offs, n,
                  out);
}

int arcb_ed25519_verify_prehashed(const uint8_t* rec, int64_t n, int* out, void* stream) {
  if (n <= 0) return 0;
  const int64_t blocks = (n + 127) / 128;
  return launch_k(ed::k_verify_prehashed, dim3((unsigned)blocks), dim3(128), 0, (cudaStream_t)stream, rec, n, out);
}

int arcb_ed25519_selftest(int op, const uint8_t* in, int64_t n, uint8_t* out, int* code, void* stream) {
  if (n <= 0) return 0;
  const int64_t blocks = (n + 127) / 128;
  return launch_k(ed::k_selftest, dim3((unsigned)blocks), dim3(128), 0, (cudaStream_t)stream, op, in, n, out, code);
}

}  // extern "C"
