// Decode-step kernels around the limb GEMM (K3-K7): embedding, RMSNorm with
// fused limb split, GEMM finalize (limb recombination + per-row scale) fused
// with residual add + next-norm sum of squares / RoPE + paged KV append /
// SwiGLU + limb split, exact split-KV paged decode attention, and repetition
// penalty + argmax.
//
// Integer semantics follow the reference CPU engine bit for bit
// (crates/arc-inference/src/cached_integer_model.rs: RMSNorm 985-1000, RoPE
// 1002-1012, SiLU 1016-1027, attention 1448-1481, penalty/argmax 1537-1548;
// crates/arc-inference/src/integer_lut.rs for exp/softmax/isqrt).
//
// Conventions:
//  * a "slot" is one token of the step's batch (B slots); a slot has a
//    position pos[b] and a page-table row pt[b * pt_stride + page].
//  * limb planes: X + l * B * K + b * K + k, l = 0..7 (signed radix-256
//    digits); lmax is the per-operand max limb count, raised by atomicMax.
//  * P: GEMM partials [8 * B, M] int32, row l * B + b; finalize zeroes what
//    it reads so the next GEMM can accumulate into it.
//  * ss: per-norm sum of squares sum((x*x) >> 16) per slot, u64 wrapping.
//    The producer of a residual stream value (embed, residual finalize) adds
//    into it, so the norm itself is a fully parallel elementwise kernel.
//  * KV cache (per layer): [page][kv_head][16][d_head] int64.
#include <climits>

#include "common.cuh"
#include "lut.cuh"

extern "C" int arcb_get_pdl(void);

using namespace q16;

namespace {

__device__ __forceinline__ uint64_t warp_sum_u64(uint64_t v) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v += (uint64_t)__shfl_xor_sync(0xffffffffu, (unsigned long long)v, m);
  return v;
}

__device__ __forceinline__ int block_max_int(int v, int* sh) {
  v = __reduce_max_sync(0xffffffffu, v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  if (w == 0) {
    int x = l < (int)(blockDim.x >> 5) ? sh[l] : INT_MIN;
    x = __reduce_max_sync(0xffffffffu, x);
    if (l == 0) sh[0] = x;
  }
  __syncthreads();
  int r = sh[0];
  __syncthreads();
  return r;
}

__device__ __forceinline__ uint64_t block_sum_u64(uint64_t v, uint64_t* sh) {
  v = warp_sum_u64(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  if (w == 0) {
    uint64_t x = l < (int)(blockDim.x >> 5) ? sh[l] : 0;
    x = warp_sum_u64(x);
    if (l == 0) sh[0] = x;
  }
  __syncthreads();
  uint64_t r = sh[0];
  __syncthreads();
  return r;
}


// Limb digits of v (slot b, column j of a [rows, ld] limb operand of B slots).
__device__ __forceinline__ void store_limbs(int8_t* X, int B, int ld, int b, int j, int64_t v, int& need) {
  int8_t d[8];
  int n = limb_split8(v, d);
  need = n > need ? n : need;
#pragma unroll
  for (int l = 0; l < 8; ++l) X[limb_row(l, b, B) * ld + j] = d[l];
}

// Recombine one output element from its limb partials and zero them.
__device__ __forceinline__ int64_t fin_elem(int* P, int M, int B, int L, int b, int m, int64_t s) {
  uint64_t acc = 0;
  for (int l = 0; l < L; ++l) {
    int* p = P + (size_t)(l * B + b) * M + m;
    acc += (uint64_t)(int64_t)(*p) << (8 * l);
    *p = 0;
  }
  return mulshr((int64_t)acc, s);
}

__device__ __forceinline__ uint64_t sq16(int64_t x) { return (uint64_t)(wmul(x, x) >> FRAC_BITS); }

// ------------------------------------------------------------------ embed
// h[b] = emb_i8[min(tok, V-1)] * scale (cached_integer_model.rs:1397-1400,
// 1821-1830).  One CTA per slot; also writes the first norm's sum of squares
// into ss[0][b] and zeroes the step's counters and the other ss slots.
__global__ void k_embed(const int* __restrict__ tokens, const int8_t* __restrict__ emb,
                        const int64_t* __restrict__ emb_s, int V, int d, int B, int64_t* __restrict__ h,
                        int* __restrict__ counters, int ncounters, uint64_t* __restrict__ ss, int nss) {
  pdl_wait_dep();
  pdl_allow_next();
  __shared__ uint64_t sh[32];
  const int b = blockIdx.x;
  const uint32_t tok = (uint32_t)tokens[b];
  const int idx = tok >= (uint32_t)V ? V - 1 : (int)tok;
  // emb_s == null: emb is a full-precision Q16 table (int64 [V, d])
  const int64_t s = emb_s ? emb_s[idx] : 0;
  const int64_t* emb64 = (const int64_t*)emb;
  uint64_t acc = 0;
  for (int j = threadIdx.x; j < d; j += blockDim.x) {
    const int64_t v = emb_s ? wmul((int64_t)emb[(size_t)idx * d + j], s) : emb64[(size_t)idx * d + j];
    h[(size_t)b * d + j] = v;
    acc += sq16(v);
  }
  acc = block_sum_u64(acc, sh);
  if (threadIdx.x == 0) ss[b] = acc;
  for (int c = threadIdx.x; c < nss - 1; c += blockDim.x) ss[(size_t)(c + 1) * B + b] = 0;
  if (b == 0)
    for (int c = threadIdx.x; c < ncounters; c += blockDim.x) counters[c] = 0;
}

// ------------------------------------------------------------------ RMSNorm apply + limbs
// y = (((x * isqrt(ss/n + 1)) >> 16) * gamma) >> 16, gamma = ONE past its end.
__global__ void k_norm_limbs(const int64_t* __restrict__ h, const uint64_t* __restrict__ ss,
                             const int64_t* __restrict__ gamma, int ngamma, int d, int B, int8_t* __restrict__ X,
                             int* __restrict__ lmax, int64_t* __restrict__ y_out) {
  pdl_wait_dep();
  pdl_allow_next();
  __shared__ int shi[32];
  const int b = blockIdx.y;
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  // one inverse RMS per warp (an integer square root and a 64-bit division),
  // broadcast to its lanes
  int64_t inv = 0;
  if ((threadIdx.x & 31) == 0) inv = rms_inv((int64_t)ss[b], d);
  inv = (int64_t)__shfl_sync(0xffffffffu, (long long)inv, 0);
  int need = 0;
  if (j < d) {
    const size_t off = (size_t)b * d + j;
    const int64_t y = rms_apply(h[off], inv, j < ngamma ? gamma[j] : ONE);
    if (y_out) y_out[off] = y;
    if (X) store_limbs(X, B, d, b, j, y, need);
  }
  need = block_max_int(need, shi);
  if (threadIdx.x == 0 && lmax) atomicMax(lmax, need);
}

// Self-contained RMSNorm (computes its own sum of squares; one CTA per slot).
__global__ void k_rmsnorm_limbs(const int64_t* __restrict__ h, const int64_t* __restrict__ gamma, int ngamma,
                                int d, int B, int8_t* __restrict__ X, int* __restrict__ lmax,
                                int64_t* __restrict__ y_out) {
  pdl_wait_dep();
  pdl_allow_next();
  __shared__ uint64_t sh[32];
  __shared__ int shi[32];
  const int b = blockIdx.x;
  const int64_t* x = h + (size_t)b * d;
  uint64_t ss = 0;
  for (int j = threadIdx.x; j < d; j += blockDim.x) ss += sq16(x[j]);
  ss = block_sum_u64(ss, sh);
  int64_t inv = 0;
  if ((threadIdx.x & 31) == 0) inv = rms_inv((int64_t)ss, d);
  inv = (int64_t)__shfl_sync(0xffffffffu, (long long)inv, 0);
  int need = 0;
  for (int j = threadIdx.x; j < d; j += blockDim.x) {
    const int64_t y = rms_apply(x[j], inv, j < ngamma ? gamma[j] : ONE);
    if (y_out) y_out[(size_t)b * d + j] = y;
    if (X) store_limbs(X, B, d, b, j, y, need);
  }
  need = block_max_int(need, shi);
  if (threadIdx.x == 0 && lmax) atomicMax(lmax, need);
}

// ------------------------------------------------------------------ finalize
// mode 0: out[b*ldo+m] = v ; mode 1: out[b*ldo+m] += v (residual) and, when
// ss_out is given, ss_out[b] += sum over the CTA of (out*out) >> 16.
__global__ void k_finalize(int* __restrict__ P, int M, int B, const int* __restrict__ lmax,
                           const int64_t* __restrict__ scales, int64_t* __restrict__ out, int ldo, int mode,
                           uint64_t* __restrict__ ss_out) {
  pdl_wait_dep();
  pdl_allow_next();
  __shared__ uint64_t sh[32];
  const int b = blockIdx.y;
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  uint64_t acc = 0;
  if (m < M) {
    const int64_t v = fin_elem(P, M, B, *lmax, b, m, scales[m]);
    int64_t* o = out + (size_t)b * ldo + m;
    const int64_t r = mode == 1 ? wadd(*o, v) : v;
    *o = r;
    acc = sq16(r);
  }
  if (ss_out) {
    acc = block_sum_u64(acc, sh);
    if (threadIdx.x == 0) atomicAdd((unsigned long long*)(ss_out + b), (unsigned long long)acc);
  }
}

// ------------------------------------------------------------------ sampling
// Repetition penalty over the newest min(count, 64) generated ids (compounding,
// newest first), then argmax with lowest-index ties (1533-1548).  Per sampled
// slot s: logits row lrow[s]; hist ring [S, 64]; writes the next token into
// tokens_next[s], appends it to gen[s, count] (cap gen_cap) and the ring, and
// advances pos_inc[s] when given.  done[s] latches on an EOS id.
__global__ void k_sample(int64_t* __restrict__ logits, int ldl, int V, const int* __restrict__ lrow,
                         int* __restrict__ hist, int* __restrict__ count, int* __restrict__ gen, int gen_cap,
                         int* __restrict__ tokens_next, int* __restrict__ pos_inc, int* __restrict__ done,
                         const int* __restrict__ eos, int n_eos) {
  pdl_wait_dep();
  pdl_allow_next();
  __shared__ int64_t sv[32];
  __shared__ int si[32];
  const int s = blockIdx.x;
  if (done && done[s]) return;
  int64_t* lg = logits + (size_t)(lrow ? lrow[s] : s) * ldl;
  const int cnt = count[s];
  // The penalty compounds per occurrence, and occurrences of different ids
  // touch different logits, so the result depends only on each id's count
  // among the newest min(cnt, 64): thread k takes history entry k, and the
  // first entry of each id applies the penalty count times (one round trip
  // instead of 64 dependent ones).
  __shared__ int ht[64];
  const int n = cnt < 64 ? cnt : 64;
  if (threadIdx.x < n) ht[threadIdx.x] = hist[s * 64 + ((cnt - 1 - threadIdx.x) & 63)];
  __syncthreads();
  if (threadIdx.x < n) {
    const int k = threadIdx.x, t = ht[k];
    bool first = t >= 0 && t < V;
    int c = 0;
    for (int j = 0; j < n; ++j) {
      c += ht[j] == t;
      first &= !(j < k && ht[j] == t);
    }
    if (first) {
      int64_t v = lg[t];
      for (int r = 0; r < c; ++r) v = penalize(v);
      lg[t] = v;
    }
  }
  __syncthreads();
  int64_t bv = INT64_MIN;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const int64_t v = lg[i];
    if (v > bv) {
      bv = v;
      bi = i;
    }
  }
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) {
    const int64_t ov = (int64_t)__shfl_xor_sync(0xffffffffu, (long long)bv, m);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, m);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) {
    sv[w] = bv;
    si[w] = bi;
  }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    bv = l < nw ? sv[l] : INT64_MIN;
    bi = l < nw ? si[l] : 0x7fffffff;
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
      const int64_t ov = (int64_t)__shfl_xor_sync(0xffffffffu, (long long)bv, m);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, m);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (l == 0) {
      if (bi == 0x7fffffff) bi = 0;  // V == 0 guard; argmax_i64 returns 0
      tokens_next[s] = bi;
      if (cnt < gen_cap) gen[(size_t)s * gen_cap + cnt] = bi;
      hist[s * 64 + (cnt & 63)] = bi;
      count[s] = cnt + 1;
      if (pos_inc) pos_inc[s] += 1;
      if (done)
        for (int e = 0; e < n_eos; ++e)
          if (eos[e] == bi) done[s] = 1;
    }
  }
}

}  // namespace

int arcb_pdl_enabled() { return arcb_get_pdl(); }

#include "../common/rng.h"

namespace {
__global__ void k_rng_i8(uint64_t key, int8_t* __restrict__ out, int64_t n) {
  pdl_wait_dep();
  pdl_allow_next();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = arcrng::weight_i8(key, (uint64_t)i);
}
}  // namespace

// ==================================================================== C ABI
// Checks udiv_small (q16.h) against the compiler's 64-bit division on the
// divisions the kernels make.  Sigmoid: every den in [den0, den1) (inside
// [ONE, 2 ONE]) against num = ONE * ONE and every num = e * ONE, e in
// [0, ONE].  Softmax weights: n_rand pseudo-random (e <= ONE, sum >= e up to
// 2^40) pairs per thread.  Mismatches are counted into *bad.
__global__ void k_check_udiv(int64_t den0, int64_t den1, int n_rand, unsigned long long* bad) {
  unsigned long long nbad = 0;
  const int64_t den = den0 + blockIdx.x;
  if (den < den1) {
    for (int64_t e = threadIdx.x; e <= ONE + 1; e += blockDim.x) {
      const int64_t num = e <= ONE ? e * ONE : ONE * ONE;
      nbad += udiv_small(num, den) != num / den;
    }
  }
  uint64_t x = 0x9E3779B97F4A7C15ull * (blockIdx.x * blockDim.x + threadIdx.x + 1);
  for (int i = 0; i < n_rand; ++i) {
    x ^= x << 13, x ^= x >> 7, x ^= x << 17;  // xorshift64
    const int64_t e = (int64_t)(x % (uint64_t)(ONE + 1));
    x ^= x << 13, x ^= x >> 7, x ^= x << 17;
    const int64_t sum = e + (int64_t)(x >> (24 + (x & 15)));  // spans many magnitudes
    if (sum == 0) continue;
    nbad += udiv_small(e * ONE, sum) != (e * ONE) / sum;
  }
  if (nbad) atomicAdd(bad, nbad);
}

extern "C" {

static int g_pdl = 1;
void arcb_set_pdl(int on) { g_pdl = on ? 1 : 0; }
int arcb_get_pdl(void) { return g_pdl; }

static inline cudaStream_t S_(void* s) { return (cudaStream_t)s; }

int arcb_embed(const int* tokens, const int8_t* emb, const int64_t* emb_s, int V, int d, int B, int64_t* h,
               int* counters, int ncounters, uint64_t* ss, int nss, void* st) {
  return launch_k(k_embed, dim3(B), dim3(512), 0, S_(st), tokens, emb, emb_s, V, d, B, h, counters, ncounters, ss, nss);
}

int arcb_norm_limbs(const int64_t* h, const uint64_t* ss, const int64_t* gamma, int ngamma, int d, int B,
                    int8_t* X, int* lmax, int64_t* y_out, void* st) {
  dim3 g((d + 255) / 256, B);
  return launch_k(k_norm_limbs, dim3(g), dim3(256), 0, S_(st), h, ss, gamma, ngamma, d, B, X, lmax, y_out);
}

int arcb_rmsnorm_limbs(const int64_t* h, const int64_t* gamma, int ngamma, int d, int B, int8_t* X, int* lmax,
                       int64_t* y_out, void* st) {
  return launch_k(k_rmsnorm_limbs, dim3(B), dim3(512), 0, S_(st), h, gamma, ngamma, d, B, X, lmax, y_out);
}

int arcb_finalize(int* P, int M, int B, const int* lmax, const int64_t* scales, int64_t* out, int ldo, int mode,
                  uint64_t* ss_out, void* st) {
  dim3 g((M + 255) / 256, B);
  return launch_k(k_finalize, dim3(g), dim3(256), 0, S_(st), P, M, B, lmax, scales, out, ldo, mode, ss_out);
}

int arcb_sample(int64_t* logits, int ldl, int V, const int* lrow, int S, int* hist, int* count, int* gen,
                int gen_cap, int* tokens_next, int* pos_inc, int* done, const int* eos, int n_eos, void* st) {
  return launch_k(k_sample, dim3(S), dim3(1024), 0, S_(st), logits, ldl, V, lrow, hist, count, gen, gen_cap, tokens_next, pos_inc, done,
                                    eos, n_eos);
}

int arcb_rng_i8(uint64_t seed, uint64_t stream, int8_t* out, int64_t n, void* st) {
  const uint64_t key = arcrng::stream_key(seed, stream);
  int blocks = (int)((n + 255) / 256);
  if (blocks > 148 * 32) blocks = 148 * 32;
  if (blocks < 1) blocks = 1;
  return launch_k(k_rng_i8, dim3(blocks), dim3(256), 0, S_(st), key, out, n);
}

// Self-check of the kernels' exact small-quotient division (see k_check_udiv).
int arcb_check_udiv(int64_t den0, int64_t den1, int n_rand, unsigned long long* bad, void* st) {
  const int blocks = (int)(den1 - den0) > 0 ? (int)(den1 - den0) : 1;
  return launch_k(k_check_udiv, dim3(blocks), dim3(256), 0, S_(st), den0, den1, n_rand, bad);
}

}  // extern "C"
