// K10 / K12 helpers: MLA latent-KV preparation, the absorbed per-head
// projections, and MoE routing (softmax_i64 + top-k).  Integer semantics are
// defined in arc_chain_b200/models/mla_moe.py (the oracle this must match);
// the building blocks are the reference's (RMSNorm, half-split RoPE, per-row
// INT8 linear, softmax_i64: crates/arc-inference/src/cached_integer_model.rs
// 221-262, 985-1012; integer_lut.rs 78-100).
#include <climits>

#include "common.cuh"
#include "lut.cuh"

using namespace q16;

namespace {

constexpr int PAGE = 16;

__device__ __forceinline__ uint64_t warp_sum_u64(uint64_t v) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v += (uint64_t)__shfl_xor_sync(0xffffffffu, (unsigned long long)v, m);
  return v;
}

__device__ uint64_t block_sum_u64(uint64_t v, uint64_t* sh) {
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
  const uint64_t r = sh[0];
  __syncthreads();
  return r;
}

// Latent KV of one slot: c = RMSNorm(kva[:r], kv_norm), k_rope = RoPE(kva[r:]),
// written as one cache row [c | k_rope] at (page, pos % 16).  grid = B.
__global__ void k_mla_kv(const int64_t* __restrict__ kva, int r, int dr, const int64_t* __restrict__ gamma,
                         int ngamma, int64_t* __restrict__ cache, const int* __restrict__ pt, int pt_stride,
                         const int* __restrict__ pos, const int64_t* __restrict__ rcos,
                         const int64_t* __restrict__ rsin, int max_seq, int* __restrict__ err) {
  pdl_wait_dep();
  pdl_allow_next();
  __shared__ uint64_t sh[32];
  const int b = blockIdx.x;
  const int dk = r + dr;
  const int64_t* x = kva + (size_t)b * dk;
  uint64_t ss = 0;
  for (int i = threadIdx.x; i < r; i += blockDim.x) ss += (uint64_t)(wmul(x[i], x[i]) >> FRAC_BITS);
  ss = block_sum_u64(ss, sh);
  const int p = pos[b];
  if (p < 0 || p >= max_seq) {
    if (threadIdx.x == 0) set_error(err, ARCB_ERR_SEQ_OVERFLOW);
    return;
  }
  const int64_t inv = rms_inv((int64_t)ss, r);
  int64_t* row = cache + ((size_t)pt[(size_t)b * pt_stride + p / PAGE] * PAGE + (p % PAGE)) * dk;
  for (int i = threadIdx.x; i < r; i += blockDim.x) row[i] = rms_apply(x[i], inv, i < ngamma ? gamma[i] : ONE);
  const int half = dr / 2;
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    int64_t x0 = x[r + i], x1 = x[r + i + half];
    rope_pair(x0, x1, rcos[(size_t)p * half + i], rsin[(size_t)p * half + i]);
    row[r + i] = x0;
    row[r + i + half] = x1;
  }
}

// Per-head batched INT8 linear, the shape shared by the two absorbed MLA
// projections: y[b, h, i] = (sum_e W[h * R + i, e] * x[b, h, e]) * s >> 16
// for i < R, e < Kd, over all B slots.  One block owns RB rows of one head:
// the rows are read from HBM once (not once per slot) into shared memory with
// a padded stride (odd word count: lanes reading one word of consecutive rows
// hit distinct banks); slots are staged SC at a time.  Thread t computes row
// t % RB for slot t / RB of the staged chunk.  The i8 x i64 products are
// summed in wrapping u64 by four accumulators (the sum modulo 2^64 does not
// depend on the order, so this equals the oracle's sequential sum).
constexpr int HL_RB = 16;
constexpr int HL_SC = 16;
constexpr int HL_THREADS = HL_RB * HL_SC;

__host__ __device__ inline size_t hl_qstride(int Kd) { return (size_t)Kd + 2; }  // i64 units
__host__ __device__ inline size_t hl_wstride(int Kd) { return (size_t)Kd + 4; }  // bytes
inline size_t hl_smem(int Kd) { return HL_SC * hl_qstride(Kd) * 8 + HL_RB * hl_wstride(Kd); }

// Stages W rows [r0, r0 + RB) of head h; returns nothing (caller syncs).
__device__ __forceinline__ void hl_stage_w(const int8_t* __restrict__ W, int h, int R, int Kd, int r0,
                                           uint8_t* ws) {
  const int words = Kd >> 2;
  const size_t wst = hl_wstride(Kd);
  for (int idx = threadIdx.x; idx < HL_RB * words; idx += blockDim.x) {
    const int rr = idx / words, c = idx - rr * words;
    uint32_t v = 0;
    if (r0 + rr < R) v = __ldg((const uint32_t*)(W + ((size_t)h * R + r0 + rr) * Kd) + c);
    *(uint32_t*)(ws + rr * wst + 4 * c) = v;
  }
}

__device__ __forceinline__ void hl_stage_x(const int64_t* __restrict__ x, size_t ld_b, size_t ld_h, int h, int Kd,
                                           int b0, int nb, int64_t* qs) {
  const size_t qst = hl_qstride(Kd);
  for (int idx = threadIdx.x; idx < nb * Kd; idx += blockDim.x) {
    const int sl = idx / Kd, e = idx - sl * Kd;
    qs[sl * qst + e] = x[(size_t)(b0 + sl) * ld_b + (size_t)h * ld_h + e];
  }
}

__device__ __forceinline__ uint64_t hl_dot(const uint8_t* wrow, const int64_t* qv, int Kd) {
  uint64_t a0 = 0, a1 = 0, a2 = 0, a3 = 0;
  const uint32_t* w4 = (const uint32_t*)wrow;
#pragma unroll 4
  for (int c = 0; c < (Kd >> 2); ++c) {
    const uint32_t w = w4[c];
    const longlong2 q01 = *(const longlong2*)(qv + 4 * c);
    const longlong2 q23 = *(const longlong2*)(qv + 4 * c + 2);
    a0 += (uint64_t)(int64_t)(int8_t)(w & 0xFF) * (uint64_t)q01.x;
    a1 += (uint64_t)(int64_t)(int8_t)((w >> 8) & 0xFF) * (uint64_t)q01.y;
    a2 += (uint64_t)(int64_t)(int8_t)((w >> 16) & 0xFF) * (uint64_t)q23.x;
    a3 += (uint64_t)(int64_t)(int8_t)(w >> 24) * (uint64_t)q23.y;
  }
  return a0 + a1 + a2 + a3;
}

// Absorbed query: Q[b, h] = [Lin_uk[h](q_nope[b, h]) | RoPE(q_rope[b, h])].
// q: [B, H, dn + dr]; W_uk: [H * r, dn] int8, scales [H * r]; Q: [B, H, r + dr].
// grid = (H, ceil(r / RB)); blocks with blockIdx.y == 0 also rotate q_rope.
__global__ void __launch_bounds__(HL_THREADS) k_mla_q(const int64_t* __restrict__ q, int H, int dn, int dr, int r,
                                                      const int8_t* __restrict__ Wuk, const int64_t* __restrict__ suk,
                                                      const int* __restrict__ pos, const int64_t* __restrict__ rcos,
                                                      const int64_t* __restrict__ rsin, int max_seq, int B,
                                                      int64_t* __restrict__ Q) {
  extern __shared__ __align__(16) int64_t hl_sm[];
  int64_t* qs = hl_sm;
  uint8_t* ws = (uint8_t*)(hl_sm + HL_SC * hl_qstride(dn));
  const int h = blockIdx.x, r0 = blockIdx.y * HL_RB;
  hl_stage_w(Wuk, h, r, dn, r0, ws);  // weights do not depend on the previous kernel
  pdl_wait_dep();
  pdl_allow_next();
  const int row = threadIdx.x % HL_RB, sl = threadIdx.x / HL_RB, i = r0 + row;
  const int64_t s = i < r ? suk[(size_t)h * r + i] : 0;
  for (int b0 = 0; b0 < B; b0 += HL_SC) {
    const int nb = min(HL_SC, B - b0);
    __syncthreads();
    hl_stage_x(q, (size_t)H * (dn + dr), dn + dr, h, dn, b0, nb, qs);
    __syncthreads();
    if (sl < nb && i < r) {
      const uint64_t acc = hl_dot(ws + row * hl_wstride(dn), qs + sl * hl_qstride(dn), dn);
      Q[((size_t)(b0 + sl) * H + h) * (r + dr) + i] = mulshr((int64_t)acc, s);
    }
  }
  if (blockIdx.y == 0) {
    const int half = dr / 2;
    for (int idx = threadIdx.x; idx < B * half; idx += blockDim.x) {
      const int b = idx / half, j = idx - b * half;
      const int p = min(max(pos[b], 0), max_seq - 1);
      const int64_t* qh = q + ((size_t)b * H + h) * (dn + dr);
      int64_t x0 = qh[dn + j], x1 = qh[dn + j + half];
      rope_pair(x0, x1, rcos[(size_t)p * half + j], rsin[(size_t)p * half + j]);
      int64_t* out = Q + ((size_t)b * H + h) * (r + dr);
      out[r + j] = x0;
      out[r + j + half] = x1;
    }
  }
}

// Per-head output projection o[b, h] = Lin_uv[h](oc[b, h]) straight into the
// limb planes of the W_o GEMM operand (and o_out when given).
// oc: [B, H, r]; W_uv: [H * dv, r].  grid = (H, ceil(dv / RB)).
__global__ void __launch_bounds__(HL_THREADS) k_mla_out(const int64_t* __restrict__ oc, int H, int r, int dv,
                                                        const int8_t* __restrict__ Wuv,
                                                        const int64_t* __restrict__ suv, int B,
                                                        int8_t* __restrict__ X, int* __restrict__ lmax,
                                                        int64_t* __restrict__ o_out) {
  extern __shared__ __align__(16) int64_t hl_sm[];
  __shared__ int need_s;
  int64_t* qs = hl_sm;
  uint8_t* ws = (uint8_t*)(hl_sm + HL_SC * hl_qstride(r));
  const int h = blockIdx.x, r0 = blockIdx.y * HL_RB;
  hl_stage_w(Wuv, h, dv, r, r0, ws);
  if (threadIdx.x == 0) need_s = 0;
  pdl_wait_dep();
  pdl_allow_next();
  const int row = threadIdx.x % HL_RB, sl = threadIdx.x / HL_RB, i = r0 + row;
  const int64_t s = i < dv ? suv[(size_t)h * dv + i] : 0;
  const int d_out = H * dv;
  int need = 0;
  for (int b0 = 0; b0 < B; b0 += HL_SC) {
    const int nb = min(HL_SC, B - b0);
    __syncthreads();
    hl_stage_x(oc, (size_t)H * r, r, h, r, b0, nb, qs);
    __syncthreads();
    if (sl < nb && i < dv) {
      const uint64_t acc = hl_dot(ws + row * hl_wstride(r), qs + sl * hl_qstride(r), r);
      const int64_t v = mulshr((int64_t)acc, s);
      const size_t off = (size_t)(b0 + sl) * d_out + (size_t)h * dv + i;
      if (o_out) o_out[off] = v;
      int8_t dg[8];
      const int n = limb_split8(v, dg);
      need = n > need ? n : need;
#pragma unroll
      for (int l = 0; l < 8; ++l) X[limb_row(l, b0 + sl, B) * d_out + (size_t)h * dv + i] = dg[l];
    }
  }
  need = __reduce_max_sync(0xffffffffu, need);
  if ((threadIdx.x & 31) == 0 && need) atomicMax(&need_s, need);
  __syncthreads();
  if (threadIdx.x == 0 && need_s) atomicMax(lmax, need_s);
}

// MoE routing of one slot: p = softmax_i64(logits[b, :E]); the top_k experts
// by (p desc, index asc) get weight p_e, the others 0; the S shared experts
// (columns E..E+S-1) get ONE.  route: [B, E + S] int64.  One warp per slot,
// lane l owning experts l, l + 32, ...: the max is exact, the wrapping sum is
// order-free, and each top-k round is a warp argmax on (p, -index).
// grid = B, block 32.
__global__ void k_moe_route(const int64_t* __restrict__ logits, int ldl, int E, int S, int top_k,
                            int64_t* __restrict__ route) {
  pdl_wait_dep();
  pdl_allow_next();
  const int b = blockIdx.x, lane = threadIdx.x;
  const int64_t* z = logits + (size_t)b * ldl;
  int64_t* out = route + (size_t)b * (E + S);
  const int64_t* lut = g_exp_lut.v;
  constexpr int PER = 8;  // E <= 256
  int64_t p[PER];
  if (E == 1) {
    p[0] = ONE;
  } else {
    int64_t m = LLONG_MIN;
#pragma unroll
    for (int j = 0; j < PER; ++j)
      if (lane + 32 * j < E) m = max(m, z[lane + 32 * j]);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) m = max(m, (int64_t)__shfl_xor_sync(0xffffffffu, (long long)m, o));
    uint64_t su = 0;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int e = lane + 32 * j;
      p[j] = e < E ? integer_exp(wsub(z[e], m), lut) : 0;
      su += (uint64_t)p[j];
    }
    const int64_t sum = (int64_t)warp_sum_u64(su);
#pragma unroll
    for (int j = 0; j < PER; ++j) p[j] = sum == 0 ? ONE / E : udiv_small(wmul(p[j], ONE), sum);
  }
  for (int e = lane; e < E + S; e += 32) out[e] = e < E ? 0 : ONE;
  __syncwarp();
  uint32_t taken = 0;  // bit j: expert lane + 32 j already chosen
  for (int t = 0; t < top_k && t < E; ++t) {
    int64_t bv = LLONG_MIN;
    int be = INT_MAX;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int e = lane + 32 * j;
      if (e < E && !(taken & (1u << j)) && (p[j] > bv || (p[j] == bv && e < be))) {
        bv = p[j];
        be = e;
      }
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      const int64_t ov = (int64_t)__shfl_xor_sync(0xffffffffu, (long long)bv, o);
      const int oe = __shfl_xor_sync(0xffffffffu, be, o);
      if (ov > bv || (ov == bv && oe < be)) {
        bv = ov;
        be = oe;
      }
    }
    if ((be & 31) == lane) {
      taken |= 1u << (be >> 5);
      out[be] = bv;
    }
  }
}

}  // namespace

extern "C" {

int arcb_mla_kv(const int64_t* kva, int r, int dr, const int64_t* gamma, int ngamma, int64_t* cache, const int* pt,
                int pt_stride, const int* pos, const int64_t* rcos, const int64_t* rsin, int max_seq, int B, int* err,
                void* st) {
  return launch_k(k_mla_kv, dim3(B), dim3(256), 0, (cudaStream_t)st, kva, r, dr, gamma, ngamma, cache, pt, pt_stride,
                  pos, rcos, rsin, max_seq, err);
}

static int hl_attr(const void* k, size_t smem) {
  if (smem <= 48 * 1024) return 0;
  return (int)cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
}

int arcb_mla_q(const int64_t* q, int H, int dn, int dr, int r, const int8_t* Wuk, const int64_t* suk, const int* pos,
               const int64_t* rcos, const int64_t* rsin, int max_seq, int B, int64_t* Q, void* st) {
  if ((dn & 3) || (dr & 1)) return -1;
  const size_t sm = hl_smem(dn);
  if (sm > 227 * 1024) return -2;
  if (int e = hl_attr((const void*)k_mla_q, sm)) return e;
  return launch_k(k_mla_q, dim3(H, (r + HL_RB - 1) / HL_RB), dim3(HL_THREADS), sm, (cudaStream_t)st, q, H, dn, dr, r,
                  Wuk, suk, pos, rcos, rsin, max_seq, B, Q);
}

int arcb_mla_out(const int64_t* oc, int H, int r, int dv, const int8_t* Wuv, const int64_t* suv, int B, int8_t* X,
                 int* lmax, int64_t* o_out, void* st) {
  if (r & 3) return -1;
  const size_t sm = hl_smem(r);
  if (sm > 227 * 1024) return -2;
  if (int e = hl_attr((const void*)k_mla_out, sm)) return e;
  return launch_k(k_mla_out, dim3(H, (dv + HL_RB - 1) / HL_RB), dim3(HL_THREADS), sm, (cudaStream_t)st, oc, H, r, dv,
                  Wuv, suv, B, X, lmax, o_out);
}

int arcb_moe_route(const int64_t* logits, int ldl, int E, int S, int top_k, int B, int64_t* route, void* st) {
  if (E > 256) return -1;
  return launch_k(k_moe_route, dim3(B), dim3(32), 0, (cudaStream_t)st, logits, ldl, E, S, top_k, route);
}

}  // extern "C"
