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

// Absorbed query of head h, slot b: Q[b,h] = [Lin_uk[h](q_nope) | RoPE(q_rope)].
// q: [B, H, dn + dr]; W_uk: [H * r, dn] int8 row-major, scales [H * r].
// grid = (H, B), block 256.
__global__ void k_mla_q(const int64_t* __restrict__ q, int H, int dn, int dr, int r, const int8_t* __restrict__ Wuk,
                        const int64_t* __restrict__ suk, const int* __restrict__ pos,
                        const int64_t* __restrict__ rcos, const int64_t* __restrict__ rsin, int max_seq,
                        int64_t* __restrict__ Q) {
  pdl_wait_dep();
  pdl_allow_next();
  extern __shared__ int64_t qn[];  // dn values
  const int h = blockIdx.x, b = blockIdx.y;
  const int64_t* qh = q + ((size_t)b * H + h) * (dn + dr);
  int64_t* out = Q + ((size_t)b * H + h) * (r + dr);
  for (int e = threadIdx.x; e < dn; e += blockDim.x) qn[e] = qh[e];
  __syncthreads();
  const int8_t* W = Wuk + (size_t)h * r * dn;
  for (int i = threadIdx.x; i < r; i += blockDim.x) {
    uint64_t acc = 0;
    const int8_t* wr = W + (size_t)i * dn;
    for (int e = 0; e < dn; ++e) acc += (uint64_t)(int64_t)wr[e] * (uint64_t)qn[e];
    out[i] = mulshr((int64_t)acc, suk[(size_t)h * r + i]);
  }
  const int p = min(max(pos[b], 0), max_seq - 1);
  const int half = dr / 2;
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    int64_t x0 = qh[dn + i], x1 = qh[dn + i + half];
    rope_pair(x0, x1, rcos[(size_t)p * half + i], rsin[(size_t)p * half + i]);
    out[r + i] = x0;
    out[r + i + half] = x1;
  }
}

// Per-head output projection o[b,h] = Lin_uv[h](oc[b,h]) straight into the
// limb planes of the W_o GEMM operand.  oc: [B, H, r]; W_uv: [H * dv, r].
// grid = (H, B), block 128.
__global__ void k_mla_out(const int64_t* __restrict__ oc, int H, int r, int dv, const int8_t* __restrict__ Wuv,
                          const int64_t* __restrict__ suv, int B, int8_t* __restrict__ X, int* __restrict__ lmax,
                          int64_t* __restrict__ o_out) {
  pdl_wait_dep();
  pdl_allow_next();
  extern __shared__ int64_t xs[];  // r values
  __shared__ int need_s;
  const int h = blockIdx.x, b = blockIdx.y;
  const int64_t* x = oc + ((size_t)b * H + h) * r;
  for (int e = threadIdx.x; e < r; e += blockDim.x) xs[e] = x[e];
  if (threadIdx.x == 0) need_s = 0;
  __syncthreads();
  const int d_out = H * dv;
  int need = 0;
  for (int i = threadIdx.x; i < dv; i += blockDim.x) {
    const int8_t* wr = Wuv + ((size_t)h * dv + i) * r;
    uint64_t acc = 0;
    for (int e = 0; e < r; ++e) acc += (uint64_t)(int64_t)wr[e] * (uint64_t)xs[e];
    const int64_t v = mulshr((int64_t)acc, suv[(size_t)h * dv + i]);
    const size_t off = (size_t)b * d_out + h * dv + i;
    if (o_out) o_out[off] = v;
    int8_t dg[8];
    const int n = limb_split8(v, dg);
    need = n > need ? n : need;
#pragma unroll
    for (int l = 0; l < 8; ++l) X[(size_t)l * B * d_out + off] = dg[l];
  }
  need = __reduce_max_sync(0xffffffffu, need);
  if ((threadIdx.x & 31) == 0 && need) atomicMax(&need_s, need);
  __syncthreads();
  if (threadIdx.x == 0 && need_s) atomicMax(lmax, need_s);
}

// MoE routing of one slot: p = softmax_i64(logits[b, :E]); the top_k experts
// by (p desc, index asc) get weight p_e, the others 0; the S shared experts
// (columns E..E+S-1) get ONE.  route: [B, E + S] int64.  grid = B, block 32.
__global__ void k_moe_route(const int64_t* __restrict__ logits, int ldl, int E, int S, int top_k,
                            int64_t* __restrict__ route) {
  pdl_wait_dep();
  pdl_allow_next();
  const int b = blockIdx.x;
  if (threadIdx.x != 0) return;
  const int64_t* z = logits + (size_t)b * ldl;
  int64_t* out = route + (size_t)b * (E + S);
  const int64_t* lut = g_exp_lut.v;
  int64_t p[256];
  if (E == 1) {
    p[0] = ONE;
  } else {
    int64_t m = z[0];
    for (int e = 1; e < E; ++e) m = z[e] > m ? z[e] : m;
    int64_t s = 0;
    for (int e = 0; e < E; ++e) {
      p[e] = integer_exp(wsub(z[e], m), lut);
      s = wadd(s, p[e]);
    }
    for (int e = 0; e < E; ++e) p[e] = s == 0 ? ONE / E : wmul(p[e], ONE) / s;
  }
  uint32_t taken[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int e = 0; e < E + S; ++e) out[e] = e < E ? 0 : ONE;
  for (int t = 0; t < top_k && t < E; ++t) {
    int best = -1;
    for (int e = 0; e < E; ++e) {
      if (taken[e >> 5] & (1u << (e & 31))) continue;
      if (best < 0 || p[e] > p[best]) best = e;
    }
    taken[best >> 5] |= 1u << (best & 31);
    out[best] = p[best];
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

int arcb_mla_q(const int64_t* q, int H, int dn, int dr, int r, const int8_t* Wuk, const int64_t* suk, const int* pos,
               const int64_t* rcos, const int64_t* rsin, int max_seq, int B, int64_t* Q, void* st) {
  return launch_k(k_mla_q, dim3(H, B), dim3(256), (size_t)dn * 8, (cudaStream_t)st, q, H, dn, dr, r, Wuk, suk, pos,
                  rcos, rsin, max_seq, Q);
}

int arcb_mla_out(const int64_t* oc, int H, int r, int dv, const int8_t* Wuv, const int64_t* suv, int B, int8_t* X,
                 int* lmax, int64_t* o_out, void* st) {
  return launch_k(k_mla_out, dim3(H, B), dim3(128), (size_t)r * 8, (cudaStream_t)st, oc, H, r, dv, Wuv, suv, B, X,
                  lmax, o_out);
}

int arcb_moe_route(const int64_t* logits, int ldl, int E, int S, int top_k, int B, int64_t* route, void* st) {
  if (E > 256) return -1;
  return launch_k(k_moe_route, dim3(B), dim3(32), 0, (cudaStream_t)st, logits, ldl, E, S, top_k, route);
}

}  // extern "C"
