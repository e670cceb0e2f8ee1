// K5: exact paged decode attention in one launch, one thread-block cluster
// per (slot, query head).
//
// Integer semantics (crates/arc-inference/src/cached_integer_model.rs:
// 1448-1476, softmax_i64 integer_lut.rs:78-100): score_j = ((q.k_j >> 16) *
// attn_scale) >> 16 with wrapping i64 dots; w = softmax_i64(scores) which
// needs the exact global max and the exact global sum of the LUT exps; and
// o = sum_j (w_j * v_j) >> 16 rounded per term.  Online (running-max)
// softmax would round differently, so the keys are split over the CTAs of a
// cluster and the three cross-CTA reductions (max, sum of exps, partial
// outputs) are exchanged through distributed shared memory between cluster
// barriers: all integer, so the result does not depend on the split.
//
// grid = (CS, n_heads, B) with cluster (CS, 1, 1); CTA rank r takes keys
// [r*ceil(T/CS), ...).  The output is written straight into the limb planes
// of the W_o GEMM operand (signed radix-256 digits) with its limb count.
#include <climits>

#include "common.cuh"
#include "lut.cuh"

using namespace q16;

int arcb_attn_paged_enabled();

namespace {

constexpr int PAGE = 16;
constexpr int NT = 128;

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint64_t ld_cluster_u64(const void* local, uint32_t rank) {
  uint32_t la = smem_u32(local), ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(la), "r"(rank));
  uint64_t v;
  asm volatile("ld.shared::cluster.u64 %0, [%1];" : "=l"(v) : "r"(ra) : "memory");
  return v;
}

__device__ __forceinline__ uint64_t warp_sum_u64(uint64_t v) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v += (uint64_t)__shfl_xor_sync(0xffffffffu, (unsigned long long)v, m);
  return v;
}

template <int CS>
__global__ void __launch_bounds__(NT) k_attn_cluster(const int64_t* __restrict__ q, const int64_t* __restrict__ Kc,
                                                     const int64_t* __restrict__ Vc, const int* __restrict__ pt,
                                                     int pt_stride, const int* __restrict__ pos, int n_heads,
                                                     int n_kv, int dk, int dv, int kst, int vst,
                                                     int64_t attn_scale, int max_T, int B,
                                                     int8_t* __restrict__ X, int* __restrict__ lmax,
                                                     int64_t* __restrict__ o_out, int* __restrict__ err) {
  pdl_wait_dep();
  pdl_allow_next();
  extern __shared__ int64_t dyn[];
  __shared__ int64_t lut[EXP_LUT_N];
  __shared__ int64_t qs[640];
  __shared__ unsigned long long xo[512];
  __shared__ int64_t red[NT / 32];
  __shared__ long long xmax;
  __shared__ unsigned long long xsum;
  __shared__ int xneed;
  int64_t* sc = dyn;  // local scores, then exps, then weights

  const uint32_t rank = cluster_rank();
  const int hq = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int T = pos[b] + 1;
  const bool bad = T > max_T || T < 1;
  if (bad && rank == 0 && tid == 0) set_error(err, ARCB_ERR_SEQ_OVERFLOW);
  const int chunk = bad ? 0 : (T + CS - 1) / CS;
  const int j0 = min(T, (int)rank * chunk), j1 = bad ? 0 : min(T, j0 + chunk);
  const int n = max(0, j1 - j0);
  const int kvh = hq * n_kv / n_heads;
  const int dq = n_heads * dk, d = n_heads * dv;
  const int* ptb = pt + (size_t)b * pt_stride;

  for (int i = tid; i < EXP_LUT_N; i += NT) lut[i] = g_exp_lut.v[i];
  for (int e = tid; e < dk; e += NT) qs[e] = bad ? 0 : q[(size_t)b * dq + hq * dk + e];
  __syncthreads();

  // ---- phase 1: scores of the local keys, local max
  int64_t mx = INT64_MIN;
  for (int jj = warp; jj < n; jj += 2 * (NT / 32)) {
    const int ja = j0 + jj, jb = ja + NT / 32;
    const bool hb = jj + NT / 32 < n;
    const int64_t* ka = Kc + (((size_t)ptb[ja / PAGE] * n_kv + kvh) * PAGE + (ja % PAGE)) * kst;
    const int64_t* kb = hb ? Kc + (((size_t)ptb[jb / PAGE] * n_kv + kvh) * PAGE + (jb % PAGE)) * kst : ka;
    uint64_t aa = 0, ab = 0;
#pragma unroll 4
    for (int e = lane; e < dk; e += 32) {
      const uint64_t qe = (uint64_t)qs[e];
      aa += qe * (uint64_t)__ldg(ka + e);
      ab += qe * (uint64_t)__ldg(kb + e);
    }
    aa = warp_sum_u64(aa);
    ab = warp_sum_u64(ab);
    const int64_t sa = attn_score((int64_t)aa, attn_scale), sb = attn_score((int64_t)ab, attn_scale);
    if (lane == 0) {
      sc[jj] = sa;
      if (hb) sc[jj + NT / 32] = sb;
    }
    mx = sa > mx ? sa : mx;
    if (hb) mx = sb > mx ? sb : mx;
  }
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  if (tid == 0) {
    int64_t m = red[0];
    for (int w = 1; w < NT / 32; ++w) m = red[w] > m ? red[w] : m;
    xmax = m;
  }
  cluster_sync();
  int64_t gmax = INT64_MIN;
#pragma unroll
  for (int r = 0; r < CS; ++r) {
    const int64_t v = (int64_t)ld_cluster_u64(&xmax, r);
    gmax = v > gmax ? v : gmax;
  }

  // ---- phase 2: exps of the local keys, local sum
  uint64_t s = 0;
  for (int jj = tid; jj < n; jj += NT) {
    const int64_t e = integer_exp(wsub(sc[jj], gmax), lut);
    sc[jj] = e;
    s += (uint64_t)e;
  }
  s = warp_sum_u64(s);
  __syncthreads();
  if (lane == 0) red[warp] = (int64_t)s;
  __syncthreads();
  if (tid == 0) {
    uint64_t t = 0;
    for (int w = 0; w < NT / 32; ++w) t += (uint64_t)red[w];
    xsum = t;
  }
  cluster_sync();
  uint64_t gs = 0;
#pragma unroll
  for (int r = 0; r < CS; ++r) gs += ld_cluster_u64(&xsum, r);
  const int64_t gsum = (int64_t)gs;

  // ---- phase 3: weights, partial outputs of the local keys
  for (int jj = tid; jj < n; jj += NT) {
    int64_t w;
    if (T == 1) w = ONE;
    else if (gsum == 0) w = ONE / T;
    else w = udiv_small(wmul(sc[jj], ONE), gsum);  // e <= gsum: quotient <= ONE
    sc[jj] = w;
  }
  __syncthreads();
  for (int e = tid; e < dv; e += NT) {
    uint64_t o0 = 0, o1 = 0;
    int jj = 0;
    for (; jj + 1 < n; jj += 2) {
      const int ja = j0 + jj, jb = ja + 1;
      const int64_t va = __ldg(Vc + (((size_t)ptb[ja / PAGE] * n_kv + kvh) * PAGE + (ja % PAGE)) * vst + e);
      const int64_t vb = __ldg(Vc + (((size_t)ptb[jb / PAGE] * n_kv + kvh) * PAGE + (jb % PAGE)) * vst + e);
      o0 += (uint64_t)mulshr(sc[jj], va);
      o1 += (uint64_t)mulshr(sc[jj + 1], vb);
    }
    if (jj < n) {
      const int ja = j0 + jj;
      o0 += (uint64_t)mulshr(sc[jj], __ldg(Vc + (((size_t)ptb[ja / PAGE] * n_kv + kvh) * PAGE + (ja % PAGE)) * vst + e));
    }
    xo[e] = o0 + o1;
  }
  if (tid == 0) xneed = 0;
  cluster_sync();

  // ---- cross-CTA sum of partial outputs; rank r finalises a slice of dh
  const int per = (dv + CS - 1) / CS;
  int need = 0;
  for (int e = (int)rank * per + tid; e < min(dv, ((int)rank + 1) * per); e += NT) {
    uint64_t o = 0;
#pragma unroll
    for (int r = 0; r < CS; ++r) o += ld_cluster_u64(&xo[e], r);
    if (bad) continue;
    const size_t off = (size_t)b * d + hq * dv + e;
    if (o_out) o_out[off] = (int64_t)o;
    if (X) {
      int8_t dg[8];
      const int nl = limb_split8((int64_t)o, dg);
      need = nl > need ? nl : need;
#pragma unroll
      for (int l = 0; l < 8; ++l) X[limb_row(l, b, B) * d + hq * dv + e] = dg[l];
    }
  }
  need = __reduce_max_sync(0xffffffffu, need);
  if (lane == 0 && need) atomicMax(&xneed, need);
  __syncthreads();
  if (tid == 0 && lmax && xneed) atomicMax(lmax, xneed);
  cluster_sync();  // no CTA may exit while a peer still reads its shared memory
}

// ---------------------------------------------------------------- TMA-fed form
// The same exact attention for standard heads (dk = dv = row stride = DH,
// DH = 64 or 128), with the cache streamed by the bulk-copy engine: the
// rows of one KV head in one page are one contiguous block (16 x DH int64,
// 16 KB at DH = 128), so CTA rank r takes whole pages [np*r/CS, np*(r+1)/CS)
// and thread 0 streams its K pages, then its V pages, through an R-stage
// shared-memory ring (cp.async.bulk, local memory only).  All page loads are
// in flight from the start up to the ring depth, and the V pages arrive
// while the cluster exchanges the max and the sum; the per-thread loops of
// the plain form wait one DRAM round trip per key pair instead.
#ifndef ARCB_ATTN_RING
#define ARCB_ATTN_RING 4
#endif
constexpr int RING = ARCB_ATTN_RING;

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

template <int CS, int DH>
__global__ void __launch_bounds__(NT) k_attn_paged(const int64_t* __restrict__ q, const int64_t* __restrict__ Kc,
                                                   const int64_t* __restrict__ Vc, const int* __restrict__ pt,
                                                   int pt_stride, const int* __restrict__ pos, int n_heads, int n_kv,
                                                   int64_t attn_scale, int max_T, int B, int8_t* __restrict__ X,
                                                   int* __restrict__ lmax, int64_t* __restrict__ o_out,
                                                   int* __restrict__ err) {
  constexpr int PB = PAGE * DH * 8;      // bytes of one page of one KV head
  constexpr int EPL = DH / 32;           // elements per lane in a dot
  constexpr int GROUPS = NT / DH;        // threads per output element in the value pass
  static_assert(NT == 128 && PAGE == 16, "pass 1 maps 4 warps x 4 keys onto one page");
  extern __shared__ __align__(128) uint8_t dsm[];
  __shared__ int64_t lut[EXP_LUT_N];
  __shared__ __align__(8) uint64_t full[RING];
  __shared__ unsigned long long xo[DH];
  __shared__ unsigned long long part[GROUPS][DH];
  __shared__ int64_t red[NT / 32];
  __shared__ long long xmax;
  __shared__ unsigned long long xsum;
  __shared__ int xneed, abort_;
  const uint32_t ring = (smem_u32(dsm) + 127u) & ~127u;
  int64_t* sc = (int64_t*)(dsm + (ring - smem_u32(dsm)) + RING * PB);
  volatile int* abort_p = &abort_;  // set by any thread whose wait ran out

  const uint32_t rank = cluster_rank();
  const int hq = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int s = 0; s < RING; ++s) mbar_init(smem_u32(&full[s]), 1);
    fence_barrier_init();
    xneed = 0;
    *abort_p = 0;
  }
  pdl_wait_dep();
  pdl_allow_next();
  const int T = pos[b] + 1;
  const bool bad = T > max_T || T < 1;
  if (bad && rank == 0 && tid == 0) set_error(err, ARCB_ERR_SEQ_OVERFLOW);
  const int npT = bad ? 0 : (T + PAGE - 1) / PAGE;
  const int p0 = npT * (int)rank / CS, p1 = npT * ((int)rank + 1) / CS;
  const int np = p1 - p0;
  const int n = bad ? 0 : max(0, min(T, p1 * PAGE) - min(T, p0 * PAGE));  // local keys
  const int kvh = hq * n_kv / n_heads;
  const int d = n_heads * DH;
  const int* ptb = pt + (size_t)b * pt_stride;
  const int uses = 2 * np;  // K pages then V pages
  int issued = 0;
  auto issue = [&](int u) {  // thread 0 only
    const bool isv = u >= np;
    const int page = ptb[p0 + (isv ? u - np : u)];
    const int64_t* src = (isv ? Vc : Kc) + ((size_t)page * n_kv + kvh) * PAGE * DH;
    const uint32_t bar = smem_u32(&full[u % RING]);
    mbar_arrive_expect_tx(bar, PB);
    bulk_g2s(ring + (u % RING) * PB, src, PB, bar);
  };
  __syncthreads();
  if (tid == 0)
    for (; issued < min(RING, uses); ++issued) issue(issued);
  for (int i = tid; i < EXP_LUT_N; i += NT) lut[i] = g_exp_lut.v[i];
  uint64_t qv[EPL];
#pragma unroll
  for (int i = 0; i < EPL; ++i) qv[i] = bad ? 0 : (uint64_t)q[(size_t)b * d + hq * DH + lane + 32 * i];

  // Waits for ring use u; false once any thread of the CTA gave up.
  auto wait_use = [&](int u) -> bool {
    if (*abort_p) return false;
    if (!mbar_wait(smem_u32(&full[u % RING]), (uint32_t)(u / RING) & 1u)) {
      *abort_p = 1;
      set_error(err, ARCB_ERR_TIMEOUT_FULL);
      return false;
    }
    return true;
  };
  // After every thread has finished with use u's stage, reissue it.
  auto release = [&](int u) {
    __syncthreads();
    if (tid == 0 && issued < uses && !*abort_p) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(issued++);
    }
  };

  // ---- pass 1: scores of the local keys (warp w: keys 4w..4w+3 of each page), local max
  int64_t mx = INT64_MIN;
  for (int pi = 0; pi < np; ++pi) {
    const bool ok = wait_use(pi);
    __syncthreads();
    if (!ok || *abort_p) break;
    const int64_t* kp = (const int64_t*)(dsm + (ring - smem_u32(dsm)) + (pi % RING) * PB);
    uint64_t acc[4];
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const int64_t* row = kp + (warp * 4 + kk) * DH;
      uint64_t a = 0;
#pragma unroll
      for (int i = 0; i < EPL; ++i) a += qv[i] * (uint64_t)row[lane + 32 * i];
      acc[kk] = a;
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint64_t a = warp_sum_u64(acc[kk]);
      const int jj = pi * PAGE + warp * 4 + kk;
      if (jj < n) {
        const int64_t sv = attn_score((int64_t)a, attn_scale);
        if (lane == 0) sc[jj] = sv;
        mx = sv > mx ? sv : mx;
      }
    }
    release(pi);
  }
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  if (tid == 0) {
    int64_t m = red[0];
    for (int w = 1; w < NT / 32; ++w) m = red[w] > m ? red[w] : m;
    xmax = m;
  }
  cluster_sync();
  int64_t gmax = INT64_MIN;
#pragma unroll
  for (int r = 0; r < CS; ++r) {
    const int64_t v = (int64_t)ld_cluster_u64(&xmax, r);
    gmax = v > gmax ? v : gmax;
  }

  // ---- pass 2: exps of the local keys, local sum
  uint64_t sacc = 0;
  for (int jj = tid; jj < n; jj += NT) {
    const int64_t e = integer_exp(wsub(sc[jj], gmax), lut);
    sc[jj] = e;
    sacc += (uint64_t)e;
  }
  sacc = warp_sum_u64(sacc);
  __syncthreads();
  if (lane == 0) red[warp] = (int64_t)sacc;
  __syncthreads();
  if (tid == 0) {
    uint64_t t = 0;
    for (int w = 0; w < NT / 32; ++w) t += (uint64_t)red[w];
    xsum = t;
  }
  cluster_sync();
  uint64_t gs = 0;
#pragma unroll
  for (int r = 0; r < CS; ++r) gs += ld_cluster_u64(&xsum, r);
  const int64_t gsum = (int64_t)gs;

  // ---- pass 3: weights, partial outputs (thread: element tid % DH, keys of parity tid / DH)
  for (int jj = tid; jj < n; jj += NT) {
    int64_t w;
    if (T == 1) w = ONE;
    else if (gsum == 0) w = ONE / T;
    else w = udiv_small(wmul(sc[jj], ONE), gsum);  // e <= gsum: quotient <= ONE
    sc[jj] = w;
  }
  __syncthreads();
  const int e = tid % DH, g = tid / DH;
  uint64_t o = 0;
  for (int pi = 0; pi < np; ++pi) {
    const int u = np + pi;
    const bool ok = wait_use(u);
    __syncthreads();
    if (!ok || *abort_p) break;
    const int64_t* vp = (const int64_t*)(dsm + (ring - smem_u32(dsm)) + (u % RING) * PB);
    const int kmax = min(PAGE, n - pi * PAGE);
#pragma unroll 4
    for (int k = g; k < kmax; k += GROUPS) o += (uint64_t)mulshr(sc[pi * PAGE + k], vp[k * DH + e]);
    release(u);
  }
  part[g][e] = o;
  __syncthreads();
  if (g == 0) {
    uint64_t t = 0;
#pragma unroll
    for (int gg = 0; gg < GROUPS; ++gg) t += part[gg][e];
    xo[e] = t;
  }
  // copies still in flight (only after an abort) must land before the CTA exits
  if (tid == 0)
    for (int u = max(0, issued - RING); u < issued; ++u) mbar_wait(smem_u32(&full[u % RING]), (uint32_t)(u / RING) & 1u);
  cluster_sync();

  // ---- cross-CTA sum of partial outputs; rank r finalises a slice of the head
  constexpr int per = (DH + CS - 1) / CS;
  int need = 0;
  for (int ee = (int)rank * per + tid; ee < min(DH, ((int)rank + 1) * per); ee += NT) {
    uint64_t acc = 0;
#pragma unroll
    for (int r = 0; r < CS; ++r) acc += ld_cluster_u64(&xo[ee], r);
    if (bad) continue;
    const size_t off = (size_t)b * d + hq * DH + ee;
    if (o_out) o_out[off] = (int64_t)acc;
    if (X) {
      int8_t dg[8];
      const int nl = limb_split8((int64_t)acc, dg);
      need = nl > need ? nl : need;
#pragma unroll
      for (int l = 0; l < 8; ++l) X[limb_row(l, b, B) * d + hq * DH + ee] = dg[l];
    }
  }
  need = __reduce_max_sync(0xffffffffu, need);
  if (lane == 0 && need) atomicMax(&xneed, need);
  __syncthreads();
  if (tid == 0 && lmax && xneed) atomicMax(lmax, xneed);
  cluster_sync();  // no CTA may exit while a peer still reads its shared memory
}

template <int CS, int DH>
int launch_paged(const int64_t* q, const int64_t* Kc, const int64_t* Vc, const int* pt, int pt_stride, const int* pos,
                 int n_heads, int n_kv, int64_t attn_scale, int max_T, int B, int8_t* X, int* lmax, int64_t* o_out,
                 int* err, cudaStream_t st) {
  const int max_pages = (max_T + PAGE - 1) / PAGE;
  const size_t smem = 128 + (size_t)RING * PAGE * DH * 8 + (size_t)((max_pages + CS - 1) / CS) * PAGE * 8;
  if (smem > 200 * 1024) return -3;
  static size_t attr = 0;
  if (smem > attr) {
    cudaError_t e = cudaFuncSetAttribute(k_attn_paged<CS, DH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return (int)e;
    attr = smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(CS, n_heads, B);
  cfg.blockDim = dim3(NT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = CS;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = arcb_pdl_enabled();
  cfg.attrs = at;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, k_attn_paged<CS, DH>, q, Kc, Vc, pt, pt_stride, pos, n_heads, n_kv,
                                     attn_scale, max_T, B, X, lmax, o_out, err);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

template <int DH>
int paged_any(const int64_t* q, const int64_t* Kc, const int64_t* Vc, const int* pt, int pt_stride, const int* pos,
              int n_heads, int n_kv, int64_t attn_scale, int max_T, int B, int cluster, int8_t* X, int* lmax,
              int64_t* o_out, int* err, cudaStream_t st) {
  switch (cluster) {
    case 1: return launch_paged<1, DH>(q, Kc, Vc, pt, pt_stride, pos, n_heads, n_kv, attn_scale, max_T, B, X, lmax, o_out, err, st);
    case 2: return launch_paged<2, DH>(q, Kc, Vc, pt, pt_stride, pos, n_heads, n_kv, attn_scale, max_T, B, X, lmax, o_out, err, st);
    case 4: return launch_paged<4, DH>(q, Kc, Vc, pt, pt_stride, pos, n_heads, n_kv, attn_scale, max_T, B, X, lmax, o_out, err, st);
    case 8: return launch_paged<8, DH>(q, Kc, Vc, pt, pt_stride, pos, n_heads, n_kv, attn_scale, max_T, B, X, lmax, o_out, err, st);
  }
  return -2;
}

template <int CS>
int launch(const int64_t* q, const int64_t* Kc, const int64_t* Vc, const int* pt, int pt_stride, const int* pos,
           int n_heads, int n_kv, int dk, int dv, int kst, int vst, int64_t attn_scale, int max_T, int B, int8_t* X, int* lmax,
           int64_t* o_out, int* err, cudaStream_t st) {
  const size_t smem = (size_t)((max_T + CS - 1) / CS + 1) * 8;
  static size_t attr = 0;
  if (smem > attr) {
    cudaError_t e = cudaFuncSetAttribute(k_attn_cluster<CS>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return (int)e;
    attr = smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(CS, n_heads, B);
  cfg.blockDim = dim3(NT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = CS;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = arcb_pdl_enabled();
  cfg.attrs = at;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, k_attn_cluster<CS>, q, Kc, Vc, pt, pt_stride, pos, n_heads, n_kv, dk, dv,
                                     kst, vst, attn_scale, max_T, B, X, lmax, o_out, err);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

}  // namespace

// General form: queries/keys of dk values, values of dv values, cache rows
// of kst / vst int64 (MLA: one shared latent head, dk = r + dr, dv = r,
// V = the first r values of the K rows).
static int attn_any(const int64_t* q, const int64_t* Kc, const int64_t* Vc, const int* pt, int pt_stride,
                    const int* pos, int n_heads, int n_kv, int dk, int dv, int kst, int vst, int64_t attn_scale,
                    int max_T, int B, int cluster, int8_t* X, int* lmax, int64_t* o_out, int* err, cudaStream_t st) {
  if (dk > 640 || dv > 512) return -1;
  switch (cluster) {
    case 1: return launch<1>(q, Kc, Vc, pt, pt_stride, pos, n_heads, n_kv, dk, dv, kst, vst, attn_scale, max_T, B, X, lmax, o_out, err, st);
    case 2: return launch<2>(q, Kc, Vc, pt, pt_stride, pos, n_heads, n_kv, dk, dv, kst, vst, attn_scale, max_T, B, X, lmax, o_out, err, st);
    case 4: return launch<4>(q, Kc, Vc, pt, pt_stride, pos, n_heads, n_kv, dk, dv, kst, vst, attn_scale, max_T, B, X, lmax, o_out, err, st);
    case 8: return launch<8>(q, Kc, Vc, pt, pt_stride, pos, n_heads, n_kv, dk, dv, kst, vst, attn_scale, max_T, B, X, lmax, o_out, err, st);
  }
  return -2;
}

extern "C" int arcb_attn_cluster(const int64_t* q, const int64_t* Kc, const int64_t* Vc, const int* pt,
                                 int pt_stride, const int* pos, int n_heads, int n_kv, int dh, int64_t attn_scale,
                                 int max_T, int B, int cluster, int8_t* X, int* lmax, int64_t* o_out, int* err,
                                 void* stream) {
  const cudaStream_t st = (cudaStream_t)stream;
  const int max_pages = (max_T + PAGE - 1) / PAGE;
  const bool fits = cluster >= 1 && 128 + (size_t)RING * PAGE * dh * 8 +
                                        (size_t)((max_pages + cluster - 1) / cluster) * PAGE * 8 <= 200 * 1024;
  if (arcb_attn_paged_enabled() && fits && (dh == 128 || dh == 64)) {
    if (dh == 128)
      return paged_any<128>(q, Kc, Vc, pt, pt_stride, pos, n_heads, n_kv, attn_scale, max_T, B, cluster, X, lmax,
                            o_out, err, st);
    return paged_any<64>(q, Kc, Vc, pt, pt_stride, pos, n_heads, n_kv, attn_scale, max_T, B, cluster, X, lmax, o_out,
                         err, st);
  }
  return attn_any(q, Kc, Vc, pt, pt_stride, pos, n_heads, n_kv, dh, dh, dh, dh, attn_scale, max_T, B, cluster, X,
                  lmax, o_out, err, st);
}

// Selects the TMA-fed form for standard heads (1, the default) or the plain
// per-thread-load form (0), process-wide; both compute the same values.
static int g_attn_paged = 1;
extern "C" void arcb_set_attn_paged(int on) { g_attn_paged = on; }
int arcb_attn_paged_enabled() { return g_attn_paged; }


extern "C" int arcb_attn_mla(const int64_t* q, const int64_t* cache, const int* pt, int pt_stride, const int* pos,
                             int n_heads, int dk, int dv, int64_t attn_scale, int max_T, int B, int cluster,
                             int64_t* o_out, int* err, void* stream) {
  return attn_any(q, cache, cache, pt, pt_stride, pos, n_heads, 1, dk, dv, dk, dk, attn_scale, max_T, B, cluster,
                  nullptr, nullptr, o_out, err, (cudaStream_t)stream);
}
