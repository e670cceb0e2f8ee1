// Exact causal attention for a prefill chunk: QB consecutive positions of one
// sequence per CTA, every K and V page streamed once for all of them.
//
// Integer semantics per (position, head), as the reference CPU engine
// (crates/arc-inference/src/cached_integer_model.rs:1448-1476,
// softmax_i64 integer_lut.rs:78-100) and the decode kernels: score_j =
// ((q.k_j >> 16) * attn_scale) >> 16 with wrapping i64 dots over keys j <= p;
// w = softmax_i64(scores) (exact max, exact sum of LUT exps, per-term
// (e_j * ONE) / sum); o = sum_j (w_j * v_j) >> 16 rounded per term.  No
// online softmax: all scores of the block stay in shared memory.
//
// Why: the decode kernel run once per position re-reads the whole prefix for
// every position of the chunk (a 1024-position chunk reads each K/V page up
// to 1024 times, times the query heads of a KV head).  Here a page is read
// once per QB positions.
//
// Two modes share the kernel (the block's "queries" read the same pages):
//  * MODE 0, prefill: grid (ceil(B / QB), n_heads).  Slots [0, nq) are the
//    chunk's positions p0, p0 + 1, ... of the sequence whose page-table row
//    is pt[0]; query i of block x is slot x * QB + i of head blockIdx.y;
//    slots [nq, B) (padding) get zero outputs.
//  * MODE 1, grouped-query decode: grid (B, n_kv).  Query i is query head
//    kvh * G + i (G = n_heads / n_kv <= QB) of slot blockIdx.x at position
//    pos[slot], pages pt[slot]: the G heads that share a KV head read each of
//    its pages once, instead of once per head.
// QB * 32 * WM threads: WM warps per query.  Output: limb planes of the W_o
// operand (limb_row layout of B slots) and the limb count (atomicMax).  The
// page ring holds `ring` pages (set per launch from the shared memory the
// scores leave).
//
// Exact int32 fast path: a 64-bit wrapping multiply-add costs about five
// integer instructions.  When the query rows and the K elements a warp reads
// fit in int32, every product fits exactly in int64, so one widening
// multiply-add per element gives the identical wrapping sum.  For V values
// that fit in int32
// the value term runs in 32-bit arithmetic: with v = vh * 2^16 + vl (vh the
// arithmetic high half, 0 <= vl < 2^16) and 0 <= w <= ONE = 2^16,
//   (w * v) >> 16 = w * vh + ((w * vl) >> 16)      (w * vl < 2^32, unsigned)
// and since the weights of one query sum to at most ONE, every partial sum of
// w * vh lies in [-2^31, 2^31) and of ((w * vl) >> 16) in [0, 2^16]: both
// int32 accumulators are exact.  Each warp checks the elements it reads and
// takes the 64-bit form for them otherwise.
#include "common.cuh"
#include "lut.cuh"

using namespace q16;

namespace ap {

constexpr int PAGE = 16;
constexpr int MAX_RING = 8;

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

template <int QB, int DH, int MODE, int WM>
__global__ void __launch_bounds__(QB * 32 * WM) k_attn_block(const int64_t* __restrict__ q, const int64_t* __restrict__ Kc,
                                                        const int64_t* __restrict__ Vc, const int* __restrict__ pt,
                                                        int pt_stride, const int* __restrict__ pos, int nq, int p0,
                                                        int n_heads, int n_kv, int64_t attn_scale, int max_T, int B,
                                                        int RING, int8_t* __restrict__ X, int* __restrict__ lmax,
                                                        int* __restrict__ err) {
  constexpr int NT = QB * 32 * WM;
  constexpr int PB = PAGE * DH * 8;  // one page of one KV head
  extern __shared__ __align__(128) uint8_t dsm[];
  __shared__ int64_t lut[EXP_LUT_N];
  __shared__ __align__(8) uint64_t full[MAX_RING];
  __shared__ int s_need, s_abort;
  __shared__ int cons[MAX_RING], last_use[MAX_RING];  // warps done with a stage; its latest use
  __shared__ int qfit[QB];  // query row fits in int32
  __shared__ int64_t red[WM][QB];
  // softmax passes: warp (wpart, qi) = part wpart of query qi
  const int tid = threadIdx.x, qi = (tid >> 5) % QB, wpart = (tid >> 5) / QB, lane = tid & 31;
  const int G = n_heads / n_kv;
  const int d = n_heads * DH;
  const uint32_t ring = (smem_u32(dsm) + 127u) & ~127u;
  uint8_t* ringp = dsm + (ring - smem_u32(dsm));
  int64_t* qs = (int64_t*)(ringp + RING * PB);  // [QB][DH]
  int64_t* sc = qs + QB * DH;                   // [QB][Tp] scores -> exps -> weights
  if (tid == 0) {
    for (int s = 0; s < RING; ++s) mbar_init(smem_u32(&full[s]), 1);
    fence_barrier_init();
    s_need = 0;
    s_abort = 0;
  }
  if (tid < QB) qfit[tid] = 1;
  if (tid < MAX_RING) cons[tid] = 0, last_use[tid] = -1;
  pdl_wait_dep();
  pdl_allow_next();
  // block geometry: live queries, their slot / head / position, the pages
  int nreal, slot, hq, kvh, pq, Tmax;
  const int* ptb;
  if (MODE == 0) {
    const int s0 = blockIdx.x * QB;
    hq = blockIdx.y;
    kvh = hq / G;
    nreal = max(0, min(QB, nq - s0));
    slot = s0 + qi;
    pq = p0 + s0 + qi;
    Tmax = nreal > 0 ? p0 + s0 + nreal : 0;  // keys of the block's last position
    ptb = pt;
  } else {
    slot = blockIdx.x;
    kvh = blockIdx.y;
    hq = kvh * G + qi;
    nreal = G;
    pq = pos[slot];
    Tmax = pq + 1;
    ptb = pt + (size_t)slot * pt_stride;
  }
  const bool bad = nreal > 0 && (Tmax > max_T || Tmax < 1 || (MODE == 0 && p0 < 0));
  if (bad && tid == 0) set_error(err, ARCB_ERR_SEQ_OVERFLOW);
  const int npg = (nreal > 0 && !bad) ? (Tmax + PAGE - 1) / PAGE : 0;
  const int Tp = npg * PAGE;
  const int uses = 2 * npg;
  auto issue = [&](int u) {  // one thread
    const bool isv = u >= npg;
    const int page = ptb[isv ? u - npg : u];
    const int64_t* src = (isv ? Vc : Kc) + ((size_t)page * n_kv + kvh) * PAGE * DH;
    const uint32_t bar = smem_u32(&full[u % RING]);
    last_use[u % RING] = u;
    mbar_arrive_expect_tx(bar, PB);
    bulk_g2s(ring + (u % RING) * PB, src, PB, bar);
  };
  __syncthreads();
  if (tid == 0)
    for (int u = 0; u < min(RING, uses); ++u) issue(u);
  for (int i = tid; i < EXP_LUT_N; i += NT) lut[i] = g_exp_lut.v[i];
  for (int i = tid; i < QB * DH; i += NT) {
    const int qq = i / DH, e = i - qq * DH;
    const size_t src = MODE == 0 ? (size_t)(blockIdx.x * QB + qq) * d + blockIdx.y * DH + e
                                 : (size_t)blockIdx.x * d + (kvh * G + qq) * DH + e;
    const int64_t v = qq < nreal && !bad ? q[src] : 0;
    qs[i] = v;
    if (v != (int64_t)(int32_t)v) qfit[qq] = 0;
  }
  // Pages are consumed warp by warp, with no block-wide barrier per page:
  // each warp waits for the stage itself (lane 0, bounded), and the last warp
  // to finish with a stage refills it with the use RING ahead.  A timeout
  // sets the abort flag, which every warp checks before its next page.
  constexpr int NW = NT / 32;
  auto wait_page = [&](int u) -> bool {
    if (*(volatile int*)&s_abort) return false;
    int got = 1;
    if (lane == 0) got = mbar_wait(smem_u32(&full[u % RING]), (uint32_t)(u / RING) & 1u) ? 1 : 0;
    got = __shfl_sync(0xffffffffu, got, 0);
    __syncwarp();
    if (!got && lane == 0) {
      s_abort = 1;
      set_error(err, ARCB_ERR_TIMEOUT_FULL);
    }
    return got != 0;
  };
  auto page_done = [&](int u) {
    __syncwarp();
    if (lane == 0) {
      __threadfence_block();  // this warp's reads of the stage come first
      const int st = u % RING;
      if (atomicAdd(&cons[st], 1) == NW - 1) {
        cons[st] = 0;
        if (u + RING < uses && !*(volatile int*)&s_abort) {
          __threadfence_block();
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          issue(u + RING);
        }
      }
    }
  };
  auto fits32 = [](int64_t v) { return v == (int64_t)(int32_t)v; };
  const bool live = qi < nreal && !bad;
  // position of query qq of the block (the last key it attends to)
  auto qpos = [&](int qq) { return MODE == 0 ? p0 + (int)blockIdx.x * QB + qq : pq; };
  // Register-tiled form (int32 pages): thread = (key kk1, slice sl); it holds
  // the slice of every query in registers and reads each K element once for
  // all of them.  S1 = 2 * QB * WM slices per key, EPS elements per slice;
  // after the reduce-scatter LQ lanes hold each query's dot.
  constexpr int S1 = NT / PAGE, EPS = DH / S1, LQ = S1 / QB;
  static_assert(S1 % QB == 0 && S1 <= 32 && EPS >= 1, "slice lanes of a key within one warp");
  const int kk1 = tid / S1, sl = tid % S1;
  __syncthreads();  // qfit complete
  bool qall = true;
  for (int qq = 0; qq < QB; ++qq) qall &= qfit[qq] != 0;
  int qreg[QB][EPS];
#pragma unroll
  for (int qq = 0; qq < QB; ++qq)
#pragma unroll
    for (int i = 0; i < EPS; ++i) qreg[qq][i] = (int)qs[qq * DH + i * S1 + sl];
  // ---- pass 1: scores of keys j <= (position of the query).  Each warp
  // takes its key(s) of the page: 32-bit products when its elements and the
  // query rows fit in int32 (decided per warp), 64-bit products otherwise;
  // the same reduce-scatter either way.
  for (int pi = 0; pi < npg; ++pi) {
    if (!wait_page(pi)) break;
    const int64_t* kr = (const int64_t*)(ringp + (pi % RING) * PB) + kk1 * DH + sl;
    int kv[EPS];
    bool fit = qall;
#pragma unroll
    for (int i = 0; i < EPS; ++i) {
      const int64_t x = kr[i * S1];
      kv[i] = (int)x;
      fit &= fits32(x);
    }
    fit = __all_sync(0xffffffffu, fit);
    uint64_t v[QB];
    if (fit) {
#pragma unroll
      for (int qq = 0; qq < QB; ++qq) {
        int64_t acc = 0;
#pragma unroll
        for (int i = 0; i < EPS; ++i) acc += (int64_t)qreg[qq][i] * (int64_t)kv[i];
        v[qq] = (uint64_t)acc;
      }
    } else {  // 64-bit products, operands re-read from shared memory
#pragma unroll
      for (int qq = 0; qq < QB; ++qq) {
        uint64_t acc = 0;
        for (int i = 0; i < EPS; ++i) acc += (uint64_t)qs[qq * DH + i * S1 + sl] * (uint64_t)kr[i * S1];
        v[qq] = acc;
      }
    }
    // reduce-scatter over the S1 lanes of this key: lane sl ends with the
    // whole dot of query sl / LQ (wrapping sums, exact)
#pragma unroll
    for (int st = 0, m = S1 / 2; m >= 1; ++st, m >>= 1) {
      const int cnt = QB >> st;
      if (cnt > 1) {
        const bool up = (sl & m) != 0;
#pragma unroll
        for (int i = 0; i < cnt / 2; ++i) {
          const uint64_t mine = up ? v[cnt / 2 + i] : v[i];
          const uint64_t other = up ? v[i] : v[cnt / 2 + i];
          v[i] = mine + (uint64_t)__shfl_xor_sync(0xffffffffu, (unsigned long long)other, m);
        }
      } else {
        v[0] += (uint64_t)__shfl_xor_sync(0xffffffffu, (unsigned long long)v[0], m);
      }
    }
    const int qq = sl / LQ, j = pi * PAGE + kk1;
    if (sl % LQ == 0 && qq < nreal && !bad && j <= qpos(qq)) sc[qq * Tp + j] = attn_score((int64_t)v[0], attn_scale);
    page_done(pi);
  }
  __syncthreads();
  bool ok = s_abort == 0;
  // ---- pass 2: exact max and sum of exps per position (WM warps per query,
  // partial results combined through shared memory)
  const int Tq = pq + 1;
  const int j0 = wpart * 32 + lane;
  constexpr int JS = 32 * WM;
  int64_t mx = INT64_MIN;
  if (ok && live)
    for (int jj = j0; jj < Tq; jj += JS) mx = sc[qi * Tp + jj] > mx ? sc[qi * Tp + jj] : mx;
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) {
    const int64_t o2 = (int64_t)__shfl_xor_sync(0xffffffffu, (long long)mx, m);
    mx = o2 > mx ? o2 : mx;
  }
  if (WM > 1) {
    if (lane == 0) red[wpart][qi] = mx;
    __syncthreads();
#pragma unroll
    for (int w = 0; w < WM; ++w) mx = red[w][qi] > mx ? red[w][qi] : mx;
    __syncthreads();
  }
  uint64_t su = 0;
  if (ok && live)
    for (int jj = j0; jj < Tq; jj += JS) {
      const int64_t ex = integer_exp(wsub(sc[qi * Tp + jj], mx), lut);
      sc[qi * Tp + jj] = ex;
      su += (uint64_t)ex;
    }
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) su += (uint64_t)__shfl_xor_sync(0xffffffffu, (unsigned long long)su, m);
  if (WM > 1) {
    if (lane == 0) red[wpart][qi] = (int64_t)su;
    __syncthreads();
    su = 0;
#pragma unroll
    for (int w = 0; w < WM; ++w) su += (uint64_t)red[w][qi];
  }
  const int64_t gsum = (int64_t)su;
  // ---- pass 3: weights in [0, ONE]; zero past each position's last key
  if (ok)
    for (int jj = j0; jj < Tp; jj += JS) {
      int64_t w = 0;
      if (live && jj < Tq) {
        if (Tq == 1) w = ONE;
        else if (gsum == 0) w = ONE / Tq;
        else w = udiv_small(wmul(sc[qi * Tp + jj], ONE), gsum);  // e <= gsum: quotient <= ONE
      }
      sc[qi * Tp + jj] = w;
    }
  // 64-bit partial outputs of pages that do not fit int32: the query rows'
  // area, free after pass 1
  unsigned long long* osl = (unsigned long long*)qs;
  for (int i = tid; i < QB * DH; i += NT) osl[i] = 0;
  __syncthreads();
  // ---- value pass: thread = element slice es (elements es + 32 i), QG
  // queries (qg0 .. qg0 + QG - 1), KPT keys of each page.  Warps whose
  // values fit in int32 use the hi/lo int32 accumulators (exact, see the
  // header); otherwise 64-bit terms added into osl.
  constexpr int EPV = DH / 32, QG = DH == 128 ? 4 : 8, QH = QB / QG, KG = NT / 32 / QH, KPT = PAGE / KG;
  static_assert(QB % QG == 0 && PAGE % KG == 0, "value-pass tiling");
  const int es = tid & 31, rest = tid >> 5, kg = rest / QH, qg0 = (rest % QH) * QG;
  const int* w32 = (const int*)sc;  // weight (qq, j): low word of sc[qq * Tp + j]
  int acch[QG][EPV];
  unsigned accl[QG][EPV];
#pragma unroll
  for (int qq = 0; qq < QG; ++qq)
#pragma unroll
    for (int i = 0; i < EPV; ++i) acch[qq][i] = 0, accl[qq][i] = 0;
  for (int pi = 0; pi < npg && ok; ++pi) {
    const int u = npg + pi;
    if (!wait_page(u)) break;
    const int64_t* vp = (const int64_t*)(ringp + (u % RING) * PB);
    int vv[KPT][EPV];
    bool fit = true;
#pragma unroll
    for (int h = 0; h < KPT; ++h)
#pragma unroll
      for (int i = 0; i < EPV; ++i) {
        const int64_t x = vp[(kg + KG * h) * DH + es + 32 * i];
        vv[h][i] = (int)x;
        fit &= fits32(x);
      }
    fit = __all_sync(0xffffffffu, fit);
#pragma unroll
    for (int h = 0; h < KPT; ++h) {
      const int j = pi * PAGE + kg + KG * h;
      if (fit) {
        int vh[EPV];
        unsigned vl[EPV];
#pragma unroll
        for (int i = 0; i < EPV; ++i) {
          const int v = vv[h][i];
          vh[i] = v >> 16;
          vl[i] = (unsigned)v & 0xffffu;
        }
#pragma unroll
        for (int qq = 0; qq < QG; ++qq) {
          const int w = w32[2 * ((qg0 + qq) * Tp + j)];  // 0 past the position's last key
#pragma unroll
          for (int i = 0; i < EPV; ++i) {
            acch[qq][i] += w * vh[i];
            accl[qq][i] += ((unsigned)w * vl[i]) >> 16;
          }
        }
      } else {
        for (int qq = 0; qq < QG; ++qq) {
          const int64_t w = sc[(qg0 + qq) * Tp + j];
          if (w == 0) continue;
#pragma unroll
          for (int i = 0; i < EPV; ++i)
            atomicAdd(osl + (qg0 + qq) * DH + es + 32 * i,
                      (unsigned long long)mulshr(w, vp[(kg + KG * h) * DH + es + 32 * i]));
        }
      }
    }
    page_done(u);
  }
  __syncthreads();
  ok = ok && s_abort == 0;
  // copies in flight (only after an abort) must land before the CTA exits
  if (tid == 0)
    for (int st = 0; st < RING; ++st)
      if (last_use[st] >= 0) mbar_wait(smem_u32(&full[st]), (uint32_t)(last_use[st] / RING) & 1u);
  // ---- both forms' partial outputs summed in shared memory (the idle ring)
  __syncthreads();
  unsigned long long* osm = (unsigned long long*)ringp;  // [QB][DH]
  for (int i = tid; i < QB * DH; i += NT) osm[i] = 0;
  __syncthreads();
#pragma unroll
  for (int qq = 0; qq < QG; ++qq)
#pragma unroll
    for (int i = 0; i < EPV; ++i) {
      const int64_t t = (int64_t)acch[qq][i] + (int64_t)accl[qq][i];
      if (t) atomicAdd(osm + (qg0 + qq) * DH + es + 32 * i, (unsigned long long)t);
    }
  for (int i = tid; i < QB * DH; i += NT)
    if (osl[i]) atomicAdd(osm + i, osl[i]);
  __syncthreads();
  // ---- limb planes of the W_o operand (zeros for padding slots and dead queries)
  int need = 0;
  for (int i = tid; i < QB * DH; i += NT) {
    const int qq = i / DH, e = i - qq * DH;
    const int sl2 = MODE == 0 ? (int)blockIdx.x * QB + qq : slot;
    const int h2 = MODE == 0 ? hq : kvh * G + qq;
    if (sl2 >= B || (MODE == 1 && qq >= G)) continue;
    int8_t dg[8];
    int nl = 0;
    if (qq < nreal && !bad && ok) nl = limb_split8((int64_t)osm[i], dg);
    else
#pragma unroll
      for (int l = 0; l < 8; ++l) dg[l] = 0;
    need = nl > need ? nl : need;
#pragma unroll
    for (int l = 0; l < 8; ++l) X[limb_row(l, sl2, B) * d + h2 * DH + e] = dg[l];
  }
  need = __reduce_max_sync(0xffffffffu, need);
  if ((tid & 31) == 0 && need) atomicMax(&s_need, need);
  __syncthreads();
  if (tid == 0 && s_need && lmax) atomicMax(lmax, s_need);
}

static size_t smem_bytes(int QB, int DH, int Tp, int ring) {
  return 128 + (size_t)ring * PAGE * DH * 8 + (size_t)QB * DH * 8 + (size_t)QB * Tp * 8;
}

template <int QB, int DH, int MODE, int WM>
int launch(const int64_t* q, const int64_t* Kc, const int64_t* Vc, const int* pt, int pt_stride, const int* pos, int nq,
           int p0, int n_heads, int n_kv, int64_t attn_scale, int max_T, int B, int Tlim, int8_t* X, int* lmax,
           int* err, cudaStream_t st) {
  const int Tp = (Tlim + PAGE - 1) / PAGE * PAGE;
  int ring = MAX_RING;
  while (ring > 2 && smem_bytes(QB, DH, Tp, ring) > 220 * 1024) --ring;
  const size_t smem = smem_bytes(QB, DH, Tp, ring);
  if (smem > 220 * 1024) return -3;
  static size_t attr = 0;
  if (smem > attr) {
    cudaError_t e = cudaFuncSetAttribute(k_attn_block<QB, DH, MODE, WM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return (int)e;
    attr = smem;
  }
  const dim3 grid = MODE == 0 ? dim3((B + QB - 1) / QB, n_heads) : dim3(B, n_kv);
  // a position beyond the score buffer is reported (ARCB_ERR_SEQ_OVERFLOW), never written past it
  const int cap = max_T < Tp ? max_T : Tp;
  return launch_k(k_attn_block<QB, DH, MODE, WM>, grid, dim3(QB * 32 * WM), smem, st, q, Kc, Vc, pt, pt_stride, pos, nq, p0,
                  n_heads, n_kv, attn_scale, cap, B, ring, X, lmax, err);
}

}  // namespace ap

extern "C" {

// Largest key count the block kernel serves with QB queries per CTA.
int arcb_attn_prefill_max_T(int dh, int qb) {
  const int fixed = 128 + 2 * ap::PAGE * dh * 8 + qb * dh * 8;
  return ((220 * 1024 - fixed) / (qb * 8)) / ap::PAGE * ap::PAGE;
}

// Causal attention of a prefill chunk: slots [0, nq) hold positions p0 ..
// p0 + nq - 1 of the sequence whose page table is pt (one row), slots
// [nq, B) are padding (zero outputs).  q: [B, n_heads * dh]; X: W_o limb
// planes of B slots (limb_row layout).  Returns -3 when the chunk's scores
// do not fit in shared memory (the caller then uses the decode kernel).
int arcb_attn_prefill(const int64_t* q, const int64_t* Kc, const int64_t* Vc, const int* pt, int nq, int p0,
                      int n_heads, int n_kv, int dh, int64_t attn_scale, int max_T, int B, int8_t* X, int* lmax,
                      int* err, void* stream) {
  cudaStream_t st = (cudaStream_t)stream;
  if (n_kv <= 0 || n_heads % n_kv) return -2;
  const int T = p0 + nq;
  const bool wide = T <= arcb_attn_prefill_max_T(dh, 16);
  // head dim 128: 8 positions per CTA, two warps per position (16 positions
  // would need more than the 128 registers a 512-thread CTA can have)
  if (dh == 128)
    return ap::launch<8, 128, 0, 2>(q, Kc, Vc, pt, 0, nullptr, nq, p0, n_heads, n_kv, attn_scale, max_T, B, T, X, lmax,
                                    err, st);
  if (dh == 64)
    return wide ? ap::launch<16, 64, 0, 1>(q, Kc, Vc, pt, 0, nullptr, nq, p0, n_heads, n_kv, attn_scale, max_T, B, T, X,
                                        lmax, err, st)
                : ap::launch<8, 64, 0, 1>(q, Kc, Vc, pt, 0, nullptr, nq, p0, n_heads, n_kv, attn_scale, max_T, B, T, X,
                                       lmax, err, st);
  return -2;
}

// Grouped-query decode attention: one CTA per (slot, KV head) serves the
// G = n_heads / n_kv query heads of that KV head (G <= 8), reading each page
// of the slot once.  Scores for up to t_lim keys (the largest position + 1
// of any slot) stay in shared memory; returns -3 when they do not fit.
int arcb_attn_gqa_block(const int64_t* q, const int64_t* Kc, const int64_t* Vc, const int* pt, int pt_stride,
                        const int* pos, int n_heads, int n_kv, int dh, int64_t attn_scale, int max_T, int t_lim, int B,
                        int8_t* X, int* lmax, int* err, void* stream) {
  cudaStream_t st = (cudaStream_t)stream;
  if (n_kv <= 0 || n_heads % n_kv || n_heads / n_kv > 8) return -2;
  if (dh == 128)
    return ap::launch<8, 128, 1, 2>(q, Kc, Vc, pt, pt_stride, pos, 0, 0, n_heads, n_kv, attn_scale, max_T, B, t_lim, X,
                                 lmax, err, st);
  if (dh == 64)
    return ap::launch<8, 64, 1, 2>(q, Kc, Vc, pt, pt_stride, pos, 0, 0, n_heads, n_kv, attn_scale, max_T, B, t_lim, X,
                                lmax, err, st);
  return -2;
}

}  // extern "C"
