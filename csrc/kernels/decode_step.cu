// K13: the whole single-stream decode step (B <= 2) as one persistent,
// cooperative kernel: one CTA per SM runs a program of phases
//   per layer: RMSNorm -> QKV GEMM (RoPE + KV append) -> attention ->
//              W_o GEMM (+ residual, next norm's sum of squares) -> RMSNorm ->
//              gate/up GEMM (SwiGLU + limbs) -> W_down GEMM (+ residual)
//   then the final RMSNorm and the LM head GEMM,
// separated by grid barriers (one arrival counter per phase, zeroed by the
// embedding kernel that precedes the step; bounded waits).
//
// Why: as separate kernels, every GEMM pays a launch, a pipeline ramp and a
// tail during which HBM idles (a new CTA cannot become resident on an SM
// until the previous kernel's CTA there leaves).  Here the TMA producer of
// each CTA streams the weight tiles of all GEMM phases back to back into its
// shared-memory ring; only the small activation tile of a stage waits for
// the barrier that makes its operand ready, so weight streaming continues
// through norms, attention and barriers, up to the ring depth.
//
// Roles (192 threads): warp 0 lane 0 TMA producer (weights run ahead, limb
// tiles after the operand's barrier), warp 1 lane 0 MMA issuer
// (tcgen05.mma kind::i8 into a double-buffered TMEM accumulator), warps 2-5
// the epilogues and the non-GEMM phases.  GEMM arithmetic, epilogue modes and
// split-tile finalisation are the fused GEMM's (fgemm_dev.cuh): every result
// is the same exact integer.
//
// Attention is split over S CTAs per (slot, head) with the exact three-pass
// softmax exchanged through global memory (atomicMax of the scores' max,
// sum of exps, wrapping sum of partial outputs), each pass closed by a
// bounded per-head counter; the last split converts the output to limbs and
// resets the scratch for the next layer.
//
// Failure handling: every wait is bounded (ARCB_WAIT_NS).  A timeout sets an
// error bit; every waiter also gives up as soon as any timeout bit is set,
// so a stuck step ends within one wait bound.  The producer then completes
// the transactions it started, and TMEM is freed before exit.
#include "fgemm_dev.cuh"

using namespace q16;

namespace ds {

using namespace fg;

constexpr int DBN = 16;  // one N tile: 8 limb planes x B <= 2 slots
constexpr int STAGES = 10;
constexpr int A_BYTES = BM * BK;
constexpr int B_BYTES = DBN * BK;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int ACC_COLS = 32;
constexpr int TMEM_COLS = 64;
constexpr int THREADS = 192;
constexpr int ATT_MAX_T = 2048;
constexpr int ABORT_BITS = ARCB_ERR_TIMEOUT_FULL | ARCB_ERR_TIMEOUT_EMPTY | ARCB_ERR_TIMEOUT_DONE |
                           ARCB_ERR_COMM_TIMEOUT;

enum Kind : int { K_NORM = 0, K_GEMM = 1, K_ATTN = 2 };

struct NormP {
  const int64_t* h;
  const unsigned long long* ss;  // [B] sum of squares (Q16) of h
  const int64_t* gamma;
  int ngamma, d, B;
  int8_t* X;  // limb planes [8][B][d]
  int* lmax;
};

struct AttnP {
  const int64_t* q;  // [B, n_heads * dh]
  const int64_t* Kc;
  const int64_t* Vc;
  const int* pt;
  int pt_stride;
  const int* pos;
  int n_heads, n_kv, dh;
  int64_t attn_scale;
  int max_T, B, S;  // S key splits per (slot, head)
  int8_t* X;        // W_o operand limb planes [8][B][n_heads * dh]
  int* lmax;
  // per (slot, head) scratch, reset by the last split: max, sum, outputs [dh], 3 counters
  long long* gmax;
  unsigned long long* gsum;
  unsigned long long* gout;
  int* cnt;
};

struct alignas(64) GemmP {
  CUtensorMap tmA;  // tiled int8 weights, box 128 x 128
  CUtensorMap tmB;  // limb operand, box 16 x 128
  int M, K, B;
  int dep_bar;      // barrier whose completion makes the limb operand ready
  const int* lmax;
  int* tile_cnt;    // per M-tile arrival counters (kept zero between uses)
  Epi E;
};

struct Phase {
  int kind, idx;
};

struct Program {
  int n_phases, n_gemms;
  const Phase* phases;
  const NormP* norms;
  const AttnP* attns;
  const GemmP* gemms;
  int* bar;  // n_phases arrival counters, zero at launch
  int* P;    // split-tile partials
  int* err;
  // optional %globaltimer stamps of CTA 0 [n_phases][2]: phase start (after
  // its barrier), phase end (before arriving)
  unsigned long long* prof;
};

__device__ __forceinline__ int ld_acq(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ bool aborted(const int* err) { return (ld_acq(err) & ABORT_BITS) != 0; }

// Bounded wait for *p >= target; false on timeout (sets `bit`) or when any
// other waiter already timed out.
__device__ bool wait_geq(const int* p, int target, int* err, int bit) {
  if (ld_acq(p) >= target) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0;; ++i) {
    if (ld_acq(p) >= target) return true;
    if ((i & 31) == 31) {
      if (aborted(err)) return false;
      if (globaltimer_ns() - t0 > ARCB_WAIT_NS) {
        set_error(err, bit);
        return false;
      }
      __nanosleep(32);
    }
  }
}

__device__ __forceinline__ void fence_to_async() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// ---------------------------------------------------------------- phases run by the 128 epilogue threads
// t: 0..127 (thread within the epilogue group)

__device__ void run_norm(const NormP& N, int t, int* s_need) {
  const int total = N.B * N.d;
  const int per = (total + gridDim.x - 1) / gridDim.x;
  const int i0 = blockIdx.x * per, i1 = min(total, i0 + per);
  int need = 0;
  for (int i = i0 + t; i < i1; i += 128) {
    const int b = i / N.d, j = i - b * N.d;
    const int64_t inv = rms_inv((int64_t)__ldcg(N.ss + b), N.d);
    const int64_t y = rms_apply(__ldcg(N.h + i), inv, j < N.ngamma ? N.gamma[j] : ONE);
    int8_t dg[8];
    const int n = limb_split8(y, dg);
    need = n > need ? n : need;
    const size_t ps = (size_t)N.B * N.d;
#pragma unroll
    for (int l = 0; l < 8; ++l) N.X[l * ps + i] = dg[l];
  }
  need = __reduce_max_sync(0xffffffffu, need);
  if ((t & 31) == 0 && need) atomicMax(s_need, need);
}

struct AttnSmem {
  int64_t sc[ATT_MAX_T];  // scores -> exps -> weights of this split's keys
  int64_t qs[256];
  unsigned long long o2[2][256];
  long long red[4];
  unsigned long long redu[4];
};

__device__ __forceinline__ uint64_t warp_sum64(uint64_t v) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v += (uint64_t)__shfl_xor_sync(0xffffffffu, (unsigned long long)v, m);
  return v;
}

// One split of one (slot, head).  Returns false when a wait was abandoned.
__device__ bool attn_unit(const AttnP& A, int u, int t, AttnSmem& sm, const int64_t* lut, int* err,
                          int* s_need) {
  const int S = A.S;
  const int bh = u / S, sp = u - bh * S;
  const int b = bh / A.n_heads, hq = bh - b * A.n_heads;
  const int warp = t >> 5, lane = t & 31;
  const int T = A.pos[b] + 1;
  const bool bad = T > A.max_T || T < 1 || T > ATT_MAX_T * S;
  if (bad && sp == 0 && t == 0) set_error(err, ARCB_ERR_SEQ_OVERFLOW);
  const int chunk = bad ? 0 : (T + S - 1) / S;
  const int j0 = min(T, sp * chunk), n = bad ? 0 : max(0, min(T, j0 + chunk) - j0);
  const int dh = A.dh, kvh = hq * A.n_kv / A.n_heads;
  const int* ptb = A.pt + (size_t)b * A.pt_stride;
  auto krow = [&](const int64_t* base, int j) {
    return base + (((size_t)ptb[j / 16] * A.n_kv + kvh) * 16 + (j % 16)) * dh;
  };
  for (int e = t; e < dh; e += 128) sm.qs[e] = bad ? 0 : __ldcg(A.q + (size_t)b * A.n_heads * dh + hq * dh + e);
  asm volatile("bar.sync 2, 128;" ::: "memory");

  // pass 1: scores (4 keys per warp per round), local max
  int64_t mx = LLONG_MIN;
  for (int jj = warp * 4; jj < n; jj += 16) {
    uint64_t acc[4] = {0, 0, 0, 0};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (jj + k < n) {
        const int64_t* kr = krow(A.Kc, j0 + jj + k);
        for (int e = lane; e < dh; e += 32) acc[k] += (uint64_t)sm.qs[e] * (uint64_t)__ldcg(kr + e);
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint64_t s = warp_sum64(acc[k]);
      if (jj + k < n) {
        const int64_t sc = attn_score((int64_t)s, A.attn_scale);
        if (lane == 0) sm.sc[jj + k] = sc;
        mx = sc > mx ? sc : mx;
      }
    }
  }
  if (lane == 0) sm.red[warp] = mx;
  asm volatile("bar.sync 2, 128;" ::: "memory");
  int* cnt = A.cnt + 3 * bh;
  if (t == 0) {
    long long m = sm.red[0];
    for (int w = 1; w < 4; ++w) m = sm.red[w] > m ? sm.red[w] : m;
    if (n > 0) atomicMax(A.gmax + bh, m);
    __threadfence();
    atomicAdd(cnt + 0, 1);
    sm.red[0] = wait_geq(cnt + 0, S, err, ARCB_ERR_TIMEOUT_DONE) ? 1 : 0;
  }
  asm volatile("bar.sync 2, 128;" ::: "memory");
  if (!sm.red[0]) return false;
  const int64_t gmax = __ldcg(A.gmax + bh);

  // pass 2: exps, local sum
  uint64_t s = 0;
  for (int jj = t; jj < n; jj += 128) {
    const int64_t e = integer_exp(wsub(sm.sc[jj], gmax), lut);
    sm.sc[jj] = e;
    s += (uint64_t)e;
  }
  s = warp_sum64(s);
  if (lane == 0) sm.redu[warp] = s;
  asm volatile("bar.sync 2, 128;" ::: "memory");
  if (t == 0) {
    const uint64_t tot = sm.redu[0] + sm.redu[1] + sm.redu[2] + sm.redu[3];
    atomicAdd(A.gsum + bh, (unsigned long long)tot);
    __threadfence();
    atomicAdd(cnt + 1, 1);
    sm.red[0] = wait_geq(cnt + 1, S, err, ARCB_ERR_TIMEOUT_DONE) ? 1 : 0;
  }
  asm volatile("bar.sync 2, 128;" ::: "memory");
  if (!sm.red[0]) return false;
  const int64_t gsum = (int64_t)__ldcg(A.gsum + bh);

  // pass 3: weights, partial outputs (thread: element pair 2*(t%64), key parity t/64)
  for (int jj = t; jj < n; jj += 128) {
    int64_t w;
    if (T == 1) w = ONE;
    else if (gsum == 0) w = ONE / T;
    else w = wmul(sm.sc[jj], ONE) / gsum;
    sm.sc[jj] = w;
  }
  asm volatile("bar.sync 2, 128;" ::: "memory");
  const int e2 = 2 * (t & 63), par = t >> 6;
  uint64_t o0 = 0, o1 = 0;
  if (e2 < dh) {
    int jj = par;
    for (; jj + 14 < n; jj += 16) {
      longlong2 v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = __ldcg((const longlong2*)(krow(A.Vc, j0 + jj + 2 * k) + e2));
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int64_t w = sm.sc[jj + 2 * k];
        o0 += (uint64_t)mulshr(w, v[k].x);
        o1 += (uint64_t)mulshr(w, v[k].y);
      }
    }
    for (; jj < n; jj += 2) {
      const longlong2 v = __ldcg((const longlong2*)(krow(A.Vc, j0 + jj) + e2));
      o0 += (uint64_t)mulshr(sm.sc[jj], v.x);
      o1 += (uint64_t)mulshr(sm.sc[jj], v.y);
    }
  }
  sm.o2[par][e2] = o0;
  sm.o2[par][e2 + 1] = o1;
  asm volatile("bar.sync 2, 128;" ::: "memory");
  unsigned long long* go = A.gout + (size_t)bh * dh;
  for (int e = t; e < dh; e += 128)
    if (n > 0) atomicAdd(go + e, sm.o2[0][e] + sm.o2[1][e]);
  __threadfence();
  asm volatile("bar.sync 2, 128;" ::: "memory");
  if (t == 0) sm.red[1] = (atomicAdd(cnt + 2, 1) == S - 1) ? 1 : 0;
  asm volatile("bar.sync 2, 128;" ::: "memory");
  if (sm.red[1]) {
    // last split: limbs of the output into the W_o operand, reset the scratch
    __threadfence();
    const int d = A.n_heads * dh;
    int need = 0;
    for (int e = t; e < dh; e += 128) {
      const int64_t o = (int64_t)__ldcg(go + e);
      go[e] = 0;
      if (bad) continue;
      int8_t dg[8];
      const int nl = limb_split8(o, dg);
      need = nl > need ? nl : need;
      const size_t off = (size_t)b * d + hq * dh + e;
      const size_t ps = (size_t)A.B * d;
#pragma unroll
      for (int l = 0; l < 8; ++l) A.X[l * ps + off] = dg[l];
    }
    need = __reduce_max_sync(0xffffffffu, need);
    if (lane == 0 && need) atomicMax(s_need, need);
    if (t == 0) {
      A.gmax[bh] = LLONG_MIN;
      A.gsum[bh] = 0;
      cnt[0] = cnt[1] = cnt[2] = 0;
    }
  }
  return true;
}

}  // namespace ds

namespace ds {

// This CTA's item range [it0, it1) of GEMM g (one N tile; stream-K split).
__device__ __forceinline__ void gemm_range(const GemmP& G, int& it0, int& it1, int& mt, int& nch) {
  mt = (G.M + BM - 1) / BM;
  nch = (G.K + BK - 1) / BK;
  const long long total = (long long)mt * nch;
  it0 = (int)(total * blockIdx.x / gridDim.x);
  it1 = (int)(total * (blockIdx.x + 1) / gridDim.x);
}

__global__ void __launch_bounds__(THREADS, 1) k_decode_step(const __grid_constant__ Program Pg) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ AttnSmem asm_;
  __shared__ int64_t lut[EXP_LUT_N];
  __shared__ int s_need, s_ok, s_flag, s_L;
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t a_base = base, b_base = base + STAGES * A_BYTES;
  const uint32_t bar = b_base + STAGES * B_BYTES;
  auto full = [&](int s) { return bar + 8u * s; };
  auto empty = [&](int s) { return bar + 8u * (STAGES + s); };
  auto seg_full = [&](int t) { return bar + 8u * (2 * STAGES + t); };
  auto seg_free = [&](int t) { return bar + 8u * (2 * STAGES + 2 + t); };
  const uint32_t mma_done = bar + 8u * (2 * STAGES + 4);
  const uint32_t tslot = bar + 8u * (2 * STAGES + 5);
  volatile uint32_t* tslot_ptr = (volatile uint32_t*)(smem_raw + (tslot - raw));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* err = Pg.err;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(seg_full(t), 1);
      mbar_init(seg_free(t), 4);
    }
    mbar_init(mma_done, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tslot, TMEM_COLS);
    tmem_relinquish();
  }
  for (int i = threadIdx.x; i < EXP_LUT_N; i += THREADS) lut[i] = g_exp_lut.v[i];
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot_ptr;
  pdl_launch();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer: weight tiles run ahead of the limb tiles
      int ga = 0, ia = 0, ia1 = 0, gb = 0, ib = 0, ib1 = 0, mta = 1, ncha = 1, mtb = 1, nchb = 1;
      auto next_nonempty = [&](int& g, int& i, int& i1, int& mt, int& nch) {
        while (g < Pg.n_gemms) {
          gemm_range(Pg.gemms[g], i, i1, mt, nch);
          if (i < i1) return;
          ++g;
        }
      };
      next_nonempty(ga, ia, ia1, mta, ncha);
      next_nonempty(gb, ib, ib1, mtb, nchb);
      int na = 0, nb = 0;
      bool ready = false, ok = true;
      uint64_t t_idle = 0;
      while (gb < Pg.n_gemms) {
        bool progressed = false;
        if (ga < Pg.n_gemms) {
          const int s = na % STAGES;
          const bool free_ = na < STAGES || mbar_try_wait(empty(s), ((uint32_t)(na / STAGES) & 1u) ^ 1u);
          if (free_) {
            const GemmP& G = Pg.gemms[ga];
            mbar_arrive_expect_tx(full(s), STAGE_BYTES);
            tma_load_2d(a_base + s * A_BYTES, &G.tmA, full(s), 0, ((ia / ncha) % mta * ncha + ia % ncha) * BM);
            ++na;
            if (++ia >= ia1) {
              ++ga;
              next_nonempty(ga, ia, ia1, mta, ncha);
            }
            progressed = true;
          }
        }
        if (nb < na) {
          const GemmP& G = Pg.gemms[gb];
          if (!ready) {
            ready = G.dep_bar < 0 || ld_acq(Pg.bar + G.dep_bar) >= (int)gridDim.x;
            if (ready) fence_to_async();  // the operand's generic writes before this TMA read
          }
          if (ready) {
            const int s = nb % STAGES;
            tma_load_2d(b_base + s * B_BYTES, &G.tmB, full(s), (ib % nchb) * BK, 0);
            ++nb;
            if (++ib >= ib1) {
              ++gb;
              next_nonempty(gb, ib, ib1, mtb, nchb);
              ready = false;
            }
            progressed = true;
          }
        }
        if (progressed) {
          t_idle = 0;
        } else {
          const uint64_t now = globaltimer_ns();
          if (t_idle == 0) t_idle = now;
          if (now - t_idle > ARCB_WAIT_NS) set_error(err, ARCB_ERR_TIMEOUT_EMPTY);
          if (aborted(err)) {
            ok = false;
            break;
          }
          __nanosleep(20);
        }
      }
      if (!ok) {
        // finish every transaction begun: limb tiles of issued stages, then wait
        while (nb < na) {
          const int s = nb % STAGES;
          tma_load_2d(b_base + s * B_BYTES, &Pg.gemms[gb < Pg.n_gemms ? gb : 0].tmB, full(s), 0, 0);
          ++nb;
        }
        for (int i = max(0, na - STAGES); i < na; ++i) mbar_wait(full(i % STAGES), (uint32_t)(i / STAGES) & 1u);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer, all GEMM phases in program order
      int i = 0, seg = 0;
      bool ok = true;
      const uint32_t idesc = idesc_i8(BM, DBN);
      for (int g = 0; g < Pg.n_gemms && ok; ++g) {
        int it0, it1, mt, nch;
        gemm_range(Pg.gemms[g], it0, it1, mt, nch);
        for (int it = it0; it < it1 && ok; ++seg) {
          const int se = min(it1, (it / nch + 1) * nch), tb = seg & 1;
          if (seg >= 2 && !mbar_wait(seg_free(tb), (uint32_t)((seg >> 1) - 1) & 1u)) {
            set_error(err, ARCB_ERR_TIMEOUT_DONE);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t dst = tmem + (uint32_t)(tb * ACC_COLS);
          for (int j = it; j < se; ++j, ++i) {
            const int s = i % STAGES;
            if (!mbar_wait(full(s), (uint32_t)(i / STAGES) & 1u)) {
              set_error(err, ARCB_ERR_TIMEOUT_FULL);
              ok = false;
              break;
            }
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < BK / 32; ++kk) {
              const uint64_t ad = sw128_kmajor_desc(a_base + s * A_BYTES + kk * 32);
              const uint64_t bd = sw128_kmajor_desc(b_base + s * B_BYTES + kk * 32);
              mma_i8(dst, ad, bd, idesc, (j > it || kk > 0) ? 1u : 0u);
            }
            mma_commit(empty(s));
          }
          mma_commit(seg_full(tb));
          it = se;
        }
      }
      // every MMA issued has completed before TMEM can be released
      mma_commit(mma_done);
      mbar_wait(mma_done, 0);
    }
  } else {
    // ---------------- epilogue warps: every phase in program order
    const int t = threadIdx.x - 64, q = warp & 3;
    pdl_wait();
    int seg = 0;
    bool ok = true;
    for (int p = 0; p < Pg.n_phases && ok; ++p) {
      if (t == 0) {
        s_ok = p == 0 || wait_geq(Pg.bar + p - 1, (int)gridDim.x, err, ARCB_ERR_TIMEOUT_DONE);
        s_need = 0;
      }
      epi_bar();
      if (!s_ok) break;
      if (Pg.prof && blockIdx.x == 0 && t == 0) Pg.prof[2 * p] = globaltimer_ns();
      const Phase ph = Pg.phases[p];
      if (ph.kind == K_NORM) {
        const NormP& N = Pg.norms[ph.idx];
        run_norm(N, t, &s_need);
        epi_bar();
        if (t == 0 && s_need) atomicMax(N.lmax, s_need);
      } else if (ph.kind == K_ATTN) {
        const AttnP& A = Pg.attns[ph.idx];
        const int units = A.B * A.n_heads * A.S;
        for (int u = blockIdx.x; u < units && ok; u += gridDim.x) ok = attn_unit(A, u, t, asm_, lut, err, &s_need);
        epi_bar();
        if (t == 0 && s_need) atomicMax(A.lmax, s_need);
      } else {
        const GemmP& G = Pg.gemms[ph.idx];
        const Epi& E = G.E;
        if (t == 0) s_L = max(1, __ldcg(G.lmax));
        epi_bar();
        const int L = s_L, B = G.B, M = G.M;
        int it0, it1, mt_n, nch;
        gemm_range(G, it0, it1, mt_n, nch);
        const int nrows = L * B;
        int need = 0;
        for (int it = it0; it < it1; ++seg) {
          const int se = min(it1, (it / nch + 1) * nch), tb = seg & 1;
          const int mt = (it / nch) % mt_n;
          if (t == 0) s_ok = mbar_wait(seg_full(tb), (uint32_t)(seg >> 1) & 1u) ? 1 : 0;
          epi_bar();
          const bool got = s_ok != 0;
          epi_bar();  // thread 0 rewrites s_ok for the next segment only after every warp has read it
          if (!got) {
            if (t == 0) set_error(err, ARCB_ERR_TIMEOUT_DONE);
            ok = false;
            break;
          }
          tc_fence_after();
          const int m = mt * BM + q * 32 + lane;
          const bool valid = m < M;
          const bool whole = (it % nch == 0) && (se - it == nch);
          const uint32_t taddr = tmem + (uint32_t)(tb * ACC_COLS) + ((uint32_t)(q * 32) << 16);
          if (whole) {
            uint32_t r[16];
            tmem_ld16(taddr, r);
            tmem_ld_wait();
            for (int b = 0; b < B; ++b) {
              uint64_t acc = 0;
#pragma unroll
              for (int l = 0; l < 8; ++l)
                if (l < L) acc += (uint64_t)(int64_t)(int)r[l * B + b] << (8 * l);
              apply_row(E, M, m, valid, b, acc, need);
            }
          } else {
            uint32_t r[16];
            tmem_ld16(taddr, r);
            tmem_ld_wait();
            if (valid) {
#pragma unroll
              for (int j = 0; j < 16; ++j)
                if (j < nrows && r[j] != 0) red_add_s32(Pg.P + (size_t)j * M + m, (int)r[j]);
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(seg_free(tb));
          if (!whole) {
            __threadfence();
            epi_bar();
            if (t == 0) {
              const int add = se - it;
              const int old = atomicAdd(G.tile_cnt + mt, add);
              s_flag = (old + add == nch) ? 1 : 0;
            }
            epi_bar();
            if (s_flag) {
              __threadfence();
              finalize_from_P<DBN>(E, Pg.P, M, m, valid, B, L, need);
              if (t == 0) G.tile_cnt[mt] = 0;
            }
            epi_bar();
          }
          it = se;
        }
        if (E.mode == SWIGLU && E.lmax_out) {
          need = __reduce_max_sync(0xffffffffu, need);
          if (lane == 0 && need > 0) atomicMax(E.lmax_out, need);
        }
      }
      // publish this phase's writes (generic and to the TMA proxy), then arrive
      fence_to_async();
      __threadfence();
      epi_bar();
      if (Pg.prof && blockIdx.x == 0 && t == 0) Pg.prof[2 * p + 1] = globaltimer_ns();
      if (t == 0) atomicAdd(Pg.bar + p, 1);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

constexpr int SMEM_DYN = 1024 + STAGES * STAGE_BYTES + 8 * (2 * STAGES + 5) + 16;

}  // namespace ds

extern "C" {

int arcb_ds_sizes(int* out) {
  out[0] = (int)sizeof(ds::NormP);
  out[1] = (int)sizeof(ds::AttnP);
  out[2] = (int)sizeof(ds::GemmP);
  out[3] = (int)sizeof(ds::Phase);
  out[4] = (int)sizeof(ds::Program);
  out[5] = (int)offsetof(ds::GemmP, E);
  out[6] = (int)sizeof(fg::Epi);
  return 0;
}

// Fills one GEMM phase record (host memory) from two encoded tensor maps and
// an epilogue descriptor.
int arcb_ds_gemm(void* out, const void* tmA, const void* tmB, int M, int K, int B, int dep_bar, const int* lmax,
                 int* tile_cnt, const void* epi) {
  ds::GemmP g;
  memset(&g, 0, sizeof(g));
  memcpy(&g.tmA, tmA, sizeof(CUtensorMap));
  memcpy(&g.tmB, tmB, sizeof(CUtensorMap));
  g.M = M;
  g.K = K;
  g.B = B;
  g.dep_bar = dep_bar;
  g.lmax = lmax;
  g.tile_cnt = tile_cnt;
  g.E = *(const fg::Epi*)epi;
  g.E.B = B;
  memcpy(out, &g, sizeof(g));
  return 0;
}

// Launches the step program (a device copy of Program is taken from host
// memory `prog`).  Cooperative: every CTA must be resident for the barriers.
int arcb_decode_step(const void* prog, void* stream) {
  static int attr = 0;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(ds::k_decode_step, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         ds::SMEM_DYN);
    if (e != cudaSuccess) return (int)e;
    attr = 1;
  }
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  ds::Program P = *(const ds::Program*)prog;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sms);
  cfg.blockDim = dim3(ds::THREADS);
  cfg.dynamicSmemBytes = ds::SMEM_DYN;
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeCooperative;
  at[0].val.cooperative = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = arcb_pdl_enabled();
  cfg.attrs = at;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, ds::k_decode_step, P);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

}  // extern "C"
