// K13: one decode step of a dense INT8 decoder (batch of 1 or 2 slots) as a
// single persistent, cooperative kernel: one CTA per SM runs every layer's
// RMSNorms, QKV / W_o / gate-up / W_down GEMMs and attention, then the final
// norm and the LM head, as a dataflow program.
//
// Why: at batch 1 a decode step streams every weight once (6.6 GB for the
// 7B architecture) and does almost no arithmetic on it, so the step is
// bound by how continuously HBM streams.  As separate kernels, each of the
// ~230 launches pays a ramp and a tail; here each SM's TMA producer streams
// its share of the weight tiles of ALL GEMMs of the step back to back into a
// shared-memory ring, independently of the activations.  Only the small limb
// tile of a stage (the activation operand) waits for its data, and it waits
// on the finest dependency that exists:
//   * QKV, gate/up, LM head: the RMSNorm before them (a grid-wide count);
//   * W_o K chunk c: the attention heads whose outputs form chunk c;
//   * W_down K chunk c: the two gate/up M tiles whose SwiGLU outputs form it.
// Grid-wide waits remain only at the two RMSNorms of a layer (the norm needs
// the sum of squares of the whole hidden vector).  While an SM waits, its
// producer keeps loading the next weight tiles up to the ring depth.
//
// Arithmetic (exact, as the reference CPU engine computes it,
// crates/arc-inference/src/cached_integer_model.rs:1381-1516): activations
// are split into 8 signed radix-256 limb planes; tcgen05.mma kind::i8 gives
// int32 per-limb partial sums in TMEM; a split-K segment recombines its
// limbs into a wrapping u64 (sum_l P_l << 8l) and adds it into the GEMM's u64
// accumulator (the recombination is linear mod 2^64, so adding recombined
// segments equals recombining the summed partials).  The CTA whose arrival
// completes a tile's chunk count finalises it: per-row scale, RoPE + paged
// KV append (QKV), SwiGLU + limb split (gate/up), logits (LM head).  The
// residual GEMMs (W_o, W_down) are finalised by the next RMSNorm: each CTA
// owns a fixed slice of the hidden vector, keeps it in registers for the
// whole step, adds the scaled residual, contributes its sum of squares, and
// after the grid-wide count writes the normalised limb planes of its slice.
// Attention (one CTA per (slot, head), pages streamed by cp.async.bulk
// through a shared-memory ring) uses the exact three-pass integer softmax:
// global max, exact sum of LUT exps, per-term rounded weights.
//
// Tensor parallelism (npeers > 1): W_o and W_down are row-parallel.  The
// CTA that completes a local tile stores its wrapping u64 row sums into this
// rank's slot of every rank's receive buffer (plain stores to peer memory),
// then adds 1 to every rank's arrival counter for the tile; the norm sums the
// npeers slots (exact, order free).  The LM head stores its vocab slice into
// every rank's logits buffer the same way.  No TMA or bulk copy reads peer
// memory; no multicast is used anywhere.
//
// Counters are monotonic: a counter that receives k arrivals per step is
// complete for step e (1, 2, ...) when it reaches k * e, so nothing is reset
// between steps; the step number e lives on the device (the last CTA of a
// step advances it).  Accumulator rows are zeroed by their single reader.
//
// Roles (224 threads): warp 0 lane 0 weight producer; warp 1 lane 0 MMA
// issuer (warp 1 owns TMEM); warps 2-5 epilogues, norms and attention;
// warp 6 lane 0 limb-tile producer (dependency polling).  Every wait is
// bounded (ARCB_WAIT_NS); a timeout sets an error bit, every waiter gives up
// once any timeout bit is set, in-flight copies are completed and TMEM is
// freed before exit.
#include <cstddef>

#include "fgemm_dev.cuh"

using namespace q16;

namespace df {

using fg::BK;
using fg::BM;
using fg::Epi;
using fg::mbar_arrive;

constexpr int BN = 16;  // MMA N: 8 limb planes x up to 2 slots
constexpr int MAXB = 2;
constexpr int A_BYTES = BM * BK;
constexpr int B_BYTES = BN * BK;
constexpr int MAX_STAGES = 12;  // weight ring depth is set per launch from the shared memory left
constexpr int ACC_COLS = 32;
constexpr int TMEM_COLS = 64;
constexpr int THREADS = 224;
constexpr int ARING = 2;
constexpr int PAGE = 16;
constexpr int NORM_PER_THREAD = 4;  // hidden elements (slot, row) owned by one epilogue thread
constexpr int ABORT_BITS = ARCB_ERR_TIMEOUT_FULL | ARCB_ERR_TIMEOUT_EMPTY | ARCB_ERR_TIMEOUT_DONE |
                           ARCB_ERR_COMM_TIMEOUT;

enum { PH_NORM = 0, PH_GEMM = 1, PH_ATTN = 2 };
// DEP_SWIGLU: the limb tile of W_down's chunk c is written into shared
// memory by this CTA's epilogue warps, from the gate/up accumulator rows of
// FFN units [128c, 128c + 128) once their gate/up tiles are complete.
enum { DEP_COUNT = 0, DEP_HEADS = 1, DEP_SWIGLU = 3 };
enum { FIN_APPLY = 0, FIN_NONE = 1, FIN_PUSH = 2 };
enum { SRC_EMBED = 0, SRC_ACC = 1, SRC_PEERS = 2 };

struct alignas(64) GemmD {
  CUtensorMap tmA;  // tiled int8 weights [mt * nch * 128, 128], box 128 x 128
  CUtensorMap tmB;  // limb operand [16, K], box 16 x 128
  int M, K, mt, nch;
  int dep;            // DEP_*: what the limb tile of a chunk waits for
  int dep_dh;         // DEP_HEADS: elements per head
  int dep_n;          // counters in dep_cnt
  unsigned dep_mul;   // a counter is ready at dep_mul * e
  const unsigned* dep_cnt;
  unsigned long long* acc;  // [B][M] split-K accumulator, zero between uses
  unsigned* tile_cnt;       // [mt] chunk arrivals (+nch per step)
  unsigned* tile_fin;       // [mt] finalised (+1 per step); FIN_APPLY, may be null
  int fin;                  // FIN_*
  int rank, npeers;
  long long* const* peer_R;   // FIN_PUSH: every rank's receive buffer [npeers][B][M] of this site
  unsigned* const* peer_arr;  // FIN_PUSH: every rank's per-tile arrivals; FIN_APPLY: one counter per rank
  const uint8_t* wptr;        // the tiled weights (16 KB per tile), for L2 prefetches
  // item order: 0 tile-major (item = mt * nch + kc: a CTA's range is a run
  // of chunks of one or two tiles), 1 chunk-major (item = kc * mt + m: a
  // range is a run of tiles of one or two chunks, so it depends on only
  // those chunks' inputs)
  int kmajor;
  // DEP_SWIGLU: gate/up accumulator [B][src_ld] (rows 2j = gate j, 2j + 1 =
  // up j), its row scales; dep_cnt = its tile counters (dep_n tiles, complete
  // at dep_mul * e chunk arrivals)
  const unsigned long long* src_acc;
  const int64_t* src_scales;
  int src_ld;
  Epi E;
};

struct NormD {
  int src, d, B, npeers;
  const int* tokens;  // SRC_EMBED
  const int8_t* emb;
  const int64_t* emb_s;
  int vocab;
  unsigned long long* acc;  // SRC_ACC: the residual GEMM's accumulator [B][d]
  const unsigned* src_cnt;  // per tile of d: SRC_ACC chunk counts, SRC_PEERS arrivals
  unsigned src_mul;         // ready at src_mul * e
  const long long* R;       // SRC_PEERS: this rank's receive buffer [npeers][B][d]
  const int64_t* scales;    // residual GEMM row scales [d]
  const int64_t* gamma;
  int ngamma;
  unsigned long long* ss;  // [2][G][B] each CTA's partial sum of squares, by step parity
  unsigned* cnt1;          // [NSUB] slices whose partial sum is stored (grid count)
  unsigned* cnt2;          // [NSUB] slices whose limb planes are written (grid count)
  int8_t* X;               // limb planes [16][d] (row l * B + b)
  // an accumulator all of whose readers are done once every CTA has passed
  // this norm's first half (QKV of this layer, or gate/up of the previous
  // one): each CTA zeroes its share of its zero_n u64 for the next step
  unsigned long long* zero_acc;
  int zero_n;
};

struct AttnD {
  // the QKV GEMM's accumulator [B][qkv_M] (rows: q heads, k heads, v heads;
  // q and k rows of a head interleaved as rotation pairs), row scales, tile
  // counters (complete at qkv_mul * e), RoPE tables [max_seq][dh / 2]
  const unsigned long long* qkv_acc;
  const int64_t* qkv_scales;
  const unsigned* qkv_cnt;
  unsigned qkv_mul;
  int qkv_M;
  const int64_t* rcos;
  const int64_t* rsin;
  int64_t* Kc;
  int64_t* Vc;
  const int* pt;
  int pt_stride;
  const int* pos;
  int n_heads, n_kv, dh;
  long long attn_scale;
  int max_T, B;
  int8_t* X;                // W_o limb planes [16][n_heads * dh]
  unsigned* head_done;      // [n_heads] (+B per step)
  // key splits: the S CTAs of a (slot, head) exchange their max, their sum
  // of exps and their partial outputs through per-split slots in global
  // memory (xmax[S], xsum[S], xout[S][dh] per (slot, head)), each round
  // closed by a counter of S arrivals per step
  int S;
  long long* xmax;
  unsigned long long* xsum;
  unsigned long long* xout;
  unsigned* acnt;
};

struct Phase {
  int kind, idx;
};

struct Prog {
  int n_phases, n_gemms, B, max_T;
  const Phase* phases;
  const NormD* norms;
  const GemmD* gemms;
  const AttnD* attns;
  unsigned* epoch;     // completed steps
  unsigned* exit_cnt;  // CTAs finished (G per step)
  int* err;
  const unsigned* lm_arr;  // CTA 0 waits for lm_arr >= lm_mul * e before exit (null: no wait)
  unsigned lm_mul;
  // optional %globaltimer timeline: [G][n_phases][2] phase start / end of
  // every CTA's epilogue group, then [G][n_gemms][4] per GEMM: first weight
  // tile issued, first limb tile issued (its dependency met), first MMA
  // issued, last MMA committed
  unsigned long long* prof;
  // optional per-CTA wait totals in ns [G][8]: 0 weight producer on free
  // stages, 1 limb producer on dependencies, 2 limb producer on free stages,
  // 3 MMA on full stages, 4 epilogue on accumulators, 5 norms' waits,
  // 6 attention (whole units), 7 kernel duration
  unsigned long long* stats;
  int pf_tiles;  // weight tiles the producer keeps requested into L2 ahead of its shared-memory ring
  int stages;    // weight ring depth (set by the launcher)
};

// ---------------------------------------------------------------- helpers
__device__ __forceinline__ unsigned ld_relaxed(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned ld_relaxed_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned ld_poll(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
// Pause between polls of a global counter: hundreds of pollers on one line
// otherwise slow down the very arrivals they wait for.
__device__ __forceinline__ void poll_pause(uint32_t i) { __nanosleep(i < 4 ? 40 : 160); }
__device__ __forceinline__ void fence_acq_rel() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ void fence_to_async() { asm volatile("fence.proxy.async.global;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ bool reached(unsigned v, unsigned target) { return (int)(v - target) >= 0; }
__device__ __forceinline__ bool aborted(const int* err) {
  return (*(volatile const int*)err & ABORT_BITS) != 0;
}
__device__ __forceinline__ unsigned atom_acq_rel_add(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// A grid-wide count is spread over NSUB counters (CTA c arrives on c % NSUB)
// so the arrivals of 148 CTAs do not serialise on one address.
constexpr int NSUB = 8;
__device__ __forceinline__ unsigned sub_target(int j, unsigned e) {
  return (unsigned)(((int)gridDim.x - j + NSUB - 1) / NSUB) * e;
}
__device__ __forceinline__ void grid_arrive(unsigned* cnt) { red_release_add(cnt + blockIdx.x % NSUB, 1u); }
__device__ __forceinline__ bool grid_done(const unsigned* cnt, unsigned e) {
  unsigned v[NSUB];
#pragma unroll
  for (int j = 0; j < NSUB; ++j) v[j] = ld_poll(cnt + j);
  bool ok = true;
#pragma unroll
  for (int j = 0; j < NSUB; ++j) ok &= reached(v[j], sub_target(j, e));
  return ok;
}
// Bounded wait for a grid count (thread-level; acquire on success).
__device__ bool wait_grid(const unsigned* cnt, unsigned e, int* err) {
  uint64_t t0 = 0;
  for (uint32_t i = 0;; ++i) {
    if (grid_done(cnt, e)) {
      fence_acq_rel();
      return true;
    }
    const uint64_t now = globaltimer_ns();
    if (t0 == 0) t0 = now;
    else if (now - t0 > ARCB_WAIT_NS) {
      set_error(err, ARCB_ERR_TIMEOUT_DONE);
      return false;
    }
    if ((i & 7) == 7 && aborted(err)) return false;
    poll_pause(i);
  }
}

__device__ __forceinline__ void red_add_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("red.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Bounded wait until *p reaches target (wrap-safe); acquire on success.
// sys: the counter is written by other GPUs.  Gives up (false) on timeout
// (setting `bit`) or once any other waiter has timed out.
__device__ bool wait_reach(const unsigned* p, unsigned target, int* err, int bit, bool sys = false) {
  uint64_t t0 = 0;
  for (uint32_t i = 0;; ++i) {
    const unsigned v = sys ? ld_relaxed_sys(p) : ld_relaxed(p);
    if (reached(v, target)) {
      if (sys) fence_acq_rel_sys();
      else fence_acq_rel();
      return true;
    }
    if ((i & 7) == 7) {
      if (aborted(err)) return false;
      const uint64_t now = globaltimer_ns();
      if (t0 == 0) t0 = now;
      else if (now - t0 > ARCB_WAIT_NS) {
        set_error(err, bit);
        return false;
      }
    }
    poll_pause(i);
  }
}

// mbarrier wait that also gives up once another waiter timed out.
__device__ bool mwait(uint32_t bar, uint32_t parity, int* err, int bit) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63) == 63) {
      if (aborted(err)) return false;
      if (globaltimer_ns() - t0 > ARCB_WAIT_NS) {
        set_error(err, bit);
        return false;
      }
    }
  }
}

__device__ __forceinline__ void gstamp(const Prog& P, int g, int k) {
  if (P.prof)
    P.prof[(size_t)gridDim.x * P.n_phases * 2 + ((size_t)blockIdx.x * P.n_gemms + g) * 4 + k] = globaltimer_ns();
}

// Item order.  kmajor = 0: tile-major (item = mt * nch + kc).  kmajor = g >
// 0: chunk groups of g chunks, each group tile-major inside (items of group
// q: (mt, q * g + j) for every mt, j < g), so a CTA's range covers a few
// chunks of a few tiles.
__device__ __forceinline__ void item_mk(const GemmD& G, int i, int& mt, int& kc) {
  if (G.kmajor) {
    const int q = i / (G.mt * G.kmajor);
    const int gw = min(G.kmajor, G.nch - q * G.kmajor);  // chunks in this group
    const int r = i - q * G.mt * G.kmajor;
    mt = r / gw;
    kc = q * G.kmajor + (r - mt * gw);
  } else {
    mt = i / G.nch;
    kc = i - mt * G.nch;
  }
}
// End of the segment (run of items of one tile) that starts at item it.
__device__ __forceinline__ int seg_end(const GemmD& G, int it, int i1) {
  if (G.kmajor) {
    const int q = it / (G.mt * G.kmajor);
    const int gw = min(G.kmajor, G.nch - q * G.kmajor);
    const int base = q * G.mt * G.kmajor;
    return min(i1, base + ((it - base) / gw + 1) * gw);
  }
  return min(i1, (it / G.nch + 1) * G.nch);
}
__device__ __forceinline__ int tile_row(const GemmD& G, int i) {
  int mt, kc;
  item_mk(G, i, mt, kc);
  return (mt * G.nch + kc) * BM;
}

__device__ __forceinline__ void range(const GemmD& G, int& i0, int& i1) {
  const long long tot = (long long)G.mt * G.nch;
  i0 = (int)(tot * blockIdx.x / gridDim.x);
  i1 = (int)(tot * (blockIdx.x + 1) / gridDim.x);
}

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

__device__ __forceinline__ uint64_t warp_sum(uint64_t v) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v += (uint64_t)__shfl_xor_sync(0xffffffffu, (unsigned long long)v, m);
  return v;
}

// Counters [c0, c1] that the limb tile of chunk kc of G waits for
// (DEP_HEADS: the attention heads of the chunk).
__device__ __forceinline__ void dep_span(const GemmD& G, int kc, int& c0, int& c1) {
  if (G.dep == DEP_HEADS) {
    c0 = kc * BK / G.dep_dh;
    c1 = min(G.dep_n - 1, (kc * BK + BK - 1) / G.dep_dh);
  } else {
    c0 = c1 = 0;
  }
}

// How many consecutive items from i (at most 8, below i1) have their limb
// dependencies met: every counter of the window is loaded at once (one L2
// round trip), then the ready prefix is counted.
constexpr int DEP_WIN = 8;
__device__ __forceinline__ int deps_ready(const GemmD& G, int i, int i1, unsigned e) {
  const unsigned target = G.dep_mul * e;
  if (G.dep == DEP_COUNT) return grid_done(G.dep_cnt, e) ? DEP_WIN : 0;
  unsigned v[DEP_WIN][2];
#pragma unroll
  for (int w = 0; w < DEP_WIN; ++w) {
    int c0 = 0, c1 = -1;
    if (i + w < i1) {
      int mt_, kc;
      item_mk(G, i + w, mt_, kc);
      dep_span(G, kc, c0, c1);
    }
    v[w][0] = c0 <= c1 ? ld_poll(G.dep_cnt + c0) : target;
    v[w][1] = c0 + 1 <= c1 ? ld_poll(G.dep_cnt + c0 + 1) : target;
  }
  int n = 0;
#pragma unroll
  for (int w = 0; w < DEP_WIN; ++w) {
    if (n == w && i + w < i1 && reached(v[w][0], target) && reached(v[w][1], target)) ++n;
  }
  return n;
}

// ---------------------------------------------------------------- shared state
struct Shared {
  int64_t lut[EXP_LUT_N];
  int64_t qs[128];                  // attention: the head's rotated query
  unsigned long long part[2][128];  // attention: partial outputs per key group
  int64_t red[4];
  unsigned long long redu[4];
  int64_t inv[MAXB];
  int ok, flag;
  volatile int a_issued, b_issued, a_stopped, b_stopped;
  // per ring stage: 1 + the last use whose weight (a) / limb (b) half was provided
  volatile int a_stage[MAX_STAGES], b_stage[MAX_STAGES];
};

// ---------------------------------------------------------------- the epilogue group's phases
// t: thread 0..127 of the epilogue warps; every call is made by all 128.

struct Ctx {
  Shared* sh;
  const Prog* P;
  int* err;
  unsigned e;
  int t, lane, q;  // q: TMEM lane quarter (warp % 4)
  uint32_t tmem;
  uint32_t seg_full0, seg_free0;
  int seg;         // accumulator segments consumed
  uint32_t aring;  // attention ring (shared address)
  uint32_t abar0;  // its barriers
  int64_t* sc;     // attention scores [max_T]
  uint8_t* smem_raw;
  uint32_t raw;
  unsigned au;     // attention ring uses so far
  int ring_n;      // weight-ring uses of the GEMM phases before the current one
  int ns;          // weight ring depth
  int staged[16];  // DEP_SWIGLU: chunk held by each 2 KB staging tile (kc % 16)
  uint32_t full0, empty0, b_base;
  int64_t hreg[NORM_PER_THREAD];  // this thread's slice of the hidden state
  uint64_t w[3];  // thread 0: waits on accumulators, norm waits, attention time (ns)
};

// thread 0 decides, everyone follows
__device__ __forceinline__ bool bcast(Ctx& C, bool v) {
  if (C.t == 0) C.sh->ok = v ? 1 : 0;
  fg::epi_bar();
  const bool r = C.sh->ok != 0;
  fg::epi_bar();
  return r;
}

// Sum over the 4 epilogue warps of per-thread values (result in every thread).
__device__ __forceinline__ uint64_t epi_sum(Ctx& C, uint64_t v, int slot) {
  v = warp_sum(v);
  if (C.lane == 0) C.sh->redu[(C.t >> 5)] = v;
  fg::epi_bar();
  const uint64_t r = C.sh->redu[0] + C.sh->redu[1] + C.sh->redu[2] + C.sh->redu[3];
  fg::epi_bar();
  (void)slot;
  return r;
}

// RMSNorm (cached_integer_model.rs:985-1000) of the hidden state, finalising
// the residual GEMM before it.  CTA c owns rows [r0, r1) of every slot and
// keeps them in registers for the whole step: (1) add the scaled residual
// (or load the embedding), (2) store this slice's sum of squares in its own
// slot, (3) after the grid-wide count, sum the G slots (exact integers),
// (4) write the normalised slice's limb planes and count them.
__device__ bool run_norm(Ctx& C, const NormD& N) {
  const int G = gridDim.x, c = blockIdx.x;
  const int d = N.d, B = N.B;
  const int r0 = (int)((long long)d * c / G), r1 = (int)((long long)d * (c + 1) / G);
  const int rows = r1 - r0, nel = rows * B;
  const unsigned e = C.e;
  const int par = (int)(e & 1u);
  bool ok = true;
  const uint64_t tn0 = C.t == 0 ? globaltimer_ns() : 0;
  if (N.src != SRC_EMBED) {
    if (C.t == 0 && rows > 0) {
      for (int tl = r0 / BM; tl <= (r1 - 1) / BM && ok; ++tl)
        ok = wait_reach(N.src_cnt + tl, N.src_mul * e, C.err, N.src == SRC_PEERS ? ARCB_ERR_COMM_TIMEOUT : ARCB_ERR_TIMEOUT_DONE,
                        N.src == SRC_PEERS);
    }
    if (!bcast(C, ok)) return false;
  }
  if (C.t == 0) C.w[1] += globaltimer_ns() - tn0;
  uint64_t sq[MAXB] = {0, 0};
#pragma unroll
  for (int k = 0; k < NORM_PER_THREAD; ++k) {
    const int idx = C.t + 128 * k;
    if (idx < nel) {
      const int b = idx / rows, m = r0 + (idx - b * rows);
      int64_t hv;
      if (N.src == SRC_EMBED) {
        const unsigned tok = (unsigned)__ldcg(N.tokens + b);
        const int ti = tok >= (unsigned)N.vocab ? N.vocab - 1 : (int)tok;
        hv = wmul((int64_t)N.emb[(size_t)ti * d + m], N.emb_s[ti]);
      } else {
        uint64_t a = 0;
        if (N.src == SRC_ACC) {
          unsigned long long* p = N.acc + (size_t)b * d + m;
          a = __ldcg(p);
          __stcg(p, 0ull);
        } else {
          for (int r = 0; r < N.npeers; ++r) a += (uint64_t)__ldcg(N.R + ((size_t)r * B + b) * d + m);
        }
        hv = wadd(C.hreg[k], mulshr((int64_t)a, N.scales[m]));
      }
      C.hreg[k] = hv;
      const uint64_t s = fg::sq16(hv);
      if (b == 0) sq[0] += s;
      else sq[1] += s;
    }
  }
  unsigned long long* ssp = N.ss + (size_t)par * G * B;
  for (int b = 0; b < B; ++b) {
    const uint64_t s = epi_sum(C, b == 0 ? sq[0] : sq[1], b);
    if (C.t == 0) __stcg(ssp + (size_t)c * B + b, (unsigned long long)s);
  }
  if (C.t == 0) {
    grid_arrive(N.cnt1);
    const uint64_t tn1 = globaltimer_ns();
    ok = wait_grid(N.cnt1, e, C.err);
    C.w[1] += globaltimer_ns() - tn1;
  }
  if (!bcast(C, ok)) return false;
  // the sum of squares of every slot: thread t adds the slots of CTAs t, t + 128
  for (int b = 0; b < B; ++b) {
    uint64_t v = 0;
    for (int cc = C.t; cc < G; cc += 128) v += (uint64_t)__ldcg(ssp + (size_t)cc * B + b);
    v = epi_sum(C, v, b);
    if (C.t == 0) C.sh->inv[b] = rms_inv((int64_t)v, d);
  }
  if (N.zero_acc) {
    const int z0 = (int)((long long)N.zero_n * c / G), z1 = (int)((long long)N.zero_n * (c + 1) / G);
    for (int z = z0 + C.t; z < z1; z += 128) __stcg(N.zero_acc + z, 0ull);
  }
  fg::epi_bar();
#pragma unroll
  for (int k = 0; k < NORM_PER_THREAD; ++k) {
    const int idx = C.t + 128 * k;
    if (idx < nel) {
      const int b = idx / rows, m = r0 + (idx - b * rows);
      const int64_t y = rms_apply(C.hreg[k], C.sh->inv[b], m < N.ngamma ? N.gamma[m] : ONE);
      int8_t dg[8];
      limb_split8(y, dg);
#pragma unroll
      for (int l = 0; l < 8; ++l) N.X[(size_t)(l * B + b) * d + m] = dg[l];
    }
  }
  fence_to_async();
  fg::epi_bar();
  if (C.t == 0) grid_arrive(N.cnt2);
  return true;
}

// Finalises row m of a completed tile (all lanes of the 4 warps together).
__device__ __forceinline__ void finish_rows(Ctx& C, const GemmD& G, int mt, int m, bool valid, const uint64_t* a,
                                            int B) {
  if (G.fin == FIN_APPLY) {
    int need = 0;
    for (int b = 0; b < B; ++b) fg::apply_row(G.E, G.M, m, valid, b, a[b], need);
    fence_to_async();
    if (G.peer_arr) {
      __threadfence_system();
      fg::epi_bar();
      if (C.t == 0)
        for (int p = 0; p < G.npeers; ++p) atomicAdd_system(G.peer_arr[p], 1u);
    } else {
      __threadfence();
      fg::epi_bar();
      if (C.t == 0 && G.tile_fin) atomicAdd(G.tile_fin + mt, 1u);
    }
  } else if (G.fin == FIN_PUSH) {
    if (valid)
      for (int p = 0; p < G.npeers; ++p)
        for (int b = 0; b < B; ++b)
          __stcg(G.peer_R[p] + ((size_t)G.rank * B + b) * G.M + m, (long long)a[b]);
    __threadfence_system();
    fg::epi_bar();
    if (C.t == 0)
      for (int p = 0; p < G.npeers; ++p) atomicAdd_system(G.peer_arr[p] + mt, 1u);
  }
}

// Byte (row r, column c) of a 16-row x 128-byte limb tile in shared memory,
// laid out as a 128-byte-swizzle TMA box writes it (16-byte granule c / 16 of
// row r sits at granule position (c / 16) ^ (r % 8)).
__device__ __forceinline__ uint32_t sw128_off(int r, int c) {
  return (uint32_t)(r * 128 + ((((c >> 4) ^ (r & 7))) << 4) + (c & 15));
}

// DEP_SWIGLU staging: the limb tile of W_down chunk kc (SwiGLU of FFN units
// [128 kc, 128 kc + 128) from the gate/up accumulator, rows 2j = gate j and
// 2j + 1 = up j, split into 8 limb planes, row l * B + b) is built once per
// CTA into one of 16 2 KB staging tiles in the (then idle) attention ring, in the
// 128-byte-swizzled layout a TMA box would have, then copied verbatim into
// the ring stage of every item that uses it.  Thread t: unit t.
__device__ bool swiglu_stage(Ctx& C, const GemmD& G, int kc, uint32_t dst) {
  const int B = C.P->B;
  bool ok = true;
  if (C.t == 0) {
    const int c0 = 2 * kc, c1 = min(G.dep_n - 1, 2 * kc + 1);
    for (int c = c0; c <= c1 && ok; ++c) ok = wait_reach(G.dep_cnt + c, G.dep_mul * C.e, C.err, ARCB_ERR_TIMEOUT_DONE);
  }
  if (!bcast(C, ok)) return false;
  const int u = kc * BK + C.t;  // FFN unit
  const bool live = u < G.K;
  const int64_t gs = live ? G.src_scales[2 * u] : 0, us = live ? G.src_scales[2 * u + 1] : 0;
  uint64_t ga[MAXB], ua[MAXB];
#pragma unroll
  for (int b = 0; b < MAXB; ++b) {
    const bool lb = live && b < B;
    const unsigned long long* ac = G.src_acc + (size_t)b * G.src_ld + 2 * u;
    ga[b] = lb ? __ldcg(ac) : 0;
    ua[b] = lb ? __ldcg(ac + 1) : 0;
  }
  uint8_t* tile = C.smem_raw + (dst - C.raw);
#pragma unroll
  for (int b = 0; b < MAXB; ++b) {
    if (b >= B) break;
    const int64_t y = swiglu(mulshr((int64_t)ga[b], gs), mulshr((int64_t)ua[b], us), C.sh->lut);
    int8_t dg[8];
    limb_split8(y, dg);  // units past K: swiglu(0, 0) = 0
#pragma unroll
    for (int l = 0; l < 8; ++l) tile[sw128_off(l * B + b, C.t)] = (uint8_t)dg[l];
  }
  return true;
}

// Writes the limb tiles of W_down items [i, i + k) (ring uses n .. n + k - 1,
// k <= SW_BATCH) into their stages.
constexpr int SW_BATCH = 8;
__device__ bool swiglu_feed(Ctx& C, const GemmD& G, int i, int k, int n) {
  bool ok = true;
  if (C.t == 0)
    for (int j = 0; j < k && ok; ++j) {
      const int nj = n + j, s = nj % C.ns;
      if (nj >= C.ns) ok = mwait(C.empty0 + 8u * s, ((uint32_t)(nj / C.ns) & 1u) ^ 1u, C.err, ARCB_ERR_TIMEOUT_EMPTY);
    }
  if (!bcast(C, ok)) return false;
  for (int j = 0; j < k; ++j) {
    int mt_, kc;
    item_mk(G, i + j, mt_, kc);
    const int slot = kc & 15;
    if (C.staged[slot] != kc) {
      fg::epi_bar();  // earlier copies out of this staging slot are done
      if (!swiglu_stage(C, G, kc, C.aring + (uint32_t)slot * B_BYTES)) return false;
      C.staged[slot] = kc;
      fg::epi_bar();
    }
    const uint4* src = (const uint4*)(C.smem_raw + (C.aring + (uint32_t)slot * B_BYTES - C.raw));
    uint4* dst = (uint4*)(C.smem_raw + (C.b_base + (uint32_t)((n + j) % C.ns) * B_BYTES - C.raw));
    dst[C.t] = src[C.t];
  }
  fence_async_smem();
  fg::epi_bar();
  if (C.t == 0)
    for (int j = 0; j < k; ++j) {
      const int s = (n + j) % C.ns;
      C.sh->b_stage[s] = n + j + 1;
      mbar_arrive(C.full0 + 8u * s);
    }
  return true;
}

__device__ bool run_gemm(Ctx& C, const GemmD& G) {
  int i0, i1;
  range(G, i0, i1);
  const int B = C.P->B, nch = G.nch;
  const unsigned target = (unsigned)nch * C.e;
  const int ring0 = C.ring_n;
  C.ring_n += i1 - i0;
  int fed = i0;  // DEP_SWIGLU: items whose limb tile is written
  for (int k = 0; k < 16; ++k) C.staged[k] = -1;
  for (int it = i0; it < i1; ++C.seg) {
    const int se = seg_end(G, it, i1), tb = C.seg & 1;
    int mt, kc0;
    item_mk(G, it, mt, kc0);
    if (G.dep == DEP_SWIGLU) {
      // limb tiles of this segment plus a batch ahead, then drain this segment
      const int want = min(i1, max(se, it + SW_BATCH));
      while (fed < want) {
        const int k = min(SW_BATCH, want - fed);
        if (!swiglu_feed(C, G, fed, k, ring0 + (fed - i0))) return false;
        fed += k;
      }
    }
    bool ok = true;
    if (C.t == 0 && !mbar_try_wait(C.seg_full0 + 8u * tb, (uint32_t)(C.seg >> 1) & 1u)) {
      const uint64_t t0 = globaltimer_ns();
      ok = mwait(C.seg_full0 + 8u * tb, (uint32_t)(C.seg >> 1) & 1u, C.err, ARCB_ERR_TIMEOUT_DONE);
      C.w[0] += globaltimer_ns() - t0;
    }
    if (!bcast(C, ok)) return false;
    tc_fence_after();
    const int m = mt * BM + C.q * 32 + C.lane;
    const bool valid = m < G.M;
    uint32_t r[16];
    tmem_ld16(C.tmem + (uint32_t)(tb * ACC_COLS) + ((uint32_t)(C.q * 32) << 16), r);
    tmem_ld_wait();
    uint64_t a[MAXB];
#pragma unroll
    for (int b = 0; b < MAXB; ++b) {
      uint64_t v = 0;
#pragma unroll
      for (int l = 0; l < 8; ++l) v += (uint64_t)(int64_t)(int)r[l * B + b] << (8 * l);
      a[b] = v;
      if (b + 1 >= B) break;
    }
    tc_fence_before();
    __syncwarp();
    if (C.lane == 0) mbar_arrive(C.seg_free0 + 8u * tb);
    const bool whole = kc0 == 0 && se - it == nch;
    if (G.fin == FIN_NONE) {
      // accumulate and signal, without waiting: the consumer finalises
      if (valid)
        for (int b = 0; b < B; ++b) {
          unsigned long long* p = G.acc + (size_t)b * G.M + m;
          if (whole) __stcg(p, (unsigned long long)a[b]);
          else if (a[b]) red_add_u64(p, (unsigned long long)a[b]);
        }
      fg::epi_bar();
      if (C.t == 0) red_release_add(G.tile_cnt + mt, (unsigned)(se - it));
    } else if (whole) {
      finish_rows(C, G, mt, m, valid, a, B);
    } else {
      if (valid)
        for (int b = 0; b < B; ++b)
          if (a[b]) red_add_u64(G.acc + (size_t)b * G.M + m, (unsigned long long)a[b]);
      fg::epi_bar();
      if (C.t == 0) {
        const unsigned add = (unsigned)(se - it);
        const unsigned old = atom_acq_rel_add(G.tile_cnt + mt, add);
        C.sh->flag = (old + add == target) ? 1 : 0;
      }
      fg::epi_bar();
      if (C.sh->flag) {
        if (valid)
          for (int b = 0; b < B; ++b) {
            unsigned long long* p = G.acc + (size_t)b * G.M + m;
            a[b] = __ldcg(p);
            __stcg(p, 0ull);
          }
        finish_rows(C, G, mt, m, valid, a, B);
      }
      fg::epi_bar();
    }
    it = se;
  }
  return true;
}

// One key split `sp` of one (slot, query head): exact attention over the
// paged cache.  The CTA streams the K pages, then the V pages, of its split
// through a shared-memory ring (cp.async.bulk); K pages that do not hold the
// step's new key are requested before the QKV tiles are final.  The S splits
// of a head exchange the global max, the exact sum of exps and their partial
// outputs through global memory; the last arriver writes the output's limb
// planes (W_o operand) and counts the head done.
__device__ bool attn_unit(Ctx& C, const AttnD& A, int b, int hq, int sp, int bh_layer) {
  Shared* sh = C.sh;
  const int t = C.t, ew = t >> 5, lane = C.lane;
  const int dh = A.dh, d = A.n_heads * dh, S = A.S;
  const int kvh = hq / (A.n_heads / A.n_kv);
  const int dq = d, dkv = A.n_kv * dh;
  const int T = __ldcg(A.pos + b) + 1;
  const bool bad = T > A.max_T || T < 1;
  if (bad && t == 0 && sp == 0) set_error(C.err, ARCB_ERR_SEQ_OVERFLOW);
  const int npT = bad ? 0 : (T + PAGE - 1) / PAGE;
  const int p0 = npT * sp / S, p1 = npT * (sp + 1) / S;
  const int np = p1 - p0;
  const int j0 = p0 * PAGE;                                    // first key of the split
  const int n = bad ? 0 : max(0, min(T, p1 * PAGE) - j0);     // keys of the split
  const uint32_t PB = (uint32_t)(PAGE * dh * 8);
  const int* ptb = A.pt + (size_t)b * A.pt_stride;
  const int uses = 2 * np;
  const unsigned u0 = C.au;
  // uses before `early` hold no key or value written this step
  const int newp = (T - 1) / PAGE - p0;  // the split-local page of the new key (if in range)
  const int early = (newp >= 0 && newp < np) ? newp : np;
  int issued = 0;
  auto issue = [&](int u) {
    const bool isv = u >= np;
    const int page = __ldcg(ptb + p0 + (isv ? u - np : u));
    const int64_t* src = (isv ? A.Vc : A.Kc) + ((size_t)page * A.n_kv + kvh) * PAGE * dh;
    const unsigned gu = u0 + (unsigned)u;
    const uint32_t bar = C.abar0 + 8u * (gu % ARING);
    mbar_arrive_expect_tx(bar, PB);
    bulk_g2s(C.aring + (gu % ARING) * PB, src, PB, bar);
  };
  bool ok = true;
  const bool owns_new = early < np;  // this split holds the step's new key and value
  if (t == 0) {
    for (; issued < min(ARING, early); ++issued) issue(issued);
    // the QKV tiles of this head (q) and, for the new key's split, of its KV head
    const int spans[3][2] = {{hq * dh, hq * dh + dh}, {dq + kvh * dh, dq + kvh * dh + dh},
                             {dq + dkv + kvh * dh, dq + dkv + kvh * dh + dh}};
    for (int k = 0; k < (owns_new ? 3 : 1) && ok; ++k)
      for (int tl = spans[k][0] / BM; tl <= (spans[k][1] - 1) / BM && ok; ++tl)
        ok = wait_reach(A.qkv_cnt + tl, A.qkv_mul * C.e, C.err, ARCB_ERR_TIMEOUT_DONE);
  }
  if (!bcast(C, ok)) {
    if (t == 0)
      for (int u = 0; u < issued; ++u) mbar_wait(C.abar0 + 8u * ((u0 + u) % ARING), ((u0 + u) / ARING) & 1u);
    C.au = u0 + (unsigned)uses;
    return false;
  }
  // finalise this head's rows of the QKV GEMM (cached_integer_model.rs:1418-1444):
  // per-row scale, half-split RoPE at the slot's position (rows of a q / k
  // head are interleaved as rotation pairs, so lanes t and t ^ 1 hold a
  // pair), and, in the split that holds the new position, the paged K / V append
  if (!bad && t < dh) {
    const int p = T - 1, half = dh / 2, i = t >> 1, role = t & 1;
    const int e_out = role ? i + half : i;
    const int64_t cs = A.rcos[(size_t)p * half + i], sn = A.rsin[(size_t)p * half + i];
    const unsigned long long* ac = A.qkv_acc + (size_t)b * A.qkv_M;
    auto rot = [&](int m) {
      const int64_t v = mulshr((int64_t)__ldcg(ac + m), A.qkv_scales[m]);
      const int64_t pv = (int64_t)__shfl_xor_sync(0xffffffffu, (long long)v, 1);
      int64_t x0 = role ? pv : v, x1 = role ? v : pv;
      rope_pair(x0, x1, cs, sn);
      return role ? x1 : x0;
    };
    sh->qs[e_out] = rot(hq * dh + t);
    if (owns_new) {
      const int page = __ldcg(ptb + p / PAGE);
      const size_t row = (((size_t)page * A.n_kv + kvh) * PAGE + (p % PAGE)) * dh;
      A.Kc[row + e_out] = rot(dq + kvh * dh + t);
      const int mv = dq + dkv + kvh * dh + t;
      A.Vc[row + t] = mulshr((int64_t)__ldcg(ac + mv), A.qkv_scales[mv]);
      fence_to_async();  // these cache writes before the bulk reads of the page
    }
  } else if (t < dh) {
    sh->qs[t] = 0;
  }
  fg::epi_bar();
  if (t == 0)
    for (; issued < min(ARING, uses); ++issued) issue(issued);
  const int EPL = dh / 32;  // 2 or 4
  uint64_t qv[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) qv[i] = i < EPL ? (uint64_t)sh->qs[lane + 32 * i] : 0;
  auto wait_use = [&](int u) -> bool {
    const unsigned gu = u0 + (unsigned)u;
    bool r = true;
    if (t == 0) r = mwait(C.abar0 + 8u * (gu % ARING), (gu / ARING) & 1u, C.err, ARCB_ERR_TIMEOUT_FULL);
    return bcast(C, r);
  };
  auto release = [&](int u) {
    fg::epi_bar();
    if (t == 0 && issued < uses) {
      fence_async_smem();
      issue(issued++);
    }
  };
  const uint8_t* ring = C.smem_raw + (C.aring - C.raw);
  long long* xmax = A.xmax + (size_t)bh_layer * S;
  unsigned long long* xsum = A.xsum + (size_t)bh_layer * S;
  unsigned long long* xout = A.xout + (size_t)bh_layer * S * dh;
  unsigned* acnt = A.acnt + 3 * bh_layer;
  const unsigned tgt = (unsigned)S * C.e;
  // pass 1: scores (epilogue warp w: keys 4w..4w+3 of each page), local max
  int64_t mx = INT64_MIN;
  for (int pi = 0; pi < np && ok; ++pi) {
    if (!(ok = wait_use(pi))) break;
    const unsigned gu = u0 + (unsigned)pi;
    const int64_t* kp = (const int64_t*)(ring + (gu % ARING) * PB);
    uint64_t acc[4];
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const int64_t* row = kp + (ew * 4 + kk) * dh;
      uint64_t sdot = qv[0] * (uint64_t)row[lane] + qv[1] * (uint64_t)row[lane + 32];
      if (EPL == 4) sdot += qv[2] * (uint64_t)row[lane + 64] + qv[3] * (uint64_t)row[lane + 96];
      acc[kk] = sdot;
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint64_t sdot = warp_sum(acc[kk]);
      const int jj = pi * PAGE + ew * 4 + kk;
      if (jj < n) {
        const int64_t sv = attn_score((int64_t)sdot, A.attn_scale);
        if (lane == 0) C.sc[jj] = sv;
        mx = sv > mx ? sv : mx;
      }
    }
    release(pi);
  }
  int64_t gmx = INT64_MIN, gsm = 0;
  if (ok) {
    // exchange 1: the global max (this split's max in its slot; all S read back)
    if (lane == 0) sh->red[ew] = mx;
    fg::epi_bar();
    if (t == 0) {
      int64_t m4 = sh->red[0];
      for (int w = 1; w < 4; ++w) m4 = sh->red[w] > m4 ? sh->red[w] : m4;
      __stcg(xmax + sp, (long long)m4);
      red_release_add(acnt + 0, 1u);
      ok = wait_reach(acnt + 0, tgt, C.err, ARCB_ERR_TIMEOUT_DONE);
      int64_t g = INT64_MIN;
      if (ok)
        for (int k = 0; k < S; ++k) {
          const int64_t v = (int64_t)__ldcg(xmax + k);
          g = v > g ? v : g;
        }
      sh->red[0] = g;
    }
    ok = bcast(C, ok);
    gmx = sh->red[0];
  }
  if (ok) {
    // pass 2: exps of the split's keys; exchange 2: their exact sum
    uint64_t su = 0;
    for (int jj = t; jj < n; jj += 128) {
      const int64_t ex = integer_exp(wsub(C.sc[jj], gmx), sh->lut);
      C.sc[jj] = ex;
      su += (uint64_t)ex;
    }
    su = warp_sum(su);
    if (lane == 0) sh->redu[ew] = su;
    fg::epi_bar();
    if (t == 0) {
      __stcg(xsum + sp, (unsigned long long)(sh->redu[0] + sh->redu[1] + sh->redu[2] + sh->redu[3]));
      red_release_add(acnt + 1, 1u);
      ok = wait_reach(acnt + 1, tgt, C.err, ARCB_ERR_TIMEOUT_DONE);
      uint64_t g = 0;
      if (ok)
        for (int k = 0; k < S; ++k) g += (uint64_t)__ldcg(xsum + k);
      sh->red[1] = (int64_t)g;
    }
    ok = bcast(C, ok);
    gsm = sh->red[1];
  }
  if (ok) {
    // pass 3: weights
    for (int jj = t; jj < n; jj += 128) {
      int64_t w;
      if (T == 1) w = ONE;
      else if (gsm == 0) w = ONE / T;
      else w = wmul(C.sc[jj], ONE) / gsm;
      C.sc[jj] = w;
    }
    fg::epi_bar();
    // value pass: thread = element t % dh, keys of group t / dh
    const int GROUPS = 128 / dh, el = t % dh, g = t / dh;
    uint64_t o = 0;
    for (int pi = 0; pi < np && ok; ++pi) {
      const int u = np + pi;
      if (!(ok = wait_use(u))) break;
      const unsigned gu = u0 + (unsigned)u;
      const int64_t* vp = (const int64_t*)(ring + (gu % ARING) * PB);
      const int kmax = min(PAGE, n - pi * PAGE);
      for (int k = g; k < kmax; k += GROUPS) o += (uint64_t)mulshr(C.sc[pi * PAGE + k], vp[k * dh + el]);
      release(u);
    }
    sh->part[g][el] = o;
  }
  // copies in flight (only after an abort) must land before the ring is reused or the CTA exits
  if (t == 0)
    for (int u = max(0, issued - ARING); u < issued; ++u) {
      const unsigned gu = u0 + (unsigned)u;
      mbar_wait(C.abar0 + 8u * (gu % ARING), (gu / ARING) & 1u);
    }
  C.au = u0 + (unsigned)uses;  // every thread agrees (after an abort the ring is not used again)
  fg::epi_bar();
  if (!ok) return false;
  // exchange 3: partial outputs in this split's slot; the last split to
  // arrive sums the S slots (exact) and writes the head's limb planes
  if (t < dh) {
    uint64_t o = 0;
    for (int g = 0; g < 128 / dh; ++g) o += sh->part[g][t];
    __stcg(xout + (size_t)sp * dh + t, (unsigned long long)o);
  }
  fg::epi_bar();
  if (t == 0) sh->flag = (atom_acq_rel_add(acnt + 2, 1u) + 1u == tgt) ? 1 : 0;
  fg::epi_bar();
  if (sh->flag) {
    if (t < dh) {
      uint64_t o = 0;
      for (int k = 0; k < S; ++k) o += (uint64_t)__ldcg(xout + (size_t)k * dh + t);
      if (!bad) {
        int8_t dg[8];
        limb_split8((int64_t)o, dg);
#pragma unroll
        for (int l = 0; l < 8; ++l) A.X[(size_t)(l * A.B + b) * d + hq * dh + t] = dg[l];
      }
    }
    fence_to_async();
    fg::epi_bar();
    if (t == 0) red_release_add(A.head_done + hq, 1u);
  }
  return true;
}

__device__ bool run_attn(Ctx& C, const AttnD& A) {
  const int units = A.B * A.n_heads * A.S;
  for (int u = blockIdx.x; u < units; u += gridDim.x) {
    const int bh = u / A.S, sp = u - bh * A.S;
    const int b = bh / A.n_heads, hq = bh - b * A.n_heads;
    const uint64_t ta = C.t == 0 ? globaltimer_ns() : 0;
    if (!attn_unit(C, A, b, hq, sp, bh)) return false;
    if (C.t == 0) C.w[2] += globaltimer_ns() - ta;
  }
  return true;
}

// ---------------------------------------------------------------- the kernel
__global__ void __launch_bounds__(THREADS, 1) k_flow(const __grid_constant__ Prog Pg) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ Shared sh;
  const int NS = Pg.stages;
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t a_base = base;
  const uint32_t b_base = a_base + NS * A_BYTES;
  const uint32_t ar_base = b_base + NS * B_BYTES;
  // attention ring: ARING pages of 16 x dh int64 (dh <= 128)
  const uint32_t sc_base = ar_base + ARING * (PAGE * 128 * 8);
  const uint32_t bar = sc_base + (uint32_t)Pg.max_T * 8u;
  auto full = [&](int s) { return bar + 8u * s; };
  auto empty = [&](int s) { return bar + 8u * (NS + s); };
  const uint32_t seg_full0 = bar + 8u * (2 * NS);
  const uint32_t seg_free0 = seg_full0 + 16u;
  const uint32_t mma_done = seg_free0 + 16u;
  const uint32_t abar0 = mma_done + 8u;
  const uint32_t tslot = abar0 + 8u * ARING;
  volatile uint32_t* tslot_ptr = (volatile uint32_t*)(smem_raw + (tslot - raw));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* err = Pg.err;
  const unsigned e = __ldcg(Pg.epoch) + 1u;
  const uint64_t t_start = globaltimer_ns();

  if (threadIdx.x == 0) {
    // a stage is full once its weight half (TMA) and its limb half (TMA, or
    // the epilogue's shared-memory writes) have both arrived
    for (int s = 0; s < NS; ++s) {
      mbar_init(full(s), 2);
      mbar_init(empty(s), 1);
      sh.a_stage[s] = 0;
      sh.b_stage[s] = 0;
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(seg_full0 + 8u * t, 1);
      mbar_init(seg_free0 + 8u * t, 4);
    }
    mbar_init(mma_done, 1);
    for (int s = 0; s < ARING; ++s) mbar_init(abar0 + 8u * s, 1);
    fence_barrier_init();
    sh.a_issued = 0;
    sh.b_issued = 0;
    sh.a_stopped = 0;
    sh.b_stopped = 0;
  }
  if (warp == 1) {
    tmem_alloc(tslot, TMEM_COLS);
    tmem_relinquish();
  }
  for (int i = threadIdx.x; i < EXP_LUT_N; i += THREADS) sh.lut[i] = g_exp_lut.v[i];
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot_ptr;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- weight producer: every GEMM's tiles of this CTA, back to back
      int n = 0;
      bool ok = true;
      uint64_t w_empty = 0;
      // L2 prefetch cursor: GEMM pg, item pi (of [pi, pi1)), npf items requested
      int pg = 0, pi = 0, pi1 = 0, npf = 0;
      range(Pg.gemms[0], pi, pi1);
      auto pf_next = [&]() {
        while (pg < Pg.n_gemms && pi >= pi1) {
          if (++pg < Pg.n_gemms) range(Pg.gemms[pg], pi, pi1);
        }
        if (pg >= Pg.n_gemms) return false;
        const uint8_t* src = Pg.gemms[pg].wptr + (size_t)tile_row(Pg.gemms[pg], pi) * BK;
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(A_BYTES) : "memory");
        ++pi;
        ++npf;
        return true;
      };
      for (int g = 0; g < Pg.n_gemms && ok; ++g) {
        const GemmD& G = Pg.gemms[g];
        int i0, i1;
        range(G, i0, i1);
        if (g + 1 < Pg.n_gemms) prefetch_tmap(&Pg.gemms[g + 1].tmA);
        for (int i = i0; i < i1; ++i, ++n) {
          while (npf < n + NS + Pg.pf_tiles && pf_next()) {
          }
          const int s = n % NS;
          if (n >= NS && !mbar_try_wait(empty(s), ((uint32_t)(n / NS) & 1u) ^ 1u)) {
            const uint64_t t0 = globaltimer_ns();
            const bool got = mwait(empty(s), ((uint32_t)(n / NS) & 1u) ^ 1u, err, ARCB_ERR_TIMEOUT_EMPTY);
            w_empty += globaltimer_ns() - t0;
            if (!got) {
              ok = false;
              break;
            }
          }
          mbar_arrive_expect_tx(full(s), A_BYTES);
          tma_load_2d(a_base + s * A_BYTES, &G.tmA, full(s), 0, tile_row(G, i));
          if (i == i0) gstamp(Pg, g, 0);
          sh.a_stage[s] = n + 1;
          sh.a_issued = n + 1;
        }
      }
      sh.a_stopped = 1;
      if (Pg.stats) Pg.stats[blockIdx.x * 8 + 0] = w_empty;
    }
  } else if (warp == 6) {
    if (lane == 0) {
      // ---------------- limb-tile producer: waits for each chunk's dependency
      int n = 0;
      bool ok = true;
      uint64_t w_dep = 0, w_empty = 0;
      for (int g = 0; g < Pg.n_gemms && ok; ++g) {
        const GemmD& G = Pg.gemms[g];
        int i0, i1;
        range(G, i0, i1);
        if (G.dep == DEP_SWIGLU) {  // the epilogue warps write these limb tiles
          n += i1 - i0;
          continue;
        }
        if (i0 < i1) prefetch_tmap(&G.tmB);
        int ready_to = i0;  // items [.., ready_to) have their dependencies met
        for (int i = i0; i < i1; ++i, ++n) {
          int mt_, kc;
          item_mk(G, i, mt_, kc);
          if (i >= ready_to) {
            uint64_t t0 = 0;
            for (uint32_t k = 0;; ++k) {
              const int r = deps_ready(G, i, i1, e);
              if (r > 0) {
                ready_to = G.dep == DEP_COUNT ? i1 : i + r;
                break;
              }
              const uint64_t now = globaltimer_ns();
              if (t0 == 0) t0 = now;
              else if (now - t0 > ARCB_WAIT_NS) {
                set_error(err, G.dep == DEP_COUNT ? ARCB_ERR_TIMEOUT_DONE : ARCB_ERR_TIMEOUT_FULL);
                ok = false;
                break;
              }
              if ((k & 7) == 7 && aborted(err)) {
                ok = false;
                break;
              }
              poll_pause(k);
            }
            if (t0) w_dep += globaltimer_ns() - t0;
            if (!ok) break;
            fence_acq_rel();
            fence_to_async();
          }
          const int s = n % NS;
          if (n >= NS && !mbar_try_wait(empty(s), ((uint32_t)(n / NS) & 1u) ^ 1u)) {
            const uint64_t t0 = globaltimer_ns();
            const bool got = mwait(empty(s), ((uint32_t)(n / NS) & 1u) ^ 1u, err, ARCB_ERR_TIMEOUT_EMPTY);
            w_empty += globaltimer_ns() - t0;
            if (!got) {
              ok = false;
              break;
            }
          }
          mbar_arrive_expect_tx(full(s), B_BYTES);
          tma_load_2d(b_base + s * B_BYTES, &G.tmB, full(s), kc * BK, 0);
          if (i == i0) gstamp(Pg, g, 1);
          sh.b_stage[s] = n + 1;
          sh.b_issued = n + 1;
        }
      }
      if (Pg.stats) {
        Pg.stats[blockIdx.x * 8 + 1] = w_dep;
        Pg.stats[blockIdx.x * 8 + 2] = w_empty;
      }
      sh.b_stopped = 1;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer: every GEMM segment in program order
      int n = 0, seg = 0;
      bool ok = true;
      uint64_t w_full = 0;
      const uint32_t idesc = idesc_i8(BM, BN);
      for (int g = 0; g < Pg.n_gemms && ok; ++g) {
        const GemmD& G = Pg.gemms[g];
        int i0, i1;
        range(G, i0, i1);
        for (int it = i0; it < i1 && ok; ++seg) {
          const int se = seg_end(G, it, i1), tb = seg & 1;
          if (seg >= 2 &&
              !mwait(seg_free0 + 8u * tb, (uint32_t)((seg >> 1) - 1) & 1u, err, ARCB_ERR_TIMEOUT_DONE)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t dst = tmem + (uint32_t)(tb * ACC_COLS);
          for (int j = it; j < se; ++j, ++n) {
            const int s = n % NS;
            if (!mbar_try_wait(full(s), (uint32_t)(n / NS) & 1u)) {
              const uint64_t t0 = globaltimer_ns();
              const bool got = mwait(full(s), (uint32_t)(n / NS) & 1u, err, ARCB_ERR_TIMEOUT_FULL);
              w_full += globaltimer_ns() - t0;
              if (!got) {
                ok = false;
                break;
              }
            }
            tc_fence_after();
            if (j == i0) gstamp(Pg, g, 2);
#pragma unroll
            for (int kk = 0; kk < BK / 32; ++kk) {
              const uint64_t ad = sw128_kmajor_desc(a_base + s * A_BYTES + kk * 32);
              const uint64_t bd = sw128_kmajor_desc(b_base + s * B_BYTES + kk * 32);
              mma_i8(dst, ad, bd, idesc, (j > it || kk > 0) ? 1u : 0u);
            }
            mma_commit(empty(s));
          }
          if (!ok) break;
          mma_commit(seg_full0 + 8u * tb);
          it = se;
        }
        if (i1 > i0) gstamp(Pg, g, 3);
      }
      mma_commit(mma_done);
      mbar_wait(mma_done, 0);
      if (Pg.stats) Pg.stats[blockIdx.x * 8 + 3] = w_full;
    }
  } else {
    // ---------------- epilogue group (warps 2..5): every phase in program order
    Ctx C;
    C.sh = &sh;
    C.P = &Pg;
    C.err = err;
    C.e = e;
    C.t = threadIdx.x - 64;
    C.lane = lane;
    C.q = warp & 3;
    C.tmem = tmem;
    C.seg_full0 = seg_full0;
    C.seg_free0 = seg_free0;
    C.seg = 0;
    C.aring = ar_base;
    C.abar0 = abar0;
    C.sc = (int64_t*)(smem_raw + (sc_base - raw));
    C.smem_raw = smem_raw;
    C.raw = raw;
    C.au = 0;
    C.ring_n = 0;
    C.ns = NS;
    C.full0 = bar;
    C.empty0 = bar + 8u * NS;
    C.b_base = b_base;
#pragma unroll
    for (int k = 0; k < NORM_PER_THREAD; ++k) C.hreg[k] = 0;
    C.w[0] = C.w[1] = C.w[2] = 0;
    for (int p = 0; p < Pg.n_phases; ++p) {
      if (Pg.prof && C.t == 0) Pg.prof[((size_t)blockIdx.x * Pg.n_phases + p) * 2] = globaltimer_ns();
      const Phase ph = Pg.phases[p];
      bool ok;
      if (ph.kind == PH_NORM) ok = run_norm(C, Pg.norms[ph.idx]);
      else if (ph.kind == PH_GEMM) ok = run_gemm(C, Pg.gemms[ph.idx]);
      else ok = run_attn(C, Pg.attns[ph.idx]);
      if (Pg.prof && C.t == 0) Pg.prof[((size_t)blockIdx.x * Pg.n_phases + p) * 2 + 1] = globaltimer_ns();
      if (!ok) break;
    }
    if (Pg.lm_arr && blockIdx.x == 0 && C.t == 0)
      wait_reach(Pg.lm_arr, Pg.lm_mul * e, err, ARCB_ERR_COMM_TIMEOUT, true);
    if (Pg.stats && C.t == 0) {
      Pg.stats[blockIdx.x * 8 + 4] = C.w[0];
      Pg.stats[blockIdx.x * 8 + 5] = C.w[1];
      Pg.stats[blockIdx.x * 8 + 6] = C.w[2];
      Pg.stats[blockIdx.x * 8 + 7] = globaltimer_ns() - t_start;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && aborted(err)) {
    // After an abort, complete every ring stage that has a copy in flight,
    // so nothing lands in shared memory after the CTA exits: the missing
    // half of a stage is filled by a dummy copy (its contents are unused).
    int nm = 0;
    for (int s2 = 0; s2 < NS; ++s2) nm = max(nm, max(sh.a_stage[s2], sh.b_stage[s2]));
    for (int u = max(0, nm - NS); u < nm; ++u) {
      const int s2 = u % NS;
      const bool has_a = sh.a_stage[s2] == u + 1, has_b = sh.b_stage[s2] == u + 1;
      if (!has_a && !has_b) continue;
      if (!has_a) {
        mbar_arrive_expect_tx(full(s2), A_BYTES);
        tma_load_2d(a_base + s2 * A_BYTES, &Pg.gemms[0].tmA, full(s2), 0, 0);
      }
      if (!has_b) {
        mbar_arrive_expect_tx(full(s2), B_BYTES);
        tma_load_2d(b_base + s2 * B_BYTES, &Pg.gemms[0].tmB, full(s2), 0, 0);
      }
      mbar_wait(full(s2), (uint32_t)(u / NS) & 1u);
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned old = atomicAdd(Pg.exit_cnt, 1u);
    if (old + 1u == gridDim.x * e) atomicExch(Pg.epoch, e);
  }
}

}  // namespace df

extern "C" {

// Record sizes and field offsets for the host-side mirrors.
int arcb_flow_layout(int* out) {
  out[0] = (int)sizeof(df::NormD);
  out[1] = (int)sizeof(df::AttnD);
  out[2] = (int)sizeof(df::GemmD);
  out[3] = (int)sizeof(df::Phase);
  out[4] = (int)sizeof(df::Prog);
  out[5] = (int)offsetof(df::GemmD, E);
  out[6] = (int)sizeof(fg::Epi);
  out[7] = df::MAX_STAGES;
  out[8] = df::ARING;
  out[9] = df::NORM_PER_THREAD;
  return 0;
}

// Fills one GEMM record (host memory, 64-byte aligned) of the step program.
int arcb_flow_gemm(void* out, const void* tmA, const void* tmB, int M, int K, int dep, int dep_dh, int dep_n,
                   unsigned dep_mul, const unsigned* dep_cnt, unsigned long long* acc, unsigned* tile_cnt,
                   unsigned* tile_fin, int fin, int rank, int npeers, long long* const* peer_R,
                   unsigned* const* peer_arr, const void* epi, int B, const void* wptr, const void* src_acc,
                   const void* src_scales, int src_ld, int kmajor) {
  if ((uintptr_t)out & 63) return -1;
  df::GemmD g;
  memset(&g, 0, sizeof(g));
  memcpy(&g.tmA, tmA, sizeof(CUtensorMap));
  memcpy(&g.tmB, tmB, sizeof(CUtensorMap));
  g.M = M;
  g.K = K;
  g.mt = (M + fg::BM - 1) / fg::BM;
  g.nch = (K + fg::BK - 1) / fg::BK;
  g.dep = dep;
  g.dep_dh = dep_dh;
  g.dep_n = dep_n;
  g.dep_mul = dep_mul;
  g.dep_cnt = dep_cnt;
  g.acc = acc;
  g.tile_cnt = tile_cnt;
  g.tile_fin = tile_fin;
  g.fin = fin;
  g.rank = rank;
  g.npeers = npeers;
  g.peer_R = peer_R;
  g.peer_arr = peer_arr;
  g.wptr = (const uint8_t*)wptr;
  g.src_acc = (const unsigned long long*)src_acc;
  g.src_scales = (const int64_t*)src_scales;
  g.src_ld = src_ld;
  g.kmajor = kmajor;
  if (epi) g.E = *(const fg::Epi*)epi;
  g.E.B = B;
  memcpy(out, &g, sizeof(g));
  return 0;
}

static int flow_dyn_smem(int ns, int max_T) {
  return 1024 + ns * (df::A_BYTES + df::B_BYTES) + df::ARING * df::PAGE * 128 * 8 + max_T * 8 +
         8 * (2 * ns + 5 + df::ARING) + 64;
}

// Weight ring depth for an attention capacity: as many 18 KB stages as the
// 227 KB of shared memory per block leaves (at most MAX_STAGES).
int arcb_flow_stages(int max_T) {
  cudaFuncAttributes fa;
  if (cudaFuncGetAttributes(&fa, df::k_flow) != cudaSuccess) return -1;
  int ns = df::MAX_STAGES;
  while (ns > 2 && flow_dyn_smem(ns, max_T) + (int)fa.sharedSizeBytes > 227 * 1024) --ns;
  return ns;
}

// Dynamic shared memory of the step kernel for an attention capacity.
int arcb_flow_smem(int max_T) {
  const int ns = arcb_flow_stages(max_T);
  return ns < 0 ? ns : flow_dyn_smem(ns, max_T);
}

// Launches one step (a copy of the Prog record is taken from host memory).
// Cooperative: every CTA (one per SM) must be resident.
int arcb_flow_launch(const void* prog, void* stream) {
  df::Prog P = *(const df::Prog*)prog;
  P.stages = arcb_flow_stages(P.max_T);
  if (P.stages < 4) return -2;
  const int smem = flow_dyn_smem(P.stages, P.max_T);
  static int attr = 0;
  if (smem > attr) {
    cudaError_t e = cudaFuncSetAttribute(df::k_flow, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return (int)e;
    attr = smem;
  }
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sms);
  cfg.blockDim = dim3(df::THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, df::k_flow, P);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

}  // extern "C"
