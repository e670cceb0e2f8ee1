// K1 (fused): persistent stream-K int8 x int64 limb GEMM with the finalize
// fused into the epilogue.  Same exact arithmetic as gemm_i8.cu (signed
// radix-256 limb planes, tcgen05.mma kind::i8, s32 partials in TMEM); what
// changes is the schedule and what happens after the MMA:
//
//  * Persistent: one CTA per SM.  The work list is every (n-tile, m-tile,
//    128-byte K chunk) item; CTA c takes a contiguous, balanced range of it,
//    so the TMA stream of weights never drains between tiles and no SM idles
//    (stream-K).  A range is cut into segments (runs of one (n, m) tile); each
//    segment accumulates into one of two TMEM buffers, so the epilogue of a
//    segment overlaps the MMAs of the next.
//  * Fused finalize: a segment that covers a whole tile finalizes straight
//    from TMEM; otherwise it adds its int32 partials into P (red.global.add)
//    and the CTA whose arrival completes the tile's counter finalizes from P
//    (integer adds: order free, exact) and zeroes what it read.
//  * Epilogue modes: store (LM head), residual add + next-norm sum of squares
//    (W_o, W_down), RoPE + paged KV append (QKV, rows of a head interleaved as
//    (e, e + d_head/2) pairs so a lane pair holds a rotation pair), SwiGLU +
//    limb split for the next GEMM (gate/up rows interleaved), partial-only
//    (tensor-parallel partials reduced by the caller).
//  * Programmatic dependent launch: the producer issues the first weight
//    tiles before griddepcontrol.wait, so weights stream in while the
//    previous kernel (norm, attention) is still finishing.
//
// Warp roles (192 threads): warp 0 lane 0 TMA producer, warp 1 lane 0 MMA
// issuer (warp 1 owns the TMEM allocation), warps 2-5 epilogue (TMEM lane
// quarter = warp % 4).  All waits are bounded (common.cuh).
#include <climits>

#include "common.cuh"
#include "lut.cuh"

using namespace q16;

namespace fg {

constexpr int BM = 128;
constexpr int BK = 128;
constexpr int NTHREADS = 192;
// Q4 tiles (group-32 4-bit weights): 128 rows x 64 bytes of nibbles (low
// nibble = even column, value = nibble - 8) then 128 rows x 2 bytes of 4-bit
// group multipliers (group g of the 128-column chunk in bits 4g..4g+3).
constexpr int Q4_TILE = 128 * 64 + 128 * 2;
constexpr int PAGE = 16;

enum Mode : int { PARTIAL = 0, STORE = 1, RESID = 2, QKV = 3, SWIGLU = 4, MOE_COMBINE = 5 };

struct Epi {
  int mode;
  const int64_t* scales;  // per fused row
  int64_t* out;           // STORE / RESID target [B, ldo]
  int ldo;
  unsigned long long* ss_out;  // RESID: next norm's sum of squares per slot
  // QKV
  int n_heads, n_kv, dh;
  int64_t* q_out;
  int64_t* Kc;
  int64_t* Vc;
  const int* pt;
  int pt_stride;
  const int* pos;
  const int64_t* rcos;
  const int64_t* rsin;
  int max_seq;
  // SWIGLU: limb planes of the next GEMM's operand [8][B][ldx]
  int8_t* X;
  int ldx;
  int* lmax_out;
  int* err;
  int B;  // slots in the step (plane stride of X = B * ldx)
  // Tensor-parallel push mode (rp = 1): partials go to every rank's P over
  // NVLink (peer pointers of a symmetric allocation), arrivals to every
  // rank's per-tile counters; tile mt is finalised on each rank by its CTA
  // mt % gridDim.x once all ranks' chunks have arrived.
  int rp;
  int npeers;
  int* const* peer_P;
  int* const* peer_cnt;
  int* const* peer_lmax;
  int* cnt_local;
  int* lmax_fin;
  // optional per-CTA %globaltimer stamps [grid][8]: 0 entry, 1 after the
  // dependency wait, 2 first stage consumed, 3 last MMA issued, 4 epilogue
  // done, 5 finaliser done, 6 exit
  unsigned long long* prof;
  // Grouped (MoE) GEMMs over stacked experts: rows come in groups of
  // grp_rows per expert; grp_koff > 0 makes group g read operand columns
  // [g * grp_koff, g * grp_koff + K) (each expert's own intermediate).
  int grp_rows;
  int grp_koff;
  // MOE_COMBINE: h[b, i] += (route[b, g] * y) >> 16 for routed experts.
  const int64_t* route;
  int route_ld;
  // Upper bound on persistent CTAs (0 = one per SM).  Fewer CTAs means
  // fewer CTAs share a tile, so less partial-sum traffic at larger batch.
  int max_ctas;
  // Rows per TMA box of the limb operand's tensor map (0 = BN).  With a box
  // smaller than BN only the boxes that hold live rows (limbs x slots) are
  // loaded, so a batch whose activations need few limbs does not stream the
  // unused limb planes.
  int b_box;
  // Expert parallelism: MOE_COMBINE reads route column g * route_gs of
  // local group g (route points at this rank's first expert column;
  // 0 = stride 1) and, with peer_h set, adds into the npeers targets
  // peer_h[p] (every rank's combine buffer) instead of out; with peer_sig
  // set every CTA, once its adds are fenced, increments every rank's
  // arrival counter peer_sig[p] by one.
  int route_gs;
  int64_t* const* peer_h;
  unsigned long long* const* peer_sig;
  // Cross-GEMM prefetch: once this CTA's producer has issued its last load,
  // it asks L2 for the first pf_tiles weight tiles that the same CTA index
  // will stream in the next GEMM (tiled int8 weights pf_w of [pf_M, pf_K],
  // one N tile, the same grid), so HBM stays busy through this GEMM's tail
  // and the next GEMM's first stages hit L2.  null = off.
  const uint8_t* pf_w;
  int pf_M, pf_K, pf_tiles;
};

// Ring depth for decode-sized tiles (BN <= 32).  A 5-stage ring (two CTAs
// per SM, so the next GEMM could prefetch during this one's tail) measured
// slower on the 7B decode (3.31 vs 3.15 ms/token): the deep ring wins.
#ifndef ARCB_FG_SMALL_STAGES
#define ARCB_FG_SMALL_STAGES 11
#endif

template <int BN, bool Q4 = false>
struct Cfg {
  static constexpr int A_BYTES = BM * BK;
  static constexpr int B_BYTES = BN * BK;
  static constexpr int Q_BYTES = Q4 ? Q4_TILE : 0;        // staging of the packed Q4 tile
  static constexpr int STAGE_BYTES = (Q4 ? Q4_TILE : A_BYTES) + B_BYTES;  // bytes TMA brings per stage
  static constexpr int STAGES = Q4 ? (BN <= 32 ? 7 : (BN <= 64 ? 6 : (BN <= 128 ? 5 : 3)))
                                   : (BN <= 32 ? ARCB_FG_SMALL_STAGES : (BN <= 64 ? 8 : (BN <= 128 ? 6 : 4)));
  static constexpr int ACC_COLS = BN < 32 ? 32 : BN;       // one TMEM accumulator
  static constexpr int TMEM_COLS = 2 * ACC_COLS;          // double buffered
  static constexpr int THREADS = Q4 ? 320 : NTHREADS;     // + 4 converter warps for Q4
  static constexpr int SMEM = 1024 + STAGES * (A_BYTES + B_BYTES + Q_BYTES) + 512;
};

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" :::); }
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld1(uint32_t taddr, uint32_t& r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(taddr));
}

__device__ __forceinline__ uint64_t sq16(int64_t x) { return (uint64_t)(wmul(x, x) >> FRAC_BITS); }

__device__ __forceinline__ uint64_t warp_sum_u64(uint64_t v) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v += (uint64_t)__shfl_xor_sync(0xffffffffu, (unsigned long long)v, m);
  return v;
}

// Applies the epilogue to output row m (fused-row index) of slot b, given the
// recombined wrapping accumulator acc = sum_k W[m,k] x_b[k].  Called by all 32
// lanes of a warp together (rows m0..m0+31) so pair exchanges can shuffle.
__device__ __forceinline__ void apply_row(const Epi& E, int M, int m, bool valid, int b, uint64_t acc,
                                          int& need) {
  const int64_t s = valid ? E.scales[m] : 0;
  const int64_t v = mulshr((int64_t)acc, s);
  const int lane = threadIdx.x & 31;
  switch (E.mode) {
    case STORE:
      if (valid) E.out[(size_t)b * E.ldo + m] = v;
      break;
    case RESID: {
      uint64_t sq = 0;
      if (valid) {
        int64_t* o = E.out + (size_t)b * E.ldo + m;
        const int64_t r = wadd(*o, v);
        *o = r;
        sq = sq16(r);
      }
      if (E.ss_out) {
        sq = warp_sum_u64(sq);
        if (lane == 0) atomicAdd(E.ss_out + b, (unsigned long long)sq);
      }
      break;
    }
    case QKV: {
      const int d = E.n_heads * E.dh, dkv = E.n_kv * E.dh, half = E.dh / 2;
      const int64_t partner = (int64_t)__shfl_xor_sync(0xffffffffu, (long long)v, 1);
      if (!valid) break;
      const int p = E.pos[b];
      if (p < 0 || p >= E.max_seq) {
        set_error(E.err, ARCB_ERR_SEQ_OVERFLOW);
        break;
      }
      const int page = E.pt[(size_t)b * E.pt_stride + p / PAGE];
      const int slot = p % PAGE;
      if (m < d + dkv) {
        const bool is_q = m < d;
        const int r = is_q ? m : m - d;
        const int head = r / E.dh, w = r % E.dh, i = w >> 1, role = w & 1;
        int64_t x0 = role ? partner : v, x1 = role ? v : partner;
        rope_pair(x0, x1, E.rcos[(size_t)p * half + i], E.rsin[(size_t)p * half + i]);
        const int e = role ? i + half : i;
        const int64_t y = role ? x1 : x0;
        if (is_q) E.q_out[(size_t)b * d + head * E.dh + e] = y;
        else E.Kc[(((size_t)page * E.n_kv + head) * PAGE + slot) * E.dh + e] = y;
      } else {
        const int j = m - d - dkv;
        E.Vc[(((size_t)page * E.n_kv + j / E.dh) * PAGE + slot) * E.dh + (j % E.dh)] = v;
      }
      break;
    }
    case SWIGLU: {
      const int64_t partner = (int64_t)__shfl_xor_sync(0xffffffffu, (long long)v, 1);
      if (valid && (m & 1) == 0) {
        const int j = m >> 1;
        const int64_t y = swiglu(v, partner, g_exp_lut.v);
        int8_t dg[8];
        const int n = limb_split8(y, dg);
        need = n > need ? n : need;
        const size_t ps = (size_t)E.ldx * E.B;
        const size_t off = (size_t)b * E.ldx + j;
#pragma unroll
        for (int l = 0; l < 8; ++l) E.X[l * ps + off] = dg[l];
      }
      break;
    }
    case MOE_COMBINE: {
      if (!valid) break;
      const int g = m / E.grp_rows, i = m - g * E.grp_rows;
      const int64_t w = E.route[(size_t)b * E.route_ld + (size_t)g * (E.route_gs ? E.route_gs : 1)];
      if (w != 0) {
        const unsigned long long add = (unsigned long long)mulshr(w, v);
        const size_t off = (size_t)b * E.ldo + i;
        if (E.peer_h) {
          for (int p = 0; p < E.npeers; ++p) atomicAdd((unsigned long long*)(E.peer_h[p] + off), add);
        } else {
          atomicAdd((unsigned long long*)(E.out + off), add);
        }
      }
      break;
    }
    default:
      break;
  }
}

// Finalises row m of a split tile from the partial buffer P: reads and
// clears its L x B int32 partials, recombines the limbs and applies the
// epilogue.  Wide tiles (BN >= 64, i.e. batches of 8 or more) read 8 slots x
// L limbs per round with every load in flight together; each load otherwise
// waits for the previous clear, and a batch of 32 slots at 3 limbs would
// serialise 96 L2 round trips.  Called by all lanes of a warp together.
template <int BN>
__device__ __forceinline__ void finalize_from_P(const Epi& E, int* P, int M, int m, bool valid, int B, int L,
                                                int& need) {
  if (BN >= 64) {
    constexpr int FS = 4;  // slots per round: 4 x L loads in flight, no spills
    for (int b0 = 0; b0 < B; b0 += FS) {
      int v[8][FS];
#pragma unroll
      for (int l = 0; l < 8; ++l)
#pragma unroll
        for (int j = 0; j < FS; ++j)
          v[l][j] = (valid && l < L && b0 + j < B) ? __ldcg(P + (size_t)(l * B + b0 + j) * M + m) : 0;
#pragma unroll
      for (int l = 0; l < 8; ++l)
#pragma unroll
        for (int j = 0; j < FS; ++j)
          if (valid && l < L && b0 + j < B) __stcg(P + (size_t)(l * B + b0 + j) * M + m, 0);
#pragma unroll
      for (int j = 0; j < FS; ++j) {
        if (b0 + j >= B) break;
        uint64_t acc = 0;
#pragma unroll
        for (int l = 0; l < 8; ++l) acc += (uint64_t)(int64_t)v[l][j] << (8 * l);
        apply_row(E, M, m, valid, b0 + j, acc, need);
      }
    }
    return;
  }
  for (int b = 0; b < B; ++b) {
    uint64_t acc = 0;
    if (valid)
      for (int l = 0; l < L; ++l) {
        int* p = P + (size_t)(l * B + b) * M + m;
        acc += (uint64_t)(int64_t)__ldcg(p) << (8 * l);
        *p = 0;
      }
    apply_row(E, M, m, valid, b, acc, need);
  }
}

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait for a counter written by other GPUs (and this GPU's CTAs).
__device__ __forceinline__ bool wait_counter_geq(const int* p, int target) {
  if (ld_acquire_sys(p) >= target) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0;; ++i) {
    if (ld_acquire_sys(p) >= target) return true;
    if ((i & 63) == 63) {
      if (globaltimer_ns() - t0 > ARCB_WAIT_NS) return false;
      __nanosleep(64);
    }
  }
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Work item -> (n-tile, m-tile, chunk); CTA c owns items [it0, it1).
struct Work {
  int Mt, nch, it0, it1;
  __device__ void range(int ntu) {
    const long long total = (long long)ntu * Mt * nch;
    it0 = (int)(total * blockIdx.x / gridDim.x);
    it1 = (int)(total * (blockIdx.x + 1) / gridDim.x);
  }
  __device__ int nt(int it) const { return it / (Mt * nch); }
  __device__ int mt(int it) const { return (it / nch) % Mt; }
  __device__ int kc(int it) const { return it % nch; }
  __device__ int seg_end(int it) const { return min(it1, (it / nch + 1) * nch); }
  // Weights are stored tiled: tile (m, k) is 128 rows x 128 bytes, contiguous,
  // at row (m * nch + k) * 128 of a [Mt * nch * 128, 128] byte matrix, so one
  // TMA box is one contiguous 16 KB DRAM block.
  __device__ int tile_row(int it) const { return (mt(it) * nch + kc(it)) * BM; }
};

template <int BN, bool Q4>
__global__ void __launch_bounds__(Cfg<BN, Q4>::THREADS, 1)
    k_gemm_fused(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M, int K,
                 int B, int n_tiles_max, int prefetch_ok, const int* __restrict__ lmax, int* __restrict__ P,
                 int* __restrict__ tile_cnt, const __grid_constant__ Epi E, const uint8_t* __restrict__ q4w) {
  using C = Cfg<BN, Q4>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t a_base = base;
  const uint32_t b_base = base + C::STAGES * C::A_BYTES;
  const uint32_t q_base = b_base + C::STAGES * C::B_BYTES;  // Q4 staging (Q_BYTES per stage)
  const uint32_t bar = q_base + C::STAGES * C::Q_BYTES;
  auto full = [&](int s) { return bar + 8u * s; };
  auto empty = [&](int s) { return bar + 8u * (C::STAGES + s); };
  auto seg_full = [&](int t) { return bar + 8u * (2 * C::STAGES + t); };
  auto seg_free = [&](int t) { return bar + 8u * (2 * C::STAGES + 2 + t); };
  auto conv = [&](int s) { return bar + 8u * (2 * C::STAGES + 4 + s); };  // Q4: A tile converted
  const uint32_t tslot = bar + 8u * (3 * C::STAGES + 4);
  volatile uint32_t* tslot_ptr = (volatile uint32_t*)(smem_raw + (tslot - raw));
  volatile int* flag_ptr = (volatile int*)(smem_raw + (tslot + 8 - raw));
  volatile int* ok_ptr = (volatile int*)(smem_raw + (tslot + 12 - raw));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  Work W{(M + BM - 1) / BM, (K + BK - 1) / BK, 0, 0};

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(seg_full(t), 1);
      mbar_init(seg_free(t), 4);
    }
    if (Q4)
      for (int s = 0; s < C::STAGES; ++s) mbar_init(conv(s), 4);
    fence_barrier_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tslot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot_ptr;
  if (E.prof && threadIdx.x == 0) E.prof[blockIdx.x * 8 + 0] = globaltimer_ns();
  pdl_launch();

  // Weight tile of work item `it` into stage s: an int8 tile by TMA, or the
  // packed Q4 tile by a bulk copy into the staging area (converted below).
  // Decode-sized tiles (BN <= 32) always load their one box; the sub-box
  // path and the batched TMEM reads below exist for BN >= 64 only, so the
  // small-batch kernels keep their original code.
  const int bbox = (BN >= 64 && E.b_box > 0 && E.b_box < BN) ? E.b_box : BN;
  auto load_b = [&](int s, int it, int kx, int rows) {
    if constexpr (BN >= 64) {
      for (int r0 = 0; r0 < rows; r0 += bbox)
        tma_load_2d(b_base + s * C::B_BYTES + r0 * BK, &tmB, full(s), kx, W.nt(it) * BN + r0);
    } else {
      tma_load_2d(b_base + s * C::B_BYTES, &tmB, full(s), kx, W.nt(it) * BN);
    }
  };
  auto load_a = [&](int s, int it) {
    if constexpr (Q4) {
      const uint8_t* src = q4w + (size_t)(W.mt(it) * W.nch + W.kc(it)) * Q4_TILE;
      asm volatile(
          "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
              q_base + s * C::Q_BYTES),
          "l"(src), "r"(Q4_TILE), "r"(full(s))
          : "memory");
    } else {
      tma_load_2d(a_base + s * C::A_BYTES, &tmA, full(s), 0, W.tile_row(it));
    }
  };
  // Weights do not depend on the previous kernel: start streaming them.
  int pre = 0;
  if (warp == 0 && lane == 0 && prefetch_ok) {
    W.range(1);
    pre = min(C::STAGES, W.it1 - W.it0);
    for (int i = 0; i < pre; ++i) {
      const int it = W.it0 + i;
      mbar_arrive_expect_tx(full(i), C::STAGE_BYTES);
      load_a(i, it);
    }
  }
  pdl_wait();
  if (E.prof && threadIdx.x == 0) E.prof[blockIdx.x * 8 + 1] = globaltimer_ns();
  const int L = max(1, *lmax);
  const int nrows = L * B;
  const int ntu = min(n_tiles_max, (nrows + BN - 1) / BN);
  W.range(ntu);
  if (E.rp && warp == 2 && lane == 0) {
    // Publish this rank's limb count before any arrival (finalisers read the
    // max over ranks), then count the n-tiles this rank has no rows for, so
    // every rank contributes n_tiles_max * nch arrivals per tile.
    for (int p = 0; p < E.npeers; ++p) atomicMax_system(E.peer_lmax[p], L);
    __threadfence_system();
    const int virt = (n_tiles_max - ntu) * W.nch;
    if (blockIdx.x == 0 && virt > 0)
      for (int mt = 0; mt < W.Mt; ++mt)
        for (int p = 0; p < E.npeers; ++p) atomicAdd_system(E.peer_cnt[p] + mt, virt);
  }

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      const int n = W.it1 - W.it0;
      int issued = 0;
      bool ok = true;
      for (int i = 0; i < n; ++i) {
        const int it = W.it0 + i, s = i % C::STAGES;
        const uint32_t ph = (uint32_t)(i / C::STAGES) & 1u;
        const int kx = W.kc(it) * BK + (E.grp_koff ? (W.mt(it) * BM / E.grp_rows) * E.grp_koff : 0);
        if (i < pre) {  // its transaction count (full box) was set before the dependency wait
          load_b(s, it, kx, BN);
          ++issued;
          continue;
        }
        if (i >= C::STAGES && !mbar_wait(empty(s), ph ^ 1u)) {
          set_error(E.err, ARCB_ERR_TIMEOUT_EMPTY);
          ok = false;
          break;
        }
        const int live = BN >= 64 ? min(BN, (min(BN, nrows - W.nt(it) * BN) + bbox - 1) / bbox * bbox) : BN;
        mbar_arrive_expect_tx(full(s), (Q4 ? Q4_TILE : C::A_BYTES) + live * BK);
        load_a(s, it);
        load_b(s, it, kx, live);
        ++issued;
      }
      if (!ok)
        for (int i = max(0, issued - C::STAGES); i < issued; ++i)
          mbar_wait(full(i % C::STAGES), (uint32_t)(i / C::STAGES) & 1u);
      if (ok && E.pf_w && E.pf_tiles > 0) {
        const int mt2 = (E.pf_M + BM - 1) / BM, nch2 = (E.pf_K + BK - 1) / BK;
        const long long tot2 = (long long)mt2 * nch2;
        const int a0 = (int)(tot2 * blockIdx.x / gridDim.x), a1 = (int)(tot2 * (blockIdx.x + 1) / gridDim.x);
        const int np = min(a1 - a0, E.pf_tiles);
        for (int j = 0; j < np; ++j) {
          const int it = a0 + j;
          const uint8_t* src = E.pf_w + ((size_t)((it / nch2) % mt2) * nch2 + (it % nch2)) * (BM * BK);
          asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(BM * BK) : "memory");
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      int i = 0, seg = 0;
      bool ok = true;
      for (int it = W.it0; it < W.it1 && ok; ++seg) {
        const int se = W.seg_end(it), tb = seg & 1;
        if (seg >= 2 && !mbar_wait(seg_free(tb), (uint32_t)((seg >> 1) - 1) & 1u)) {
          set_error(E.err, ARCB_ERR_TIMEOUT_DONE);
          break;
        }
        tc_fence_after();
        const int n0 = W.nt(it) * BN;
        const int n_mma = (min(BN, nrows - n0) + 15) & ~15;
        const uint32_t idesc = idesc_i8(BM, n_mma);
        const uint32_t dst = tmem + (uint32_t)(tb * C::ACC_COLS);
        for (int j = it; j < se; ++j, ++i) {
          const int s = i % C::STAGES;
          if (!mbar_wait(Q4 ? conv(s) : full(s), (uint32_t)(i / C::STAGES) & 1u)) {
            set_error(E.err, ARCB_ERR_TIMEOUT_FULL);
            ok = false;
            break;
          }
          tc_fence_after();
          if (E.prof && i == 0) E.prof[blockIdx.x * 8 + 2] = globaltimer_ns();
#pragma unroll
          for (int kk = 0; kk < BK / 32; ++kk) {
            const uint64_t ad = sw128_kmajor_desc(a_base + s * C::A_BYTES + kk * 32);
            const uint64_t bd = sw128_kmajor_desc(b_base + s * C::B_BYTES + kk * 32);
            mma_i8(dst, ad, bd, idesc, (j > it || kk > 0) ? 1u : 0u);
          }
          mma_commit(empty(s));
        }
        mma_commit(seg_full(tb));
        if (E.prof) E.prof[blockIdx.x * 8 + 3] = globaltimer_ns();
        it = se;
      }
    }
  } else if (Q4 && warp >= 6) {
    // ---------------- Q4 converter warps 6..9: packed tile -> swizzled int8 A
    const int r = threadIdx.x - 192;  // tile row
    const int n = W.it1 - W.it0;
    for (int i = 0; i < n; ++i) {
      const int s = i % C::STAGES;
      if (!mbar_wait(full(s), (uint32_t)(i / C::STAGES) & 1u)) {
        set_error(E.err, ARCB_ERR_TIMEOUT_FULL);
        break;
      }
      const uint8_t* st = smem_raw + (q_base + s * C::Q_BYTES - raw);
      const uint4* nib = (const uint4*)(st + r * 64);
      const uint32_t mul = *(const uint16_t*)(st + 128 * 64 + r * 2);
      uint8_t* arow = smem_raw + (a_base + s * C::A_BYTES - raw) + r * 128;
#pragma unroll
      for (int c2 = 0; c2 < 4; ++c2) {  // 16 nibble bytes = 32 columns = one group
        const uint4 v = nib[c2];
        const int m = (int)((mul >> (4 * c2)) & 0xF);
        const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int h = 0; h < 2; ++h) {  // two 16-column output granules
          uint32_t o[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint32_t word = w4[h * 2 + (k >> 1)];
            const uint32_t b0 = (word >> (16 * (k & 1))) & 0xFF, b1 = (word >> (16 * (k & 1) + 8)) & 0xFF;
            const int v0 = ((int)(b0 & 15) - 8) * m, v1 = ((int)(b0 >> 4) - 8) * m;
            const int v2 = ((int)(b1 & 15) - 8) * m, v3 = ((int)(b1 >> 4) - 8) * m;
            o[k] = (uint32_t)(v0 & 0xFF) | ((uint32_t)(v1 & 0xFF) << 8) | ((uint32_t)(v2 & 0xFF) << 16) |
                   ((uint32_t)(v3 & 0xFF) << 24);
          }
          const int g16 = c2 * 2 + h;  // 16-byte granule index in the 128-byte row
          *(uint4*)(arow + ((g16 ^ (r & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(conv(s));
    }
  } else {
    // ---------------- epilogue warps 2..5
    const int q = warp & 3;
    int seg = 0;
    for (int it = W.it0; it < W.it1; ++seg) {
      const int se = W.seg_end(it), tb = seg & 1;
      const int nt = W.nt(it), mt = W.mt(it);
      // One thread waits (bounded); the four warps then branch together, since
      // the named barriers below have no timeout of their own.
      if (warp == 2 && lane == 0) *ok_ptr = mbar_wait(seg_full(tb), (uint32_t)(seg >> 1) & 1u) ? 1 : 0;
      epi_bar();
      const bool got = *ok_ptr != 0;
      epi_bar();
      if (!got) {
        set_error(E.err, ARCB_ERR_TIMEOUT_DONE);
        break;
      }
      tc_fence_after();
      const int m = mt * BM + q * 32 + lane;
      const bool valid = m < M;
      const int n0 = nt * BN;
      const int n_mma = (min(BN, nrows - n0) + 15) & ~15;
      const bool whole = (W.kc(it) == 0) && (se - it == W.nch);
      const bool direct = whole && ntu == 1 && E.mode != PARTIAL && !E.rp;
      const uint32_t taddr = tmem + (uint32_t)(tb * C::ACC_COLS) + ((uint32_t)(q * 32) << 16);
      int need = 0;
      if (BN >= 64 && direct && (B & 7) == 0) {
        // 8 slots x L limbs per TMEM read batch (columns l * B + b0 .. + 7)
        for (int b0 = 0; b0 < B; b0 += 8) {
          uint32_t r[8][8];
#pragma unroll
          for (int l = 0; l < 8; ++l)
            if (l < L) tmem_ld8(taddr + (uint32_t)(l * B + b0), r[l]);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            uint64_t acc = 0;
#pragma unroll
            for (int l = 0; l < 8; ++l)
              if (l < L) acc += (uint64_t)(int64_t)(int)r[l][j] << (8 * l);
            apply_row(E, M, m, valid, b0 + j, acc, need);
          }
        }
      } else if (direct) {
        for (int b = 0; b < B; ++b) {
          uint32_t r[8];
          for (int l = 0; l < L; ++l) tmem_ld1(taddr + (uint32_t)(l * B + b), r[l]);
          tmem_ld_wait();
          uint64_t acc = 0;
          for (int l = 0; l < L; ++l) acc += (uint64_t)(int64_t)(int)r[l] << (8 * l);
          apply_row(E, M, m, valid, b, acc, need);
        }
      } else {
        for (int c0 = 0; c0 < n_mma; c0 += 16) {
          uint32_t r[16];
          tmem_ld16(taddr + (uint32_t)c0, r);
          tmem_ld_wait();
          if (valid) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int n = n0 + c0 + j;
              if (n < nrows && r[j] != 0) {
                if (E.rp) {
                  for (int p = 0; p < E.npeers; ++p) red_add_s32(E.peer_P[p] + (size_t)n * M + m, (int)r[j]);
                } else {
                  red_add_s32(P + (size_t)n * M + m, (int)r[j]);
                }
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(seg_free(tb));
      if (E.rp) {
        __threadfence_system();
        epi_bar();
        if (warp == 2 && lane == 0)
          for (int p = 0; p < E.npeers; ++p) atomicAdd_system(E.peer_cnt[p] + mt, se - it);
      } else if (!direct && E.mode != PARTIAL) {
        __threadfence();
        epi_bar();
        if (warp == 2 && lane == 0) {
          const int add = se - it;
          const int old = atomicAdd(tile_cnt + mt, add);
          *flag_ptr = (old + add == ntu * W.nch) ? 1 : 0;
        }
        epi_bar();
        const bool last = *flag_ptr != 0;
        if (last) {
          __threadfence();
          finalize_from_P<BN>(E, P, M, m, valid, B, L, need);
          if (warp == 2 && lane == 0) tile_cnt[mt] = 0;
        }
        epi_bar();
      }
      if (E.mode == SWIGLU && E.lmax_out) {
        need = __reduce_max_sync(0xffffffffu, need);
        if (lane == 0 && need > 0) atomicMax(E.lmax_out, need);
      }
      it = se;
    }
    if (E.prof && warp == 2 && lane == 0) E.prof[blockIdx.x * 8 + 4] = globaltimer_ns();
    if (E.peer_sig) {
      __threadfence_system();
      epi_bar();
      if (warp == 2 && lane == 0)
        for (int p = 0; p < E.npeers; ++p) atomicAdd_system(E.peer_sig[p], 1ull);
    }
    if (E.rp && E.mode != PARTIAL) {
      // ---- finaliser: tiles mt = blockIdx.x (mod grid) of this rank's copy
      const int target = E.npeers * n_tiles_max * W.nch;
      for (int mt = blockIdx.x; mt < W.Mt; mt += gridDim.x) {
        if (warp == 2 && lane == 0) *ok_ptr = wait_counter_geq(E.cnt_local + mt, target) ? 1 : 0;
        epi_bar();
        const bool ok = *ok_ptr != 0;
        epi_bar();
        if (!ok) {
          if (warp == 2 && lane == 0) set_error(E.err, ARCB_ERR_COMM_TIMEOUT);
          continue;
        }
        __threadfence_system();
        const int Lf = min(8, max(L, ld_acquire_sys(E.lmax_fin)));
        const int m = mt * BM + q * 32 + lane;
        const bool valid = m < M;
        int need = 0;
        finalize_from_P<BN>(E, P, M, m, valid, B, Lf, need);
        epi_bar();
        if (warp == 2 && lane == 0) E.cnt_local[mt] = 0;
      }
      if (E.prof && warp == 2 && lane == 0) E.prof[blockIdx.x * 8 + 5] = globaltimer_ns();
    }
  }
  if (E.prof && threadIdx.x == 0) E.prof[blockIdx.x * 8 + 6] = globaltimer_ns();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

static int num_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

template <int BN, bool Q4>
int launch(const CUtensorMap* a, const CUtensorMap* b, int M, int K, int B, const int* lmax, int* P, int* cnt,
           const Epi& E, cudaStream_t st, int pdl, const uint8_t* q4w) {
  using C = Cfg<BN, Q4>;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(k_gemm_fused<BN, Q4>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return (int)e;
    attr = true;
  }
  const int n_tiles_max = (8 * B + BN - 1) / BN;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(E.max_ctas > 0 && E.max_ctas < num_sms() ? E.max_ctas : num_sms());
  cfg.blockDim = dim3(C::THREADS);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, k_gemm_fused<BN, Q4>, *a, *b, M, K, B, n_tiles_max,
                                     (int)(n_tiles_max == 1), lmax, P, cnt, E, q4w);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

}  // namespace fg

extern "C" {

// Box height for the fused GEMM's limb operand: all 8 planes of B slots fit
// one N tile up to B = 32 (so the work list is known before the dependency
// wait and weight prefetch is allowed); larger batches tile N by 256.
int arcb_fgemm_bn(int B) {
  const int want = 8 * B;
  if (want <= 16) return 16;
  if (want <= 32) return 32;
  if (want <= 64) return 64;
  if (want <= 128) return 128;
  return 256;
}

// Fused GEMM + epilogue.  `epi` points to an fg::Epi in host memory (copied
// into the launch).  tile_cnt: zeroed int array with one entry per M tile.
int arcb_fgemm(const void* tmA, const void* tmB, int M, int K, int B, int bn, const int* lmax, int* P,
               int* tile_cnt, const void* epi, int pdl, void* stream) {
  const CUtensorMap* a = (const CUtensorMap*)tmA;
  const CUtensorMap* b = (const CUtensorMap*)tmB;
  fg::Epi E = *(const fg::Epi*)epi;
  pdl = pdl && arcb_pdl_enabled();
  E.B = B;
  cudaStream_t st = (cudaStream_t)stream;
  switch (bn) {
    case 16: return fg::launch<16, false>(a, b, M, K, B, lmax, P, tile_cnt, E, st, pdl, nullptr);
    case 32: return fg::launch<32, false>(a, b, M, K, B, lmax, P, tile_cnt, E, st, pdl, nullptr);
    case 64: return fg::launch<64, false>(a, b, M, K, B, lmax, P, tile_cnt, E, st, pdl, nullptr);
    case 128: return fg::launch<128, false>(a, b, M, K, B, lmax, P, tile_cnt, E, st, pdl, nullptr);
    case 256: return fg::launch<256, false>(a, b, M, K, B, lmax, P, tile_cnt, E, st, pdl, nullptr);
  }
  return -3;
}

int arcb_fgemm_epi_size(void) { return (int)sizeof(fg::Epi); }

// K2: same GEMM with Q4 group-32 weights, dequantised to int8 in shared
// memory (value = (nibble - 8) * group multiplier, exact); `q4w` holds the
// tiles produced by arc_chain_b200.ops.int_ops.pack_q4 (Q4_TILE bytes each,
// tile (m, k) at index m * nch + k).
int arcb_fgemm_q4(const uint8_t* q4w, const void* tmB, int M, int K, int B, int bn, const int* lmax, int* P,
                  int* tile_cnt, const void* epi, int pdl, void* stream) {
  const CUtensorMap* b = (const CUtensorMap*)tmB;
  fg::Epi E = *(const fg::Epi*)epi;
  E.B = B;
  pdl = pdl && arcb_pdl_enabled();
  cudaStream_t st = (cudaStream_t)stream;
  if ((uintptr_t)q4w & 15) return -4;
  switch (bn) {
    case 16: return fg::launch<16, true>(b, b, M, K, B, lmax, P, tile_cnt, E, st, pdl, q4w);
    case 32: return fg::launch<32, true>(b, b, M, K, B, lmax, P, tile_cnt, E, st, pdl, q4w);
    case 64: return fg::launch<64, true>(b, b, M, K, B, lmax, P, tile_cnt, E, st, pdl, q4w);
    case 128: return fg::launch<128, true>(b, b, M, K, B, lmax, P, tile_cnt, E, st, pdl, q4w);
    case 256: return fg::launch<256, true>(b, b, M, K, B, lmax, P, tile_cnt, E, st, pdl, q4w);
  }
  return -3;
}

}  // extern "C"
