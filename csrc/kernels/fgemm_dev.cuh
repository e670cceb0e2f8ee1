// Device-side pieces of the persistent fused limb GEMM shared by the
// per-GEMM kernel (gemm_fused.cu) and the persistent decode-step kernel
// (decode_step.cu): the epilogue descriptor, tile configuration, epilogue
// row application, split-tile finalisation, bounded waits and the stream-K
// work list.  See gemm_fused.cu for the design.
#pragma once
#include <climits>

#include "common.cuh"
#include "lut.cuh"

namespace fg {

using namespace q16;

constexpr int BM = 128;
constexpr int BK = 128;
constexpr int NTHREADS = 192;
// Q4 tiles (group-32 4-bit weights): 128 rows x 64 bytes of nibbles (low
// nibble = even column, value = nibble - 8) then 128 rows x 2 bytes of 4-bit
// group multipliers (group g of the 128-column chunk in bits 4g..4g+3).
constexpr int Q4_TILE = 128 * 64 + 128 * 2;
constexpr int PAGE = 16;

// STORE_PEERS: STORE into every rank's buffer peer_h[p] (the vocab-parallel
// LM head's all-gather); kept apart from STORE so the plain store stays one
// instruction in the unrolled epilogue loops.
enum Mode : int { PARTIAL = 0, STORE = 1, RESID = 2, QKV = 3, SWIGLU = 4, MOE_COMBINE = 5, STORE_PEERS = 6 };

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
  // Tensor-parallel reduce mode (rp = 1, row-parallel GEMMs): the split-K
  // partials of a tile are summed in this GPU's P as in the one-GPU path;
  // the CTA that completes the tile recombines its limbs and stores the
  // wrapping int64 row sums into slot `rank` of every rank's receive buffer
  // peer_R[p] ([npeers][B][M], peer pointers of a symmetric allocation),
  // then adds 1 to every rank's arrival counter peer_cnt[p][tile].  Tile t
  // is finalised on each rank by its CTA t % gridDim.x once cnt_local[t]
  // reaches npeers: it sums the npeers slots and applies the epilogue.
  int rp;
  int npeers;
  int rank;
  int64_t* const* peer_R;
  int* const* peer_cnt;
  int* cnt_local;
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
  // peer_h[p] (every rank's combine buffer) instead of out.  STORE_PEERS
  // stores each row into every rank's buffer peer_h[p] (the vocab-parallel
  // LM head's all-gather; peer_h[p] already points at this rank's column
  // offset).  With peer_sig set every CTA, once its writes are fenced,
  // increments every rank's arrival counter peer_sig[p] by one.
  int route_gs;
  int64_t* const* peer_h;
  unsigned long long* const* peer_sig;
  // Work schedule of launches with several n-tiles: 0 = round-robin whole
  // tiles / n-tile groups (struct Work), 1 = plain stream-K.
  int sched;
  // Tensor-parallel reduce-scatter + all-gather (rp = 1 and rs_ag = 1), for
  // large batches on 4+ ranks: the completed tile's sums go only to its
  // owner rank (m-tile index mod npeers) and bump only the owner's counter;
  // the owner sums the npeers slots, stores the total into every rank's
  // final area (slot npeers of peer_R) and bumps every rank's final counter
  // (cnt at offset rs_cnt_off); every rank then applies the epilogue to all
  // tiles from its final area.  Each rank sends 2 (N - 1) / N of a tile's
  // bytes instead of N - 1 times them.
  int rs_ag;
  int rs_cnt_off;
  // Token-dispatch expert parallelism: with peer_h set and ep_rows > 0, the
  // MOE_COMBINE add of gathered slot b goes only to its owner rank
  // b / ep_rows, at row b % ep_rows of that rank's combine buffer (each rank
  // owns ep_rows consecutive slots).  0 = add into every rank's buffer.
  int ep_rows;
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
    case STORE_PEERS:  // GEMM -> all-gather: the row lands in every rank's buffer
      if (valid)
        for (int p = 0; p < E.npeers; ++p) __stcg((long long*)(E.peer_h[p] + (size_t)b * E.ldo + m), (long long)v);
      break;
    case RESID: {
      uint64_t sq = 0;
      if (valid) {
        int64_t* o = E.out + (size_t)b * E.ldo + m;
        // L2 read: in the persistent step kernel another CTA may have updated
        // this row since this SM last cached it
        const int64_t r = wadd(__ldcg(o), v);
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
#pragma unroll
        for (int l = 0; l < 8; ++l) E.X[limb_row(l, b, E.B) * E.ldx + j] = dg[l];
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
        if (E.peer_h && E.ep_rows > 0) {
          const int p = b / E.ep_rows;
          atomicAdd((unsigned long long*)(E.peer_h[p] + (size_t)(b - p * E.ep_rows) * E.ldo + i), add);
        } else if (E.peer_h) {
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

// SWIGLU epilogue for two consecutive slots b, b + 1 at once (acc0, acc1:
// row m's recombined sums of those slots).  Rows come in (gate, up) pairs;
// the gate lane computes slot b's output and the up lane slot b + 1's, one
// shuffle giving each the partner value it lacks.  Called by all 32 lanes.
__device__ __forceinline__ void swiglu_pair(const Epi& E, int M, int m, bool valid, int b, uint64_t acc0,
                                            uint64_t acc1, int& need) {
  const int64_t s = valid ? E.scales[m] : 0;
  const int64_t v0 = mulshr((int64_t)acc0, s), v1 = mulshr((int64_t)acc1, s);
  const bool gate = (m & 1) == 0;
  // gate lane sends its slot-(b+1) gate, up lane its slot-b up value
  const int64_t other = (int64_t)__shfl_xor_sync(0xffffffffu, (long long)(gate ? v1 : v0), 1);
  const int bs = gate ? b : b + 1;
  if (valid && bs < E.B) {
    const int64_t y = gate ? swiglu(v0, other, g_exp_lut.v) : swiglu(other, v1, g_exp_lut.v);
    int8_t dg[8];
    const int n = limb_split8(y, dg);
    need = n > need ? n : need;
    const int j = m >> 1;
#pragma unroll
    for (int l = 0; l < 8; ++l) E.X[limb_row(l, bs, E.B) * E.ldx + j] = dg[l];
  }
}

// Tensor-parallel reduce mode: stores this rank's recombined sum of row m,
// slot b into slot `rank` of every rank's receive buffer (plain stores to
// peer memory; the caller fences and signals once the tile is complete).
__device__ __forceinline__ void push_row(const Epi& E, int M, int B, int m, bool valid, int b, uint64_t acc) {
  if (!valid) return;
  const size_t off = ((size_t)E.rank * B + b) * M + m;
  if (E.rs_ag) {  // reduce-scatter: only the tile's owner
    __stcg((long long*)(E.peer_R[(m / BM) % E.npeers] + off), (long long)acc);
    return;
  }
  for (int p = 0; p < E.npeers; ++p) __stcg((long long*)(E.peer_R[p] + off), (long long)acc);
}

// The row's destination: every rank's receive buffer (PUSH, the rp mode) or
// the epilogue.  Callers branch on E.rp once per tile and run a loop
// instantiated for one of the two, so the unrolled loops carry one path.
template <bool PUSH>
__device__ __forceinline__ void emit_row(const Epi& E, int M, int B, int m, bool valid, int b, uint64_t acc,
                                         int& need) {
  if constexpr (PUSH) push_row(E, M, B, m, valid, b, acc);
  else apply_row(E, M, m, valid, b, acc, need);
}

// Applies the epilogue to row m of FG consecutive slots b0.. whose sums
// are already in registers.  RESID loads the FG hidden-state values first,
// so their latencies overlap instead of adding up slot by slot; the other
// modes go through apply_row.  Called by all lanes of a warp together.
template <int FG>
__device__ __forceinline__ void apply_rows(const Epi& E, int M, int m, bool valid, int b0, int nb,
                                           const uint64_t (&acc)[FG], int& need) {
  if (E.mode == RESID) {
    const int64_t s = valid ? E.scales[m] : 0;
    int64_t h[FG];
#pragma unroll
    for (int j = 0; j < FG; ++j) h[j] = (valid && j < nb) ? __ldcg(E.out + (size_t)(b0 + j) * E.ldo + m) : 0;
#pragma unroll
    for (int j = 0; j < FG; ++j) {
      if (j >= nb) break;
      uint64_t sq = 0;
      if (valid) {
        const int64_t r = wadd(h[j], mulshr((int64_t)acc[j], s));
        E.out[(size_t)(b0 + j) * E.ldo + m] = r;
        sq = sq16(r);
      }
      if (E.ss_out) {
        sq = warp_sum_u64(sq);
        if ((threadIdx.x & 31) == 0) atomicAdd(E.ss_out + b0 + j, (unsigned long long)sq);
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < FG; ++j)
      if (j < nb) apply_row(E, M, m, valid, b0 + j, acc[j], need);
  }
}

// Reduce-scatter owner: row m of slots [bb0, bb1) summed over the npeers
// slots and stored into every rank's final area (slot npeers of peer_R);
// four slots' loads in flight at a time.
__device__ __forceinline__ void owner_sum_to_all(const Epi& E, int M, int m, bool valid, int B, int bb0, int bb1) {
  if (!valid) return;
  const int64_t* R = E.peer_R[E.rank];
  constexpr int FG = 4;
  for (int b0 = bb0; b0 < bb1; b0 += FG) {
    uint64_t acc[FG] = {0, 0, 0, 0};
    for (int r = 0; r < E.npeers; ++r)
#pragma unroll
      for (int j = 0; j < FG; ++j)
        if (b0 + j < bb1) acc[j] += (uint64_t)__ldcg((const long long*)(R + ((size_t)r * B + b0 + j) * M + m));
    for (int p = 0; p < E.npeers; ++p)
#pragma unroll
      for (int j = 0; j < FG; ++j)
        if (b0 + j < bb1)
          __stcg((long long*)(E.peer_R[p] + ((size_t)E.npeers * B + b0 + j) * M + m), (long long)acc[j]);
  }
}

// All-gather receiver: row m of slots [bb0, bb1) from this rank's final
// area, eight slots at a time.
__device__ __forceinline__ void finalize_from_F(const Epi& E, int M, int m, bool valid, int B, int& need, int bb0,
                                                int bb1) {
  const int64_t* F = E.peer_R[E.rank] + (size_t)E.npeers * B * M;
  constexpr int FG = 8;
  for (int b0 = bb0; b0 < bb1; b0 += FG) {
    uint64_t acc[FG];
#pragma unroll
    for (int j = 0; j < FG; ++j)
      acc[j] = (valid && b0 + j < bb1) ? (uint64_t)__ldcg((const long long*)(F + (size_t)(b0 + j) * M + m)) : 0;
    apply_rows<FG>(E, M, m, valid, b0, bb1 - b0, acc, need);
  }
}

// Tensor-parallel finaliser: row m of slots [bb0, bb1) is the wrapping sum
// of the npeers ranks' slots of this rank's receive buffer (exact, so the
// order does not matter and every rank computes the same value); four
// slots' loads in flight at a time.
__device__ __forceinline__ void finalize_from_R(const Epi& E, int M, int m, bool valid, int B, int& need, int bb0,
                                                int bb1) {
  const int64_t* R = E.peer_R[E.rank];
  constexpr int FG = 4;
  for (int b0 = bb0; b0 < bb1; b0 += FG) {
    uint64_t acc[FG] = {0, 0, 0, 0};
    if (valid)
      for (int r = 0; r < E.npeers; ++r)
#pragma unroll
        for (int j = 0; j < FG; ++j)
          if (b0 + j < bb1) acc[j] += (uint64_t)__ldcg((const long long*)(R + ((size_t)r * B + b0 + j) * M + m));
    apply_rows<FG>(E, M, m, valid, b0, bb1 - b0, acc, need);
  }
}

// Finalises row m of a split tile from the partial buffer P: reads and
// clears its L x B int32 partials, recombines the limbs and applies the
// epilogue (or, in tensor-parallel reduce mode, pushes the sums).  Wide tiles (BN >= 64, i.e. batches of 8 or more) read 8 slots x
// L limbs per round with every load in flight together; each load otherwise
// waits for the previous clear, and a batch of 32 slots at 3 limbs would
// serialise 96 L2 round trips.  Called by all lanes of a warp together.
template <int BN, bool PUSH = false>
__device__ __forceinline__ void finalize_from_P(const Epi& E, int* P, int M, int m, bool valid, int B, int L,
                                                int& need, int bb0 = 0, int bb1 = -1) {
  // slots [bb0, bb1) of the partial buffer (row l * B + b); the whole batch by default
  if (bb1 < 0) bb1 = B;
  if constexpr (BN >= 64) {
    constexpr int FS = 4;  // slots per round: 4 x L loads in flight, no spills
    for (int b0 = bb0; b0 < bb1; b0 += FS) {
      int v[8][FS];
#pragma unroll
      for (int l = 0; l < 8; ++l)
#pragma unroll
        for (int j = 0; j < FS; ++j)
          v[l][j] = (valid && l < L && b0 + j < bb1) ? __ldcg(P + (size_t)(l * B + b0 + j) * M + m) : 0;
#pragma unroll
      for (int l = 0; l < 8; ++l)
#pragma unroll
        for (int j = 0; j < FS; ++j)
          if (valid && l < L && b0 + j < bb1) __stcg(P + (size_t)(l * B + b0 + j) * M + m, 0);
#pragma unroll
      for (int j = 0; j < FS; ++j) {
        if (b0 + j >= bb1) break;
        uint64_t acc = 0;
#pragma unroll
        for (int l = 0; l < 8; ++l) acc += (uint64_t)(int64_t)v[l][j] << (8 * l);
        emit_row<PUSH>(E, M, B, m, valid, b0 + j, acc, need);
      }
    }
  } else {
    for (int b = bb0; b < bb1; ++b) {
      uint64_t acc = 0;
      if (valid)
        for (int l = 0; l < L; ++l) {
          int* p = P + (size_t)(l * B + b) * M + m;
          acc += (uint64_t)(int64_t)__ldcg(p) << (8 * l);
          *p = 0;
        }
      emit_row<PUSH>(E, M, B, m, valid, b, acc, need);
    }
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

// Work item -> (m-tile, n-tile, chunk).  Three schedules:
//
// Stream-K (one n-tile): items are numbered tile by tile, chunk innermost,
// and CTA c takes one balanced contiguous range.
//
// Several n-tiles, at least two waves of tiles (hybrid): the first `waves`
// full waves are handed out whole and round-robin (CTA c runs tiles c,
// c + grid, ..., tile = mt * ntu + nt), so at any moment the grid works on
// about grid / ntu weight tiles, each shared through L2 by the CTAs on its
// n-tiles; a contiguous range would walk the n-tiles of one weight tile on
// a single CTA, re-reading it from DRAM once per n-tile.  The remaining
// tiles (between one and two waves) are split stream-K.  Item numbers of
// the round-robin part are [c * dpn, (c + 1) * dpn) for CTA c; the
// stream-K part starts at dp_end = waves * grid * nch.
//
// Several n-tiles, fewer than two waves (grouped): the grid is cut into ntu
// equal groups (grid / ntu CTAs each; the few CTAs left over get no items);
// group g = c % ntu runs stream-K over the m-tiles of n-tile g, numbered
// it = g * Mt * nch + mt * nch + chunk.  The CTAs of equal rank in different
// groups walk the same (m-tile, chunk) sequence at the same time, so each
// weight tile comes from DRAM once and is shared through L2.
//
// A round-robin tile starts at a CTA-dependent chunk `rot` and wraps (the
// chunks' partial sums are exact, so their order does not matter): the
// ntu CTAs on one weight tile, and the CTAs on one n-tile, then read any
// given chunk at different moments within the tile's window instead of all
// at once from one L2 location.  kpos(it) is the item's position in its
// tile, kc(it) the chunk it loads.
struct Work {
  int Mt, nch, it0, it1, ntu = 1;
  int dpn = 0, dp_end = 0, sk0 = 0, per = 0;  // per > 0: grouped (items per group)
  int rot = 0;
  __device__ void range(int ntu_, bool multi = false) {
    ntu = ntu_;
    const long long T = (long long)ntu * Mt;
    const int G = (int)gridDim.x, c = (int)blockIdx.x;
    if (multi && ntu > 1 && T < 2LL * G && G >= ntu) {
      const int Gg = G / ntu;  // CTAs per group
      per = Mt * nch;
      if (c >= Gg * ntu) {
        it0 = it1 = sk0 = 0;
        return;
      }
      const int g = c % ntu, r = c / ntu;
      it0 = sk0 = g * per + (int)((long long)per * r / Gg);
      it1 = g * per + (int)((long long)per * (r + 1) / Gg);
      return;
    }
    int waves = multi && ntu > 1 ? (int)(T / G) - 1 : 0;
    if (waves < 0) waves = 0;
    dpn = waves * nch;
    dp_end = waves * G * nch;
    rot = (int)(((long long)(c % ntu) * max(1, nch / ntu) + (long long)(c / ntu) * 3) % nch);
    const long long total = (T - (long long)waves * G) * nch;
    sk0 = dp_end + (int)(total * c / G);
    it1 = dp_end + (int)(total * (c + 1) / G);
    it0 = dpn ? c * dpn : sk0;
  }
  // number of items of this CTA, and its i-th item
  __device__ int count() const { return dpn + (it1 - sk0); }
  __device__ int item(int i) const { return i < dpn ? it0 + i : sk0 + (i - dpn); }
  // the item after a segment that ended at se
  __device__ int next(int se) const { return (dpn && se == it0 + dpn) ? sk0 : se; }
  __device__ int tile(int it) const {  // (mt, nt) index = mt * ntu + nt
    if (per) return ((it % per) / nch) * ntu + it / per;
    return it < dp_end ? (int)blockIdx.x + ((it - it0) / nch) * (int)gridDim.x : it / nch;
  }
  __device__ int nt(int it) const { return per ? it / per : tile(it) % ntu; }
  __device__ int mt(int it) const { return per ? (it % per) / nch : tile(it) / ntu; }
  __device__ int kpos(int it) const { return it % nch; }
  __device__ int kc(int it) const {
    const int k = it % nch;
    return it < dp_end ? (k + rot < nch ? k + rot : k + rot - nch) : k;
  }
  __device__ int seg_end(int it) const {
    return it < dp_end ? (it / nch + 1) * nch : min(it1, (it / nch + 1) * nch);
  }
  // Weights are stored tiled: tile (m, k) is 128 rows x 128 bytes, contiguous,
  // at row (m * nch + k) * 128 of a [Mt * nch * 128, 128] byte matrix, so one
  // TMA box is one contiguous 16 KB DRAM block.
  __device__ int tile_row(int it) const { return (mt(it) * nch + kc(it)) * BM; }
};
}  // namespace fg
