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
#include "fgemm_dev.cuh"

using namespace q16;

namespace fg {

// MB: the launch has several 32-slot blocks (B > 32, 256-row tiles only).
template <int BN, bool Q4, bool MB>
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
  // b_row: first operand row of the item's n-tile; tile: weight tile index
  // (m-tile * chunks + chunk) in the tiled weight layout.
  auto load_b = [&](int s, int b_row, int kx, int rows) {
    if constexpr (BN >= 64) {
      for (int r0 = 0; r0 < rows; r0 += bbox)
        tma_load_2d(b_base + s * C::B_BYTES + r0 * BK, &tmB, full(s), kx, b_row + r0);
    } else {
      tma_load_2d(b_base + s * C::B_BYTES, &tmB, full(s), kx, b_row);
    }
  };
  auto load_a = [&](int s, int tile) {
    if constexpr (Q4) {
      const uint8_t* src = q4w + (size_t)tile * Q4_TILE;
      asm volatile(
          "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
              q_base + s * C::Q_BYTES),
          "l"(src), "r"(Q4_TILE), "r"(full(s))
          : "memory");
    } else {
      tma_load_2d(a_base + s * C::A_BYTES, &tmA, full(s), 0, tile * BM);
    }
  };
  // Weights do not depend on the previous kernel: start streaming them.
  // The work list depends only on B (n-tiles = slot blocks), not on the limb
  // count, so it is known before the dependency wait.
  // Only launches with B > 32 (256-row tiles) have several 32-slot blocks;
  // the others have one block of B slots, which the compiler is told.
  constexpr bool MULTI = MB;
  const int S = MULTI ? limb_slots(B) : B;
  const int ntu = MULTI ? n_tiles_max : 1;  // = ceil(B / S)
  int pre = 0;
  if (warp == 0 && lane == 0 && prefetch_ok) {
    W.range(ntu, MULTI && E.sched == 0);
    pre = min(C::STAGES, W.count());
    for (int i = 0; i < pre; ++i) {
      const int it = W.item(i);
      mbar_arrive_expect_tx(full(i), C::STAGE_BYTES);
      load_a(i, W.mt(it) * W.nch + W.kc(it));
    }
  }
  pdl_wait();
  if (E.prof && threadIdx.x == 0) E.prof[blockIdx.x * 8 + 1] = globaltimer_ns();
  const int L = max(1, *lmax);
  const int nrows = L * S;  // live rows of every n-tile: L limbs of S slots
  W.range(ntu, MULTI && E.sched == 0);

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      // One thread issues every stage, so its per-stage work bounds the
      // kernel at large batch (a 256-row stage is ~0.14 us of MMA): the item
      // -> (tile, chunk) mapping is evaluated once per segment (tile) and
      // the chunk, stage and parity then advance by increments.
      const int live = BN >= 64 ? min(BN, (min(BN, nrows) + bbox - 1) / bbox * bbox) : BN;
      const uint32_t tx_bytes = (Q4 ? Q4_TILE : C::A_BYTES) + live * BK;
      int issued = 0, i = 0, s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int it = W.item(0); it < W.it1 && ok; it = W.next(W.seg_end(it))) {
        const int se = W.seg_end(it), mt_ = W.mt(it), nch = W.nch;
        const int b_row = W.nt(it) * BN;
        const int kx_off = E.grp_koff ? (mt_ * BM / E.grp_rows) * E.grp_koff : 0;
        const int tile0 = mt_ * nch;
        int kc = W.kc(it);
        for (int j = it; j < se; ++j, ++i) {
          const int kx = kc * BK + kx_off;
          if (i < pre) {  // its transaction count (full box) was set before the dependency wait
            load_b(s, b_row, kx, BN);
          } else {
            if (i >= C::STAGES && !mbar_wait(empty(s), ph ^ 1u)) {
              set_error(E.err, ARCB_ERR_TIMEOUT_EMPTY);
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(full(s), tx_bytes);
            load_a(s, tile0 + kc);
            load_b(s, b_row, kx, live);
          }
          ++issued;
          if (++kc == nch) kc = 0;
          if (++s == C::STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      if (!ok)
        for (int i = max(0, issued - C::STAGES); i < issued; ++i)
          mbar_wait(full(i % C::STAGES), (uint32_t)(i / C::STAGES) & 1u);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      int i = 0, seg = 0;
      bool ok = true;
      for (int it = W.item(0); it < W.it1 && ok; ++seg) {
        const int se = W.seg_end(it), tb = seg & 1;
        if (seg >= 2 && !mbar_wait(seg_free(tb), (uint32_t)((seg >> 1) - 1) & 1u)) {
          set_error(E.err, ARCB_ERR_TIMEOUT_DONE);
          break;
        }
        tc_fence_after();
        const int n_mma = (min(BN, nrows) + 15) & ~15;
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
        it = W.next(se);
      }
    }
  } else if (Q4 && warp >= 6) {
    // ---------------- Q4 converter warps 6..9: packed tile -> swizzled int8 A
    const int r = threadIdx.x - 192;  // tile row
    const int n = W.count();
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
    for (int it = W.item(0); it < W.it1; ++seg) {
      const int se = W.seg_end(it), tb = seg & 1;
      const int nt = MULTI ? W.nt(it) : 0, mt = MULTI ? W.mt(it) : it / W.nch, tl = MULTI ? W.tile(it) : mt;
      const int sb0 = nt * S, nb = min(S, B - sb0);  // slots of this n-tile
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
      const int n_mma = (min(BN, nrows) + 15) & ~15;
      const bool whole = (W.kpos(it) == 0) && (se - it == W.nch);
      const bool direct = whole && E.mode != PARTIAL;
      const uint32_t taddr = tmem + (uint32_t)(tb * C::ACC_COLS) + ((uint32_t)(q * 32) << 16);
      int need = 0;
      // A tile covered by this CTA alone is recombined from TMEM; its rows go
      // to the epilogue or, in the rp mode, to every rank's receive buffer.
      // Only the epilogue form has the unrolled 8-slot batches (the push is
      // the rare multi-GPU case), so the hot loops carry a single path.
      if (BN >= 64 && direct && !E.rp && (nb & 7) == 0) {
        // 8 slots x L limbs per TMEM read batch (tile columns l * S + s0 .. + 7)
        for (int s0 = 0; s0 < nb; s0 += 8) {
          uint32_t r[8][8];
#pragma unroll
          for (int l = 0; l < 8; ++l)
            if (l < L) tmem_ld8(taddr + (uint32_t)(l * S + s0), r[l]);
          tmem_ld_wait();
          if (E.mode == SWIGLU) {
            // slot pairs: the gate lane (even row) finishes slot j and the up
            // lane (odd row) slot j + 1, so no lane of the pair idles
#pragma unroll
            for (int j = 0; j < 8; j += 2) {
              uint64_t a0 = 0, a1 = 0;
#pragma unroll
              for (int l = 0; l < 8; ++l)
                if (l < L) {
                  a0 += (uint64_t)(int64_t)(int)r[l][j] << (8 * l);
                  a1 += (uint64_t)(int64_t)(int)r[l][j + 1] << (8 * l);
                }
              swiglu_pair(E, M, m, valid, sb0 + s0 + j, a0, a1, need);
            }
          } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              uint64_t acc = 0;
#pragma unroll
              for (int l = 0; l < 8; ++l)
                if (l < L) acc += (uint64_t)(int64_t)(int)r[l][j] << (8 * l);
              apply_row(E, M, m, valid, sb0 + s0 + j, acc, need);
            }
          }
        }
      } else if (direct) {
        for (int s = 0; s < nb; ++s) {
          uint32_t r[8];
          for (int l = 0; l < L; ++l) tmem_ld1(taddr + (uint32_t)(l * S + s), r[l]);
          tmem_ld_wait();
          uint64_t acc = 0;
          for (int l = 0; l < L; ++l) acc += (uint64_t)(int64_t)(int)r[l] << (8 * l);
          if (E.rp) push_row(E, M, B, m, valid, sb0 + s, acc);
          else apply_row(E, M, m, valid, sb0 + s, acc, need);
        }
      } else if (!MULTI || ntu == 1) {
        // one slot block: tile column c is partial row c
        for (int c0 = 0; c0 < n_mma; c0 += 16) {
          uint32_t r[16];
          tmem_ld16(taddr + (uint32_t)c0, r);
          tmem_ld_wait();
          if (valid) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int n = c0 + j;
              if (n < nrows && r[j] != 0) red_add_s32(P + (size_t)n * M + m, (int)r[j]);
            }
          }
        }
      } else {
        // tile column c = l * S + s holds partial row l * B + sb0 + s = c + l * (B - S) + sb0;
        // l is advanced column by column (no division on the tail's critical path)
        int lc = 0, sc = 0;
        for (int c0 = 0; c0 < n_mma; c0 += 16) {
          uint32_t r[16];
          tmem_ld16(taddr + (uint32_t)c0, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int c = c0 + j, l = lc, s = sc;
            if (++sc == S) {
              sc = 0;
              ++lc;
            }
            const int n = c + l * (B - S) + sb0;
            if (valid) {
              if (c < nrows && s < nb && r[j] != 0) red_add_s32(P + (size_t)n * M + m, (int)r[j]);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(seg_free(tb));
      bool pushed = direct;  // rp: this CTA completed the tile and stored its sums
      if (!direct && E.mode != PARTIAL) {
        __threadfence();
        epi_bar();
        if (warp == 2 && lane == 0) {
          const int add = se - it;
          const int old = atomicAdd(tile_cnt + tl, add);
          *flag_ptr = (old + add == W.nch) ? 1 : 0;
        }
        epi_bar();
        const bool last = *flag_ptr != 0;
        if (last) {
          __threadfence();
          if (E.rp) finalize_from_P<BN, true>(E, P, M, m, valid, B, L, need, sb0, sb0 + nb);
          else finalize_from_P<BN, false>(E, P, M, m, valid, B, L, need, sb0, sb0 + nb);
          if (warp == 2 && lane == 0) tile_cnt[tl] = 0;
        }
        pushed = last;
        epi_bar();
      }
      if (E.rp && pushed) {
        // the tile's sums are in every rank's receive buffer: signal each rank once
        __threadfence_system();
        epi_bar();
        if (warp == 2 && lane == 0) {
          if (E.rs_ag) atomicAdd_system(E.peer_cnt[mt % E.npeers] + tl, 1);
          else
            for (int p = 0; p < E.npeers; ++p) atomicAdd_system(E.peer_cnt[p] + tl, 1);
        }
      }
      if (E.mode == SWIGLU && E.lmax_out) {
        need = __reduce_max_sync(0xffffffffu, need);
        if (lane == 0 && need > 0) atomicMax(E.lmax_out, need);
      }
      it = W.next(se);
    }
    if (E.prof && warp == 2 && lane == 0) E.prof[blockIdx.x * 8 + 4] = globaltimer_ns();
    if (E.peer_sig) {
      __threadfence_system();
      epi_bar();
      if (warp == 2 && lane == 0)
        for (int p = 0; p < E.npeers; ++p) atomicAdd_system(E.peer_sig[p], 1ull);
    }
    if (E.rp && E.mode != PARTIAL && E.rs_ag) {
      // ---- reduce-scatter owner: every tile of this rank's m-tiles (all of
      // them first, since they wait only on partial pushes), then the
      // all-gather receiver for every tile
      for (int t = blockIdx.x; t < W.Mt * ntu; t += gridDim.x) {
        const int mt = t / ntu, nt = t - mt * ntu;
        if (mt % E.npeers != E.rank) continue;
        const int sb0 = nt * S, nb = min(S, B - sb0);
        if (warp == 2 && lane == 0) *ok_ptr = wait_counter_geq(E.cnt_local + t, E.npeers) ? 1 : 0;
        epi_bar();
        const bool ok = *ok_ptr != 0;
        epi_bar();
        if (!ok) {
          if (warp == 2 && lane == 0) set_error(E.err, ARCB_ERR_COMM_TIMEOUT);
          continue;
        }
        __threadfence_system();
        const int m = mt * BM + q * 32 + lane;
        owner_sum_to_all(E, M, m, m < M, B, sb0, sb0 + nb);
        __threadfence_system();
        epi_bar();
        if (warp == 2 && lane == 0) {
          E.cnt_local[t] = 0;
          for (int p = 0; p < E.npeers; ++p) atomicAdd_system(E.peer_cnt[p] + E.rs_cnt_off + t, 1);
        }
      }
      for (int t = blockIdx.x; t < W.Mt * ntu; t += gridDim.x) {
        const int mt = t / ntu, nt = t - mt * ntu;
        const int sb0 = nt * S, nb = min(S, B - sb0);
        if (warp == 2 && lane == 0) *ok_ptr = wait_counter_geq(E.cnt_local + E.rs_cnt_off + t, 1) ? 1 : 0;
        epi_bar();
        const bool ok = *ok_ptr != 0;
        epi_bar();
        if (!ok) {
          if (warp == 2 && lane == 0) set_error(E.err, ARCB_ERR_COMM_TIMEOUT);
          continue;
        }
        __threadfence_system();
        const int m = mt * BM + q * 32 + lane;
        int need = 0;
        finalize_from_F(E, M, m, m < M, B, need, sb0, sb0 + nb);
        epi_bar();
        if (warp == 2 && lane == 0) E.cnt_local[E.rs_cnt_off + t] = 0;
      }
      if (E.prof && warp == 2 && lane == 0) E.prof[blockIdx.x * 8 + 5] = globaltimer_ns();
    } else if (E.rp && E.mode != PARTIAL) {
      // ---- finaliser: (m-tile, n-tile) t = blockIdx.x (mod grid) of this rank's copy
      const int target = E.npeers;  // one arrival per rank per tile
      for (int t = blockIdx.x; t < W.Mt * ntu; t += gridDim.x) {
        const int mt = t / ntu, nt = t - mt * ntu;
        const int sb0 = nt * S, nb = min(S, B - sb0);
        if (warp == 2 && lane == 0) *ok_ptr = wait_counter_geq(E.cnt_local + t, target) ? 1 : 0;
        epi_bar();
        const bool ok = *ok_ptr != 0;
        epi_bar();
        if (!ok) {
          if (warp == 2 && lane == 0) set_error(E.err, ARCB_ERR_COMM_TIMEOUT);
          continue;
        }
        __threadfence_system();
        const int m = mt * BM + q * 32 + lane;
        const bool valid = m < M;
        int need = 0;
        finalize_from_R(E, M, m, valid, B, need, sb0, sb0 + nb);
        epi_bar();
        if (warp == 2 && lane == 0) E.cnt_local[t] = 0;
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

template <int BN, bool Q4, bool MB = false>
int launch(const CUtensorMap* a, const CUtensorMap* b, int M, int K, int B, const int* lmax, int* P, int* cnt,
           const Epi& E, cudaStream_t st, int pdl, const uint8_t* q4w) {
  using C = Cfg<BN, Q4>;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(k_gemm_fused<BN, Q4, MB>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return (int)e;
    attr = true;
  }
  const int n_tiles_max = (B + limb_slots(B) - 1) / limb_slots(B);  // slot blocks = n-tiles
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
  cudaError_t e = cudaLaunchKernelEx(&cfg, k_gemm_fused<BN, Q4, MB>, *a, *b, M, K, B, n_tiles_max, 1, lmax, P, cnt,
                                     E, q4w);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

}  // namespace fg

extern "C" {

// N-tile height of the fused GEMM's limb operand: all 8 planes of B <= 32
// slots in one tile; larger batches use 256-row tiles of 32-slot blocks
// (limb_row layout), one tile per block.
int arcb_fgemm_bn(int B) {
  const int want = 8 * B;
  if (want <= 16) return 16;
  if (want <= 32) return 32;
  if (want <= 64) return 64;
  if (want <= 128) return 128;
  return 256;
}

// Fused GEMM + epilogue.  `epi` points to an fg::Epi in host memory (copied
// into the launch).  tile_cnt: zeroed int array with one entry per (M tile,
// N tile), ceil(M / 128) * ceil(B / 32) + 1 entries.  The limb operand uses
// the limb_row layout (common.cuh); the partial buffer P has rows l * B + b.
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
    case 256:
      return B > 32 ? fg::launch<256, false, true>(a, b, M, K, B, lmax, P, tile_cnt, E, st, pdl, nullptr)
                    : fg::launch<256, false, false>(a, b, M, K, B, lmax, P, tile_cnt, E, st, pdl, nullptr);
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
    case 256:
      return B > 32 ? fg::launch<256, true, true>(b, b, M, K, B, lmax, P, tile_cnt, E, st, pdl, q4w)
                    : fg::launch<256, true, false>(b, b, M, K, B, lmax, P, tile_cnt, E, st, pdl, q4w);
  }
  return -3;
}

}  // extern "C"
