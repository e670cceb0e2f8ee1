// K1: exact int8-weight x int64-activation GEMM on the 5th-gen tensor cores.
//
// The reference computes every linear layer as out_i = ((sum_j w_ij * x_j) *
// s_i) >> 16 with i8 weights and full i64 Q16 activations, in wrapping i64
// (crates/arc-inference/src/cached_integer_model.rs:221-262).  Here each
// activation is split into signed radix-256 digits ("limb planes", digits in
// [-128, 127]); plane l of all tokens forms rows l*B + b of the B operand.
// tcgen05.mma kind::i8 (s8 x s8 -> s32, accumulator in TMEM) produces the
// per-limb partial P_l = sum_j w_ij * d_lj exactly: |P_l| <= 127*128*K < 2^31
// for K < 132k.  The epilogue adds the int32 partials into a global [rows, M]
// buffer with red.global.add (split-K partials are integers, so the sum is
// order independent and exact); a finalize kernel forms
// acc = sum_l P_l << 8l in wrapping u64, which equals the reference's wrapping
// i64 dot product, then applies (acc * s) >> 16 and the fused epilogue op.
//
// One weight tile read serves all limbs and all tokens: weights are the M
// operand (128 rows per CTA, TMEM lanes), limbs x tokens the N operand.
// Warp roles: warp 0 lane 0 = TMA producer, warp 1 lane 0 = MMA issuer,
// warps 0-3 = epilogue (TMEM lanes 32w..32w+31).  Every wait is bounded
// (common.cuh) and reports through the error word.
#include "common.cuh"

namespace {

constexpr int BM = 128;     // weight rows per CTA = TMEM lanes
constexpr int BK = 128;     // K bytes per pipeline stage = one 128-byte swizzle row
constexpr int NTHREADS = 128;

template <int BN>
struct Cfg {
  static constexpr int A_BYTES = BM * BK;
  static constexpr int B_BYTES = BN * BK;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (BN >= 256) ? 4 : (BN >= 128 ? 6 : 8);
  static constexpr int TMEM_COLS = BN < 32 ? 32 : BN;
  static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + (2 * STAGES + 2) * 8 + 16;
};

template <int BN>
__global__ void __launch_bounds__(NTHREADS, 1)
    k_gemm_i8(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
              int M, int K, int B, int chunks_per_split, const int* __restrict__ lmax,
              int* __restrict__ P, int* __restrict__ err) {
  using C = Cfg<BN>;
  const int L = *lmax;
  const int nrows = L * B;
  const int n0 = blockIdx.y * BN;
  if (n0 >= nrows) return;
  const int m0 = blockIdx.x * BM;
  const int nchunks = (K + BK - 1) / BK;
  const int kc0 = blockIdx.z * chunks_per_split;
  const int kc1 = min(nchunks, kc0 + chunks_per_split);
  if (kc0 >= kc1) return;
  const int nk = kc1 - kc0;
  const int n_valid = min(BN, nrows - n0);
  const int n_mma = (n_valid + 15) & ~15;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t a_base = base;
  const uint32_t b_base = base + C::STAGES * C::A_BYTES;
  const uint32_t bar_base = b_base + C::STAGES * C::B_BYTES;
  auto full = [&](int s) { return bar_base + 8u * s; };
  auto empty = [&](int s) { return bar_base + 8u * (C::STAGES + s); };
  const uint32_t done = bar_base + 8u * (2 * C::STAGES);
  const uint32_t tslot = done + 8u;
  volatile uint32_t* tslot_ptr = (volatile uint32_t*)(smem_raw + (tslot - raw));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    mbar_init(done, 1);
    fence_barrier_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 0) {
    tmem_alloc(tslot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot_ptr;

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer
    int issued = 0;
    bool ok = true;
    for (int i = 0; i < nk; ++i) {
      const int s = i % C::STAGES;
      const uint32_t ph = (uint32_t)(i / C::STAGES) & 1u;
      if (i >= C::STAGES && !mbar_wait(empty(s), ph ^ 1u)) {
        set_error(err, ARCB_ERR_TIMEOUT_EMPTY);
        ok = false;
        break;
      }
      mbar_arrive_expect_tx(full(s), C::STAGE_BYTES);
      const int kx = (kc0 + i) * BK;
      tma_load_2d(a_base + s * C::A_BYTES, &tmA, full(s), kx, m0);
      tma_load_2d(b_base + s * C::B_BYTES, &tmB, full(s), kx, n0);
      ++issued;
    }
    if (!ok) {
      // Drain copies still in flight before the CTA can exit (bounded).
      int first = issued > C::STAGES ? issued - C::STAGES : 0;
      for (int i = first; i < issued; ++i)
        mbar_wait(full(i % C::STAGES), (uint32_t)(i / C::STAGES) & 1u);
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer (single thread)
    const uint32_t idesc = idesc_i8(BM, n_mma);
    for (int i = 0; i < nk; ++i) {
      const int s = i % C::STAGES;
      const uint32_t ph = (uint32_t)(i / C::STAGES) & 1u;
      if (!mbar_wait(full(s), ph)) {
        set_error(err, ARCB_ERR_TIMEOUT_FULL);
        break;
      }
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < BK / 32; ++kk) {
        const uint64_t ad = sw128_kmajor_desc(a_base + s * C::A_BYTES + kk * 32);
        const uint64_t bd = sw128_kmajor_desc(b_base + s * C::B_BYTES + kk * 32);
        mma_i8(tmem, ad, bd, idesc, (i > 0 || kk > 0) ? 1u : 0u);
      }
      mma_commit(empty(s));
    }
    mma_commit(done);
  }
  __syncwarp();

  // ---------------- epilogue: TMEM -> int32 partial sums in global memory
  // warp-uniform decision: tcgen05.ld below is .sync.aligned
  const bool have = __shfl_sync(0xffffffffu, mbar_wait(done, 0) ? 1 : 0, 0) != 0;
  if (!have) set_error(err, ARCB_ERR_TIMEOUT_DONE);
  tc_fence_after();
  if (have) {
    const int m = m0 + warp * 32 + lane;
    for (int c0 = 0; c0 < n_mma; c0 += 16) {
      uint32_t r[16];
      tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, r);
      tmem_ld_wait();
      if (m < M) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int n = n0 + c0 + j;
          const int v = (int)r[j];
          if (n < nrows && v != 0) red_add_s32(P + (size_t)n * M + m, v);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

template <int BN>
int launch(const CUtensorMap* a, const CUtensorMap* b, int M, int K, int B, int ksplit,
           const int* lmax, int* P, int* err, cudaStream_t st) {
  using C = Cfg<BN>;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(k_gemm_i8<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return (int)e;
    attr = true;
  }
  const int nchunks = (K + BK - 1) / BK;
  if (ksplit < 1) ksplit = 1;
  if (ksplit > nchunks) ksplit = nchunks;
  const int cps = (nchunks + ksplit - 1) / ksplit;
  ksplit = (nchunks + cps - 1) / cps;
  dim3 grid((M + BM - 1) / BM, (8 * B + BN - 1) / BN, ksplit);
  k_gemm_i8<BN><<<grid, NTHREADS, C::SMEM, st>>>(*a, *b, M, K, B, cps, lmax, P, err);
  return (int)cudaGetLastError();
}

}  // namespace

extern "C" {

// Weight/limb operand tensor maps: 2-D int8 [rows, cols] row-major, box
// {128 bytes of K, box_rows}, 128-byte swizzle, zero fill out of bounds.
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                  CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                  CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiledFn)p;
  }
  return fn;
}

// Writes a 128-byte CUtensorMap into `out`.  Returns 0 on success.
int arcb_tmap_i8(void* out, const void* ptr, int64_t rows, int64_t cols, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return -1;
  if (((uintptr_t)ptr & 15) || (cols & 15)) return -2;  // TMA: 16-byte aligned base and row stride
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn((CUtensorMap*)out, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, (void*)ptr, dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return (int)r;
}

// Box height the launcher below uses for the limb operand, given B tokens.
int arcb_gemm_bn(int B) {
  int want = 4 * B;
  if (want <= 16) return 16;
  if (want <= 32) return 32;
  if (want <= 64) return 64;
  if (want <= 128) return 128;
  return 256;
}

// P[l*B+b, m] += sum_k W[m,k] * X[l*B+b, k]  for l < *lmax (device value).
int arcb_gemm_i8(const void* tmA, const void* tmB, int M, int K, int B, int bn, int ksplit,
                 const int* lmax, int* P, int* err, void* stream) {
  cudaStream_t st = (cudaStream_t)stream;
  const CUtensorMap* a = (const CUtensorMap*)tmA;
  const CUtensorMap* b = (const CUtensorMap*)tmB;
  switch (bn) {
    case 16: return launch<16>(a, b, M, K, B, ksplit, lmax, P, err, st);
    case 32: return launch<32>(a, b, M, K, B, ksplit, lmax, P, err, st);
    case 64: return launch<64>(a, b, M, K, B, ksplit, lmax, P, err, st);
    case 128: return launch<128>(a, b, M, K, B, ksplit, lmax, P, err, st);
    case 256: return launch<256>(a, b, M, K, B, ksplit, lmax, P, err, st);
  }
  return -3;
}

}  // extern "C"
