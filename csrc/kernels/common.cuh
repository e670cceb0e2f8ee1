// Shared device helpers for the sm_100a kernels: error reporting, bounded
// waits, mbarrier / TMA / tcgen05 inline-PTX wrappers.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../common/q16.h"

// Error word bits written by kernels (host reads them with arcb_get_error).
enum ArcbErr : int {
  ARCB_ERR_TIMEOUT_FULL = 1,     // MMA side waited too long for a TMA stage
  ARCB_ERR_TIMEOUT_EMPTY = 2,    // producer waited too long for a free stage
  ARCB_ERR_TIMEOUT_DONE = 4,     // epilogue waited too long for the accumulator
  ARCB_ERR_BOUNDS = 8,           // an index check failed (access skipped)
  ARCB_ERR_COMM_TIMEOUT = 16,    // a cross-GPU flag wait ran out
  ARCB_ERR_SEQ_OVERFLOW = 32,    // position beyond the RoPE table / page table
};

// Default bound on any spin: 2 s of %globaltimer.
#ifndef ARCB_WAIT_NS
#define ARCB_WAIT_NS 2000000000ull
#endif

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void set_error(int* err, int code) {
  if (err) atomicOr(err, code);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: returns false (after ARCB_WAIT_NS) instead of spinning forever.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255) == 255 && globaltimer_ns() - t0 > ARCB_WAIT_NS) return false;
  }
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"((uint64_t)map), "r"(bar), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)map) : "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::i8, s32 accumulate.
__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on an mbarrier once all prior tcgen05.mma of this thread complete.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

// 32 lanes x 16 columns of 32-bit from TMEM (warp w reads lanes 32w..32w+31).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                 "=r"(r[7])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor, K-major, 128-byte swizzle: rows of 128
// bytes, 8-row atoms of 1024 bytes (SBO), version 1 (sm_100).
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFF) >> 4);   // start address
  d |= (uint64_t)(16 >> 4) << 16;           // LBO (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;         // SBO
  d |= (uint64_t)1 << 46;                   // version
  d |= (uint64_t)2 << 61;                   // SWIZZLE_128B
  return d;
}

// Instruction descriptor: kind::i8, s8 x s8 -> s32, both K-major.
__host__ __device__ __forceinline__ uint32_t idesc_i8(int M, int N) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ---------------------------------------------------------------- PDL
// Programmatic dependent launch: a kernel launched with the PDL attribute
// may start while its predecessor still runs; it must call pdl_wait()
// before touching anything the predecessor writes.  Both are no-ops for a
// normal launch.
__device__ __forceinline__ void pdl_wait_dep() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_allow_next() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// Process-wide switch (arcb_set_pdl) read by every launcher.
int arcb_pdl_enabled();

template <typename... KArgs, typename... Args>
static inline int launch_k(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                           Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = arcb_pdl_enabled();
  cfg.attrs = at;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, k, ((KArgs)args)...);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

// ---------------------------------------------------------------- misc
__device__ __forceinline__ void red_add_s32(int* p, int v) {
  asm volatile("red.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int64_t shfl_xor_i64(int64_t v, int m) {
  return (int64_t)__shfl_xor_sync(0xffffffffu, (long long)v, m);
}

// Limb-operand layout: the row of limb plane l of slot b when B slots are
// split into limbs.  Slots are grouped in blocks of S = min(B, 32); a block
// occupies 8 * S consecutive rows, limb-major inside (row l * S + slot), so
// one 256-row N tile of the fused GEMM holds every limb of its 32 slots and
// can recombine them from TMEM.  For B <= 32 this is the single block
// row = l * B + b.
__host__ __device__ __forceinline__ int limb_slots(int B) { return B < 32 ? B : 32; }
__host__ __device__ __forceinline__ size_t limb_row(int l, int b, int B) {
  if (B <= 32) return (size_t)l * B + b;  // one block: no division
  return (size_t)(b >> 5) * 256 + (size_t)l * 32 + (size_t)(b & 31);
}

// Signed-digit limb split of one value into 8 int8 planes.
__device__ __forceinline__ int limb_split8(int64_t x, int8_t* d) {
  int need = 0;
  int64_t r = x;
#pragma unroll
  for (int l = 0; l < 8; ++l) {
    int8_t dl = (int8_t)(uint8_t)((uint64_t)r & 0xFF);
    d[l] = dl;
    r = q16::wsub(r, (int64_t)dl) >> 8;
    if (r == 0 && need == 0) need = l + 1;
  }
  if (x == 0) return 0;
  return need == 0 ? 8 : need;
}
