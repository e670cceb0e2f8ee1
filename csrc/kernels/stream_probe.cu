// Weight-streaming probe: how fast one persistent CTA per SM can stream a
// large read-only buffer into a shared-memory ring with the bulk-copy
// engine, without any MMA.  Used to size the decode GEMMs' load path.
//   mode 0: 2-D tensor-map loads of 128 x 128-byte boxes (16 KB), as the
//           fused GEMM loads its weight tiles;
//   mode 1: 1-D bulk copies (cp.async.bulk) of `tile` contiguous bytes.
// CTA c streams the contiguous range [c, c+1) * n / grid of tiles through a
// `stages`-deep ring; a consumer thread waits for each stage and frees it.
#include "common.cuh"

namespace {

__device__ __forceinline__ void probe_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__global__ void __launch_bounds__(64, 1) k_stream_probe(const __grid_constant__ CUtensorMap tm, const uint8_t* src,
                                                        long long n_tiles, int tile, int stages, int mode,
                                                        int* err) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t bar = base + (uint32_t)stages * tile;
  auto full = [&](int s) { return bar + 8u * s; };
  auto empty = [&](int s) { return bar + 8u * (stages + s); };
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    fence_barrier_init();
  }
  __syncthreads();
  const long long t0 = n_tiles * blockIdx.x / gridDim.x, t1 = n_tiles * (blockIdx.x + 1) / gridDim.x;
  const int n = (int)(t1 - t0);
  if (threadIdx.x == 0) {
    for (int i = 0; i < n; ++i) {
      const int s = i % stages;
      if (i >= stages && !mbar_wait(empty(s), ((uint32_t)(i / stages) & 1u) ^ 1u)) {
        set_error(err, ARCB_ERR_TIMEOUT_EMPTY);
        break;
      }
      mbar_arrive_expect_tx(full(s), tile);
      const long long t = t0 + i;
      if (mode == 0) {
        for (int r = 0; r < tile / (128 * 128); ++r)
          tma_load_2d(base + s * tile + r * 16384, &tm, full(s), 0, (int)((t * (tile / 16384) + r) * 128));
      } else {
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                base + s * tile),
            "l"(src + t * tile), "r"(tile), "r"(full(s))
            : "memory");
      }
    }
  } else if (threadIdx.x == 32) {
    for (int i = 0; i < n; ++i) {
      const int s = i % stages;
      if (!mbar_wait(full(s), (uint32_t)(i / stages) & 1u)) {
        set_error(err, ARCB_ERR_TIMEOUT_FULL);
        break;
      }
      probe_arrive(empty(s));
    }
  }
  __syncthreads();
}

}  // namespace

extern "C" int arcb_stream_probe(const void* tmap, const uint8_t* src, long long nbytes, int tile, int stages, int mode,
                                 int grid, int* err, void* stream) {
  if (tile % 16384 || stages < 1) return -1;
  const size_t smem = 1024 + (size_t)stages * tile + 16 * stages + 64;
  if (smem > 227 * 1024) return -2;
  cudaError_t e = cudaFuncSetAttribute(k_stream_probe, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return (int)e;
  k_stream_probe<<<grid, 64, smem, (cudaStream_t)stream>>>(*(const CUtensorMap*)tmap, src, nbytes / tile, tile, stages,
                                                             mode, err);
  return (int)cudaGetLastError();
}
