// Allocation-free entry point of the fused limb GEMM; see gemm_noalloc.h for
// who needs it, its limits and its sharing rules.  It has no counterpart in
// the reference.
#include "gemm_noalloc.h"

#include "fgemm_dev.cuh"

#include <cuda_runtime.h>

#include <mutex>

extern "C" int arcb_fgemm(const void* tmA, const void* tmB, int M, int K, int B, int bn, const int* lmax, int* P,
                          int* tile_cnt, const void* epi, int pdl, void* stream);

namespace {

constexpr unsigned kWords = ARCB_NOALLOC_SCRATCH_BYTES / 4u;
constexpr unsigned kCounterWords = 4096u;  // tile counters first, partials after

// The library's own scratch: tile counters, then int32 partial sums.  In host
// code this name is only a stand-in for the device array, so its device
// address is looked up per device below and passed to the kernel.
static __device__ __align__(256) int g_fgemm_scratch[kWords];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
int* g_dev_ptr[kMaxDevices] = {};

// Set-up, once per device, with that device current.
int scratch_for_current_device(int** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev < 0 || dev >= kMaxDevices) return ARCB_NOALLOC_ERR_ARGS;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_dev_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_fgemm_scratch);
    if (e != cudaSuccess || !p) return ARCB_NOALLOC_ERR_SYMBOL;
    g_dev_ptr[dev] = (int*)p;
  }
  *out = g_dev_ptr[dev];
  return 0;
}

}  // namespace

extern "C" int arcb_fgemm_noalloc(const void* tmA, const void* tmB, int M, int K, int B, int bn, const int* lmax,
                                  const void* epi, void* stream) {
  if (!tmA || !tmB || !lmax || !epi || M <= 0 || K <= 0 || B <= 0) return ARCB_NOALLOC_ERR_ARGS;
  // Partial-only mode leaves its result in the scratch array; the push and
  // peer-target modes write other GPUs' buffers that the caller allocated.
  const fg::Epi* E = (const fg::Epi*)epi;
  if (E->mode == fg::PARTIAL || E->rp || E->peer_h || E->peer_sig) return ARCB_NOALLOC_ERR_MODE;
  const long long tiles = (long long)((M + 127) / 128) * ((B + limb_slots(B) - 1) / limb_slots(B)) + 1;
  if (tiles > ARCB_NOALLOC_MAX_TILES + 1) return ARCB_NOALLOC_ERR_TOO_MANY_TILES;
  const long long partials = 8ll * B * (long long)M;
  if (partials > (long long)ARCB_NOALLOC_MAX_PARTIALS) return ARCB_NOALLOC_ERR_PARTIALS;
  int* base = nullptr;
  int rc = scratch_for_current_device(&base);
  if (rc) return rc;
  int* cnt = base;
  int* P = base + kCounterWords;
  cudaStream_t st = (cudaStream_t)stream;
  // The kernel expects zeroed counters and partials; clear the part this call uses.
  cudaError_t e = cudaMemsetAsync(cnt, 0, (size_t)tiles * sizeof(int), st);
  if (e == cudaSuccess) e = cudaMemsetAsync(P, 0, (size_t)partials * sizeof(int), st);
  if (e != cudaSuccess) return (int)e;
  return arcb_fgemm(tmA, tmB, M, K, B, bn, lmax, P, cnt, epi, 1, stream);
}
