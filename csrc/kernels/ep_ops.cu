// K11 (expert-parallel combine, second half): after a rank's grouped down
// GEMM has added its experts' routing-weighted outputs into every rank's
// combine buffer `delta` (peer atomics, MOE_COMBINE epilogue of
// gemm_fused.cu) and each of its CTAs has bumped every rank's arrival
// counter, this kernel waits until all ranks' arrivals for this call are in
// (bounded; a timeout sets ARCB_ERR_COMM_TIMEOUT and goes on), then folds
// h += delta (wrapping) and clears delta.  Integer adds make the result
// independent of the order in which peers' contributions landed.
//
// The call count lives on the device (`epoch`, advanced by the block that
// finishes last), so the kernel is CUDA-graph safe: call e waits for
// cnt >= (e + 1) * per_call.  per_call = 0 skips the wait (the NCCL path,
// where an all-reduce already summed delta).
#include <algorithm>

#include "common.cuh"

namespace {

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__global__ void k_ep_wait_apply(const unsigned long long* __restrict__ cnt, unsigned long long* __restrict__ epoch,
                                unsigned long long per_call, int64_t* __restrict__ h, int64_t* __restrict__ delta,
                                int64_t n, int* __restrict__ done, int* __restrict__ err) {
  pdl_wait_dep();
  __shared__ int ok;
  const unsigned long long ep = *(volatile unsigned long long*)epoch;
  if (threadIdx.x == 0) {
    ok = 1;
    if (per_call) {
      const unsigned long long target = (ep + 1) * per_call;
      if (ld_acquire_u64(cnt) < target) {
        const uint64_t t0 = globaltimer_ns();
        while (ld_acquire_u64(cnt) < target) {
          if (globaltimer_ns() - t0 > ARCB_WAIT_NS) {
            ok = 0;
            break;
          }
          __nanosleep(128);
        }
      }
    }
  }
  __syncthreads();
  if (!ok && threadIdx.x == 0) set_error(err, ARCB_ERR_COMM_TIMEOUT);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    h[i] = (int64_t)((uint64_t)h[i] + (uint64_t)delta[i]);
    delta[i] = 0;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(done, 1) == (int)gridDim.x - 1) {
      *epoch = ep + 1;
      *done = 0;
      __threadfence();
    }
  }
  pdl_allow_next();
}

}  // namespace

extern "C" {

// cnt: this rank's arrival counter (u64); epoch: u64 call count; done: int
// scratch (zero); h, delta: n int64.
int arcb_ep_wait_apply(const void* cnt, void* epoch, unsigned long long per_call, int64_t* h, int64_t* delta, int64_t n,
                       int* done, int* err, void* stream) {
  const int64_t blocks = std::min<int64_t>(148, (n + 1023) / 1024);
  return launch_k(k_ep_wait_apply, dim3((unsigned)std::max<int64_t>(1, blocks)), dim3(256), 0, (cudaStream_t)stream,
                  (const unsigned long long*)cnt, (unsigned long long*)epoch, per_call, h, delta, n, done, err);
}

}  // extern "C"
