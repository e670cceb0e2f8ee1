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

// K10 (expert-parallel token dispatch).  Tokens live on the rank that owns
// their request (attention, router and dense layers run on each rank's own
// B slots); the experts are sharded over the ranks.  Before a MoE layer's
// expert GEMMs, every rank stores its slots' normalised-activation limb
// planes (X: limb_row layout of B slots, ldx = d bytes per row) and routing
// weights (route: [B, G] int64) into every rank's gathered buffers at slot
// offset rank * B (gathered layout: limb_row of N * B slots), writes its limb
// count into slot `rank` of every rank's counts[], fences, and bumps every
// rank's arrival counter once per CTA.  Block 0 then waits (bounded) until
// all N ranks' CTAs of this call have arrived, and writes the gathered limb
// count (the max over ranks) to gcnt and zeroes the expert GEMM's limb
// counter zero_cnt.  Peer memory is written with plain 16-byte stores (no
// TMA, no multicast).  Each rank's grouped expert GEMMs then read only this
// GPU's gathered copy.
//
// Buffer reuse: a rank writes a peer's gathered buffers for layer j + 1 only
// after its own combine wait of layer j, which needs the arrivals of every
// CTA of the peer's down GEMM of layer j, which runs after the peer's
// gate/up GEMM (the only reader of the gathered planes) and reads the
// gathered routing weights itself before arriving; so one set of gathered
// buffers serves every layer.
__global__ void k_ep_dispatch(const int8_t* __restrict__ X, int B, int ldx, const int64_t* __restrict__ route, int G,
                              const int* __restrict__ lcnt, int rank, int npeers, int8_t* const* __restrict__ peer_X,
                              int64_t* const* __restrict__ peer_route, int* const* __restrict__ peer_counts,
                              unsigned long long* const* __restrict__ peer_sig, const unsigned long long* __restrict__ cnt,
                              unsigned long long* __restrict__ epoch, int* __restrict__ gcnt, int* __restrict__ zero_cnt,
                              int* __restrict__ err) {
  pdl_wait_dep();
  const int NB = npeers * B;
  const int row16 = ldx / 16;                     // 16-byte chunks per limb row
  const int64_t nx = (int64_t)8 * B * row16;      // limb-plane chunks
  const int64_t nr = (int64_t)B * G * 8 / 16;     // routing-weight chunks
  const int64_t tot = nx + nr;
  for (int p = 0; p < npeers; ++p) {
    int8_t* dX = peer_X[p];
    int64_t* dR = peer_route[p];
    for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < tot; c += (int64_t)gridDim.x * blockDim.x) {
      if (c < nx) {
        const int64_t r = c / row16;
        const int l = (int)(r / B), b = (int)(r - (int64_t)l * B), k = (int)(c - r * row16);
        const int4 v = *(const int4*)(X + limb_row(l, b, B) * ldx + (size_t)k * 16);
        *(int4*)(dX + limb_row(l, rank * B + b, NB) * ldx + (size_t)k * 16) = v;
      } else {
        const int64_t k = c - nx;  // route rows are contiguous: [B, G] -> rows rank * B ..
        const int4 v = *(const int4*)((const int8_t*)route + k * 16);
        *(int4*)((int8_t*)(dR + (size_t)rank * B * G) + k * 16) = v;
      }
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) peer_counts[p][rank] = *lcnt;
  }
  __threadfence_system();  // every thread's peer stores, before the CTA's arrival
  __syncthreads();
  if (threadIdx.x == 0)
    for (int p = 0; p < npeers; ++p) atomicAdd_system(peer_sig[p], 1ull);
  if (blockIdx.x == 0) {
    __shared__ int ok;
    if (threadIdx.x == 0) {
      const unsigned long long ep = *(volatile unsigned long long*)epoch;
      const unsigned long long target = (ep + 1) * (unsigned long long)npeers * gridDim.x;
      ok = 1;
      if (ld_acquire_u64(cnt) < target) {
        const uint64_t t0 = globaltimer_ns();
        while (ld_acquire_u64(cnt) < target) {
          if (globaltimer_ns() - t0 > ARCB_WAIT_NS) {
            ok = 0;
            break;
          }
          __nanosleep(64);
        }
      }
      if (!ok) set_error(err, ARCB_ERR_COMM_TIMEOUT);
      int m = 0;
      const int* cts = peer_counts[rank];
      for (int p = 0; p < npeers; ++p) {
        const int v = ((volatile const int*)cts)[p];
        m = v > m ? v : m;
      }
      *gcnt = m;
      *zero_cnt = 0;
      *epoch = ep + 1;
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

// Token dispatch (see k_ep_dispatch).  X: this rank's limb planes of B
// slots, ldx a multiple of 16; route: [B, G] int64 (B * G even); peer_*:
// device arrays of npeers peer pointers; cnt/epoch: this rank's u64 arrival
// counter and call count; gcnt: gathered limb count (out); zero_cnt: a
// counter the next GEMM raises (zeroed here).  The grid size must be the
// same on every rank (it is part of the arrival target).
int arcb_ep_dispatch(const int8_t* X, int B, int ldx, const int64_t* route, int G, const int* lcnt, int rank,
                     int npeers, void* const* peer_X, void* const* peer_route, void* const* peer_counts,
                     void* const* peer_sig, const void* cnt, void* epoch, int* gcnt, int* zero_cnt, int blocks,
                     int* err, void* stream) {
  if (ldx % 16 || (B * G) % 2 || blocks < 1) return -2;
  return launch_k(k_ep_dispatch, dim3(blocks), dim3(256), 0, (cudaStream_t)stream, X, B, ldx, route, G, lcnt, rank,
                  npeers, (int8_t* const*)peer_X, (int64_t* const*)peer_route, (int* const*)peer_counts,
                  (unsigned long long* const*)peer_sig, (const unsigned long long*)cnt, (unsigned long long*)epoch,
                  gcnt, zero_cnt, err);
}

}  // extern "C"
