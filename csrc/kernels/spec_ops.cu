// Speculative-decoding verification: repetition penalty + argmax for the k+1
// verify positions of each lane.
//
// The reference's greedy step (crates/arc-inference/src/cached_integer_model.rs:
// 1533-1548) penalises the newest 64 generated ids, compounding, newest
// first, then takes the first maximum.  When the target model scores the
// draft tokens d_1..d_k in one forward, position i (0..k) must see exactly
// the history a plain decode would have seen: the lane's confirmed tokens
// followed by d_1..d_i.  CTA (lane, i) applies the penalty over d_i, ..., d_1
// and then the confirmed ring (newest first) until 64 ids have been applied,
// and writes argmax to y[lane * (k + 1) + i].  Logits rows are slot-major:
// row = lane * (k + 1) + i.
#include <climits>

#include "common.cuh"

using namespace q16;

namespace {

__global__ void k_verify_sample(int64_t* __restrict__ logits, int ldl, int V, int k,
                                const int* __restrict__ drafts, const int* __restrict__ hist,
                                const int* __restrict__ count, int* __restrict__ y) {
  pdl_wait_dep();
  pdl_allow_next();
  __shared__ int64_t sv[32];
  __shared__ int si[32];
  const int lane = blockIdx.y, i = blockIdx.x;
  const int row = lane * (k + 1) + i;
  int64_t* lg = logits + (size_t)row * ldl;
  if (threadIdx.x == 0) {
    int applied = 0;
    for (int j = i; j >= 1 && applied < 64; --j, ++applied) {
      const int t = drafts[lane * k + j - 1];
      if (t >= 0 && t < V) lg[t] = penalize(lg[t]);
    }
    const int cnt = count[lane];
    for (int kk = 0; kk < cnt && applied < 64; ++kk, ++applied) {
      const int t = hist[lane * 64 + ((cnt - 1 - kk) & 63)];
      if (t >= 0 && t < V) lg[t] = penalize(lg[t]);
    }
  }
  __syncthreads();
  int64_t bv = INT64_MIN;
  int bi = 0x7fffffff;
  for (int v = threadIdx.x; v < V; v += blockDim.x) {
    const int64_t x = lg[v];
    if (x > bv) {
      bv = x;
      bi = v;
    }
  }
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) {
    const int64_t ov = (int64_t)__shfl_xor_sync(0xffffffffu, (long long)bv, m);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, m);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) {
    sv[w] = bv;
    si[w] = bi;
  }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    bv = l < nw ? sv[l] : INT64_MIN;
    bi = l < nw ? si[l] : 0x7fffffff;
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
      const int64_t ov = (int64_t)__shfl_xor_sync(0xffffffffu, (long long)bv, m);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, m);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (l == 0) y[row] = bi == 0x7fffffff ? 0 : bi;
  }
}

}  // namespace

extern "C" int arcb_verify_sample(int64_t* logits, int ldl, int V, int lanes, int k, const int* drafts,
                                  const int* hist, const int* count, int* y, void* stream) {
  return launch_k(k_verify_sample, dim3(k + 1, lanes), dim3(1024), 0, (cudaStream_t)stream, logits, ldl, V, k,
                  drafts, hist, count, y);
}
