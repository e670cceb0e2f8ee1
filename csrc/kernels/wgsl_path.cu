// CUDA restatement of the reference's GPU compute-shader decode path
// (crates/arc-gpu/src/transformer.wgsl): the same nine kernels with the same
// workgroup shapes and buffer rules, so a token step launched in the order
// of GpuForward::forward_one_token reproduces that path's outputs bit for
// bit (the host restatement csrc/ref/wgsl_forward.cpp is the oracle).  The
// arithmetic is in csrc/common/wgsl_math.h.  Every buffer is passed with its
// length: loads past it read 0 and stores past it are dropped.
//
// This path is kept for fidelity with the reference's GPU numbers and to
// document its deviations from the CPU integer engine; the exact engine is
// the product (gemm_fused.cu, attn_cluster.cu, decode_ops.cu).
#include <cuda_runtime.h>
#include <stdint.h>

#include "../common/wgsl_math.h"

namespace {

template <typename T>
__device__ __forceinline__ T ld(const T* p, long long n, long long i) {
  return (i >= 0 && i < n) ? p[i] : T(0);
}
template <typename T>
__device__ __forceinline__ void st(T* p, long long n, long long i, T v) {
  if (i >= 0 && i < n) p[i] = v;
}

// transformer.wgsl:122-175, one workgroup of 256
__global__ void __launch_bounds__(256) k_wg_layernorm(const int32_t* in, long long n_in, int32_t* out,
                                                      long long n_out, const int32_t* gamma, long long n_g,
                                                      int size) {
  __shared__ int32_t sh[256];
  const int tid = threadIdx.x;
  int32_t s = 0;
  for (int i = tid; i < size; i += 256) s = wg::add(s, ld(in, n_in, i));
  sh[tid] = s;
  __syncthreads();
  for (int st2 = 128; st2 > 0; st2 >>= 1) {
    if (tid < st2) sh[tid] = wg::add(sh[tid], sh[tid + st2]);
    __syncthreads();
  }
  const int32_t mean = wg::div(sh[0], size);
  __syncthreads();
  int32_t v = 0;
  for (int i = tid; i < size; i += 256) {
    const int32_t d = wg::sub(ld(in, n_in, i), mean);
    v = wg::add(v, wg::mul(d, d) >> 16);
  }
  sh[tid] = v;
  __syncthreads();
  for (int st2 = 128; st2 > 0; st2 >>= 1) {
    if (tid < st2) sh[tid] = wg::add(sh[tid], sh[tid + st2]);
    __syncthreads();
  }
  const int32_t istd = wg::inv_std(wg::div(sh[0], size));
  for (int i = tid; i < size; i += 256) st(out, n_out, i, wg::ln_elem(ld(in, n_in, i), mean, istd, ld(gamma, n_g, i)));
}

// transformer.wgsl:185-227, one workgroup of 256
__global__ void __launch_bounds__(256) k_wg_quantize(const int32_t* in, long long n_in, uint32_t* out, long long n_out,
                                                     int32_t* scale) {
  __shared__ int32_t sh[256];
  const int tid = threadIdx.x;
  int32_t mx = 0;
  for (int i = tid; i < 16384; i += 256) {
    const int32_t av = wg::abs_wrap(ld(in, n_in, i));
    mx = av > mx ? av : mx;
  }
  sh[tid] = mx;
  __syncthreads();
  for (int st2 = 128; st2 > 0; st2 >>= 1) {
    if (tid < st2) sh[tid] = sh[tid + st2] > sh[tid] ? sh[tid + st2] : sh[tid];
    __syncthreads();
  }
  const int32_t amax = sh[0] > 1 ? sh[0] : 1;
  const int32_t a127 = amax / 127;
  const int32_t sf = a127 > 1 ? a127 : 1;
  if (tid == 0 && scale) *scale = sf;
  for (int i = tid; i < 4096; i += 256) {
    uint32_t p = 0;
    for (int k = 0; k < 4; ++k) p |= wg::quant_byte(ld(in, n_in, 4LL * i + k), sf) << (8 * k);
    st(out, n_out, i, p);
  }
}

// transformer.wgsl:64-109, one thread per output row
__global__ void __launch_bounds__(256) k_wg_matmul(const uint32_t* w, long long n_w, const uint32_t* in, long long n_in,
                                                   int32_t* out, long long n_out, int in_size, int out_size,
                                                   const int32_t* scales, long long n_s) {
  const int row = blockIdx.x * 256 + threadIdx.x;
  if (row >= out_size) return;
  const int pc = in_size / 4;
  const long long off = (long long)row * pc;
  int32_t acc = 0;
  for (int j = 0; j < pc; ++j) {
    const uint32_t a = ld(w, n_w, off + j), x = ld(in, n_in, (long long)j);
#pragma unroll
    for (int b = 0; b < 4; ++b) acc = wg::add(acc, wg::mul(wg::ext_i8(a, b), wg::ext_i8(x, b)));
  }
  st(out, n_out, (long long)row, wg::mul(acc, ld(scales, n_s, (long long)row) >> 8));
}

// transformer.wgsl:236-256
__global__ void __launch_bounds__(256) k_wg_rope(int32_t* x, long long n, const int32_t* cs, const int32_t* sn,
                                                 long long n_tab, int pos, int dh, int n_heads) {
  const int idx = blockIdx.x * 256 + threadIdx.x;
  const int half = dh / 2;
  if (idx >= n_heads * half) return;
  const int head = idx / half, i = idx % half, base = head * dh;
  int32_t x0 = ld(x, n, (long long)base + i), x1 = ld(x, n, (long long)base + i + half);
  wg::rope(x0, x1, ld(cs, n_tab, (long long)pos * half + i), ld(sn, n_tab, (long long)pos * half + i));
  st(x, n, (long long)base + i, x0);
  st(x, n, (long long)base + i + half, x1);
}

// transformer.wgsl:271-345, one workgroup of 32 per head
__global__ void __launch_bounds__(32) k_wg_attention(const int32_t* q, long long n_q, const uint32_t* kc,
                                                     const uint32_t* vc, long long n_kv, const int32_t* ks,
                                                     const int32_t* vs, long long n_s, int32_t* out, long long n_out,
                                                     int dh, int n_heads, int n_kv_heads, int seq, int d_kv,
                                                     int32_t attn_scale) {
  __shared__ int32_t sc[2048];
  const int head = blockIdx.x, tid = threadIdx.x;
  for (int i = tid; i < 2048; i += 32) sc[i] = 0;  // workgroup memory starts zeroed
  __syncthreads();
  const int kvh = head * n_kv_heads / n_heads;
  if (tid < seq) {
    const int j = tid;
    int32_t dot = 0;
    const long long koff = (long long)j * d_kv + (long long)kvh * dh;
    for (int d = 0; d < dh / 4; ++d) {
      const uint32_t kp = ld(kc, n_kv, koff / 4 + d);
      for (int k = 0; k < 4; ++k) dot = wg::add(dot, wg::mul(ld(q, n_q, (long long)head * dh + d * 4 + k), wg::ext_i8(kp, k)));
    }
    sc[j] = wg::score(dot, ld(ks, n_s, (long long)j), attn_scale);
  }
  __syncthreads();
  if (tid == 0) {
    int32_t mx = -999999;
    for (int j = 0; j < seq; ++j) {
      const int32_t v = j < 2048 ? sc[j] : 0;
      mx = v > mx ? v : mx;
    }
    int32_t sum = 0;
    for (int j = 0; j < seq; ++j) {
      const int32_t e = wg::exp_lin(wg::sub(j < 2048 ? sc[j] : 0, mx));
      if (j < 2048) sc[j] = e;
      sum = wg::add(sum, e);
    }
    if (sum > 0)
      for (int j = 0; j < seq && j < 2048; ++j) sc[j] = wg::div(wg::mul(sc[j], 65536), sum);
  }
  __syncthreads();
  const int dpt = dh / 32 > 1 ? dh / 32 : 1;
  const int d0 = tid * dpt, d1 = min(dh, d0 + dpt);
  for (int d = d0; d < d1; ++d) {
    int32_t acc = 0;
    for (int j = 0; j < seq; ++j) {
      const long long voff = (long long)j * d_kv + (long long)kvh * dh;
      const int32_t vv = wg::mul(wg::ext_i8(ld(vc, n_kv, voff / 4 + d / 4), d % 4), ld(vs, n_s, (long long)j));
      acc = wg::add(acc, wg::mul(j < 2048 ? sc[j] : 0, vv) >> 16);
    }
    st(out, n_out, (long long)head * dh + d, acc);
  }
}

// transformer.wgsl:352-358 and 365-368 (threads = workgroups x 256)
__global__ void __launch_bounds__(256) k_wg_silu(int32_t* g, const int32_t* u, long long n) {
  const long long i = (long long)blockIdx.x * 256 + threadIdx.x;
  st(g, n, i, wg::silu_mul(ld(g, n, i), ld(u, n, i)));
}
__global__ void __launch_bounds__(256) k_wg_residual(int32_t* h, const int32_t* a, long long n) {
  const long long i = (long long)blockIdx.x * 256 + threadIdx.x;
  st(h, n, i, wg::add(ld(h, n, i), ld(a, n, i)));
}

// transformer.wgsl:378-414, one workgroup of 256
__global__ void __launch_bounds__(256) k_wg_argmax(const int32_t* in, long long n_in, uint32_t* result) {
  __shared__ uint32_t si[256];
  __shared__ int32_t sv[256];
  const int tid = threadIdx.x;
  uint32_t bi = (uint32_t)tid;
  int32_t bv = -2147483647;
  for (int i = tid; i < 32000; i += 256) {
    const int32_t v = ld(in, n_in, (long long)i);
    if (v > bv) {
      bv = v;
      bi = (uint32_t)i;
    }
  }
  si[tid] = bi;
  sv[tid] = bv;
  __syncthreads();
  for (int s = 128; s > 0; s >>= 1) {
    if (tid < s && sv[tid + s] > sv[tid]) {
      sv[tid] = sv[tid + s];
      si[tid] = si[tid + s];
    }
    __syncthreads();
  }
  if (tid == 0) result[0] = si[0];
}

inline int ret() { return (int)cudaGetLastError(); }

}  // namespace

extern "C" {

int arcb_wg_layernorm(const int32_t* in, long long n_in, int32_t* out, long long n_out, const int32_t* gamma,
                      long long n_g, int size, void* stream) {
  k_wg_layernorm<<<1, 256, 0, (cudaStream_t)stream>>>(in, n_in, out, n_out, gamma, n_g, size);
  return ret();
}

int arcb_wg_quantize(const int32_t* in, long long n_in, uint32_t* out, long long n_out, int32_t* scale, void* stream) {
  k_wg_quantize<<<1, 256, 0, (cudaStream_t)stream>>>(in, n_in, out, n_out, scale);
  return ret();
}

int arcb_wg_matmul(const uint32_t* w, long long n_w, const uint32_t* in, long long n_in, int32_t* out, long long n_out,
                   int in_size, int out_size, const int32_t* scales, long long n_s, void* stream) {
  if (out_size <= 0) return 0;
  k_wg_matmul<<<(out_size + 255) / 256, 256, 0, (cudaStream_t)stream>>>(w, n_w, in, n_in, out, n_out, in_size,
                                                                          out_size, scales, n_s);
  return ret();
}

int arcb_wg_rope(int32_t* x, long long n, const int32_t* cs, const int32_t* sn, long long n_tab, int pos, int dh,
                 int n_heads, void* stream) {
  const int total = n_heads * (dh / 2);
  if (total <= 0) return 0;
  k_wg_rope<<<(total + 255) / 256, 256, 0, (cudaStream_t)stream>>>(x, n, cs, sn, n_tab, pos, dh, n_heads);
  return ret();
}

int arcb_wg_attention(const int32_t* q, long long n_q, const uint32_t* kc, const uint32_t* vc, long long n_kv,
                      const int32_t* ks, const int32_t* vs, long long n_s, int32_t* out, long long n_out, int dh,
                      int n_heads, int n_kv_heads, int seq, int d_kv, int32_t attn_scale, void* stream) {
  k_wg_attention<<<n_heads, 32, 0, (cudaStream_t)stream>>>(q, n_q, kc, vc, n_kv, ks, vs, n_s, out, n_out, dh, n_heads,
                                                           n_kv_heads, seq, d_kv, attn_scale);
  return ret();
}

int arcb_wg_silu(int32_t* g, const int32_t* u, long long n, void* stream) {
  if (n <= 0) return 0;
  k_wg_silu<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(g, u, n);
  return ret();
}

int arcb_wg_residual(int32_t* h, const int32_t* a, long long n, void* stream) {
  if (n <= 0) return 0;
  k_wg_residual<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(h, a, n);
  return ret();
}

int arcb_wg_argmax(const int32_t* in, long long n_in, uint32_t* result, void* stream) {
  k_wg_argmax<<<1, 256, 0, (cudaStream_t)stream>>>(in, n_in, result);
  return ret();
}

}  // extern "C"
