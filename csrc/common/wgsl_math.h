// Arithmetic of the reference's GPU compute-shader path (crates/arc-gpu/src/
// transformer.wgsl, driven by gpu_forward.rs), restated for the host
// restatement (csrc/ref/wgsl_forward.cpp) and the CUDA kernels
// (csrc/kernels/wgsl_path.cu).  That path computes a different function
// from the CPU integer engine: 32-bit activations, i8-quantised matmul
// inputs, mean-subtracting LayerNorm with an f32 square root, an i8 KV
// cache, a piecewise-linear exp, a leaky-ReLU "SiLU" and a thread-ordered
// argmax.
//
// WGSL integer semantics kept here: i32 + - * wrap modulo 2^32; >> on i32 is
// arithmetic; e1 / e2 truncates toward zero and yields e1 when e2 == 0 or
// when e1 = INT_MIN and e2 = -1; u32(i32) reinterprets the bits; i32(f32)
// truncates toward zero.  Loads past the end of a buffer read 0 and stores
// past it are dropped (the robust-access choice this restatement makes; the
// WGSL specification leaves the value implementation-defined).
#pragma once
#include <math.h>
#include <stdint.h>

#if defined(__CUDACC__)
#define WG_HD __host__ __device__ __forceinline__
#else
#define WG_HD inline
#endif

namespace wg {

WG_HD int32_t add(int32_t a, int32_t b) { return (int32_t)((uint32_t)a + (uint32_t)b); }
WG_HD int32_t sub(int32_t a, int32_t b) { return (int32_t)((uint32_t)a - (uint32_t)b); }
WG_HD int32_t mul(int32_t a, int32_t b) { return (int32_t)((uint32_t)a * (uint32_t)b); }
WG_HD int32_t div(int32_t a, int32_t b) {
  if (b == 0 || (a == INT32_MIN && b == -1)) return a;
  return a / b;
}
WG_HD int32_t neg(int32_t a) { return sub(0, a); }

// signed byte idx of a little-endian packed word (transformer.wgsl:47-50)
WG_HD int32_t ext_i8(uint32_t packed, uint32_t idx) { return (int32_t)(int8_t)(uint8_t)((packed >> (idx * 8u)) & 0xFFu); }

// inv_std of the LayerNorm kernels (transformer.wgsl:167, 468)
WG_HD int32_t inv_std(int32_t variance) {
  int32_t v = add(variance, 1);
  v = v > 1 ? v : 1;
  const int32_t r = (int32_t)sqrtf((float)v);
  return div(65536, r > 1 ? r : 1);
}

// one normalised, gamma-scaled element (transformer.wgsl:172-173)
WG_HD int32_t ln_elem(int32_t x, int32_t mean, int32_t istd, int32_t gamma) {
  const int32_t norm = mul(sub(x, mean), istd) >> 16;
  return mul(norm, gamma) >> 16;
}

// quantisation of one value with scale factor s, clamped to [-127, 127]
WG_HD uint32_t quant_byte(int32_t v, int32_t s) {
  int32_t q = div(v, s);
  q = q < -127 ? -127 : (q > 127 ? 127 : q);
  return (uint32_t)q & 0xFFu;
}

WG_HD int32_t abs_wrap(int32_t v) { return v >= 0 ? v : neg(v); }

// RoPE rotation of a pair (transformer.wgsl:254-255)
WG_HD void rope(int32_t& x0, int32_t& x1, int32_t c, int32_t s) {
  const int32_t a = sub(mul(x0, c) >> 16, mul(x1, s) >> 16);
  const int32_t b = add(mul(x0, s) >> 16, mul(x1, c) >> 16);
  x0 = a;
  x1 = b;
}

// attention score from a dot product (transformer.wgsl:293)
WG_HD int32_t score(int32_t dot, int32_t k_scale, int32_t attn_scale) {
  return mul(mul(dot >> 16, k_scale) >> 16, attn_scale) >> 16;
}

// piecewise-linear exp of x = score - max (transformer.wgsl:313-318)
WG_HD int32_t exp_lin(int32_t x) {
  const int32_t e = x > -65536 * 8 ? add(65536, x) : 0;
  return e > 0 ? e : 0;
}

// leaky "SiLU" times up (transformer.wgsl:352-358)
WG_HD int32_t silu_mul(int32_t g, int32_t u) { return mul(g > 0 ? g : (g >> 2), u) >> 16; }

}  // namespace wg
