// Device copy of the Q16 exp LUT, built at compile time by the reference's
// recurrence (crates/arc-inference/src/integer_lut.rs:24-51).
#pragma once
#include "../common/q16.h"

struct ExpLut {
  int64_t v[q16::EXP_LUT_N];
};

constexpr ExpLut make_exp_lut() {
  ExpLut t{};
  t.v[256] = q16::ONE;
  for (int i = 255; i >= 0; --i) t.v[i] = (t.v[i + 1] * q16::EXP_DECAY) >> q16::FRAC_BITS;
  return t;
}

// Global (L1-cached) rather than __constant__: lookups are data-dependent,
// and divergent constant-bank reads serialise across a warp.
static __device__ const ExpLut g_exp_lut = make_exp_lut();
