// The reference's small full-sequence integer transformer (the model behind
// its cross-platform determinism benchmark): i64 Q16 weights, LayerNorm
// with gamma/beta, multi-head attention over the whole sequence, ReLU FFN,
// LCG-seeded test models, greedy generate + BLAKE3 output hash
// (crates/arc-inference/src/integer_engine.rs:16-38 matmul, 44-84
// layernorm, 90-137 attention, 140-237 block, 240-305 model, 309-377
// build_test_model; crates/arc-bench/src/integer_bench.rs).
//
// Semantics kept exactly: wrapping i64 products and sums; masked attention
// scores are -8 * ONE (not -infinity) and still enter the softmax, so when a
// row's maximum is negative later positions contribute and every position
// must be recomputed each step: generate re-runs the whole sequence per
// token, as the reference does.
#include <stdint.h>
#include <string.h>

#include <vector>

#include "../common/q16.h"
#include "arcref.h"
#include "blake3.h"

using namespace q16;

namespace {

struct Block {
  std::vector<int64_t> wq, wk, wv, wo, ff1, ff2, g1, b1, g2, b2;
};

struct Toy {
  int vocab, d, h, dh, ff, layers;
  int64_t attn_scale;
  std::vector<int64_t> emb, lm, fg, fb;
  std::vector<Block> blocks;
};

// argmax_i64: the first maximal index (integer_lut.rs:103-113).
int argmax_first(const int64_t* x, int n) {
  int b = 0;
  for (int i = 1; i < n; ++i)
    if (x[i] > x[b]) b = i;
  return b;
}

// out[i] = (sum_j W[i, j] x[j]) >> 16 (no bias in the model's uses).
void matmul(const std::vector<int64_t>& W, const int64_t* x, int in, int out, int64_t* y) {
  for (int i = 0; i < out; ++i) {
    uint64_t acc = 0;
    const int64_t* w = W.data() + (size_t)i * in;
    for (int j = 0; j < in; ++j) acc += (uint64_t)w[j] * (uint64_t)x[j];
    y[i] = (int64_t)acc >> FRAC_BITS;
  }
}

void layernorm(const int64_t* x, int n, const std::vector<int64_t>& g, const std::vector<int64_t>& b, int64_t* y) {
  uint64_t s = 0;
  for (int i = 0; i < n; ++i) s += (uint64_t)x[i];
  const int64_t mean = tdiv((int64_t)s, n);
  uint64_t vs = 0;
  for (int i = 0; i < n; ++i) {
    const int64_t diff = wsub(x[i], mean);
    vs += (uint64_t)(wmul(diff, diff) >> FRAC_BITS);
  }
  const int64_t var = tdiv((int64_t)vs, n);
  const int64_t inv = integer_isqrt(wadd(var, 1));
  for (int i = 0; i < n; ++i) {
    const int64_t diff = wsub(x[i], mean);
    const int64_t nm = wmul(diff, inv) >> FRAC_BITS;
    y[i] = wadd(wmul(nm, g[i]) >> FRAC_BITS, b[i]);
  }
}

uint64_t lcg_step(uint64_t& r) {
  r = r * 6364136223846793005ull + 1442695040888963407ull;
  return r;
}

std::vector<int64_t> gen_vec(uint64_t& r, size_t n) {
  std::vector<int64_t> v(n);
  for (size_t i = 0; i < n; ++i) v[i] = (int64_t)(lcg_step(r) >> 33) % 13107 - 6553;
  return v;
}

int64_t isqrt_floor(int64_t v) {
  int64_t s = 0;
  while ((s + 1) * (s + 1) <= v) ++s;
  return s;
}

// Forward over the whole sequence; logits of the last position.
void forward(const Toy& m, const uint32_t* toks, int T, int64_t* logits) {
  const int d = m.d, dh = m.dh;
  std::vector<int64_t> x((size_t)T * d, 0), nx((size_t)T * d), q((size_t)T * d), k((size_t)T * d),
      v((size_t)T * d), att((size_t)T * d), r1((size_t)T * d), hid(m.ff), f2(d);
  for (int t = 0; t < T; ++t)
    if ((int)toks[t] < m.vocab) memcpy(&x[(size_t)t * d], &m.emb[(size_t)toks[t] * d], sizeof(int64_t) * d);
  std::vector<int64_t> sc(T), p(T);
  for (const Block& bk : m.blocks) {
    for (int t = 0; t < T; ++t) layernorm(&x[(size_t)t * d], d, bk.g1, bk.b1, &nx[(size_t)t * d]);
    for (int t = 0; t < T; ++t) {
      matmul(bk.wq, &nx[(size_t)t * d], d, d, &q[(size_t)t * d]);
      matmul(bk.wk, &nx[(size_t)t * d], d, d, &k[(size_t)t * d]);
      matmul(bk.wv, &nx[(size_t)t * d], d, d, &v[(size_t)t * d]);
    }
    for (int hh = 0; hh < m.h; ++hh) {
      const int o = hh * dh;
      for (int i = 0; i < T; ++i) {
        for (int j = 0; j < T; ++j) {
          if (j > i) {
            sc[j] = -8 * ONE;
            continue;
          }
          uint64_t dot = 0;
          for (int e = 0; e < dh; ++e) dot += (uint64_t)q[(size_t)i * d + o + e] * (uint64_t)k[(size_t)j * d + o + e];
          sc[j] = wmul((int64_t)dot >> FRAC_BITS, m.attn_scale) >> FRAC_BITS;
        }
        arcref_softmax(sc.data(), T, p.data());
        for (int e = 0; e < dh; ++e) {
          uint64_t acc = 0;
          for (int j = 0; j < T; ++j) acc += (uint64_t)p[j] * (uint64_t)v[(size_t)j * d + o + e];
          att[(size_t)i * d + o + e] = (int64_t)acc >> FRAC_BITS;
        }
      }
    }
    for (int t = 0; t < T; ++t) {
      matmul(bk.wo, &att[(size_t)t * d], d, d, f2.data());
      for (int e = 0; e < d; ++e) r1[(size_t)t * d + e] = wadd(x[(size_t)t * d + e], f2[e]);
    }
    for (int t = 0; t < T; ++t) {
      const int64_t* xr = &r1[(size_t)t * d];
      layernorm(xr, d, bk.g2, bk.b2, nx.data());
      matmul(bk.ff1, nx.data(), d, m.ff, hid.data());
      for (int e = 0; e < m.ff; ++e) hid[e] = hid[e] > 0 ? hid[e] : 0;
      matmul(bk.ff2, hid.data(), m.ff, d, f2.data());
      for (int e = 0; e < d; ++e) x[(size_t)t * d + e] = wadd(xr[e], f2[e]);
    }
  }
  std::vector<int64_t> last(d);
  layernorm(&x[(size_t)(T - 1) * d], d, m.fg, m.fb, last.data());
  matmul(m.lm, last.data(), d, m.vocab, logits);
}

}  // namespace

extern "C" {

void* arcref_toy_build(int vocab, int d, int h, int ff, int layers) {
  Toy* m = new Toy();
  m->vocab = vocab;
  m->d = d;
  m->h = h;
  m->dh = d / h;
  m->ff = ff;
  m->layers = layers;
  uint64_t r = 42;
  m->emb = gen_vec(r, (size_t)vocab * d);
  m->lm = gen_vec(r, (size_t)vocab * d);
  m->fg.assign(d, ONE);
  m->fb.assign(d, 0);
  switch (m->dh) {
    case 32: m->attn_scale = 11585; break;
    case 64: m->attn_scale = 8192; break;
    case 128: m->attn_scale = 5793; break;
    default: m->attn_scale = ONE / (isqrt_floor(m->dh) + 1); break;
  }
  for (int l = 0; l < layers; ++l) {
    Block b;
    b.wq = gen_vec(r, (size_t)d * d);
    b.wk = gen_vec(r, (size_t)d * d);
    b.wv = gen_vec(r, (size_t)d * d);
    b.wo = gen_vec(r, (size_t)d * d);
    b.ff1 = gen_vec(r, (size_t)ff * d);
    b.ff2 = gen_vec(r, (size_t)d * ff);
    b.g1.assign(d, ONE);
    b.b1.assign(d, 0);
    b.g2.assign(d, ONE);
    b.b2.assign(d, 0);
    m->blocks.push_back(std::move(b));
  }
  return m;
}

void arcref_toy_free(void* h) { delete (Toy*)h; }

void arcref_toy_forward(void* h, const uint32_t* toks, int n, int64_t* logits) { forward(*(Toy*)h, toks, n, logits); }

// Greedy generate (argmax, lowest index on ties; stops after emitting eos);
// returns the count and writes BLAKE3(LE u32 tokens) to hash32.
int arcref_toy_generate(void* h, const uint32_t* prompt, int n, int max_tokens, uint32_t eos, uint32_t* out,
                        uint8_t* hash32) {
  const Toy& m = *(Toy*)h;
  std::vector<uint32_t> toks(prompt, prompt + n);
  std::vector<int64_t> logits(m.vocab);
  int cnt = 0;
  for (int s = 0; s < max_tokens; ++s) {
    forward(m, toks.data(), (int)toks.size(), logits.data());
    const uint32_t nx = (uint32_t)argmax_first(logits.data(), m.vocab);
    out[cnt++] = nx;
    toks.push_back(nx);
    if (nx == eos) break;
  }
  std::vector<uint8_t> b(4 * (size_t)cnt);
  for (int i = 0; i < cnt; ++i)
    for (int k = 0; k < 4; ++k) b[4 * i + k] = (uint8_t)(out[i] >> (8 * k));
  arcb3::hash(b.data(), b.size(), hash32);
  return cnt;
}

}  // extern "C"
