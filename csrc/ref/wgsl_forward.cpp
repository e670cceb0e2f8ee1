// Host restatement of the reference's GPU compute-shader decode path: the
// nine kernels of crates/arc-gpu/src/transformer.wgsl, dispatched in the
// order of GpuForward::forward_one_token (gpu_forward.rs:656-720), with the
// buffer sizes of GpuForward::upload_model (gpu_forward.rs:458-570).
//
// It documents how that path differs from the CPU integer engine and is the
// oracle of the CUDA restatement (csrc/kernels/wgsl_path.cu).  As wired in
// the reference, the per-token hidden state is uploaded as zeros
// (gpu_forward.rs:664-666) and the i8 KV caches and their scales are never
// written, so every layer's output is zero and the argmax returns token 0;
// the hidden input is a parameter here so the arithmetic can be exercised
// on real values.
//
// Buffer rules follow the shaders: the quantiser scans 16384 inputs and
// writes 4096 packed words whatever the vector length (loads past a buffer
// read 0, stores past it are dropped, words past 4096 keep older contents);
// attention scores only the first 32 positions (one thread each) and
// softmaxes seq_len entries of a zero-initialised 2048-entry array; argmax
// scans 32000 logits with 256 threads and keeps the lower thread on ties.
#include <stdint.h>
#include <string.h>

#include <vector>

#include "../common/wgsl_math.h"

namespace {

using wg::add;
using wg::mul;

struct Buf {  // i32 buffer with the shaders' out-of-bounds rules
  std::vector<int32_t> v;
  explicit Buf(size_t n = 0) : v(n, 0) {}
  int32_t ld(long long i) const { return (i >= 0 && (size_t)i < v.size()) ? v[(size_t)i] : 0; }
  void st(long long i, int32_t x) {
    if (i >= 0 && (size_t)i < v.size()) v[(size_t)i] = x;
  }
};
struct Words {
  std::vector<uint32_t> v;
  explicit Words(size_t n = 0) : v(n, 0u) {}
  uint32_t ld(long long i) const { return (i >= 0 && (size_t)i < v.size()) ? v[(size_t)i] : 0u; }
  void st(long long i, uint32_t x) {
    if (i >= 0 && (size_t)i < v.size()) v[(size_t)i] = x;
  }
};

Words pack(const int8_t* w, size_t n) {  // 4 signed bytes per little-endian word
  Words p((n + 3) / 4);
  for (size_t i = 0; i < n; ++i) p.v[i / 4] |= ((uint32_t)(uint8_t)w[i]) << (8 * (i % 4));
  return p;
}
Buf trunc32(const int64_t* s, size_t n) {  // `x as i32`
  Buf b(n);
  for (size_t i = 0; i < n; ++i) b.v[i] = (int32_t)(uint32_t)(uint64_t)s[i];
  return b;
}

struct Mat {
  Words w;
  Buf s;
  int in, out;
};

struct Layer {
  Mat q, k, v, o, gate, up, down;
  Buf an, fn;
  Words kc, vc;  // i8 KV caches (never written by the reference path)
  Buf ks, vs;
};

struct Model {
  int n_layers, d, dff, dh, nh, nkv, vocab, d_kv, max_seq;
  int32_t attn_scale;
  std::vector<Layer> L;
  Mat lm;
  Buf fnorm, cosb, sinb;
  // activations, sized as in upload_model
  Buf hidden, normed, q, k, v, attn_out, proj, gate, up, ff_out, logits;
  Words packed;
  int32_t qscale = 0;
};

// transformer.wgsl:122-175
void layernorm(const Buf& in, Buf& out, const Buf& gamma, int size) {
  int32_t s = 0;
  for (int i = 0; i < size; ++i) s = add(s, in.ld(i));
  const int32_t mean = wg::div(s, size);
  int32_t var = 0;
  for (int i = 0; i < size; ++i) {
    const int32_t dlt = wg::sub(in.ld(i), mean);
    var = add(var, mul(dlt, dlt) >> 16);
  }
  const int32_t istd = wg::inv_std(wg::div(var, size));
  for (int i = 0; i < size; ++i) out.st(i, wg::ln_elem(in.ld(i), mean, istd, gamma.ld(i)));
}

// transformer.wgsl:185-227
void quantize(const Buf& in, Words& out, int32_t& scale) {
  int32_t mx = 0;
  for (int i = 0; i < 16384; ++i) {
    const int32_t av = wg::abs_wrap(in.ld(i));
    mx = av > mx ? av : mx;
  }
  const int32_t amax = mx > 1 ? mx : 1;
  const int32_t a127 = amax / 127;
  const int32_t sf = a127 > 1 ? a127 : 1;
  scale = sf;
  for (int i = 0; i < 4096; ++i) {
    uint32_t p = 0;
    for (int k = 0; k < 4; ++k) p |= wg::quant_byte(in.ld(4 * i + k), sf) << (8 * k);
    out.st(i, p);
  }
}

// transformer.wgsl:64-109 (scale_offset 0)
void matmul(const Mat& m, const Words& in, Buf& out) {
  const int pc = m.in / 4;
  for (int row = 0; row < m.out; ++row) {
    int32_t acc = 0;
    for (int j = 0; j < pc; ++j) {
      const uint32_t w = m.w.ld((long long)row * pc + j), x = in.ld(j);
      for (int b = 0; b < 4; ++b) acc = add(acc, mul(wg::ext_i8(w, b), wg::ext_i8(x, b)));
    }
    out.st(row, mul(acc, m.s.ld(row) >> 8));
  }
}

// transformer.wgsl:236-256
void rope(Buf& x, const Model& M, int pos, int n_heads) {
  const int half = M.dh / 2;
  for (int idx = 0; idx < n_heads * half; ++idx) {
    const int head = idx / half, i = idx % half, base = head * M.dh;
    int32_t x0 = x.ld(base + i), x1 = x.ld(base + i + half);
    wg::rope(x0, x1, M.cosb.ld((long long)pos * half + i), M.sinb.ld((long long)pos * half + i));
    x.st(base + i, x0);
    x.st(base + i + half, x1);
  }
}

// transformer.wgsl:271-345, one workgroup of 32 threads per head
void attention(Model& M, const Layer& Ly, int seq) {
  const int dh = M.dh;
  for (int head = 0; head < M.nh; ++head) {
    const int kvh = head * M.nkv / M.nh;
    Buf sc(2048);
    for (int j = 0; j < 32 && j < seq; ++j) {
      int32_t dot = 0;
      const long long koff = (long long)j * M.d_kv + kvh * dh;
      for (int dd = 0; dd < dh / 4; ++dd) {
        const uint32_t kp = Ly.kc.ld(koff / 4 + dd);
        for (int b = 0; b < 4; ++b) dot = add(dot, mul(M.q.ld(head * dh + dd * 4 + b), wg::ext_i8(kp, b)));
      }
      sc.st(j, wg::score(dot, Ly.ks.ld(j), M.attn_scale));
    }
    int32_t mx = -999999;
    for (int j = 0; j < seq; ++j) mx = sc.ld(j) > mx ? sc.ld(j) : mx;
    int32_t sum = 0;
    for (int j = 0; j < seq; ++j) {
      const int32_t e = wg::exp_lin(wg::sub(sc.ld(j), mx));
      sc.st(j, e);
      sum = add(sum, e);
    }
    if (sum > 0)
      for (int j = 0; j < seq; ++j) sc.st(j, wg::div(mul(sc.ld(j), 65536), sum));
    const int dpt = dh / 32 > 1 ? dh / 32 : 1;
    for (int t = 0; t < 32; ++t)
      for (int dd = t * dpt; dd < dh && dd < t * dpt + dpt; ++dd) {
        int32_t acc = 0;
        for (int j = 0; j < seq; ++j) {
          const long long voff = (long long)j * M.d_kv + kvh * dh;
          const int32_t vv = mul(wg::ext_i8(Ly.vc.ld(voff / 4 + dd / 4), dd % 4), Ly.vs.ld(j));
          acc = add(acc, mul(sc.ld(j), vv) >> 16);
        }
        M.attn_out.st(head * dh + dd, acc);
      }
  }
}

// transformer.wgsl:378-414
int argmax(const Buf& in) {
  uint32_t idx[256];
  int32_t val[256];
  for (int t = 0; t < 256; ++t) {
    uint32_t bi = (uint32_t)t;
    int32_t bv = -2147483647;
    for (int i = t; i < 32000; i += 256) {
      const int32_t x = in.ld(i);
      if (x > bv) {
        bv = x;
        bi = (uint32_t)i;
      }
    }
    idx[t] = bi;
    val[t] = bv;
  }
  for (int stride = 128; stride > 0; stride >>= 1)
    for (int t = 0; t < stride; ++t)
      if (val[t + stride] > val[t]) {
        val[t] = val[t + stride];
        idx[t] = idx[t + stride];
      }
  return (int)idx[0];
}

Mat make_mat(const int8_t* w, const int64_t* s, int out, int in) {
  Mat m;
  m.w = pack(w, (size_t)out * in);
  m.s = trunc32(s, (size_t)out);
  m.in = in;
  m.out = out;
  return m;
}

}  // namespace

extern "C" {

void* arcwg_new(int n_layers, int d, int dff, int dh, int nh, int nkv, int vocab, int32_t attn_scale) {
  Model* M = new Model();
  M->n_layers = n_layers;
  M->d = d;
  M->dff = dff;
  M->dh = dh;
  M->nh = nh;
  M->nkv = nkv;
  M->vocab = vocab;
  M->d_kv = nkv * dh;
  M->max_seq = 2048;
  M->attn_scale = attn_scale;
  M->L.resize(n_layers);
  for (auto& Ly : M->L) {
    Ly.kc = Words(((size_t)M->max_seq * M->d_kv + 3) / 4);
    Ly.vc = Words(((size_t)M->max_seq * M->d_kv + 3) / 4);
    Ly.ks = Buf(M->max_seq);
    Ly.vs = Buf(M->max_seq);
  }
  M->hidden = Buf(d);
  M->normed = Buf(d);
  M->packed = Words(((size_t)(d > dff ? d : dff) + 3) / 4);
  M->q = Buf(d);
  M->k = Buf(M->d_kv);
  M->v = Buf(M->d_kv);
  M->attn_out = Buf(d);
  M->proj = Buf(d);
  M->gate = Buf(dff);
  M->up = Buf(dff);
  M->ff_out = Buf(d);
  M->logits = Buf(vocab);
  return M;
}

void arcwg_free(void* h) { delete (Model*)h; }

// w[7] / s[7]: wq wk wv wo gate up down (int8 [out, in] row-major, int64 scales)
int arcwg_set_layer(void* h, int l, const int8_t* const* w, const int64_t* const* s, const int64_t* an,
                    const int64_t* fn) {
  Model* M = (Model*)h;
  if (l < 0 || l >= M->n_layers || M->d % 4 || M->dff % 4) return -1;
  Layer& Ly = M->L[l];
  const int d = M->d, dkv = M->d_kv, dff = M->dff;
  Ly.q = make_mat(w[0], s[0], d, d);
  Ly.k = make_mat(w[1], s[1], dkv, d);
  Ly.v = make_mat(w[2], s[2], dkv, d);
  Ly.o = make_mat(w[3], s[3], d, d);
  Ly.gate = make_mat(w[4], s[4], dff, d);
  Ly.up = make_mat(w[5], s[5], dff, d);
  Ly.down = make_mat(w[6], s[6], d, dff);
  Ly.an = trunc32(an, d);
  Ly.fn = trunc32(fn, d);
  return 0;
}

int arcwg_set_head(void* h, const int8_t* out_w, const int64_t* out_s, const int64_t* fnorm, const int64_t* rcos,
                   const int64_t* rsin, int rope_rows) {
  Model* M = (Model*)h;
  M->lm = make_mat(out_w, out_s, M->vocab, M->d);
  M->fnorm = trunc32(fnorm, M->d);
  M->cosb = trunc32(rcos, (size_t)rope_rows * (M->dh / 2));
  M->sinb = trunc32(rsin, (size_t)rope_rows * (M->dh / 2));
  return 0;
}

// One token at position pos from the hidden input (d values; the reference
// uploads zeros).  Writes the logits (vocab) and returns the argmax token.
int arcwg_forward(void* h, const int32_t* hidden_in, int pos, int32_t* logits_out) {
  Model* M = (Model*)h;
  memcpy(M->hidden.v.data(), hidden_in, sizeof(int32_t) * M->d);
  for (int l = 0; l < M->n_layers; ++l) {
    const Layer& Ly = M->L[l];
    layernorm(M->hidden, M->normed, Ly.an, M->d);
    quantize(M->normed, M->packed, M->qscale);
    matmul(Ly.q, M->packed, M->q);
    matmul(Ly.k, M->packed, M->k);
    matmul(Ly.v, M->packed, M->v);
    rope(M->q, *M, pos, M->nh);
    rope(M->k, *M, pos, M->nkv);
    attention(*M, Ly, pos + 1);
    quantize(M->attn_out, M->packed, M->qscale);
    matmul(Ly.o, M->packed, M->proj);
    for (int i = 0; i < M->d; ++i) M->hidden.v[i] = add(M->hidden.v[i], M->proj.v[i]);
    layernorm(M->hidden, M->normed, Ly.fn, M->d);
    quantize(M->normed, M->packed, M->qscale);
    matmul(Ly.gate, M->packed, M->gate);
    matmul(Ly.up, M->packed, M->up);
    for (int i = 0; i < M->dff; ++i) M->gate.v[i] = wg::silu_mul(M->gate.v[i], M->up.v[i]);
    quantize(M->gate, M->packed, M->qscale);
    matmul(Ly.down, M->packed, M->ff_out);
    for (int i = 0; i < M->d; ++i) M->hidden.v[i] = add(M->hidden.v[i], M->ff_out.v[i]);
  }
  layernorm(M->hidden, M->normed, M->fnorm, M->d);
  quantize(M->normed, M->packed, M->qscale);
  matmul(M->lm, M->packed, M->logits);
  if (logits_out) memcpy(logits_out, M->logits.v.data(), sizeof(int32_t) * M->vocab);
  return argmax(M->logits);
}

}  // extern "C"
