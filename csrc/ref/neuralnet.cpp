// Native NeuralNet reader / writer / forward passes; the format and the two
// executions are described in neuralnet.h.  Restated from the behaviour of
// crates/arc-vm/src/inference.rs (from_bytes 132-211, to_bytes 213-270,
// forward 282-381, infer_*_size 387-422) and, for the integer form, of
// I8Weights::quantize_f32 (crates/arc-inference/src/cached_integer_model.rs:
// 36-62) and the Q16 primitives of integer_lut.rs.
//
// Float semantics that decide bits:
//  * every f32 sum is a left-to-right fold that starts at -0.0 (the
//    reference's edition-2024 toolchain folds `Sum` for floats from -0.0);
//  * `a += w * x` is a rounded product then a rounded add: this file is built
//    with -ffp-contract=off so no fused multiply-add is formed;
//  * max is NaN-ignoring (f32::max, fmaxf);
//  * exp is the C library's expf, the function Rust's f32::exp calls on
//    Linux;
//  * Rust's float -> integer casts saturate and send NaN to 0; C++ casts of
//    out-of-range values are undefined, so every such cast goes through a
//    saturating helper.
#include "ref/neuralnet.h"

#include <math.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <string>
#include <vector>

#include "common/q16.h"
#include "ref/arcref.h"

using q16::ONE;

namespace {

struct NNLayer {
  int kind = ARCNN_RELU;
  int64_t rows = 0, cols = 0;  // dense out x in; embedding vocab x dim; layernorm n
  std::vector<float> a, b;     // W / gamma / table; bias / beta
  float eps = 0.0f;
  // integer form
  std::vector<int8_t> qw;
  std::vector<int64_t> qs, qa, qb;
  int64_t qeps = 1;
};

int64_t sat_i64(double v) {
  if (v != v) return 0;
  if (v >= 9223372036854775808.0) return INT64_MAX;
  if (v <= -9223372036854775808.0) return INT64_MIN;
  return (int64_t)v;
}

// round(v * ONE), half away from zero, saturated: a Q16 value from an f32.
int64_t to_q16(float v) { return sat_i64(round((double)v * (double)ONE)); }

float fold_sum(const float* p, int64_t n) {
  float s = -0.0f;
  for (int64_t i = 0; i < n; ++i) s = s + p[i];
  return s;
}

// I8Weights::quantize_f32 of one row.
void quantize_row(const float* w, int64_t cols, int8_t* q, int64_t* scale) {
  float am = 0.0f;
  for (int64_t j = 0; j < cols; ++j) am = fmaxf(am, fabsf(w[j]));
  am = fmaxf(am, 1e-10f);
  const float inv = 127.0f / am;
  for (int64_t j = 0; j < cols; ++j) {
    float r = roundf(w[j] * inv);
    r = std::min(std::max(r, -127.0f), 127.0f);
    q[j] = (r != r) ? 0 : (int8_t)r;
  }
  const int64_t s = q16::tdiv(q16::wadd(q16::wmul(sat_i64(am), ONE), 126), 127);
  *scale = std::max<int64_t>(s, 1);
}

void build_int(NNLayer& L) {
  switch (L.kind) {
    case ARCNN_DENSE:
      L.qw.resize((size_t)(L.rows * L.cols));
      L.qs.resize((size_t)L.rows);
      L.qb.resize((size_t)L.rows);
      for (int64_t i = 0; i < L.rows; ++i) {
        quantize_row(L.a.data() + i * L.cols, L.cols, L.qw.data() + i * L.cols, &L.qs[i]);
        L.qb[i] = to_q16(L.b[i]);
      }
      break;
    case ARCNN_LAYERNORM:
      L.qa.resize(L.a.size());
      L.qb.resize(L.b.size());
      for (size_t i = 0; i < L.a.size(); ++i) L.qa[i] = to_q16(L.a[i]);
      for (size_t i = 0; i < L.b.size(); ++i) L.qb[i] = to_q16(L.b[i]);
      L.qeps = std::max<int64_t>(1, to_q16(L.eps));
      break;
    case ARCNN_EMBEDDING:
      L.qa.resize(L.a.size());
      for (size_t i = 0; i < L.a.size(); ++i) L.qa[i] = to_q16(L.a[i]);
      break;
    default:
      break;
  }
}

// Width of one embedding row as the VM's forward sees it: an empty table has
// no first row, so out-of-vocabulary inputs emit nothing.
int64_t emb_dim(const NNLayer& L) { return L.rows == 0 ? 0 : L.cols; }

// Saturating f32 -> usize, then the table bound: the row index, or -1.
int64_t emb_index_f32(float x, int64_t vocab) {
  if (!(x >= 0.0f)) return vocab > 0 ? 0 : -1;  // negative and NaN saturate to 0
  if ((double)x >= (double)vocab) return -1;
  return (int64_t)x;
}

// Q16 index: the integer part, negatives saturated to 0 as the f32 path does.
int64_t emb_index_q16(int64_t x, int64_t vocab) {
  const int64_t i = x < 0 ? 0 : (x >> 16);
  return i < vocab ? i : -1;
}

struct Rd {
  const uint8_t* p;
  size_t n, off = 0;
  std::string err;
  bool u32(uint32_t& v) {
    if (n - off < 4) {
      err = "unexpected end of model data at offset " + std::to_string(off) + " (need 4 bytes)";
      return false;
    }
    memcpy(&v, p + off, 4);
    off += 4;
    return true;
  }
  bool f32s(std::vector<float>& v, uint64_t count) {
    if ((n - off) / 4 < count) {
      err = "unexpected end of model data at offset " + std::to_string(off) + " (need " +
            std::to_string(count) + " f32 values)";
      return false;
    }
    v.resize((size_t)count);
    if (count) memcpy(v.data(), p + off, (size_t)count * 4);
    off += (size_t)count * 4;
    return true;
  }
};

bool parse_with(const uint8_t* d, size_t len, int base, std::vector<NNLayer>& out, size_t& used,
                std::string& err) {
  Rd r{d, len};
  if (len < 4) {
    err = "model data too short (need at least 4 bytes for header)";
    return false;
  }
  uint32_t nl = 0;
  r.u32(nl);
  out.clear();
  for (uint32_t i = 0; i < nl; ++i) {
    if (r.off >= len) {
      err = "unexpected end of data before layer " + std::to_string(i);
      return false;
    }
    const int tag = (int)d[r.off++] - base;
    NNLayer L;
    L.kind = tag;
    uint32_t u = 0, v = 0;
    switch (tag) {
      case ARCNN_DENSE:
        if (!r.u32(u) || !r.u32(v) || !r.f32s(L.a, (uint64_t)u * v) || !r.f32s(L.b, u)) break;
        L.rows = u;
        L.cols = v;
        break;
      case ARCNN_RELU:
      case ARCNN_SOFTMAX:
        break;
      case ARCNN_LAYERNORM: {
        std::vector<float> e;
        if (!r.u32(u) || !r.f32s(L.a, u) || !r.f32s(L.b, u) || !r.f32s(e, 1)) break;
        L.rows = u;
        L.eps = e[0];
        break;
      }
      case ARCNN_EMBEDDING:
        if (!r.u32(u) || !r.u32(v) || !r.f32s(L.a, (uint64_t)u * v)) break;
        L.rows = u;
        L.cols = v;
        break;
      default:
        err = "unknown layer tag " + std::to_string(tag + base) + " at layer " + std::to_string(i);
        return false;
    }
    if (!r.err.empty()) {
      err = r.err;
      return false;
    }
    out.push_back(std::move(L));
  }
  used = r.off;
  return true;
}

}  // namespace

struct arcnn_net {
  std::vector<NNLayer> layers;
  int tag_base = 0;
};

extern "C" {

static arcnn_net* parse(const uint8_t* data, size_t len, char* err, int errlen) {
  std::vector<NNLayer> layers;
  std::string e, first_err;
  size_t used = 0;
  int pick = -1;
  for (int base = 0; base <= 1 && pick < 0; ++base) {
    if (parse_with(data, len, base, layers, used, e) && used == len) pick = base;
    if (base == 0) first_err = e;
  }
  if (pick < 0) {
    // the VM's own rule: numbering 0..4, bytes after the last layer ignored
    if (parse_with(data, len, 0, layers, used, e)) {
      pick = 0;
    } else {
      if (err && errlen > 0) snprintf(err, (size_t)errlen, "%s", first_err.c_str());
      return nullptr;
    }
  }
  auto* net = new arcnn_net();
  net->layers = std::move(layers);
  net->tag_base = pick;
  for (auto& L : net->layers) build_int(L);
  return net;
}

// No C++ exception (an allocation failure on a huge but well-formed file)
// crosses the C ABI.
arcnn_net* arcnn_parse(const uint8_t* data, size_t len, char* err, int errlen) {
  try {
    return parse(data, len, err, errlen);
  } catch (const std::exception& e) {
    if (err && errlen > 0) snprintf(err, (size_t)errlen, "parse failed: %s", e.what());
    return nullptr;
  }
}

arcnn_net* arcnn_new(void) { return new arcnn_net(); }

static int add_layer(arcnn_net* net, int kind, int64_t rows, int64_t cols, const float* a,
                     const float* b, float eps) {
  NNLayer L;
  L.kind = kind;
  switch (kind) {
    case ARCNN_DENSE:
      L.rows = rows;
      L.cols = cols;
      L.a.assign(a, a + rows * cols);
      L.b.assign(b, b + rows);
      break;
    case ARCNN_LAYERNORM:
      L.rows = rows;
      L.a.assign(a, a + rows);
      L.b.assign(b, b + rows);
      L.eps = eps;
      break;
    case ARCNN_EMBEDDING:
      L.rows = rows;
      L.cols = cols;
      L.a.assign(a, a + rows * cols);
      break;
    case ARCNN_RELU:
    case ARCNN_SOFTMAX:
      break;
    default:
      return -1;
  }
  build_int(L);
  net->layers.push_back(std::move(L));
  return 0;
}

int arcnn_add_layer(arcnn_net* net, int kind, int64_t rows, int64_t cols, const float* a,
                    const float* b, float eps) {
  try {
    return add_layer(net, kind, rows, cols, a, b, eps);
  } catch (const std::exception&) {
    return -2;
  }
}

void arcnn_free(arcnn_net* net) { delete net; }

int arcnn_tag_base(const arcnn_net* net) { return net->tag_base; }
int64_t arcnn_num_layers(const arcnn_net* net) { return (int64_t)net->layers.size(); }

int arcnn_layer(const arcnn_net* net, int64_t i, int64_t* rows, int64_t* cols, float* eps) {
  if (i < 0 || i >= (int64_t)net->layers.size()) return -1;
  const NNLayer& L = net->layers[(size_t)i];
  if (rows) *rows = L.rows;
  if (cols) *cols = L.cols;
  if (eps) *eps = L.eps;
  return L.kind;
}

int64_t arcnn_layer_data(const arcnn_net* net, int64_t i, int which, float* out, int64_t cap) {
  if (i < 0 || i >= (int64_t)net->layers.size()) return -1;
  const std::vector<float>& v = which == 0 ? net->layers[(size_t)i].a : net->layers[(size_t)i].b;
  if (out && cap >= (int64_t)v.size() && !v.empty()) memcpy(out, v.data(), v.size() * 4);
  return (int64_t)v.size();
}

int64_t arcnn_input_size(const arcnn_net* net) {
  for (const auto& L : net->layers) {
    if (L.kind == ARCNN_DENSE) return L.rows == 0 ? 0 : L.cols;
    if (L.kind == ARCNN_EMBEDDING) return L.rows;
    if (L.kind == ARCNN_LAYERNORM) return L.rows;
  }
  return 0;
}

int64_t arcnn_output_size(const arcnn_net* net) {
  for (auto it = net->layers.rbegin(); it != net->layers.rend(); ++it) {
    if (it->kind == ARCNN_DENSE) return it->rows;
    if (it->kind == ARCNN_EMBEDDING) return emb_dim(*it);
    if (it->kind == ARCNN_LAYERNORM) return it->rows;
  }
  return 0;
}

int64_t arcnn_serialize(const arcnn_net* net, int tag_base, uint8_t* out, int64_t cap) {
  std::vector<uint8_t> buf;
  auto put32 = [&](uint32_t v) {
    uint8_t t[4];
    memcpy(t, &v, 4);
    buf.insert(buf.end(), t, t + 4);
  };
  auto putf = [&](const std::vector<float>& v) {
    const uint8_t* p = (const uint8_t*)v.data();
    buf.insert(buf.end(), p, p + v.size() * 4);
  };
  put32((uint32_t)net->layers.size());
  for (const auto& L : net->layers) {
    buf.push_back((uint8_t)(L.kind + tag_base));
    switch (L.kind) {
      case ARCNN_DENSE:  // an empty weight list has no first row: cols is written as 0
        put32((uint32_t)L.rows);
        put32((uint32_t)(L.rows == 0 ? 0 : L.cols));
        putf(L.a);
        putf(L.b);
        break;
      case ARCNN_LAYERNORM: {
        put32((uint32_t)L.rows);
        putf(L.a);
        putf(L.b);
        std::vector<float> e{L.eps};
        putf(e);
        break;
      }
      case ARCNN_EMBEDDING:
        put32((uint32_t)L.rows);
        put32((uint32_t)emb_dim(L));
        putf(L.a);
        break;
      default:
        break;
    }
  }
  if (out && cap >= (int64_t)buf.size()) memcpy(out, buf.data(), buf.size());
  return (int64_t)buf.size();
}

int64_t arcnn_output_len(const arcnn_net* net, int64_t n) {
  for (const auto& L : net->layers) {
    if (L.kind == ARCNN_DENSE) n = L.rows;
    else if (L.kind == ARCNN_EMBEDDING) n *= emb_dim(L);
  }
  return n;
}

void arcnn_softmax_f32(const float* x, int64_t n, float* out) {
  if (n == 0) return;
  float mx = -INFINITY;
  for (int64_t i = 0; i < n; ++i) mx = fmaxf(mx, x[i]);
  for (int64_t i = 0; i < n; ++i) out[i] = expf(x[i] - mx);
  const float s = fold_sum(out, n);
  if (s == 0.0f) {
    const float u = 1.0f / (float)n;
    for (int64_t i = 0; i < n; ++i) out[i] = u;
    return;
  }
  for (int64_t i = 0; i < n; ++i) out[i] = out[i] / s;
}

int64_t arcnn_forward_f32(const arcnn_net* net, const float* x, int64_t n, float* out, int64_t cap) {
  const int64_t total = arcnn_output_len(net, n);
  if (!out || cap < total) return total;
  std::vector<float> a(x, x + n), nx;
  for (const auto& L : net->layers) {
    const int64_t m = (int64_t)a.size();
    switch (L.kind) {
      case ARCNN_DENSE: {
        nx.assign((size_t)L.rows, 0.0f);
        const int64_t k = std::min(L.cols, m);
        for (int64_t i = 0; i < L.rows; ++i) {
          const float* w = L.a.data() + i * L.cols;
          float acc = L.b[(size_t)i];
          for (int64_t j = 0; j < k; ++j) acc += w[j] * a[(size_t)j];
          nx[(size_t)i] = acc;
        }
        a.swap(nx);
        break;
      }
      case ARCNN_RELU:
        for (auto& v : a) v = v > 0.0f ? v : 0.0f;
        break;
      case ARCNN_SOFTMAX:
        nx.resize(a.size());
        arcnn_softmax_f32(a.data(), m, nx.data());
        a.swap(nx);
        break;
      case ARCNN_LAYERNORM: {
        const float nf = (float)m;
        const float mean = fold_sum(a.data(), m) / nf;
        float vs = -0.0f;
        for (int64_t i = 0; i < m; ++i) vs = vs + (a[(size_t)i] - mean) * (a[(size_t)i] - mean);
        const float inv = 1.0f / sqrtf(vs / nf + L.eps);
        for (int64_t i = 0; i < m; ++i) {
          const float g = i < (int64_t)L.a.size() ? L.a[(size_t)i] : 1.0f;
          const float b = i < (int64_t)L.b.size() ? L.b[(size_t)i] : 0.0f;
          a[(size_t)i] = (a[(size_t)i] - mean) * inv * g + b;
        }
        break;
      }
      case ARCNN_EMBEDDING: {
        const int64_t dim = emb_dim(L);
        nx.assign((size_t)(m * dim), 0.0f);
        for (int64_t t = 0; t < m; ++t) {
          const int64_t r = emb_index_f32(a[(size_t)t], L.rows);
          if (r >= 0) std::copy_n(L.a.data() + r * L.cols, dim, nx.data() + t * dim);
        }
        a.swap(nx);
        break;
      }
      default:
        break;
    }
  }
  std::copy(a.begin(), a.end(), out);
  return total;
}

int64_t arcnn_forward_q16(const arcnn_net* net, const int64_t* x, int64_t n, int64_t* out,
                          int64_t cap) {
  using q16::wadd;
  using q16::wmul;
  using q16::wsub;
  const int64_t total = arcnn_output_len(net, n);
  if (!out || cap < total) return total;
  std::vector<int64_t> a(x, x + n), nx;
  for (const auto& L : net->layers) {
    const int64_t m = (int64_t)a.size();
    switch (L.kind) {
      case ARCNN_DENSE: {
        nx.assign((size_t)L.rows, 0);
        const int64_t k = std::min(L.cols, m);
        for (int64_t i = 0; i < L.rows; ++i) {
          const int8_t* w = L.qw.data() + i * L.cols;
          int64_t acc = 0;
          for (int64_t j = 0; j < k; ++j) acc = wadd(acc, wmul(w[j], a[(size_t)j]));
          nx[(size_t)i] = wadd(wmul(acc, L.qs[(size_t)i]) >> 16, L.qb[(size_t)i]);
        }
        a.swap(nx);
        break;
      }
      case ARCNN_RELU:
        for (auto& v : a) v = std::max<int64_t>(v, 0);
        break;
      case ARCNN_SOFTMAX:
        nx.resize(a.size());
        arcref_softmax(a.data(), m, nx.data());
        a.swap(nx);
        break;
      case ARCNN_LAYERNORM: {
        if (m == 0) break;
        int64_t s = 0;
        for (auto v : a) s = wadd(s, v);
        const int64_t mean = s / m;
        int64_t vs = 0;
        for (auto v : a) {
          const int64_t d = wsub(v, mean);
          vs = wadd(vs, wmul(d, d) >> 16);
        }
        const int64_t inv = q16::integer_isqrt(std::max<int64_t>(1, wadd(vs / m, L.qeps)));
        for (int64_t i = 0; i < m; ++i) {
          const int64_t g = i < (int64_t)L.qa.size() ? L.qa[(size_t)i] : ONE;
          const int64_t b = i < (int64_t)L.qb.size() ? L.qb[(size_t)i] : 0;
          a[(size_t)i] = wadd(q16::mulshr(q16::mulshr(wsub(a[(size_t)i], mean), inv), g), b);
        }
        break;
      }
      case ARCNN_EMBEDDING: {
        const int64_t dim = emb_dim(L);
        nx.assign((size_t)(m * dim), 0);
        for (int64_t t = 0; t < m; ++t) {
          const int64_t r = emb_index_q16(a[(size_t)t], L.rows);
          if (r >= 0) std::copy_n(L.qa.data() + r * L.cols, dim, nx.data() + t * dim);
        }
        a.swap(nx);
        break;
      }
      default:
        break;
    }
  }
  std::copy(a.begin(), a.end(), out);
  return total;
}

}  // extern "C"
