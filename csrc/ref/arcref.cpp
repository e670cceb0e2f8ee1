// arcref: the CPU oracle.  Bit-exact restatement of CachedIntegerModel
// (crates/arc-inference/src/cached_integer_model.rs) written from its
// semantics; see arcref.h for the API.
#include "arcref.h"

#include <fcntl.h>
#include <stdio.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <condition_variable>
#include <functional>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../common/q16.h"
#include "blake3.h"
#include "../common/rng.h"

using namespace q16;

// ---------------------------------------------------------------------------
// Thread pool: one parallel_for at a time, static chunking.
// ---------------------------------------------------------------------------
namespace {

// Set on the pool's worker threads: a parallel_for issued from inside a job
// runs inline instead of waiting for the pool that is running it.
thread_local bool t_pool_worker = false;

// One job at a time: callers on other host threads (ctypes releases the GIL)
// queue on call_mu_ rather than sharing the job slot.
class Pool {
 public:
  explicit Pool(int n) { resize(n); }
  ~Pool() { stop(); }
  int size() const { return threads_; }
  // Not concurrent with parallel_for.  New workers start at the current job
  // generation, so they wait for the next job instead of taking a finished
  // one.
  void resize(int n) {
    std::lock_guard<std::mutex> call(call_mu_);
    stop();
    if (n < 1) n = 1;
    quit_ = false;
    threads_ = n;
    const uint64_t g = gen_;
    for (int i = 0; i < n - 1; ++i) workers_.emplace_back([this, i, g] { loop(i + 1, g); });
  }
  // Runs f(lo, hi) over [0, n) split into size() contiguous ranges.
  void parallel_for(int64_t n, const std::function<void(int64_t, int64_t)>& f) {
    if (n < 2 || t_pool_worker) {
      f(0, n);
      return;
    }
    std::lock_guard<std::mutex> call(call_mu_);
    const int t = size();
    if (t == 1) {
      f(0, n);
      return;
    }
    {
      std::unique_lock<std::mutex> lk(mu_);
      job_ = &f;
      n_ = n;
      pending_ = t - 1;
      ++gen_;
    }
    cv_.notify_all();
    run_range(0, t, n, f);
    std::unique_lock<std::mutex> lk(mu_);
    done_cv_.wait(lk, [this] { return pending_ == 0; });
    job_ = nullptr;
  }

 private:
  static void run_range(int idx, int t, int64_t n, const std::function<void(int64_t, int64_t)>& f) {
    int64_t per = (n + t - 1) / t;
    int64_t lo = idx * per, hi = std::min<int64_t>(n, lo + per);
    if (lo < hi) f(lo, hi);
  }
  void loop(int idx, uint64_t seen) {
    t_pool_worker = true;
    for (;;) {
      const std::function<void(int64_t, int64_t)>* job;
      int64_t n;
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] { return quit_ || gen_ != seen; });
        if (quit_) return;
        seen = gen_;
        job = job_;
        n = n_;
      }
      run_range(idx, size(), n, *job);
      std::unique_lock<std::mutex> lk(mu_);
      if (--pending_ == 0) done_cv_.notify_all();
    }
  }
  void stop() {
    {
      std::unique_lock<std::mutex> lk(mu_);
      quit_ = true;
    }
    cv_.notify_all();
    for (auto& w : workers_) w.join();
    workers_.clear();
  }
  std::vector<std::thread> workers_;
  std::mutex call_mu_, mu_;
  std::condition_variable cv_, done_cv_;
  const std::function<void(int64_t, int64_t)>* job_ = nullptr;
  int64_t n_ = 0;
  int threads_ = 1;
  int pending_ = 0;
  uint64_t gen_ = 0;
  bool quit_ = false;
};

Pool& pool() {
  static Pool p([] {
    const char* e = getenv("ARCREF_THREADS");
    int n = e ? atoi(e) : (int)std::thread::hardware_concurrency();
    return n > 0 ? n : 1;
  }());
  return p;
}

const int64_t* exp_lut() {
  static int64_t t[EXP_LUT_N];
  static bool init = [] {
    build_exp_lut(t);
    return true;
  }();
  (void)init;
  return t;
}

// ---------------------------------------------------------------------------
// Weights
// ---------------------------------------------------------------------------
struct I8W {
  const int8_t* data = nullptr;
  const int64_t* scales = nullptr;
  int64_t rows = 0, cols = 0;
};

// Reference per-row Q4 (Q4WeightsX86): bias-8 nibbles, low nibble = even col.
struct Q4W {
  std::vector<uint8_t> data;
  std::vector<int64_t> scales;
  int64_t rows = 0, cols = 0;
};

struct Vec64 {
  const int64_t* p = nullptr;
  int64_t n = 0;
};

struct Layer {
  I8W wq, wk, wv, wo, gate, up, down;
  Vec64 attn_norm, ffn_norm;
};

// Q4WeightsX86::from_i8 (cached_integer_model.rs:670-701).
Q4W q4_from_i8(const I8W& w) {
  Q4W q;
  q.rows = w.rows;
  q.cols = w.cols;
  int64_t bc = (w.cols + 1) / 2;
  q.data.resize(w.rows * bc);
  q.scales.resize(w.rows);
  for (int64_t i = 0; i < w.rows; ++i) {
    const int8_t* row = w.data + i * w.cols;
    int am = 1;
    for (int64_t j = 0; j < w.cols; ++j) am = std::max(am, std::abs((int)row[j]));
    int64_t qpu = std::max<int64_t>(1, (am + 6) / 7);
    for (int64_t p = 0; p < bc; ++p) {
      int v0 = std::clamp<int>((int16_t)row[2 * p] / (int16_t)qpu, -8, 7);
      int v1 = 2 * p + 1 < w.cols ? std::clamp<int>((int16_t)row[2 * p + 1] / (int16_t)qpu, -8, 7) : 0;
      q.data[i * bc + p] = (uint8_t)(((v0 + 8) & 0xF) | (((v1 + 8) & 0xF) << 4));
    }
    q.scales[i] = wmul(w.scales[i], qpu);
  }
  return q;
}

// dot_i8_i64 (221-245): wrapping i64 sum of i8*i64.  The order of a wrapping
// sum does not change its value, so any vectorisation is exact.
__attribute__((target_clones("avx512f", "avx2", "default")))
int64_t dot_i8_i64(const int8_t* w, const int64_t* x, int64_t n) {
  uint64_t acc = 0;
  for (int64_t j = 0; j < n; ++j) acc += (uint64_t)(int64_t)w[j] * (uint64_t)x[j];
  return (int64_t)acc;
}

int64_t dot_q4_i64(const uint8_t* d, const int64_t* x, int64_t cols) {
  uint64_t acc = 0;
  int64_t bc = cols / 2;
  for (int64_t p = 0; p < bc; ++p) {
    int64_t lo = (int64_t)(d[p] & 0xF) - 8, hi = (int64_t)(d[p] >> 4) - 8;
    acc += (uint64_t)lo * (uint64_t)x[2 * p] + (uint64_t)hi * (uint64_t)x[2 * p + 1];
  }
  return (int64_t)acc;
}

void matmul_i8(const I8W& w, const int64_t* x, int64_t* out) {
  auto body = [&](int64_t lo, int64_t hi) {
    for (int64_t i = lo; i < hi; ++i)
      out[i] = mulshr(dot_i8_i64(w.data + i * w.cols, x, w.cols), w.scales[i]);
  };
  if (w.rows * w.cols < (1 << 20)) body(0, w.rows);
  else pool().parallel_for(w.rows, body);
}

// matmul_q4_full (955-978).
void matmul_q4(const Q4W& w, const int64_t* x, int64_t* out) {
  int64_t bc = w.cols / 2;
  auto body = [&](int64_t lo, int64_t hi) {
    for (int64_t i = lo; i < hi; ++i)
      out[i] = mulshr(dot_q4_i64(w.data.data() + i * bc, x, w.cols), w.scales[i]);
  };
  if (w.rows * w.cols < (1 << 20)) body(0, w.rows);
  else pool().parallel_for(w.rows, body);
}

// layernorm (985-1000): RMSNorm with gamma = ONE past gamma's end.
void rmsnorm(const int64_t* x, int64_t n, const int64_t* g, int64_t ng, int64_t* out) {
  if (n == 0) return;
  int64_t ss = 0;
  for (int64_t i = 0; i < n; ++i) ss = wadd(ss, wmul(x[i], x[i]) >> FRAC_BITS);
  int64_t inv = rms_inv(ss, n);
  for (int64_t i = 0; i < n; ++i) out[i] = rms_apply(x[i], inv, i < ng ? g[i] : ONE);
}

void softmax(const int64_t* x, int64_t n, int64_t* out) {
  if (n == 0) return;
  if (n == 1) {
    out[0] = ONE;
    return;
  }
  const int64_t* lut = exp_lut();
  int64_t m = x[0];
  for (int64_t i = 1; i < n; ++i) m = std::max(m, x[i]);
  int64_t s = 0;
  for (int64_t i = 0; i < n; ++i) {
    out[i] = integer_exp(wsub(x[i], m), lut);
    s = wadd(s, out[i]);
  }
  if (s == 0) {
    for (int64_t i = 0; i < n; ++i) out[i] = ONE / n;
    return;
  }
  for (int64_t i = 0; i < n; ++i) out[i] = wmul(out[i], ONE) / s;
}

}  // namespace

// ---------------------------------------------------------------------------
// Model
// ---------------------------------------------------------------------------
struct arcref_model {
  arcref_config cfg{};
  I8W emb, out;
  // Full-precision Q16 embedding [vocab, d] (GGUF-loaded models keep one:
  // cached_integer_model.rs:1719-1723); null -> i8 * scale per row.
  const int64_t* emb_q16 = nullptr;
  Vec64 final_norm, rope_cos, rope_sin;
  std::vector<Layer> layers;
  // Q4 mode
  bool q4 = false;
  std::vector<Q4W> q4w;  // per layer 7 matrices, then the LM head
  // storage for file loads
  void* map = nullptr;
  size_t map_len = 0;
  std::vector<int64_t> owned;  // aligned copies of i64 vectors from the file
  // vocab JSON bytes of the loaded file, written back verbatim by
  // arcref_save_file; "[]" (an empty list) when there is none
  std::string vocab_json = "[]";
};

struct arcref_cache {
  std::vector<std::vector<int64_t>> k, v;
  int64_t seq_len = 0;
  // set when a forward was asked for a position past the RoPE tables (the
  // reference indexes them unchecked and panics there)
  bool overflow = false;
  std::vector<int64_t> last_hidden;
};

namespace {

struct Reader {
  const uint8_t* p;
  size_t n, off = 0;
  bool ok = true;
  std::string err;
  // Compares against the bytes left (no off + k, which a corrupted size
  // field could wrap).
  bool need(size_t k, const char* what) {
    if (!ok) return false;
    if (k > n - off) {
      ok = false;
      err = std::string("truncated file reading ") + what;
      return false;
    }
    return true;
  }
  // `count` items of `size` bytes, checked before anything is allocated.
  bool need_items(uint64_t count, uint64_t size, const char* what) {
    if (!ok) return false;
    if (size && count > (n - off) / size) {
      ok = false;
      err = std::string("size field exceeds the file reading ") + what;
      return false;
    }
    return true;
  }
  uint64_t u64(const char* what) {
    if (!need(8, what)) return 0;
    uint64_t v;
    memcpy(&v, p + off, 8);
    off += 8;
    return v;
  }
};

// Reads `vec` (u64 len + LE i64 items) into owned storage; returns offset.
bool read_vec(Reader& r, std::vector<std::pair<size_t, size_t>>& spans, std::vector<int64_t>& owned,
              const char* what) {
  uint64_t len = r.u64(what);
  if (!r.need_items(len, 8, what)) return false;
  size_t at = owned.size();
  owned.resize(at + len);
  memcpy(owned.data() + at, r.p + r.off, len * 8);
  r.off += len * 8;
  spans.push_back({at, (size_t)len});
  return true;
}

bool read_i8w(Reader& r, I8W& w, std::vector<std::pair<size_t, size_t>>& spans,
              std::vector<int64_t>& owned, const char* what) {
  const uint64_t rows = r.u64(what), cols = r.u64(what);
  uint64_t bytes = 0;
  if (!r.need_items(rows, 8, what)) return false;
  if (__builtin_mul_overflow(rows, cols, &bytes) || bytes > r.n - r.off - rows * 8) {
    r.ok = false;
    r.err = std::string("size field exceeds the file reading ") + what;
    return false;
  }
  w.rows = (int64_t)rows;
  w.cols = (int64_t)cols;
  size_t at = owned.size();
  owned.resize(at + w.rows);
  memcpy(owned.data() + at, r.p + r.off, w.rows * 8);
  spans.push_back({at, (size_t)w.rows});
  r.off += w.rows * 8;
  if (!r.need((size_t)(w.rows * w.cols), what)) return false;
  w.data = (const int8_t*)(r.p + r.off);
  r.off += w.rows * w.cols;
  return true;
}

}  // namespace

extern "C" {

static arcref_model* load_file(const char* path, char* err, int errlen) {
  auto fail = [&](const std::string& m) -> arcref_model* {
    if (err && errlen > 0) snprintf(err, errlen, "%s", m.c_str());
    return nullptr;
  };
  int fd = open(path, O_RDONLY);
  if (fd < 0) return fail(std::string("open failed: ") + path);
  struct stat st;
  fstat(fd, &st);
  size_t len = (size_t)st.st_size;
  void* map = mmap(nullptr, len, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (map == MAP_FAILED) return fail("mmap failed");
  auto* m = new arcref_model();
  m->map = map;
  m->map_len = len;
  Reader r{(const uint8_t*)map, len};
  if (len < 10 || memcmp(map, "ARC-INT8", 8) != 0) {
    arcref_free(m);
    return fail("Not an ARC-INT8 file");
  }
  r.off = 10;  // magic + version + minor (minor byte ignored, as the reference does)
  arcref_config& c = m->cfg;
  c.n_layers = r.u64("cfg");
  c.d_model = r.u64("cfg");
  c.n_heads = r.u64("cfg");
  c.n_kv_heads = r.u64("cfg");
  c.d_ff = r.u64("cfg");
  c.d_head = r.u64("cfg");
  c.d_kv = r.u64("cfg");
  c.vocab = r.u64("cfg");
  c.max_seq = r.u64("cfg");
  c.attn_scale = (int64_t)r.u64("attn_scale");
  std::vector<std::pair<size_t, size_t>> spans;
  read_vec(r, spans, m->owned, "rope_cos");
  read_vec(r, spans, m->owned, "rope_sin");
  read_i8w(r, m->emb, spans, m->owned, "embedding");
  read_i8w(r, m->out, spans, m->owned, "output");
  read_vec(r, spans, m->owned, "final_norm");
  // every layer holds 7 matrices (16-byte headers) and 2 vectors (8-byte
  // lengths) at least: a larger count is a corrupted header, refused before
  // anything is allocated for it
  if (r.ok && c.n_layers > 0 && (uint64_t)c.n_layers > (r.n - r.off) / (7 * 16 + 2 * 8)) {
    arcref_free(m);
    return fail("layer count exceeds the file");
  }
  m->layers.resize(c.n_layers);
  for (int64_t l = 0; l < c.n_layers && r.ok; ++l) {
    Layer& L = m->layers[l];
    read_i8w(r, L.wq, spans, m->owned, "wq");
    read_i8w(r, L.wk, spans, m->owned, "wk");
    read_i8w(r, L.wv, spans, m->owned, "wv");
    read_i8w(r, L.wo, spans, m->owned, "wo");
    read_i8w(r, L.gate, spans, m->owned, "gate");
    read_i8w(r, L.up, spans, m->owned, "up");
    read_i8w(r, L.down, spans, m->owned, "down");
    read_vec(r, spans, m->owned, "attn_norm");
    read_vec(r, spans, m->owned, "ffn_norm");
  }
  if (!r.ok) {
    std::string e = r.err;
    arcref_free(m);
    return fail(e);
  }
  // u64 length + vocab JSON; a missing or short tail leaves the empty list
  if (len - r.off >= 8) {
    uint64_t vl;
    memcpy(&vl, r.p + r.off, 8);
    if (len - r.off - 8 >= vl) m->vocab_json.assign((const char*)r.p + r.off + 8, (size_t)vl);
  }
  // Resolve spans now that `owned` has stopped growing.
  size_t si = 0;
  auto vec_at = [&](Vec64& v) {
    v.p = m->owned.data() + spans[si].first;
    v.n = (int64_t)spans[si].second;
    ++si;
  };
  auto sc_at = [&](I8W& w) {
    w.scales = m->owned.data() + spans[si].first;
    ++si;
  };
  vec_at(m->rope_cos);
  vec_at(m->rope_sin);
  sc_at(m->emb);
  sc_at(m->out);
  vec_at(m->final_norm);
  for (auto& L : m->layers) {
    sc_at(L.wq);
    sc_at(L.wk);
    sc_at(L.wv);
    sc_at(L.wo);
    sc_at(L.gate);
    sc_at(L.up);
    sc_at(L.down);
    vec_at(L.attn_norm);
    vec_at(L.ffn_norm);
  }
  // the forward pass indexes every matrix with the config's dimensions
  std::string bad;
  auto want = [&](const I8W& w, int64_t rows, int64_t cols, const char* name) {
    if (bad.empty() && (w.rows != rows || w.cols != cols))
      bad = std::string(name) + " is " + std::to_string(w.rows) + " x " + std::to_string(w.cols) +
            ", the config needs " + std::to_string(rows) + " x " + std::to_string(cols);
  };
  if (c.n_heads < 1 || c.n_kv_heads < 1 || c.d_head < 2 || c.n_heads * c.d_head != c.d_model ||
      c.n_kv_heads * c.d_head != c.d_kv || c.vocab < 1)
    bad = "inconsistent config (heads x d_head must equal d_model and d_kv)";
  want(m->emb, c.vocab, c.d_model, "embedding");
  want(m->out, c.vocab, c.d_model, "output");
  for (const Layer& L : m->layers) {
    want(L.wq, c.d_model, c.d_model, "wq");
    want(L.wk, c.d_kv, c.d_model, "wk");
    want(L.wv, c.d_kv, c.d_model, "wv");
    want(L.wo, c.d_model, c.d_model, "wo");
    want(L.gate, c.d_ff, c.d_model, "gate");
    want(L.up, c.d_ff, c.d_model, "up");
    want(L.down, c.d_model, c.d_ff, "down");
  }
  if (!bad.empty()) {
    arcref_free(m);
    return fail(bad);
  }
  return m;
}

arcref_model* arcref_load_file(const char* path, char* err, int errlen) {
  try {
    return load_file(path, err, errlen);
  } catch (const std::exception& e) {  // no C++ exception crosses the C ABI
    if (err && errlen > 0) snprintf(err, errlen, "load failed: %s", e.what());
    return nullptr;
  }
}

int arcref_save_file(const arcref_model* m, const char* path, const char* vocab_json,
                     int64_t vocab_len, char* err, int errlen) {
  FILE* f = fopen(path, "wb");
  if (!f) {
    if (err && errlen > 0) snprintf(err, errlen, "open failed: %s", path);
    return -1;
  }
  bool ok = true;
  auto put = [&](const void* p, size_t n) {
    if (ok && n) ok = fwrite(p, 1, n, f) == n;
  };
  auto u64 = [&](uint64_t v) { put(&v, 8); };
  auto vec = [&](const Vec64& v) {
    u64((uint64_t)v.n);
    put(v.p, (size_t)v.n * 8);
  };
  auto i8w = [&](const I8W& w) {
    u64((uint64_t)w.rows);
    u64((uint64_t)w.cols);
    put(w.scales, (size_t)w.rows * 8);
    put(w.data, (size_t)(w.rows * w.cols));
  };
  const arcref_config& c = m->cfg;
  put("ARC-INT8\x02\x00", 10);
  for (int64_t v : {c.n_layers, c.d_model, c.n_heads, c.n_kv_heads, c.d_ff, c.d_head, c.d_kv,
                    c.vocab, c.max_seq})
    u64((uint64_t)v);
  u64((uint64_t)c.attn_scale);
  vec(m->rope_cos);
  vec(m->rope_sin);
  i8w(m->emb);
  i8w(m->out);
  vec(m->final_norm);
  for (const Layer& L : m->layers) {
    for (const I8W* w : {&L.wq, &L.wk, &L.wv, &L.wo, &L.gate, &L.up, &L.down}) i8w(*w);
    vec(L.attn_norm);
    vec(L.ffn_norm);
  }
  const char* vj = vocab_json ? vocab_json : m->vocab_json.data();
  const size_t vl = vocab_json ? (size_t)vocab_len : m->vocab_json.size();
  u64((uint64_t)vl);
  put(vj, vl);
  ok = (fclose(f) == 0) && ok;
  if (!ok && err && errlen > 0) snprintf(err, errlen, "write failed: %s", path);
  return ok ? 0 : -1;
}

arcref_model* arcref_from_arrays(const arcref_config* cfg, const void* const* ptrs,
                                 const int64_t* lens) {
  auto* m = new arcref_model();
  m->cfg = *cfg;
  const arcref_config& c = m->cfg;
  int pi = 0, li = 0;
  auto i8w = [&](I8W& w, int64_t rows, int64_t cols) {
    w.data = (const int8_t*)ptrs[pi++];
    w.scales = (const int64_t*)ptrs[pi++];
    w.rows = rows;
    w.cols = cols;
  };
  i8w(m->emb, c.vocab, c.d_model);
  i8w(m->out, c.vocab, c.d_model);
  m->final_norm = {(const int64_t*)ptrs[pi++], lens[li++]};
  int64_t rl = lens[li++];
  m->rope_cos = {(const int64_t*)ptrs[pi++], rl};
  m->rope_sin = {(const int64_t*)ptrs[pi++], rl};
  m->layers.resize(c.n_layers);
  for (auto& L : m->layers) {
    i8w(L.wq, c.d_model, c.d_model);
    i8w(L.wk, c.d_kv, c.d_model);
    i8w(L.wv, c.d_kv, c.d_model);
    i8w(L.wo, c.d_model, c.d_model);
    i8w(L.gate, c.d_ff, c.d_model);
    i8w(L.up, c.d_ff, c.d_model);
    i8w(L.down, c.d_model, c.d_ff);
    L.attn_norm = {(const int64_t*)ptrs[pi++], lens[li++]};
    L.ffn_norm = {(const int64_t*)ptrs[pi++], lens[li++]};
  }
  return m;
}

void arcref_free(arcref_model* m) {
  if (!m) return;
  if (m->map) munmap(m->map, m->map_len);
  delete m;
}

void arcref_get_config(const arcref_model* m, arcref_config* out) { *out = m->cfg; }

void arcref_enable_q4(arcref_model* m) {
  m->q4w.clear();
  for (auto& L : m->layers)
    for (const I8W* w : {&L.wq, &L.wk, &L.wv, &L.wo, &L.gate, &L.up, &L.down})
      m->q4w.push_back(q4_from_i8(*w));
  m->q4w.push_back(q4_from_i8(m->out));
  m->q4 = true;
}

arcref_cache* arcref_cache_new(const arcref_model* m) {
  auto* c = new arcref_cache();
  c->k.resize(m->cfg.n_layers);
  c->v.resize(m->cfg.n_layers);
  return c;
}
void arcref_cache_free(arcref_cache* c) { delete c; }
int arcref_cache_overflow(const arcref_cache* c) { return c->overflow ? 1 : 0; }
int64_t arcref_cache_len(const arcref_cache* c) { return c->seq_len; }
void arcref_cache_truncate(arcref_cache* c, int64_t len) {
  if (len >= c->seq_len) return;
  for (size_t l = 0; l < c->k.size(); ++l) {
    size_t per = c->seq_len ? c->k[l].size() / c->seq_len : 0;
    c->k[l].resize(per * len);
    c->v[l].resize(per * len);
  }
  c->seq_len = len;
}
void arcref_last_hidden(const arcref_cache* c, int64_t* out) {
  std::copy(c->last_hidden.begin(), c->last_hidden.end(), out);
}

// forward_one_token (1381-1516).
void arcref_forward(arcref_model* m, arcref_cache* cache, uint32_t token, int64_t* logits) {
  const arcref_config& c = m->cfg;
  const int64_t d = c.d_model, dh = c.d_head, half = dh / 2;
  const int64_t pos = cache->seq_len;
  if ((pos + 1) * half > m->rope_cos.n || (pos + 1) * half > m->rope_sin.n) {
    cache->overflow = true;
    std::fill(logits, logits + c.vocab, 0);
    return;
  }
  const int64_t* lut = exp_lut();
  int64_t idx = std::min<int64_t>((int64_t)token, c.vocab - 1);
  std::vector<int64_t> h(d), n(d), q(d), kb(c.d_kv), vb(c.d_kv), ao(d), pr(d), g(c.d_ff),
      u(c.d_ff), fo(d);
  // embedding_q16: the model's own table, or i8 * scale (1821-1830)
  if (m->emb_q16)
    for (int64_t j = 0; j < d; ++j) h[j] = m->emb_q16[idx * d + j];
  else
    for (int64_t j = 0; j < d; ++j) h[j] = wmul((int64_t)m->emb.data[idx * d + j], m->emb.scales[idx]);
  auto mm = [&](int li, const I8W& w, const int64_t* x, int64_t* o) {
    if (m->q4) matmul_q4(m->q4w[li], x, o);
    else matmul_i8(w, x, o);
  };
  for (int64_t l = 0; l < c.n_layers; ++l) {
    const Layer& L = m->layers[l];
    int base = (int)(l * 7);
    rmsnorm(h.data(), d, L.attn_norm.p, L.attn_norm.n, n.data());
    mm(base + 0, L.wq, n.data(), q.data());
    mm(base + 1, L.wk, n.data(), kb.data());
    mm(base + 2, L.wv, n.data(), vb.data());
    auto rope = [&](int64_t* v) {
      for (int64_t i = 0; i < half; ++i)
        rope_pair(v[i], v[i + half], m->rope_cos.p[pos * half + i], m->rope_sin.p[pos * half + i]);
    };
    for (int64_t hh = 0; hh < c.n_heads; ++hh) rope(q.data() + hh * dh);
    for (int64_t hh = 0; hh < c.n_kv_heads; ++hh) rope(kb.data() + hh * dh);
    auto& K = cache->k[l];
    auto& V = cache->v[l];
    K.insert(K.end(), kb.begin(), kb.end());
    V.insert(V.end(), vb.begin(), vb.end());
    const int64_t T = pos + 1;
    auto head = [&](int64_t lo, int64_t hi) {
      std::vector<int64_t> sc(T), w(T);
      for (int64_t hq = lo; hq < hi; ++hq) {
        int64_t kvh = hq * c.n_kv_heads / c.n_heads;
        const int64_t* qh = q.data() + hq * dh;
        for (int64_t j = 0; j < T; ++j) {
          const int64_t* kr = K.data() + j * c.d_kv + kvh * dh;
          uint64_t dot = 0;
          for (int64_t e = 0; e < dh; ++e) dot += (uint64_t)qh[e] * (uint64_t)kr[e];
          sc[j] = attn_score((int64_t)dot, c.attn_scale);
        }
        softmax(sc.data(), T, w.data());
        int64_t* o = ao.data() + hq * dh;
        for (int64_t e = 0; e < dh; ++e) o[e] = 0;
        for (int64_t j = 0; j < T; ++j) {
          const int64_t* vr = V.data() + j * c.d_kv + kvh * dh;
          for (int64_t e = 0; e < dh; ++e) o[e] = wadd(o[e], mulshr(w[j], vr[e]));
        }
      }
    };
    if (T * c.n_heads * dh < (1 << 18)) head(0, c.n_heads);
    else pool().parallel_for(c.n_heads, head);
    mm(base + 3, L.wo, ao.data(), pr.data());
    for (int64_t i = 0; i < d; ++i) h[i] = wadd(h[i], pr[i]);
    rmsnorm(h.data(), d, L.ffn_norm.p, L.ffn_norm.n, n.data());
    mm(base + 4, L.gate, n.data(), g.data());
    mm(base + 5, L.up, n.data(), u.data());
    for (int64_t j = 0; j < c.d_ff; ++j) g[j] = swiglu(g[j], u[j], lut);
    mm(base + 6, L.down, g.data(), fo.data());
    for (int64_t i = 0; i < d; ++i) h[i] = wadd(h[i], fo[i]);
  }
  cache->seq_len = pos + 1;
  cache->last_hidden = h;
  rmsnorm(h.data(), d, m->final_norm.p, m->final_norm.n, n.data());
  if (m->q4) matmul_q4(m->q4w.back(), n.data(), logits);
  else matmul_i8(m->out, n.data(), logits);
}

// generate (1518-1557).
int64_t arcref_generate(arcref_model* m, const uint32_t* prompt, int64_t n_prompt,
                        int64_t max_tokens, const uint32_t* eos, int64_t n_eos,
                        uint32_t* out_tokens, uint8_t* hash32) {
  arcref_cache* cache = arcref_cache_new(m);
  std::vector<int64_t> logits(m->cfg.vocab);
  arcref_forward(m, cache, 1, logits.data());  // BOS
  for (int64_t i = 0; i < n_prompt; ++i) arcref_forward(m, cache, prompt[i], logits.data());
  int64_t ng = 0;
  for (int64_t t = 0; t < max_tokens && !cache->overflow; ++t) {
    uint32_t last = ng > 0 ? out_tokens[ng - 1] : (n_prompt > 0 ? prompt[n_prompt - 1] : 0);
    arcref_forward(m, cache, last, logits.data());
    if (cache->overflow) break;
    for (int64_t k = ng - 1, cnt = 0; k >= 0 && cnt < 64; --k, ++cnt) {
      uint32_t ti = out_tokens[k];
      if ((int64_t)ti < m->cfg.vocab) logits[ti] = penalize(logits[ti]);
    }
    int64_t best = 0, bv = INT64_MIN;
    for (int64_t i = 0; i < m->cfg.vocab; ++i)
      if (logits[i] > bv) {
        bv = logits[i];
        best = i;
      }
    out_tokens[ng++] = (uint32_t)best;
    bool stop = false;
    for (int64_t e = 0; e < n_eos; ++e) stop |= (eos[e] == (uint32_t)best);
    if (stop) break;
  }
  const bool overflow = cache->overflow;
  arcref_cache_free(cache);
  if (overflow) return -1;
  std::vector<uint8_t> bytes(ng * 4);
  for (int64_t i = 0; i < ng; ++i) {
    uint32_t t = out_tokens[i];
    bytes[4 * i] = (uint8_t)t;
    bytes[4 * i + 1] = (uint8_t)(t >> 8);
    bytes[4 * i + 2] = (uint8_t)(t >> 16);
    bytes[4 * i + 3] = (uint8_t)(t >> 24);
  }
  arcb3::hash(bytes.data(), bytes.size(), hash32);
  return ng;
}

// weight_hash (1598-1617): i8 bytes then LE i64 scales, per matrix.
void arcref_weight_hash(const arcref_model* m, uint8_t* hash32) {
  arcb3::Hasher h;
  h.init();
  auto add = [&](const I8W& w) {
    h.update(w.data, (size_t)(w.rows * w.cols));
    h.update(w.scales, (size_t)w.rows * 8);  // little-endian host
  };
  add(m->emb);
  add(m->out);
  for (auto& L : m->layers)
    for (const I8W* w : {&L.wq, &L.wk, &L.wv, &L.wo, &L.gate, &L.up, &L.down}) add(*w);
  h.finalize(hash32);
}

int64_t arcref_integer_exp(int64_t x) { return integer_exp(x, exp_lut()); }
int64_t arcref_integer_isqrt(int64_t x) { return integer_isqrt(x); }
int64_t arcref_silu(int64_t x) { return silu(x, exp_lut()); }
void arcref_softmax(const int64_t* x, int64_t n, int64_t* out) { softmax(x, n, out); }
void arcref_rmsnorm(const int64_t* x, int64_t n, const int64_t* gamma, int64_t ng, int64_t* out) {
  rmsnorm(x, n, gamma, ng, out);
}
void arcref_matmul_i8(const int8_t* w, const int64_t* s, const int64_t* x, int64_t rows,
                      int64_t cols, int64_t* out) {
  I8W m;
  m.data = w;
  m.scales = s;
  m.rows = rows;
  m.cols = cols;
  matmul_i8(m, x, out);
}

void arcref_blake3(const void* data, size_t len, uint8_t* out32) { arcb3::hash(data, len, out32); }
void* arcref_blake3_new(void) {
  auto* h = new arcb3::Hasher();
  h->init();
  return h;
}
void arcref_blake3_update(void* h, const void* data, size_t len) {
  ((arcb3::Hasher*)h)->update(data, len);
}
void arcref_blake3_push_chunk_cv(void* h, const uint32_t* cv8, uint64_t total_chunks) {
  auto* hh = (arcb3::Hasher*)h;
  hh->push_chunk_cv(cv8, total_chunks);
  hh->chunk_counter = total_chunks;
}
void arcref_blake3_finalize(void* h, uint8_t* out32) { ((arcb3::Hasher*)h)->finalize(out32); }
void arcref_blake3_free(void* h) { delete (arcb3::Hasher*)h; }

void arcref_rng_fill_i8(uint64_t seed, uint64_t stream, int8_t* out, int64_t n) {
  uint64_t key = arcrng::stream_key(seed, stream);
  pool().parallel_for(n, [&](int64_t lo, int64_t hi) {
    for (int64_t i = lo; i < hi; ++i) out[i] = arcrng::weight_i8(key, (uint64_t)i);
  });
}
void arcref_rng_u64(uint64_t seed, uint64_t stream, uint64_t* out, int64_t n) {
  uint64_t key = arcrng::stream_key(seed, stream);
  for (int64_t i = 0; i < n; ++i) out[i] = arcrng::at(key, (uint64_t)i);
}

int arcref_num_threads(void) { return pool().size(); }
void arcref_set_threads(int n) { pool().resize(n); }

}  // extern "C"

extern "C" void arcref_blake3_push_subtree_cv(void* h, const uint32_t* cv8, int level, uint64_t total_chunks) {
  ((arcb3::Hasher*)h)->push_subtree_cv(cv8, level, total_chunks);
}

// ---------------------------------------------------------------- BLAKE3 modes and batch commits
// Batch transaction commitments: item i hashed as derive_key(context,
// [domain_i] ++ data[offs[i] .. offs[i+1])) (the domain byte only when
// `domains` is given); the CPU counterpart of the GPU batch kernel
// (reference: crates/arc-gpu/src/lib.rs:70-91 cpu_batch_commit{,_domain}).
extern "C" void* arcref_blake3_new_derive(const char* context, size_t clen) {
  auto* h = new arcb3::Hasher();
  h->init_derive_key(context, clen);
  return h;
}
extern "C" void* arcref_blake3_new_keyed(const uint8_t* key32) {
  auto* h = new arcb3::Hasher();
  h->init_keyed(key32);
  return h;
}
extern "C" void arcref_blake3_context_key(const char* context, size_t clen, uint32_t* key8) {
  arcb3::derive_context_key(context, clen, key8);
}
extern "C" void arcref_blake3_batch_commit(const uint8_t* data, const int64_t* offs, int64_t n,
                                           const uint8_t* domains, const char* context, size_t clen,
                                           uint8_t* out32) {
  uint32_t k[8];
  arcb3::derive_context_key(context, clen, k);
  pool().parallel_for(n, [&](int64_t lo, int64_t hi) {
    for (int64_t i = lo; i < hi; ++i) {
      arcb3::Hasher h;
      h.init();
      memcpy(h.key, k, 32);
      memcpy(h.cv, k, 32);
      h.mode = arcb3::DERIVE_KEY_MATERIAL;
      if (domains) h.update(domains + i, 1);
      h.update(data + offs[i], (size_t)(offs[i + 1] - offs[i]));
      h.finalize(out32 + 32 * i);
    }
  });
}
// Merkle root over 32-byte leaves: each layer hashes adjacent pairs (64-byte
// payloads) with the batch commitment; an odd layer is padded with a zero
// hash; no leaves -> zero hash; one leaf -> the leaf
// (reference: crates/arc-gpu/src/lib.rs:414-460 gpu_merkle_root).
extern "C" void arcref_merkle_root(const uint8_t* leaves, int64_t n, const char* context, size_t clen,
                                   uint8_t* out32) {
  if (n == 0) {
    memset(out32, 0, 32);
    return;
  }
  std::vector<uint8_t> cur(leaves, leaves + 32 * n);
  int64_t m = n;
  while (m > 1) {
    if (m & 1) {
      cur.resize(32 * (m + 1), 0);
      ++m;
    }
    const int64_t np = m / 2;
    std::vector<int64_t> offs(np + 1);
    for (int64_t i = 0; i <= np; ++i) offs[i] = 64 * i;
    std::vector<uint8_t> nxt(32 * np);
    arcref_blake3_batch_commit(cur.data(), offs.data(), np, nullptr, context, clen, nxt.data());
    cur.swap(nxt);
    m = np;
  }
  memcpy(out32, cur.data(), 32);
}

// Installs a full-precision Q16 embedding table (borrowed; the caller keeps
// it alive for the model's lifetime).
extern "C" void arcref_set_embedding_q16(arcref_model* m, const int64_t* q16) { m->emb_q16 = q16; }
