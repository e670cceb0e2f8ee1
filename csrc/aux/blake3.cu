// A1: BLAKE3 on the GPU for GB-scale hashing (the model's weight hash).
//
// BLAKE3 (O'Connor, Aumasson, Neves, Wilcox-O'Hearn) splits input into
// 1 KiB chunks whose chaining values (CVs) combine in a binary tree whose
// complete subtrees are aligned powers of two.  Kernel 1 hashes every chunk
// but the last one (one thread per chunk, 16 compressions); kernel 2 merges
// aligned pairs of CVs into parent CVs, level by level; the host finishes the
// few remaining merges and the final chunk (which may carry the ROOT flag)
// with the incremental C++ hasher.  The input is a virtual concatenation of
// device segments (pointer, length), as the reference's weight_hash streams
// i8 data then LE i64 scales per matrix (cached_integer_model.rs:1598-1617);
// reference kernel for comparison: crates/arc-gpu/src/blake3.wgsl.
#include <cuda_runtime.h>
#include <stdint.h>

#include "../kernels/common.cuh"

namespace {

__constant__ uint32_t IV[8] = {0x6A09E667u, 0xBB67AE85u, 0x3C6EF372u, 0xA54FF53Au,
                               0x510E527Fu, 0x9B05688Cu, 0x1F83D9ABu, 0x5BE0CD19u};
constexpr uint32_t CHUNK_START = 1u, CHUNK_END = 2u, PARENT = 4u;

__device__ __forceinline__ uint32_t rotr(uint32_t x, int n) { return __funnelshift_r(x, x, n); }

__device__ __forceinline__ void g(uint32_t& a, uint32_t& b, uint32_t& c, uint32_t& d, uint32_t mx, uint32_t my) {
  a = a + b + mx;
  d = rotr(d ^ a, 16);
  c = c + d;
  b = rotr(b ^ c, 12);
  a = a + b + my;
  d = rotr(d ^ a, 8);
  c = c + d;
  b = rotr(b ^ c, 7);
}

// Compression returning the 8-word chaining value.
__device__ void compress_cv(uint32_t cv[8], const uint32_t m0[16], uint64_t counter, uint32_t len,
                            uint32_t flags) {
  uint32_t s[16] = {cv[0], cv[1], cv[2], cv[3], cv[4], cv[5], cv[6], cv[7],
                    IV[0], IV[1], IV[2], IV[3], (uint32_t)counter, (uint32_t)(counter >> 32), len, flags};
  uint32_t m[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) m[i] = m0[i];
#pragma unroll
  for (int r = 0; r < 7; ++r) {
    g(s[0], s[4], s[8], s[12], m[0], m[1]);
    g(s[1], s[5], s[9], s[13], m[2], m[3]);
    g(s[2], s[6], s[10], s[14], m[4], m[5]);
    g(s[3], s[7], s[11], s[15], m[6], m[7]);
    g(s[0], s[5], s[10], s[15], m[8], m[9]);
    g(s[1], s[6], s[11], s[12], m[10], m[11]);
    g(s[2], s[7], s[8], s[13], m[12], m[13]);
    g(s[3], s[4], s[9], s[14], m[14], m[15]);
    if (r < 6) {  // message permutation 2,6,3,10,7,0,4,13,1,11,12,5,9,14,15,8
      const uint32_t t[16] = {m[2], m[6], m[3], m[10], m[7], m[0], m[4], m[13],
                              m[1], m[11], m[12], m[5], m[9], m[14], m[15], m[8]};
#pragma unroll
      for (int i = 0; i < 16; ++i) m[i] = t[i];
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) cv[i] = s[i] ^ s[i + 8];
}

// Byte `off` of the virtual concatenation.
__device__ __forceinline__ int find_seg(const int64_t* offs, int n, int64_t off) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (offs[mid] <= off) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

__global__ void k_chunk_cvs(const uint8_t* const* __restrict__ segs, const int64_t* __restrict__ offs, int nseg,
                            int64_t n_chunks, int64_t chunk_base, uint32_t* __restrict__ cvs) {
  pdl_wait_dep();
  const int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (c >= n_chunks) return;
  uint32_t cv[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) cv[i] = IV[i];
  const int64_t base = c * 1024;
  int si = find_seg(offs, nseg, base);
  for (int blk = 0; blk < 16; ++blk) {
    uint32_t m[16];
    const int64_t o = base + blk * 64;
    while (si + 1 < nseg && offs[si + 1] <= o) ++si;
    const int64_t in_seg = o - offs[si];
    const uint8_t* p = segs[si] + in_seg;
    const bool fast = (si + 1 >= nseg || offs[si + 1] >= o + 64) && (((uintptr_t)p & 15) == 0);
    if (fast) {
      const uint4* q = (const uint4*)p;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint4 v = __ldg(q + k);
        m[4 * k] = v.x;
        m[4 * k + 1] = v.y;
        m[4 * k + 2] = v.z;
        m[4 * k + 3] = v.w;
      }
    } else {
      int sj = si;
      for (int w = 0; w < 16; ++w) {
        uint32_t word = 0;
        for (int b = 0; b < 4; ++b) {
          const int64_t ob = o + 4 * w + b;
          while (sj + 1 < nseg && offs[sj + 1] <= ob) ++sj;
          word |= (uint32_t)segs[sj][ob - offs[sj]] << (8 * b);
        }
        m[w] = word;
      }
    }
    const uint32_t flags = (blk == 0 ? CHUNK_START : 0u) | (blk == 15 ? CHUNK_END : 0u);
    compress_cv(cv, m, (uint64_t)(chunk_base + c), 64, flags);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) cvs[c * 8 + i] = cv[i];
}

// parents[i] = parent(cvs[2i], cvs[2i+1]) (non-root), i < n_pairs.
__global__ void k_parents(const uint32_t* __restrict__ cvs, int64_t n_pairs, uint32_t* __restrict__ out) {
  pdl_wait_dep();
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n_pairs) return;
  uint32_t m[16], cv[8];
#pragma unroll
  for (int k = 0; k < 16; ++k) m[k] = cvs[i * 16 + k];
#pragma unroll
  for (int k = 0; k < 8; ++k) cv[k] = IV[k];
  compress_cv(cv, m, 0, 64, PARENT);
#pragma unroll
  for (int k = 0; k < 8; ++k) out[i * 8 + k] = cv[k];
}

// ---------------------------------------------------------------- batch commitments
// One thread per item: derive_key(context, [domain_i] ++ item_i), where the
// context key (the material hasher's key words) is derived on the host.
// Items are byte ranges [offs[i], offs[i+1]) of one buffer of `nwords` 32-bit
// words (the host pads it to a multiple of 16 bytes); a word straddling two
// aligned words is assembled with a funnel shift.  Items of more than one
// chunk keep the chaining-value stack in local memory (depth MAXD: items up
// to 2^MAXD KiB).
constexpr uint32_t ROOT_F = 8u, DKM = 64u;
constexpr int MAXD = 20;

struct Key8 {
  uint32_t w[8];
};

__device__ __forceinline__ uint32_t item_word(const uint32_t* __restrict__ buf, int64_t nwords, int64_t start,
                                              int dom, uint32_t dbyte, int64_t vlen, int64_t vpos) {
  if (vpos >= vlen) return 0;
  uint32_t w;
  if (dom && vpos == 0) {
    // the domain byte, then the first three data bytes
    w = dbyte;
    for (int j = 1; j < 4; ++j) {
      if (j >= vlen) break;
      const int64_t a = start + j - 1;
      w |= ((buf[a >> 2] >> (8 * (a & 3))) & 0xFFu) << (8 * j);
    }
    return w;
  }
  const int64_t a = start + vpos - dom;
  const int64_t aw = a >> 2;
  const int sh = (int)(a & 3) * 8;
  const uint32_t w0 = __ldg(buf + aw);
  const uint32_t w1 = (sh && aw + 1 < nwords) ? __ldg(buf + aw + 1) : 0u;
  w = sh ? __funnelshift_r(w0, w1, sh) : w0;
  const int64_t rem = vlen - vpos;
  if (rem < 4) w &= 0xFFFFFFFFu >> (8 * (4 - (int)rem));
  return w;
}

__global__ void k_batch_commit(const uint32_t* __restrict__ buf, int64_t nwords, const int64_t* __restrict__ offs,
                               int64_t n, const uint8_t* __restrict__ domains, Key8 key, uint32_t* __restrict__ out) {
  pdl_wait_dep();
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int64_t start = offs[i], len = offs[i + 1] - start;
  const int dom = domains ? 1 : 0;
  const uint32_t dbyte = domains ? domains[i] : 0u;
  const int64_t vlen = len + dom;
  const int64_t nch = vlen == 0 ? 1 : (vlen + 1023) / 1024;
  uint32_t stack[MAXD][8];
  int sp = 0;
  uint32_t cv[8];
  for (int64_t c = 0; c < nch; ++c) {
#pragma unroll
    for (int k = 0; k < 8; ++k) cv[k] = key.w[k];
    const int64_t clen = min((int64_t)1024, vlen - c * 1024);
    const int nb = clen <= 0 ? 1 : (int)((clen + 63) / 64);
    for (int blk = 0; blk < nb; ++blk) {
      const int64_t v0 = c * 1024 + blk * 64;
      uint32_t m[16];
#pragma unroll
      for (int w = 0; w < 16; ++w) m[w] = item_word(buf, nwords, start, dom, dbyte, vlen, v0 + 4 * w);
      const uint32_t blen = (uint32_t)max((int64_t)0, min((int64_t)64, clen - blk * 64));
      uint32_t f = DKM | (blk == 0 ? CHUNK_START : 0u) | (blk == nb - 1 ? CHUNK_END : 0u);
      if (nch == 1 && blk == nb - 1) f |= ROOT_F;
      compress_cv(cv, m, (uint64_t)c, blen, f);
    }
    if (c + 1 < nch) {
      // merge completed subtrees: one parent per trailing zero bit of the count
      uint64_t t = (uint64_t)c + 1;
      while ((t & 1) == 0 && sp > 0) {
        uint32_t pm[16];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          pm[k] = stack[sp - 1][k];
          pm[8 + k] = cv[k];
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) cv[k] = key.w[k];
        compress_cv(cv, pm, 0, 64, DKM | PARENT);
        --sp;
        t >>= 1;
      }
      if (sp >= MAXD) return;  // unreachable: the host bounds the item length
#pragma unroll
      for (int k = 0; k < 8; ++k) stack[sp][k] = cv[k];
      ++sp;
    }
  }
  for (int j = sp - 1; j >= 0; --j) {
    uint32_t pm[16];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      pm[k] = stack[j][k];
      pm[8 + k] = cv[k];
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) cv[k] = key.w[k];
    compress_cv(cv, pm, 0, 64, DKM | PARENT | (j == 0 ? ROOT_F : 0u));
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) out[i * 8 + k] = cv[k];
}

// One Merkle layer: out[i] = commit(in[2i] ++ in[2i+1]), in[n_in] = zero hash.
__global__ void k_merkle_layer(const uint32_t* __restrict__ in, int64_t n_in, Key8 key, uint32_t* __restrict__ out) {
  pdl_wait_dep();
  pdl_allow_next();
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= (n_in + 1) / 2) return;
  uint32_t m[16], cv[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    m[k] = in[(2 * i) * 8 + k];
    m[8 + k] = 2 * i + 1 < n_in ? in[(2 * i + 1) * 8 + k] : 0u;
    cv[k] = key.w[k];
  }
  compress_cv(cv, m, 0, 64, DKM | CHUNK_START | CHUNK_END | ROOT_F);
#pragma unroll
  for (int k = 0; k < 8; ++k) out[i * 8 + k] = cv[k];
}

}  // namespace

extern "C" {

// Batch commitments of n items (see k_batch_commit).  buf: 4-byte aligned,
// nbytes a multiple of 4 and >= offs[n]; domains: n bytes or null; key8: the
// derive_key context key words; out: n x 32 bytes.  Items longer than
// 2^MAXD KiB are refused (-2).
int arcb_blake3_batch_commit(const void* buf, int64_t nbytes, const int64_t* offs, int64_t n, const uint8_t* domains,
                             const uint32_t* key8, int64_t max_item_len, uint32_t* out, void* stream) {
  if (n <= 0) return 0;
  if (((uintptr_t)buf & 3) || (nbytes & 3)) return -1;
  if (max_item_len + 1 > ((int64_t)1024 << MAXD)) return -2;
  Key8 k;
  for (int j = 0; j < 8; ++j) k.w[j] = key8[j];
  const int64_t blocks = (n + 127) / 128;
  return launch_k(k_batch_commit, dim3((unsigned)blocks), dim3(128), 0, (cudaStream_t)stream, (const uint32_t*)buf,
                  nbytes / 4, offs, n, domains, k, out);
}

// Merkle root of n 32-byte leaves into out (8 words).  scratch: at least
// 2 * 32 * ((n + 1) / 2) bytes, used as two ping-pong layers.
int arcb_merkle_root(const uint32_t* leaves, int64_t n, const uint32_t* key8, uint32_t* scratch, uint32_t* out,
                     void* stream) {
  cudaStream_t st = (cudaStream_t)stream;
  if (n <= 0) return (int)cudaMemsetAsync(out, 0, 32, st);
  if (n == 1) return (int)cudaMemcpyAsync(out, leaves, 32, cudaMemcpyDeviceToDevice, st);
  Key8 k;
  for (int j = 0; j < 8; ++j) k.w[j] = key8[j];
  const int64_t half = (n + 1) / 2;
  uint32_t* bufs[2] = {scratch, scratch + 8 * half};
  const uint32_t* cur = leaves;
  int64_t m = n;
  int side = 0;
  while (m > 1) {
    const int64_t mo = (m + 1) / 2;
    uint32_t* dst = mo == 1 ? out : bufs[side];
    const int64_t blocks = (mo + 127) / 128;
    const int e = launch_k(k_merkle_layer, dim3((unsigned)blocks), dim3(128), 0, st, cur, m, k, dst);
    if (e) return e;
    cur = dst;
    side ^= 1;
    m = mo;
  }
  return 0;
}

// chunk_base: index of the first chunk in the whole stream (the chunk
// counter input of BLAKE3's compression).
int arcb_blake3_chunk_cvs(const void* seg_ptrs, const int64_t* seg_offs, int nseg, int64_t n_chunks,
                          int64_t chunk_base, uint32_t* cvs, void* stream) {
  if (n_chunks <= 0) return 0;
  const int64_t blocks = (n_chunks + 127) / 128;
  return launch_k(k_chunk_cvs, dim3((unsigned)blocks), dim3(128), 0, (cudaStream_t)stream,
                  (const uint8_t* const*)seg_ptrs, seg_offs, nseg, n_chunks, chunk_base, cvs);
}

int arcb_blake3_parents(const uint32_t* cvs, int64_t n_pairs, uint32_t* out, void* stream) {
  if (n_pairs <= 0) return 0;
  const int64_t blocks = (n_pairs + 127) / 128;
  return launch_k(k_parents, dim3((unsigned)blocks), dim3(128), 0, (cudaStream_t)stream, cvs, n_pairs, out);
}

}  // extern "C"
