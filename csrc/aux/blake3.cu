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

}  // namespace

extern "C" {

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
