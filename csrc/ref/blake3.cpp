// BLAKE3 hash, keyed-hash and derive-key modes, from the specification.  See blake3.h.
#include "blake3.h"

#include <string.h>

namespace arcb3 {

static const uint8_t PERM[16] = {2, 6, 3, 10, 7, 0, 4, 13, 1, 11, 12, 5, 9, 14, 15, 8};

static inline uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

static inline void g(uint32_t* s, int a, int b, int c, int d, uint32_t mx, uint32_t my) {
  s[a] = s[a] + s[b] + mx;
  s[d] = rotr(s[d] ^ s[a], 16);
  s[c] = s[c] + s[d];
  s[b] = rotr(s[b] ^ s[c], 12);
  s[a] = s[a] + s[b] + my;
  s[d] = rotr(s[d] ^ s[a], 8);
  s[c] = s[c] + s[d];
  s[b] = rotr(s[b] ^ s[c], 7);
}

void compress(const uint32_t cv[8], const uint32_t block[16], uint64_t counter,
              uint32_t block_len, uint32_t flags, uint32_t out[16]) {
  uint32_t s[16] = {cv[0], cv[1], cv[2], cv[3], cv[4], cv[5], cv[6], cv[7],
                    IV[0], IV[1], IV[2], IV[3], (uint32_t)counter,
                    (uint32_t)(counter >> 32), block_len, flags};
  uint32_t m[16];
  memcpy(m, block, 64);
  for (int r = 0; r < 7; ++r) {
    g(s, 0, 4, 8, 12, m[0], m[1]);
    g(s, 1, 5, 9, 13, m[2], m[3]);
    g(s, 2, 6, 10, 14, m[4], m[5]);
    g(s, 3, 7, 11, 15, m[6], m[7]);
    g(s, 0, 5, 10, 15, m[8], m[9]);
    g(s, 1, 6, 11, 12, m[10], m[11]);
    g(s, 2, 7, 8, 13, m[12], m[13]);
    g(s, 3, 4, 9, 14, m[14], m[15]);
    if (r < 6) {
      uint32_t t[16];
      for (int i = 0; i < 16; ++i) t[i] = m[PERM[i]];
      memcpy(m, t, 64);
    }
  }
  for (int i = 0; i < 8; ++i) {
    out[i] = s[i] ^ s[i + 8];
    out[i + 8] = s[i + 8] ^ cv[i];
  }
}

static inline void load_block(const uint8_t* b, uint32_t w[16]) {
  for (int i = 0; i < 16; ++i)
    w[i] = (uint32_t)b[4 * i] | ((uint32_t)b[4 * i + 1] << 8) |
           ((uint32_t)b[4 * i + 2] << 16) | ((uint32_t)b[4 * i + 3] << 24);
}

static void parent_cv(const uint32_t key[8], const uint32_t l[8], const uint32_t r[8], uint32_t flags,
                      uint32_t out8[8]) {
  uint32_t blk[16], o[16];
  memcpy(blk, l, 32);
  memcpy(blk + 8, r, 32);
  compress(key, blk, 0, 64, PARENT | flags, o);
  memcpy(out8, o, 32);
}

void Hasher::init() {
  mode = 0;
  memcpy(key, IV, 32);
  memcpy(cv, IV, 32);
  chunk_counter = 0;
  block_len = 0;
  blocks_compressed = 0;
  stack_len = 0;
  memset(block, 0, 64);
}

void Hasher::init_keyed(const uint8_t key32[32]) {
  init();
  for (int i = 0; i < 8; ++i)
    key[i] = (uint32_t)key32[4 * i] | ((uint32_t)key32[4 * i + 1] << 8) | ((uint32_t)key32[4 * i + 2] << 16) |
             ((uint32_t)key32[4 * i + 3] << 24);
  memcpy(cv, key, 32);
  mode = KEYED_HASH;
}

void derive_context_key(const char* context, size_t len, uint32_t key_out[8]) {
  Hasher h;
  h.init();
  h.mode = DERIVE_KEY_CONTEXT;
  h.update(context, len);
  uint8_t k[32];
  h.finalize(k);
  for (int i = 0; i < 8; ++i)
    key_out[i] = (uint32_t)k[4 * i] | ((uint32_t)k[4 * i + 1] << 8) | ((uint32_t)k[4 * i + 2] << 16) |
                 ((uint32_t)k[4 * i + 3] << 24);
}

void Hasher::init_derive_key(const char* context, size_t len) {
  uint32_t k[8];
  derive_context_key(context, len, k);
  init();
  memcpy(key, k, 32);
  memcpy(cv, k, 32);
  mode = DERIVE_KEY_MATERIAL;
}

void Hasher::push_chunk_cv(const uint32_t cv_in[8], uint64_t total_chunks) {
  uint32_t c[8];
  memcpy(c, cv_in, 32);
  while ((total_chunks & 1) == 0) {
    --stack_len;
    parent_cv(key, stack[stack_len], c, mode, c);
    total_chunks >>= 1;
  }
  memcpy(stack[stack_len++], c, 32);
}

void Hasher::push_subtree_cv(const uint32_t cv_in[8], int level, uint64_t total_chunks) {
  uint32_t c[8];
  memcpy(c, cv_in, 32);
  uint64_t t = total_chunks >> level;
  while ((t & 1) == 0) {
    --stack_len;
    parent_cv(key, stack[stack_len], c, mode, c);
    t >>= 1;
  }
  memcpy(stack[stack_len++], c, 32);
  chunk_counter = total_chunks;
}

void Hasher::update(const void* data, size_t len) {
  const uint8_t* p = (const uint8_t*)data;
  while (len > 0) {
    // A full chunk is only closed once more input arrives, so the final
    // chunk can still receive the ROOT flag.
    if (blocks_compressed * BLOCK_LEN + block_len == CHUNK_LEN) {
      uint32_t w[16], o[16];
      load_block(block, w);
      uint32_t flags = mode | CHUNK_END | (blocks_compressed == 0 ? CHUNK_START : 0);
      compress(cv, w, chunk_counter, block_len, flags, o);
      ++chunk_counter;
      push_chunk_cv(o, chunk_counter);
      memcpy(cv, key, 32);
      blocks_compressed = 0;
      block_len = 0;
      memset(block, 0, 64);
    }
    if (block_len == BLOCK_LEN) {
      uint32_t w[16], o[16];
      load_block(block, w);
      uint32_t flags = mode | (blocks_compressed == 0 ? CHUNK_START : 0);
      compress(cv, w, chunk_counter, 64, flags, o);
      memcpy(cv, o, 32);
      ++blocks_compressed;
      block_len = 0;
      memset(block, 0, 64);
    }
    size_t take = BLOCK_LEN - block_len;
    if (take > len) take = len;
    memcpy(block + block_len, p, take);
    block_len += (uint32_t)take;
    p += take;
    len -= take;
  }
}

void Hasher::finalize(uint8_t out[32]) const {
  uint32_t w[16], o[16];
  uint8_t blk[64];
  memset(blk, 0, 64);
  memcpy(blk, block, block_len);
  load_block(blk, w);
  uint32_t flags = mode | CHUNK_END | (blocks_compressed == 0 ? CHUNK_START : 0);
  uint32_t res[8];
  if (stack_len == 0) {
    compress(cv, w, chunk_counter, block_len, flags | ROOT, o);
    memcpy(res, o, 32);
  } else {
    compress(cv, w, chunk_counter, block_len, flags, o);
    uint32_t c[8];
    memcpy(c, o, 32);
    for (int i = stack_len - 1; i >= 0; --i)
      parent_cv(key, stack[i], c, mode | (i == 0 ? ROOT : 0), c);
    memcpy(res, c, 32);
  }
  for (int i = 0; i < 8; ++i) {
    out[4 * i] = (uint8_t)res[i];
    out[4 * i + 1] = (uint8_t)(res[i] >> 8);
    out[4 * i + 2] = (uint8_t)(res[i] >> 16);
    out[4 * i + 3] = (uint8_t)(res[i] >> 24);
  }
}

void hash(const void* data, size_t len, uint8_t out[32]) {
  Hasher h;
  h.init();
  h.update(data, len);
  h.finalize(out);
}

}  // namespace arcb3
