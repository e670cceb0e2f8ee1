// Portable BLAKE3 (hash, keyed-hash and derive-key modes), written from the BLAKE3 specification
// (O'Connor, Aumasson, Neves, Wilcox-O'Hearn, 2020).  Used for the
// attestation triple: model hash, input hash and output hash
// (reference: crates/arc-crypto/src/hash.rs:77-80 hash_bytes = BLAKE3;
//  crates/arc-inference/src/cached_integer_model.rs:1553-1555, 1598-1617).
#pragma once
#include <stddef.h>
#include <stdint.h>

namespace arcb3 {

constexpr uint32_t IV[8] = {0x6A09E667u, 0xBB67AE85u, 0x3C6EF372u, 0xA54FF53Au,
                            0x510E527Fu, 0x9B05688Cu, 0x1F83D9ABu, 0x5BE0CD19u};
constexpr uint32_t CHUNK_START = 1u, CHUNK_END = 2u, PARENT = 4u, ROOT = 8u, KEYED_HASH = 16u,
                   DERIVE_KEY_CONTEXT = 32u, DERIVE_KEY_MATERIAL = 64u;
constexpr size_t BLOCK_LEN = 64, CHUNK_LEN = 1024;

void compress(const uint32_t cv[8], const uint32_t block[16], uint64_t counter,
              uint32_t block_len, uint32_t flags, uint32_t out[16]);

// Incremental hasher (tree built with the spec's chaining-value stack).
struct Hasher {
  uint32_t key[8];
  uint32_t mode;  // flags added to every compression (0, KEYED_HASH or a DERIVE_KEY_* flag)
  // current chunk state
  uint32_t cv[8];
  uint64_t chunk_counter;
  uint8_t block[64];
  uint32_t block_len;
  uint32_t blocks_compressed;
  // chaining value stack (54 levels covers 2^64 bytes)
  uint32_t stack[54][8];
  int stack_len;

  void init();
  void init_keyed(const uint8_t key32[32]);
  // derive_key(context, .): the context string hashed in DERIVE_KEY_CONTEXT
  // mode gives the key of the material hash (DERIVE_KEY_MATERIAL mode).
  void init_derive_key(const char* context, size_t len);
  void update(const void* data, size_t len);
  void finalize(uint8_t out[32]) const;
  // Merge a finished chunk's chaining value whose chunk index is
  // `total_chunks - 1`; exposed so a device-side chunk hasher can feed it.
  void push_chunk_cv(const uint32_t cv_in[8], uint64_t total_chunks);
  // Merge the CV of a complete aligned subtree of 2^level chunks that ends
  // at chunk count `total_chunks` (a multiple of 2^level).
  void push_subtree_cv(const uint32_t cv_in[8], int level, uint64_t total_chunks);
};

void hash(const void* data, size_t len, uint8_t out[32]);
// Key words of derive_key(context): the material hasher's key.
void derive_context_key(const char* context, size_t len, uint32_t key_out[8]);

}  // namespace arcb3
