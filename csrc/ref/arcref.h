// arcref: bit-exact C++ restatement of the reference CPU integer engine
// (crates/arc-inference/src/cached_integer_model.rs, CachedIntegerModel).
// It is the correctness oracle for every GPU path and the timed same-box
// CPU baseline.  C ABI so Python binds it with ctypes.
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct arcref_config {
  int64_t n_layers, d_model, n_heads, n_kv_heads, d_ff, d_head, d_kv, vocab, max_seq;
  int64_t attn_scale;
} arcref_config;

typedef struct arcref_model arcref_model;
typedef struct arcref_cache arcref_cache;

// Load an ARC-INT8 v2 file (cached_integer_model.rs:1783-1864).  Returns NULL
// and writes a message into `err` on failure.
arcref_model* arcref_load_file(const char* path, char* err, int errlen);

// Write the model as an ARC-INT8 v2 file, the bytes save_weights writes
// (cached_integer_model.rs:1560-1595): header, RoPE tables, embedding and
// output matrices, final norm, per layer 7 matrices and 2 norms, then u64
// length + vocab JSON.  `vocab_json` (`vocab_len` UTF-8 bytes) is stored as
// given; NULL stores the vocab bytes of the file the model was loaded from
// ("[]" when there were none).  Q4 mode does not change what is written (the
// INT8 weights).  Returns 0, or -1 with a message in `err`.
int arcref_save_file(const arcref_model* m, const char* path, const char* vocab_json,
                     int64_t vocab_len, char* err, int errlen);

// Build a model over caller-owned arrays (not copied; they must outlive the
// model).  `ptrs` order: emb_data, emb_scales, out_data, out_scales,
// final_norm, rope_cos, rope_sin, then per layer wq, wq_s, wk, wk_s, wv, wv_s,
// wo, wo_s, gate, gate_s, up, up_s, down, down_s, attn_norm, ffn_norm.
// `lens` order: final_norm, rope (cos and sin each), then per layer
// attn_norm, ffn_norm.
arcref_model* arcref_from_arrays(const arcref_config* cfg, const void* const* ptrs,
                                 const int64_t* lens);
void arcref_free(arcref_model* m);
void arcref_get_config(const arcref_model* m, arcref_config* out);

// Convert every matrix to the reference's per-row Q4 (Q4WeightsX86::from_i8,
// cached_integer_model.rs:670-701) and use it in forward (enable_q4, 181-193).
void arcref_enable_q4(arcref_model* m);

// Greedy generate with the reference's quirks (1518-1557).  Returns the number
// of generated tokens (<= max_tokens); writes BLAKE3(LE u32 tokens) to hash32.
// Returns -1 when the sequence runs past the RoPE tables (the reference's
// max_seq), where the reference's unchecked indexing panics.
int64_t arcref_generate(arcref_model* m, const uint32_t* prompt, int64_t n_prompt,
                        int64_t max_tokens, const uint32_t* eos, int64_t n_eos,
                        uint32_t* out_tokens, uint8_t* hash32);

// Single-token forward for kernel tests.
arcref_cache* arcref_cache_new(const arcref_model* m);
void arcref_cache_free(arcref_cache* c);
int64_t arcref_cache_len(const arcref_cache* c);
void arcref_cache_truncate(arcref_cache* c, int64_t len);
// A position past the RoPE tables writes zero logits and sets the cache's
// overflow flag (arcref_cache_overflow) instead of reading past them.
void arcref_forward(arcref_model* m, arcref_cache* c, uint32_t token, int64_t* logits);
int arcref_cache_overflow(const arcref_cache* c);
// Hidden state after the last layer (before the final norm) of the last
// forward call, d_model values.
void arcref_last_hidden(const arcref_cache* c, int64_t* out);

// weight_hash (1598-1617).
void arcref_weight_hash(const arcref_model* m, uint8_t* hash32);

// Primitive exports (tests compare kernels and the Python restatement).
int64_t arcref_integer_exp(int64_t x);
int64_t arcref_integer_isqrt(int64_t x);
int64_t arcref_silu(int64_t x);
void arcref_softmax(const int64_t* x, int64_t n, int64_t* out);
void arcref_rmsnorm(const int64_t* x, int64_t n, const int64_t* gamma, int64_t ng,
                    int64_t* out);
// out[i] = ((sum_j w[i,j]*x[j]) * s[i]) >> 16, wrapping.
void arcref_matmul_i8(const int8_t* w, const int64_t* s, const int64_t* x, int64_t rows,
                      int64_t cols, int64_t* out);

void arcref_blake3(const void* data, size_t len, uint8_t* out32);
// Incremental BLAKE3 for streams (weight hash over device buffers).
void* arcref_blake3_new(void);
void arcref_blake3_update(void* h, const void* data, size_t len);
void arcref_blake3_push_chunk_cv(void* h, const uint32_t* cv8, uint64_t total_chunks);
void arcref_blake3_finalize(void* h, uint8_t* out32);
void arcref_blake3_free(void* h);

// Seeded generator (csrc/common/rng.h): int8 weights in [-127,127] / raw u64.
void arcref_rng_fill_i8(uint64_t seed, uint64_t stream, int8_t* out, int64_t n);
void arcref_rng_u64(uint64_t seed, uint64_t stream, uint64_t* out, int64_t n);

int arcref_num_threads(void);
void arcref_set_threads(int n);

#ifdef __cplusplus
}
#endif
