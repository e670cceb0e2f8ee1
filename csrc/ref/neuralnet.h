// arcnn: native reader, writer and forward passes of the reference VM's
// tagged f32 MLP format ("NeuralNet", crates/arc-vm/src/inference.rs:21-55,
// 132-381) and of the files scripts/create_model.py writes.
//
// File layout (little-endian): u32 n_layers, then per layer one tag byte and
// its payload:
//   Dense      u32 rows, u32 cols, f32 W[rows*cols] row-major, f32 bias[rows]
//   ReLU, Softmax   no payload
//   LayerNorm  u32 n, f32 gamma[n], f32 beta[n], f32 eps
//   Embedding  u32 vocab, u32 dim, f32 table[vocab*dim]
// The VM numbers the tags 0..4 (Dense, ReLU, Softmax, LayerNorm, Embedding)
// and create_model.py 1..5.  arcnn_parse takes the numbering under which the
// whole image parses exactly (the VM's when both do, as for a file of only
// ReLU / Softmax layers); failing both, the VM's own rule (0..4, bytes after
// the last layer ignored, inference.rs:132-211).
//
// Two executions:
//   arcnn_forward_f32  the VM's f32 forward (inference.rs:282-381) with the
//                      same operation order: left-to-right sums that start
//                      at -0.0 (Rust's f32 Sum), NaN-ignoring max, libm expf,
//                      saturating float -> index casts.  Built without
//                      floating-point contraction.
//   arcnn_forward_q16  the same network in the integer engine's arithmetic:
//                      per-row INT8 Dense (I8Weights::quantize_f32,
//                      cached_integer_model.rs:36-62) with a Q16 bias,
//                      ReLU, softmax_i64, integer LayerNorm, Q16 embedding.
//                      Deterministic on every platform.
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ARCNN_DENSE = 0, ARCNN_RELU = 1, ARCNN_SOFTMAX = 2, ARCNN_LAYERNORM = 3, ARCNN_EMBEDDING = 4 };

typedef struct arcnn_net arcnn_net;

// Parse a file image.  Returns NULL and writes a message to `err` on failure.
arcnn_net* arcnn_parse(const uint8_t* data, size_t len, char* err, int errlen);
// An empty network to fill with arcnn_add_layer.
arcnn_net* arcnn_new(void);
// Append a layer.  Dense: a = W [rows*cols], b = bias [rows].  LayerNorm:
// a = gamma [rows], b = beta [rows], eps.  Embedding: a = table [rows*cols].
// ReLU / Softmax take no arrays.  Returns 0, -1 for an unknown kind, or -2
// when the layer could not be allocated.
int arcnn_add_layer(arcnn_net* net, int kind, int64_t rows, int64_t cols, const float* a,
                    const float* b, float eps);
void arcnn_free(arcnn_net* net);

// 0 for the VM numbering, 1 for create_model.py's.
int arcnn_tag_base(const arcnn_net* net);
int64_t arcnn_num_layers(const arcnn_net* net);
// Kind of layer i (or -1); writes its rows / cols (0 where not applicable).
int arcnn_layer(const arcnn_net* net, int64_t i, int64_t* rows, int64_t* cols, float* eps);
// Copies array `which` (0: W / gamma / table, 1: bias / beta) of layer i into
// `out` when it holds `cap` floats; returns the array's length.
int64_t arcnn_layer_data(const arcnn_net* net, int64_t i, int which, float* out, int64_t cap);
// infer_input_size / infer_output_size (inference.rs:387-422).
int64_t arcnn_input_size(const arcnn_net* net);
int64_t arcnn_output_size(const arcnn_net* net);

// Serialise (NeuralNet::to_bytes, inference.rs:213-270) under tag numbering
// `tag_base`.  Writes when `cap` suffices; returns the byte count.
int64_t arcnn_serialize(const arcnn_net* net, int tag_base, uint8_t* out, int64_t cap);

// Output length of a forward pass over n inputs.
int64_t arcnn_output_len(const arcnn_net* net, int64_t n);
// Forward passes: write arcnn_output_len(net, n) values when `cap` suffices;
// return that length.
int64_t arcnn_forward_f32(const arcnn_net* net, const float* x, int64_t n, float* out, int64_t cap);
int64_t arcnn_forward_q16(const arcnn_net* net, const int64_t* x, int64_t n, int64_t* out,
                          int64_t cap);
// The VM's softmax of one vector (also used to classify outputs).
void arcnn_softmax_f32(const float* x, int64_t n, float* out);

#ifdef __cplusplus
}
#endif
