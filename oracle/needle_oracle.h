/*
 * needle_oracle.h — CPU restatement of rustyneedle's Needle-3 token loop.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the parity checker for the
 * B200 kernels and the timed CPU baseline in bench.py. The product
 * (rustyneedle_b200) never links, loads or calls it.
 *
 * Two numeric modes restate the two code paths the reference compiles:
 *   NBO_MODE_INT   — the aarch64 integer kernels (crates/kernels/src/neon.rs,
 *                    panel.rs; matrix.rs:204-214,402-420): int8 activations per
 *                    128-group, exact int32 group sums, ordered f32 combine.
 *                    This is the parity target of the GPU path.
 *   NBO_MODE_FLOAT — the portable float kernels every other target runs
 *                    (matrix.rs:216-219,422-440; kernels/src/attention.rs:262-275).
 *                    This is what rustyneedle executes on an x86-64 host.
 *
 * Every function returns 0 on success or a negative status; the message of
 * the last failure on the calling thread is available from nbo_last_error().
 */
#ifndef NEEDLE_ORACLE_H
#define NEEDLE_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { NBO_MODE_INT = 0, NBO_MODE_FLOAT = 1 };

typedef struct nbo_model nbo_model;
typedef struct nbo_session nbo_session;

const char* nbo_last_error(void);

/* Model::open (crates/model/src/model.rs:52-56) with a numeric mode and a
 * worker-thread count for the fork-join sections (0 = all host cores). */
int nbo_model_open(const char* path, int mode, int threads, nbo_model** out);
/* Model::with_depth (model.rs:63-66); status -3 carries no model. */
int nbo_model_with_depth(const nbo_model* model, int depth, nbo_model** out);
void nbo_model_free(nbo_model* model);
int nbo_model_active_layers(const nbo_model* model, int32_t* out, int cap);
/* Header geometry as 8 integers: vocab, output_vocab, d_model, heads,
 * kv_heads, layers, head_dim, max_seq_len. */
void nbo_model_geometry(const nbo_model* model, int32_t* out8);
void nbo_model_set_threads(nbo_model* model, int threads);

/* Session (crates/model/src/session.rs). */
nbo_session* nbo_session_new(const nbo_model* model);
nbo_session* nbo_session_clone(const nbo_session* session);
void nbo_session_free(nbo_session* session);
size_t nbo_session_len(const nbo_session* session);
// Session::head_output / pooled_readout: values written (at most cap), -1 without a head `code`.
long nbo_session_head_output(const nbo_session* session, int code, float* out, size_t cap);
long nbo_session_pooled_readout(const nbo_session* session, int code, float* out, size_t cap);

// Whistle (whistle/src/cross.rs): the cross-attention memory of an encoder
// output [frames][d_model], its per-layer keys/values, and a push through the
// cross-attention hook; the archive's text vocabulary size (0 without audio).
typedef struct nbo_cross_memory nbo_cross_memory;
int nbo_cross_memory_new(const nbo_model* model, const float* encoded, size_t frames, nbo_cross_memory** out);
void nbo_cross_memory_free(nbo_cross_memory* memory);
size_t nbo_cross_memory_read(const nbo_cross_memory* memory, int layer, int8_t* keys, float* key_scales, int8_t* values,
                             float* value_scales);
int nbo_session_push_cross(nbo_session* session, uint32_t token, const nbo_cross_memory* memory);
size_t nbo_model_text_vocab(const nbo_model* model);
void nbo_session_push(nbo_session* session, uint32_t token);
/* push that also records the lane stream after every active layer:
 * trace holds depth × lanes × d_model floats. */
void nbo_session_push_traced(nbo_session* session, uint32_t token, float* trace);
void nbo_session_feed(nbo_session* session, const uint32_t* tokens, size_t count);
void nbo_session_logits(const nbo_session* session, float* out);
void nbo_session_hidden(const nbo_session* session, float* out);
/* The int8 KV cache of one layer: keys/values [positions][kv_heads][dim],
 * scales [kv_heads][positions]. Returns the position count. */
size_t nbo_session_cache(const nbo_session* session, int layer, int8_t* keys, float* key_scales, int8_t* values,
                         float* value_scales);

/* Runs `count` sessions one decode step each, one session per worker
 * (the reference runs independent sequences on separate threads). */
void nbo_sessions_step(nbo_session** sessions, size_t count, const uint32_t* tokens, float* logits, int threads);

/* Generator pieces (crates/generate/src/generator.rs:147-194). */
int32_t nbo_argmax(const float* values, size_t count);
int32_t nbo_argmax_allowed(const float* values, const uint8_t* allowed, size_t count);
void nbo_allowed_statistics(const float* logits, size_t count, uint32_t token, const uint8_t* allowed, float* probability,
                            float* mass);

/* Kernel-level primitives (crates/kernels/src/{walsh,ops}.rs). */
void nbo_walsh(float* values, size_t count);
float nbo_fast_exp(float value);
float nbo_sigmoid(float value);
void nbo_softmax(float* values, size_t count);
void nbo_kronecker(const float* input, const float* left, size_t left_size, const float* right, size_t right_size,
                   float* output, int mode);
void nbo_sinkhorn(float* logits, size_t size, size_t iterations);
void nbo_zero_centred_norm(const float* input, const float* gains, float* output, size_t count);
void nbo_fake_quantise_int8(float* values, size_t count);
float nbo_quantise_int8(const float* values, int8_t* codes, size_t count);
void nbo_rotary(float* head, size_t dim, size_t position, float theta);
int nbo_ladder_order(int layers, int32_t* out);
int nbo_ladder_select(int layers, int depth, int32_t* out);
float nbo_half_to_f32(uint16_t bits);

/* One codebook-quantised product of archive tensor `tensor` with an input
 * of the matrix's column count, over rows [first_row, first_row+rows).
 * With NBO_MODE_INT the per-(row, group) int32 sums are written to
 * group_sums (rows × groups) when it is non-NULL. */
int nbo_matrix_product(const nbo_model* model, int tensor, const float* input, size_t first_row, size_t rows,
                       float* out, int32_t* group_sums);
/* QuantisedMatrix::dequantise_row (crates/kernels/src/matrix.rs:140-153). */
int nbo_matrix_dequantise_row(const nbo_model* model, int tensor, size_t row, float* out);
/* Shape of archive tensor `tensor`: kind, rows, columns, group, bits. */
int nbo_tensor_info(const nbo_model* model, int tensor, int64_t* out5);
/* A codebook product of one input through a matrix given in the archive's
 * representation (QuantisedMatrix, crates/kernels/src/matrix.rs:123-165):
 * packed bits-wide indices (rows × cols·bits/8 bytes), the 2^bits levels and
 * fp16 norms per 128-column group; mode NBO_MODE_INT or NBO_MODE_FLOAT.
 * sums (may be NULL) receives the INT path's per-group int32 sums. */
int nbo_product_raw(int mode, uint32_t bits, const uint8_t* packed, const float* levels, const uint16_t* norms, size_t rows,
                    size_t cols, const float* input, float* out, int32_t* sums);
/* attend_head (crates/kernels/src/attention.rs:53-77) of one head over count
   positions given directly: keys, values [count][dim] int8; scales [count]. */
int nbo_attend_head_raw(int mode, const int8_t* query, float query_scale, const int8_t* keys, const float* key_scales,
                        const int8_t* values, const float* value_scales, size_t count, size_t dim, float* out);
/* LaneWeights::route of one layer for the session in `slot` (crates/model/src/lanes.rs:45-80):
   stream [lanes][d_model]; input [d_model], post [lanes], residual [lanes][lanes]. */
int nbo_route(const nbo_model* model, int layer, int slot, const float* stream, float* input, float* post, float* residual);
/* HadamardWeights::apply of one layer (crates/model/src/hadamard.rs:260-304). */
int nbo_hadamard_apply(const nbo_model* model, int layer, const float* input, float* out);

#ifdef __cplusplus
}
#endif
#endif
