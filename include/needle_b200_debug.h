/*
 * needle_b200_debug.h — kernel-level test hooks of the B200 Needle-3 library.
 *
 * These entry points are not part of the drop-in boundary (needle_b200.h):
 * the parity tests use them to compare single kernels with the CPU
 * restatement. Buffers are host memory; each call synchronises.
 */
#ifndef NEEDLE_B200_DEBUG_H
#define NEEDLE_B200_DEBUG_H

#include "needle_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Element-wise device math on the model's GPU: op 0 = f32::exp as the host
 * libm computes it, 1 = sigmoid (crates/kernels/src/ops.rs:69-71),
 * 2 = fast_exp (ops.rs:83-90), 3 = silu (ops.rs:74-76), 4 = the Sinkhorn
 * reciprocal 1 / max(x, f32::MIN_POSITIVE) (ops.rs:206, 211) for x <= 4 (the
 * row and column totals never exceed 4). */
nb_status nb_debug_math(nb_model* model, int op, const float* in, float* out, size_t count);

/* QuantisedMatrix::prepare + multiply_vector (crates/kernels/src/matrix.rs:123-165)
 * of `count` inputs through one device matrix: which = 0 the fused
 * q/k/v/gate rows of `layer`, 1 its out_proj, 2 the tied embedding (logits).
 * in: count × columns floats; out: count × rows floats. */
nb_status nb_debug_project(nb_model* model, int which, uint32_t layer, const float* in, size_t count, float* out);

/* HadamardWeights::apply (crates/model/src/hadamard.rs:260-304) of one layer
 * on `count` inputs of d_model values. */
nb_status nb_debug_hadamard(nb_model* model, uint32_t layer, const float* in, size_t count, float* out);

/* The product microbenchmark (no model): QuantisedMatrix::prepare +
 * multiply_vector (crates/kernels/src/matrix.rs:123-165) of `count` inputs
 * through a matrix given in the archive's representation — packed bits-wide
 * indices per row (rows × cols·bits/8 bytes, matrix.rs:622-631), the 2^bits
 * codebook levels and fp16 norms per 128-column group — on device `device`.
 * bits 2 or 4, cols 512 or 2048. in: count × cols floats; out: count × rows
 * floats. With reps > 0, *ms_per_product (may be NULL) receives the mean device
 * time of the product kernel alone, activations already quantised. */
nb_status nb_debug_product(int device, uint32_t bits, const uint8_t* packed, const float* levels, const uint16_t* norms, uint32_t rows,
                           uint32_t cols, const float* in, uint32_t count, float* out, uint32_t reps, float* ms_per_product);

/* Failure detection test: the next `count` routing CTAs (k_route) on the
 * model's GPU each give up a short bounded wait on a barrier no copy will
 * complete, set the engine's error flag and return once their own copies have
 * landed (nothing asynchronous outlives them); the next
 * synchronising call that ran them returns NB_ERR_TIMEOUT, as for any device
 * wait that gave up. The session that ran them is left inconsistent; other
 * sessions and models are not affected. No reference counterpart. */
nb_status nb_debug_expire_waits(nb_model* model, uint32_t count);

/* A plain streaming read of a `bytes`-long device buffer (a multiple of 16)
 * on device `device`, through L2 with 16-byte loads, four 512-thread CTAs per
 * SM, `passes` (1-4096) reads of the whole buffer per launch: *ms_per_read
 * receives the mean device time of one read of the buffer over `reps`
 * launches after three untimed ones (CUDA events). Below the L2 size it
 * measures the L2 read bandwidth, well above it the HBM read bandwidth. No
 * reference counterpart: the denominator of the batch-1 roofline. */
nb_status nb_debug_read_bandwidth(int device, size_t bytes, uint32_t passes, uint32_t reps, float* ms_per_read);

/* The session's final hidden state (session.rs:140-143): d_model floats. */
nb_status nb_debug_hidden(nb_session* session, float* out);

/* The int8 KV cache of one layer in the reference's layout
 * (model/src/attention.rs:37-45): keys/values [len][kv_heads][64],
 * scales [kv_heads][len]. */
nb_status nb_debug_kv(nb_session* session, uint32_t layer, int8_t* keys, float* key_scales, int8_t* values,
                      float* value_scales);

/* Replays the attention of every active layer over the batch's current
 * positions `reps` times (per layer the step's launches, one per group of
 * sequences, one after another) and reports the mean device time of one
 * layer's attention (CUDA events on the model's stream) and the KV bytes it
 * must read (keys, values and their scales of every attended position). */
nb_status nb_debug_time_attention(nb_batch* batch, uint32_t reps, float* ms_per_launch, double* bytes_per_launch);

/* A cross memory's keys, key scales, values and value scales of one decoder
 * layer: [frames][heads][64] int8 and [frames][heads] f32 each. */
nb_status nb_debug_cross_memory(const nb_cross_memory* memory, int layer, int8_t* keys, float* key_scales, int8_t* values,
                                float* value_scales);

/* Kernels in the batch's step graph (the last one recorded; 0 before the
 * first step). No reference counterpart: the bench's launch count. */
nb_status nb_debug_step_kernels(nb_batch* batch, uint32_t* kernels);

#ifdef __cplusplus
}
#endif
#endif
