// kernels.h — host launchers of the kernels in kernels.cu.
#pragma once

#include <cuda_runtime.h>

#include <vector>

#include "exactmath.h"
#include "layout.h"

namespace nbk {

void set_exp_constants(const nbx::ExpConstants& constants, const nbx::ExceptionSet& exceptions, cudaStream_t stream);
cudaError_t configure(const nbl::ModelDev& md, int t_cap);
// Kernels the calling thread has launched or recorded into a graph so far
// (the token loop's launchers; the test hooks are not counted).
long launch_counter();
void note_launch();

void launch_embed(const nbl::ModelDev& md, const nbl::Work& w, int M, cudaStream_t st);
// One decoder layer of M tokens. `distinct`: every token of the pass belongs
// to a different sequence (a decode step, or a one-token feed). `engram`: the
// host copy of the layer's engram site, or null.
void launch_layer(const nbl::ModelDev& md, const nbl::LayerDev& L, const nbl::EngramDev* engram, const nbl::CrossLayerDev* cross,
                  const nbl::Work& w, const nbl::KvDev& kv, int M, int layer, int slot, int t_cap, bool distinct, cudaStream_t st);
// CrossWeights::memory of `frames` encoder rows (device): `rows` (frames · d
// floats), `act`/`act_scale` (a K = d activation buffer of `act_rows` rows)
// and `kv` (frames · 2d floats) are scratch; keys/values [layers][frames]
// [heads][64] and their scales [layers][frames][heads] are written.
cudaError_t cross_memory(const nbl::ModelDev& md, const std::vector<nbl::CrossLayerDev>& layers, const float* encoded, int frames,
                         const float* sin_tab, const float* cos_tab, float gate, float* rows, int8_t* act, float* act_scale,
                         int act_rows, float* kv, int8_t* keys, float* kscale, int8_t* values, float* vscale, cudaStream_t st);
void launch_final(const nbl::ModelDev& md, const nbl::Work& w, float* hidden, int M, cudaStream_t st);
// ProbeHead::observe of cell row `row` (0: the embedding, layer + 1) of every
// token of the pass; `stream` holds the lanes after that layer.
void launch_observe(const nbl::ModelDev& md, const nbl::Work& w, const float* stream, int M, int row, cudaStream_t st);
// ProbeHead::pooled (into `pooled`, queries · d) and, with project_out,
// ProbeHead::project (into `out`) of head h (`head`: its host copy) of the
// session in `slot`; `rows`
// (device) lists the model's nrows cell rows; readouts: nrows · probes · d
// floats, weights: nrows · probes floats; act/act_scale: a zeroed one-token
// activation buffer of K-chunk-major rows `act_rows`.
void head_output(const nbl::ModelDev& md, const nbl::HeadDev& head, int h, int slot, const int32_t* rows, int nrows, float* readouts,
                 float* weights, float* pooled, int8_t* act, float* act_scale, int act_rows, float* out, bool project_out,
                 cudaStream_t st);
// Codebook rows dequantised to f32 (QuantisedMatrix::dequantise_row).
void dense_rows(const uint8_t* packed, uint32_t row_bytes, uint32_t bits, const float* levels, const float* norms, int rows, int cols,
                float inv_sqrt_group, float* out, cudaStream_t st);
void fill(float* p, size_t n, float value, cudaStream_t st);
void launch_logits(const nbl::ModelDev& md, const float* hidden, const int32_t* slots, int B, int8_t* act, float* act_scale,
                   float* logits, cudaStream_t st);
void launch_select(const float* logits, int V, const uint32_t* mask, const int32_t* active, uint32_t* next, float* peaks, int B,
                   cudaStream_t st);
void launch_stats(const float* logits, int V, const uint32_t* mask, const int32_t* active, const uint32_t* next,
                  const float* peaks, float* stats, int stats_stride, int B, cudaStream_t st);
void launch_advance(nbl::TokenMeta* meta, int B, cudaStream_t st);
// The attention of a pass (with the head step when `heads`, and the output
// projection's activation step where the shapes allow); false when k_prep
// must still run.
bool launch_attention(const nbl::ModelDev& md, const nbl::LayerDev& L, const nbl::Work& w, const nbl::KvDev& kv, int M, int layer,
                      int t_cap, bool heads, cudaStream_t st);
void launch_debug_hadamard(const nbl::ModelDev& md, const nbl::LayerDev& L, const float* in, float* out, int M, cudaStream_t st);
void launch_debug_math(int op, const float* in, float* out, int n, cudaStream_t st);
void launch_debug_project(const nbl::ModelDev& md, const nbl::QMat& W, const float* in, int K, int M, int8_t* act,
                          float* act_scale, float* out, int out_stride, cudaStream_t st);

cudaError_t launch_product_bench(const nbl::QMat& W, const float* in, int M, int8_t* act, float* act_scale, int act_rows, float* out,
                                 int* error, int reps, float* ms, cudaStream_t st);

// Failure detection test hook: the next `count` k_route CTAs each give up a
// short bounded wait on a barrier no copy completes, set the engine's error
// flag, wait for their own copies and return.
cudaError_t set_expire_route(int count, cudaStream_t st);

// A streaming read of `bytes` (a multiple of 16) from `data` through L2,
// `passes` times per launch; three untimed launches then `reps` timed ones;
// *ms = the mean device time of one launch.
cudaError_t launch_read_bench(const void* data, size_t bytes, int passes, uint32_t* sink, int reps, float* ms, cudaStream_t st);

// The allocation-free product: tokens per call the file-scope scratch holds.
constexpr int STATIC_MAX_TOKENS = 256;
// Looks up this device's copy of the scratch once (cudaGetSymbolAddress with
// the device current; it may load the module, so it belongs before any stream
// capture). Later calls return at once.
cudaError_t static_scratch_setup(int device);
// k_prep + the tensor-core product of M ≤ STATIC_MAX_TOKENS inputs (K = 512,
// 16-byte aligned) into out [M][W.rows]; synchronises `st` and reports in
// *wait_failed whether a bounded wait of the product gave up.
cudaError_t launch_static_project(int device, const nbl::ModelDev& md, const nbl::QMat& W, const float* in, int M, float* out,
                                  cudaStream_t st, int* wait_failed);

// A byte automaton for device grammar masks (grammar.cu): transitions
// [num_states][256] (0 = byte rejected; state 0 = no call machine), complete
// [num_states], the vocabulary's pieces as bytes + offsets [vocab + 1], the
// call's start state and marker ids, and an error word (bit 0: a state out of
// range was met).
struct AutomatonDev {
  const uint32_t* transitions = nullptr;
  const uint8_t* complete = nullptr;
  const uint8_t* bytes = nullptr;
  const uint32_t* offsets = nullptr;
  uint32_t* error = nullptr;
  uint32_t num_states = 0, start = 0, call_start = 0, call_end = 0;
  int vocab = 0;
};
// TokenBytes::allowed for `count` sequences: mask [count][vocab / 32] words.
cudaError_t automaton_mask(const AutomatonDev& a, const uint32_t* states, int count, uint32_t* mask, cudaStream_t st);
// TokenBytes::advance plus the call markers of run_turn for `count` sequences.
cudaError_t automaton_advance(const AutomatonDev& a, const uint32_t* next, int count, uint32_t* states,
                              cudaStream_t st);

}  // namespace nbk
