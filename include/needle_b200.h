/*
 * needle_b200.h — C ABI of the B200-native Needle-3 token loop.
 *
 * This is the drop-in boundary for rustyneedle's model + generation layers.
 * Each entry point names the reference interface it replaces (paths are
 * inside the rustyneedle workspace). Plain pointers and sizes only; every
 * call returns an nb_status and never aborts on bad input. The message of the
 * last failure on the calling thread is returned by nb_last_error().
 *
 * Threading: an nb_model is immutable once opened and may be shared by host
 * threads (the reference's Arc<Model>, docs/library.md:150). Sessions and
 * batches are single-thread objects (Send, not Sync), like rustyneedle's
 * Session. All device work of a model runs on that model's CUDA stream.
 */
#ifndef NEEDLE_B200_H
#define NEEDLE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum nb_status {
  NB_OK = 0,
  NB_ERR_IO = -1,               /* CactError::Io (crates/cact/src/error.rs:6) */
  NB_ERR_ARCHIVE = -2,          /* CactError::{Truncated, WrongTag, UnknownElementKind, BadLayout, OutOfBounds} */
  NB_ERR_DEPTH = -3,            /* ModelError::Depth (crates/model/src/model.rs:15) */
  NB_ERR_ARGUMENT = -4,         /* a null pointer, an out-of-range token id or size */
  NB_ERR_UNSUPPORTED = -5,      /* an archive feature this build does not run (conv taps, engram, probe heads) */
  NB_ERR_CUDA = -6,             /* a CUDA runtime failure; the message names the call */
  NB_ERR_CONTEXT_OVERFLOW = -7, /* RawTurn.overflow (crates/generate/src/generator.rs:77-89) */
  NB_ERR_KV_EXHAUSTED = -8,     /* the device KV page pool has no free page */
  NB_ERR_TIMEOUT = -9,          /* a bounded device wait gave up */
  NB_ERR_NO_DEVICE = -10        /* no CUDA device, or the library was built for another architecture */
} nb_status;

typedef struct nb_model nb_model;
typedef struct nb_session nb_session;
typedef struct nb_batch nb_batch;

typedef struct nb_options {
  int32_t device;          /* CUDA ordinal; -1 = the current device */
  uint32_t max_sessions;   /* concurrent sessions on this model (0 = 256) */
  uint32_t kv_pages;       /* 64-position KV pages in the pool (0 = enough for max_sessions at max_seq_len) */
  uint32_t max_batch_tokens; /* tokens in one forward pass (prefill chunk; 0 = 1024) */
} nb_options;

typedef struct nb_model_config {
  uint32_t vocab, output_vocab, d_model, num_heads, num_kv_heads, num_layers, head_dim, max_seq_len, hada_n, lanes;
  uint32_t depth;          /* active layers */
  int32_t active_layers[64];
  float rope_theta;
} nb_model_config;

typedef struct nb_step_stats {
  float probability;       /* allowed_statistics().probability (generator.rs:182-194) */
  float mass;              /* allowed_statistics().mass */
  int32_t status;          /* NB_OK or NB_ERR_CONTEXT_OVERFLOW for this sequence */
} nb_step_stats;

const char* nb_last_error(void);

/* Model::open (crates/model/src/model.rs:52-56): reads the .cact archive
 * (crates/cact/src/archive.rs:37-70, layout.rs:190-209), repacks every
 * codebook-quantised matrix into its device layout and uploads it once.
 * `options` may be NULL. */
nb_status nb_model_open(const char* path, const nb_options* options, nb_model** out);

/* Model::with_depth (model.rs:63-66, ladder.rs:22-29): a new handle over the
 * same device weights running the first `depth` rungs of the bisection ladder.
 * NB_ERR_DEPTH when depth is outside [2, layers]. */
nb_status nb_model_with_depth(const nb_model* model, uint32_t depth, nb_model** out);

/* Model::config (model.rs:80-82) and Model::active_layers (model.rs:76-78). */
nb_status nb_model_get_config(const nb_model* model, nb_model_config* out);

/* Drops one handle; device memory is freed with the last handle of a model. */
void nb_model_release(nb_model* model);

/* Session::new (crates/model/src/session.rs:30-42). */
nb_status nb_session_create(nb_model* model, nb_session** out);

/* Session: Clone — the prefix cache (generator.rs:36-47). KV pages are shared
 * copy-on-write; the clone costs no device copy until one side appends into a
 * shared partial page. */
nb_status nb_session_clone(const nb_session* session, nb_session** out);

void nb_session_release(nb_session* session);

/* Session::feed (session.rs:56-70): the prompt runs as batched forward
 * passes; results are bit-identical to pushing the tokens one at a time. */
nb_status nb_session_feed(nb_session* session, const uint32_t* ids, size_t count);

/* Several sessions' Session::feed (session.rs:56-70) in one call: their
 * prompts are packed, in session order, into shared forward passes of up to
 * the model's batch-token capacity (options.max_batch_tokens); each session's
 * state is bit-identical to feeding it alone. ids[i] holds counts[i] tokens
 * of sessions[i]. The sessions must be distinct and belong to one model with
 * the same active layers. No reference counterpart: the reference prefills
 * one session at a time (prefill.rs:10-99). */
nb_status nb_sessions_feed(nb_session* const* sessions, const uint32_t* const* ids, const size_t* counts, size_t n);

/* Session::push (session.rs:72-148): one token through every active layer. */
nb_status nb_session_push(nb_session* session, uint32_t id);

/* Session::logits (session.rs:166-177) into a caller-owned host buffer of
 * at least output_vocab floats. */
nb_status nb_session_logits(nb_session* session, float* out, size_t capacity);

/* Session::head_output (session.rs:150-154): the probe head `code`'s
 * projection of its pooled readout (ProbeHead::pooled and ::project,
 * heads.rs:85-125), observed over every token the session has fed. Writes
 * min(capacity, n) floats to `out` and n to *count (may be NULL).
 * NB_ERR_ARGUMENT when the model has no head with that code (the reference's
 * None). */
nb_status nb_session_head_output(nb_session* session, uint32_t code, float* out, size_t capacity, size_t* count);

/* Session::pooled_readout (session.rs:156-160): the pooled readout itself,
 * queries x d_model floats (Engine::embed reads head 2's, CONFIDENCE_HEAD, engine.rs:110-120). */
nb_status nb_session_pooled_readout(nb_session* session, uint32_t code, float* out, size_t capacity, size_t* count);

/* Whistle (crates/whistle): a cross-attention memory of one encoder output.
 * CrossWeights::memory (whistle/src/cross.rs:58-99): the gated positional
 * signal added to `encoded` ([frames][d_model] f32, host memory), then every
 * decoder layer's int8 keys and values. NB_ERR_UNSUPPORTED when the archive
 * carries no audio section; frames in 1..2048 (a 30-second window is 1500). */
typedef struct nb_cross_memory nb_cross_memory;
typedef struct nb_token_automaton nb_token_automaton;
nb_status nb_cross_memory_create(nb_model* model, const float* encoded, size_t frames, nb_cross_memory** out);
void nb_cross_memory_release(nb_cross_memory* memory);

/* Session::push_with(token, Some(CrossState)) for every later pass of the
 * session (session.rs:126-128, whistle lib.rs:255-293): each layer's cross
 * attention over `memory` runs after its self-attention residual. NULL
 * detaches. The session keeps the memory alive; clones share it. */
nb_status nb_session_set_cross(nb_session* session, nb_cross_memory* memory);

/* AudioManifest::text_vocab (crates/cact/src/layout.rs:265-279): the ids below
 * it are text, those from it on name languages; 0 without an audio section. */
size_t nb_model_text_vocab(const nb_model* model);

/* Session::len (session.rs:44-46). */
size_t nb_session_len(const nb_session* session);

/* Greedy selection of generator.rs:99-116 for one session: logits, the
 * optional packed grammar bitset (V/32 words, bit set = allowed), argmax or
 * argmax_allowed (generator.rs:147-165, falling back to the unrestricted
 * argmax when nothing is allowed) and allowed_statistics; the chosen token is
 * then pushed. `stats` may be NULL. */
nb_status nb_session_step(nb_session* session, const uint32_t* mask_bits, uint32_t* next, nb_step_stats* stats);

/* Batched decode (no reference equivalent: run_turn's loop,
 * generator.rs:99-130, over B independent sessions). The batch owns a CUDA
 * graph of one step; the sessions must all belong to `model`. */
nb_status nb_batch_create(nb_model* model, nb_session* const* sessions, uint32_t count, nb_batch** out);
void nb_batch_release(nb_batch* batch);

/* One greedy step of every session in the batch, all on device: logits,
 * mask, argmax, statistics and the push of the chosen tokens. mask_bits is
 * count × (output_vocab/32) words or NULL (unconstrained); next receives
 * count token ids; stats (count entries) may be NULL. A sequence whose context
 * is full is not stepped: its stats.status is NB_ERR_CONTEXT_OVERFLOW and its
 * next id is UINT32_MAX. */
nb_status nb_batch_step(nb_batch* batch, const uint32_t* mask_bits, uint32_t* next, nb_step_stats* stats);

/* Device-resident variant for callers that keep data on the GPU: mask_bits
 * (may be NULL) and next (count uint32) are device pointers on the model's
 * device. stats_device must be NULL: statistics come from nb_batch_step. */
nb_status nb_batch_step_device(nb_batch* batch, const uint32_t* mask_bits_device, uint32_t* next_device,
                               nb_step_stats* stats_device);

/* `steps` greedy steps of the batch back to back on the device, without a
 * host round trip between them (unconstrained, or under per-step device
 * masks: steps × count × (output_vocab/32) words). tokens_device (steps ×
 * count, may be NULL) receives the chosen ids; elapsed_ms (may be NULL) the
 * device time of the run, measured with CUDA events on the model's stream.
 * Fails with NB_ERR_CONTEXT_OVERFLOW, before any work, when a session cannot
 * take `steps` more tokens. */
nb_status nb_batch_run(nb_batch* batch, uint32_t steps, const uint32_t* mask_bits_device, uint32_t* tokens_device,
                       float* elapsed_ms);

/* Device grammar masks. The reference builds each constrained step's mask on
 * the host: TokenBytes::allowed (crates/grammar/src/mask.rs:28-42) steps a
 * clone of the call machine through every vocabulary piece, and
 * TokenBytes::advance (mask.rs:44-49) steps the live machine with the chosen
 * piece, inside run_turn (crates/generate/src/generator.rs:102-124). Here the
 * caller compiles the machine into a byte automaton and both operations run on
 * the device for a whole batch.
 *
 * transitions: num_states × 256 next states (0 = the byte is rejected; a value
 * with the top bit set also rejects the byte and leaves the machine in the state
 * of the low 31 bits, as the reference's array and object stages change state on
 * some bytes they reject, machine.rs:357-364, 444-451, 495-505); state 0
 * means "no call machine" and must not be complete. complete[s] != 0: the
 * machine is done (CallMachine::is_complete, call.rs:83-85), so only call_end is
 * allowed. start_state: the state grammar.start() enters after call_start.
 * token_bytes / token_offsets (vocab + 1 entries): each output id's piece as
 * TokenBytes::bytes gives it (mask.rs:24-26; an empty range = no bytes, never
 * allowed). vocab must equal the model's output vocabulary. The arrays are
 * copied; they may be freed on return. */
#define NB_AUTOMATON_MAX_STATES (1u << 20)
#define NB_AUTOMATON_MAX_PIECE 255u
nb_status nb_token_automaton_create(nb_model* model, const uint32_t* transitions, uint32_t num_states,
                                    const uint8_t* complete, uint32_t start_state, const uint8_t* token_bytes,
                                    const uint32_t* token_offsets, uint32_t vocab, uint32_t call_start,
                                    uint32_t call_end, nb_token_automaton** out);
void nb_token_automaton_release(nb_token_automaton* automaton);

/* Mask words (count × vocab/32, the layout nb_batch_step_device takes) for
 * `count` sequences whose automaton states are states_device[0..count): all ids
 * for state 0, call_end alone for a complete state, else the ids whose bytes the
 * automaton accepts from that state (TokenBytes::allowed). Device pointers;
 * queued on the model's stream, no synchronisation. */
nb_status nb_token_automaton_mask(nb_token_automaton* automaton, const uint32_t* states_device, uint32_t count,
                                  uint32_t* mask_bits_device);

/* Advances states_device with the chosen ids next_device (generator.rs:118-124):
 * call_start with state 0 enters start_state, call_end returns to 0, any other
 * id steps the automaton through its bytes and keeps the last accepted state;
 * UINT32_MAX (a sequence not stepped) leaves the state. Queued on the model's
 * stream, no synchronisation. */
nb_status nb_token_automaton_advance(nb_token_automaton* automaton, const uint32_t* next_device, uint32_t count,
                                     uint32_t* states_device);

/* Waits for the model's stream and reports NB_ERR_ARGUMENT if a mask or an
 * advance since the last check met a state >= num_states (such a sequence was
 * masked as unconstrained and not advanced); clears the report. */
nb_status nb_token_automaton_check(nb_token_automaton* automaton);

/* A compiled tool-call grammar: the byte automaton of CallGrammar's
 * CallMachine (crates/grammar/src/call.rs:33-174) for the tools JSON that
 * CallGrammar::from_tools_json takes (call.rs:16-31, 47-49; the schemas as
 * schema::compile reads them, schema.rs:29-141), ready for
 * nb_token_automaton_create. Host only: no GPU is needed.
 *
 * require_call != 0 is CallGrammar::require_call (call.rs:51-55): no empty
 * call list, and with permitted (permitted_count indices into the tool list)
 * only those tools; permitted must be NULL without require_call. The
 * automaton's states are the call machine's reachable states (state 0 = no
 * machine); exploring more than max_states (0 = NB_AUTOMATON_MAX_STATES)
 * fails with NB_ERR_UNSUPPORTED, the caller then keeps building masks on the
 * host. Malformed JSON fails with NB_ERR_ARGUMENT. */
typedef struct nb_call_grammar nb_call_grammar;
nb_status nb_call_grammar_compile(const char* tools_json, int require_call, const uint32_t* permitted, size_t permitted_count,
                                  uint32_t max_states, nb_call_grammar** out);
/* Its number of states S (state 0 included). */
uint32_t nb_call_grammar_states(const nb_call_grammar* grammar);
/* Copies its tables: transitions (S × 256), complete (S) and the start state
 * (CallMachine::start, call.rs:57-59), in nb_token_automaton_create's form. */
nb_status nb_call_grammar_tables(const nb_call_grammar* grammar, uint32_t* transitions, uint8_t* complete,
                                 uint32_t* start_state);
void nb_call_grammar_release(nb_call_grammar* grammar);

/* Waits for the model's stream. */
nb_status nb_model_synchronize(nb_model* model);

/* Builds the table of inputs where this host's libm expf differs from the
 * correctly rounded exponential (used by the device sigmoid to reproduce
 * f32::exp exactly) and writes it to `path`. Runs on the host CPU. */
nb_status nb_build_expf_table(const char* path);

/* Allocation-free codebook product. It has no counterpart in the reference.
 * It serves callers that may not allocate device memory — a host that has
 * given all of the GPU's memory to its own pool, or a thread that must not
 * take the device-wide synchronisation cudaMalloc/cudaFree imply — with the
 * product of one device matrix, the same result the model's own passes
 * compute with it: which = 0
 * the fused q/k/v/gate rows of `layer`, 1 its out_proj, 2 the tied embedding.
 * in_device: count × 512 floats (16-byte aligned), out_device: count × rows
 * floats, both device memory of the model's GPU; stream: a cudaStream_t of that
 * GPU, or NULL for the model's stream. Returns when the product is complete.
 * Its scratch is a fixed array of the library, one per GPU, that holds at most
 * 256 tokens: a larger count fails with NB_ERR_ARGUMENT, before any work. The
 * first call on a GPU looks the array up (make it before any stream capture).
 * Every call shares the array: calls that overlap in time race on it. */
nb_status nb_model_project_static(nb_model* model, int which, uint32_t layer, const float* in_device, uint32_t count,
                                  float* out_device, void* stream);

#ifdef __cplusplus
}
#endif
#endif
