// Device grammar masks over a token automaton.
//
// The reference builds each constrained step's mask on the host:
// TokenBytes::allowed (crates/grammar/src/mask.rs:28-42) clones the call
// machine once per vocabulary piece and steps it byte by byte, and
// TokenBytes::advance (mask.rs:44-49) steps the live machine with the chosen
// piece. Here the machine is given as a byte automaton — transitions
// [state][256]: the next state; 0 = the byte is rejected; the top bit set =
// the byte is rejected and the machine moves to the state in the low 31 bits
// (the reference's array and object stages change state on some bytes they
// reject) — compiled by the caller (nb_call_grammar_compile builds it from the
// tools JSON), and both operations run on the device for a whole batch:
//
//   states[b] == 0      no call machine (generator.rs:110, argmax over all ids)
//   complete[states[b]] the machine is done; only call_end is allowed
//                       (generator.rs:103, `active.is_complete()`)
//   otherwise           token t is allowed when its bytes are non-empty and
//                       every byte is accepted (mask.rs:31-40)
//
// and the advance follows generator.rs:118-124: call_start with no machine
// enters `start`, call_end leaves it, any other token steps the machine
// through its bytes until the first rejected one (TokenBytes::advance's
// `all`), which leaves the state or moves it where the top bit says.
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"

namespace nbk {

constexpr int AUTOMATON_THREADS = 256;
constexpr int AUTOMATON_ROUNDS = 4;  // tokens per thread: a CTA covers 1024 ids
constexpr uint32_t AUTOMATON_BAD_STATE = 1u;
constexpr uint32_t REJECT_MOVES = 0x80000000u;  // a rejected byte that still changes the state

// grid (ceil(V / 1024), count), block 256. Each warp's 32 consecutive ids form
// one mask word (ballot). The first byte of every piece is looked up in the
// sequence's own transition row, staged in shared memory; the remaining bytes
// walk the table, which stays in L2 (4 bytes × 256 per state).
__global__ void __launch_bounds__(AUTOMATON_THREADS)
    k_automaton_mask(const uint32_t* __restrict__ transitions, uint32_t num_states, const uint8_t* __restrict__ complete,
                     const uint8_t* __restrict__ bytes, const uint32_t* __restrict__ offsets, int vocab,
                     uint32_t call_end, const uint32_t* __restrict__ states, uint32_t* __restrict__ mask,
                     uint32_t* __restrict__ error) {
  __shared__ uint32_t s_row[256];
  const int b = blockIdx.y, tid = threadIdx.x, lane = tid & 31;
  const int words = vocab / 32;
  uint32_t s = states[b];
  const bool bad = s >= num_states;
  if (bad) {
    if (tid == 0 && blockIdx.x == 0) atomicOr(error, AUTOMATON_BAD_STATE);
    s = 0;  // reported through the error word; masked as unconstrained
  }
  const bool done = s != 0 && complete[s] != 0;
  const bool walk = s != 0 && !done;
  if (walk) s_row[tid] = transitions[(size_t)s * 256 + tid];
  __syncthreads();
  const int base = blockIdx.x * AUTOMATON_THREADS * AUTOMATON_ROUNDS;
#pragma unroll
  for (int r = 0; r < AUTOMATON_ROUNDS; ++r) {
    const int t = base + r * AUTOMATON_THREADS + tid;
    bool ok = false;
    if (t < vocab) {
      if (!walk) {
        ok = done ? (uint32_t)t == call_end : true;
      } else {
        const uint32_t o = offsets[t], e = offsets[t + 1];
        if (e > o) {
          // a rejection, with or without a state change, ends the walk: the
          // entry is then 0 or has the top bit set, both not positive as int32
          int32_t q = (int32_t)s_row[bytes[o]];
          for (uint32_t k = o + 1; q > 0 && k < e; ++k) q = (int32_t)transitions[(size_t)q * 256 + bytes[k]];
          ok = q > 0;
        }
      }
    }
    const uint32_t word = __ballot_sync(0xffffffffu, ok);
    const int first = t - lane;
    if (lane == 0 && first < vocab) mask[(size_t)b * words + (first >> 5)] = word;
  }
}

// One thread per sequence. next[b] == UINT32_MAX marks a sequence that was not
// stepped (full context); its state stays.
__global__ void k_automaton_advance(const uint32_t* __restrict__ transitions, uint32_t num_states,
                                    const uint8_t* __restrict__ bytes, const uint32_t* __restrict__ offsets, int vocab,
                                    uint32_t start, uint32_t call_start, uint32_t call_end,
                                    const uint32_t* __restrict__ next, int count, uint32_t* __restrict__ states,
                                    uint32_t* __restrict__ error) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= count) return;
  const uint32_t t = next[b];
  uint32_t s = states[b];
  if (t == 0xffffffffu) return;
  if (s >= num_states) {
    atomicOr(error, AUTOMATON_BAD_STATE);
    return;
  }
  if (t == call_start && s == 0) {
    s = start;
  } else if (t == call_end) {
    s = 0;
  } else if (s != 0 && t < (uint32_t)vocab) {
    for (uint32_t k = offsets[t], e = offsets[t + 1]; k < e; ++k) {
      const uint32_t q = transitions[(size_t)s * 256 + bytes[k]];
      if (q == 0) break;
      if (q & REJECT_MOVES) {
        s = q & ~REJECT_MOVES;
        break;
      }
      s = q;
    }
  }
  states[b] = s;
}

cudaError_t automaton_mask(const AutomatonDev& a, const uint32_t* states, int count, uint32_t* mask, cudaStream_t st) {
  if (count <= 0) return cudaSuccess;
  const int per_cta = AUTOMATON_THREADS * AUTOMATON_ROUNDS;
  const dim3 grid((unsigned)((a.vocab + per_cta - 1) / per_cta), (unsigned)count);
  k_automaton_mask<<<grid, AUTOMATON_THREADS, 0, st>>>(a.transitions, a.num_states, a.complete, a.bytes, a.offsets,
                                                       a.vocab, a.call_end, states, mask, a.error);
  note_launch();
  return cudaGetLastError();
}

cudaError_t automaton_advance(const AutomatonDev& a, const uint32_t* next, int count, uint32_t* states,
                              cudaStream_t st) {
  if (count <= 0) return cudaSuccess;
  k_automaton_advance<<<(count + 127) / 128, 128, 0, st>>>(a.transitions, a.num_states, a.bytes, a.offsets, a.vocab,
                                                          a.start, a.call_start, a.call_end, next, count, states,
                                                          a.error);
  note_launch();
  return cudaGetLastError();
}

}  // namespace nbk
