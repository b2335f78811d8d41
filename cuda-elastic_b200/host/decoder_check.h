// Acceptance check of the llama2c decoder drop-in (decoder_b200), restating
// the reference's decoder oracle (applications/loom_private/decoder/
// oracle.h, oracle.cpp:31-229): the analytic token progression, upstream
// llama2.c's normalization invariants on every (sequence, step), and a dense
// double-precision evaluation of up to 8 sampled sequences. The check defines
// what a valid run is; nothing here produces outputs for the GPU path.
#pragma once

#include <cstdint>
#include <vector>

namespace ce_host {

struct DecoderShape {
  long long batch, width, vocab, steps;
};

struct DecoderExpect {
  std::vector<int32_t> tokens;      // [batch][steps]
  std::vector<long long> sampled;   // increasing sequence indices
  std::vector<double> normalized;   // [sampled][steps][width]
  std::vector<double> logits;       // [sampled][steps][vocab]
  std::vector<double> probabilities;
  bool consistent = true;           // dense argmax reproduced the progression
};

// Tokens of every sequence and the dense double results of the sampled ones
// (oracle.cpp:86-123), on host threads.
DecoderExpect decoder_expect(const DecoderShape &shape);

// Compares the device outputs (host copies: generated [batch][steps],
// normalized [steps][batch][width], logits and probabilities
// [steps][batch][vocab]) with the expectation; prints the first 8 mismatches
// of each kind and a summary line to stderr (oracle.cpp:125-229).
bool decoder_check(const DecoderShape &shape, const DecoderExpect &expect, const int32_t *generated,
                   const float *normalized, const float *logits, const float *probabilities);

}  // namespace ce_host
