// The device sampler with no device allocation: its working arrays and result word live
// in one file-scope device array (sample_static.cu).  No counterpart in the reference.
#pragma once

#include "frame.hpp"

namespace navi::qwen3tts {

// Largest vocabulary the static scratch holds.
constexpr int SAMPLE_STATIC_MAX_VOCAB = 32768;

// Same arguments, result and numerics as Frame::sample.  Throws navi::Error with
// NAVI_E_ARG for a vocabulary above SAMPLE_STATIC_MAX_VOCAB.
int sample_static(const Device & dev, const float * d_logits, int vocab, const Sampling & s, uint64_t seed, int frame_index,
                  int codebook, int suppress_from, int eos_id, const uint8_t * d_seen);

} // namespace navi::qwen3tts
