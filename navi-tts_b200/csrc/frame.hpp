// navi::qwen3tts::Frame on B200: the host side of the persistent frame kernel.
// Interface of the reference's Frame (model/qwen3tts/frame.h:24-71).
#pragma once

#include "runtime.hpp"

#include <cstdint>
#include <memory>
#include <string>

namespace navi::qwen3tts {

struct Sampling {                  // frame.h:24-31, plus top-p and the stream choice
    float temperature = 0.9f;
    int top_k = 50;
    float top_p = 1.0f;
    float repetition_penalty = 1.05f;
    float cp_temperature = 0.9f;
    int cp_top_k = 50;
    float cp_top_p = 1.0f;
    int min_frames = 2;
    int rng = 0;                   // 0 PCG (the reference's stream), 1 Philox
};

struct FrameOptions {              // frame.h:33-36
    int blocks_per_mp = 1;
    uint64_t deadline_us = 200000;   // longest single device-side wait
};

struct KvCache {                   // talker.h:20-24
    int n_layer = 0, max_pos = 0, kv_dim = 0;
    uint16_t ** k = nullptr;       // host array of n_layer device pointers, [max_pos][kv_dim] f16
    uint16_t ** v = nullptr;
    int n_used = 0;
};

struct FrameResult {               // frame.h:38-44
    bool ok = false;
    bool eos = false;
    int32_t codes[16] = {};
    double us = 0;
    int status = 0;
    std::string error;
};

class Frame {
public:
    static std::unique_ptr<Frame> create(const Device & dev, const DeviceWeights & w, const FrameOptions & opt = {});
    ~Frame();

    // The frame keeps MAX_SLOTS stream slots, each with its repetition set and step embedding;
    // the single-stream calls use slot 0 unless told otherwise.
    static constexpr int MAX_SLOTS = 4;

    void reset(int slot = 0);
    FrameResult run_first(const float * d_hidden, const float * d_logits, const float * d_trailing, const Sampling & s,
                          uint64_t seed, int frame_index, int slot = 0);
    FrameResult run(KvCache & kv, int n_past, const float * d_trailing, const Sampling & s, uint64_t seed, int frame_index);
    // launch only; collect() synchronises and returns the last launch's result
    int enqueue(KvCache & kv, int n_past, const float * d_trailing, const Sampling & s, uint64_t seed, int frame_index,
                std::string & err);
    FrameResult collect();
    // Batched decode: nb (1, 2 or 4) streams in distinct slots decode one frame each in one
    // launch that reads every weight once: stream i at position n_past[i] of its own KV cache,
    // with its own trailing row, seed and frame index. collect_batch fills out[0..nb).
    int enqueue_batch(int nb, const int * slots, KvCache * const * kvs, const int * n_past, const float * const * d_trailing,
                      const Sampling & s, const uint64_t * seeds, const int * frame_index, std::string & err);
    void collect_batch(FrameResult * out);
    // Frame 0 of nb (2 or 4) streams in one launch (run_first of each, together): stream i
    // from the post-norm hidden and codec logits of its prefill; collect_batch gives the results.
    int enqueue_first_batch(int nb, const int * slots, const float * const * d_hidden, const float * const * d_logits,
                            const float * const * d_trailing, const Sampling & s, const uint64_t * seeds, const int * frame_index,
                            std::string & err);
    // One talker decoder layer alone (the layer phases of the frame: q/k/v, attention over
    // positions [0, n_past) plus the new one, o, gate/up, down) on the f32 input d_x at
    // position n_past, writing the f32 residual stream after the layer to d_out and the
    // layer's K/V row n_past (configs[0]'s single-layer decode step).
    FrameResult run_layer(int layer, const float * d_x, KvCache & kv, int n_past, float * d_out);

    const float * d_step_out(int slot = 0) const;
    void set_step_in(const float * d_step, int slot = 0);
    int grid_blocks() const;
    // host copies of the last launch's talker hidden, logits and code-predictor logits of
    // stream `index` of that launch
    void inspect(float * hidden, float * logits, float * clogits, int index = 0) const;
    // phase trace of the last launch on CTA `cta` (ns): start, then 4 stamps per phase
    void set_profile(bool on, int cta = 0);
    int profile(uint64_t * out, int cap) const;
    // the device sampler alone (one CTA) on device logits
    static int sample(const Device & dev, const float * d_logits, int vocab, const Sampling & s, uint64_t seed, int frame_index,
                      int codebook, int suppress_from, int eos_id, const uint8_t * d_seen);

    struct Impl;

private:
    Frame() = default;
    std::unique_ptr<Impl> impl_;
};

} // namespace navi::qwen3tts
