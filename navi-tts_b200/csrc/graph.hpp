// navi::qwen3tts::Graph on B200: the per-utterance loop (reference model/qwen3tts/graph.h:22-79,
// graph.cpp:52-111) over this build's talker prefill and frame kernel. It starts from token
// ids (the text tokenizer is not part of this build) and returns the 16 codes of every frame.
#pragma once

#include "frame.hpp"
#include "talker.hpp"

#include <cstdint>
#include <functional>
#include <memory>
#include <span>
#include <string>
#include <vector>

namespace navi::qwen3tts {

struct SynthRequest {              // graph.h:24-34, from token ids
    std::span<const std::int32_t> ids;
    std::string language = "english";
    std::span<const float> speaker;   // [hidden]
    std::uint64_t seed = 0;
    int max_frames = 600;
    Sampling sampling;
};

struct SynthStats {                // graph.h:36-41
    int n_tokens = 0, n_frames = 0;
    bool hit_cap = false, eos = false;
    double prefill_ms = 0, frames_ms = 0, total_ms = 0, ttfc_ms = 0;   // ttfc: time to the first frame's codes
};

class Graph {
public:
    static std::unique_ptr<Graph> create(const Device & dev, const DeviceWeights & w, const FrameOptions & fopt = {},
                                         int max_prompt_tokens = 1024, int max_frames = 2048);
    ~Graph();
    // Codes of every frame go to on_codes (16 per frame) as they are decoded.
    SynthStats synth(const SynthRequest & req, const std::function<void(const std::int32_t * codes)> & on_codes);
    Talker & talker();
    Frame & frame();

private:
    Graph() = default;
    int hidden_ = 0;
    std::unique_ptr<Talker> talker_;
    std::unique_ptr<Frame> frame_;
};

} // namespace navi::qwen3tts
