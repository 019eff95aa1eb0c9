// navi::qwen3tts::Graph on B200: the per-utterance loop (reference model/qwen3tts/graph.h:22-79,
// graph.cpp:52-111) over this build's talker prefill, frame kernel and vocoder. It starts from
// token ids (the text tokenizer is not part of this build), hands the 16 codes of every frame to
// on_codes and streams the PCM of each vocoder batch to on_pcm.
#pragma once

#include "frame.hpp"
#include "talker.hpp"
#include "vocoder.hpp"

#include <cstdint>
#include <functional>
#include <memory>
#include <span>
#include <string>
#include <vector>

namespace navi::qwen3tts {

// Streaming batch sizes in frames (graph.h:29-30): the first vocoder call takes 4 frames (time
// to first audio), the later ones 16. The PCM does not depend on the batching.
constexpr int STREAM_FIRST_BATCH = 4;
constexpr int STREAM_BATCH = 16;

struct SynthRequest {              // graph.h:32-41, from token ids
    std::span<const std::int32_t> ids;
    std::string language = "english";
    std::span<const float> speaker;   // [hidden]
    std::uint64_t seed = 0;
    int max_frames = 600;
    Sampling sampling;
    int vocoder_batch = 0;            // frames per vocoder call; 0 = the vocoder's max_chunk_frames
    int first_batch = 0;              // frames in the first call; 0 = vocoder_batch
};

struct SynthStats {                // graph.h:43-48
    int n_tokens = 0, n_frames = 0;
    bool hit_cap = false, eos = false;
    double prefill_ms = 0, frames_ms = 0, vocoder_ms = 0, total_ms = 0;
    double ttfc_ms = 0;               // time to the first frame's codes
    double ttfa_ms = 0;               // time to the first PCM batch (0 without a PCM consumer)
    double audio_s = 0, rtf = 0;      // seconds of audio; total_ms / 1000 / audio_s
};

class Graph {
public:
    // A talker (prompts up to max_prompt_tokens, KV for max_prompt_tokens + max_frames + 1
    // positions), a frame kernel and, for vocoder_chunk > 0, a vocoder decoding up to
    // vocoder_chunk frames per pass (graph.cpp:22-44 without tokenizer and speaker encoder).
    // max_streams (1..4): the streams synth_batch takes, each with its own talker (KV cache)
    // and vocoder state.
    static std::unique_ptr<Graph> create(const Device & dev, const DeviceWeights & w, const FrameOptions & fopt = {},
                                         int max_prompt_tokens = 1024, int max_frames = 2048, int vocoder_chunk = 32,
                                         int max_streams = 1);
    ~Graph();

    using CodesFn = std::function<void(const std::int32_t * codes)>;
    using PcmFn = std::function<void(std::span<const float> pcm)>;
    // Synthesises `req`. Codes of every frame go to on_codes (16 per frame) as they are
    // decoded; without on_pcm the vocoder is not run (codes only). With it, the frames are
    // vocoded in batches of first_batch, then vocoder_batch frames, plus the remainder at
    // the end, and each batch's 24 kHz f32 PCM goes to on_pcm. Throws navi::Error on a
    // failed frame or vocoder pass.
    SynthStats synth(const SynthRequest & req, const CodesFn & on_codes, const PcmFn & on_pcm = {});

    // Up to max_streams requests at once: each stream gets its prompt and prefill on its own
    // talker (and KV cache), frame 0, then the streams still running decode their frames
    // together in batched launches (Frame::enqueue_batch, 4 / 2 / 1 streams per launch) until
    // each reaches EOS or its max_frames; every stream's frames go through its own vocoder as
    // in synth(). The requests must share their sampling settings (seeds, frame caps and
    // prompts are per stream). Callbacks get the stream's index in reqs. Stream i's codes equal synth(reqs[i])'s
    // whenever its draws agree, which they do unless a float rounding difference of the batched
    // attention split moves a draw that sits on a boundary. Times are from the call's start.
    using StreamCodesFn = std::function<void(int stream, const std::int32_t * codes)>;
    using StreamPcmFn = std::function<void(int stream, std::span<const float> pcm)>;
    std::vector<SynthStats> synth_batch(std::span<const SynthRequest> reqs, const StreamCodesFn & on_codes,
                                        const StreamPcmFn & on_pcm = {});
    int max_streams() const { return static_cast<int>(talkers_.size()); }
    Talker & talker();
    Frame & frame();
    Vocoder * vocoder();          // null when created with vocoder_chunk = 0

private:
    Graph() = default;
    int hidden_ = 0;
    int sample_rate_ = 24000, upsample_ = 1920;
    std::vector<std::unique_ptr<Talker>> talkers_;     // [0] is synth()'s
    std::unique_ptr<Frame> frame_;
    std::vector<std::unique_ptr<Vocoder>> vocoders_;
    std::vector<std::int32_t> codes_;
    std::vector<float> pcm_;
};

} // namespace navi::qwen3tts
