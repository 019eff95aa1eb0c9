// navi::qwen3tts::Talker on B200: the prompt and the prefill of the talker, which fill the
// KV cache the frame kernel decodes from. Interface of the reference's Talker
// (model/qwen3tts/talker.h:20-67).
#pragma once

#include "frame.hpp"
#include "runtime.hpp"

#include <cstdint>
#include <memory>
#include <span>
#include <string>

namespace navi::qwen3tts {

struct Prompt {                    // talker.h:26-32: device rows, valid until the next build_prompt
    const float * prefill = nullptr;   // [n_prefill][hidden]
    const float * trailing = nullptr;  // [n_trailing][hidden] text rows fed one per frame
    const float * tts_pad = nullptr;   // [hidden] fed once the trailing rows run out
    int n_prefill = 0, n_trailing = 0;
};

class Talker {
public:
    static std::unique_ptr<Talker> create(const Device & dev, const DeviceWeights & w, int max_prompt_tokens = 1024,
                                          int max_positions = 4096);
    ~Talker();

    // ids: the tokenised "<|im_start|>assistant\n{text}<|im_end|>\n<|im_start|>assistant\n"
    // (3 header ids, the text, 5 trailer ids); language: "" or "auto" for none; speaker: [hidden].
    const Prompt & build_prompt(std::span<const std::int32_t> ids, const std::string & language, std::span<const float> speaker);
    // Runs the prompt's prefill rows through every layer at positions 0..n-1 and fills kv().
    void prefill(const Prompt & p);

    KvCache & kv();
    const float * d_hidden() const;   // post-norm hidden of the last prefill row [hidden]
    const float * d_logits() const;   // its codec logits [talker vocab]
    double last_ms() const;

    struct Impl;

private:
    Talker() = default;
    std::unique_ptr<Impl> impl_;
};

} // namespace navi::qwen3tts
