// The per-utterance loop (reference model/qwen3tts/graph.cpp:52-111): prompt and prefill, then
// frame 0 from the prefill's hidden and logits and frame i >= 1 at KV position n_prefill + i - 1,
// each fed the i-th trailing text row (tts_pad once they run out), until EOS or max_frames.
#include "graph.hpp"

#include "../../include/navi_b200.h"

#include <chrono>

namespace navi::qwen3tts {

std::unique_ptr<Graph> Graph::create(const Device & dev, const DeviceWeights & w, const FrameOptions & fopt, int max_prompt_tokens,
                                     int max_frames) {
    std::unique_ptr<Graph> g(new Graph());
    g->hidden_ = w.params().talker.hidden;
    g->talker_ = Talker::create(dev, w, max_prompt_tokens, max_prompt_tokens + max_frames + 1);
    g->frame_ = Frame::create(dev, w, fopt);
    return g;
}

Graph::~Graph() = default;
Talker & Graph::talker() { return *talker_; }
Frame & Graph::frame() { return *frame_; }

SynthStats Graph::synth(const SynthRequest & req, const std::function<void(const std::int32_t * codes)> & on_codes) {
    using clock = std::chrono::steady_clock;
    const auto t0 = clock::now();
    auto ms_since = [&](clock::time_point a) { return std::chrono::duration<double, std::milli>(clock::now() - a).count(); };
    SynthStats st;
    st.n_tokens = static_cast<int>(req.ids.size()) - 8;
    if (st.n_tokens < 1) fail("synth: empty text", NAVI_E_ARG);
    if (req.max_frames < 1) fail("synth: max_frames must be positive", NAVI_E_ARG);
    const Prompt & pr = talker_->build_prompt(req.ids, req.language, req.speaker);
    talker_->prefill(pr);
    st.prefill_ms = ms_since(t0);
    KvCache & kv = talker_->kv();
    if (pr.n_prefill + req.max_frames > kv.max_pos) fail("synth: prompt + max_frames exceed the KV cache", NAVI_E_KV_FULL);
    frame_->reset();
    for (int i = 0; i < req.max_frames; ++i) {
        const float * trailing = i < pr.n_trailing ? pr.trailing + static_cast<size_t>(i) * hidden_ : pr.tts_pad;
        const FrameResult r = i == 0 ? frame_->run_first(talker_->d_hidden(), talker_->d_logits(), trailing, req.sampling, req.seed, 0)
                                     : frame_->run(kv, pr.n_prefill + i - 1, trailing, req.sampling, req.seed, i);
        if (!r.ok) fail("synth: frame " + std::to_string(i) + ": " + r.error, r.status ? r.status : NAVI_E_LAUNCH);
        st.frames_ms += r.us / 1000.0;
        if (r.eos) {
            st.eos = true;
            break;
        }
        on_codes(r.codes);
        if (st.n_frames == 0) st.ttfc_ms = ms_since(t0);
        ++st.n_frames;
    }
    st.hit_cap = !st.eos;
    st.total_ms = ms_since(t0);
    return st;
}

} // namespace navi::qwen3tts
