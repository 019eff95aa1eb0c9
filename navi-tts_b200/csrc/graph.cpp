// The per-utterance loop (reference model/qwen3tts/graph.cpp:52-111): prompt and prefill, then
// frame 0 from the prefill's hidden and logits and frame i >= 1 at KV position n_prefill + i - 1,
// each fed the i-th trailing text row (tts_pad once they run out), until EOS or max_frames.
// Frames wait for the vocoder in a pending list that is flushed once it holds first_batch
// frames (the first time) or vocoder_batch frames (afterwards), and once more at the end.
#include "graph.hpp"

#include "../../include/navi_b200.h"

#include <algorithm>
#include <chrono>

namespace navi::qwen3tts {

std::unique_ptr<Graph> Graph::create(const Device & dev, const DeviceWeights & w, const FrameOptions & fopt, int max_prompt_tokens,
                                     int max_frames, int vocoder_chunk) {
    std::unique_ptr<Graph> g(new Graph());
    const Params & p = w.params();
    g->hidden_ = p.talker.hidden;
    if (p.codec_sample_rate > 0) g->sample_rate_ = p.codec_sample_rate;
    if (p.codec_upsample > 0) g->upsample_ = p.codec_upsample;
    g->talker_ = Talker::create(dev, w, max_prompt_tokens, max_prompt_tokens + max_frames + 1);
    g->frame_ = Frame::create(dev, w, fopt);
    if (vocoder_chunk > 0) g->vocoder_ = Vocoder::create(dev, w, vocoder_chunk, max_frames);
    g->codes_.reserve(static_cast<size_t>(max_frames) * 16);
    return g;
}

Graph::~Graph() = default;
Talker & Graph::talker() { return *talker_; }
Frame & Graph::frame() { return *frame_; }
Vocoder * Graph::vocoder() { return vocoder_.get(); }

SynthStats Graph::synth(const SynthRequest & req, const CodesFn & on_codes, const PcmFn & on_pcm) {
    using clock = std::chrono::steady_clock;
    const auto t0 = clock::now();
    auto ms_since = [&](clock::time_point a) { return std::chrono::duration<double, std::milli>(clock::now() - a).count(); };
    SynthStats st;
    st.n_tokens = static_cast<int>(req.ids.size()) - 8;
    if (st.n_tokens < 1) fail("synth: empty text", NAVI_E_ARG);
    if (req.max_frames < 1) fail("synth: max_frames must be positive", NAVI_E_ARG);
    const bool audio = static_cast<bool>(on_pcm);
    if (audio && !vocoder_) fail("synth: PCM requested from a graph created without a vocoder", NAVI_E_ARG);
    const Prompt & pr = talker_->build_prompt(req.ids, req.language, req.speaker);
    talker_->prefill(pr);
    st.prefill_ms = ms_since(t0);
    KvCache & kv = talker_->kv();
    if (pr.n_prefill + req.max_frames > kv.max_pos) fail("synth: prompt + max_frames exceed the KV cache", NAVI_E_KV_FULL);
    frame_->reset();
    codes_.clear();

    // vocoder batching (graph.cpp:73-87)
    int batch = 0, first = 0;
    if (audio) {
        vocoder_->reset();
        const int maxc = vocoder_->max_chunk_frames();
        batch = req.vocoder_batch > 0 ? std::min(req.vocoder_batch, maxc) : maxc;
        first = req.first_batch > 0 ? std::min(req.first_batch, batch) : batch;
    }
    int pending = 0;
    bool first_audio = true;
    auto flush = [&](bool final) {
        if (!audio || pending == 0 || (!final && pending < (first_audio ? first : batch))) return;
        const auto tv = clock::now();
        const size_t off = codes_.size() - static_cast<size_t>(pending) * 16;
        pcm_.resize(static_cast<size_t>(pending) * vocoder_->samples_per_frame());
        vocoder_->decode_into(std::span<const std::int32_t>(codes_.data() + off, static_cast<size_t>(pending) * 16), pending,
                              pcm_.data());
        st.vocoder_ms += ms_since(tv);
        pending = 0;
        if (first_audio) {
            st.ttfa_ms = ms_since(t0);
            first_audio = false;
        }
        on_pcm(std::span<const float>(pcm_.data(), pcm_.size()));
    };

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
        codes_.insert(codes_.end(), r.codes, r.codes + 16);
        if (on_codes) on_codes(r.codes);
        if (st.n_frames == 0) st.ttfc_ms = ms_since(t0);
        ++st.n_frames;
        ++pending;
        flush(false);
    }
    st.hit_cap = !st.eos;
    flush(true);
    st.total_ms = ms_since(t0);
    st.audio_s = static_cast<double>(st.n_frames) * upsample_ / sample_rate_;
    st.rtf = st.audio_s > 0 ? st.total_ms / 1000.0 / st.audio_s : 0.0;
    return st;
}

} // namespace navi::qwen3tts
