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
                                     int max_frames, int vocoder_chunk, int max_streams) {
    std::unique_ptr<Graph> g(new Graph());
    const Params & p = w.params();
    g->hidden_ = p.talker.hidden;
    if (p.codec_sample_rate > 0) g->sample_rate_ = p.codec_sample_rate;
    if (p.codec_upsample > 0) g->upsample_ = p.codec_upsample;
    if (max_streams < 1 || max_streams > Frame::MAX_SLOTS)
        fail("graph: max_streams must be in 1.." + std::to_string(Frame::MAX_SLOTS), NAVI_E_ARG);
    for (int s = 0; s < max_streams; ++s) {
        g->talkers_.push_back(Talker::create(dev, w, max_prompt_tokens, max_prompt_tokens + max_frames + 1));
        if (vocoder_chunk > 0) g->vocoders_.push_back(Vocoder::create(dev, w, vocoder_chunk, max_frames));
    }
    g->frame_ = Frame::create(dev, w, fopt);
    g->codes_.reserve(static_cast<size_t>(max_frames) * 16);
    return g;
}

Graph::~Graph() = default;
Talker & Graph::talker() { return *talkers_[0]; }
Frame & Graph::frame() { return *frame_; }
Vocoder * Graph::vocoder() { return vocoders_.empty() ? nullptr : vocoders_[0].get(); }

SynthStats Graph::synth(const SynthRequest & req, const CodesFn & on_codes, const PcmFn & on_pcm) {
    Talker * talker_ = talkers_[0].get();
    Vocoder * vocoder_ = vocoder();
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

namespace navi::qwen3tts {

std::vector<SynthStats> Graph::synth_batch(std::span<const SynthRequest> reqs, const StreamCodesFn & on_codes, const StreamPcmFn & on_pcm) {
    using clock = std::chrono::steady_clock;
    const auto t0 = clock::now();
    auto ms_since = [&](clock::time_point a) { return std::chrono::duration<double, std::milli>(clock::now() - a).count(); };
    const int n = static_cast<int>(reqs.size());
    if (n < 1 || n > max_streams()) fail("synth_batch: 1.." + std::to_string(max_streams()) + " requests per call", NAVI_E_ARG);
    const bool audio = static_cast<bool>(on_pcm);
    if (audio && vocoders_.empty()) fail("synth_batch: PCM requested from a graph created without a vocoder", NAVI_E_ARG);
    for (const SynthRequest & r : reqs) {
        const Sampling & a = r.sampling, & b = reqs[0].sampling;
        if (a.temperature != b.temperature || a.top_k != b.top_k || a.top_p != b.top_p || a.repetition_penalty != b.repetition_penalty ||
            a.cp_temperature != b.cp_temperature || a.cp_top_k != b.cp_top_k || a.cp_top_p != b.cp_top_p || a.min_frames != b.min_frames ||
            a.rng != b.rng)
            fail("synth_batch: the streams of one call share their sampling settings", NAVI_E_ARG);
    }
    std::vector<SynthStats> st(static_cast<size_t>(n));
    struct Live {
        const Prompt * pr = nullptr;
        int frame = 0, pending = 0, first = 0, batch = 0;
        bool first_audio = true, done = false;
        std::vector<std::int32_t> codes;
        std::vector<float> pcm;
    };
    std::vector<Live> L(static_cast<size_t>(n));
    auto flush = [&](int s, bool final) {
        Live & l = L[static_cast<size_t>(s)];
        if (!audio || l.pending == 0 || (!final && l.pending < (l.first_audio ? l.first : l.batch))) return;
        const auto tv = clock::now();
        Vocoder & v = *vocoders_[static_cast<size_t>(s)];
        const size_t off = l.codes.size() - static_cast<size_t>(l.pending) * 16;
        l.pcm.resize(static_cast<size_t>(l.pending) * v.samples_per_frame());
        v.decode_into(std::span<const std::int32_t>(l.codes.data() + off, static_cast<size_t>(l.pending) * 16), l.pending, l.pcm.data());
        st[static_cast<size_t>(s)].vocoder_ms += ms_since(tv);
        l.pending = 0;
        if (l.first_audio) {
            st[static_cast<size_t>(s)].ttfa_ms = ms_since(t0);
            l.first_audio = false;
        }
        on_pcm(s, std::span<const float>(l.pcm.data(), l.pcm.size()));
    };
    // a decoded frame of stream s: EOS ends it, otherwise its codes are kept and vocoded
    auto take = [&](int s, const FrameResult & r) {
        Live & l = L[static_cast<size_t>(s)];
        SynthStats & ss = st[static_cast<size_t>(s)];
        if (!r.ok) fail("synth_batch: stream " + std::to_string(s) + " frame " + std::to_string(l.frame) + ": " + r.error,
                        r.status ? r.status : NAVI_E_LAUNCH);
        ss.frames_ms += r.us / 1000.0;
        ++l.frame;
        if (r.eos) {
            ss.eos = true;
            l.done = true;
            return;
        }
        l.codes.insert(l.codes.end(), r.codes, r.codes + 16);
        if (on_codes) on_codes(s, r.codes);
        if (ss.n_frames == 0) ss.ttfc_ms = ms_since(t0);
        ++ss.n_frames;
        ++l.pending;
        flush(s, false);
        if (l.frame >= reqs[static_cast<size_t>(s)].max_frames) l.done = true;
    };
    // prompts and prefills of every stream (graph.cpp:52-72 per stream)
    for (int s = 0; s < n; ++s) {
        const SynthRequest & req = reqs[static_cast<size_t>(s)];
        SynthStats & ss = st[static_cast<size_t>(s)];
        Live & l = L[static_cast<size_t>(s)];
        ss.n_tokens = static_cast<int>(req.ids.size()) - 8;
        if (ss.n_tokens < 1) fail("synth_batch: empty text", NAVI_E_ARG);
        if (req.max_frames < 1) fail("synth_batch: max_frames must be positive", NAVI_E_ARG);
        Talker & tk = *talkers_[static_cast<size_t>(s)];
        const auto tp = clock::now();
        l.pr = &tk.build_prompt(req.ids, req.language, req.speaker);
        tk.prefill(*l.pr);
        ss.prefill_ms = ms_since(tp);
        if (l.pr->n_prefill + req.max_frames > tk.kv().max_pos) fail("synth_batch: prompt + max_frames exceed the KV cache", NAVI_E_KV_FULL);
        frame_->reset(s);
        if (audio) {
            Vocoder & v = *vocoders_[static_cast<size_t>(s)];
            v.reset();
            const int maxc = v.max_chunk_frames();
            l.batch = req.vocoder_batch > 0 ? std::min(req.vocoder_batch, maxc) : maxc;
            l.first = req.first_batch > 0 ? std::min(req.first_batch, l.batch) : l.batch;
        }
    }
    // frame 0 of every stream: 4 or 2 at a time in one launch, a last single one alone
    for (int s0 = 0; s0 < n;) {
        const int left = n - s0;
        const int nb = left >= 4 ? 4 : left >= 2 ? 2 : 1;
        const float * hid[Frame::MAX_SLOTS], * lg[Frame::MAX_SLOTS], * trail[Frame::MAX_SLOTS];
        int slots[Frame::MAX_SLOTS], fidx[Frame::MAX_SLOTS];
        uint64_t seeds[Frame::MAX_SLOTS];
        for (int j = 0; j < nb; ++j) {
            const int s = s0 + j;
            const Live & l = L[static_cast<size_t>(s)];
            Talker & tk = *talkers_[static_cast<size_t>(s)];
            hid[j] = tk.d_hidden();
            lg[j] = tk.d_logits();
            trail[j] = l.pr->n_trailing > 0 ? l.pr->trailing : l.pr->tts_pad;
            slots[j] = s;
            fidx[j] = 0;
            seeds[j] = reqs[static_cast<size_t>(s)].seed;
        }
        if (nb == 1) {
            take(s0, frame_->run_first(hid[0], lg[0], trail[0], reqs[static_cast<size_t>(s0)].sampling, seeds[0], 0, s0));
        } else {
            std::string err;
            const int stt = frame_->enqueue_first_batch(nb, slots, hid, lg, trail, reqs[0].sampling, seeds, fidx, err);
            if (stt != NAVI_OK) fail("synth_batch: " + err, stt);
            FrameResult res[Frame::MAX_SLOTS];
            frame_->collect_batch(res);
            for (int j = 0; j < nb; ++j) take(s0 + j, res[j]);
        }
        s0 += nb;
    }
    // frames >= 1 of the running streams, together: groups of 4, 2 and 1 streams per launch
    for (;;) {
        std::vector<int> live;
        for (int s = 0; s < n; ++s)
            if (!L[static_cast<size_t>(s)].done) live.push_back(s);
        if (live.empty()) break;
        size_t at = 0;
        while (at < live.size()) {
            const size_t left = live.size() - at;
            const int nb = left >= 4 ? 4 : left >= 2 ? 2 : 1;
            int slots[Frame::MAX_SLOTS], n_past[Frame::MAX_SLOTS], fidx[Frame::MAX_SLOTS];
            KvCache * kvs[Frame::MAX_SLOTS];
            const float * trail[Frame::MAX_SLOTS];
            uint64_t seeds[Frame::MAX_SLOTS];
            for (int j = 0; j < nb; ++j) {
                const int s = live[at + static_cast<size_t>(j)];
                const Live & l = L[static_cast<size_t>(s)];
                const int i = l.frame;
                slots[j] = s;
                kvs[j] = &talkers_[static_cast<size_t>(s)]->kv();
                n_past[j] = l.pr->n_prefill + i - 1;
                trail[j] = i < l.pr->n_trailing ? l.pr->trailing + static_cast<size_t>(i) * hidden_ : l.pr->tts_pad;
                seeds[j] = reqs[static_cast<size_t>(s)].seed;
                fidx[j] = i;
            }
            std::string err;
            const int stt = frame_->enqueue_batch(nb, slots, kvs, n_past, trail, reqs[static_cast<size_t>(slots[0])].sampling, seeds, fidx, err);
            if (stt != NAVI_OK) fail("synth_batch: " + err, stt);
            FrameResult res[Frame::MAX_SLOTS];
            frame_->collect_batch(res);
            for (int j = 0; j < nb; ++j) take(slots[j], res[j]);
            at += static_cast<size_t>(nb);
        }
    }
    for (int s = 0; s < n; ++s) {
        SynthStats & ss = st[static_cast<size_t>(s)];
        ss.hit_cap = !ss.eos;
        flush(s, true);
        ss.total_ms = ms_since(t0);
        ss.audio_s = static_cast<double>(ss.n_frames) * upsample_ / sample_rate_;
        ss.rtf = ss.audio_s > 0 ? ss.total_ms / 1000.0 / ss.audio_s : 0.0;
    }
    return st;
}

} // namespace navi::qwen3tts
