// navi-b200: the command-line front of this build, over the C ABI (include/navi_b200.h).
// Mirrors the reference's `info` and `synth` subcommands (runtime/cli/main.cpp:59-72,
// 247-279) without the text tokenizer: `synth` takes the prompt's token ids.
//
//   navi-b200 info  [--model FILE] [--device N]
//   navi-b200 synth --model FILE (--ids "i,j,..." | --ids-file FILE) --speaker EMB --out OUT.wav
//                   [--seed N] [--language L] [--max-frames N] [--greedy] [--first-batch N]
//                   [--batch N] [--device N]
//
// --ids are the tokenised "<|im_start|>assistant\n{text}<|im_end|>\n<|im_start|>assistant\n"
// (3 header ids, the text, 5 trailer ids), as navi_talker_build_prompt takes them. --speaker
// is a speaker embedding of the talker's hidden size: a 1-D float32 .npy, or raw
// little-endian float32. The WAV is 16-bit PCM mono at the codec's sample rate.
#include "../../include/navi_b200.h"

#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

namespace {

struct Args {
    std::string cmd, model, ids, ids_file, speaker, out, language = "english";
    unsigned long long seed = 0;
    int max_frames = 600, first_batch = 4, batch = 16, device = 0;
    bool greedy = false;
};

int usage(const char * argv0) {
    std::fprintf(stderr,
                 "%s\n"
                 "usage: %s info  [--model FILE] [--device N]\n"
                 "       %s synth --model FILE (--ids \"i,j,...\" | --ids-file FILE) --speaker EMB(.npy|.f32) --out OUT.wav\n"
                 "                [--seed N] [--language L] [--max-frames N] [--greedy] [--first-batch N] [--batch N] [--device N]\n"
                 "  --ids: the tokenised prompt template (3 header ids, the text, 5 trailer ids)\n",
                 navi_version(), argv0, argv0);
    return 2;
}

Args parse(int argc, char ** argv) {
    Args a;
    if (argc < 2) throw std::invalid_argument("no command");
    a.cmd = argv[1];
    for (int i = 2; i < argc; ++i) {
        const std::string s = argv[i];
        auto next = [&](const char * what) -> std::string {
            if (i + 1 >= argc) throw std::invalid_argument(std::string(what) + " needs a value");
            return argv[++i];
        };
        if (s == "--model" || s == "-m") a.model = next("--model");
        else if (s == "--ids") a.ids = next("--ids");
        else if (s == "--ids-file") a.ids_file = next("--ids-file");
        else if (s == "--speaker") a.speaker = next("--speaker");
        else if (s == "--out") a.out = next("--out");
        else if (s == "--language") a.language = next("--language");
        else if (s == "--seed") a.seed = std::stoull(next("--seed"));
        else if (s == "--max-frames") a.max_frames = std::stoi(next("--max-frames"));
        else if (s == "--first-batch") a.first_batch = std::stoi(next("--first-batch"));
        else if (s == "--batch") a.batch = std::stoi(next("--batch"));
        else if (s == "--device") a.device = std::stoi(next("--device"));
        else if (s == "--greedy") a.greedy = true;
        else throw std::invalid_argument("unknown option " + s);
    }
    return a;
}

void check(int st, const char * what) {
    if (st != NAVI_OK) throw std::runtime_error(std::string(what) + ": " + navi_last_error());
}

std::vector<int32_t> parse_ids(const std::string & text) {
    std::vector<int32_t> ids;
    std::string tok;
    std::stringstream ss(text);
    while (ss >> tok) {   // commas and white space both separate
        std::stringstream ts(tok);
        std::string part;
        while (std::getline(ts, part, ','))
            if (!part.empty()) ids.push_back(static_cast<int32_t>(std::stol(part)));
    }
    return ids;
}

std::vector<char> read_file(const std::string & path) {
    std::ifstream f(path, std::ios::binary);
    if (!f) throw std::runtime_error("cannot open " + path);
    return std::vector<char>((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
}

// A 1-D little-endian float32 .npy (format 1.0-3.0), or raw float32.
std::vector<float> read_f32(const std::string & path) {
    const std::vector<char> b = read_file(path);
    size_t off = 0;
    if (b.size() >= 10 && std::memcmp(b.data(), "\x93NUMPY", 6) == 0) {
        const int major = static_cast<unsigned char>(b[6]);
        size_t hlen, hstart;
        if (major == 1) { hlen = static_cast<unsigned char>(b[8]) | (static_cast<unsigned char>(b[9]) << 8); hstart = 10; }
        else {
            if (b.size() < 12) throw std::runtime_error(path + ": truncated .npy header");
            hlen = 0;
            for (int k = 0; k < 4; ++k) hlen |= static_cast<size_t>(static_cast<unsigned char>(b[8 + k])) << (8 * k);
            hstart = 12;
        }
        if (hstart + hlen > b.size()) throw std::runtime_error(path + ": truncated .npy header");
        const std::string h(b.data() + hstart, hlen);
        if (h.find("'<f4'") == std::string::npos) throw std::runtime_error(path + ": not a little-endian float32 .npy");
        if (h.find("'fortran_order': True") != std::string::npos) throw std::runtime_error(path + ": fortran-ordered .npy");
        off = hstart + hlen;
    }
    if ((b.size() - off) % 4) throw std::runtime_error(path + ": size is not a whole number of float32");
    std::vector<float> v((b.size() - off) / 4);
    std::memcpy(v.data(), b.data() + off, v.size() * 4);
    return v;
}

void put_u32(std::vector<uint8_t> & o, uint32_t v) { for (int k = 0; k < 4; ++k) o.push_back(static_cast<uint8_t>(v >> (8 * k))); }
void put_u16(std::vector<uint8_t> & o, uint16_t v) { o.push_back(static_cast<uint8_t>(v)); o.push_back(static_cast<uint8_t>(v >> 8)); }

// 16-bit PCM mono RIFF/WAVE: samples clamped to [-1, 1], scaled by 32767, rounded to nearest.
void write_wav(const std::string & path, const std::vector<float> & pcm, int rate) {
    const uint32_t data = static_cast<uint32_t>(pcm.size() * 2);
    std::vector<uint8_t> o;
    o.reserve(44 + data);
    o.insert(o.end(), {'R', 'I', 'F', 'F'});
    put_u32(o, 36 + data);
    o.insert(o.end(), {'W', 'A', 'V', 'E', 'f', 'm', 't', ' '});
    put_u32(o, 16);
    put_u16(o, 1);                                   // PCM
    put_u16(o, 1);                                   // mono
    put_u32(o, static_cast<uint32_t>(rate));
    put_u32(o, static_cast<uint32_t>(rate) * 2);     // byte rate
    put_u16(o, 2);                                   // block align
    put_u16(o, 16);                                  // bits per sample
    o.insert(o.end(), {'d', 'a', 't', 'a'});
    put_u32(o, data);
    for (float x : pcm) {
        const float c = std::fmax(-1.f, std::fmin(1.f, x));
        put_u16(o, static_cast<uint16_t>(static_cast<int16_t>(std::lrintf(c * 32767.f))));
    }
    std::ofstream f(path, std::ios::binary);
    if (!f.write(reinterpret_cast<const char *>(o.data()), static_cast<std::streamsize>(o.size()))) throw std::runtime_error("cannot write " + path);
}

int cmd_info(const Args & a) {
    int n = 0;
    check(navi_device_count(&n), "device count");
    std::printf("navi-b200 %s: %d device(s)\n", navi_version(), n);
    navi_device * dev = nullptr;
    check(navi_device_open(a.device, &dev), "device open");
    navi_device_info di{};
    check(navi_device_get_info(dev, &di), "device info");
    std::printf("device %d: %s, sm_%d%d, %d SMs, %zu KB shared memory per CTA, %zu MB L2, %.1f / %.1f GB free\n", di.ordinal, di.name,
                di.cc_major, di.cc_minor, di.multiprocessors, di.smem_per_block_optin / 1024, di.l2_bytes >> 20, di.vram_free / 1e9,
                di.vram_total / 1e9);
    if (!a.model.empty()) {
        navi_weights * w = nullptr;
        check(navi_weights_upload(dev, a.model.c_str(), &w), "weights");
        navi_params p{};
        check(navi_weights_get_params(w, &p), "params");
        std::printf("model %s: %.2f GB on the device\n", a.model.c_str(), navi_weights_bytes(w) / 1e9);
        std::printf("  talker %d layers, hidden %d, %d/%d heads x %d, ff %d, vocab %d\n", p.talker.n_layer, p.talker.hidden, p.talker.n_head,
                    p.talker.n_kv_head, p.talker.head_dim, p.talker.ff, p.talker.vocab);
        std::printf("  code predictor %d layers, hidden %d, vocab %d, %d code groups\n", p.cp.n_layer, p.cp.hidden, p.cp.vocab, p.n_code_groups);
        std::printf("  vocoder %d codebooks x %d, decoder dim %d, %d samples per frame at %d Hz\n", p.vq_n_q, p.vq_codebook_size, p.decoder_dim,
                    p.codec_upsample, p.sample_rate);
        navi_weights_free(w);
    }
    navi_device_close(dev);
    return 0;
}

struct PcmSink {
    std::vector<float> pcm;
    int batches = 0;
};
void on_pcm(const float * pcm, int n, void * user) {
    auto * s = static_cast<PcmSink *>(user);
    s->pcm.insert(s->pcm.end(), pcm, pcm + n);
    ++s->batches;
}

int cmd_synth(const Args & a) {
    if (a.model.empty() || (a.ids.empty() && a.ids_file.empty()) || a.speaker.empty() || a.out.empty())
        throw std::invalid_argument("synth needs --model, --ids or --ids-file, --speaker and --out");
    std::string id_text = a.ids;
    if (id_text.empty()) {
        const std::vector<char> b = read_file(a.ids_file);
        id_text.assign(b.data(), b.size());
    }
    const std::vector<int32_t> ids = parse_ids(id_text);
    if (ids.size() < 9) throw std::invalid_argument("--ids: the template alone is 8 ids; the text needs at least one more");
    const std::vector<float> spk = read_f32(a.speaker);
    const auto t0 = std::chrono::steady_clock::now();
    navi_device * dev = nullptr;
    check(navi_device_open(a.device, &dev), "device open");
    navi_weights * w = nullptr;
    check(navi_weights_upload(dev, a.model.c_str(), &w), "weights");
    navi_params p{};
    check(navi_weights_get_params(w, &p), "params");
    if (static_cast<int>(spk.size()) != p.talker.hidden)
        throw std::invalid_argument("--speaker has " + std::to_string(spk.size()) + " values; the talker's hidden size is " +
                                    std::to_string(p.talker.hidden));
    navi_frame_opts fo{1, 0};
    navi_graph * g = nullptr;
    check(navi_graph_create(dev, w, &fo, static_cast<int>(ids.size()) + 16, a.max_frames, a.batch, &g), "graph");
    const double load_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    // the model's generation defaults (graph.h:36, Sampling), greedy on request
    navi_sampling s{};
    s.temperature = a.greedy ? 0.f : p.temperature;
    s.top_k = p.top_k;
    s.top_p = p.top_p;
    s.repetition_penalty = p.repetition_penalty;
    s.cp_temperature = a.greedy ? 0.f : p.cp_temperature;
    s.cp_top_k = p.cp_top_k;
    s.cp_top_p = p.cp_top_p;
    s.min_frames = 2;
    s.rng = NAVI_RNG_PCG;
    PcmSink sink;
    navi_synth_stats st{};
    check(navi_graph_synth(g, ids.data(), static_cast<int>(ids.size()), a.language.c_str(), spk.data(), &s, a.seed, a.max_frames,
                           a.first_batch, a.batch, nullptr, 0, on_pcm, &sink, &st),
          "synth");
    write_wav(a.out, sink.pcm, p.sample_rate);
    std::fprintf(stderr,
                 "load %.0f ms | %d tokens, %d frames (%s) | prefill %.1f ms, frames %.1f ms (%.2f ms/frame), vocoder %.1f ms in %d "
                 "batches | ttfa %.1f ms | %.2f s audio in %.1f ms, RTF %.4f | %s\n",
                 load_ms, st.n_tokens, st.n_frames, st.eos ? "eos" : "cap", st.prefill_ms, st.frames_ms,
                 st.n_frames ? st.frames_ms / st.n_frames : 0.0, st.vocoder_ms, sink.batches, st.ttfa_ms, st.audio_s, st.total_ms, st.rtf,
                 a.out.c_str());
    navi_graph_destroy(g);
    navi_weights_free(w);
    navi_device_close(dev);
    return 0;
}

} // namespace

int main(int argc, char ** argv) {
    try {
        if (argc < 2 || std::strcmp(argv[1], "-h") == 0 || std::strcmp(argv[1], "--help") == 0) return usage(argv[0]);
        const Args a = parse(argc, argv);
        if (a.cmd == "info") return cmd_info(a);
        if (a.cmd == "synth") return cmd_synth(a);
        return usage(argv[0]);
    } catch (const std::invalid_argument & e) {
        std::fprintf(stderr, "navi-b200: %s\n", e.what());
        return usage(argv[0]);
    } catch (const std::exception & e) {
        std::fprintf(stderr, "navi-b200: %s\n", e.what());
        return 1;
    }
}
