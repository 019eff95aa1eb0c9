// navi-b200: the command-line front of this build, over the C ABI (include/navi_b200.h).
// Mirrors the reference's `info`, `synth` and `bench` subcommands (runtime/cli/main.cpp:59-72,
// 219-279; runtime/bench/bench.cpp:98-155) without the text tokenizer and the speaker encoder:
// `synth` and `bench` take the prompt's token ids and a speaker embedding.
//
//   navi-b200 info  [--model FILE] [--device N]
//   navi-b200 bench --model FILE [--ids "i,j,..." | --ids-file FILE] [--speaker EMB] [--seed N]
//                   [--repeats N] [--warmup N] [--batch N] [--max-frames N] [--out results.jsonl]
//   navi-b200 synth --model FILE (--ids "i,j,..." | --ids-file FILE) --speaker EMB --out OUT.wav
//                   [--seed N] [--language L] [--max-frames N] [--greedy] [--first-batch N]
//                   [--batch N] [--device N]
//
// --ids are the tokenised "<|im_start|>assistant\n{text}<|im_end|>\n<|im_start|>assistant\n"
// (3 header ids, the text, 5 trailer ids), as navi_talker_build_prompt takes them. --speaker
// is a speaker embedding of the talker's hidden size: a 1-D float32 .npy, or raw
// little-endian float32. The WAV is 16-bit PCM mono at the codec's sample rate.
#include "../../include/navi_b200.h"

#include <algorithm>
#include <chrono>
#include <ctime>
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
    int max_frames = 600, first_batch = 4, batch = 16, device = 0, repeats = 1, warmup = 1;
    bool greedy = false, seed_set = false, batch_set = false;
};

int usage(const char * argv0) {
    std::fprintf(stderr,
                 "%s\n"
                 "usage: %s info  [--model FILE] [--device N]\n"
                 "       %s synth --model FILE (--ids \"i,j,...\" | --ids-file FILE) --speaker EMB(.npy|.f32) --out OUT.wav\n"
                 "                [--seed N] [--language L] [--max-frames N] [--greedy] [--first-batch N] [--batch N] [--device N]\n"
                 "       %s bench --model FILE [--ids \"i,j,...\" | --ids-file FILE] [--speaker EMB] [--seed N] [--repeats N]\n"
                 "                [--warmup N] [--batch N] [--max-frames N] [--device N] [--out results.jsonl]\n"
                 "  --ids: the tokenised prompt template (3 header ids, the text, 5 trailer ids)\n",
                 navi_version(), argv0, argv0, argv0);
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
        else if (s == "--seed") { a.seed = std::stoull(next("--seed")); a.seed_set = true; }
        else if (s == "--repeats") a.repeats = std::stoi(next("--repeats"));
        else if (s == "--warmup") a.warmup = std::stoi(next("--warmup"));
        else if (s == "--max-frames") a.max_frames = std::stoi(next("--max-frames"));
        else if (s == "--first-batch") a.first_batch = std::stoi(next("--first-batch"));
        else if (s == "--batch") { a.batch = std::stoi(next("--batch")); a.batch_set = true; }
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
std::vector<uint8_t> wav_bytes(const std::vector<float> & pcm, int rate) {
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
    return o;
}

void write_wav(const std::string & path, const std::vector<float> & pcm, int rate) {
    const std::vector<uint8_t> o = wav_bytes(pcm, rate);
    std::ofstream f(path, std::ios::binary);
    if (!f.write(reinterpret_cast<const char *>(o.data()), static_cast<std::streamsize>(o.size()))) throw std::runtime_error("cannot write " + path);
}

// SHA-256 (FIPS 180-4) of a byte string, as lowercase hex: the WAV digest the reference's bench
// line records (bench.cpp:150-151).
std::string sha256_hex(const std::vector<uint8_t> & msg) {
    static const uint32_t K[64] = {
        0x428a2f98, 0x71374491, 0xb5c0fbcf, 0xe9b5dba5, 0x3956c25b, 0x59f111f1, 0x923f82a4, 0xab1c5ed5, 0xd807aa98, 0x12835b01, 0x243185be,
        0x550c7dc3, 0x72be5d74, 0x80deb1fe, 0x9bdc06a7, 0xc19bf174, 0xe49b69c1, 0xefbe4786, 0x0fc19dc6, 0x240ca1cc, 0x2de92c6f, 0x4a7484aa,
        0x5cb0a9dc, 0x76f988da, 0x983e5152, 0xa831c66d, 0xb00327c8, 0xbf597fc7, 0xc6e00bf3, 0xd5a79147, 0x06ca6351, 0x14292967, 0x27b70a85,
        0x2e1b2138, 0x4d2c6dfc, 0x53380d13, 0x650a7354, 0x766a0abb, 0x81c2c92e, 0x92722c85, 0xa2bfe8a1, 0xa81a664b, 0xc24b8b70, 0xc76c51a3,
        0xd192e819, 0xd6990624, 0xf40e3585, 0x106aa070, 0x19a4c116, 0x1e376c08, 0x2748774c, 0x34b0bcb5, 0x391c0cb3, 0x4ed8aa4a, 0x5b9cca4f,
        0x682e6ff3, 0x748f82ee, 0x78a5636f, 0x84c87814, 0x8cc70208, 0x90befffa, 0xa4506ceb, 0xbef9a3f7, 0xc67178f2};
    uint32_t h[8] = {0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a, 0x510e527f, 0x9b05688c, 0x1f83d9ab, 0x5be0cd19};
    std::vector<uint8_t> m(msg);
    const uint64_t bits = static_cast<uint64_t>(msg.size()) * 8;
    m.push_back(0x80);
    while (m.size() % 64 != 56) m.push_back(0);
    for (int k = 7; k >= 0; --k) m.push_back(static_cast<uint8_t>(bits >> (8 * k)));
    auto rotr = [](uint32_t x, int n) { return (x >> n) | (x << (32 - n)); };
    for (size_t blk = 0; blk < m.size(); blk += 64) {
        uint32_t w[64];
        for (int t = 0; t < 16; ++t)
            w[t] = (uint32_t(m[blk + 4 * t]) << 24) | (uint32_t(m[blk + 4 * t + 1]) << 16) | (uint32_t(m[blk + 4 * t + 2]) << 8) |
                   uint32_t(m[blk + 4 * t + 3]);
        for (int t = 16; t < 64; ++t) {
            const uint32_t s0 = rotr(w[t - 15], 7) ^ rotr(w[t - 15], 18) ^ (w[t - 15] >> 3);
            const uint32_t s1 = rotr(w[t - 2], 17) ^ rotr(w[t - 2], 19) ^ (w[t - 2] >> 10);
            w[t] = w[t - 16] + s0 + w[t - 7] + s1;
        }
        uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
        for (int t = 0; t < 64; ++t) {
            const uint32_t t1 = hh + (rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25)) + ((e & f) ^ (~e & g)) + K[t] + w[t];
            const uint32_t t2 = (rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22)) + ((a & b) ^ (a & c) ^ (b & c));
            hh = g; g = f; f = e; e = d + t1; d = c; c = b; b = a; a = t1 + t2;
        }
        h[0] += a; h[1] += b; h[2] += c; h[3] += d; h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
    }
    char out[65];
    for (int k = 0; k < 8; ++k) std::snprintf(out + 8 * k, 9, "%08x", h[k]);
    return std::string(out, 64);
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

// The reference's bench harness (runtime/bench/bench.h:27-43, bench.cpp:98-155): load, then the
// utterance through the serving path (Graph::synth) after `warmup` untimed ones, one JSON line per
// repeat with the same fields. This build has no tokenizer or speaker encoder: the prompt is --ids
// (default: a fixed 20-token text in the Qwen template, for models with the full text vocabulary)
// and the speaker --speaker (default: the zero embedding). talker_ms / cp_ms stay null, as in the
// reference: the frame is one launch.
int cmd_bench(const Args & a) {
    if (a.model.empty()) throw std::invalid_argument("bench needs --model");
    using clock = std::chrono::steady_clock;
    auto ms_since = [](clock::time_point t) { return std::chrono::duration<double, std::milli>(clock::now() - t).count(); };
    const auto t0 = clock::now();
    navi_params p{};
    int n_tensors = 0, n_missing = 0, n_bad = 0, n_unused = 0;
    check(navi_model_probe(a.model.c_str(), &p, &n_tensors, &n_missing, &n_bad, &n_unused), "model");
    const double map_ms = ms_since(t0);
    std::vector<int32_t> ids;
    if (!a.ids.empty() || !a.ids_file.empty()) {
        std::string id_text = a.ids;
        if (id_text.empty()) {
            const std::vector<char> b = read_file(a.ids_file);
            id_text.assign(b.data(), b.size());
        }
        ids = parse_ids(id_text);
    } else {
        if (p.text_vocab < 151936) throw std::invalid_argument("bench: this model's text vocabulary needs --ids");
        ids = {151644, 77091, 198};   // <|im_start|> assistant \n
        for (int i = 1; i <= 20; ++i) ids.push_back(static_cast<int32_t>((static_cast<uint64_t>(i) * 2654435761ull) % 150000ull));
        for (int32_t t : {151645, 198, 151644, 77091, 198}) ids.push_back(t);
    }
    if (ids.size() < 9) throw std::invalid_argument("--ids: the template alone is 8 ids; the text needs at least one more");
    std::vector<float> spk = a.speaker.empty() ? std::vector<float>(static_cast<size_t>(p.talker.hidden), 0.f) : read_f32(a.speaker);
    if (static_cast<int>(spk.size()) != p.talker.hidden) throw std::invalid_argument("--speaker size is not the talker's hidden size");
    navi_device * dev = nullptr;
    check(navi_device_open(a.device, &dev), "device open");
    navi_device_info di{};
    check(navi_device_get_info(dev, &di), "device info");
    const auto tu = clock::now();
    navi_weights * w = nullptr;
    check(navi_weights_upload(dev, a.model.c_str(), &w), "weights");
    const double upload_ms = ms_since(tu);
    const uint64_t wbytes = navi_weights_bytes(w);
    // streaming batches 4 then 16 (graph.h:29-30), or --batch throughout
    const int first = a.batch_set ? a.batch : 4, batch = a.batch_set ? a.batch : 16;
    navi_frame_opts fo{1, 0};
    navi_graph * g = nullptr;
    check(navi_graph_create(dev, w, &fo, static_cast<int>(ids.size()) + 16, a.max_frames, batch, &g), "graph");
    navi_sampling s{};
    s.temperature = p.temperature; s.top_k = p.top_k; s.top_p = p.top_p; s.repetition_penalty = p.repetition_penalty;
    s.cp_temperature = p.cp_temperature; s.cp_top_k = p.cp_top_k; s.cp_top_p = p.cp_top_p; s.min_frames = 2; s.rng = NAVI_RNG_PCG;
    const uint64_t seed = a.seed_set ? a.seed : 2;   // the reference's bench seed (bench.h:21)
    char name[512] = {0};
    for (int r = 0; r < std::max(1, a.repeats); ++r) {
        PcmSink sink;
        navi_synth_stats st{};
        for (int i = 0; i < a.warmup + 1; ++i) {
            sink = PcmSink{};
            check(navi_graph_synth(g, ids.data(), static_cast<int>(ids.size()), a.language.c_str(), spk.data(), &s, seed, a.max_frames, first,
                                   batch, nullptr, 0, on_pcm, &sink, &st),
                  "synth");
        }
        const std::vector<uint8_t> wav = wav_bytes(sink.pcm, p.sample_rate);
        if (!a.out.empty() && a.out.size() > 4 && a.out.compare(a.out.size() - 4, 4, ".wav") == 0) write_wav(a.out, sink.pcm, p.sample_rate);
        const std::time_t now = std::time(nullptr);
        char ts[32];
        std::strftime(ts, sizeof ts, "%Y-%m-%dT%H:%M:%SZ", std::gmtime(&now));
        std::snprintf(name, sizeof name, "%s", a.model.c_str());
        std::ostringstream j;
        j.setf(std::ios::fixed);
        j.precision(4);
        const double nf = st.n_frames;
        j << "{\"ts\": \"" << ts << "\", \"git\": \"" << navi_version() << "\", \"gfx\": \"sm_" << di.cc_major << di.cc_minor
          << "a\", \"device\": \"" << di.name << "\", \"multiprocessors\": " << di.multiprocessors << ", \"model\": \"" << name
          << "\", \"weight_bytes\": " << wbytes << ", \"load_map_ms\": " << map_ms << ", \"load_upload_ms\": " << upload_ms
          << ", \"upload_gbps\": " << (upload_ms > 0 ? wbytes / 1e6 / upload_ms : 0.0) << ", \"prefill_ms\": " << st.prefill_ms
          << ", \"frame_ms\": " << (nf ? st.frames_ms / nf : 0.0) << ", \"talker_ms\": null, \"cp_ms\": null, \"vocoder_ms_per_frame\": "
          << (nf ? st.vocoder_ms / nf : 0.0) << ", \"ttfa_ms\": " << st.ttfa_ms << ", \"rtf\": " << st.rtf << ", \"n_frames\": " << st.n_frames
          << ", \"wav_sha256\": \"" << sha256_hex(wav) << "\", \"text\": \"" << ids.size() - 8 << " text token ids\", \"seed\": " << seed
          << "}";
        const std::string line = j.str();
        if (a.out.empty() || (a.out.size() > 4 && a.out.compare(a.out.size() - 4, 4, ".wav") == 0)) {
            std::printf("%s\n", line.c_str());
        } else {
            std::ofstream f(a.out, std::ios::app);
            if (!f) throw std::runtime_error("cannot open " + a.out + " for append");
            f << line << '\n';
            std::fprintf(stderr, "appended to %s: %d frames, prefill %.1f ms, %.2f ms/frame, ttfa %.1f ms, RTF %.4f\n", a.out.c_str(),
                         st.n_frames, st.prefill_ms, nf ? st.frames_ms / nf : 0.0, st.ttfa_ms, st.rtf);
        }
    }
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
        if (a.cmd == "bench") return cmd_bench(a);
        return usage(argv[0]);
    } catch (const std::invalid_argument & e) {
        std::fprintf(stderr, "navi-b200: %s\n", e.what());
        return usage(argv[0]);
    } catch (const std::exception & e) {
        std::fprintf(stderr, "navi-b200: %s\n", e.what());
        return 1;
    }
}
