// Checker (test infrastructure only): runs the reference engine's own talker prompt and
// prefill on the CPU.
//
// model/qwen3tts/talker.hip of the reference, its kernel launches rewritten for the host
// emulator by oracle/hip_to_host.py (oracle/_build/talker_host.cpp), compiled with kernels.h,
// params.cpp, navi_file.cpp and device_weights.cpp against the host stand-in for the HIP
// runtime (oracle/hipsim), and used as the reference's Graph uses it (graph.cpp:22-50):
// DeviceWeights::upload with Talker::fused_groups, Talker::create, build_prompt, prefill.
//
// Usage: ref_talker_check NAVI REQUEST OUT
//   REQUEST: i32 n_ids, i32 ids[n_ids], i32 len, language bytes, f32 speaker[hidden]
//   OUT:     i32 n_prefill, i32 n_trailing, f32 prefill[n_prefill][H], trailing[n_trailing][H],
//            tts_pad[H], hidden[H], logits[V], then per layer K, V rows [n_prefill][kv_dim] f16
#include "talker_host.cpp"

#include "device_standin.hpp"
#include "model/qwen3tts/params.h"
#include "runtime/weights/device_weights.h"
#include "runtime/weights/navi_file.h"

#include <cstdio>
#include <fstream>
#include <iterator>
#include <string>
#include <vector>

int main(int argc, char ** argv) {
    if (argc != 4) {
        std::fprintf(stderr, "usage: %s NAVI REQUEST OUT\n", argv[0]);
        return 2;
    }
    try {
        std::vector<char> b;
        {
            std::ifstream is(argv[2], std::ios::binary);
            b.assign(std::istreambuf_iterator<char>(is), std::istreambuf_iterator<char>());
        }
        size_t at = 0;
        auto take = [&](void * dst, size_t n) {
            if (at + n > b.size()) throw std::runtime_error("request truncated");
            std::memcpy(dst, b.data() + at, n);
            at += n;
        };
        int32_t n_ids = 0, nl = 0;
        take(&n_ids, 4);
        std::vector<int32_t> ids(static_cast<size_t>(n_ids));
        take(ids.data(), ids.size() * 4);
        take(&nl, 4);
        std::string language(static_cast<size_t>(nl), '\0');
        take(language.data(), language.size());

        navi::Device dev = navi::Device::open();
        navi::NaviFile file = navi::NaviFile::open(argv[1]);
        const auto p = navi::qwen3tts::read_params(file);
        const int H = p.talker.hidden;
        std::vector<float> speaker(static_cast<size_t>(H));
        take(speaker.data(), speaker.size() * 4);
        const std::string pre = "talker.";
        auto select = [&](const navi::TensorInfo & t) { return t.name.compare(0, pre.size(), pre) == 0 && t.dtype != navi::DType::U8; };
        navi::DeviceWeights w = navi::DeviceWeights::upload(file, select, navi::qwen3tts::Talker::fused_groups(p));
        auto tal = navi::qwen3tts::Talker::create(dev, w, p, std::max(n_ids, 16), std::max(n_ids, 16) + 16);
        const auto & pr = tal->build_prompt(ids, language, speaker);
        tal->prefill(pr);
        std::ofstream os(argv[3], std::ios::binary);
        auto put = [&](const void * src, size_t n) { os.write(static_cast<const char *>(src), static_cast<std::streamsize>(n)); };
        put(&pr.n_prefill, 4);
        put(&pr.n_trailing, 4);
        put(pr.prefill, static_cast<size_t>(pr.n_prefill) * H * 4);
        put(pr.trailing, static_cast<size_t>(pr.n_trailing) * H * 4);
        put(pr.tts_pad, static_cast<size_t>(H) * 4);
        put(tal->d_hidden(), static_cast<size_t>(H) * 4);
        put(tal->d_logits(), static_cast<size_t>(p.talker.vocab) * 4);
        auto & kv = tal->kv();
        for (int l = 0; l < kv.n_layer; ++l) {
            put(kv.k[static_cast<size_t>(l)], static_cast<size_t>(pr.n_prefill) * kv.kv_dim * 2);
            put(kv.v[static_cast<size_t>(l)], static_cast<size_t>(pr.n_prefill) * kv.kv_dim * 2);
        }
        return 0;
    } catch (const std::exception & e) {
        std::fprintf(stderr, "ref_talker_check: %s\n", e.what());
        return 3;
    }
}
