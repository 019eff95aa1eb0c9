// Checker (test infrastructure only): links the reference engine's own .navi
// reader and tensor table (runtime/weights/navi_file.cpp, model/qwen3tts/params.cpp,
// compiled from the reference sources into oracle/_ref/) and reports, as JSON,
// what the reference makes of a .navi file: its hyperparameters and whether its
// expected_tensors/validate accept the tensor table.
#include "model/qwen3tts/params.h"
#include "runtime/weights/navi_file.h"

#include <cstdio>
#include <exception>

int main(int argc, char ** argv) {
    if (argc < 2) { std::fprintf(stderr, "usage: %s file.navi\n", argv[0]); return 2; }
    try {
        navi::NaviFile f = navi::NaviFile::open(argv[1]);
        const auto p = navi::qwen3tts::read_params(f);
        const auto v = navi::qwen3tts::validate(f, p);
        std::printf("{\"ok\": %s, \"missing\": %zu, \"shape_mismatch\": %zu, \"unused\": %zu, \"n_tensors\": %zu,",
                    v.ok() ? "true" : "false", v.missing.size(), v.shape_mismatch.size(), v.unused.size(), f.tensors().size());
        std::printf(" \"talker\": [%d, %d, %d, %d, %d, %d, %d], \"cp\": [%d, %d, %d, %d, %d, %d, %d],",
                    p.talker.hidden, p.talker.n_layer, p.talker.n_head, p.talker.n_kv_head, p.talker.head_dim, p.talker.ff,
                    p.talker.vocab, p.cp.hidden, p.cp.n_layer, p.cp.n_head, p.cp.n_kv_head, p.cp.head_dim, p.cp.ff, p.cp.vocab);
        std::printf(" \"codec_eos\": %d, \"decoder_dim\": %d, \"upsample\": %d, \"rms_eps\": %.9g, \"rope_theta\": %.9g,",
                    p.codec_eos_id, p.vocoder_decoder_dim, p.codec_upsample, p.talker.rms_eps, p.talker.rope_theta);
        std::printf(" \"first_missing\": \"%s\", \"first_mismatch\": \"%s\", \"data_offset\": %llu}\n",
                    v.missing.empty() ? "" : v.missing[0].c_str(),
                    v.shape_mismatch.empty() ? "" : v.shape_mismatch[0].c_str(),
                    static_cast<unsigned long long>(f.data_offset()));
        return v.ok() ? 0 : 1;
    } catch (const std::exception & e) {
        std::printf("{\"error\": \"%s\"}\n", e.what());
        return 3;
    }
}
