// Checker (test infrastructure only): runs the reference engine's own vocoder on the CPU.
//
// model/qwen3tts/vocoder.hip of the reference, its kernel launches rewritten by
// oracle/hip_to_host.py for the host emulator (oracle/_build/vocoder_host.cpp), is compiled
// with kernels.h, params.cpp, navi_file.cpp and device_weights.cpp against the host
// stand-in for the HIP runtime (oracle/hipsim): every grid runs block after block, each block
// as cooperative fibers. The device handle the reference's Vocoder::create takes comes from
// hipsim/device_standin.hpp.
// Used as in the reference's tests/test_vocoder.cpp: DeviceWeights::upload of the decoder
// tensors it does not own, Vocoder::create, decode.
//
// Usage: ref_vocoder_check NAVI CODES OUT [MAX_CHUNK [STAGES]]
//   CODES  int32 [n_frames][16];  OUT  f32 PCM [n_frames * samples_per_frame]
//   STAGES (optional) a directory: every stage of the first chunk as <name>.f32 + <name>.shape
#include "vocoder_host.cpp"

#include "device_standin.hpp"
#include "model/qwen3tts/params.h"
#include "runtime/device/device.h"
#include "runtime/weights/device_weights.h"
#include "runtime/weights/navi_file.h"

#include <cstdio>
#include <fstream>
#include <iterator>
#include <string>
#include <vector>

int main(int argc, char ** argv) {
    if (argc < 4) {
        std::fprintf(stderr, "usage: %s NAVI CODES OUT [MAX_CHUNK [STAGES]]\n", argv[0]);
        return 2;
    }
    try {
        std::vector<int32_t> codes;
        {
            std::ifstream is(argv[2], std::ios::binary);
            std::vector<char> b((std::istreambuf_iterator<char>(is)), std::istreambuf_iterator<char>());
            codes.resize(b.size() / 4);
            std::memcpy(codes.data(), b.data(), codes.size() * 4);
        }
        const int max_chunk = argc > 4 ? std::atoi(argv[4]) : 32;
        navi::Device dev = navi::Device::open();
        navi::NaviFile file = navi::NaviFile::open(argv[1]);
        const auto params = navi::qwen3tts::read_params(file);
        const std::string dec = "codec.decoder.";
        auto select = [&](const navi::TensorInfo & t) {
            return t.name.compare(0, dec.size(), dec) == 0 && !navi::qwen3tts::vocoder_owns_tensor(t.name);
        };
        navi::DeviceWeights w = navi::DeviceWeights::upload(file, select);
        auto voc = navi::qwen3tts::Vocoder::create(dev, file, w, params, max_chunk);
        const int n_q = params.vq_n_q, n_frames = static_cast<int>(codes.size()) / n_q;
        // the hook's state lives as long as the vocoder uses the hook
        const std::string dir = argc > 5 ? argv[5] : "";
        bool first_chunk = true;
        std::vector<std::string> seen;
        if (!dir.empty()) {
            voc->set_stage_hook([&](const std::string & name, const float * buf, int rows, int cols) {
                for (const auto & s : seen)
                    if (s == name) first_chunk = false;
                if (!first_chunk) return;
                seen.push_back(name);
                std::ofstream(dir + "/" + name + ".f32", std::ios::binary).write(reinterpret_cast<const char *>(buf),
                                                                               static_cast<std::streamsize>(rows) * cols * 4);
                std::ofstream(dir + "/" + name + ".shape") << rows << " " << cols << "\n";
            });
        }
        std::vector<float> pcm;
        voc->decode(codes, n_frames, pcm);
        std::ofstream(argv[3], std::ios::binary).write(reinterpret_cast<const char *>(pcm.data()), static_cast<std::streamsize>(pcm.size() * 4));
        return 0;
    } catch (const std::exception & e) {
        std::fprintf(stderr, "ref_vocoder_check: %s\n", e.what());
        return 3;
    }
}
