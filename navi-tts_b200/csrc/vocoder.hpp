// navi::qwen3tts::Vocoder on B200: the streaming codec decoder, codes [T][16] -> PCM
// [T * 1920] clamped to [-1, 1].  Interface of the reference's Vocoder
// (model/qwen3tts/vocoder.h:27-55).  Every convolution, transposed convolution and
// linear layer of the decoder runs as an implicit GEMM on the tcgen05 tensor cores
// (conv.hpp); the row-local pieces (RVQ gather, norms, RoPE, sliding-window attention,
// depthwise conv + LayerNorm, the 1-channel output conv) are small CUDA kernels.
#pragma once

#include "runtime.hpp"

#include <cstdint>
#include <functional>
#include <memory>
#include <span>
#include <vector>

namespace navi::qwen3tts {

class Vocoder {
public:
    // max_chunk_frames: frames decoded per pass (longer inputs are cut into chunks).
    // max_frames is accepted for interface parity; the attention ring only needs
    // sliding_window + max_chunk_frames rows.
    static std::unique_ptr<Vocoder> create(const Device & dev, const DeviceWeights & w, int max_chunk_frames = 32,
                                           int max_frames = 4096);
    ~Vocoder();

    // Zeroes every conv history and the position counter (a new utterance).
    void reset();
    // Appends n_frames * samples_per_frame() samples to pcm. codes: [n_frames][n_q] ids.
    void decode(std::span<const std::int32_t> codes, int n_frames, std::vector<float> & pcm);
    // The same into a caller buffer of at least n_frames * samples_per_frame() floats.
    void decode_into(std::span<const std::int32_t> codes, int n_frames, float * pcm);

    int samples_per_frame() const;
    int max_chunk_frames() const;
    double last_ms() const;   // device time of the last decode call

    // Called after each stage with a device buffer [rows][cols] (the stream is synchronised
    // first); stage names: rvq, pre_conv, layer<l>, pre_transformer, up<j>, dec0,
    // dec<b>, pcm (vocoder.hip:227-233).
    using StageHook = std::function<void(const char * name, const float * d_buf, int rows, int cols)>;
    void set_stage_hook(StageHook hook);

    struct Impl;

private:
    Vocoder() = default;
    std::unique_ptr<Impl> impl_;
};

} // namespace navi::qwen3tts
