// The standalone device sampler without any device allocation.
//
// Frame::sample allocates its result word per call (cudaMallocAsync) and stages the
// sampler's working arrays in dynamic shared memory sized by the vocabulary.  Some
// callers cannot allocate at all: a real-time audio thread, whose latency budget rules out
// calls that may block in the driver or grow a memory pool, and a serving process that
// reserves every device byte for weights and KV caches at start-up, where any later
// allocation can fail under memory pressure.  This variant allocates nothing:
// the result word and all of the sampler's working arrays (logits copy, exp values,
// candidate ids and ranks, histograms, reduction words) live in
// one file-scope device array of fixed size.
//
// Set-up: the first call on a device, with that device current, takes the array's
// device address with cudaGetSymbolAddress (which may load the module) and caches it, so
// the first call per device should come before any stream capture on that device.
//
// Zeroing: no part of the scratch has to start at zero.  The kernel writes the logits
// copy and every other working word before it reads it, clears the histograms at the start
// of each call, and writes the result word unconditionally.
//
// Sharing: all calls on one device use the same array, so two calls in flight at once
// would race on it.  This file holds a per-device host lock from launch until the result
// has been copied back, which serialises calls from different threads or different
// navi_device handles of the same GPU; work enqueued by other means that reads or writes
// the array is not covered by the lock.
#include "sample_static.hpp"
#include "frame_kernel.cuh"
#include "sampler.cuh"

#include "navi_b200.h"

#include <mutex>
#include <string>

namespace navi::fk {

using namespace navi::dev;

constexpr size_t SAMPLE_STATIC_OUT_BYTES = 256;   // result word, padded to keep the arrays 256-byte aligned
constexpr size_t SAMPLE_STATIC_BYTES =
    SAMPLE_STATIC_OUT_BYTES + static_cast<size_t>(sample_scratch_floats(navi::qwen3tts::SAMPLE_STATIC_MAX_VOCAB)) * sizeof(float);

static __device__ __align__(256) unsigned char g_sample_scratch[SAMPLE_STATIC_BYTES];

// One CTA of NCT threads; the arrays are laid out for this call's vocabulary V.
__global__ void __launch_bounds__(NCT, 1) k_sample_static(const float * logits, int V, SampleCfg cfg, unsigned char * scratch) {
    const SampleScratch sc = sampler_layout(reinterpret_cast<float *>(scratch + SAMPLE_STATIC_OUT_BYTES), V);
    for (int i = threadIdx.x; i < V; i += NCT) sc.s[i] = logits[i];
    named_sync(BID, NCT);
    const int c = sample_cta<NCT>(V, cfg, sc, BID);
    if (threadIdx.x == 0) *reinterpret_cast<int *>(scratch) = c;
}

} // namespace navi::fk

namespace navi::qwen3tts {

namespace {

constexpr int MAX_DEVICES = 64;
std::mutex g_lock[MAX_DEVICES];
unsigned char * g_addr[MAX_DEVICES] = {};

// Device address of the scratch array; the caller holds g_lock[ordinal] and has made the
// device current.
unsigned char * scratch_of(int ordinal) {
    if (!g_addr[ordinal]) {
        void * p = nullptr;
        const cudaError_t rc = cudaGetSymbolAddress(&p, navi::fk::g_sample_scratch);
        if (rc != cudaSuccess || !p)
            fail(std::string("cudaGetSymbolAddress(sampler scratch) failed: ") + cudaGetErrorString(rc), NAVI_E_CUDA);
        g_addr[ordinal] = static_cast<unsigned char *>(p);
    }
    return g_addr[ordinal];
}

} // namespace

int sample_static(const Device & dev, const float * d_logits, int vocab, const Sampling & s, uint64_t seed, int frame_index,
                  int codebook, int suppress_from, int eos_id, const uint8_t * d_seen) {
    if (vocab <= 0 || vocab > SAMPLE_STATIC_MAX_VOCAB)
        fail("vocab " + std::to_string(vocab) + " outside 1.." + std::to_string(SAMPLE_STATIC_MAX_VOCAB) +
                 ": the static sampler scratch holds at most that many logits",
             NAVI_E_ARG);
    const int ordinal = dev.info().ordinal;
    if (ordinal < 0 || ordinal >= MAX_DEVICES) fail("device ordinal out of range for the static sampler", NAVI_E_ARG);
    navi::dev::SampleCfg c{};
    if (codebook == 0) {
        c.temperature = s.temperature; c.top_k = s.top_k; c.top_p = s.top_p;
        c.talker_mods = 1; c.suppress_from = suppress_from; c.eos_id = eos_id; c.min_frames = s.min_frames;
        c.repetition_penalty = d_seen ? s.repetition_penalty : 0.f;
        c.seen = d_seen;
    } else {
        c.temperature = s.cp_temperature; c.top_k = s.cp_top_k; c.top_p = s.cp_top_p;
    }
    c.rng = s.rng; c.seed = seed; c.frame_index = frame_index; c.codebook = codebook;
    c.pcg_seed = navi::dev::pcg_draw_seed(seed, frame_index, codebook);

    std::lock_guard<std::mutex> hold(g_lock[ordinal]);
    dev.make_current();
    unsigned char * scratch = scratch_of(ordinal);
    navi::fk::k_sample_static<<<1, navi::fk::NCT, 0, dev.stream()>>>(d_logits, vocab, c, scratch);
    NAVI_CUDA(cudaGetLastError());
    int h = -1;
    NAVI_CUDA(cudaMemcpyAsync(&h, scratch, sizeof(int), cudaMemcpyDeviceToHost, dev.stream()));
    NAVI_CUDA(cudaStreamSynchronize(dev.stream()));
    return h;
}

} // namespace navi::qwen3tts
