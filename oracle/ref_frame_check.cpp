// Checker (test infrastructure only): runs the reference engine's own frame code on the CPU.
//
// model/qwen3tts/frame.hip (with its headers, model/qwen3tts/params.cpp,
// runtime/weights/navi_file.cpp and device_weights.cpp) is compiled from the reference
// sources against this repository's host stand-in for the HIP runtime (oracle/hipsim):
// device functions become host functions, one thread block of the kernel runs as 256
// cooperative fibers (simt.hpp), and the reference's own Frame::Impl::launch computes the
// per-frame seeds and starts k_frame on a one-block grid (the grid barrier then never
// waits). Device memory is host memory. Math functions are the host C library's, so float
// results are the reference's algorithm with glibc's expf / powf / sincosf in place of the
// GPU's; integer work (seeds, radix select, draw walk) is the reference's exactly.
//
// Usage: ref_frame_check IN OUT, binary request / response (oracle/ref_frame.py):
//   mode 0  frame: Frame::run at n_past on a given step embedding and KV cache
//   mode 1  frame 0: Frame::run_first on given hidden and logits
//   mode 2  seeds: B.talker_seed / B.cp_seed of launch(seed, frame_index) for a list
//   mode 3  sampler: tl_sample (codebook 0) or cp_sample (codebook >= 1) on given logits
#include "model/qwen3tts/frame.hip"
#include "model/qwen3tts/params.h"
#include "runtime/weights/navi_file.h"

#include <cstdio>
#include <fstream>
#include <iterator>
#include <stdexcept>
#include <string>
#include <vector>

namespace {

using navi::qwen3tts::Frame;

struct In {
    std::vector<char> b;
    size_t at = 0;
    template <class T> T get() {
        if (at + sizeof(T) > b.size()) throw std::runtime_error("request truncated");
        T v;
        std::memcpy(&v, b.data() + at, sizeof(T));
        at += sizeof(T);
        return v;
    }
    template <class T> std::vector<T> arr(size_t n) {
        std::vector<T> v(n);
        if (at + n * sizeof(T) > b.size()) throw std::runtime_error("request truncated");
        std::memcpy(v.data(), b.data() + at, n * sizeof(T));
        at += n * sizeof(T);
        return v;
    }
};

struct Out {
    std::vector<char> b;
    template <class T> void put(T v) { b.insert(b.end(), reinterpret_cast<char *>(&v), reinterpret_cast<char *>(&v) + sizeof(T)); }
    template <class T> void arr(const T * p, size_t n) {
        b.insert(b.end(), reinterpret_cast<const char *>(p), reinterpret_cast<const char *>(p) + n * sizeof(T));
    }
};

template <class T> T * host_alloc(size_t n) { return static_cast<T *>(std::calloc(n ? n : 1, sizeof(T))); }

// The frame of Frame::create (frame.hip:684-774) on the mapped file: weights are pointers
// into the mapping, the work buffers host memory, a one-block grid.
struct Setup {
    navi::NaviFile f;
    navi::qwen3tts::Params p;
    Frame::Impl I;
    explicit Setup(const std::string & path) : f(navi::NaviFile::open(path)), p(navi::qwen3tts::read_params(f)) {
        using namespace navi::qwen3tts;
        const auto & tp = p.talker;
        const auto & cp = p.cp;
        I.p = p;
        I.TP = {tp.hidden, tp.n_head, tp.n_kv_head, tp.head_dim, tp.ff, tp.vocab, tp.n_layer, tp.rms_eps, static_cast<float>(tp.rope_theta)};
        I.CP = {cp.hidden, cp.n_head, cp.n_kv_head, cp.head_dim, cp.ff, cp.vocab, cp.n_layer, cp.rms_eps, static_cast<float>(cp.rope_theta)};
        auto h16 = [&](const std::string & n) { return static_cast<const uint16_t *>(f.data(f.get(n))); };
        auto h32 = [&](const std::string & n) { return static_cast<const float *>(f.data(f.get(n))); };
        auto layer = [&](auto & W, const std::string & prefix, int l) {
            const std::string lp = prefix + ".layers." + std::to_string(l) + ".";
            W.attn_norm[l] = h32(lp + "input_layernorm.weight");
            W.ffn_norm[l] = h32(lp + "post_attention_layernorm.weight");
            W.q_norm[l] = h32(lp + "self_attn.q_norm.weight");
            W.k_norm[l] = h32(lp + "self_attn.k_norm.weight");
            W.wq[l] = h16(lp + "self_attn.q_proj.weight");
            W.wk[l] = h16(lp + "self_attn.k_proj.weight");
            W.wv[l] = h16(lp + "self_attn.v_proj.weight");
            W.wo[l] = h16(lp + "self_attn.o_proj.weight");
            W.w_gate[l] = h16(lp + "mlp.gate_proj.weight");
            W.w_up[l] = h16(lp + "mlp.up_proj.weight");
            W.w_down[l] = h16(lp + "mlp.down_proj.weight");
        };
        for (int l = 0; l < tp.n_layer; ++l) layer(I.TW, "talker.model", l);
        for (int l = 0; l < cp.n_layer; ++l) layer(I.CW, "talker.code_predictor.model", l);
        I.TW.output_norm = h32("talker.model.norm.weight");
        I.TW.codec_head = h16("talker.codec_head.weight");
        I.CW.output_norm = h32("talker.code_predictor.model.norm.weight");
        I.CW.talker_codec_embd = h16("talker.model.codec_embedding.weight");
        for (int i = 0; i < 15; ++i) {
            I.CW.codec_embd[i] = h16("talker.code_predictor.model.codec_embedding." + std::to_string(i) + ".weight");
            I.CW.lm_head[i] = h16("talker.code_predictor.lm_head." + std::to_string(i) + ".weight");
        }
        auto & B = I.B;
        const int Q = tp.n_head * tp.head_dim, KV = tp.n_kv_head * tp.head_dim;
        const int CQ = cp.n_head * cp.head_dim, CKV = cp.n_kv_head * cp.head_dim;
        B.x = host_alloc<float>(tp.hidden); B.q = host_alloc<float>(Q); B.k = host_alloc<float>(KV); B.v = host_alloc<float>(KV);
        B.attn = host_alloc<float>(Q); B.h = host_alloc<float>(tp.ff); B.hidden_out = host_alloc<float>(tp.hidden);
        B.logits = host_alloc<float>(tp.vocab); B.seen = host_alloc<uint8_t>(tp.vocab);
        B.cx = host_alloc<float>(cp.hidden); B.cq = host_alloc<float>(CQ); B.ck = host_alloc<float>(CKV); B.cv = host_alloc<float>(CKV);
        B.cattn = host_alloc<float>(CQ); B.ch = host_alloc<float>(cp.ff); B.clogits = host_alloc<float>(15ull * cp.vocab);
        B.ckcache = host_alloc<uint16_t>(static_cast<size_t>(cp.n_layer) * 16 * CKV);
        B.cvcache = host_alloc<uint16_t>(static_cast<size_t>(cp.n_layer) * 16 * CKV);
        B.codes = host_alloc<int32_t>(16);
        B.step_out = host_alloc<float>(tp.hidden);
        B.bar = host_alloc<unsigned>(3);
        B.eos_id = p.codec_eos_id;
        B.suppress_from = tp.vocab - 1024;
        B.spin_cap = 1ull << 40;
        I.grid = 1;
    }
};

int run_k_frame(const void *, dim3 grid, dim3 block, void ** args) {
    using namespace navi::qwen3tts;
    if (grid.x != 1) return 1;
    auto & TP = *static_cast<TlParams *>(args[0]);
    auto & TW = *static_cast<TlWeights *>(args[1]);
    auto & CP = *static_cast<CpParams *>(args[2]);
    auto & CW = *static_cast<CpWeights *>(args[3]);
    auto & B = *static_cast<Work *>(args[4]);
    simt::run_block(block.x, simt::Dim{0, 0, 0}, simt::Dim{1, 1, 1}, [&]() { k_frame(TP, TW, CP, CW, B); });
    return 0;
}

navi::qwen3tts::Sampling read_sampling(In & in) {
    navi::qwen3tts::Sampling s;
    s.temperature = in.get<float>();
    s.top_k = in.get<int32_t>();
    s.repetition_penalty = in.get<float>();
    s.cp_temperature = in.get<float>();
    s.cp_top_k = in.get<int32_t>();
    s.min_frames = in.get<int32_t>();
    return s;
}

} // namespace

int main(int argc, char ** argv) {
    if (argc != 3) {
        std::fprintf(stderr, "usage: %s REQUEST RESPONSE\n", argv[0]);
        return 2;
    }
    try {
        In in;
        {
            std::ifstream is(argv[1], std::ios::binary);
            in.b.assign(std::istreambuf_iterator<char>(is), std::istreambuf_iterator<char>());
        }
        const auto mode = in.get<int32_t>();
        const auto plen = in.get<int32_t>();
        const auto pchars = in.arr<char>(static_cast<size_t>(plen));
        Setup S(std::string(pchars.begin(), pchars.end()));
        auto & I = S.I;
        auto & B = I.B;
        const auto & tp = S.p.talker;
        const auto & cp = S.p.cp;
        Out out;
        if (mode == 0 || mode == 1) {
            simsim::set_launch_runner(run_k_frame);
            const auto s = read_sampling(in);
            const auto seed = in.get<uint64_t>();
            const auto frame_index = in.get<int32_t>();
            const auto seen = in.arr<uint8_t>(static_cast<size_t>(tp.vocab));
            std::memcpy(B.seen, seen.data(), seen.size());
            const auto trailing = in.arr<float>(static_cast<size_t>(tp.hidden));
            std::vector<float> step, hid, lg;
            std::vector<std::vector<uint16_t>> kc, vc;
            int n_past = 0;
            const int KV = tp.n_kv_head * tp.head_dim;
            B.trailing = trailing.data();
            if (mode == 0) {
                n_past = in.get<int32_t>();
                step = in.arr<float>(static_cast<size_t>(tp.hidden));
                for (int l = 0; l < tp.n_layer; ++l) {
                    kc.push_back(in.arr<uint16_t>(static_cast<size_t>(n_past + 1) * KV));
                    vc.push_back(in.arr<uint16_t>(static_cast<size_t>(n_past + 1) * KV));
                    B.kcache[l] = kc.back().data();
                    B.vcache[l] = vc.back().data();
                }
                // Frame::run (frame.hip:798-810) with the step embedding given
                B.skip_talker = 0;
                B.n_past = n_past;
                B.step_in = step.data();
            } else {
                hid = in.arr<float>(static_cast<size_t>(tp.hidden));
                lg = in.arr<float>(static_cast<size_t>(tp.vocab));
                // Frame::run_first (frame.hip:787-796)
                B.skip_talker = 1;
                B.hidden_in = hid.data();
                B.logits_in = lg.data();
                B.step_in = nullptr;
            }
            const auto r = I.launch(s, seed, frame_index);
            out.put<int32_t>(r.ok ? 1 : 0);
            out.arr(B.codes, 16);
            out.put<uint64_t>(B.talker_seed);
            out.put<uint64_t>(B.cp_seed);
            out.arr(B.hidden_out, static_cast<size_t>(tp.hidden));
            out.arr(B.logits, static_cast<size_t>(tp.vocab));
            out.arr(B.clogits, 15ull * cp.vocab);
            out.arr(B.step_out, static_cast<size_t>(tp.hidden));
            out.arr(B.seen, static_cast<size_t>(tp.vocab));
            if (mode == 0)
                for (int l = 0; l < tp.n_layer; ++l) {
                    out.arr(kc[l].data() + static_cast<size_t>(n_past) * KV, static_cast<size_t>(KV));
                    out.arr(vc[l].data() + static_cast<size_t>(n_past) * KV, static_cast<size_t>(KV));
                }
        } else if (mode == 2) {
            simsim::set_launch_runner([](const void *, dim3, dim3, void **) { return 0; });   // seeds only: the kernel does not run
            const auto n = in.get<int32_t>();
            for (int i = 0; i < n; ++i) {
                const auto seed = in.get<uint64_t>();
                const auto fi = in.get<int32_t>();
                (void) I.launch(navi::qwen3tts::Sampling{}, seed, fi);
                out.put<uint64_t>(B.talker_seed);
                out.put<uint64_t>(B.cp_seed);
            }
        } else if (mode == 3) {
            using namespace navi::qwen3tts;
            simsim::set_launch_runner([](const void *, dim3, dim3, void **) { return 0; });
            const auto n = in.get<int32_t>();
            static float xs[VEC_MAX];
            static float red[32];
            static SampleScratch samp;
            for (int i = 0; i < n; ++i) {
                const auto s = read_sampling(in);
                const auto seed = in.get<uint64_t>();
                const auto fi = in.get<int32_t>();
                const auto codebook = in.get<int32_t>();
                const int V = codebook == 0 ? tp.vocab : cp.vocab;
                const auto logits = in.arr<float>(static_cast<size_t>(V));
                const auto seen = in.arr<uint8_t>(static_cast<size_t>(tp.vocab));
                (void) I.launch(s, seed, fi);   // sets the sampling fields and the seeds of B
                std::memcpy(B.seen, seen.data(), seen.size());
                std::memset(B.codes, 0xff, 16 * sizeof(int32_t));
                if (codebook == 0) {
                    std::memcpy(B.logits, logits.data(), logits.size() * sizeof(float));
                    simt::run_block(256, simt::Dim{0, 0, 0}, simt::Dim{1, 1, 1}, [&]() { tl_sample(I.TP, B, xs, red, samp); });
                } else {
                    std::memcpy(B.clogits + static_cast<size_t>(codebook - 1) * V, logits.data(), logits.size() * sizeof(float));
                    simt::run_block(256, simt::Dim{0, 0, 0}, simt::Dim{1, 1, 1}, [&]() { cp_sample(I.CP, B, codebook, xs, red, samp); });
                }
                out.put<int32_t>(B.codes[codebook]);
            }
        } else {
            throw std::runtime_error("unknown mode");
        }
        std::ofstream os(argv[2], std::ios::binary);
        os.write(out.b.data(), static_cast<std::streamsize>(out.b.size()));
        return 0;
    } catch (const std::exception & e) {
        std::fprintf(stderr, "ref_frame_check: %s\n", e.what());
        return 3;
    }
}
