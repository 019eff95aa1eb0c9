// Host side of the persistent frame kernel: weight tables, the phase programs, the
// exchange and cache buffers, and one cooperative launch per frame
// (reference: Frame::create / launch / run_first / run, model/qwen3tts/frame.hip:653-810).
#include "frame.hpp"
#include "frame_kernel.cuh"

#include "../../include/navi_b200.h"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <vector>

namespace navi::fk {
__global__ void k_frame(const __grid_constant__ Args A);
__global__ void k_frame_batch(const __grid_constant__ Args A);

// Re-lays out an R x K row-major f16 matrix into per-CTA slices (layout in frame_kernel.cuh):
// each thread moves one 8-column chunk (16 bytes).
__global__ void k_slice_layout(const __half * __restrict__ W, __half * __restrict__ out, int R, int K, int G) {
    const int nk = K / 8;
    const size_t units = static_cast<size_t>(R) * nk;
    for (size_t u = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; u < units; u += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const int r = static_cast<int>(u / nk), kc = static_cast<int>(u % nk);
        const int b = static_cast<int>((static_cast<long long>(r + 1) * G + R - 1) / R) - 1;   // the CTA whose rows hold r
        int r0, r1;
        split_rows(R, b, G, r0, r1);
        const size_t dst = static_cast<size_t>(r0) * K + (static_cast<size_t>(kc) * (r1 - r0) + (r - r0)) * 8;
        *reinterpret_cast<uint4 *>(out + dst) = *reinterpret_cast<const uint4 *>(W + static_cast<size_t>(r) * K + kc * 8);
    }
}
__global__ void k_sample(const float * logits, int V, navi::dev::SampleCfg cfg, int * out);
} // namespace navi::fk

namespace navi::qwen3tts {

using namespace navi::fk;

namespace {

int cdiv(int a, int b) { return (a + b - 1) / b; }

// cos[hd/2] then sin[hd/2] of RoPE at integer position pos: the angle is the f32 product
// pos * inv_freq (as the reference forms it), cos and sin are taken in double and rounded.
void rope_row(const std::vector<float> & inv_freq, int pos, float * out) {
    const size_t h2 = inv_freq.size();
    for (size_t i = 0; i < h2; ++i) {
        const float ang = static_cast<float>(pos) * inv_freq[i];
        out[i] = static_cast<float>(std::cos(static_cast<double>(ang)));
        out[h2 + i] = static_cast<float>(std::sin(static_cast<double>(ang)));
    }
}

} // namespace

struct Frame::Impl {
    int ordinal = 0;
    cudaStream_t stream = nullptr;
    Dims d{};
    ModelW * dmw = nullptr;
    __half * wslices = nullptr;   // the frame's copy of its weight matrices in per-CTA slice layout
    Phase * prog_full = nullptr;
    Phase * prog_first = nullptr;
    Phase * prog_layers = nullptr;   // [TL][LAYER_PHASES]: one talker layer alone, then XOUT
    Phase * prog_batch[MAX_B + 1] = {};   // batched programs of 2 and 4 streams
    Phase * prog_batch_first[MAX_B + 1] = {};   // their frame-0 form (the code predictor only)
    int n_batch_first[MAX_B + 1] = {};
    int sample_phase_first[MAX_B + 1][NCB] = {};
    int n_batch[MAX_B + 1] = {};
    int thead_phase[MAX_B + 1] = {};
    int sample_phase[MAX_B + 1][NCB] = {};
    int n_full = 0, n_first = 0;
    Work w{};
    float * inv_t = nullptr, * inv_c = nullptr;
    std::vector<float> inv_t_h, inv_c_h;   // host copies (RoPE tables)
    // talker RoPE rows [cos | sin] of the positions seen so far, computed once each: a frame's
    // launch copies its row instead of evaluating 128 double-precision cos / sin
    std::vector<float> rope_rows;
    const float * rope_at(int pos) {
        const size_t hd = 2 * inv_t_h.size();
        while (rope_rows.size() < (static_cast<size_t>(pos) + 1) * hd) {
            const size_t at = rope_rows.size();
            rope_rows.resize(at + hd);
            rope_row(inv_t_h, static_cast<int>(at / hd), rope_rows.data() + at);
        }
        return rope_rows.data() + static_cast<size_t>(pos) * hd;
    }
    float * rope_c = nullptr;               // [NCB][HD] code-predictor cos | sin at positions 0..15
    float * step[MAX_B][2] = {};   // per slot: the step embedding a frame reads and the one it writes
    int cur[MAX_B] = {};
    uint8_t * seen = nullptr;       // [MAX_B][TV] per slot
    int last_nb = 1;
    uint32_t tag = 0;
    uint32_t last_tag = 0;
    bool pending = false;
    int grid = 0;
    uint32_t scratch_floats = 0;
    int cp_keep_layers = 0;   // code-predictor layers held in L2 by cache policy
    uint64_t timeout_ns = 0;
    uint32_t poll_ns = 0;
    int eos = 0, suppress_from = 0;
    size_t ll_bytes = 0;
    // tensor maps of each slot's talker KV cache ([MAX_B][MAX_TL][K, V] in device memory), and
    // the host copies with the cache pointers and length they were encoded for
    uint8_t * kvmaps = nullptr;
    std::vector<uint8_t> kvmap_host[MAX_B];
    const void * kvmap_src[MAX_B][MAX_TL][2] = {};
    int kvmap_pos[MAX_B] = {};
    uint64_t * ll_base = nullptr;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    int32_t * h_out = nullptr;   // pinned: 4 control words + MAX_B x 16 codes (the device block's layout)
    unsigned long long * prof = nullptr;
    bool prof_on = false;
    int prof_cta = 0;
    int last_nphase = 0;
    std::vector<void *> owned;

    template <class T> T * alloc(size_t n) {
        void * p = nullptr;
        NAVI_CUDA(cudaMalloc(&p, n * sizeof(T)));
        NAVI_CUDA(cudaMemset(p, 0, n * sizeof(T)));
        owned.push_back(p);
        return static_cast<T *>(p);
    }

    // Talker attention of a stream: its KV head's cached positions in `split` ranges of
    // `chunk` positions (at least 8 per split, at most `per` splits), one range per CTA.
    static void attn_plan(int n_past, int per, int & split, int & chunk) {
        split = std::min(per, std::max(1, cdiv(n_past, 8)));
        chunk = std::max(1, cdiv(n_past, split));
        split = std::max(1, cdiv(n_past, chunk));
    }

    // One stream of a launch.
    struct StreamIn {
        int slot = 0;
        const float * step_in = nullptr;   // null: the slot's own step embedding
        const float * trailing = nullptr;
        KvCache * kv = nullptr;
        int n_past = 0;
        uint64_t seed = 0;
        int frame_index = 0;
        const float * hidden = nullptr;    // batched frame 0: the prefill's post-norm hidden
        const float * logits = nullptr;    // and its codec logits
    };

    static constexpr int LAYER_PHASES = 6;

    // Per-mode launch shape: streams nb -> shared-memory layout and ring.
    struct Mode {
        int xcols = 2, cp_slots = 1;
        uint32_t part_floats = 0, ysum_off = 0, ring = 0, smem = 0;
    };
    Mode modes[MAX_B + 1];

    // The tensor maps of slot sl's KV cache (boxes of KV_BOX positions x one KV head), encoded
    // again only when the cache's pointers or length change (once per request); null when the
    // cache's layout does not suit them (the kernel then copies the rows one by one).
    const uint8_t * kv_maps(int sl, const KvCache & kv) {
        bool same = kvmap_pos[sl] == kv.max_pos;
        for (int l = 0; l < d.TL && same; ++l) same = kvmap_src[sl][l][0] == kv.k[l] && kvmap_src[sl][l][1] == kv.v[l];
        uint8_t * dst = kvmaps + static_cast<size_t>(sl) * MAX_TL * 2 * TMAP_BYTES;
        if (same) return kvmap_pos[sl] > 0 ? dst : nullptr;
        static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
        if (!encode) {
            cudaDriverEntryPointQueryResult q{};
            void * fn = nullptr;
            NAVI_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
            if (q != cudaDriverEntryPointSuccess || !fn) fail("frame: cuTensorMapEncodeTiled unavailable", NAVI_E_CUDA);
            encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
        }
        std::vector<uint8_t> & h = kvmap_host[sl];
        h.assign(static_cast<size_t>(MAX_TL) * 2 * TMAP_BYTES, 0);
        bool ok = kv.kv_dim == d.KV && kv.max_pos > 0;
        const cuuint64_t dims[2] = {static_cast<cuuint64_t>(d.KV), static_cast<cuuint64_t>(kv.max_pos)};
        const cuuint64_t strides[1] = {static_cast<cuuint64_t>(d.KV) * 2};
        const cuuint32_t box[2] = {static_cast<cuuint32_t>(d.HD), static_cast<cuuint32_t>(KV_BOX)};
        const cuuint32_t estr[2] = {1, 1};
        for (int l = 0; l < d.TL && ok; ++l)
            for (int c = 0; c < 2 && ok; ++c) {
                const void * base = c ? static_cast<const void *>(kv.v[l]) : static_cast<const void *>(kv.k[l]);
                if (reinterpret_cast<std::uintptr_t>(base) & 15u) { ok = false; break; }
                CUtensorMap * m = reinterpret_cast<CUtensorMap *>(h.data() + (static_cast<size_t>(l) * 2 + c) * TMAP_BYTES);
                ok = encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
            }
        for (int l = 0; l < d.TL; ++l) {
            kvmap_src[sl][l][0] = kv.k[l];
            kvmap_src[sl][l][1] = kv.v[l];
        }
        kvmap_pos[sl] = ok ? kv.max_pos : -1;
        if (!ok) return nullptr;
        NAVI_CUDA(cudaMemcpyAsync(dst, h.data(), h.size(), cudaMemcpyHostToDevice, stream));
        NAVI_CUDA(cudaStreamSynchronize(stream));
        return dst;
    }

    // layer >= 0: the single-layer program of that talker layer, from step_in into layer_out.
    // hidden_in / logits_in: frame 0 of one stream (the code predictor only).
    int launch(const StreamIn * in, int nb, const float * hidden_in, const float * logits_in, const Sampling & s, std::string & err,
               int layer = -1, float * layer_out = nullptr) {
        NAVI_CUDA(cudaSetDevice(ordinal));
        Args A{};
        const bool first = hidden_in != nullptr || (nb > 1 && in[0].hidden != nullptr);
        if (nb == 1) {
            A.prog = layer >= 0 ? prog_layers + static_cast<size_t>(layer) * LAYER_PHASES : first ? prog_first : prog_full;
            A.nphase = layer >= 0 ? LAYER_PHASES : first ? n_first : n_full;
        } else {
            A.prog = first ? prog_batch_first[nb] : prog_batch[nb];
            A.nphase = first ? n_batch_first[nb] : n_batch[nb];
            A.thead_phase = thead_phase[nb];
            for (int cb = 0; cb < NCB; ++cb) A.sample_phase[cb] = first ? sample_phase_first[nb][cb] : sample_phase[nb][cb];
        }
        A.mw = dmw;
        A.d = d;
        A.w = w;
        A.grid = grid;
        A.nb = nb;
        const Mode & M = modes[nb];
        A.xcols = M.xcols;
        A.cp_slots = M.cp_slots;
        A.attn_per = std::max(1, std::min(MAX_SPLIT, grid / (d.NKV * nb)));
        if (tag > 0xF0000000u) {   // tags about to wrap: clear every exchange word once
            NAVI_CUDA(cudaMemsetAsync(ll_base, 0, ll_bytes, stream));
            NAVI_CUDA(cudaMemsetAsync(w.ctl, 0, 16, stream));
            tag = 0;
        }
        tag += 4096;
        A.tag_base = tag;
        for (int i = 0; i < nb; ++i) {
            const StreamIn & q = in[i];
            A.n_past[i] = q.n_past;
            attn_plan(q.n_past, A.attn_per, A.attn_split[i], A.attn_chunk[i]);
            if (!first) {
                if (A.attn_chunk[i] + 1 > MAX_ATTN_CHUNK + 1) {
                    err = "KV length " + std::to_string(q.n_past) + " needs " + std::to_string(A.attn_chunk[i]) +
                          " positions per attention split; the kernel takes at most " + std::to_string(MAX_ATTN_CHUNK);
                    return NAVI_E_KV_FULL;
                }
                const uint64_t krows = static_cast<uint64_t>(A.attn_chunk[i] + KV_BOX - 1) / KV_BOX * KV_BOX;   // whole boxes
                const uint64_t kvb = 2ull * krows * d.HD * 2 + 2ull * d.HD * 4;
                if (kvb > M.ring) {
                    err = "KV length " + std::to_string(q.n_past) + " needs " + std::to_string(kvb) + "-byte attention slices; the ring holds " +
                          std::to_string(M.ring);
                    return NAVI_E_KV_FULL;
                }
            }
            const int sl = q.slot;
            A.step_in[i] = q.step_in ? q.step_in : step[sl][cur[sl]];
            A.trailing[i] = q.trailing;
            A.step_out[i] = layer >= 0 ? layer_out : step[sl][cur[sl] ^ 1];
            A.seen[i] = seen + static_cast<size_t>(sl) * d.TV;
            if (q.kv) {
                for (int l = 0; l < d.TL; ++l) {
                    A.kc[i][l] = reinterpret_cast<__half *>(q.kv->k[l]);
                    A.vc[i][l] = reinterpret_cast<__half *>(q.kv->v[l]);
                }
                // boxed loads pay off once a split covers several boxes' worth of positions (a
                // 4-stream launch at KV 512: 128); a short split is faster as 32 row copies in flight
                A.kvmap[i] = A.attn_chunk[i] > 2 * KV_BOX ? kv_maps(sl, *q.kv) : nullptr;
            }
            if (!first) std::memcpy(A.rope_t[i], rope_at(q.n_past), 2 * inv_t_h.size() * sizeof(float));
            A.first_hidden[i] = nb > 1 ? q.hidden : nullptr;
            A.first_logits[i] = nb > 1 ? q.logits : nullptr;
            A.seed[i] = q.seed;
            A.frame_index[i] = q.frame_index;
            for (int cb = 0; cb < NCB; ++cb) A.pcg_seed[i][cb] = navi::dev::pcg_draw_seed(q.seed, q.frame_index, cb);
        }
        A.hidden_in = hidden_in;
        A.logits_in = logits_in;
        A.inv_freq_t = inv_t;
        A.inv_freq_c = inv_c;
        A.rope_c = rope_c;
        A.temp = s.temperature; A.top_p = s.top_p; A.rep = s.repetition_penalty; A.top_k = s.top_k;
        A.cp_temp = s.cp_temperature; A.cp_top_p = s.cp_top_p; A.cp_top_k = s.cp_top_k;
        A.min_frames = s.min_frames; A.rng = s.rng;
        A.eos_id = eos;
        A.suppress_from = suppress_from;
        A.timeout_ns = timeout_ns;
        A.poll_ns = poll_ns;
        A.ring_bytes = M.ring;
        A.cp_keep_layers = cp_keep_layers;
        A.scratch_floats = scratch_floats;
        A.part_floats = M.part_floats;
        A.ysum_off = M.ysum_off;
        A.prof = prof_on ? prof : nullptr;
        if (prof_on) NAVI_CUDA(cudaMemsetAsync(prof, 0, static_cast<size_t>(PROF_STRIDE) * grid * sizeof(unsigned long long), stream));
        A.prof_cta = prof_cta;
        last_nphase = A.nphase;
        NAVI_CUDA(cudaEventRecord(ev0, stream));
        void * args[] = {&A};
        const void * kern = nb > 1 ? reinterpret_cast<const void *>(&k_frame_batch) : reinterpret_cast<const void *>(&k_frame);
        const cudaError_t e = cudaLaunchCooperativeKernel(kern, dim3(grid), dim3(NTHR), args, M.smem, stream);
        if (e != cudaSuccess) {
            (void) cudaGetLastError();
            err = std::string("cooperative launch failed: ") + cudaGetErrorString(e);
            return NAVI_E_LAUNCH;
        }
        NAVI_CUDA(cudaEventRecord(ev1, stream));
        // the 4 control words and the codes are one block in device memory: one copy
        NAVI_CUDA(cudaMemcpyAsync(h_out, w.ctl, (4 + static_cast<size_t>(nb) * NCB) * sizeof(int32_t), cudaMemcpyDeviceToHost, stream));
        if (layer < 0)
            for (int i = 0; i < nb; ++i) cur[in[i].slot] ^= 1;
        last_tag = tag;
        last_nb = nb;
        pending = true;
        return NAVI_OK;
    }

    // Results of the last launch, one per stream (out[0..last_nb)).
    void collect(FrameResult * out) {
        const int nb = std::max(1, last_nb);
        if (!pending) {
            for (int i = 0; i < nb; ++i) { out[i] = FrameResult{}; out[i].status = NAVI_E_ARG; out[i].error = "no frame enqueued"; }
            return;
        }
        pending = false;
        NAVI_CUDA(cudaSetDevice(ordinal));
        NAVI_CUDA(cudaStreamSynchronize(stream));
        float ms = 0.f;
        NAVI_CUDA(cudaEventElapsedTime(&ms, ev0, ev1));
        const uint32_t * ctl = reinterpret_cast<const uint32_t *>(h_out);
        const bool failed = ctl[2] == last_tag || ctl[0] != last_tag;
        for (int i = 0; i < nb; ++i) {
            FrameResult & r = out[i];
            r = FrameResult{};
            r.us = ms * 1000.0;
            if (failed) {
                r.status = NAVI_E_TIMEOUT;
                r.error = "device wait timed out in phase " + std::to_string(ctl[1]) + " (CTA " + std::to_string(ctl[3]) +
                          "): the cooperative grid could not run to completion";
                continue;
            }
            std::memcpy(r.codes, h_out + 4 + i * NCB, sizeof(r.codes));
            r.eos = r.codes[0] == eos;
            r.ok = true;
        }
    }
    FrameResult collect() {
        FrameResult r[MAX_B];
        collect(r);
        return r[0];
    }
};

std::unique_ptr<Frame> Frame::create(const Device & dev, const DeviceWeights & wts, const FrameOptions & opt) {
    std::unique_ptr<Frame> f(new Frame());
    f->impl_ = std::make_unique<Impl>();
    Impl & I = *f->impl_;
    dev.make_current();
    I.ordinal = dev.info().ordinal;
    I.stream = dev.stream();
    const Params & p = wts.params();
    const auto & tp = p.talker;
    const auto & cp = p.cp;
    // shapes the kernel is built for
    if (tp.hidden != cp.hidden || tp.n_head != cp.n_head || tp.n_kv_head != cp.n_kv_head || tp.head_dim != cp.head_dim || tp.ff != cp.ff)
        fail("frame: the talker and code predictor must share hidden/heads/head_dim/ff", NAVI_E_SHAPE);
    if (tp.n_layer > MAX_TL || cp.n_layer > MAX_CP) fail("frame: too many layers for the kernel", NAVI_E_SHAPE);
    if (p.n_code_groups != NCB) fail("frame: the kernel is built for 16 codebooks", NAVI_E_SHAPE);
    // the attention code is specialised at compile time (shape-generic code ran several times slower)
    if (tp.head_dim != KHD || tp.n_head != KGR * tp.n_kv_head)
        fail("frame: the kernel is built for head_dim " + std::to_string(KHD) + " and " + std::to_string(KGR) +
                 " query heads per KV head",
             NAVI_E_SHAPE);
    const int Q = tp.n_head * tp.head_dim, KV = tp.n_kv_head * tp.head_dim;
    if (tp.hidden % 256 || Q % 256 || tp.ff % 256) fail("frame: hidden, n_head*head_dim and ff must be multiples of 256", NAVI_E_SHAPE);
    if (opt.blocks_per_mp != 1) fail("frame: blocks_per_mp must be 1 (one CTA per SM)", NAVI_E_ARG);
    Dims & d = I.d;
    d.H = tp.hidden; d.NH = tp.n_head; d.NKV = tp.n_kv_head; d.HD = tp.head_dim; d.F = tp.ff;
    d.TV = tp.vocab; d.CV = cp.vocab; d.TL = tp.n_layer; d.CL = cp.n_layer;
    d.Q = Q; d.KV = KV; d.QKV = Q + 2 * KV; d.GROUP = tp.n_head / tp.n_kv_head;
    d.eps_t = tp.rms_eps; d.eps_c = cp.rms_eps;
    if (d.NKV * d.CL > dev.info().multiprocessors) fail("frame: code-predictor attention needs a CTA per (KV head, layer)", NAVI_E_SHAPE);
    I.eos = p.codec_eos_id;
    I.suppress_from = tp.vocab - 1024;   // HF suppress_tokens = range(vocab - 1024, vocab) minus EOS (frame.hip:760)
    I.timeout_ns = (opt.deadline_us ? opt.deadline_us : 200000ull) * 1000ull;
    if (const char * env = std::getenv("NAVI_POLL_NS")) I.poll_ns = static_cast<uint32_t>(std::atoi(env));

    // weight tables: the frame streams its own copy of every matrix, re-laid out per CTA slice
    I.grid = dev.info().multiprocessors * opt.blocks_per_mp;
    const int Gs = I.grid;
    size_t slice_elems = 0;
    const size_t per_layer = static_cast<size_t>(d.QKV) * d.H + static_cast<size_t>(d.H) * d.Q + 2ull * d.F * d.H + static_cast<size_t>(d.H) * d.F;
    slice_elems = per_layer * (d.TL + d.CL) + static_cast<size_t>(d.TV) * d.H + static_cast<size_t>(NCB - 1) * d.CV * d.H;
    I.wslices = I.alloc<__half>(slice_elems);
    size_t slice_at = 0;
    auto sliced = [&](const __half * W, int R, int K) {
        __half * out = I.wslices + slice_at;
        slice_at += static_cast<size_t>(R) * K;
        if (K % 8) fail("frame: matrix width must be a multiple of 8", NAVI_E_SHAPE);
        k_slice_layout<<<1184, 256, 0, I.stream>>>(W, out, R, K, Gs);
        NAVI_CUDA(cudaGetLastError());
        return static_cast<const __half *>(out);
    };
    ModelW hw{};
    auto f16p = [&](const std::string & n) { return reinterpret_cast<const __half *>(wts.get(n).ptr); };
    auto f32p = [&](const std::string & n) { return wts.get(n).as<float>(); };
    auto layer = [&](const std::string & prefix, int l) {
        const std::string lp = prefix + ".layers." + std::to_string(l) + ".";
        LayerW L{};
        L.ln1 = f32p(lp + "input_layernorm.weight");
        L.ln2 = f32p(lp + "post_attention_layernorm.weight");
        L.qn = f32p(lp + "self_attn.q_norm.weight");
        L.kn = f32p(lp + "self_attn.k_norm.weight");
        const __half * wq = f16p(lp + "self_attn.q_proj.weight");
        const __half * wk = f16p(lp + "self_attn.k_proj.weight");
        const __half * wv = f16p(lp + "self_attn.v_proj.weight");
        if (wk != wq + static_cast<size_t>(Q) * d.H || wv != wk + static_cast<size_t>(KV) * d.H)
            fail("frame: q/k/v of " + lp + " are not adjacent in the weight arena", NAVI_E_FORMAT);
        L.wqkv = sliced(wq, d.QKV, d.H);
        L.wo = sliced(f16p(lp + "self_attn.o_proj.weight"), d.H, d.Q);
        L.wg = sliced(f16p(lp + "mlp.gate_proj.weight"), d.F, d.H);
        L.wu = sliced(f16p(lp + "mlp.up_proj.weight"), d.F, d.H);
        L.wd = sliced(f16p(lp + "mlp.down_proj.weight"), d.H, d.F);
        return L;
    };
    for (int l = 0; l < d.TL; ++l) hw.tl[l] = layer("talker.model", l);
    for (int l = 0; l < d.CL; ++l) hw.cp[l] = layer("talker.code_predictor.model", l);
    hw.tl_norm = f32p("talker.model.norm.weight");
    hw.cp_norm = f32p("talker.code_predictor.model.norm.weight");
    hw.codec_head = sliced(f16p("talker.codec_head.weight"), d.TV, d.H);
    hw.tl_emb = f16p("talker.model.codec_embedding.weight");
    for (int i = 0; i < NCB - 1; ++i) {
        hw.cp_emb[i] = f16p("talker.code_predictor.model.codec_embedding." + std::to_string(i) + ".weight");
        hw.lm_head[i] = sliced(f16p("talker.code_predictor.lm_head." + std::to_string(i) + ".weight"), d.CV, d.H);
    }
    NAVI_CUDA(cudaStreamSynchronize(I.stream));
    I.dmw = I.alloc<ModelW>(1);
    NAVI_CUDA(cudaMemcpy(I.dmw, &hw, sizeof(ModelW), cudaMemcpyHostToDevice));

    // phase programs: with the talker step, and frame 0 (code predictor only)
    auto build = [&](bool with_talker) {
        std::vector<Phase> v;
        if (with_talker) {
            for (int l = 0; l < d.TL; ++l)
                for (uint8_t op : {TQKV, TATTN, TO, TGU, TDOWN}) v.push_back({op, 1, static_cast<uint8_t>(l), 0});
            v.push_back({THEAD, 1, 0, 0});
        }
        for (int l = 0; l < d.CL; ++l)
            for (uint8_t op : {CQKV, CATTN, CO, CGU, CDOWN}) v.push_back({op, 2, static_cast<uint8_t>(l), 0});
        v.push_back({CHEAD, 2, 0, 1});
        for (int pos = 2; pos < NCB; ++pos) {
            for (int l = 0; l < d.CL; ++l)
                for (uint8_t op : {CQKV, CATTN, CO, CGU, CDOWN}) v.push_back({op, 1, static_cast<uint8_t>(l), static_cast<uint8_t>(pos)});
            v.push_back({CHEAD, 1, 0, static_cast<uint8_t>(pos)});
        }
        v.push_back({FINAL, 1, 0, 0});
        return v;
    };
    const auto pf = build(true), p0 = build(false);
    std::vector<Phase> pl;
    for (int l = 0; l < d.TL; ++l) {
        pl.push_back({TQKV, 1, static_cast<uint8_t>(l), POS_STEP_IN});
        for (uint8_t op : {TATTN, TO, TGU, TDOWN}) pl.push_back({op, 1, static_cast<uint8_t>(l), 0});
        pl.push_back({XOUT, 1, static_cast<uint8_t>(l), 0});
    }
    I.prog_layers = I.alloc<Phase>(pl.size());
    NAVI_CUDA(cudaMemcpy(I.prog_layers, pl.data(), pl.size() * sizeof(Phase), cudaMemcpyHostToDevice));
    I.n_full = static_cast<int>(pf.size());
    I.n_first = static_cast<int>(p0.size());
    if (I.n_full >= 4096) fail("frame: phase program too long", NAVI_E_SHAPE);
    I.prog_full = I.alloc<Phase>(pf.size());
    I.prog_first = I.alloc<Phase>(p0.size());
    NAVI_CUDA(cudaMemcpy(I.prog_full, pf.data(), pf.size() * sizeof(Phase), cudaMemcpyHostToDevice));
    NAVI_CUDA(cudaMemcpy(I.prog_first, p0.data(), p0.size() * sizeof(Phase), cudaMemcpyHostToDevice));
    // batched programs (nb streams, one input column each): the talker step, THEAD (which also
    // publishes every stream's post-norm hidden), the codebook-0 draws (SAMPLE: CTA s draws
    // stream s), code-predictor position 0 on the hidden, then for positions 1..15 the pass on
    // the embedding of the code drawn last, its head and the draw; FINAL assembles the step
    // embeddings from the published codes
    for (int nb : {2, 4}) {
        std::vector<Phase> v;
        const uint8_t c = static_cast<uint8_t>(nb);
        for (int l = 0; l < d.TL; ++l)
            for (uint8_t op : {TQKV, TATTN, TO, TGU, TDOWN}) v.push_back({op, c, static_cast<uint8_t>(l), 0});
        I.thead_phase[nb] = static_cast<int>(v.size());
        v.push_back({THEAD, c, 0, 0});
        I.sample_phase[nb][0] = static_cast<int>(v.size());
        v.push_back({SAMPLE, c, 0, 0});
        for (int pos = 0; pos < NCB; ++pos) {
            for (int l = 0; l < d.CL; ++l)
                for (uint8_t op : {CQKV, CATTN, CO, CGU, CDOWN}) v.push_back({op, c, static_cast<uint8_t>(l), static_cast<uint8_t>(pos)});
            if (pos == 0) continue;
            v.push_back({CHEAD, c, 0, static_cast<uint8_t>(pos)});
            I.sample_phase[nb][pos] = static_cast<int>(v.size());
            v.push_back({SAMPLE, c, 0, static_cast<uint8_t>(pos)});
        }
        v.push_back({FINAL, c, 0, 0});
        if (v.size() >= 4096) fail("frame: batched phase program too long", NAVI_E_SHAPE);
        I.n_batch[nb] = static_cast<int>(v.size());
        I.prog_batch[nb] = I.alloc<Phase>(v.size());
        NAVI_CUDA(cudaMemcpy(I.prog_batch[nb], v.data(), v.size() * sizeof(Phase), cudaMemcpyHostToDevice));
        // frame 0: the same from the first SAMPLE on (codebook 0 drawn from each stream's
        // prefill logits, position 0 on its prefill hidden)
        const int cut = I.sample_phase[nb][0];
        std::vector<Phase> f(v.begin() + cut, v.end());
        for (int cb = 0; cb < NCB; ++cb) I.sample_phase_first[nb][cb] = I.sample_phase[nb][cb] - cut;
        I.n_batch_first[nb] = static_cast<int>(f.size());
        I.prog_batch_first[nb] = I.alloc<Phase>(f.size());
        NAVI_CUDA(cudaMemcpy(I.prog_batch_first[nb], f.data(), f.size() * sizeof(Phase), cudaMemcpyHostToDevice));
    }

    // exchange words (one allocation, cleared when tags wrap)
    const size_t n_x = 1ull * MAXC * d.H, n_qkv = 1ull * MAXC * d.QKV, n_attn = 1ull * MAXC * d.Q, n_h = 1ull * MAXC * d.F,
                 n_lg = 1ull * MAX_B * d.TV, n_clg = static_cast<size_t>(MAX_B) * (NCB - 1) * d.CV,
                 n_part = static_cast<size_t>(MAX_SPLIT) * d.NH * (d.HD + 2), n_hid = 1ull * MAX_B * d.H, n_code = 1ull * MAX_B * NCB;
    const size_t n_ll = n_x + n_qkv + n_attn + n_h + n_lg + n_clg + n_part + n_hid + n_code;
    I.ll_base = I.alloc<uint64_t>(n_ll);
    I.ll_bytes = n_ll * sizeof(uint64_t);
    uint64_t * q = I.ll_base;
    I.w.x = q; q += n_x;
    I.w.qkv = q; q += n_qkv;
    I.w.attn = q; q += n_attn;
    I.w.h = q; q += n_h;
    I.w.logits = q; q += n_lg;
    I.w.clogits = q; q += n_clg;
    I.w.part = q; q += n_part;
    I.w.hid_x = q; q += n_hid;
    I.w.code_x = q;
    I.seen = I.alloc<uint8_t>(static_cast<size_t>(MAX_B) * d.TV);
    I.kvmaps = I.alloc<uint8_t>(static_cast<size_t>(MAX_B) * MAX_TL * 2 * TMAP_BYTES + 64);
    if (reinterpret_cast<std::uintptr_t>(I.kvmaps) & 63u) fail("frame: tensor-map storage is not 64-byte aligned", NAVI_E_CUDA);
    // control words [4] then the codes [MAX_B][16]: a launch's results leave in one copy
    I.w.ctl = I.alloc<unsigned>(4 + static_cast<size_t>(MAX_B) * NCB);
    I.w.codes = reinterpret_cast<int32_t *>(I.w.ctl + 4);
    I.w.hidden = I.alloc<float>(static_cast<size_t>(MAX_B) * d.H);
    for (int sl = 0; sl < MAX_B; ++sl) {
        I.step[sl][0] = I.alloc<float>(d.H);
        I.step[sl][1] = I.alloc<float>(d.H);
    }
    // RoPE inverse frequencies theta^(-2t/hd), computed in double, stored as f32
    auto inv = [&](double theta, std::vector<float> & v) {
        v.resize(d.HD / 2);
        for (int t = 0; t < d.HD / 2; ++t) v[t] = static_cast<float>(1.0 / std::pow(theta, 2.0 * t / d.HD));
        float * dv = I.alloc<float>(v.size());
        NAVI_CUDA(cudaMemcpy(dv, v.data(), v.size() * sizeof(float), cudaMemcpyHostToDevice));
        return dv;
    };
    I.inv_t = inv(tp.rope_theta, I.inv_t_h);
    I.inv_c = inv(cp.rope_theta, I.inv_c_h);
    {
        std::vector<float> tab(static_cast<size_t>(NCB) * d.HD);
        for (int pos = 0; pos < NCB; ++pos) rope_row(I.inv_c_h, pos, tab.data() + static_cast<size_t>(pos) * d.HD);
        I.rope_c = I.alloc<float>(tab.size());
        NAVI_CUDA(cudaMemcpy(I.rope_c, tab.data(), tab.size() * sizeof(float), cudaMemcpyHostToDevice));
    }

    // shared memory: everything but the ring is sized from the shapes; the ring takes the rest
    const int G = I.grid, Vmax = std::max(d.TV, d.CV);
    const uint32_t xin = static_cast<uint32_t>(MAXC) * std::max(d.H, std::max(d.Q, d.F));
    const uint32_t samp = navi::dev::sample_scratch_floats(Vmax);
    // attention scratch: code predictor [q, k, v, scores, m/l, per-warp P.V]; talker split
    // [q, k, v, new K/V row, m/l, per-warp P.V, scores]; talker combine [splits][m, l, acc]
    const uint32_t pvf = static_cast<uint32_t>(NCW * MAX_GROUP * d.HD);
    const uint32_t att = std::max({2u * MAX_GROUP * d.HD + 4u * d.HD + 2u * MAX_GROUP * NCB + 4u * MAX_GROUP + pvf,
                                   static_cast<uint32_t>(MAX_GROUP * d.HD + 3 * d.HD + 2 * MAX_GROUP) + pvf +
                                       static_cast<uint32_t>(MAX_GROUP * (MAX_ATTN_CHUNK + 1)),
                                   static_cast<uint32_t>(std::min(MAX_SPLIT, I.grid / d.NKV) * (d.HD + 2))});
    I.scratch_floats = std::max(xin, std::max(samp, att));
    const int max_nr = std::max({cdiv(d.QKV, G), cdiv(d.H, G), cdiv(d.F, G), cdiv(d.TV, G), cdiv(d.CV, G)});
    const uint32_t optin = static_cast<uint32_t>(dev.info().smem_optin);
    const uint32_t H4 = 4u * d.H;
    const uint32_t max_chunk = std::max({H4 + static_cast<uint32_t>(cdiv(d.QKV, G) * d.H * 2), static_cast<uint32_t>(cdiv(d.H, G) * d.Q * 2),
                                         H4 + static_cast<uint32_t>(2 * cdiv(d.F, G) * d.H * 2), static_cast<uint32_t>(cdiv(d.H, G) * d.F * 2),
                                         H4 + static_cast<uint32_t>(cdiv(d.TV, G) * d.H * 2), H4 + static_cast<uint32_t>(cdiv(d.CV, G) * d.H * 2),
                                         static_cast<uint32_t>(2 * 8 * d.HD * 2 + 2 * d.HD * 4)});
    // per stream count: the residual columns and code-predictor K/V slots in shared memory, and
    // the ring that takes the rest
    uint32_t smem_max = 0;
    for (int nb : {1, 2, 4}) {
        Impl::Mode & M = I.modes[nb];
        M.xcols = std::max(2, nb);
        M.cp_slots = cdiv(nb * d.CL * d.NKV, G);
        // per warp: columns x (gate, up) x rows; then the summed [columns x (gate, up)][rows]
        M.ysum_off = static_cast<uint32_t>(NCW * 2 * M.xcols * max_nr);
        M.part_floats = M.ysum_off + static_cast<uint32_t>(2 * M.xcols * max_nr);
        if (nb * d.NKV > G) fail("frame: batched attention needs a CTA per (stream, KV head)", NAVI_E_SHAPE);
        const SmemLayout L0 = smem_layout(d, 0, I.scratch_floats, M.part_floats, M.xcols, M.cp_slots);
        if (L0.total + 16384 > optin) fail("frame: shared memory too small for the model shape", NAVI_E_SHAPE);
        M.ring = (optin - L0.total) / 128 * 128;
        if (max_chunk > M.ring) fail("frame: a phase's weight slice does not fit the shared-memory ring", NAVI_E_SHAPE);
        M.smem = smem_layout(d, M.ring, I.scratch_floats, M.part_floats, M.xcols, M.cp_slots).total;
        smem_max = std::max(smem_max, M.smem);
    }
    // The code predictor's weights are read 15 times a frame; as many whole layers as fit in
    // about 70% of L2 are marked evict-last (NAVI_L2_KEEP_LAYERS overrides the count).
    {
        const double layer_bytes = 2.0 * (static_cast<double>(d.QKV) * d.H + static_cast<double>(d.H) * d.Q + 2.0 * d.F * d.H +
                                          static_cast<double>(d.H) * d.F);
        int keep = static_cast<int>(0.7 * static_cast<double>(dev.info().l2_bytes) / layer_bytes);
        if (const char * env = std::getenv("NAVI_L2_KEEP_LAYERS")) keep = std::atoi(env);
        I.cp_keep_layers = std::max(0, std::min(keep, d.CL));
    }
    for (const void * kern : {reinterpret_cast<const void *>(&k_frame), reinterpret_cast<const void *>(&k_frame_batch)}) {
        NAVI_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_max));
        int occ = 0;
        NAVI_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, NTHR, smem_max));
        if (occ < 1) fail("frame: the frame kernel cannot be resident with " + std::to_string(smem_max) + " bytes of shared memory", NAVI_E_SHAPE);
    }
    NAVI_CUDA(cudaEventCreate(&I.ev0));
    NAVI_CUDA(cudaEventCreate(&I.ev1));
    void * h = nullptr;
    NAVI_CUDA(cudaMallocHost(&h, (MAX_B * NCB + 4) * sizeof(int32_t)));
    I.h_out = static_cast<int32_t *>(h);
    return f;
}

Frame::~Frame() {
    if (!impl_) return;
    cudaSetDevice(impl_->ordinal);
    if (impl_->pending) cudaStreamSynchronize(impl_->stream);
    if (impl_->ev0) cudaEventDestroy(impl_->ev0);
    if (impl_->ev1) cudaEventDestroy(impl_->ev1);
    if (impl_->h_out) cudaFreeHost(impl_->h_out);
    for (void * p : impl_->owned) cudaFree(p);
}

void Frame::reset(int slot) {
    Impl & I = *impl_;
    if (slot < 0 || slot >= MAX_B) fail("frame: slot out of range", NAVI_E_ARG);
    NAVI_CUDA(cudaSetDevice(I.ordinal));
    NAVI_CUDA(cudaMemsetAsync(I.seen + static_cast<size_t>(slot) * I.d.TV, 0, static_cast<size_t>(I.d.TV), I.stream));
}

FrameResult Frame::run_first(const float * d_hidden, const float * d_logits, const float * d_trailing, const Sampling & s,
                             uint64_t seed, int frame_index, int slot) {
    Impl & I = *impl_;
    FrameResult r;
    if (slot < 0 || slot >= MAX_B) { r.status = NAVI_E_ARG; r.error = "slot out of range"; return r; }
    std::string err;
    Impl::StreamIn in;
    in.slot = slot;
    in.trailing = d_trailing;
    in.seed = seed;
    in.frame_index = frame_index;
    const int st = I.launch(&in, 1, d_hidden, d_logits, s, err);
    if (st != NAVI_OK) { r.status = st; r.error = err; return r; }
    return I.collect();
}

int Frame::enqueue_batch(int nb, const int * slots, KvCache * const * kvs, const int * n_past, const float * const * d_trailing,
                         const Sampling & s, const uint64_t * seeds, const int * frame_index, std::string & err) {
    Impl & I = *impl_;
    if (nb != 1 && nb != 2 && nb != 4) { err = "a batched frame takes 1, 2 or 4 streams"; return NAVI_E_ARG; }
    Impl::StreamIn in[MAX_B];
    bool used[MAX_B] = {};
    for (int i = 0; i < nb; ++i) {
        KvCache & kv = *kvs[i];
        if (slots[i] < 0 || slots[i] >= MAX_B || used[slots[i]]) { err = "stream slots must be distinct, in 0.." + std::to_string(MAX_B - 1); return NAVI_E_ARG; }
        used[slots[i]] = true;
        if (n_past[i] < 0 || n_past[i] >= kv.max_pos) { err = "KV cache full"; return NAVI_E_KV_FULL; }
        if (kv.n_layer != I.d.TL || kv.kv_dim != I.d.KV) { err = "KV cache layout does not match the talker"; return NAVI_E_ARG; }
        if (!d_trailing[i]) { err = "NULL trailing row"; return NAVI_E_ARG; }
        in[i].slot = slots[i];
        in[i].trailing = d_trailing[i];
        in[i].kv = &kv;
        in[i].n_past = n_past[i];
        in[i].seed = seeds[i];
        in[i].frame_index = frame_index[i];
    }
    const int st = I.launch(in, nb, nullptr, nullptr, s, err);
    if (st == NAVI_OK)
        for (int i = 0; i < nb; ++i) kvs[i]->n_used = n_past[i] + 1;
    return st;
}

void Frame::collect_batch(FrameResult * out) { impl_->collect(out); }

int Frame::enqueue_first_batch(int nb, const int * slots, const float * const * d_hidden, const float * const * d_logits,
                               const float * const * d_trailing, const Sampling & s, const uint64_t * seeds, const int * frame_index,
                               std::string & err) {
    Impl & I = *impl_;
    if (nb != 2 && nb != 4) { err = "a batched frame 0 takes 2 or 4 streams"; return NAVI_E_ARG; }
    Impl::StreamIn in[MAX_B];
    bool used[MAX_B] = {};
    for (int i = 0; i < nb; ++i) {
        if (slots[i] < 0 || slots[i] >= MAX_B || used[slots[i]]) { err = "stream slots must be distinct, in 0.." + std::to_string(MAX_B - 1); return NAVI_E_ARG; }
        used[slots[i]] = true;
        if (!d_hidden[i] || !d_logits[i] || !d_trailing[i]) { err = "NULL hidden, logits or trailing row"; return NAVI_E_ARG; }
        in[i].slot = slots[i];
        in[i].hidden = d_hidden[i];
        in[i].logits = d_logits[i];
        in[i].trailing = d_trailing[i];
        in[i].seed = seeds[i];
        in[i].frame_index = frame_index[i];
    }
    return I.launch(in, nb, nullptr, nullptr, s, err);
}

int Frame::enqueue(KvCache & kv, int n_past, const float * d_trailing, const Sampling & s, uint64_t seed, int frame_index,
                   std::string & err) {
    const int slot = 0;
    KvCache * k = &kv;
    return enqueue_batch(1, &slot, &k, &n_past, &d_trailing, s, &seed, &frame_index, err);
}

FrameResult Frame::run(KvCache & kv, int n_past, const float * d_trailing, const Sampling & s, uint64_t seed, int frame_index) {
    std::string err;
    const int st = enqueue(kv, n_past, d_trailing, s, seed, frame_index, err);
    if (st != NAVI_OK) { FrameResult r; r.status = st; r.error = err; return r; }
    return impl_->collect();
}

FrameResult Frame::run_layer(int layer, const float * d_x, KvCache & kv, int n_past, float * d_out) {
    Impl & I = *impl_;
    FrameResult r;
    if (layer < 0 || layer >= I.d.TL) { r.status = NAVI_E_ARG; r.error = "layer " + std::to_string(layer) + " out of range"; return r; }
    if (!d_x || !d_out) { r.status = NAVI_E_ARG; r.error = "NULL input or output"; return r; }
    if (n_past < 0 || n_past >= kv.max_pos) { r.status = NAVI_E_KV_FULL; r.error = "KV cache full"; return r; }
    if (kv.n_layer != I.d.TL || kv.kv_dim != I.d.KV) { r.status = NAVI_E_ARG; r.error = "KV cache layout does not match the talker"; return r; }
    std::string err;
    Impl::StreamIn in;
    in.step_in = d_x;
    in.kv = &kv;
    in.n_past = n_past;
    const int st = I.launch(&in, 1, nullptr, nullptr, Sampling{}, err, layer, d_out);
    if (st != NAVI_OK) { r.status = st; r.error = err; return r; }
    return I.collect();
}

FrameResult Frame::collect() { return impl_->collect(); }

const float * Frame::d_step_out(int slot) const {
    if (slot < 0 || slot >= MAX_B) return nullptr;
    return impl_->step[slot][impl_->cur[slot]];
}

void Frame::set_step_in(const float * d_step, int slot) {
    Impl & I = *impl_;
    if (slot < 0 || slot >= MAX_B) fail("frame: slot out of range", NAVI_E_ARG);
    NAVI_CUDA(cudaSetDevice(I.ordinal));
    NAVI_CUDA(cudaMemcpyAsync(I.step[slot][I.cur[slot]], d_step, static_cast<size_t>(I.d.H) * sizeof(float), cudaMemcpyDeviceToDevice,
                              I.stream));
}

int Frame::grid_blocks() const { return impl_->grid; }

void Frame::set_profile(bool on, int cta) {
    Impl & I = *impl_;
    if (on && !I.prof) I.prof = I.alloc<unsigned long long>(static_cast<size_t>(PROF_STRIDE) * I.grid);
    I.prof_on = on;
    I.prof_cta = cta < 0 ? -1 : std::min(cta, I.grid - 1);
}

int Frame::profile(uint64_t * out, int cap) const {
    const Impl & I = *impl_;
    if (!I.prof) return 0;
    NAVI_CUDA(cudaSetDevice(I.ordinal));
    NAVI_CUDA(cudaStreamSynchronize(I.stream));
    // per traced CTA: out[0] = launch start, out[1 + 4p + k] = stamp k of phase p
    const int per = 4 * I.last_nphase + 1;
    const int nct = I.prof_cta < 0 ? I.grid : 1;
    std::vector<unsigned long long> tmp(static_cast<size_t>(PROF_STRIDE) * nct);
    NAVI_CUDA(cudaMemcpy(tmp.data(), I.prof, tmp.size() * sizeof(unsigned long long), cudaMemcpyDeviceToHost));
    int n = 0;
    for (int c = 0; c < nct && n + per <= cap; ++c) {
        const unsigned long long * src = tmp.data() + static_cast<size_t>(c) * PROF_STRIDE;
        out[n] = src[4 * I.last_nphase];
        for (int i = 0; i + 1 < per; ++i) out[n + 1 + i] = src[i];
        n += per;
    }
    return n;
}

void Frame::inspect(float * hidden, float * logits, float * clogits, int index) const {
    const Impl & I = *impl_;
    if (index < 0 || index >= MAX_B) fail("frame: stream index out of range", NAVI_E_ARG);
    NAVI_CUDA(cudaSetDevice(I.ordinal));
    NAVI_CUDA(cudaStreamSynchronize(I.stream));
    if (hidden)
        NAVI_CUDA(cudaMemcpy(hidden, I.w.hidden + static_cast<size_t>(index) * I.d.H, static_cast<size_t>(I.d.H) * sizeof(float),
                             cudaMemcpyDeviceToHost));
    auto unpack = [](const uint64_t * src, size_t n, float * dst) {
        std::vector<uint64_t> tmp(n);
        NAVI_CUDA(cudaMemcpy(tmp.data(), src, n * sizeof(uint64_t), cudaMemcpyDeviceToHost));
        for (size_t i = 0; i < n; ++i) {
            const uint32_t b = static_cast<uint32_t>(tmp[i]);
            std::memcpy(&dst[i], &b, 4);
        }
    };
    if (logits) unpack(I.w.logits + static_cast<size_t>(index) * I.d.TV, static_cast<size_t>(I.d.TV), logits);
    if (clogits) unpack(I.w.clogits + static_cast<size_t>(index) * (NCB - 1) * I.d.CV, static_cast<size_t>(NCB - 1) * I.d.CV, clogits);
}

int Frame::sample(const Device & dev, const float * d_logits, int vocab, const Sampling & s, uint64_t seed, int frame_index,
                  int codebook, int suppress_from, int eos_id, const uint8_t * d_seen) {
    dev.make_current();
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
    int * d_out = nullptr;
    NAVI_CUDA(cudaMallocAsync(reinterpret_cast<void **>(&d_out), sizeof(int), dev.stream()));
    const size_t smem = static_cast<size_t>(navi::dev::sample_scratch_floats(vocab)) * sizeof(float);
    NAVI_CUDA(cudaFuncSetAttribute(reinterpret_cast<const void *>(&k_sample), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(smem)));
    k_sample<<<1, NCT, smem, dev.stream()>>>(d_logits, vocab, c, d_out);
    NAVI_CUDA(cudaGetLastError());
    int h = -1;
    NAVI_CUDA(cudaMemcpyAsync(&h, d_out, sizeof(int), cudaMemcpyDeviceToHost, dev.stream()));
    NAVI_CUDA(cudaFreeAsync(d_out, dev.stream()));
    NAVI_CUDA(cudaStreamSynchronize(dev.stream()));
    return h;
}

} // namespace navi::qwen3tts
