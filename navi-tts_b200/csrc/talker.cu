// Kernels and host side of the talker prompt and prefill (reference: model/qwen3tts/talker.hip:21-399).
//
// The prefill runs the prompt rows (T <= max_prompt_tokens) through the 28 talker layers at
// positions 0..T-1. Its GEMMs (T x K times K x N, f16 weights) run on the tensor cores with
// mma.sync m16n8k16: each f32 activation enters as two f16 values, hi = f16(x) and
// lo = f16(x - hi), so the products keep about 22 bits of the activation while the weights
// stay exact f16; accumulation is f32.
#include "talker.hpp"
#include "conv.hpp"
#include "device.cuh"

#include "../../include/navi_b200.h"

#include <cuda_fp16.h>

#include <cmath>
#include <cstring>
#include <vector>

namespace navi::qwen3tts {

namespace {

using namespace navi::dev;

__device__ __forceinline__ float silu_f(float v) { return v / (1.f + expf(-v)); }

// rows[t] = f32(table[ids[t]])
__global__ void k_gather_rows(const __half * table, const int * ids, int width, float * out) {
    const __half * src = table + static_cast<size_t>(ids[blockIdx.x]) * width;
    float * dst = out + static_cast<size_t>(blockIdx.x) * width;
    for (int i = threadIdx.x; i < width; i += blockDim.x) dst[i] = __half2float(src[i]);
}

// out[t] = (ia[t] >= 0 ? A[ia[t]] : 0) + (ib[t] >= 0 ? B[ib[t]] : 0) + (t == spk_row ? spk : 0)
__global__ void k_assemble_rows(const float * A, const float * B, const float * spk, const int * ia, const int * ib, int spk_row, int width,
                                float * out) {
    const int t = blockIdx.x;
    const float * a = ia[t] >= 0 ? A + static_cast<size_t>(ia[t]) * width : nullptr;
    const float * b = ib[t] >= 0 ? B + static_cast<size_t>(ib[t]) * width : nullptr;
    float * dst = out + static_cast<size_t>(t) * width;
    for (int i = threadIdx.x; i < width; i += blockDim.x) {
        float v = 0.f;
        if (a) v += a[i];
        if (b) v += b[i];
        if (t == spk_row) v += spk[i];
        dst[i] = v;
    }
}

// out[r] = x[r] * rsqrt(mean(x[r]^2) + eps) * w; one block of 256 threads per row.
__global__ void k_rmsnorm(const float * x, const float * w, int H, float eps, float * out) {
    navi::dev::griddep_wait();
    navi::dev::griddep_launch_dependents();
    __shared__ float red[8];
    const float * xr = x + static_cast<size_t>(blockIdx.x) * H;
    float * yr = out + static_cast<size_t>(blockIdx.x) * H;
    float ss = 0.f;
    for (int i = threadIdx.x; i < H; i += blockDim.x) ss += xr[i] * xr[i];
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) tot += red[k];
    const float scale = rsqrtf(tot / static_cast<float>(H) + eps);
    for (int i = threadIdx.x; i < H; i += blockDim.x) yr[i] = xr[i] * scale * w[i];
}

// GEMM epilogues of the prefill (y = epi(x W^T + bias)); the GEMMs run on the tcgen05 conv
// kernel as K = 1 layers with the weights read in place by TMA (conv.hpp).
enum { EPI_NONE = 0, EPI_SILU = 1, EPI_RESIDUAL = 2 };

// Per row t (position pos0 + t): RMSNorm of every q and k head (head_dim 128: one warp per
// head, 4 values a lane), rotate-half RoPE with the host table's cos/sin for the position, q
// in place; then the f16 K (after RoPE) and V rows into the cache (talker.hip:43-80).
__global__ void k_qk_norm_rope(float * qkv, int row_stride, const float * q_norm, const float * k_norm, int NH, int NKV, float eps,
                               const float * rope, int pos0, __half * kcache, __half * vcache) {
    navi::dev::griddep_wait();
    navi::dev::griddep_launch_dependents();
    constexpr int HD = 128, H2 = 64;
    const int t = blockIdx.x, pos = pos0 + t, lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    float * row = qkv + static_cast<size_t>(t) * row_stride;
    const float * cs = rope + static_cast<size_t>(pos) * HD;
    for (int h = warp; h < NH + NKV; h += nw) {
        float * v = row + h * HD;   // q heads, then k heads (k follows q in the row)
        const float * w = h < NH ? q_norm : k_norm;
        float e[4], ss = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) { e[k] = v[lane + 32 * k]; ss += e[k] * e[k]; }
        ss = warp_sum(ss);
        const float scale = rsqrtf(ss / static_cast<float>(HD) + eps);
#pragma unroll
        for (int k = 0; k < 4; ++k) e[k] = e[k] * scale * w[lane + 32 * k];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int i = lane + 32 * k;
            const float c = cs[i], s = cs[H2 + i], x0 = e[k], x1 = e[k + 2];
            v[i] = x0 * c - x1 * s;
            v[i + H2] = x0 * s + x1 * c;
        }
    }
    __syncthreads();
    const int KV = NKV * HD;
    const float * kr = row + NH * HD, * vr = kr + KV;
    for (int i = threadIdx.x; i < KV; i += blockDim.x) {
        kcache[static_cast<size_t>(pos) * KV + i] = __float2half_rn(kr[i]);
        vcache[static_cast<size_t>(pos) * KV + i] = __float2half_rn(vr[i]);
    }
}

// Causal GQA attention of the prefill: block (t, h) over keys 0..pos0 + t from the f16 cache
// (talker.hip:86-117); scores in shared memory, softmax in f32.
constexpr int MAX_KEYS = 1024;
__global__ void k_prefill_attn(const float * qkv, int row_stride, const __half * kcache, const __half * vcache, int NH, int NKV, int pos0,
                               float * out) {
    navi::dev::griddep_wait();
    navi::dev::griddep_launch_dependents();
    constexpr int HD = 128;
    __shared__ float sc[MAX_KEYS];
    __shared__ float red[8];
    const int t = blockIdx.x, h = blockIdx.y, n = pos0 + t + 1, g = h / (NH / NKV), KV = NKV * HD;
    const float * q = qkv + static_cast<size_t>(t) * row_stride + h * HD;
    const float scale = rsqrtf(static_cast<float>(HD));
    float m = -INFINITY;
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
        const __half2 * kr = reinterpret_cast<const __half2 *>(kcache + static_cast<size_t>(j) * KV + g * HD);
        float d = 0.f;
        for (int i = 0; i < HD / 2; ++i) {
            const float2 kk = __half22float2(kr[i]);
            d = fmaf(q[2 * i], kk.x, d);
            d = fmaf(q[2 * i + 1], kk.y, d);
        }
        sc[j] = d * scale;
        m = fmaxf(m, sc[j]);
    }
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    float mx = -INFINITY;
    for (int k = 0; k < static_cast<int>(blockDim.x >> 5); ++k) mx = fmaxf(mx, red[k]);
    __syncthreads();
    float s = 0.f;
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
        sc[j] = expf(sc[j] - mx);
        s += sc[j];
    }
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    float tot = 0.f;
    for (int k = 0; k < static_cast<int>(blockDim.x >> 5); ++k) tot += red[k];
    for (int i = threadIdx.x; i < HD; i += blockDim.x) {
        float acc = 0.f;
        for (int j = 0; j < n; ++j) acc = fmaf(sc[j], __half2float(vcache[static_cast<size_t>(j) * KV + g * HD + i]), acc);
        out[(static_cast<size_t>(t) * NH + h) * HD + i] = acc / tot;
    }
}

// cos[hd/2] then sin[hd/2] at integer position pos: f32 angle pos * inv_freq, cos and sin in
// double, rounded (the oracle's RoPE).
void rope_rows(double theta, int head_dim, int n_pos, std::vector<float> & out) {
    const int h2 = head_dim / 2;
    out.resize(static_cast<size_t>(n_pos) * head_dim);
    for (int t = 0; t < h2; ++t) {
        const float inv = static_cast<float>(1.0 / std::pow(theta, 2.0 * t / head_dim));
        for (int p = 0; p < n_pos; ++p) {
            const float ang = static_cast<float>(p) * inv;
            out[static_cast<size_t>(p) * head_dim + t] = static_cast<float>(std::cos(static_cast<double>(ang)));
            out[static_cast<size_t>(p) * head_dim + h2 + t] = static_cast<float>(std::sin(static_cast<double>(ang)));
        }
    }
}

struct Layer {
    const float * ln1, * ln2, * qn, * kn;
    const __half * wqkv, * wo, * wgu, * wd;   // q|k|v and gate|up adjacent in the arena
};

} // namespace

struct Talker::Impl {
    int ordinal = 0;
    cudaStream_t stream = nullptr;
    Params p;
    int H = 0, Q = 0, KVD = 0, F = 0, QKV = 0, NH = 0, NKV = 0, TV = 0, TH = 0;
    int max_prompt = 0;
    std::vector<void *> owned;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    double last_ms = 0;
    const __half * text_emb = nullptr, * codec_emb = nullptr, * fc1 = nullptr, * fc2 = nullptr, * head = nullptr;
    const float * fc1_b = nullptr, * fc2_b = nullptr, * final_norm = nullptr;
    std::vector<Layer> layers;
    std::vector<uint16_t *> kptr, vptr;
    KvCache kv;
    float * rope = nullptr;   // [max_pos][HD]
    int * d_ids = nullptr, * d_cids = nullptr, * d_ia = nullptr, * d_ib = nullptr;
    float * text_rows = nullptr, * fc1_out = nullptr, * proj = nullptr, * codec_rows = nullptr, * d_spk = nullptr;
    float * pre_rows = nullptr, * trail_rows = nullptr, * tts_pad = nullptr;
    Prompt prompt;
    float * x = nullptr, * n = nullptr, * qkv = nullptr, * att = nullptr, * gu = nullptr, * hid = nullptr, * logits = nullptr;

    template <class T> T * alloc(size_t n_elems) {
        void * ptr = nullptr;
        NAVI_CUDA(cudaMalloc(&ptr, n_elems * sizeof(T)));
        NAVI_CUDA(cudaMemset(ptr, 0, n_elems * sizeof(T)));
        owned.push_back(ptr);
        return static_cast<T *>(ptr);
    }

    int sms = 148;
    conv::Workspace ws;

    static conv::Conv gemm_desc(const __half * W, const float * bias, int xs, int M, int K, int N, int ys, int epi, bool gate) {
        conv::Conv c;
        c.w_rm = W;
        c.w_ld = K;
        c.Cout = N;
        c.Cin = K;
        c.K = 1;
        c.x_stride = xs;
        c.T = M;
        c.pro = gate ? conv::PRO_SILU_GATE : conv::PRO_NONE;
        c.epi = epi == EPI_SILU ? conv::EPI_SILU : epi == EPI_RESIDUAL ? conv::EPI_RESIDUAL : conv::EPI_NONE;
        c.bias = bias;
        c.y_stride = ys;
        c.r_stride = ys;
        c.weights_settled = true;   // the weight arena was uploaded before any prefill
        return c;
    }

    // y[M][N] (row stride ys) = epi(op(x)[M][K] W[N][K]^T + bias); op = silu(gate) * up when
    // gate (x rows [gate K | up K]); EPI_RESIDUAL adds res (may alias y).  norm_w: the same
    // launch also writes the rows of y RMS-normalised with these weights into norm_out.
    void gemm(const __half * W, const float * bias, const float * in, int xs, int M, int K, int N, float * out, int ys, int epi,
              bool gate = false, const float * res = nullptr, const float * norm_w = nullptr, float * norm_out = nullptr) {
        conv::Conv c = gemm_desc(W, bias, xs, M, K, N, ys, epi, gate);
        c.x = in;
        c.y = out;
        c.resid = res;
        c.norm_w = norm_w;
        c.norm_out = norm_out;
        c.norm_eps = p.talker.rms_eps;
        conv::launch(c, ws, sms, stream);
    }
};

std::unique_ptr<Talker> Talker::create(const Device & dev, const DeviceWeights & w, int max_prompt_tokens, int max_positions) {
    std::unique_ptr<Talker> t(new Talker());
    t->impl_ = std::make_unique<Impl>();
    Impl & I = *t->impl_;
    dev.make_current();
    I.ordinal = dev.info().ordinal;
    I.stream = dev.stream();
    I.p = w.params();
    const auto & tp = I.p.talker;
    if (tp.head_dim != 128) fail("talker: the prefill kernels are built for head_dim 128", NAVI_E_SHAPE);
    if (max_prompt_tokens < 9 || max_prompt_tokens > MAX_KEYS) fail("talker: max_prompt_tokens must be in 9..1024", NAVI_E_ARG);
    if (max_positions < max_prompt_tokens) fail("talker: max_positions below max_prompt_tokens", NAVI_E_ARG);
    I.H = tp.hidden; I.NH = tp.n_head; I.NKV = tp.n_kv_head; I.Q = tp.n_head * tp.head_dim; I.KVD = tp.n_kv_head * tp.head_dim;
    I.F = tp.ff; I.QKV = I.Q + 2 * I.KVD; I.TV = tp.vocab; I.TH = I.p.text_hidden;
    I.max_prompt = max_prompt_tokens;
    auto f16p = [&](const std::string & name) { return reinterpret_cast<const __half *>(w.get(name).ptr); };
    auto f32p = [&](const std::string & name) { return w.get(name).as<float>(); };
    I.text_emb = f16p("talker.model.text_embedding.weight");
    I.codec_emb = f16p("talker.model.codec_embedding.weight");
    I.fc1 = f16p("talker.text_projection.linear_fc1.weight");
    I.fc1_b = f32p("talker.text_projection.linear_fc1.bias");
    I.fc2 = f16p("talker.text_projection.linear_fc2.weight");
    I.fc2_b = f32p("talker.text_projection.linear_fc2.bias");
    I.head = f16p("talker.codec_head.weight");
    I.final_norm = f32p("talker.model.norm.weight");
    for (int l = 0; l < tp.n_layer; ++l) {
        const std::string lp = "talker.model.layers." + std::to_string(l) + ".";
        Layer ly{};
        ly.ln1 = f32p(lp + "input_layernorm.weight");
        ly.ln2 = f32p(lp + "post_attention_layernorm.weight");
        ly.qn = f32p(lp + "self_attn.q_norm.weight");
        ly.kn = f32p(lp + "self_attn.k_norm.weight");
        ly.wqkv = f16p(lp + "self_attn.q_proj.weight");
        ly.wo = f16p(lp + "self_attn.o_proj.weight");
        ly.wgu = f16p(lp + "mlp.gate_proj.weight");
        ly.wd = f16p(lp + "mlp.down_proj.weight");
        if (f16p(lp + "self_attn.k_proj.weight") != ly.wqkv + static_cast<size_t>(I.Q) * I.H ||
            f16p(lp + "self_attn.v_proj.weight") != ly.wqkv + static_cast<size_t>(I.Q + I.KVD) * I.H ||
            f16p(lp + "mlp.up_proj.weight") != ly.wgu + static_cast<size_t>(I.F) * I.H)
            fail("talker: q/k/v or gate/up are not adjacent in the weight arena", NAVI_E_FORMAT);
        I.layers.push_back(ly);
    }
    I.kv.n_layer = tp.n_layer;
    I.kv.max_pos = max_positions;
    I.kv.kv_dim = I.KVD;
    for (int l = 0; l < tp.n_layer; ++l) {
        I.kptr.push_back(I.alloc<uint16_t>(static_cast<size_t>(max_positions) * I.KVD));
        I.vptr.push_back(I.alloc<uint16_t>(static_cast<size_t>(max_positions) * I.KVD));
    }
    I.kv.k = I.kptr.data();
    I.kv.v = I.vptr.data();
    {
        std::vector<float> tab;
        rope_rows(tp.rope_theta, tp.head_dim, max_positions, tab);
        I.rope = I.alloc<float>(tab.size());
        NAVI_CUDA(cudaMemcpy(I.rope, tab.data(), tab.size() * sizeof(float), cudaMemcpyHostToDevice));
    }
    const size_t M = static_cast<size_t>(max_prompt_tokens) + 8;
    I.d_ids = I.alloc<int>(M); I.d_cids = I.alloc<int>(16); I.d_ia = I.alloc<int>(M); I.d_ib = I.alloc<int>(M);
    I.text_rows = I.alloc<float>(M * I.TH); I.fc1_out = I.alloc<float>(M * I.TH); I.proj = I.alloc<float>(M * I.H);
    I.codec_rows = I.alloc<float>(16 * I.H); I.d_spk = I.alloc<float>(I.H);
    I.pre_rows = I.alloc<float>(M * I.H); I.trail_rows = I.alloc<float>(M * I.H); I.tts_pad = I.alloc<float>(I.H);
    I.x = I.alloc<float>(M * I.H); I.n = I.alloc<float>(M * I.H); I.qkv = I.alloc<float>(M * I.QKV);
    I.att = I.alloc<float>(M * I.Q); I.gu = I.alloc<float>(M * 2 * I.F);
    I.hid = I.alloc<float>(I.H); I.logits = I.alloc<float>(I.TV);
    // split-K workspace of the tensor-core GEMMs: the most any of them needs at any row count
    I.sms = dev.info().multiprocessors;
    {
        std::size_t part = 0;
        const struct { int K, N, xs; bool gate; } shapes[] = {{I.TH, I.TH, I.TH, false}, {I.TH, I.H, I.TH, false}, {I.H, I.QKV, I.H, false},
                                                             {I.Q, I.H, I.Q, false}, {I.H, 2 * I.F, I.H, false}, {I.F, I.H, 2 * I.F, true},
                                                             {I.H, I.TV, I.H, false}};
        for (int m = 1; m <= max_prompt_tokens + 8; ++m)
            for (const auto & g : shapes) part = std::max(part, conv::partial_need(Impl::gemm_desc(nullptr, nullptr, g.xs, m, g.K, g.N, g.N, EPI_NONE, g.gate), I.sms));
        I.ws.partial = I.alloc<float>(std::max<std::size_t>(part, 1));
        I.ws.partial_cap = part;
        I.ws.err = I.alloc<int>(1);
    }
    NAVI_CUDA(cudaEventCreate(&I.ev0));
    NAVI_CUDA(cudaEventCreate(&I.ev1));
    return t;
}

Talker::~Talker() {
    if (!impl_) return;
    cudaSetDevice(impl_->ordinal);
    if (impl_->ev0) cudaEventDestroy(impl_->ev0);
    if (impl_->ev1) cudaEventDestroy(impl_->ev1);
    for (void * ptr : impl_->owned) cudaFree(ptr);
}

const Prompt & Talker::build_prompt(std::span<const std::int32_t> ids, const std::string & language, std::span<const float> speaker) {
    Impl & I = *impl_;
    const Params & p = I.p;
    NAVI_CUDA(cudaSetDevice(I.ordinal));
    if (ids.size() < 9) fail("talker: prompt ids too short (need role header, text, and the trailer)", NAVI_E_ARG);
    if (static_cast<int>(ids.size()) > I.max_prompt) fail("talker: prompt longer than max_prompt_tokens", NAVI_E_ARG);
    if (static_cast<int>(speaker.size()) != I.H) fail("talker: speaker embedding must be [hidden]", NAVI_E_ARG);
    for (const int32_t id : ids)
        if (id < 0 || id >= p.text_vocab) fail("talker: token id out of the text vocabulary", NAVI_E_ARG);
    const int n_text = static_cast<int>(ids.size()) - 8;
    std::vector<int> tids(ids.begin(), ids.begin() + 3 + n_text);
    const int i_bos = static_cast<int>(tids.size()); tids.push_back(p.tts_bos_id);
    const int i_eos = static_cast<int>(tids.size()); tids.push_back(p.tts_eos_id);
    const int i_pad = static_cast<int>(tids.size()); tids.push_back(p.tts_pad_id);
    const int n_rows = static_cast<int>(tids.size());
    std::vector<int> cids;
    if (language.empty() || language == "auto") {
        cids = {p.codec_nothink_id, p.codec_think_bos_id, p.codec_think_eos_id};
    } else {
        const auto it = p.language_ids.find(language);
        if (it == p.language_ids.end()) fail("talker: unknown language '" + language + "'", NAVI_E_ARG);
        cids = {p.codec_think_id, p.codec_think_bos_id, it->second, p.codec_think_eos_id};
    }
    const int n_think = static_cast<int>(cids.size());
    cids.push_back(p.codec_pad_id);
    cids.push_back(p.codec_bos_id);
    // prefill rows: header, think rows (+ tts_pad), speaker (+ tts_pad), codec_pad (+ tts_bos),
    // codec_bos (+ the first text row); trailing rows: the other text rows, then tts_eos
    std::vector<int> ia, ib;
    for (int r = 0; r < 3; ++r) { ia.push_back(r); ib.push_back(-1); }
    for (int r = 0; r < n_think; ++r) { ia.push_back(i_pad); ib.push_back(r); }
    const int spk_row = static_cast<int>(ia.size());
    ia.push_back(i_pad); ib.push_back(-1);
    ia.push_back(i_bos); ib.push_back(n_think);
    ia.push_back(3); ib.push_back(n_think + 1);
    const int n_prefill = static_cast<int>(ia.size());
    for (int r = 1; r < n_text; ++r) { ia.push_back(3 + r); ib.push_back(-1); }
    ia.push_back(i_eos); ib.push_back(-1);
    const int n_trailing = static_cast<int>(ia.size()) - n_prefill;

    NAVI_CUDA(cudaMemcpyAsync(I.d_ids, tids.data(), tids.size() * sizeof(int), cudaMemcpyHostToDevice, I.stream));
    NAVI_CUDA(cudaMemcpyAsync(I.d_cids, cids.data(), cids.size() * sizeof(int), cudaMemcpyHostToDevice, I.stream));
    NAVI_CUDA(cudaMemcpyAsync(I.d_spk, speaker.data(), I.H * sizeof(float), cudaMemcpyHostToDevice, I.stream));
    NAVI_CUDA(cudaMemcpyAsync(I.d_ia, ia.data(), ia.size() * sizeof(int), cudaMemcpyHostToDevice, I.stream));
    NAVI_CUDA(cudaMemcpyAsync(I.d_ib, ib.data(), ib.size() * sizeof(int), cudaMemcpyHostToDevice, I.stream));
    k_gather_rows<<<n_rows, 256, 0, I.stream>>>(I.text_emb, I.d_ids, I.TH, I.text_rows);
    NAVI_CUDA(cudaGetLastError());
    I.gemm(I.fc1, I.fc1_b, I.text_rows, I.TH, n_rows, I.TH, I.TH, I.fc1_out, I.TH, EPI_SILU);
    I.gemm(I.fc2, I.fc2_b, I.fc1_out, I.TH, n_rows, I.TH, I.H, I.proj, I.H, EPI_NONE);
    k_gather_rows<<<static_cast<unsigned>(cids.size()), 256, 0, I.stream>>>(I.codec_emb, I.d_cids, I.H, I.codec_rows);
    k_assemble_rows<<<n_prefill, 256, 0, I.stream>>>(I.proj, I.codec_rows, I.d_spk, I.d_ia, I.d_ib, spk_row, I.H, I.pre_rows);
    k_assemble_rows<<<n_trailing, 256, 0, I.stream>>>(I.proj, I.codec_rows, I.d_spk, I.d_ia + n_prefill, I.d_ib + n_prefill, -1, I.H,
                                                       I.trail_rows);
    NAVI_CUDA(cudaMemcpyAsync(I.tts_pad, I.proj + static_cast<size_t>(i_pad) * I.H, I.H * sizeof(float), cudaMemcpyDeviceToDevice,
                              I.stream));
    NAVI_CUDA(cudaGetLastError());
    // the host vectors above must outlive the copies
    NAVI_CUDA(cudaStreamSynchronize(I.stream));
    I.prompt.prefill = I.pre_rows;
    I.prompt.trailing = I.trail_rows;
    I.prompt.tts_pad = I.tts_pad;
    I.prompt.n_prefill = n_prefill;
    I.prompt.n_trailing = n_trailing;
    return I.prompt;
}

void Talker::prefill(const Prompt & pr) {
    Impl & I = *impl_;
    const auto & tp = I.p.talker;
    NAVI_CUDA(cudaSetDevice(I.ordinal));
    const int T = pr.n_prefill, H = I.H;
    if (T < 1 || T > I.max_prompt) fail("talker: prefill rows outside 1..max_prompt_tokens", NAVI_E_ARG);
    if (T > I.kv.max_pos) fail("talker: prompt exceeds the KV cache", NAVI_E_KV_FULL);
    NAVI_CUDA(cudaEventRecord(I.ev0, I.stream));
    NAVI_CUDA(cudaMemcpyAsync(I.x, pr.prefill, static_cast<size_t>(T) * H * sizeof(float), cudaMemcpyDeviceToDevice, I.stream));
    for (int l = 0; l < tp.n_layer; ++l) {
        const Layer & ly = I.layers[static_cast<size_t>(l)];
        __half * kc = reinterpret_cast<__half *>(I.kptr[static_cast<size_t>(l)]);
        __half * vc = reinterpret_cast<__half *>(I.vptr[static_cast<size_t>(l)]);
        if (l == 0) NAVI_CUDA(navi::dev::launch_pdl(k_rmsnorm, dim3(T), dim3(256), 0, I.stream, I.x, ly.ln1, H, tp.rms_eps, I.n));
        I.gemm(ly.wqkv, nullptr, I.n, H, T, H, I.QKV, I.qkv, I.QKV, EPI_NONE);
        NAVI_CUDA(navi::dev::launch_pdl(k_qk_norm_rope, dim3(T), dim3(256), 0, I.stream, I.qkv, I.QKV, ly.qn, ly.kn, I.NH, I.NKV, tp.rms_eps,
                                        I.rope, 0, kc, vc));
        NAVI_CUDA(navi::dev::launch_pdl(k_prefill_attn, dim3(T, I.NH), dim3(128), 0, I.stream, I.qkv, I.QKV, kc, vc, I.NH, I.NKV, 0, I.att));
        // the RMSNorms after the O projection and (but for the last layer) after the down
        // projection are written by those GEMMs' launches
        I.gemm(ly.wo, nullptr, I.att, I.Q, T, I.Q, H, I.x, H, EPI_RESIDUAL, false, I.x, ly.ln2, I.n);
        I.gemm(ly.wgu, nullptr, I.n, H, T, H, 2 * I.F, I.gu, 2 * I.F, EPI_NONE);
        const bool last = l + 1 == tp.n_layer;
        I.gemm(ly.wd, nullptr, I.gu, 2 * I.F, T, I.F, H, I.x, H, EPI_RESIDUAL, true, I.x, last ? nullptr : I.layers[static_cast<size_t>(l + 1)].ln1,
               last ? nullptr : I.n);
    }
    // the last row: final norm and the codec head
    NAVI_CUDA(navi::dev::launch_pdl(k_rmsnorm, dim3(1), dim3(256), 0, I.stream, I.x + static_cast<size_t>(T - 1) * H, I.final_norm, H,
                                    tp.rms_eps, I.hid));
    I.gemm(I.head, nullptr, I.hid, H, 1, H, I.TV, I.logits, I.TV, EPI_NONE);
    NAVI_CUDA(cudaGetLastError());
    NAVI_CUDA(cudaEventRecord(I.ev1, I.stream));
    NAVI_CUDA(cudaEventSynchronize(I.ev1));
    float ms = 0.f;
    NAVI_CUDA(cudaEventElapsedTime(&ms, I.ev0, I.ev1));
    I.last_ms = ms;
    int err = 0;
    NAVI_CUDA(cudaMemcpy(&err, I.ws.err, sizeof(int), cudaMemcpyDeviceToHost));
    if (err) {
        NAVI_CUDA(cudaMemset(I.ws.err, 0, sizeof(int)));
        if (err == conv::ERR_ALIGN) fail("talker: a tensor-core GEMM's weight ring is misaligned for swizzled tiles", NAVI_E_SHAPE);
        fail("talker: a tensor-core GEMM wait passed its deadline", NAVI_E_TIMEOUT);
    }
    I.kv.n_used = T;
}

KvCache & Talker::kv() { return impl_->kv; }
const float * Talker::d_hidden() const { return impl_->hid; }
const float * Talker::d_logits() const { return impl_->logits; }
double Talker::last_ms() const { return impl_->last_ms; }

} // namespace navi::qwen3tts
