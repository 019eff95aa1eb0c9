// Kernels and host side of the streaming codec decoder (reference:
// model/qwen3tts/vocoder.hip:1-644).  decode_chunk() runs the same stage order as the
// reference (vocoder.hip:261-343); every GEMM-shaped stage is one conv::launch (tcgen05
// implicit GEMM), the rest are the small row-local kernels below.
#include "vocoder.hpp"

#include "conv.hpp"
#include "device.cuh"

#include "../../include/navi_b200.h"

#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <exception>
#include <utility>
#include <vector>

namespace navi::qwen3tts {

namespace {

using namespace navi::dev;

constexpr int NQ_MAX = 32;

// ---- row-local kernels ---------------------------------------------------------------------------

struct RvqArgs {
    const __half * first;
    const __half * rest[NQ_MAX];
    const int * codes;
    float * e;
    int n_q, vq;
};

// e[t] = [ first[c0] | sum_{q >= 1} rest_{q-1}[c_q] ]   (vocoder.hip:113-131)
__global__ void k_rvq(const RvqArgs a) {
    navi::dev::griddep_wait();
    navi::dev::griddep_launch_dependents();
    const int t = blockIdx.x;
    const int * c = a.codes + t * a.n_q;
    float * e = a.e + static_cast<std::size_t>(t) * 2 * a.vq;
    for (int i = threadIdx.x; i < a.vq; i += blockDim.x) {
        e[i] = __half2float(a.first[static_cast<std::size_t>(c[0]) * a.vq + i]);
        float v = 0.f;
        for (int q = 1; q < a.n_q; ++q) v += __half2float(a.rest[q - 1][static_cast<std::size_t>(c[q]) * a.vq + i]);
        e[a.vq + i] = v;
    }
}

__device__ __forceinline__ float block_sum256(float v, float * red) {
    v = warp_sum(v);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) t += red[k];
    return t;
}

// Finishes QKV row t and appends it to the attention ring (vocoder.hip:59-82): the row is
// the sum, in split order, of the QKV projection's `splits` split-K partial slices ([T][3 HD]
// each; the projection has no bias), or, with splits == 0, already in qkv.  blockIdx.y picks
// the part: 0 = q, rotate-half RoPE at position pos0 + t in place; 1 = k, rotated into qkv
// and ring slot pos & (ring - 1); 2 = v, into qkv and the ring slot.  blockIdx.z picks a
// group of QKV_THREADS / hd heads (hd <= QKV_THREADS), one thread per element for the
// partial loads, staged in shared memory for the rotation.
constexpr int QKV_THREADS = 256;
// Chunks of up to this many rows take k_qkv_rope_append (one launch fewer per layer: 4-frame
// chunk 0.837 -> 0.808 ms); a 16-frame chunk measured 1.080 -> 1.143 ms with it and keeps the
// separate reduction + k_rope_append.
constexpr int QKV_FUSED_ROWS = 8;
__global__ void __launch_bounds__(QKV_THREADS) k_qkv_rope_append(const float * partial, int splits, float * qkv, int nh, int hd,
                                                                 const int * pos0p, int ring, const float * inv_freq, float * kc, float * vc) {
    const int pos0 = *pos0p;
    navi::dev::griddep_wait();
    navi::dev::griddep_launch_dependents();
    __shared__ float buf[QKV_THREADS];
    const int t = blockIdx.x, part = blockIdx.y, pos = pos0 + t, slot = pos & (ring - 1);
    const int HD = nh * hd, half = hd / 2, hpc = QKV_THREADS / hd, h0 = blockIdx.z * hpc;
    const int nheads = min(hpc, nh - h0), cnt = nheads * hd;
    const std::size_t n = static_cast<std::size_t>(gridDim.x) * 3 * HD;
    const std::size_t off = static_cast<std::size_t>(part) * HD + static_cast<std::size_t>(h0) * hd;
    float * row = qkv + static_cast<std::size_t>(t) * 3 * HD + off;
    const int e = threadIdx.x;
    if (e < cnt) buf[e] = splits > 0 ? navi::dev::sum_slices(partial + static_cast<std::size_t>(t) * 3 * HD + off + e, splits, n) : row[e];
    __syncthreads();
    if (part == 2) {
        if (e < cnt) {
            row[e] = buf[e];
            vc[static_cast<std::size_t>(slot) * HD + static_cast<std::size_t>(h0) * hd + e] = buf[e];
        }
        return;
    }
    if (e < nheads * half) {
        const int h = e / half, p = e % half;
        const float ang = static_cast<float>(pos) * inv_freq[p];
        const float cs = cosf(ang), sn = sinf(ang);
        const float x0 = buf[h * hd + p], x1 = buf[h * hd + p + half];
        const float r0 = x0 * cs - x1 * sn, r1 = x1 * cs + x0 * sn;
        row[h * hd + p] = r0;
        row[h * hd + p + half] = r1;
        if (part == 1) {
            float * kd = kc + static_cast<std::size_t>(slot) * HD + static_cast<std::size_t>(h0 + h) * hd;
            kd[p] = r0;
            kd[p + half] = r1;
        }
    }
}

// Rotate-half RoPE on q (in place) and k of row t at position pos0 + t; k and v go to
// ring slot pos & (ring - 1) (vocoder.hip:59-82).  qkv rows: [q | k | v], HD each.  Chunks
// of more than QKV_FUSED_ROWS rows: after the QKV projection's own split-K reduction.
__global__ void k_rope_append(float * qkv, int nh, int hd, const int * pos0p, int ring, const float * inv_freq, float * kc, float * vc) {
    const int pos0 = *pos0p;
    navi::dev::griddep_wait();
    navi::dev::griddep_launch_dependents();
    const int t = blockIdx.x, pos = pos0 + t, slot = pos & (ring - 1);
    const int HD = nh * hd, half = hd / 2;
    float * row = qkv + static_cast<std::size_t>(t) * 3 * HD;
    for (int i = threadIdx.x; i < nh * half; i += blockDim.x) {
        const int h = i / half, p = i % half;
        const float ang = static_cast<float>(pos) * inv_freq[p];
        const float cs = cosf(ang), sn = sinf(ang);
        float * q = row + h * hd;
        float * k = row + HD + h * hd;
        const float q0 = q[p], q1 = q[p + half];
        q[p] = q0 * cs - q1 * sn;
        q[p + half] = q1 * cs + q0 * sn;
        const float k0 = k[p], k1 = k[p + half];
        const float r0 = k0 * cs - k1 * sn, r1 = k1 * cs + k0 * sn;
        k[p] = r0;
        k[p + half] = r1;
        float * kd = kc + static_cast<std::size_t>(slot) * HD + h * hd;
        kd[p] = r0;
        kd[p + half] = r1;
    }
    for (int i = threadIdx.x; i < HD; i += blockDim.x) vc[static_cast<std::size_t>(slot) * HD + i] = row[2 * HD + i];
}

// Sliding-window causal attention of row t, head h over keys (pos - window, pos]
// (vocoder.hip:85-111).  128 threads: thread j scores key k0 + j; thread i < hd sums
// output dimension i.  window <= 128, hd <= 128.
__global__ void k_window_attn(const float * qkv, int nh, int hd, const int * pos0p, int window, int ring, float scale, const float * kc,
                              const float * vc, float * out) {
    const int pos0 = *pos0p;
    navi::dev::griddep_wait();
    navi::dev::griddep_launch_dependents();
    __shared__ float q[128], pr[128], red[4];
    const int t = blockIdx.x, h = blockIdx.y, pos = pos0 + t, tid = threadIdx.x;
    const int HD = nh * hd;
    const int k0 = max(0, pos - window + 1), n = pos - k0 + 1;
    if (tid < hd) q[tid] = qkv[static_cast<std::size_t>(t) * 3 * HD + h * hd + tid];
    __syncthreads();
    float s = -INFINITY;
    if (tid < n) {
        const float * k = kc + static_cast<std::size_t>((k0 + tid) & (ring - 1)) * HD + h * hd;
        float d = 0.f;
        for (int i = 0; i < hd; ++i) d += q[i] * k[i];
        s = d * scale;
    }
    float m = warp_max(s);
    if ((tid & 31) == 0) red[tid >> 5] = m;
    __syncthreads();
    m = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    __syncthreads();
    const float e = tid < n ? expf(s - m) : 0.f;
    float z = warp_sum(e);
    if ((tid & 31) == 0) red[tid >> 5] = z;
    __syncthreads();
    z = red[0] + red[1] + red[2] + red[3];
    pr[tid] = e / z;
    __syncthreads();
    if (tid < hd) {
        float acc = 0.f;
        for (int j = 0; j < n; ++j) acc += pr[j] * vc[static_cast<std::size_t>((k0 + j) & (ring - 1)) * HD + h * hd + tid];
        out[static_cast<std::size_t>(t) * HD + h * hd + tid] = acc;
    }
}

// Next chunk's history of a k = 7 conv, the last 6 rows of [hist ; x[0..T)] (x rows of C
// floats), into hist_out, a buffer other than hist (vocoder.hip:133-141): the block that
// reads x rows [r0, r1) copies those of them that land there; block 0 also keeps the old
// history rows when T < 6.
__device__ __forceinline__ void next_hist6(const float * x, const float * hist, int T, int C, int r0, int r1, float * hist_out) {
    for (int t = max(r0, T - 6); t < min(r1, T); ++t)
        for (int c = threadIdx.x; c < C; c += blockDim.x)
            hist_out[static_cast<std::size_t>(t - (T - 6)) * C + c] = x[static_cast<std::size_t>(t) * C + c];
    if (blockIdx.x == 0)
        for (int q = 0; q < 6 - T; ++q)
            for (int c = threadIdx.x; c < C; c += blockDim.x)
                hist_out[static_cast<std::size_t>(q) * C + c] = hist[static_cast<std::size_t>(q + T) * C + c];
}

// ConvNeXt front: depthwise causal conv (k = 7, history of 6 rows) + LayerNorm over the
// channels (vocoder.hip:20-56).  256 threads per row, C <= 2048.
__global__ void k_dwconv_ln(const __half * W, const float * bias, const float * x, const float * hist, int C, const float * lw,
                            const float * lb, float eps, float * y, float * hist_out) {
    navi::dev::griddep_wait();
    navi::dev::griddep_launch_dependents();
    __shared__ float red[8];
    const int t = blockIdx.x;
    next_hist6(x, hist, gridDim.x, C, t, t + 1, hist_out);
    float v[8];
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const int ch = threadIdx.x + k * 256;
        float acc = 0.f;
        if (ch < C) {
            acc = bias[ch];
#pragma unroll
            for (int j = 0; j < 7; ++j) {
                const int tt = t - 6 + j;
                const float xv = tt >= 0 ? x[static_cast<std::size_t>(tt) * C + ch] : hist[static_cast<std::size_t>(6 + tt) * C + ch];
                acc += __half2float(W[ch * 7 + j]) * xv;
            }
        }
        v[k] = acc;
        s += acc;
    }
    const float mean = block_sum256(s, red) / static_cast<float>(C);
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const int ch = threadIdx.x + k * 256;
        if (ch < C) ss += (v[k] - mean) * (v[k] - mean);
    }
    const float inv = rsqrtf(block_sum256(ss, red) / static_cast<float>(C) + eps);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const int ch = threadIdx.x + k * 256;
        if (ch < C) y[static_cast<std::size_t>(t) * C + ch] = (v[k] - mean) * inv * lw[ch] + lb[ch];
    }
}

// Output conv: 1 channel, k = 7, SnakeBeta prologue, clamp to [-1, 1] (vocoder.hip:338-339).
// 256 rows per block; the Snake'd window [t0 - 6, t0 + 256) is staged channel-major.
constexpr int FROWS = 256;
__global__ void k_final_conv(const __half * W, const float * bias, const float * x, const float * hist, const float * sa, const float * sb,
                             int T, int Cin, float * y, float * hist_out) {
    navi::dev::griddep_wait();
    navi::dev::griddep_launch_dependents();
    extern __shared__ float fs[];
    constexpr int NR = FROWS + 6;
    float * xs = fs;                 // [Cin][NR]
    float * ws = fs + Cin * NR;      // [Cin][7]
    const int t0 = blockIdx.x * FROWS;
    next_hist6(x, hist, T, Cin, t0, t0 + FROWS, hist_out);
    constexpr int U = 8;   // loads in flight per thread
    for (int i0 = threadIdx.x; i0 < NR * Cin; i0 += FROWS * U) {
        float v[U];
#pragma unroll
        for (int k = 0; k < U; ++k) {
            const int i = i0 + k * FROWS;
            v[k] = 0.f;
            if (i < NR * Cin) {
                const int r = i / Cin, ci = i % Cin, gr = t0 - 6 + r;
                if (gr >= 0) v[k] = gr < T ? __ldg(x + static_cast<std::size_t>(gr) * Cin + ci) : 0.f;
                else v[k] = __ldg(hist + static_cast<std::size_t>(6 + gr) * Cin + ci);
            }
        }
#pragma unroll
        for (int k = 0; k < U; ++k) {
            const int i = i0 + k * FROWS;
            if (i < NR * Cin) {
                const int r = i / Cin, ci = i % Cin;
                const float s = sinf(v[k] * __ldg(sa + ci));
                xs[ci * NR + r] = v[k] + s * s * __ldg(sb + ci);
            }
        }
    }
    for (int i = threadIdx.x; i < Cin * 7; i += blockDim.x) ws[i] = __half2float(W[i]);
    __syncthreads();
    const int t = t0 + threadIdx.x;
    if (t >= T) return;
    float acc = bias[0];
    for (int ci = 0; ci < Cin; ++ci) {
#pragma unroll
        for (int j = 0; j < 7; ++j) acc += ws[ci * 7 + j] * xs[ci * NR + threadIdx.x + j];
    }
    y[t] = fminf(fmaxf(acc, -1.f), 1.f);
}

// One GEMM-shaped stage: its packed weights and fixed operands, plus its input history.
struct CV {
    conv::Conv c;
    float * hist = nullptr;   // history [H][Cin] read by the next launch
    float * hist2 = nullptr;  // the other buffer: the launch writes the next history there
    int H = 0;
};

} // namespace

struct Vocoder::Impl {
    cudaStream_t stream = nullptr;
    Params p;
    int sms = 148;
    int Cmax = 0, ring = 0, pos0 = 0, spf = 0;
    int L = 0, VH = 0, HD = 0, CD = 0, VQ = 0, DD = 0, FF = 0, nh = 0, hd = 0, window = 0;
    float eps = 0;
    std::vector<void *> owned;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    double last_ms = 0;
    StageHook hook;

    const __half * cb_first = nullptr;
    std::vector<const __half *> cb_rest;
    CV rvq_proj, pre_conv, in_proj, out_proj, dec0;
    struct Layer {
        const float * ln1 = nullptr, * ln2 = nullptr;
        CV qkv, o, gateup, down;
        float * kc = nullptr, * vc = nullptr;
    };
    std::vector<Layer> layers;
    const float * final_norm = nullptr;
    CV up_conv[2];
    struct Cnx {
        const __half * dw = nullptr;
        const float * dw_bias = nullptr, * ln_w = nullptr, * ln_b = nullptr;
        float * hist = nullptr, * hist2 = nullptr;   // history; the launch writes the next one into hist2
        CV pw1, pw2;
    } cnx[2];
    struct Block {
        CV up;
        CV c1[3], c2[3];
        int rate = 0, Cin = 0, Cout = 0;
    } blocks[4];
    struct Final {
        const __half * w = nullptr;
        const float * bias = nullptr, * sa = nullptr, * sb = nullptr;
        float * hist = nullptr, * hist2 = nullptr;   // history; the launch writes the next one into hist2
        int Cin = 0;
    } fin;
    float * inv_freq = nullptr;

    int * d_codes = nullptr;
    float * e = nullptr, * h = nullptr, * a = nullptr, * x = nullptr, * n = nullptr, * qkv = nullptr, * att = nullptr, * gu = nullptr,
          * u = nullptr, * A = nullptr, * B = nullptr, * G = nullptr, * d = nullptr, * pcm = nullptr;
    float * P[4] = {}, * Q[4] = {};
    int * h_codes = nullptr;     // pinned
    // The chunk's first position, read by the attention kernels from device memory so that a
    // chunk's launches are the same for every chunk of a length and history parity: those are
    // captured as a CUDA graph (after one eager chunk of that kind) and replayed.
    int * d_pos0 = nullptr;
    int * h_pos0 = nullptr;      // pinned
    int flip = 0;                // chunks decoded since create, mod 2 (every history pair swaps once a chunk)
    struct ChunkGraph { int T, flip; cudaGraphExec_t exec; };
    std::vector<ChunkGraph> graphs;
    std::vector<std::pair<int, int>> seen;   // (T, flip) run eagerly once
    std::vector<int> uncapturable;            // lengths whose capture the runtime refused
    void run_chunk(int T);
    void advance(int T);
    float * h_pcm = nullptr;     // pinned
    int * h_err = nullptr;       // pinned
    conv::Workspace ws;
    conv::Workspace ws_gu;   // the gate/up projections' two partial slices, read by the down projections

    template <class T> T * alloc(std::size_t n_elems) {
        void * ptr = nullptr;
        NAVI_CUDA(cudaMalloc(&ptr, std::max<std::size_t>(n_elems, 1) * sizeof(T)));
        owned.push_back(ptr);
        NAVI_CUDA(cudaMemsetAsync(ptr, 0, std::max<std::size_t>(n_elems, 1) * sizeof(T), stream));
        return static_cast<T *>(ptr);
    }
    template <class T> T * upload(const std::vector<T> & v) {
        T * ptr = alloc<T>(v.size());
        NAVI_CUDA(cudaMemcpyAsync(ptr, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice, stream));
        NAVI_CUDA(cudaStreamSynchronize(stream));
        return ptr;
    }

    void snap(const char * name, const float * buf, int rows, int cols) {
        if (!hook) return;
        NAVI_CUDA(cudaStreamSynchronize(stream));
        hook(name, buf, rows, cols);
    }

    // norm_w: also writes the rows of y RMS-normalised with these weights into norm_out
    // defer: a split-K launch leaves its partial sums in the workspace (wsp, else ws); returns
    // their slice count.  x_slices 2: xin holds the 2 partial slices of such a launch, [T][x_stride] each
    int run(CV & cv, const float * xin, int T, int x_stride, float * y, int y_stride, const float * resid = nullptr,
            const float * norm_w = nullptr, float * norm_out = nullptr, bool defer = false, const conv::Workspace * wsp = nullptr,
            int x_slices = 1) {
        conv::Conv c = cv.c;
        c.weights_settled = true;   // packed in create(), which synchronises before returning
        c.x = xin;
        c.T = T;
        c.x_stride = x_stride;
        c.hist = cv.hist;
        c.hist_out = cv.hist2;    // the conv kernel writes the next history itself
        c.y = y;
        c.y_stride = y_stride;
        c.resid = resid;
        c.r_stride = y_stride;
        c.norm_w = norm_w;
        c.norm_out = norm_out;
        c.norm_eps = eps;
        c.defer_reduce = defer;
        c.x_slices = x_slices;
        c.x_slice_stride = x_slices > 1 ? static_cast<std::size_t>(T) * x_stride : 0;
        const int splits = conv::launch(c, wsp ? *wsp : ws, sms, stream);
        std::swap(cv.hist, cv.hist2);
        return splits;
    }

    void decode_chunk(int T);
};

namespace {

const __half * f16_of(const DeviceWeights & w, const std::string & name) {
    const DeviceTensor & t = w.get(name);
    if (t.info.dtype != DType::F16) fail("vocoder: " + name + " is not f16", NAVI_E_FORMAT);
    return t.as<__half>();
}
const float * f32_of(const DeviceWeights & w, const std::string & name) {
    const DeviceTensor & t = w.get(name);
    if (t.info.dtype != DType::F32) fail("vocoder: " + name + " is not f32", NAVI_E_FORMAT);
    return t.as<float>();
}
std::vector<float> host_f32(const DeviceWeights & w, const std::string & name, cudaStream_t s) {
    const DeviceTensor & t = w.get(name);
    if (t.info.dtype != DType::F32) fail("vocoder: " + name + " is not f32", NAVI_E_FORMAT);
    std::vector<float> v(t.info.numel());
    NAVI_CUDA(cudaMemcpyAsync(v.data(), t.ptr, v.size() * sizeof(float), cudaMemcpyDeviceToHost, s));
    NAVI_CUDA(cudaStreamSynchronize(s));
    return v;
}

const std::string DEC = "codec.decoder.";

} // namespace

void Vocoder::Impl::decode_chunk(int T) {
    {
        RvqArgs ra{};
        ra.first = cb_first;
        for (std::size_t q = 0; q < cb_rest.size(); ++q) ra.rest[q] = cb_rest[q];
        ra.codes = d_codes;
        ra.e = e;
        ra.n_q = p.vq_n_q;
        ra.vq = VQ;
        NAVI_CUDA(navi::dev::launch_pdl(k_rvq, dim3(T), dim3(256), 0, stream, ra));
        NAVI_CUDA(cudaGetLastError());
    }
    run(rvq_proj, e, T, CD, h, CD);
    snap("rvq", h, T, CD);
    run(pre_conv, h, T, CD, a, L);
    snap("pre_conv", a, T, L);
    // Every RMSNorm of the transformer (kernels.h:342 at vocoder.hip:274, 285, 291) is
    // applied by the launch of the conv that writes its input row: n = norm(x).
    run(in_proj, a, T, L, x, VH, nullptr, layers.empty() ? final_norm : layers[0].ln1, n);
    const float scale = 1.f / std::sqrt(static_cast<float>(hd));
    for (std::size_t l = 0; l < layers.size(); ++l) {
        Layer & ly = layers[l];
        if (T <= QKV_FUSED_ROWS) {
            const int qs = run(ly.qkv, n, T, VH, qkv, 3 * HD, nullptr, nullptr, nullptr, true);
            const int hpc = QKV_THREADS / hd;
            NAVI_CUDA(navi::dev::launch_pdl(k_qkv_rope_append, dim3(T, 3, (nh + hpc - 1) / hpc), dim3(QKV_THREADS), 0, stream, ws.partial, qs,
                                            qkv, nh, hd, d_pos0, ring, inv_freq, ly.kc, ly.vc));
        } else {
            run(ly.qkv, n, T, VH, qkv, 3 * HD);
            NAVI_CUDA(navi::dev::launch_pdl(k_rope_append, dim3(T), dim3(256), 0, stream, qkv, nh, hd, d_pos0, ring, inv_freq, ly.kc, ly.vc));
        }
        NAVI_CUDA(navi::dev::launch_pdl(k_window_attn, dim3(T, nh), dim3(128), 0, stream, qkv, nh, hd, d_pos0, window, ring, scale, ly.kc, ly.vc, att));
        NAVI_CUDA(cudaGetLastError());
        run(ly.o, att, T, HD, x, VH, x, ly.ln2, n);
        // gate/up: a launch that splits K in two leaves both partial slices, and the down
        // projection's staging adds them (one reduction launch fewer per layer)
        conv::Conv cg = ly.gateup.c;
        cg.T = T;
        const bool fold = conv::plan(cg, sms).splits == 2;
        if (fold && run(ly.gateup, n, T, VH, gu, 2 * FF, nullptr, nullptr, nullptr, true, &ws_gu) != 2)
            fail("vocoder: the gate/up projection did not split in two", NAVI_E_SHAPE);
        if (!fold) run(ly.gateup, n, T, VH, gu, 2 * FF);
        run(ly.down, fold ? ws_gu.partial : gu, T, 2 * FF, x, VH, x, l + 1 < layers.size() ? layers[l + 1].ln1 : final_norm, n, false,
            nullptr, fold ? 2 : 1);
        snap(("layer" + std::to_string(l)).c_str(), x, T, VH);
    }
    run(out_proj, n, T, VH, u, L);
    snap("pre_transformer", u, T, L);

    int R = T;
    const float * src = u;
    for (int j = 0; j < 2; ++j) {
        float * dst = j == 0 ? A : B;
        float * tmp = j == 0 ? B : A;
        const int r = p.upsampling_ratios[static_cast<std::size_t>(j)];
        run(up_conv[j], src, R, L, dst, r * L);   // phases folded: output row t*r + phase, dense
        R *= r;
        Cnx & cx = cnx[j];
        NAVI_CUDA(navi::dev::launch_pdl(k_dwconv_ln, dim3(R), dim3(256), 0, stream, cx.dw, cx.dw_bias, dst, cx.hist, L, cx.ln_w, cx.ln_b, 1e-6f, tmp,
                                        cx.hist2));
        NAVI_CUDA(cudaGetLastError());
        std::swap(cx.hist, cx.hist2);
        run(cx.pw1, tmp, R, L, G, 4 * L);
        run(cx.pw2, G, R, 4 * L, dst, L, dst);
        snap(("up" + std::to_string(j)).c_str(), dst, R, L);
        src = dst;
    }
    run(dec0, src, R, L, d, DD);
    snap("dec0", d, R, DD);
    const float * in = d;
    int width = DD;
    for (int b = 0; b < 4; ++b) {
        Block & bk = blocks[b];
        run(bk.up, in, R, width, P[b], bk.rate * bk.Cout);
        R *= bk.rate;
        width = bk.Cout;
        for (int k = 0; k < 3; ++k) {
            run(bk.c1[k], P[b], R, width, Q[b], width);
            run(bk.c2[k], Q[b], R, width, P[b], width, P[b]);
        }
        snap(("dec" + std::to_string(b + 1)).c_str(), P[b], R, width);
        in = P[b];
    }
    const int fsmem = (FROWS + 6) * fin.Cin * 4 + fin.Cin * 7 * 4;
    NAVI_CUDA(navi::dev::launch_pdl(k_final_conv, dim3((R + FROWS - 1) / FROWS), dim3(FROWS), fsmem, stream, fin.w, fin.bias, in, fin.hist, fin.sa, fin.sb, R, fin.Cin, pcm,
                                    fin.hist2));
    NAVI_CUDA(cudaGetLastError());
    std::swap(fin.hist, fin.hist2);
    snap("pcm", pcm, R, 1);
    pos0 += T;
    flip ^= 1;
}

// Every history pair (read by a chunk's launch, its successor written by it), in one order.
template <class F> void each_hist_pair(Vocoder::Impl & I, F && f) {
    const auto cv = [&](CV & c) { f(c.hist, c.hist2); };
    cv(I.rvq_proj); cv(I.pre_conv); cv(I.in_proj);
    for (auto & ly : I.layers) { cv(ly.qkv); cv(ly.o); cv(ly.gateup); cv(ly.down); }
    cv(I.out_proj);
    for (int j = 0; j < 2; ++j) {
        cv(I.up_conv[j]);
        f(I.cnx[j].hist, I.cnx[j].hist2);
        cv(I.cnx[j].pw1); cv(I.cnx[j].pw2);
    }
    cv(I.dec0);
    for (auto & bk : I.blocks) {
        cv(bk.up);
        for (int k = 0; k < 3; ++k) { cv(bk.c1[k]); cv(bk.c2[k]); }
    }
    f(I.fin.hist, I.fin.hist2);
}

// What decode_chunk does to the host-side state (each history pair swapped once, the position
// advanced), for a chunk whose launches ran from a graph.
void Vocoder::Impl::advance(int T) {
    each_hist_pair(*this, [](float *& a, float *& b) { std::swap(a, b); });
    pos0 += T;
    flip ^= 1;
}

// One chunk of T frames: from its graph when one exists for (T, history parity); else eagerly,
// the first time, and captured the second (the capture advances the host state as an eager
// run would, and the graph's launch then runs that chunk). With a stage hook, always eagerly.
void Vocoder::Impl::run_chunk(int T) {
    if (hook) { decode_chunk(T); return; }
    for (const auto & g : graphs)
        if (g.T == T && g.flip == flip) {
            NAVI_CUDA(cudaGraphLaunch(g.exec, stream));
            advance(T);
            return;
        }
    const std::pair<int, int> key{T, flip};
    bool before = false;
    for (const auto & k : seen) before = before || k == key;
    bool refused = false;
    for (int u : uncapturable) refused = refused || u == T;
    if (!before || refused || graphs.size() >= 32) {
        if (!before) seen.push_back(key);
        decode_chunk(T);
        return;
    }
    // capture: the enqueue code runs without executing, so keep the state to fall back to
    const int f0 = flip, p0 = pos0;
    std::vector<float *> saved;
    each_hist_pair(*this, [&](float *& a, float *& b) { saved.push_back(a); saved.push_back(b); });
    cudaGraph_t g = nullptr;
    NAVI_CUDA(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
    bool enqueued = true;
    try {
        decode_chunk(T);
    } catch (const std::exception &) {
        enqueued = false;
    }
    const cudaError_t end = cudaStreamEndCapture(stream, &g);
    cudaGraphExec_t e = nullptr;
    const cudaError_t inst = (enqueued && end == cudaSuccess && g) ? cudaGraphInstantiate(&e, g, 0) : cudaErrorStreamCaptureInvalidated;
    if (g) cudaGraphDestroy(g);
    if (inst != cudaSuccess) {
        (void) cudaGetLastError();
        uncapturable.push_back(T);
        // undo what the capture did to the state, then run the chunk eagerly
        std::size_t i = 0;
        each_hist_pair(*this, [&](float *& a, float *& b) { a = saved[i++]; b = saved[i++]; });
        flip = f0;
        pos0 = p0;
        decode_chunk(T);
        return;
    }
    graphs.push_back({T, f0, e});
    NAVI_CUDA(cudaGraphLaunch(e, stream));
}

std::unique_ptr<Vocoder> Vocoder::create(const Device & dev, const DeviceWeights & w, int max_chunk_frames, int /*max_frames*/) {
    std::unique_ptr<Vocoder> v(new Vocoder());
    v->impl_ = std::make_unique<Impl>();
    Impl & I = *v->impl_;
    dev.make_current();
    I.stream = dev.stream();
    I.p = w.params();
    const Params & p = I.p;
    I.sms = dev.info().multiprocessors;
    if (max_chunk_frames < 1) fail("vocoder: max_chunk_frames must be >= 1", NAVI_E_ARG);
    I.Cmax = max_chunk_frames;
    if (p.upsampling_ratios.size() != 2 || p.upsample_rates.size() != 4) fail("vocoder: expected 2 upsampling ratios and 4 upsample rates", NAVI_E_SHAPE);
    const auto & vp = p.vocoder;
    if (vp.n_head != vp.n_kv_head) fail("vocoder: GQA not supported in the pre-transformer", NAVI_E_SHAPE);
    if (vp.head_dim > 128 || vp.head_dim % 2 || p.sliding_window > 128 || p.sliding_window < 1)
        fail("vocoder: head_dim and sliding window must be <= 128", NAVI_E_SHAPE);
    if (p.vq_n_q > NQ_MAX || p.vq_n_q < 2) fail("vocoder: unsupported number of codebooks", NAVI_E_SHAPE);
    I.L = p.vq_latent; I.VH = vp.hidden; I.nh = vp.n_head; I.hd = vp.head_dim; I.HD = I.nh * I.hd; I.CD = p.vq_codebook_dim;
    I.VQ = I.CD / 2; I.DD = p.decoder_dim; I.FF = vp.ff; I.window = p.sliding_window; I.eps = vp.rms_eps;
    if (I.L > 2048) fail("vocoder: latent width above 2048", NAVI_E_SHAPE);
    const cudaStream_t s = I.stream;

    auto pack = [&](std::vector<conv::PackSrc> srcs, int Cout, int Cin, int K) {
        __half * dst = I.alloc<__half>(conv::packed_elems(Cout, Cin, K));
        conv::pack(srcs, Cout, Cin, K, dst, s);
        return static_cast<const __half *>(dst);
    };
    auto direct = [&](const std::string & name, int co0, int co1, int ci0, int ci1, int K) {
        conv::PackSrc ps;
        ps.p = f16_of(w, name);
        ps.co0 = co0; ps.co1 = co1; ps.ci0 = ci0; ps.ci1 = ci1;
        ps.s_co = static_cast<long long>(ci1 - ci0) * K; ps.s_ci = K; ps.s_tap = 1;
        return ps;
    };
    auto make = [&](std::vector<conv::PackSrc> srcs, int Cout, int Cin, int K, int dil, const float * bias, int pro = conv::PRO_NONE,
                    int epi = conv::EPI_NONE) {
        CV cv;
        cv.c.w = pack(std::move(srcs), Cout, Cin, K);
        cv.c.Cout = Cout; cv.c.Cin = Cin; cv.c.K = K; cv.c.dil = dil; cv.c.bias = bias; cv.c.pro = pro; cv.c.epi = epi;
        cv.H = (K - 1) * dil;
        if (cv.H > 0) {
            cv.hist = I.alloc<float>(static_cast<std::size_t>(cv.H) * Cin);
            cv.hist2 = I.alloc<float>(static_cast<std::size_t>(cv.H) * Cin);
        }
        return cv;
    };
    auto snake = [&](const std::string & prefix, CV & cv) {
        const auto al = host_f32(w, prefix + ".alpha", s), be = host_f32(w, prefix + ".beta", s);
        std::vector<float> ea(al.size()), ib(be.size());
        for (std::size_t i = 0; i < al.size(); ++i) {
            ea[i] = std::exp(al[i]);
            ib[i] = 1.f / (std::exp(be[i]) + 1e-9f);
        }
        cv.c.snake_a = I.upload(ea);
        cv.c.snake_b = I.upload(ib);
        cv.c.pro = conv::PRO_SNAKE;
    };
    auto folded_bias = [&](const std::string & name, int phases) {
        const auto b = host_f32(w, name, s);
        std::vector<float> f(b.size() * phases);
        for (std::size_t i = 0; i < f.size(); ++i) f[i] = b[i % b.size()];
        return static_cast<const float *>(I.upload(f));
    };
    auto trans = [&](const std::string & name, int Cin, int Cout_b, int k, int stride) {
        conv::PackSrc ps;
        ps.p = f16_of(w, name);
        ps.co0 = 0; ps.co1 = Cout_b * stride; ps.ci0 = 0; ps.ci1 = Cin;
        ps.trans = 1; ps.cout_b = Cout_b; ps.k = k; ps.stride = stride;
        return ps;
    };

    // RVQ (vocoder.hip:264-265, 527-546): codebooks gathered by id, both output projections
    // as one GEMM over [first | rest].
    const std::string q = DEC + "quantizer.";
    I.cb_first = f16_of(w, q + "rvq_first.vq.layers.0._codebook.codebook");
    for (int i = 0; i < p.vq_n_q - p.vq_n_semantic; ++i)
        I.cb_rest.push_back(f16_of(w, q + "rvq_rest.vq.layers." + std::to_string(i) + "._codebook.codebook"));
    if (p.vq_n_semantic != 1) fail("vocoder: one semantic codebook expected", NAVI_E_SHAPE);
    I.rvq_proj = make({direct(q + "rvq_first.output_proj.weight", 0, I.CD, 0, I.VQ, 1), direct(q + "rvq_rest.output_proj.weight", 0, I.CD, I.VQ, 2 * I.VQ, 1)},
                      I.CD, I.CD, 1, 1, nullptr);
    I.pre_conv = make({direct(DEC + "pre_conv.conv.weight", 0, I.L, 0, I.CD, 3)}, I.L, I.CD, 3, 1, f32_of(w, DEC + "pre_conv.conv.bias"));
    const std::string pt = DEC + "pre_transformer.";
    I.in_proj = make({direct(pt + "input_proj.weight", 0, I.VH, 0, I.L, 1)}, I.VH, I.L, 1, 1, f32_of(w, pt + "input_proj.bias"));
    I.out_proj = make({direct(pt + "output_proj.weight", 0, I.L, 0, I.VH, 1)}, I.L, I.VH, 1, 1, f32_of(w, pt + "output_proj.bias"));
    I.final_norm = f32_of(w, pt + "norm.weight");

    I.ring = 8;
    while (I.ring < I.window + I.Cmax) I.ring *= 2;
    {
        std::vector<float> inv(static_cast<std::size_t>(I.hd / 2));
        for (int i = 0; i < I.hd / 2; ++i) inv[static_cast<std::size_t>(i)] = static_cast<float>(1.0 / std::pow(vp.rope_theta, (2.0 * i) / I.hd));
        I.inv_freq = I.upload(inv);
    }
    for (int l = 0; l < vp.n_layer; ++l) {
        const std::string lp = pt + "layers." + std::to_string(l) + ".";
        Impl::Layer ly;
        ly.ln1 = f32_of(w, lp + "input_layernorm.weight");
        ly.ln2 = f32_of(w, lp + "post_attention_layernorm.weight");
        ly.qkv = make({direct(lp + "self_attn.q_proj.weight", 0, I.HD, 0, I.VH, 1), direct(lp + "self_attn.k_proj.weight", I.HD, 2 * I.HD, 0, I.VH, 1),
                       direct(lp + "self_attn.v_proj.weight", 2 * I.HD, 3 * I.HD, 0, I.VH, 1)},
                      3 * I.HD, I.VH, 1, 1, nullptr);
        ly.o = make({direct(lp + "self_attn.o_proj.weight", 0, I.VH, 0, I.HD, 1)}, I.VH, I.HD, 1, 1, nullptr, conv::PRO_NONE, conv::EPI_SCALE_RESIDUAL);
        ly.o.c.scale = f32_of(w, lp + "self_attn_layer_scale.scale");
        ly.gateup = make({direct(lp + "mlp.gate_proj.weight", 0, I.FF, 0, I.VH, 1), direct(lp + "mlp.up_proj.weight", I.FF, 2 * I.FF, 0, I.VH, 1)},
                         2 * I.FF, I.VH, 1, 1, nullptr);
        ly.down = make({direct(lp + "mlp.down_proj.weight", 0, I.VH, 0, I.FF, 1)}, I.VH, I.FF, 1, 1, nullptr, conv::PRO_SILU_GATE,
                       conv::EPI_SCALE_RESIDUAL);
        ly.down.c.scale = f32_of(w, lp + "mlp_layer_scale.scale");
        ly.kc = I.alloc<float>(static_cast<std::size_t>(I.ring) * I.HD);
        ly.vc = I.alloc<float>(static_cast<std::size_t>(I.ring) * I.HD);
        I.layers.push_back(ly);
    }

    for (int j = 0; j < 2; ++j) {
        const int r = p.upsampling_ratios[static_cast<std::size_t>(j)];
        const std::string up = DEC + "upsample." + std::to_string(j) + ".";
        I.up_conv[j] = make({trans(up + "0.conv.weight", I.L, I.L, r, r)}, r * I.L, I.L, 1, 1, folded_bias(up + "0.conv.bias", r));
        Impl::Cnx & cx = I.cnx[j];
        cx.dw = f16_of(w, up + "1.dwconv.conv.weight");
        cx.dw_bias = f32_of(w, up + "1.dwconv.conv.bias");
        cx.ln_w = f32_of(w, up + "1.norm.weight");
        cx.ln_b = f32_of(w, up + "1.norm.bias");
        cx.hist = I.alloc<float>(static_cast<std::size_t>(6) * I.L);
        cx.hist2 = I.alloc<float>(static_cast<std::size_t>(6) * I.L);
        cx.pw1 = make({direct(up + "1.pwconv1.weight", 0, 4 * I.L, 0, I.L, 1)}, 4 * I.L, I.L, 1, 1, f32_of(w, up + "1.pwconv1.bias"),
                      conv::PRO_NONE, conv::EPI_GELU);
        cx.pw2 = make({direct(up + "1.pwconv2.weight", 0, I.L, 0, 4 * I.L, 1)}, I.L, 4 * I.L, 1, 1, f32_of(w, up + "1.pwconv2.bias"),
                      conv::PRO_NONE, conv::EPI_SCALE_RESIDUAL);
        cx.pw2.c.scale = f32_of(w, up + "1.gamma");
    }

    I.dec0 = make({direct(DEC + "decoder.0.conv.weight", 0, I.DD, 0, I.L, 7)}, I.DD, I.L, 7, 1, f32_of(w, DEC + "decoder.0.conv.bias"));
    int width = I.DD, rows = 4;
    const int dils[3] = {1, 3, 9};
    for (int b = 0; b < 4; ++b) {
        Impl::Block & bk = I.blocks[b];
        bk.rate = p.upsample_rates[static_cast<std::size_t>(b)];
        bk.Cin = width;
        bk.Cout = width / 2;
        const std::string bp = DEC + "decoder." + std::to_string(b + 1) + ".block.";
        bk.up = make({trans(bp + "1.conv.weight", bk.Cin, bk.Cout, 2 * bk.rate, bk.rate)}, bk.rate * bk.Cout, bk.Cin, 2, 1,
                     folded_bias(bp + "1.conv.bias", bk.rate));
        snake(bp + "0", bk.up);
        for (int k = 0; k < 3; ++k) {
            const std::string rp = bp + std::to_string(2 + k) + ".";
            bk.c1[k] = make({direct(rp + "conv1.conv.weight", 0, bk.Cout, 0, bk.Cout, 7)}, bk.Cout, bk.Cout, 7, dils[k], f32_of(w, rp + "conv1.conv.bias"));
            snake(rp + "act1", bk.c1[k]);
            bk.c2[k] = make({direct(rp + "conv2.conv.weight", 0, bk.Cout, 0, bk.Cout, 1)}, bk.Cout, bk.Cout, 1, 1, f32_of(w, rp + "conv2.conv.bias"),
                            conv::PRO_SNAKE, conv::EPI_RESIDUAL);
            snake(rp + "act2", bk.c2[k]);
            bk.c2[k].c.epi = conv::EPI_RESIDUAL;
        }
        rows *= bk.rate;
        I.P[b] = I.alloc<float>(static_cast<std::size_t>(rows) * I.Cmax * bk.Cout);
        I.Q[b] = I.alloc<float>(static_cast<std::size_t>(rows) * I.Cmax * bk.Cout);
        width = bk.Cout;
    }
    I.spf = rows;
    if (p.codec_upsample && rows != p.codec_upsample)
        fail("vocoder: upsample chain gives " + std::to_string(rows) + " samples/frame, config says " + std::to_string(p.codec_upsample), NAVI_E_SHAPE);
    const int n_up = 4;
    I.fin.w = f16_of(w, DEC + "decoder." + std::to_string(n_up + 2) + ".conv.weight");
    I.fin.bias = f32_of(w, DEC + "decoder." + std::to_string(n_up + 2) + ".conv.bias");
    I.fin.Cin = width;
    I.fin.hist = I.alloc<float>(static_cast<std::size_t>(6) * width);
    I.fin.hist2 = I.alloc<float>(static_cast<std::size_t>(6) * width);
    {
        CV tmp;
        snake(DEC + "decoder." + std::to_string(n_up + 1), tmp);
        I.fin.sa = tmp.c.snake_a;
        I.fin.sb = tmp.c.snake_b;
    }
    const int fsmem = (FROWS + 6) * width * 4 + width * 7 * 4;
    if (fsmem > 227 * 1024) fail("vocoder: output conv width too large", NAVI_E_SHAPE);
    NAVI_CUDA(cudaFuncSetAttribute(k_final_conv, cudaFuncAttributeMaxDynamicSharedMemorySize, fsmem));

    const std::size_t C = static_cast<std::size_t>(I.Cmax);
    I.d_codes = I.alloc<int>(C * p.vq_n_q);
    I.e = I.alloc<float>(C * I.CD); I.h = I.alloc<float>(C * I.CD); I.a = I.alloc<float>(C * I.L);
    I.x = I.alloc<float>(C * I.VH); I.n = I.alloc<float>(C * I.VH); I.qkv = I.alloc<float>(C * 3 * I.HD);
    I.att = I.alloc<float>(C * I.HD); I.gu = I.alloc<float>(C * 2 * I.FF); I.u = I.alloc<float>(C * I.L);
    I.A = I.alloc<float>(4 * C * I.L); I.B = I.alloc<float>(4 * C * I.L); I.G = I.alloc<float>(4 * C * 4 * I.L);
    I.d = I.alloc<float>(4 * C * I.DD);
    I.pcm = I.alloc<float>(C * I.spf);

    // split-K workspace: the largest any stage needs at any chunk length up to Cmax
    std::size_t part = 0;
    for (int T = 1; T <= I.Cmax; ++T) {
        auto need = [&](const CV & cv, int R) {
            conv::Conv c = cv.c;
            c.T = R;
            part = std::max(part, conv::partial_need(c, I.sms));
        };
        need(I.rvq_proj, T); need(I.pre_conv, T); need(I.in_proj, T); need(I.out_proj, T);
        for (auto & ly : I.layers) { need(ly.qkv, T); need(ly.o, T); need(ly.gateup, T); need(ly.down, T); }
        int R = T;
        for (int j = 0; j < 2; ++j) {
            need(I.up_conv[j], R);
            R *= p.upsampling_ratios[static_cast<std::size_t>(j)];
            need(I.cnx[j].pw1, R); need(I.cnx[j].pw2, R);
        }
        need(I.dec0, R);
        for (auto & bk : I.blocks) {
            need(bk.up, R);
            R *= bk.rate;
            for (int k = 0; k < 3; ++k) { need(bk.c1[k], R); need(bk.c2[k], R); }
        }
    }
    I.ws.partial = I.alloc<float>(part);
    I.ws.partial_cap = part;
    I.ws.err = I.alloc<int>(1);
    I.ws_gu = I.ws;
    I.ws_gu.partial_cap = 2ull * I.Cmax * 2 * I.FF;
    I.ws_gu.partial = I.alloc<float>(I.ws_gu.partial_cap);

    NAVI_CUDA(cudaMallocHost(&I.h_codes, C * p.vq_n_q * sizeof(int)));
    NAVI_CUDA(cudaMallocHost(&I.h_pos0, sizeof(int)));
    I.d_pos0 = I.alloc<int>(1);
    NAVI_CUDA(cudaMallocHost(&I.h_pcm, C * I.spf * sizeof(float)));
    NAVI_CUDA(cudaMallocHost(&I.h_err, sizeof(int)));
    NAVI_CUDA(cudaEventCreate(&I.ev0));
    NAVI_CUDA(cudaEventCreate(&I.ev1));
    NAVI_CUDA(cudaStreamSynchronize(s));
    v->reset();
    return v;
}

Vocoder::~Vocoder() {
    if (!impl_) return;
    Impl & I = *impl_;
    (void) cudaStreamSynchronize(I.stream);
    if (I.ev0) (void) cudaEventDestroy(I.ev0);
    if (I.ev1) (void) cudaEventDestroy(I.ev1);
    for (const auto & g : I.graphs) (void) cudaGraphExecDestroy(g.exec);
    if (I.h_codes) (void) cudaFreeHost(I.h_codes);
    if (I.h_pos0) (void) cudaFreeHost(I.h_pos0);
    if (I.h_pcm) (void) cudaFreeHost(I.h_pcm);
    if (I.h_err) (void) cudaFreeHost(I.h_err);
    for (void * ptr : I.owned) (void) cudaFree(ptr);
}

void Vocoder::reset() {
    Impl & I = *impl_;
    I.pos0 = 0;
    auto zero = [&](float * ptr, std::size_t n) {
        if (ptr) NAVI_CUDA(cudaMemsetAsync(ptr, 0, n * sizeof(float), I.stream));
    };
    auto zero_cv = [&](CV & cv) {
        zero(cv.hist, static_cast<std::size_t>(cv.H) * cv.c.Cin);
        zero(cv.hist2, static_cast<std::size_t>(cv.H) * cv.c.Cin);
    };
    zero_cv(I.pre_conv);
    zero_cv(I.dec0);
    for (auto & cx : I.cnx) {
        zero(cx.hist, static_cast<std::size_t>(6) * I.L);
        zero(cx.hist2, static_cast<std::size_t>(6) * I.L);
    }
    for (auto & bk : I.blocks) {
        zero_cv(bk.up);
        for (auto & c1 : bk.c1) zero_cv(c1);
    }
    zero(I.fin.hist, static_cast<std::size_t>(6) * I.fin.Cin);
    zero(I.fin.hist2, static_cast<std::size_t>(6) * I.fin.Cin);
    // KV rings need no clearing: attention reads only positions <= pos, all written before use.
    NAVI_CUDA(cudaStreamSynchronize(I.stream));
}

void Vocoder::decode_into(std::span<const std::int32_t> codes, int n_frames, float * out) {
    Impl & I = *impl_;
    const int nq = I.p.vq_n_q;
    if (n_frames < 0 || codes.size() < static_cast<std::size_t>(n_frames) * nq) fail("vocoder: codes shorter than n_frames x n_q", NAVI_E_ARG);
    for (std::size_t i = 0; i < static_cast<std::size_t>(n_frames) * nq; ++i)
        if (codes[i] < 0 || codes[i] >= I.p.vq_codebook_size) fail("vocoder: code id " + std::to_string(codes[i]) + " outside the codebook", NAVI_E_ARG);
    if (I.pos0 + n_frames > (1 << 30)) fail("vocoder: position counter overflow", NAVI_E_ARG);
    NAVI_CUDA(cudaEventRecord(I.ev0, I.stream));
    for (int f0 = 0; f0 < n_frames; f0 += I.Cmax) {
        const int T = std::min(I.Cmax, n_frames - f0);
        std::memcpy(I.h_codes, codes.data() + static_cast<std::size_t>(f0) * nq, static_cast<std::size_t>(T) * nq * sizeof(int));
        NAVI_CUDA(cudaMemcpyAsync(I.d_codes, I.h_codes, static_cast<std::size_t>(T) * nq * sizeof(int), cudaMemcpyHostToDevice, I.stream));
        *I.h_pos0 = I.pos0;
        NAVI_CUDA(cudaMemcpyAsync(I.d_pos0, I.h_pos0, sizeof(int), cudaMemcpyHostToDevice, I.stream));
        I.run_chunk(T);
        const std::size_t ns = static_cast<std::size_t>(T) * I.spf;
        NAVI_CUDA(cudaMemcpyAsync(I.h_pcm, I.pcm, ns * sizeof(float), cudaMemcpyDeviceToHost, I.stream));
        NAVI_CUDA(cudaMemcpyAsync(I.h_err, I.ws.err, sizeof(int), cudaMemcpyDeviceToHost, I.stream));
        NAVI_CUDA(cudaStreamSynchronize(I.stream));
        if (const int e = *I.h_err) {
            NAVI_CUDA(cudaMemsetAsync(I.ws.err, 0, sizeof(int), I.stream));
            NAVI_CUDA(cudaStreamSynchronize(I.stream));
            if (e == conv::ERR_ALIGN) fail("vocoder: a tensor-core conv's weight ring is misaligned for swizzled tiles", NAVI_E_SHAPE);
            fail("vocoder: a tensor-core conv wait passed its deadline", NAVI_E_TIMEOUT);
        }
        std::memcpy(out + static_cast<std::size_t>(f0) * I.spf, I.h_pcm, ns * sizeof(float));
    }
    NAVI_CUDA(cudaEventRecord(I.ev1, I.stream));
    NAVI_CUDA(cudaEventSynchronize(I.ev1));
    float ms = 0.f;
    NAVI_CUDA(cudaEventElapsedTime(&ms, I.ev0, I.ev1));
    I.last_ms = ms;
}

void Vocoder::decode(std::span<const std::int32_t> codes, int n_frames, std::vector<float> & pcm) {
    const std::size_t old = pcm.size();
    pcm.resize(old + static_cast<std::size_t>(std::max(n_frames, 0)) * impl_->spf);
    try {
        decode_into(codes, n_frames, pcm.data() + old);
    } catch (...) {
        pcm.resize(old);
        throw;
    }
}

void Vocoder::set_stage_hook(StageHook hook) { impl_->hook = std::move(hook); }
int Vocoder::samples_per_frame() const { return impl_->spf; }
int Vocoder::max_chunk_frames() const { return impl_->Cmax; }
double Vocoder::last_ms() const { return impl_->last_ms; }

} // namespace navi::qwen3tts
