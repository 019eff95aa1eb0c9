// Kernels and host side of the talker prompt and prefill (reference: model/qwen3tts/talker.hip:21-399).
//
// The prefill runs the prompt rows (T <= max_prompt_tokens) through the 28 talker layers at
// positions 0..T-1. Its GEMMs (T x K times K x N, f16 weights) run on the tcgen05 conv kernel
// (conv.hpp) and its causal attention on mma.sync tiles (k_prefill_attn_mma); in both, each
// f32 operand enters as two f16 values, hi = f16(x) and lo = f16(x - hi), so the products keep
// about 22 bits of it while the f16 weights and cache rows stay exact; accumulation is f32.
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

// The QKV projection's split-K sum with the per-head q/k RMSNorm, RoPE and the KV-cache store
// (talker.hip:43-80), one launch a layer: CTA (t, h) of 128 threads finishes head h of row t,
// the NH q heads, then the NKV k heads, then the NKV v heads, a thread per dimension. The head is the sum, in split order, of the projection's
// `splits` partial slices ([T][QKV] each, no bias), or, with splits == 0, already in qkv. q
// and k heads take the RMSNorm (sum of squares: lane l adds dims l, l+32, l+64, l+96, then a
// warp sum) and the rotate-half RoPE (pairs (i, i + 64), host cos/sin table) back into qkv;
// k and v heads also go to the f16 cache rows at position pos0 + t.
__global__ void __launch_bounds__(128) k_qkv_reduce_norm_rope(const float * partial, int splits, float * qkv, int row_stride,
                                                             const float * q_norm, const float * k_norm, int NH, int NKV, float eps,
                                                             const float * rope, int pos0, __half * kcache, __half * vcache) {
    navi::dev::griddep_wait();
    navi::dev::griddep_launch_dependents();
    constexpr int HD = 128, H2 = 64;
    __shared__ float buf[HD];
    __shared__ float sc;
    const int t = blockIdx.x, h = blockIdx.y, e = threadIdx.x, pos = pos0 + t;
    const size_t at = static_cast<size_t>(t) * row_stride + static_cast<size_t>(h) * HD + e;
    const float v = splits > 0 ? sum_slices(partial + at, splits, static_cast<size_t>(gridDim.x) * row_stride) : qkv[at];
    const int KV = NKV * HD;
    if (h >= NH + NKV) {   // v head
        qkv[at] = v;
        vcache[static_cast<size_t>(pos) * KV + static_cast<size_t>(h - NH - NKV) * HD + e] = __float2half_rn(v);
        return;
    }
    buf[e] = v;
    __syncthreads();
    if (e < 32) {
        float ss = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) ss += buf[e + 32 * k] * buf[e + 32 * k];
        ss = warp_sum(ss);
        if (e == 0) sc = rsqrtf(ss / static_cast<float>(HD) + eps);
    }
    __syncthreads();
    const float x = v * sc * (h < NH ? q_norm : k_norm)[e];
    buf[e] = x;
    __syncthreads();
    const float * cs = rope + static_cast<size_t>(pos) * HD;
    const int i = e & (H2 - 1);
    const float c = cs[i], sn = cs[H2 + i], x0 = buf[i], x1 = buf[i + H2];
    const float r = e < H2 ? x0 * c - x1 * sn : x0 * sn + x1 * c;
    qkv[at] = r;
    if (h >= NH) kcache[static_cast<size_t>(pos) * KV + static_cast<size_t>(h - NH) * HD + e] = __float2half_rn(r);
}

// ---- causal GQA attention of the prefill on the tensor cores ----------------------------------
//
// What it computes is the reference's k_prefill_attention (talker.hip:84-117): for row t at
// position pos0 + t and query head h, softmax(q K^T / sqrt(128)) V over the cached keys
// 0..pos0 + t of KV head h / (NH / NKV), with K (after RoPE) and V as f16 cache rows.
//
// How: flash-attention tiles. A CTA takes 64 query rows of one head (4 warps x 16 rows) and
// walks the key range in tiles of 64 keys, double-buffered in shared memory by cp.async.
// Scores and P.V run as mma.sync m16n8k16 (f16 operands, f32 accumulators) with an online
// softmax in registers, so the key count has no cap. The f32 operands enter as two f16
// halves: q = hi + lo against the exact f16 K rows, and p = hi + lo against the exact f16 V
// rows, which keeps about 22 bits of q and p; softmax, the running max and sum stay f32.
// Shared-memory rows are 256 bytes (128 f16), stored with their 16-byte chunks XOR-swizzled
// by (row & 7) so the ldmatrix row gathers hit eight different bank groups.
constexpr int PA_HD = 128;          // head_dim the kernel is built for
constexpr int PA_QT = 64;           // query rows per CTA
constexpr int PA_KT = 64;           // keys per tile
constexpr int PA_WARPS = PA_QT / 16;
constexpr int PA_THREADS = PA_WARPS * 32;
constexpr uint32_t PA_ROW = PA_HD * 2;                                   // bytes per f16 row
constexpr uint32_t PA_TILE = PA_KT * PA_ROW;                             // one K or V tile
constexpr uint32_t PA_SMEM = 2 * PA_QT * PA_ROW + 2 * 2 * PA_TILE;       // q hi, q lo; 2 x (K, V)

__device__ __forceinline__ uint32_t pa_swz(int row, int chunk) { return static_cast<uint32_t>(row) * PA_ROW + ((chunk ^ (row & 7)) << 4); }

__device__ __forceinline__ void pa_ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void pa_ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
// c (16x8 f32) += a (16x16 f16, row) * b (16x8 f16, col)
__device__ __forceinline__ void pa_mma(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pa_pack(float lo_elem, float hi_elem) {
    const __half2 h = __floats2half2_rn(lo_elem, hi_elem);
    return *reinterpret_cast<const uint32_t *>(&h);
}
// f32 pair -> (f16 hi pair, f16 lo pair) with v = hi + lo to about 22 bits
__device__ __forceinline__ void pa_split(float a, float b, uint32_t & hi, uint32_t & lo) {
    const float ha = __half2float(__float2half_rn(a)), hb = __half2float(__float2half_rn(b));
    hi = pa_pack(ha, hb);
    lo = pa_pack(a - ha, b - hb);
}

// K and V rows [k0, k0 + PA_KT) of KV head g into one buffer pair (rows past n_keys: zeros).
__device__ __forceinline__ void pa_load_kv(uint8_t * kbuf, uint8_t * vbuf, const __half * kc, const __half * vc, int KV, int g, int k0,
                                           int n_keys) {
    for (int i = threadIdx.x; i < PA_KT * 16; i += PA_THREADS) {
        const int r = i >> 4, c = i & 15, key = k0 + r;
        const uint32_t o = pa_swz(r, c);
        if (key < n_keys) {
            const size_t src = static_cast<size_t>(key) * KV + g * PA_HD + c * 8;
            cp_async16(kbuf + o, kc + src);
            cp_async16(vbuf + o, vc + src);
        } else {
            *reinterpret_cast<uint4 *>(kbuf + o) = make_uint4(0, 0, 0, 0);
            *reinterpret_cast<uint4 *>(vbuf + o) = make_uint4(0, 0, 0, 0);
        }
    }
    cp_async_commit();
}

__global__ void __launch_bounds__(PA_THREADS) k_prefill_attn_mma(const float * qkv, int row_stride, const __half * kcache,
                                                                  const __half * vcache, int T, int NH, int NKV, int pos0, float * out) {
    navi::dev::griddep_wait();
    navi::dev::griddep_launch_dependents();
    extern __shared__ __align__(128) uint8_t pa_smem[];
    uint8_t * qhi = pa_smem;
    uint8_t * qlo = qhi + PA_QT * PA_ROW;
    uint8_t * kvb = qlo + PA_QT * PA_ROW;   // [2][K tile, V tile]
    const int h = blockIdx.y, g = h / (NH / NKV), KV = NKV * PA_HD;
    const int t0 = blockIdx.x * PA_QT, rows = min(PA_QT, T - t0);
    const int n_keys = pos0 + t0 + rows;   // keys any row of this CTA sees
    const int n_tiles = (n_keys + PA_KT - 1) / PA_KT;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gq = lane >> 2, tq = lane & 3;

    pa_load_kv(kvb, kvb + PA_TILE, kcache, vcache, KV, g, 0, n_keys);
    // this CTA's query rows as f16 hi / lo (rows past T: zeros)
    for (int i = threadIdx.x; i < PA_QT * 16; i += PA_THREADS) {
        const int r = i >> 4, c = i & 15;
        uint4 hv = make_uint4(0, 0, 0, 0), lv = make_uint4(0, 0, 0, 0);
        if (r < rows) {
            const float * q = qkv + static_cast<size_t>(t0 + r) * row_stride + h * PA_HD + c * 8;
            const float4 a = *reinterpret_cast<const float4 *>(q), b = *reinterpret_cast<const float4 *>(q + 4);
            pa_split(a.x, a.y, hv.x, lv.x);
            pa_split(a.z, a.w, hv.y, lv.y);
            pa_split(b.x, b.y, hv.z, lv.z);
            pa_split(b.z, b.w, hv.w, lv.w);
        }
        *reinterpret_cast<uint4 *>(qhi + pa_swz(r, c)) = hv;
        *reinterpret_cast<uint4 *>(qlo + pa_swz(r, c)) = lv;
    }

    const float scale = rsqrtf(static_cast<float>(PA_HD));
    const int qrow0 = warp * 16;                       // this warp's rows within the tile
    const int pos_a = pos0 + t0 + qrow0 + gq;          // positions of this thread's two rows
    const int pos_b = pos_a + 8;
    float o[16][4];
#pragma unroll
    for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
    const uint32_t sq_hi = smem_addr(qhi), sq_lo = smem_addr(qlo);

    for (int kt = 0; kt < n_tiles; ++kt) {
        const int buf = kt & 1;
        if (kt + 1 < n_tiles) {
            uint8_t * nb = kvb + (buf ^ 1) * 2 * PA_TILE;
            pa_load_kv(nb, nb + PA_TILE, kcache, vcache, KV, g, (kt + 1) * PA_KT, n_keys);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const uint32_t sk = smem_addr(kvb + buf * 2 * PA_TILE), sv = sk + PA_TILE;
        const int k0 = kt * PA_KT;
        // S = q K^T for this warp's 16 rows and the tile's 64 keys
        float s[8][4];
#pragma unroll
        for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
        for (int ks = 0; ks < PA_HD / 16; ++ks) {
            uint32_t ah[4], al[4];
            const int ar = qrow0 + (lane & 7) + ((lane >> 3) & 1) * 8, ac = ks * 2 + (lane >> 4);
            pa_ldsm_x4(ah, sq_hi + pa_swz(ar, ac));
            pa_ldsm_x4(al, sq_lo + pa_swz(ar, ac));
#pragma unroll
            for (int np = 0; np < 4; ++np) {   // key n-tiles 2np, 2np + 1
                uint32_t b[4];
                const int kr = np * 16 + (lane & 7) + (lane >> 4) * 8, kc = ks * 2 + ((lane >> 3) & 1);
                pa_ldsm_x4(b, sk + pa_swz(kr, kc));
                pa_mma(s[2 * np], ah, b[0], b[1]);
                pa_mma(s[2 * np], al, b[0], b[1]);
                pa_mma(s[2 * np + 1], ah, b[2], b[3]);
                pa_mma(s[2 * np + 1], al, b[2], b[3]);
            }
        }
        // scale, causal mask, online softmax (rows gq and gq + 8 of the warp)
        float mx_a = m_a, mx_b = m_b;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int key = k0 + j * 8 + 2 * tq;
            s[j][0] = key <= pos_a ? s[j][0] * scale : -INFINITY;
            s[j][1] = key + 1 <= pos_a ? s[j][1] * scale : -INFINITY;
            s[j][2] = key <= pos_b ? s[j][2] * scale : -INFINITY;
            s[j][3] = key + 1 <= pos_b ? s[j][3] * scale : -INFINITY;
            mx_a = fmaxf(mx_a, fmaxf(s[j][0], s[j][1]));
            mx_b = fmaxf(mx_b, fmaxf(s[j][2], s[j][3]));
        }
#pragma unroll
        for (int off = 1; off < 4; off <<= 1) {
            mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, off));
            mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, off));
        }
        // key 0 is in the first tile and every row sees it, so the maxima are finite here
        const float al_a = expf(m_a - mx_a), al_b = expf(m_b - mx_b);
        m_a = mx_a;
        m_b = mx_b;
        l_a *= al_a;
        l_b *= al_b;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            o[j][0] *= al_a; o[j][1] *= al_a;
            o[j][2] *= al_b; o[j][3] *= al_b;
        }
        uint32_t ph[4][4], pl[4][4];   // P as the A operand of P.V, per 16-key step
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float p0 = expf(s[j][0] - m_a), p1 = expf(s[j][1] - m_a);
            const float p2 = expf(s[j][2] - m_b), p3 = expf(s[j][3] - m_b);
            l_a += p0 + p1;
            l_b += p2 + p3;
            const int st = j >> 1, hi_half = (j & 1) * 2;   // n-tile 2st -> a0/a1, 2st + 1 -> a2/a3
            pa_split(p0, p1, ph[st][hi_half], pl[st][hi_half]);
            pa_split(p2, p3, ph[st][hi_half + 1], pl[st][hi_half + 1]);
        }
        // O += P V over the tile's 4 key steps and the 16 dim n-tiles
#pragma unroll
        for (int st = 0; st < 4; ++st) {
#pragma unroll
            for (int dp = 0; dp < 8; ++dp) {   // dim n-tiles 2dp, 2dp + 1
                uint32_t b[4];
                const int vr = st * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, vc = dp * 2 + (lane >> 4);
                pa_ldsm_x4_t(b, sv + pa_swz(vr, vc));
                pa_mma(o[2 * dp], ph[st], b[0], b[1]);
                pa_mma(o[2 * dp], pl[st], b[0], b[1]);
                pa_mma(o[2 * dp + 1], ph[st], b[2], b[3]);
                pa_mma(o[2 * dp + 1], pl[st], b[2], b[3]);
            }
        }
        __syncthreads();   // the buffer is refilled two tiles on
    }
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
        l_a += __shfl_xor_sync(0xffffffffu, l_a, off);
        l_b += __shfl_xor_sync(0xffffffffu, l_b, off);
    }
    const float inv_a = 1.f / l_a, inv_b = 1.f / l_b;
    const int ra = t0 + qrow0 + gq, rb = ra + 8;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const int d = j * 8 + 2 * tq;
        if (ra < T) *reinterpret_cast<float2 *>(out + (static_cast<size_t>(ra) * NH + h) * PA_HD + d) = make_float2(o[j][0] * inv_a, o[j][1] * inv_a);
        if (rb < T) *reinterpret_cast<float2 *>(out + (static_cast<size_t>(rb) * NH + h) * PA_HD + d) = make_float2(o[j][2] * inv_b, o[j][3] * inv_b);
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
    // the gate/up projection's two split-K partial slices when the down projection sums them
    // (ws_gu.partial, 2 x rows x 2 ff), for prompts of up to GU_FOLD_ROWS rows
    static constexpr int GU_FOLD_ROWS = 64;
    conv::Workspace ws_gu;

    // The prefill's launches for one prompt length, captured as a CUDA graph after the first
    // (eager) prefill of that length: about 280 launches with their host-side planning and
    // tensor-map encoding replay as one graph launch. The launches read and write only this
    // object's buffers, so a graph stays valid for its lifetime.
    std::vector<std::pair<int, cudaGraphExec_t>> graphs;
    std::vector<int> uncapturable;
    void enqueue_prefill(int T);
    void capture_prefill(int T);

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
    // defer: a split-K launch leaves its partial sums in ws.partial for the caller's own
    // reduction; returns their slice count (0: out is final)
    int gemm(const __half * W, const float * bias, const float * in, int xs, int M, int K, int N, float * out, int ys, int epi,
             bool gate = false, const float * res = nullptr, const float * norm_w = nullptr, float * norm_out = nullptr, bool defer = false) {
        conv::Conv c = gemm_desc(W, bias, xs, M, K, N, ys, epi, gate);
        c.x = in;
        c.y = out;
        c.resid = res;
        c.norm_w = norm_w;
        c.norm_out = norm_out;
        c.norm_eps = p.talker.rms_eps;
        c.defer_reduce = defer;
        return conv::launch(c, ws, sms, stream);
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
    if (max_prompt_tokens < 9) fail("talker: max_prompt_tokens must be at least 9", NAVI_E_ARG);
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
        I.ws_gu = I.ws;
        I.ws_gu.partial_cap = 2ull * Impl::GU_FOLD_ROWS * 2 * I.F;
        I.ws_gu.partial = I.alloc<float>(I.ws_gu.partial_cap);
    }
    NAVI_CUDA(cudaFuncSetAttribute(reinterpret_cast<const void *>(&k_prefill_attn_mma), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(PA_SMEM)));
    NAVI_CUDA(cudaEventCreate(&I.ev0));
    NAVI_CUDA(cudaEventCreate(&I.ev1));
    return t;
}

Talker::~Talker() {
    if (!impl_) return;
    cudaSetDevice(impl_->ordinal);
    if (impl_->ev0) cudaEventDestroy(impl_->ev0);
    if (impl_->ev1) cudaEventDestroy(impl_->ev1);
    for (const auto & g : impl_->graphs) cudaGraphExecDestroy(g.second);
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
    NAVI_CUDA(cudaSetDevice(I.ordinal));
    const int T = pr.n_prefill, H = I.H;
    if (T < 1 || T > I.max_prompt) fail("talker: prefill rows outside 1..max_prompt_tokens", NAVI_E_ARG);
    if (T > I.kv.max_pos) fail("talker: prompt exceeds the KV cache", NAVI_E_KV_FULL);
    NAVI_CUDA(cudaEventRecord(I.ev0, I.stream));
    NAVI_CUDA(cudaMemcpyAsync(I.x, pr.prefill, static_cast<size_t>(T) * H * sizeof(float), cudaMemcpyDeviceToDevice, I.stream));
    cudaGraphExec_t ge = nullptr;
    for (const auto & g : I.graphs)
        if (g.first == T) ge = g.second;
    if (ge) NAVI_CUDA(cudaGraphLaunch(ge, I.stream));
    else I.enqueue_prefill(T);
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
    if (!ge) I.capture_prefill(T);
}

// The 28 layers and the codec head over the T rows in x (the layer loop of prefill).
void Talker::Impl::enqueue_prefill(int T) {
    Impl & I = *this;
    const auto & tp = I.p.talker;
    const int H = I.H;
    for (int l = 0; l < tp.n_layer; ++l) {
        const Layer & ly = I.layers[static_cast<size_t>(l)];
        __half * kc = reinterpret_cast<__half *>(I.kptr[static_cast<size_t>(l)]);
        __half * vc = reinterpret_cast<__half *>(I.vptr[static_cast<size_t>(l)]);
        if (l == 0) NAVI_CUDA(navi::dev::launch_pdl(k_rmsnorm, dim3(T), dim3(256), 0, I.stream, I.x, ly.ln1, H, tp.rms_eps, I.n));
        // the QKV projection leaves its split-K partials; one launch sums them, norms and ropes
        // q and k, and stores the K/V cache rows
        const int qs = I.gemm(ly.wqkv, nullptr, I.n, H, T, H, I.QKV, I.qkv, I.QKV, EPI_NONE, false, nullptr, nullptr, nullptr, true);
        NAVI_CUDA(navi::dev::launch_pdl(k_qkv_reduce_norm_rope, dim3(T, I.NH + 2 * I.NKV), dim3(128), 0, I.stream, I.ws.partial, qs, I.qkv,
                                        I.QKV, ly.qn, ly.kn, I.NH, I.NKV, tp.rms_eps, I.rope, 0, kc, vc));
        NAVI_CUDA(navi::dev::launch_pdl(k_prefill_attn_mma, dim3((T + PA_QT - 1) / PA_QT, I.NH), dim3(PA_THREADS), PA_SMEM, I.stream, I.qkv,
                                        I.QKV, kc, vc, T, I.NH, I.NKV, 0, I.att));
        // the RMSNorms after the O projection and (but for the last layer) after the down
        // projection are written by those GEMMs' launches
        I.gemm(ly.wo, nullptr, I.att, I.Q, T, I.Q, H, I.x, H, EPI_RESIDUAL, false, I.x, ly.ln2, I.n);
        // gate/up: a launch that splits K in two leaves both partial slices, and the down
        // projection's staging adds them (one reduction launch fewer per layer)
        const bool fold = T <= GU_FOLD_ROWS && conv::plan(gemm_desc(ly.wgu, nullptr, H, T, H, 2 * I.F, 2 * I.F, EPI_NONE, false), sms).splits == 2;
        if (fold) {
            conv::Conv c = gemm_desc(ly.wgu, nullptr, H, T, H, 2 * I.F, 2 * I.F, EPI_NONE, false);
            c.x = I.n;
            c.y = I.gu;
            c.defer_reduce = true;
            if (conv::launch(c, ws_gu, sms, stream) != 2) fail("talker: the gate/up projection did not split in two", NAVI_E_SHAPE);
        } else {
            I.gemm(ly.wgu, nullptr, I.n, H, T, H, 2 * I.F, I.gu, 2 * I.F, EPI_NONE);
        }
        const bool last = l + 1 == tp.n_layer;
        {
            conv::Conv c = gemm_desc(ly.wd, nullptr, 2 * I.F, T, I.F, H, H, EPI_RESIDUAL, true);
            c.x = fold ? ws_gu.partial : I.gu;
            if (fold) {
                c.x_slices = 2;
                c.x_slice_stride = static_cast<std::size_t>(T) * 2 * I.F;
            }
            c.y = I.x;
            c.resid = I.x;
            c.norm_w = last ? nullptr : I.layers[static_cast<size_t>(l + 1)].ln1;
            c.norm_out = last ? nullptr : I.n;
            c.norm_eps = tp.rms_eps;
            conv::launch(c, ws, sms, stream);
        }
    }
    // the last row: final norm and the codec head
    NAVI_CUDA(navi::dev::launch_pdl(k_rmsnorm, dim3(1), dim3(256), 0, I.stream, I.x + static_cast<size_t>(T - 1) * H, I.final_norm, H,
                                    tp.rms_eps, I.hid));
    I.gemm(I.head, nullptr, I.hid, H, 1, H, I.TV, I.logits, I.TV, EPI_NONE);
}

// Records enqueue_prefill(T) as a CUDA graph (at most 16 lengths). A length whose capture the
// runtime refuses keeps running eagerly; the refusal leaves no error behind.
void Talker::Impl::capture_prefill(int T) {
    if (graphs.size() >= 16) return;
    for (int u : uncapturable)
        if (u == T) return;
    cudaGraph_t g = nullptr;
    NAVI_CUDA(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
    bool enqueued = true;
    try {
        enqueue_prefill(T);
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
        return;
    }
    graphs.emplace_back(T, e);
}

KvCache & Talker::kv() { return impl_->kv; }
const float * Talker::d_hidden() const { return impl_->hid; }
const float * Talker::d_logits() const { return impl_->logits; }
double Talker::last_ms() const { return impl_->last_ms; }

} // namespace navi::qwen3tts
