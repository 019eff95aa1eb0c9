// Implicit-GEMM causal Conv1d on tcgen05 (see conv.hpp for the math and the GEMM view).
//
// CTA = 6 warps:
//   warp 0      one lane streams the CTA's weight tiles (16 KB each, one per (channel
//               block, tap)) into a 4-deep shared-memory ring with bulk copies;
//   warp 1      allocates the tensor-memory accumulator; one lane issues the MMAs
//               (M = 128 channels, N = BN rows, K = 16) and commits their completion
//               to the ring's and the window's "empty" barriers;
//   warps 2-5   stage the input window of each channel block (history / input rows,
//               prologue, f16 hi/lo split) into one of two window buffers, then run the
//               epilogue: tensor-memory loads (warp w reads lanes 32 (w % 4) ..), bias,
//               activation / residual, stores; with split-K the CTA that finishes a
//               tile last sums the partials in split order (deterministic).
// Every mbarrier wait is bounded by a deadline; a CTA that passes it sets the error
// word, stops waiting (its remaining waits return at once) and still frees its
// tensor memory.
#include "conv.hpp"

#include "device.cuh"
#include "umma.cuh"

#include "conv_api.hpp"

#include <algorithm>
#include <atomic>
#include <string>

namespace navi::conv {

namespace {

using namespace navi::dev;

constexpr int SMEM_MAX = 232448;      // opt-in dynamic shared memory per CTA on sm_100
constexpr int BARS_BYTES = 256;

struct KArgs {
    const __half * w;
    const float * x, * hist, * sa, * sb, * bias, * resid, * scale;
    float * y, * partial;
    unsigned * counters;
    int * err;
    int Cout, Cin, K, dil, H, T, x_stride, y_stride, r_stride;
    int BN, CB, cb_per_split, splits;
    int lbo, wrows, tmem_cols;
    unsigned long long timeout_ns;
};

struct Bars {
    uint64_t wfull[NSTAGE], wempty[NSTAGE], afull[2], aempty[2], done;
    uint32_t tmem;
    int abort;
    int last;
};
static_assert(sizeof(Bars) <= BARS_BYTES, "barrier block");

__device__ bool bwait(uint64_t * bar, uint32_t parity, Bars & B, const KArgs & a) {
    if (*reinterpret_cast<volatile int *>(&B.abort)) return false;
    uint64_t t0 = 0;
    for (uint32_t n = 1;; ++n) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((n & 63u) == 0) {
            if (*reinterpret_cast<volatile int *>(&B.abort)) return false;
            const uint64_t now = globaltimer();
            if (t0 == 0) {
                t0 = now;
            } else if (now - t0 > a.timeout_ns) {
                *reinterpret_cast<volatile int *>(&B.abort) = 1;
                atomicExch(a.err, 1);
                return false;
            }
        }
    }
}

template <int EPI>
__device__ __forceinline__ float finish(float v, const KArgs & a, int t, int co) {
    if (a.bias) v += a.bias[co];
    if (EPI == EPI_GELU) {
        v = 0.5f * v * (1.f + erff(v * 0.70710678118654752f));
    } else if (EPI == EPI_RESIDUAL) {
        v += a.resid[static_cast<std::size_t>(t) * a.r_stride + co];
    } else if (EPI == EPI_SCALE_RESIDUAL) {
        v = v * a.scale[co] + a.resid[static_cast<std::size_t>(t) * a.r_stride + co];
    }
    return v;
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// Stages one channel block's window: rows r = u/8, u/8 + 16, ... of k chunk u % 8.
template <int PRO>
__device__ __forceinline__ void stage_window(const KArgs & a, uint8_t * hi, uint8_t * lo, int c0, int t0, int u) {
    const bool valid = c0 < a.Cin;   // Cin % 8 == 0: a chunk is wholly inside or outside
    float ca[8], cb[8];
    if (PRO == PRO_SNAKE && valid) {
        const float4 a0 = *reinterpret_cast<const float4 *>(a.sa + c0), a1 = *reinterpret_cast<const float4 *>(a.sa + c0 + 4);
        const float4 b0 = *reinterpret_cast<const float4 *>(a.sb + c0), b1 = *reinterpret_cast<const float4 *>(a.sb + c0 + 4);
        ca[0] = a0.x; ca[1] = a0.y; ca[2] = a0.z; ca[3] = a0.w; ca[4] = a1.x; ca[5] = a1.y; ca[6] = a1.z; ca[7] = a1.w;
        cb[0] = b0.x; cb[1] = b0.y; cb[2] = b0.z; cb[3] = b0.w; cb[4] = b1.x; cb[5] = b1.y; cb[6] = b1.z; cb[7] = b1.w;
    }
    for (int r = u >> 3; r < a.wrows; r += 16) {
        const int gr = t0 - a.H + r;
        float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (valid) {
            const float * src = nullptr;
            if (gr >= 0 && gr < a.T) src = a.x + static_cast<std::size_t>(gr) * a.x_stride + c0;
            else if (gr < 0 && a.hist) src = a.hist + static_cast<std::size_t>(a.H + gr) * a.Cin + c0;
            if (src) {
                const float4 p0 = *reinterpret_cast<const float4 *>(src), p1 = *reinterpret_cast<const float4 *>(src + 4);
                v[0] = p0.x; v[1] = p0.y; v[2] = p0.z; v[3] = p0.w; v[4] = p1.x; v[5] = p1.y; v[6] = p1.z; v[7] = p1.w;
                if (PRO == PRO_SILU_GATE) {
                    const float4 q0 = *reinterpret_cast<const float4 *>(src + a.Cin), q1 = *reinterpret_cast<const float4 *>(src + a.Cin + 4);
                    const float up[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
                    for (int i = 0; i < 8; ++i) v[i] = v[i] / (1.f + expf(-v[i])) * up[i];
                }
            }
            if (PRO == PRO_SNAKE) {
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float s = sinf(v[i] * ca[i]);
                    v[i] += s * s * cb[i];
                }
            }
        }
        float h[8], l[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            h[i] = __half2float(__float2half_rn(v[i]));
            l[i] = v[i] - h[i];
        }
        *reinterpret_cast<uint4 *>(hi + r * 16) = make_uint4(pack_h2(h[0], h[1]), pack_h2(h[2], h[3]), pack_h2(h[4], h[5]), pack_h2(h[6], h[7]));
        *reinterpret_cast<uint4 *>(lo + r * 16) = make_uint4(pack_h2(l[0], l[1]), pack_h2(l[2], l[3]), pack_h2(l[4], l[5]), pack_h2(l[6], l[7]));
    }
}

template <int PRO, int EPI>
__global__ void __launch_bounds__(NTHREADS, 1) k_conv(const KArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t * ring = smem;
    uint8_t * win = smem + NSTAGE * TILE_BYTES;
    const int win_bytes = 8 * a.lbo;                       // one buffer's hi (or lo) planes
    Bars & B = *reinterpret_cast<Bars *>(win + 4 * win_bytes);

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int t0 = blockIdx.x * a.BN, mt = blockIdx.y, sp = blockIdx.z;
    const int c_begin = sp * a.cb_per_split, c_end = min(a.CB, c_begin + a.cb_per_split);
    const int NC = c_end - c_begin;

    if (threadIdx.x == 0) {
        for (int i = 0; i < NSTAGE; ++i) {
            mbar_init(&B.wfull[i], 1);
            mbar_init(&B.wempty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&B.afull[i], 128);
            mbar_init(&B.aempty[i], 1);
        }
        mbar_init(&B.done, 1);
        B.abort = 0;
        B.last = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        umma::tmem_alloc(&B.tmem, a.tmem_cols);
        umma::tmem_relinquish();
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tmem = B.tmem;

    if (warp == 0) {
        if (lane == 0) {
            const __half * wt = a.w + static_cast<std::size_t>(mt) * a.CB * a.K * TILE_ELEMS;
            const int NIT = NC * a.K;
            for (int it = 0; it < NIT; ++it) {
                const int s = it % NSTAGE;
                if (it >= NSTAGE && !bwait(&B.wempty[s], ((it / NSTAGE) - 1) & 1, B, a)) break;
                mbar_arrive_expect_tx(&B.wfull[s], TILE_BYTES);
                const int c = c_begin + it / a.K, j = it % a.K;
                bulk_g2s(ring + s * TILE_BYTES, wt + (static_cast<std::size_t>(c) * a.K + j) * TILE_ELEMS, TILE_BYTES, &B.wfull[s]);
            }
            // tail: every issued tile has been consumed before the CTA may exit
            for (int it = max(0, NIT - NSTAGE); it < NIT; ++it) bwait(&B.wempty[it % NSTAGE], (it / NSTAGE) & 1, B, a);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = umma::idesc_f16_f32(BM, a.BN);
            const uint32_t ring_a = smem_addr(ring), win_a = smem_addr(win);
            int it = 0;
            for (int ci = 0; ci < NC; ++ci) {
                const int b = ci & 1;
                if (!bwait(&B.afull[b], (ci >> 1) & 1, B, a)) break;
                umma::fence_after_sync();
                const uint32_t hi_a = win_a + (b * 2) * win_bytes, lo_a = hi_a + win_bytes;
                for (int j = 0; j < a.K; ++j, ++it) {
                    const int s = it % NSTAGE;
                    if (!bwait(&B.wfull[s], (it / NSTAGE) & 1, B, a)) break;
                    umma::fence_after_sync();
                    const uint32_t sa = ring_a + s * TILE_BYTES;
                    const uint32_t shift = static_cast<uint32_t>(j * a.dil * 16);
#pragma unroll
                    for (int ks = 0; ks < BK / 16; ++ks) {
                        const uint64_t ad = umma::desc_kmajor(sa + ks * 2 * (BM * 16), BM * 16, 128);
                        const uint64_t bh = umma::desc_kmajor(hi_a + ks * 2 * a.lbo + shift, a.lbo, 128);
                        const uint64_t bl = umma::desc_kmajor(lo_a + ks * 2 * a.lbo + shift, a.lbo, 128);
                        umma::mma_f16(tmem, ad, bh, idesc, (ci | j | ks) != 0);
                        umma::mma_f16(tmem, ad, bl, idesc, true);
                    }
                    umma::commit(&B.wempty[s]);
                }
                umma::commit(&B.aempty[b]);
            }
            umma::commit(&B.done);
        }
    } else {
        const int u = threadIdx.x - 64;                  // 0..127
        const int kc = u & 7;
        for (int ci = 0; ci < NC; ++ci) {
            const int b = ci & 1;
            if (ci >= 2 && !bwait(&B.aempty[b], ((ci >> 1) - 1) & 1, B, a)) break;
            uint8_t * hi = win + (b * 2) * win_bytes + kc * a.lbo;
            stage_window<PRO>(a, hi, hi + win_bytes, (c_begin + ci) * BK + kc * 8, t0, u);
            fence_proxy_async_smem();
            mbar_arrive(&B.afull[b]);
        }
        const bool ok = bwait(&B.done, 0, B, a);
        umma::fence_after_sync();
        const int q = warp & 3;
        const int co = mt * BM + q * 32 + lane;
        const uint32_t tq = tmem + (static_cast<uint32_t>(q * 32) << 16);
        for (int cc = 0; cc < a.BN; cc += 16) {
            float v[16];
            umma::tmem_ld16(tq + cc, v);
            if (!ok) continue;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const int t = t0 + cc + i;
                if (t >= a.T || co >= a.Cout) continue;
                if (a.splits > 1) a.partial[(static_cast<std::size_t>(sp) * a.T + t) * a.Cout + co] = v[i];
                else a.y[static_cast<std::size_t>(t) * a.y_stride + co] = finish<EPI>(v[i], a, t, co);
            }
        }
        if (a.splits > 1) {
            __threadfence();
            named_sync(1, 128);
            const int tile = blockIdx.y * gridDim.x + blockIdx.x;
            if (u == 0) B.last = (atomicAdd(&a.counters[tile], 1u) == static_cast<unsigned>(a.splits - 1)) ? 1 : 0;
            named_sync(1, 128);
            if (B.last) {
                __threadfence();
                if (co < a.Cout) {
                    const int tend = min(a.T, t0 + a.BN);
                    for (int t = t0; t < tend; ++t) {
                        float s = 0.f;
                        for (int k = 0; k < a.splits; ++k) s += __ldcg(a.partial + (static_cast<std::size_t>(k) * a.T + t) * a.Cout + co);
                        a.y[static_cast<std::size_t>(t) * a.y_stride + co] = finish<EPI>(s, a, t, co);
                    }
                }
                if (u == 0) a.counters[tile] = 0u;
            }
        }
    }
    umma::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        umma::fence_after_sync();
        umma::tmem_dealloc(tmem, a.tmem_cols);
    }
}

struct PackArgs {
    PackSrc s[MAX_PACK_SRC];
    int n, Cout, Cin, K, CB;
};

__global__ void k_pack(const PackArgs pa, __half * dst, std::size_t n) {
    for (std::size_t i = static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<std::size_t>(gridDim.x) * blockDim.x) {
        const std::size_t tile = i / TILE_ELEMS;
        const int e = static_cast<int>(i % TILE_ELEMS);
        const int kc = e / (BM * 8), rem = e % (BM * 8);
        const int col = rem / 8, cil = kc * 8 + rem % 8;
        const int j = static_cast<int>(tile % pa.K);
        const std::size_t t2 = tile / pa.K;
        const int cb = static_cast<int>(t2 % pa.CB), m = static_cast<int>(t2 / pa.CB);
        const int co = m * BM + col, ci = cb * BK + cil;
        __half v = __float2half_rn(0.f);
        if (co < pa.Cout && ci < pa.Cin) {
            for (int k = 0; k < pa.n; ++k) {
                const PackSrc & s = pa.s[k];
                if (co < s.co0 || co >= s.co1 || ci < s.ci0 || ci >= s.ci1) continue;
                const long long c = co - s.co0, d = ci - s.ci0;
                if (s.trans) {
                    const long long ph = c / s.cout_b, cc = c % s.cout_b, m2 = pa.K - 1 - j;
                    v = s.p[d * s.cout_b * s.k + cc * s.k + ph + m2 * s.stride];
                } else {
                    v = s.p[c * s.s_co + d * s.s_ci + j * s.s_tap];
                }
                break;
            }
        }
        dst[i] = v;
    }
}

template <int PRO, int EPI>
void launch_t(const KArgs & ka, dim3 grid, std::size_t smem, cudaStream_t stream) {
    static std::atomic<uint64_t> attr{0};   // devices whose attribute is set, one bit per ordinal < 64
    int dev = 0;
    NAVI_CUDA(cudaGetDevice(&dev));
    const uint64_t bit = 1ull << (dev & 63);
    if (!(attr.load() & bit)) {
        NAVI_CUDA(cudaFuncSetAttribute(k_conv<PRO, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_MAX));
        attr.fetch_or(bit);
    }
    k_conv<PRO, EPI><<<grid, NTHREADS, smem, stream>>>(ka);
}

__global__ void k_fold_bias(const float * b, int n, int phases, float * out) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n * phases; i += gridDim.x * blockDim.x) out[i] = b[i % n];
}

int lbo_for(int wrows) { return ((wrows + 7) / 8 * 8 + 1) * 16; }   // plane stride = 16 (mod 128): conflict-free stores
std::size_t smem_for(int BN, int H) { return static_cast<std::size_t>(NSTAGE) * TILE_BYTES + 4ull * 8 * lbo_for(BN + H) + BARS_BYTES; }

} // namespace

void pack(const std::vector<PackSrc> & srcs, int Cout, int Cin, int K, __half * dst, cudaStream_t stream) {
    if (srcs.empty() || srcs.size() > MAX_PACK_SRC) fail("conv pack: 1.." + std::to_string(MAX_PACK_SRC) + " sources", NAVI_E_SHAPE);
    PackArgs pa{};
    for (std::size_t i = 0; i < srcs.size(); ++i) pa.s[i] = srcs[i];
    pa.n = static_cast<int>(srcs.size());
    pa.Cout = Cout; pa.Cin = Cin; pa.K = K; pa.CB = ceil_div(Cin, BK);
    const std::size_t n = packed_elems(Cout, Cin, K);
    k_pack<<<static_cast<unsigned>(std::min<std::size_t>((n + 255) / 256, 148 * 32)), 256, 0, stream>>>(pa, dst, n);
    NAVI_CUDA(cudaGetLastError());
}

Plan plan(const Conv & c, int sms) {
    Plan p;
    p.MT = ceil_div(c.Cout, BM);
    p.CB = ceil_div(c.Cin, BK);
    const int H = (c.K - 1) * c.dil;
    int BN = 16;
    while (BN < c.T && BN < 256) BN *= 2;
    while (BN > 16 && smem_for(BN, H) > static_cast<std::size_t>(SMEM_MAX)) BN /= 2;
    // row-heavy layers: smaller row tiles until the grid covers the SMs (not below 64 rows)
    while (BN > 64 && p.MT * ceil_div(c.T, BN) < sms) BN /= 2;
    const int target = sms * 3 / 4;
    for (;;) {
        const int tiles = p.MT * ceil_div(c.T, BN);
        int splits = 1, cbps = p.CB;
        if (tiles < target && p.CB > 1) {
            const int want = std::min(p.CB, ceil_div(sms, tiles));
            cbps = ceil_div(p.CB, want);
            splits = ceil_div(p.CB, cbps);
        }
        const bool enough = tiles * splits >= target;
        if (enough || BN <= 16 || ceil_div(c.T, BN / 2) == ceil_div(c.T, BN)) {
            p.BN = BN;
            p.NT = ceil_div(c.T, BN);
            p.splits = splits;
            p.cb_per_split = cbps;
            break;
        }
        BN /= 2;
    }
    p.lbo = lbo_for(p.BN + H);
    p.tmem_cols = std::max(32, p.BN);
    p.smem = smem_for(p.BN, H);
    if (p.smem > static_cast<std::size_t>(SMEM_MAX)) fail("conv: window of " + std::to_string(H) + " history rows does not fit", NAVI_E_SHAPE);
    return p;
}

std::size_t partial_need(const Conv & c, int sms) {
    const Plan p = plan(c, sms);
    return p.splits > 1 ? static_cast<std::size_t>(p.splits) * c.T * c.Cout : 0;
}
int counters_need(const Conv & c, int sms) {
    const Plan p = plan(c, sms);
    return p.splits > 1 ? p.NT * p.MT : 0;
}

void launch(const Conv & c, const Workspace & ws, int sms, cudaStream_t stream) {
    if (c.T <= 0) return;
    if (c.Cin % 8 || c.x_stride % 4 || c.K < 1 || c.dil < 1 || !c.w || !c.x || !c.y)
        fail("conv: Cin and the input row stride must be multiples of 8 and 4", NAVI_E_SHAPE);
    if ((reinterpret_cast<std::uintptr_t>(c.x) | reinterpret_cast<std::uintptr_t>(c.hist) | reinterpret_cast<std::uintptr_t>(c.w)) & 15u)
        fail("conv: input, history and weights must be 16-byte aligned", NAVI_E_SHAPE);
    if (c.pro == PRO_SNAKE && (!c.snake_a || !c.snake_b || ((reinterpret_cast<std::uintptr_t>(c.snake_a) | reinterpret_cast<std::uintptr_t>(c.snake_b)) & 15u)))
        fail("conv: Snake coefficients missing or misaligned", NAVI_E_SHAPE);
    if (c.pro == PRO_SILU_GATE && c.hist) fail("conv: gated input has no history", NAVI_E_SHAPE);
    if ((c.epi == EPI_RESIDUAL || c.epi == EPI_SCALE_RESIDUAL) && !c.resid) fail("conv: residual missing", NAVI_E_SHAPE);
    if (c.epi == EPI_SCALE_RESIDUAL && !c.scale) fail("conv: layer scale missing", NAVI_E_SHAPE);
    const Plan p = plan(c, sms);
    if (p.splits > 1) {
        if (static_cast<std::size_t>(p.splits) * c.T * c.Cout > ws.partial_cap || p.NT * p.MT > ws.n_counters)
            fail("conv: split-K workspace too small", NAVI_E_SHAPE);
    }
    KArgs ka{};
    ka.w = c.w; ka.x = c.x; ka.hist = c.hist; ka.sa = c.snake_a; ka.sb = c.snake_b; ka.bias = c.bias;
    ka.resid = c.resid; ka.scale = c.scale; ka.y = c.y; ka.partial = ws.partial; ka.counters = ws.counters; ka.err = ws.err;
    ka.Cout = c.Cout; ka.Cin = c.Cin; ka.K = c.K; ka.dil = c.dil; ka.H = (c.K - 1) * c.dil; ka.T = c.T;
    ka.x_stride = c.x_stride; ka.y_stride = c.y_stride; ka.r_stride = c.r_stride;
    ka.BN = p.BN; ka.CB = p.CB; ka.cb_per_split = p.cb_per_split; ka.splits = p.splits;
    ka.lbo = p.lbo; ka.wrows = p.BN + ka.H; ka.tmem_cols = p.tmem_cols; ka.timeout_ns = ws.timeout_ns;
    const dim3 grid(p.NT, p.MT, p.splits);
#define NAVI_CONV_CASE(PR, EP) \
    if (c.pro == PR && c.epi == EP) { launch_t<PR, EP>(ka, grid, p.smem, stream); NAVI_CUDA(cudaGetLastError()); return; }
    NAVI_CONV_CASE(PRO_NONE, EPI_NONE)
    NAVI_CONV_CASE(PRO_NONE, EPI_GELU)
    NAVI_CONV_CASE(PRO_NONE, EPI_SCALE_RESIDUAL)
    NAVI_CONV_CASE(PRO_SILU_GATE, EPI_SCALE_RESIDUAL)
    NAVI_CONV_CASE(PRO_SNAKE, EPI_NONE)
    NAVI_CONV_CASE(PRO_SNAKE, EPI_RESIDUAL)
    NAVI_CONV_CASE(PRO_NONE, EPI_RESIDUAL)
    NAVI_CONV_CASE(PRO_SNAKE, EPI_GELU)
#undef NAVI_CONV_CASE
    fail("conv: no instantiation for prologue " + std::to_string(c.pro) + " epilogue " + std::to_string(c.epi), NAVI_E_SHAPE);
}

} // namespace navi::conv

namespace navi {

int conv_once(const Device & dev, const navi_conv_args & a) {
    using namespace navi::conv;
    dev.make_current();
    const cudaStream_t s = dev.stream();
    const int P = a.trans_stride > 0 ? a.trans_stride : 1;
    if (P > 1 && (a.epi != EPI_NONE || a.dil != 1)) fail("conv: a transposed conv takes no residual epilogue and no dilation", NAVI_E_ARG);
    std::vector<void *> own;
    auto alloc = [&](std::size_t bytes) {
        void * p = nullptr;
        NAVI_CUDA(cudaMalloc(&p, std::max<std::size_t>(bytes, 16)));
        own.push_back(p);
        NAVI_CUDA(cudaMemsetAsync(p, 0, std::max<std::size_t>(bytes, 16), s));
        return p;
    };
    int st = NAVI_OK;
    try {
        Conv c;
        c.Cout = a.Cout * P; c.Cin = a.Cin; c.K = a.K; c.dil = a.dil;
        PackSrc ps;
        ps.p = reinterpret_cast<const __half *>(a.w);
        ps.co0 = 0; ps.co1 = c.Cout; ps.ci0 = 0; ps.ci1 = a.Cin;
        if (P > 1) {
            ps.trans = 1; ps.cout_b = a.Cout; ps.k = a.K * P; ps.stride = P;
        } else {
            ps.s_co = static_cast<long long>(a.Cin) * a.K; ps.s_ci = a.K; ps.s_tap = 1;
        }
        __half * wp = static_cast<__half *>(alloc(packed_elems(c.Cout, c.Cin, c.K) * sizeof(__half)));
        pack({ps}, c.Cout, c.Cin, c.K, wp, s);
        c.w = wp;
        c.x = a.x; c.x_stride = a.x_stride; c.T = a.T; c.hist = a.hist;
        c.pro = a.pro; c.snake_a = a.snake_a; c.snake_b = a.snake_b;
        c.epi = a.epi; c.resid = a.resid; c.r_stride = a.y_stride; c.scale = a.scale;
        c.y = a.y; c.y_stride = a.y_stride;
        c.bias = a.bias;
        if (a.bias && P > 1) {
            float * fb = static_cast<float *>(alloc(static_cast<std::size_t>(c.Cout) * sizeof(float)));
            k_fold_bias<<<(c.Cout + 255) / 256, 256, 0, s>>>(a.bias, a.Cout, P, fb);
            NAVI_CUDA(cudaGetLastError());
            c.bias = fb;
        }
        const int sms = dev.info().multiprocessors;
        Workspace ws;
        ws.partial_cap = partial_need(c, sms);
        ws.partial = static_cast<float *>(alloc(ws.partial_cap * sizeof(float)));
        ws.n_counters = std::max(1, counters_need(c, sms));
        ws.counters = static_cast<unsigned *>(alloc(static_cast<std::size_t>(ws.n_counters) * sizeof(unsigned)));
        ws.err = static_cast<int *>(alloc(sizeof(int)));
        launch(c, ws, sms, s);
        int err = 0;
        NAVI_CUDA(cudaMemcpyAsync(&err, ws.err, sizeof(int), cudaMemcpyDeviceToHost, s));
        NAVI_CUDA(cudaStreamSynchronize(s));
        if (err) st = NAVI_E_TIMEOUT;
    } catch (...) {
        (void) cudaStreamSynchronize(s);
        for (void * p : own) (void) cudaFree(p);
        throw;
    }
    for (void * p : own) (void) cudaFree(p);
    if (st != NAVI_OK) fail("conv: a tensor-core conv wait passed its deadline", st);
    return st;
}

} // namespace navi
