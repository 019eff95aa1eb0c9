// Implicit-GEMM causal Conv1d on tcgen05 (see conv.hpp for the math and the GEMM view).
//
// Persistent CTA (one per SM at most) over work units = (row tile, channel tile, K split),
// 10 warps:
//   warp 0      one lane streams the units' weight tiles (16 KB each, one per (channel
//               block, tap)) into a 4-deep shared-memory ring with bulk copies;
//   warp 1      allocates two tensor-memory accumulators (2 x BN columns); one lane
//               issues the MMAs (M = 128 channels, N = BN rows, K = 16) and commits their
//               completion to the ring's, the window's and the accumulator's barriers;
//   warps 2-5   stage the input window of each channel block (history / input rows,
//               prologue, f16 hi/lo split) into one of two window buffers;
//   warps 6-9   epilogue: tensor-memory loads (warp w reads lanes 32 (w % 4) ..), bias,
//               activation / residual, stores; with split-K each split stores its partial
//               sums and k_splitk_reduce adds them in split order (deterministic) and
//               applies the epilogue (k_reduce_norm, one CTA per row, when the layer
//               after the conv starts with an RMS norm: it also writes the norm).
// So unit n's epilogue, unit n+1's MMAs and unit n+2's window staging overlap.
// Every mbarrier wait is bounded by a deadline; a CTA that passes it sets the error
// word, stops waiting (its remaining waits return at once) and still frees its
// tensor memory.
#include "conv.hpp"

#include <cuda.h>
#include <cudaTypedefs.h>

#include "device.cuh"
#include "umma.cuh"

#include "conv_api.hpp"

#include <algorithm>
#include <cstring>
#include <atomic>
#include <string>

namespace navi::conv {

namespace {

using namespace navi::dev;

constexpr int SMEM_MAX = 232448;      // opt-in dynamic shared memory per CTA on sm_100
constexpr int BARS_BYTES = 512;
constexpr int MAXST = 14;             // weight tiles the ring (or the resident set) can hold

struct KArgs {
    const __half * w;
    const float * x, * hist, * sa, * sb, * bias, * resid, * scale;
    float * y, * partial;
    float * hist_out;                 // next chunk's history, or null
    int * err;
    int Cout, Cin, K, dil, H, T, x_stride, y_stride, r_stride;
    int x_slices;                     // 2: x holds two split-K partial slices, summed while staging
    long long x_sstride;              // elements from one slice to the next
    int BN, NT, MT, CB, cb_per_split, splits;
    int lbo, wrows, tmem_cols;
    int nst;                          // weight-ring stages
    int tmaw;                         // 1: weights are a row-major matrix read by TMA (128B-swizzled tiles)
    int resident;                     // 1: the CTA's tiles are loaded once and reused by every unit
    int early_weights;                // 1: the weight stream need not wait for the previous kernel
    unsigned long long timeout_ns;
    const float * norm_w;             // row RMS norm of y into norm_out ([T][Cout]), or null
    float * norm_out;
    float norm_eps;
};

struct Bars {
    uint64_t wfull[MAXST], wempty[MAXST], afull[2], aempty[2], tfull[2], tempty[2], edone;
    uint32_t tmem;
    int abort;
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
                atomicExch(a.err, ERR_TIMEOUT);
                return false;
            }
        }
    }
}

// A wait that ignores the abort flag (bounded by its own, longer deadline): the tensor-memory
// release waits so for every epilogue thread, which arrives on the barrier on every path.
__device__ void bwait_drain(uint64_t * bar, uint32_t parity, const KArgs & a) {
    const uint64_t t0 = globaltimer();
    while (!mbar_try_wait(bar, parity))
        if (globaltimer() - t0 > 4 * a.timeout_ns) {
            atomicExch(a.err, ERR_TIMEOUT);
            return;
        }
}

// v already includes the bias; r is the residual row value, sc the channel's layer scale.
template <int EPI>
__device__ __forceinline__ float finish(float v, float sc, float r) {
    if (EPI == EPI_GELU) return 0.5f * v * (1.f + erff(v * 0.70710678118654752f));
    if (EPI == EPI_RESIDUAL) return v + r;
    if (EPI == EPI_SCALE_RESIDUAL) return v * sc + r;
    if (EPI == EPI_SILU) return v / (1.f + expf(-v));
    return v;
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// Window staging, software-pipelined: thread u owns k chunk u % 8 (channels c0..c0+7 of
// the block) and rows u/8 + 16 i of each batch of 16 * SR<PRO> window rows.  The loads of
// the next batch (possibly of the next channel block or unit) are issued before the
// current batch is converted, so a thread keeps a batch in flight while it converts.
// A gated input may arrive as the two split-K partial slices of the projection that made it
// (its reduction folded into this launch): the second slice's rows ride along in e/f.
template <int PRO> struct SR {
    static constexpr int n = PRO == PRO_SILU_GATE ? 2 : 4;
    static constexpr int ne = PRO == PRO_SILU_GATE ? n : 1;
};

template <int PRO>
struct Rows {
    float4 p0[SR<PRO>::n], p1[SR<PRO>::n], q0[SR<PRO>::n], q1[SR<PRO>::n];
    float4 e0[SR<PRO>::ne], e1[SR<PRO>::ne], f0[SR<PRO>::ne], f1[SR<PRO>::ne];
};

template <int PRO>
__device__ __forceinline__ void load_rows(Rows<PRO> & R, const KArgs & a, int c0, int t0, int rb) {
    constexpr int N = SR<PRO>::n;
    const bool valid = c0 < a.Cin;   // Cin % 8 == 0: a chunk is wholly inside or outside
#pragma unroll
    for (int k = 0; k < N; ++k) {
        const int r = rb + 16 * k, gr = t0 - a.H + r;
        const float * src = nullptr;
        if (valid && r < a.wrows) {
            if (gr >= 0 && gr < a.T) src = a.x + static_cast<std::size_t>(gr) * a.x_stride + c0;
            else if (gr < 0 && a.hist) src = a.hist + static_cast<std::size_t>(a.H + gr) * a.Cin + c0;
        }
        const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
        R.p0[k] = src ? __ldg(reinterpret_cast<const float4 *>(src)) : z;
        R.p1[k] = src ? __ldg(reinterpret_cast<const float4 *>(src + 4)) : z;
        if constexpr (PRO == PRO_SILU_GATE) {
            R.q0[k] = src ? __ldg(reinterpret_cast<const float4 *>(src + a.Cin)) : z;
            R.q1[k] = src ? __ldg(reinterpret_cast<const float4 *>(src + a.Cin + 4)) : z;
            if (a.x_slices > 1) {   // the second partial slice (gated input has no history)
                const float * s1 = src ? src + a.x_sstride : nullptr;
                R.e0[k] = s1 ? __ldcg(reinterpret_cast<const float4 *>(s1)) : z;
                R.e1[k] = s1 ? __ldcg(reinterpret_cast<const float4 *>(s1 + 4)) : z;
                R.f0[k] = s1 ? __ldcg(reinterpret_cast<const float4 *>(s1 + a.Cin)) : z;
                R.f1[k] = s1 ? __ldcg(reinterpret_cast<const float4 *>(s1 + a.Cin + 4)) : z;
            }
        }
    }
}

template <int PRO>
__device__ __forceinline__ void store_rows(const Rows<PRO> & R, const KArgs & a, uint8_t * hi, uint8_t * lo, int c0, int rb) {
    constexpr int N = SR<PRO>::n;
    float ca[8], cb[8];
    const bool valid = c0 < a.Cin;
    if (PRO == PRO_SNAKE) {
        if (valid) {
            const float4 a0 = __ldg(reinterpret_cast<const float4 *>(a.sa + c0)), a1 = __ldg(reinterpret_cast<const float4 *>(a.sa + c0 + 4));
            const float4 b0 = __ldg(reinterpret_cast<const float4 *>(a.sb + c0)), b1 = __ldg(reinterpret_cast<const float4 *>(a.sb + c0 + 4));
            ca[0] = a0.x; ca[1] = a0.y; ca[2] = a0.z; ca[3] = a0.w; ca[4] = a1.x; ca[5] = a1.y; ca[6] = a1.z; ca[7] = a1.w;
            cb[0] = b0.x; cb[1] = b0.y; cb[2] = b0.z; cb[3] = b0.w; cb[4] = b1.x; cb[5] = b1.y; cb[6] = b1.z; cb[7] = b1.w;
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) ca[i] = cb[i] = 0.f;
        }
    }
#pragma unroll
    for (int k = 0; k < N; ++k) {
        const int r = rb + 16 * k;
        if (r >= a.wrows) break;
        float v[8] = {R.p0[k].x, R.p0[k].y, R.p0[k].z, R.p0[k].w, R.p1[k].x, R.p1[k].y, R.p1[k].z, R.p1[k].w};
        if constexpr (PRO == PRO_SILU_GATE) {
            float up[8] = {R.q0[k].x, R.q0[k].y, R.q0[k].z, R.q0[k].w, R.q1[k].x, R.q1[k].y, R.q1[k].z, R.q1[k].w};
            if (a.x_slices > 1) {
                // slice 0 + slice 1 (+ 0, the absent bias): the split-K reduction's own sum
                const float g1[8] = {R.e0[k].x, R.e0[k].y, R.e0[k].z, R.e0[k].w, R.e1[k].x, R.e1[k].y, R.e1[k].z, R.e1[k].w};
                const float u1[8] = {R.f0[k].x, R.f0[k].y, R.f0[k].z, R.f0[k].w, R.f1[k].x, R.f1[k].y, R.f1[k].z, R.f1[k].w};
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    v[i] = (v[i] + g1[i]) + 0.f;
                    up[i] = (up[i] + u1[i]) + 0.f;
                }
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = v[i] / (1.f + __expf(-v[i])) * up[i];
        }
        if (PRO == PRO_SNAKE) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float sn = __sinf(v[i] * ca[i]);
                v[i] += sn * sn * cb[i];
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

// Work unit u (row tile nt fastest, then channel tile mt, then split sp).
struct Unit {
    int t0, mt, sp, c_begin, nc;
};
__device__ __forceinline__ Unit unit_of(const KArgs & a, int u) {
    Unit w;
    const int nt = u % a.NT, r = u / a.NT;
    w.mt = r % a.MT;
    w.sp = r / a.MT;
    w.t0 = nt * a.BN;
    w.c_begin = w.sp * a.cb_per_split;
    w.nc = min(a.CB, w.c_begin + a.cb_per_split) - w.c_begin;
    return w;
}

template <int EPI>
__device__ __forceinline__ void load_resid(float (&rr)[16], const KArgs & a, int t, int co, bool live) {
    const int nv = min(16, a.T - t);
#pragma unroll
    for (int i = 0; i < 16; ++i) rr[i] = (live && i < nv) ? a.resid[static_cast<std::size_t>(t + i) * a.r_stride + co] : 0.f;
}

// Stores one unit's accumulator (BN rows x this thread's channel); the residual rows of
// the next 16-row batch are loaded before the current batch is stored.
template <int EPI>
__device__ __forceinline__ void epilogue_unit(const KArgs & a, const Unit & w, uint32_t tacc, int q, int lane, bool ok) {
    constexpr bool RES = EPI == EPI_RESIDUAL || EPI == EPI_SCALE_RESIDUAL;
    const int co = w.mt * BM + q * 32 + lane;
    const bool live = ok && co < a.Cout;
    const float bco = (a.bias && live && a.splits == 1) ? a.bias[co] : 0.f;
    const float sco = (EPI == EPI_SCALE_RESIDUAL && live) ? a.scale[co] : 1.f;
    const uint32_t tq = tacc + (static_cast<uint32_t>(q * 32) << 16);
    const bool fin = live && a.splits == 1;
    float rr[16], rn[16];
    // after an abort the accumulator holds nothing to read: the warp skips its tensor-memory
    // loads (tcgen05.ld is warp-collective, so the decision is the warp's)
    if (!__all_sync(0xffffffffu, ok)) return;
    if (RES) load_resid<EPI>(rr, a, w.t0, co, fin);
    for (int cc = 0; cc < a.BN; cc += 16) {
        float v[16];
        __syncwarp();                        // tcgen05.ld is warp-collective (.sync.aligned)
        umma::tmem_ld16(tq + cc, v);
        if (RES && cc + 16 < a.BN) load_resid<EPI>(rn, a, w.t0 + cc + 16, co, fin && w.t0 + cc + 16 < a.T);
        const int nv = min(16, a.T - (w.t0 + cc));
        if (live && a.splits > 1) {
#pragma unroll
            for (int i = 0; i < 16; ++i)
                if (i < nv) a.partial[(static_cast<std::size_t>(w.sp) * a.T + w.t0 + cc + i) * a.Cout + co] = v[i];
        } else if (live) {
#pragma unroll
            for (int i = 0; i < 16; ++i)
                if (i < nv) a.y[static_cast<std::size_t>(w.t0 + cc + i) * a.y_stride + co] = finish<EPI>(v[i] + bco, sco, rr[i]);
        }
        if (RES) {
#pragma unroll
            for (int i = 0; i < 16; ++i) rr[i] = rn[i];
        }
    }
    __syncwarp();
}

// Persistent: CTA b takes units b, b + grid, ...; every role walks the same unit list,
// so the weight ring, the two window buffers and the two accumulators run as pipelines
// across unit boundaries.
template <int PRO, int EPI>
__global__ void __launch_bounds__(NTHREADS, 1) k_conv(const KArgs a, const __grid_constant__ CUtensorMap tmw) {
    // launched after the previous kernel of the stream may still run: every role that reads
    // its outputs waits for it below; the weight stream (warp 0) does not when the weights
    // are settled, so the first tiles load while the previous kernel finishes
    navi::dev::griddep_launch_dependents();
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t * ring = smem;
    uint8_t * win = smem + a.nst * TILE_BYTES;
    const int win_bytes = 8 * a.lbo;                       // one buffer's hi (or lo) planes
    Bars & B = *reinterpret_cast<Bars *>(win + 4 * win_bytes);

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int n_units = a.NT * a.MT * a.splits;

    if (threadIdx.x == 0) {
        for (int i = 0; i < a.nst; ++i) {
            mbar_init(&B.wfull[i], 1);
            mbar_init(&B.wempty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&B.afull[i], 128);
            mbar_init(&B.aempty[i], 1);
            mbar_init(&B.tfull[i], 1);
            mbar_init(&B.tempty[i], 128);
        }
        mbar_init(&B.edone, 128);
        B.abort = 0;
        if (a.tmaw && (smem_addr(ring) & 1023u)) {   // 128B-swizzled tiles need 1024-byte alignment
            B.abort = 1;                              // no role issues a copy or an MMA
            atomicExch(a.err, ERR_ALIGN);
        }
        fence_mbar_init();
    }
    if (warp == 1) {
        __syncwarp();
        umma::tmem_alloc(&B.tmem, a.tmem_cols);
        umma::tmem_relinquish();
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tmem = B.tmem;
    if (warp != 0 || !a.early_weights) navi::dev::griddep_wait();

    if (warp == 0) {
        if (lane == 0 && a.resident) {
            // one channel tile, no split: every unit of this CTA uses the same CB * K tiles
            const int nit = a.CB * a.K;
            for (int i = 0; i < nit && !B.abort; ++i) {
                mbar_arrive_expect_tx(&B.wfull[i], TILE_BYTES);
                if (a.tmaw) umma::tma_load_2d(ring + i * TILE_BYTES, &tmw, (i / a.K) * BK, 0, &B.wfull[i]);
                else bulk_g2s(ring + i * TILE_BYTES, a.w + static_cast<std::size_t>(i) * TILE_ELEMS, TILE_BYTES, &B.wfull[i]);
            }
        } else if (lane == 0) {
            const int NST = a.nst;
            int it = 0;
            for (int un = blockIdx.x; un < n_units; un += gridDim.x) {
                const Unit w = unit_of(a, un);
                const __half * wt = a.w + (static_cast<std::size_t>(w.mt) * a.CB + w.c_begin) * a.K * TILE_ELEMS;
                const int nit = w.nc * a.K;   // tiles of this unit are contiguous
                for (int i = 0; i < nit; ++i, ++it) {
                    const int s = it % NST;
                    if (it >= NST && !bwait(&B.wempty[s], ((it / NST) - 1) & 1, B, a)) break;
                    if (B.abort) break;
                    mbar_arrive_expect_tx(&B.wfull[s], TILE_BYTES);
                    if (a.tmaw) umma::tma_load_2d(ring + s * TILE_BYTES, &tmw, (w.c_begin + i / a.K) * BK, w.mt * BM, &B.wfull[s]);
                    else bulk_g2s(ring + s * TILE_BYTES, wt + static_cast<std::size_t>(i) * TILE_ELEMS, TILE_BYTES, &B.wfull[s]);
                }
            }
            // tail: every issued tile has been consumed before the CTA may exit
            for (int k = max(0, it - NST); k < it; ++k) bwait(&B.wempty[k % NST], (k / NST) & 1, B, a);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = umma::idesc_f16_f32(BM, a.BN);
            const uint32_t ring_a = smem_addr(ring), win_a = smem_addr(win);
            int it = 0, cg = 0, k = 0;
            for (int un = blockIdx.x; un < n_units; un += gridDim.x, ++k) {
                const Unit w = unit_of(a, un);
                const int acc = k & 1;
                if (k >= 2 && !bwait(&B.tempty[acc], ((k >> 1) - 1) & 1, B, a)) break;
                umma::fence_after_sync();
                const uint32_t d = tmem + static_cast<uint32_t>(acc * a.BN);
                bool first = true;
                for (int ci = 0; ci < w.nc; ++ci, ++cg) {
                    const int b = cg & 1;
                    if (!bwait(&B.afull[b], (cg >> 1) & 1, B, a)) break;
                    umma::fence_after_sync();
                    const uint32_t hi_a = win_a + (b * 2) * win_bytes, lo_a = hi_a + win_bytes;
                    for (int j = 0; j < a.K; ++j, ++it) {
                        int s;
                        if (a.resident) {
                            s = (w.c_begin + ci) * a.K + j;
                            if (k == 0 && !bwait(&B.wfull[s], 0, B, a)) break;
                        } else {
                            s = it % a.nst;
                            if (!bwait(&B.wfull[s], (it / a.nst) & 1, B, a)) break;
                        }
                        umma::fence_after_sync();
                        const uint32_t sa = ring_a + s * TILE_BYTES;
                        const uint32_t shift = static_cast<uint32_t>(j * a.dil * 16);
#pragma unroll
                        for (int ks = 0; ks < BK / 16; ++ks) {
                            const uint64_t ad = a.tmaw ? umma::desc_kmajor_sw128(sa + ks * 32)
                                                       : umma::desc_kmajor(sa + ks * 2 * (BM * 16), BM * 16, 128);
                            const uint64_t bh = umma::desc_kmajor(hi_a + ks * 2 * a.lbo + shift, a.lbo, 128);
                            const uint64_t bl = umma::desc_kmajor(lo_a + ks * 2 * a.lbo + shift, a.lbo, 128);
                            umma::mma_f16(d, ad, bh, idesc, !first);
                            umma::mma_f16(d, ad, bl, idesc, true);
                            first = false;
                        }
                        if (!a.resident) umma::commit(&B.wempty[s]);
                    }
                    umma::commit(&B.aempty[b]);
                }
                umma::commit(&B.tfull[acc]);
            }
        }
    } else if (warp < 6) {
        // cursor over (unit, channel block, batch) of this CTA; the next position's loads
        // are in flight while the current batch is converted and stored
        const int u = threadIdx.x - 64;                  // 0..127
        const int kc = u & 7;
        const int per = 16 * SR<PRO>::n;
        const int nb = (a.wrows + per - 1) / per;        // batches per channel block
        int un = blockIdx.x, ci = 0, bi = 0, cg = 0;
        Unit w = unit_of(a, un);
        Rows<PRO> cur, nxt;
        load_rows<PRO>(cur, a, (w.c_begin + ci) * BK + kc * 8, w.t0, (u >> 3) + bi * per);
        while (un < n_units) {
            int un2 = un, ci2 = ci, bi2 = bi + 1;
            Unit w2 = w;
            if (bi2 == nb) {
                bi2 = 0;
                if (++ci2 == w.nc) {
                    ci2 = 0;
                    un2 += gridDim.x;
                    if (un2 < n_units) w2 = unit_of(a, un2);
                }
            }
            if (un2 < n_units) load_rows<PRO>(nxt, a, (w2.c_begin + ci2) * BK + kc * 8, w2.t0, (u >> 3) + bi2 * per);
            const int b = cg & 1;
            if (bi == 0 && cg >= 2 && !bwait(&B.aempty[b], ((cg >> 1) - 1) & 1, B, a)) break;
            uint8_t * hi = win + (b * 2) * win_bytes + kc * a.lbo;
            store_rows<PRO>(cur, a, hi, hi + win_bytes, (w.c_begin + ci) * BK + kc * 8, (u >> 3) + bi * per);
            if (bi == nb - 1) {
                fence_proxy_async_smem();
                mbar_arrive(&B.afull[b]);
                ++cg;
            }
            cur = nxt;
            un = un2; ci = ci2; bi = bi2; w = w2;
        }
    } else {
        const int q = warp & 3;                          // tensor-memory lane quadrant of this warp
        if (a.hist_out) {
            // the next chunk's history, the last H rows of [hist; x], spread over every CTA's
            // epilogue threads while they wait for their first accumulator
            const int n = a.H * a.Cin, et = threadIdx.x - 6 * 32;
            for (int e = blockIdx.x * 128 + et; e < n; e += gridDim.x * 128) {
                const int r = e / a.Cin, ch = e - r * a.Cin, src = r + a.T;
                a.hist_out[e] = src < a.H ? a.hist[static_cast<std::size_t>(src) * a.Cin + ch]
                                          : a.x[static_cast<std::size_t>(src - a.H) * a.x_stride + ch];
            }
        }
        int k = 0;
        for (int un = blockIdx.x; un < n_units; un += gridDim.x, ++k) {
            const Unit w = unit_of(a, un);
            const int acc = k & 1;
            const bool ok = bwait(&B.tfull[acc], (k >> 1) & 1, B, a);
            umma::fence_after_sync();
            epilogue_unit<EPI>(a, w, tmem + static_cast<uint32_t>(acc * a.BN), q, lane, ok);
            umma::fence_before_sync();
            mbar_arrive(&B.tempty[acc]);
        }
        mbar_arrive(&B.edone);                           // no tensor-memory reads after this
    }
    // Free the accumulators only after every epilogue thread's last tensor-memory read.
    if (warp == 1) {
        if (lane == 0) bwait_drain(&B.edone, 0, a);
        __syncwarp();
        umma::fence_after_sync();
        umma::tmem_dealloc(tmem, a.tmem_cols);
    }
}

// Split-K reduction: y[t][co] = epi(bias[co] + sum over splits, in split order, of the
// partial sums) -- one thread per output, up to eight splits' loads in flight at a time.
template <int EPI>
__global__ void k_splitk_reduce(const float * partial, int splits, int T, int Cout, const float * bias, const float * scale,
                                const float * resid, int r_stride, float * y, int y_stride) {
    navi::dev::griddep_wait();
    navi::dev::griddep_launch_dependents();
    const std::size_t n = static_cast<std::size_t>(T) * Cout;
    const std::size_t i = static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int t = static_cast<int>(i / Cout), co = static_cast<int>(i % Cout);
    const float acc = sum_slices(partial + i, splits, n);
    const float v = acc + (bias ? bias[co] : 0.f);
    const float r = (EPI == EPI_RESIDUAL || EPI == EPI_SCALE_RESIDUAL) ? resid[static_cast<std::size_t>(t) * r_stride + co] : 0.f;
    y[static_cast<std::size_t>(t) * y_stride + co] = finish<EPI>(v, EPI == EPI_SCALE_RESIDUAL ? scale[co] : 1.f, r);
}

// Split-K reduction fused with the RMS norm that follows the conv, one CTA of RN_THREADS
// threads per row t (a thread per channel, so the partial loads have the parallelism of
// k_splitk_reduce): y[t] as k_splitk_reduce computes it (splits == 0: y[t] is already
// final, written by the conv's own epilogue), then norm_out[t][co] = y[t][co] *
// rsqrt(mean(y[t]^2) + eps) * norm_w[co] (the decoder transformer's RMSNorm:
// model/qwen3tts/kernels.h:342, called at model/qwen3tts/vocoder.hip:274, 285, 291).
constexpr int RN_THREADS = 1024;

template <int EPI>
__global__ void __launch_bounds__(RN_THREADS) k_reduce_norm(const float * partial, int splits, int T, int Cout, const float * bias,
                                                            const float * scale, const float * resid, int r_stride, float * y,
                                                            int y_stride, const float * norm_w, float eps, float * norm_out) {
    griddep_wait();
    griddep_launch_dependents();
    __shared__ float red[RN_THREADS / 32];
    const std::size_t n = static_cast<std::size_t>(T) * Cout;
    const int t = blockIdx.x;
    float * yr = y + static_cast<std::size_t>(t) * y_stride;
    float ss = 0.f;
    for (int co = threadIdx.x; co < Cout; co += RN_THREADS) {
        float v;
        if (splits > 0) {
            const float acc = sum_slices(partial + static_cast<std::size_t>(t) * Cout + co, splits, n);
            const float r = (EPI == EPI_RESIDUAL || EPI == EPI_SCALE_RESIDUAL) ? resid[static_cast<std::size_t>(t) * r_stride + co] : 0.f;
            v = finish<EPI>(acc + (bias ? bias[co] : 0.f), EPI == EPI_SCALE_RESIDUAL ? scale[co] : 1.f, r);
            yr[co] = v;
        } else {
            v = yr[co];
        }
        ss += v * v;
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int k = 0; k < RN_THREADS / 32; ++k) tot += red[k];
    const float inv = rsqrtf(tot / static_cast<float>(Cout) + eps);
    float * nr = norm_out + static_cast<std::size_t>(t) * Cout;
    for (int co = threadIdx.x; co < Cout; co += RN_THREADS) nr[co] = yr[co] * inv * norm_w[co];
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
void launch_t(const KArgs & ka, const CUtensorMap & tm, dim3 grid, std::size_t smem, cudaStream_t stream, bool reduce) {
    static std::atomic<uint64_t> attr{0};   // devices whose attribute is set, one bit per ordinal < 64
    int dev = 0;
    NAVI_CUDA(cudaGetDevice(&dev));
    const uint64_t bit = 1ull << (dev & 63);
    if (!(attr.load() & bit)) {
        NAVI_CUDA(cudaFuncSetAttribute(k_conv<PRO, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_MAX));
        attr.fetch_or(bit);
    }
    NAVI_CUDA(navi::dev::launch_pdl(k_conv<PRO, EPI>, grid, dim3(NTHREADS), smem, stream, ka, tm));
    if (!reduce) return;
    if (ka.norm_out) {
        NAVI_CUDA(navi::dev::launch_pdl(k_reduce_norm<EPI>, dim3(static_cast<unsigned>(ka.T)), dim3(RN_THREADS), 0, stream, ka.partial,
                                        ka.splits > 1 ? ka.splits : 0, ka.T, ka.Cout, ka.bias, ka.scale, ka.resid, ka.r_stride, ka.y,
                                        ka.y_stride, ka.norm_w, ka.norm_eps, ka.norm_out));
    } else if (ka.splits > 1) {
        const std::size_t n = static_cast<std::size_t>(ka.T) * ka.Cout;
        NAVI_CUDA(navi::dev::launch_pdl(k_splitk_reduce<EPI>, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, stream, ka.partial,
                                        ka.splits, ka.T, ka.Cout, ka.bias, ka.scale, ka.resid, ka.r_stride, ka.y, ka.y_stride));
    }
}

__global__ void k_fold_bias(const float * b, int n, int phases, float * out) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n * phases; i += gridDim.x * blockDim.x) out[i] = b[i % n];
}

int lbo_for(int wrows) { return ((wrows + 7) / 8 * 8 + 1) * 16; }   // plane stride = 16 (mod 128): conflict-free stores
std::size_t win_bytes_for(int BN, int H) { return 4ull * 8 * lbo_for(BN + H); }
std::size_t smem_for(int BN, int H, int nst = NSTAGE) { return static_cast<std::size_t>(nst) * TILE_BYTES + win_bytes_for(BN, H) + BARS_BYTES; }

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
    // Cost model (measured on B200): the MMA issuer is the bottleneck at small row tiles
    // (about 65 ns per tcgen05.mma for N up to 128 at the clocks these short launches run
    // at), so time ~ waves x (MMAs per unit); a unit also pays ~1 us of staging / epilogue
    // latency, a split-K launch a reduction pass.  Candidates: row tiles 256 .. 16 that fit
    // shared memory, channel-block splits 1 .. CB; the cheapest wins.
    double best = 1e30;
    for (int BN = 256; BN >= 16; BN /= 2) {
        if (smem_for(BN, H) > static_cast<std::size_t>(SMEM_MAX)) continue;
        if (BN > 16 && BN / 2 >= c.T) continue;                      // a smaller tile covers every row
        const int tiles = p.MT * ceil_div(c.T, BN);
        for (int want = 1; want <= p.CB; want = want < p.CB ? std::min(p.CB, want * 2) : p.CB + 1) {
            const int cbps = ceil_div(p.CB, want), splits = ceil_div(p.CB, cbps);
            const int units = tiles * splits;
            const double waves = static_cast<double>(ceil_div(units, sms));
            const double unit_us = cbps * c.K * (2.0 * BK / 16) * 0.065 + 1.0 + BN / 256.0;
            double us = waves * unit_us;
            if (splits > 1) us += 3.0 + static_cast<double>(splits + 2) * c.T * c.Cout * 4.0 / 3.0e6;
            if (us < best - 1e-9) {
                best = us;
                p.BN = BN;
                p.NT = ceil_div(c.T, BN);
                p.splits = splits;
                p.cb_per_split = cbps;
            }
        }
    }
    p.lbo = lbo_for(p.BN + H);
    p.tmem_cols = std::max(32, 2 * p.BN);   // two accumulators: the epilogue of one unit overlaps the next
    // weight ring: every stage the shared memory left after the windows holds; the whole
    // tile set when every unit of a CTA uses the same tiles (one channel tile, no split)
    const int fit = static_cast<int>((SMEM_MAX - win_bytes_for(p.BN, H) - BARS_BYTES) / TILE_BYTES);
    const int max_st = std::min(MAXST, fit);
    p.resident = p.MT == 1 && p.splits == 1 && p.CB * c.K <= max_st;
    p.nst = p.resident ? p.CB * c.K : std::max(NSTAGE, max_st);
    p.smem = smem_for(p.BN, H, p.nst);
    if (p.smem > static_cast<std::size_t>(SMEM_MAX)) fail("conv: window of " + std::to_string(H) + " history rows does not fit", NAVI_E_SHAPE);
    return p;
}

void weight_map(const __half * w, int Cout, int Cin, int ld, void * out) {
    if ((reinterpret_cast<std::uintptr_t>(w) & 15u) || ld % 8 || ld < Cin)
        fail("conv: row-major weights need a 16-byte aligned base and a row stride multiple of 8 >= Cin", NAVI_E_SHAPE);
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(Cin), static_cast<cuuint64_t>(Cout)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
    const cuuint32_t box[2] = {BK, BM};   // 64 f16 = 128 B inner (the swizzle span) x 128 rows
    const cuuint32_t estr[2] = {1, 1};
    // the driver entry point is looked up at run time, so the library loads without libcuda
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    if (!encode) {
        cudaDriverEntryPointQueryResult q{};
        void * fn = nullptr;
        NAVI_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
        if (q != cudaDriverEntryPointSuccess || !fn) fail("conv: cuTensorMapEncodeTiled unavailable", NAVI_E_CUDA);
        encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    const CUresult r = encode(static_cast<CUtensorMap *>(out), CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half *>(w), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) fail("conv: cuTensorMapEncodeTiled failed (" + std::to_string(static_cast<int>(r)) + ")", NAVI_E_CUDA);
}

std::size_t partial_need(const Conv & c, int sms) {
    const Plan p = plan(c, sms);
    return p.splits > 1 ? static_cast<std::size_t>(p.splits) * c.T * c.Cout : 0;
}

int launch(const Conv & c, const Workspace & ws, int sms, cudaStream_t stream) {
    if (c.T <= 0) return 0;
    if (c.Cin % 8 || c.x_stride % 4 || c.K < 1 || c.dil < 1 || !(c.w || c.w_rm) || !c.x || !c.y)
        fail("conv: Cin and the input row stride must be multiples of 8 and 4", NAVI_E_SHAPE);
    if ((reinterpret_cast<std::uintptr_t>(c.x) | reinterpret_cast<std::uintptr_t>(c.hist) | reinterpret_cast<std::uintptr_t>(c.w)) & 15u)
        fail("conv: input, history and weights must be 16-byte aligned", NAVI_E_SHAPE);
    if (c.pro == PRO_SNAKE && (!c.snake_a || !c.snake_b || ((reinterpret_cast<std::uintptr_t>(c.snake_a) | reinterpret_cast<std::uintptr_t>(c.snake_b)) & 15u)))
        fail("conv: Snake coefficients missing or misaligned", NAVI_E_SHAPE);
    if (c.pro == PRO_SILU_GATE && c.hist) fail("conv: gated input has no history", NAVI_E_SHAPE);
    if (c.x_slices != 1 && (c.x_slices != 2 || c.pro != PRO_SILU_GATE || c.x_slice_stride % 4 ||
                            c.x_slice_stride < static_cast<std::size_t>(c.T) * c.x_stride))
        fail("conv: a folded reduction takes the 2 partial slices of a gated input, 16-byte aligned and apart", NAVI_E_SHAPE);
    if (c.hist_out && c.hist_out == c.hist) fail("conv: the next history needs a buffer of its own", NAVI_E_ARG);
    if ((c.epi == EPI_RESIDUAL || c.epi == EPI_SCALE_RESIDUAL) && !c.resid) fail("conv: residual missing", NAVI_E_SHAPE);
    if (c.epi == EPI_SCALE_RESIDUAL && !c.scale) fail("conv: layer scale missing", NAVI_E_SHAPE);
    if (c.norm_w && (!c.norm_out || c.norm_out == c.y)) fail("conv: the row norm needs an output buffer of its own", NAVI_E_ARG);
    if (c.defer_reduce && (c.epi != EPI_NONE || c.norm_w)) fail("conv: a deferred split-K reduction takes no epilogue and no row norm", NAVI_E_ARG);
    const Plan p = plan(c, sms);
    if (p.splits > 1) {
        if (static_cast<std::size_t>(p.splits) * c.T * c.Cout > ws.partial_cap)
            fail("conv: split-K workspace too small", NAVI_E_SHAPE);
    }
    KArgs ka{};
    ka.w = c.w; ka.x = c.x; ka.hist = c.hist; ka.sa = c.snake_a; ka.sb = c.snake_b; ka.bias = c.bias;
    ka.resid = c.resid; ka.scale = c.scale; ka.y = c.y; ka.partial = ws.partial; ka.err = ws.err;
    ka.hist_out = c.hist ? c.hist_out : nullptr;
    ka.Cout = c.Cout; ka.Cin = c.Cin; ka.K = c.K; ka.dil = c.dil; ka.H = (c.K - 1) * c.dil; ka.T = c.T;
    ka.x_stride = c.x_stride; ka.y_stride = c.y_stride; ka.r_stride = c.r_stride;
    ka.x_slices = c.x_slices; ka.x_sstride = static_cast<long long>(c.x_slice_stride);
    ka.BN = p.BN; ka.NT = p.NT; ka.MT = p.MT; ka.CB = p.CB; ka.cb_per_split = p.cb_per_split; ka.splits = p.splits;
    ka.lbo = p.lbo; ka.wrows = p.BN + ka.H; ka.tmem_cols = p.tmem_cols; ka.timeout_ns = ws.timeout_ns;
    ka.nst = p.nst; ka.resident = p.resident ? 1 : 0;
    ka.early_weights = c.weights_settled ? 1 : 0;
    ka.norm_w = c.norm_w; ka.norm_out = c.norm_w ? c.norm_out : nullptr; ka.norm_eps = c.norm_eps;
    CUtensorMap tm;
    std::memset(&tm, 0, sizeof tm);
    if (c.w_rm) {
        if (c.K != 1) fail("conv: row-major (TMA) weights are for K == 1 layers", NAVI_E_SHAPE);
        weight_map(c.w_rm, c.Cout, c.Cin, c.w_ld, &tm);
        ka.tmaw = 1;
    }
    const dim3 grid(std::min(p.NT * p.MT * p.splits, sms));   // persistent: one CTA per SM at most
#define NAVI_CONV_CASE(PR, EP) \
    if (c.pro == PR && c.epi == EP) {                                                                      \
        launch_t<PR, EP>(ka, tm, grid, p.smem, stream, !c.defer_reduce);                                   \
        NAVI_CUDA(cudaGetLastError());                                                                     \
        return c.defer_reduce && p.splits > 1 ? p.splits : 0;                                              \
    }
    NAVI_CONV_CASE(PRO_NONE, EPI_NONE)
    NAVI_CONV_CASE(PRO_NONE, EPI_GELU)
    NAVI_CONV_CASE(PRO_NONE, EPI_SCALE_RESIDUAL)
    NAVI_CONV_CASE(PRO_SILU_GATE, EPI_SCALE_RESIDUAL)
    NAVI_CONV_CASE(PRO_SNAKE, EPI_NONE)
    NAVI_CONV_CASE(PRO_SNAKE, EPI_RESIDUAL)
    NAVI_CONV_CASE(PRO_NONE, EPI_RESIDUAL)
    NAVI_CONV_CASE(PRO_SNAKE, EPI_GELU)
    NAVI_CONV_CASE(PRO_NONE, EPI_SILU)
    NAVI_CONV_CASE(PRO_SILU_GATE, EPI_RESIDUAL)
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
        if (a.rowmajor) {
            if (P > 1 || a.K != 1) fail("conv: row-major weights are for K == 1 layers", NAVI_E_ARG);
            c.w_rm = reinterpret_cast<const __half *>(a.w);
            c.w_ld = a.Cin;
        } else {
            __half * wp = static_cast<__half *>(alloc(packed_elems(c.Cout, c.Cin, c.K) * sizeof(__half)));
            pack({ps}, c.Cout, c.Cin, c.K, wp, s);
            c.w = wp;
        }
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
        ws.err = static_cast<int *>(alloc(sizeof(int)));
        launch(c, ws, sms, s);
        int err = 0;
        NAVI_CUDA(cudaMemcpyAsync(&err, ws.err, sizeof(int), cudaMemcpyDeviceToHost, s));
        NAVI_CUDA(cudaStreamSynchronize(s));
        if (err) st = err == ERR_ALIGN ? NAVI_E_SHAPE : NAVI_E_TIMEOUT;
    } catch (...) {
        (void) cudaStreamSynchronize(s);
        for (void * p : own) (void) cudaFree(p);
        throw;
    }
    for (void * p : own) (void) cudaFree(p);
    if (st == NAVI_E_SHAPE) fail("conv: the weight ring is not 1024-byte aligned for the swizzled tiles", st);
    if (st != NAVI_OK) fail("conv: a tensor-core conv wait passed its deadline", st);
    return st;
}

} // namespace navi
