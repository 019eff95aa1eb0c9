// Implicit-GEMM causal Conv1d on the sm_100a tensor cores (tcgen05, accumulator in
// tensor memory): the vocoder's convolutions, transposed convolutions and linear layers
// (reference: model/qwen3tts/kernels.h:72-242, k_conv, and its ConvArgs).
//
//   y[t][co] = epi( bias[co] + sum_j sum_ci W[co][ci][j] * pro(x~[t - (K-1-j) dil][ci]) )
//
// x~[r] is row r of the input for r >= 0 and row H + r of the conv's history ([H][Cin],
// H = (K-1) dil, zeros when absent) for r < 0.  A transposed conv of stride s is the same
// sum with its s phases folded into the output channels (co' = phase * Cout + co, rows
// t * s + phase of a dense output), so it needs no special case here.
//
// GEMM view per CTA: D[co][t] (128 channels x BN rows, f32 in tensor memory) accumulates
// over (channel block of 64, tap): A = a 128 x 64 tile of the packed weights (bulk copy
// from global), B = the input window rows [t0 - H, t0 + BN) of that channel block in
// shared memory, read by tap j at a start row shifted by j * dil.  Activations enter the
// MMA as two f16 halves (hi = f16(v), lo = f16(v - hi)) against f16 weights, so the
// products keep ~21 bits of the f32 activation.
#pragma once

#include "runtime.hpp"

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <vector>

namespace navi::conv {

enum Pro : int { PRO_NONE = 0, PRO_SNAKE = 1, PRO_SILU_GATE = 2 };
enum Epi : int { EPI_NONE = 0, EPI_GELU = 1, EPI_RESIDUAL = 2, EPI_SCALE_RESIDUAL = 3, EPI_SILU = 4 };

constexpr int BM = 128;                      // output channels per tile (MMA M)
constexpr int BK = 64;                       // input channels per block
constexpr int TILE_ELEMS = BM * BK;          // one packed weight tile: [8 k chunks][128 co][8]
constexpr int TILE_BYTES = TILE_ELEMS * 2;
constexpr int NSTAGE = 4;                    // fewest weight tiles in flight per CTA
constexpr int NTHREADS = 320;                // warp 0 weights, warp 1 MMA, warps 2-5 windows, warps 6-9 epilogue

// One source block of a packed weight.  Logical weight W(co, tap, ci) for co in
// [co0, co1), ci in [ci0, ci1):
//   direct:  p[(co - co0) s_co + (ci - ci0) s_ci + tap s_tap]
//   trans:   p is a ConvTranspose1d weight [ci][cout_b][k] of stride `stride`; with
//            c = co - co0, phase = c / cout_b, m = taps - 1 - tap:
//            p[(ci - ci0) cout_b k + (c % cout_b) k + phase + m stride]   (vocoder.hip:373-385)
struct PackSrc {
    const __half * p = nullptr;
    int co0 = 0, co1 = 0, ci0 = 0, ci1 = 0;
    long long s_co = 0, s_ci = 0, s_tap = 0;
    int trans = 0, cout_b = 0, k = 0, stride = 0;
};
constexpr int MAX_PACK_SRC = 4;

inline int ceil_div(int a, int b) { return (a + b - 1) / b; }
inline std::size_t packed_elems(int Cout, int Cin, int K) {
    return static_cast<std::size_t>(ceil_div(Cout, BM)) * ceil_div(Cin, BK) * K * TILE_ELEMS;
}
// Writes the packed tiles of a [Cout][K][Cin] logical weight (zero outside every source).
void pack(const std::vector<PackSrc> & srcs, int Cout, int Cin, int K, __half * dst, cudaStream_t stream);

struct Conv {
    const __half * w = nullptr;              // packed tiles
    // or, for K == 1 (a linear layer), the weight as stored: row-major [Cout][w_ld] f16, read
    // by TMA in 128 x 64 boxes (16-byte aligned base, w_ld % 8 == 0); no packed copy needed
    const __half * w_rm = nullptr;
    int w_ld = 0;
    int Cout = 0, Cin = 0, K = 1, dil = 1;
    const float * x = nullptr;               // rows [T][x_stride]; SILU_GATE: row = [gate | up], Cin each
    int x_stride = 0, T = 0;
    // 2: x holds the 2 split-K partial slices an earlier launch left with defer_reduce (slice 1
    // at x + x_slice_stride, rows [T][x_stride] each); the staging sums them in slice order, the
    // values that launch's own reduction would have written (it must have had no bias).
    // PRO_SILU_GATE only.
    int x_slices = 1;
    std::size_t x_slice_stride = 0;
    const float * hist = nullptr;            // [H][Cin] or null
    // when set (with hist): receives the last H rows of [hist; x], i.e. the next chunk's
    // history, written by the launch itself ([H][Cin], a buffer other than hist)
    float * hist_out = nullptr;
    int pro = PRO_NONE;
    const float * snake_a = nullptr, * snake_b = nullptr;   // e^alpha, 1/(e^beta + 1e-9)   [Cin]
    int epi = EPI_NONE;
    const float * bias = nullptr;            // [Cout] or null
    const float * resid = nullptr;           // EPI_RESIDUAL / EPI_SCALE_RESIDUAL: rows [T][r_stride]
    int r_stride = 0;
    const float * scale = nullptr;           // EPI_SCALE_RESIDUAL: [Cout]
    float * y = nullptr;                     // rows [T][y_stride]
    int y_stride = 0;
    // true when no kernel still in flight in the stream writes the weights (they were packed
    // or uploaded before a synchronisation): the weight stream may then start before the
    // previous kernel in the stream has finished
    bool weights_settled = false;
    // when set: also writes norm_out[t][co] = y[t][co] * rsqrt(mean_co y[t][co]^2 + norm_eps)
    // * norm_w[co] (rows [T][Cout]), the RMS norm of a following layer, in the split-K
    // reduction's launch (or one row-norm launch when the conv is not split)
    const float * norm_w = nullptr;
    float * norm_out = nullptr;
    float norm_eps = 0.f;
    // when set: a split-K launch leaves its partial sums in the workspace for the caller to
    // reduce (slice k at partial + k T Cout, rows [T][Cout], bias not included); EPI_NONE only
    bool defer_reduce = false;
};

struct Plan {
    int BN = 16, NT = 1, MT = 1, CB = 1, splits = 1, cb_per_split = 1, lbo = 0, tmem_cols = 32;
    int nst = NSTAGE;                        // weight-ring stages
    bool resident = false;                   // weights loaded once per CTA
    std::size_t smem = 0;
};
Plan plan(const Conv & c, int sms);

// Values of the error word a conv launch leaves in Workspace::err (0: none).
constexpr int ERR_TIMEOUT = 1;               // a CTA's wait passed its deadline
constexpr int ERR_ALIGN = 2;                 // the weight ring misses the 1024-byte alignment of swizzled tiles

struct Workspace {
    float * partial = nullptr;               // split-K partial sums
    std::size_t partial_cap = 0;             // elements
    int * err = nullptr;                     // ERR_TIMEOUT / ERR_ALIGN, set by a failing CTA
    unsigned long long timeout_ns = 2000000000ull;
};
// Encodes the TMA map of a row-major [Cout][ld] f16 weight (out: a CUtensorMap).
void weight_map(const __half * w, int Cout, int Cin, int ld, void * out);
// Elements of split-K partial storage a launch of `c` needs.
std::size_t partial_need(const Conv & c, int sms);

// Returns the number of split-K partial slices left in ws.partial (Conv::defer_reduce), else 0
// (y holds the result).
int launch(const Conv & c, const Workspace & ws, int sms, cudaStream_t stream);

} // namespace navi::conv
