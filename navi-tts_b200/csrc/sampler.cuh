// The frame sampler, run by the NT consumer threads of a CTA.
//
// Semantics follow the reference's device sampler (model/qwen3tts/frame.hip):
// codebook-0 logit modifications tl_modified_logit (413-419); greedy argmax with
// the lowest index on ties (block_argmax 178-203); temperature, then the exact
// k-th largest by monotone float keys with 4 radix passes of 8 bits
// (block_kth_largest 225-256) and candidates v >= threshold; e_i = exp(v_i - max);
// the normaliser summed in the order of the reference's 256-thread block_sum
// (runtime/device/kernel_util.h:20-34); the multinomial walk over the nonzero e_i
// in index order (block_draw 263-296); PCG32 per-draw state and splitmix64 seeds
// (169-175, 284-286, 497, 581-586, 658-659).  Added here: top-p after top-k
// (candidates ordered by value descending, ties to the lower index; the shortest
// prefix whose cumulative probability reaches top_p is kept and renormalised) and
// a Philox4x32-10 stream keyed by the request seed with counter (frame, codebook).
//
// Every floating-point step is one IEEE binary32 rounding (explicit __f*_rn
// intrinsics, no contraction), and exp is this file's own exactly-specified
// function, so the draw is reproducible bit for bit on the host.
#pragma once

#include "device.cuh"

namespace navi::dev {


struct SampleCfg {
    float temperature;   // <= 0: greedy
    int top_k;           // 0 or >= V: off
    float top_p;         // outside (0, 1): off
    int rng;             // 0 PCG, 1 Philox
    uint64_t seed;       // request seed
    int frame_index;
    int codebook;        // 0 talker, 1.. code predictor
    uint64_t pcg_seed;   // per-draw PCG seed (host-computed splitmix64 chain)
    // codebook-0 modifications
    int talker_mods;
    int suppress_from, eos_id, min_frames;
    float repetition_penalty;
    const uint8_t * seen;   // global [V]
};

struct SampleScratch {
    float * s;        // [V] in: logits; then the modified, tempered values; then (top-p) keep flags
    float * e;        // [V] e^(v - max) of the candidates, 0 elsewhere
    int * idx;        // [V] candidate ids (nonzero e) in index order
    int * ord;        // [V] candidate masks; then (top-p) candidate positions by rank
    unsigned * hist;  // [2][256] radix histograms; [256, 384): values and e of the first 64 candidates
    float * red;      // [64]
};

// Floats of shared or global scratch the sampler takes for V logits (the layout of
// sampler_layout below).
__host__ __device__ constexpr uint32_t sample_scratch_floats(int V) { return 4u * V + 512 + 64; }

// The scratch arrays at base (16-byte aligned).
__host__ __device__ inline SampleScratch sampler_layout(float * base, int V) {
    SampleScratch sc;
    sc.s = base;
    sc.e = base + V;
    sc.idx = reinterpret_cast<int *>(base + 2 * V);
    sc.ord = reinterpret_cast<int *>(base + 3 * V);
    sc.hist = reinterpret_cast<unsigned *>(base + 4 * V);
    sc.red = base + 4 * V + 512;
    return sc;
}

// exp(x), exactly specified: Cody-Waite reduction x = n*ln2 + r (fdlibm hi/lo split
// of ln2), a degree-7 Taylor polynomial for e^r by Horner's rule with fused
// multiply-adds, and an exact power-of-two scaling with one final rounding.
__device__ __forceinline__ float pow2i(int k) { return __uint_as_float(static_cast<uint32_t>(k + 127) << 23); }

__device__ __forceinline__ float exp_spec(float x) {
    if (x != x) return x;
    if (x > 0x1.62e43p+6f) return __int_as_float(0x7f800000);
    if (x < -0x1.9fe36ap+6f) return 0.0f;
    const float n = rintf(__fmul_rn(x, 0x1.715476p+0f));
    float r = __fmaf_rn(-n, 0x1.62e4p-1f, x);
    r = __fmaf_rn(-n, 0x1.7f7d1cp-20f, r);
    float p = 0x1.a01a02p-13f;
    p = __fmaf_rn(p, r, 0x1.6c16c2p-10f);
    p = __fmaf_rn(p, r, 0x1.111112p-7f);
    p = __fmaf_rn(p, r, 0x1.555556p-5f);
    p = __fmaf_rn(p, r, 0x1.555556p-3f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    int ni = static_cast<int>(n);
    if (ni > 127) { p = __fmul_rn(p, pow2i(127)); ni -= 127; }
    else if (ni < -126) { p = __fmul_rn(p, pow2i(ni + 64)); ni = -64; }
    return __fmul_rn(p, pow2i(ni));
}

__host__ __device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

// The per-draw PCG seed (frame.hip:581-586, 658-659, 497): the talker's stream is
// splitmix64(seed ^ frame * 0xA24BAED4963EE407); codebook c >= 1 of the code predictor uses
// splitmix64(talker ^ 0x9FB21C651E98DF25) + c * 0xD1B54A32D192ED03. The frame launch and the
// standalone samplers all derive their seeds here.
__host__ __device__ __forceinline__ uint64_t pcg_draw_seed(uint64_t seed, int frame_index, int codebook) {
    const uint64_t tl = splitmix64(seed ^ (static_cast<uint64_t>(static_cast<int64_t>(frame_index)) * 0xA24BAED4963EE407ull));
    if (codebook == 0) return tl;
    return splitmix64(tl ^ 0x9FB21C651E98DF25ull) + static_cast<uint64_t>(codebook) * 0xD1B54A32D192ED03ull;
}

__device__ __forceinline__ uint32_t pcg32_next(uint64_t & s) {
    const uint64_t old = s;
    s = old * 6364136223846793005ull + 1442695040888963407ull;
    const uint32_t xs = static_cast<uint32_t>(((old >> 18u) ^ old) >> 27u);
    const uint32_t rot = static_cast<uint32_t>(old >> 59u);
    return (xs >> rot) | (xs << ((0u - rot) & 31u));
}

__device__ __forceinline__ uint32_t philox_word0(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint32_t k0, uint32_t k1) {
#pragma unroll
    for (int round = 0; round < 10; ++round) {
        const uint32_t lo0 = 0xD2511F53u * c0, hi0 = __umulhi(0xD2511F53u, c0);
        const uint32_t lo1 = 0xCD9E8D57u * c2, hi1 = __umulhi(0xCD9E8D57u, c2);
        const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
        c0 = n0; c1 = lo1; c2 = n2; c3 = lo0;
        k0 += 0x9E3779B9u; k1 += 0xBB67AE85u;
    }
    return c0;
}

__device__ __forceinline__ float draw_uniform(const SampleCfg & c) {
    uint32_t w;
    if (c.rng == 0) {
        uint64_t st = c.pcg_seed * 0x9E3779B97F4A7C15ull + 0xBF58476D1CE4E5B9ull + 1ull;
        (void) pcg32_next(st); (void) pcg32_next(st); (void) pcg32_next(st);
        w = pcg32_next(st);
    } else {
        w = philox_word0(static_cast<uint32_t>(c.frame_index), static_cast<uint32_t>(c.codebook), 0u, 0u,
                         static_cast<uint32_t>(c.seed), static_cast<uint32_t>(c.seed >> 32));
    }
    return __fmul_rn(static_cast<float>(w >> 8), 1.0f / 16777216.0f);
}

__device__ __forceinline__ uint32_t float_key(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_float(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// Bin of a value's distance below the block max (mx - v >= 0; +inf for v = -inf): the
// distance's exponent and top five mantissa bits, 32 bins an octave from 2^-3 (bin 0 also
// takes every smaller distance) to 2^5 (bin 255 also takes every larger one). The bin never
// decreases as the distance grows, so it never increases with v: every value of a lower bin
// is larger than every value of a higher one.
__device__ __forceinline__ int dist_bin(float mx, float v) {
    const int key = static_cast<int>(__float_as_uint(__fsub_rn(mx, v)) >> 18) - (124 << 5);
    return min(max(key, 0), 255);
}

// The k-th largest of s[0..V) by monotone float keys: 8-bit radix passes, top byte first, one
// warp resolving the digit from the histogram (2 barriers a pass); the passes stop early once
// the bin holding the k-th key holds exactly the keys still needed (then every key of that bin
// is a candidate, and a threshold with the low bits zero selects the same set; not used when
// that threshold would be +0, where -0 compares equal). The top byte (sign and exponent) puts
// most keys in a handful of bins, so that pass counts into one histogram per warp (in e and
// idx, unused until the candidates are formed) when they fit. Called by all NT threads.
template <int NT>
__device__ __forceinline__ float kth_radix(int V, int kth, const SampleScratch & S, int bid) {
    constexpr int NW = NT / 32;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const float * s = S.s;
    unsigned * hist = S.hist;
    int * ired = reinterpret_cast<int *>(S.red);
    unsigned * whist = reinterpret_cast<unsigned *>(S.e);
    const bool priv = NW * 256 <= 2 * V;
    for (int i = tid; i < 512; i += NT) hist[i] = 0u;
    if (priv)
        for (int i = tid; i < NW * 256; i += NT) whist[i] = 0u;
    named_sync(bid, NT);
    uint32_t prefix = 0, mask = 0;
    int need = kth;
    for (int pass = 3; pass >= 0; --pass) {
        const int shift = pass * 8;
        unsigned * h = hist + (pass & 1) * 256;
        if (pass == 3 && priv) {
            unsigned * hw = whist + wid * 256;
            for (int i = tid; i < V; i += NT) atomicAdd(&hw[float_key(s[i]) >> 24], 1u);
            named_sync(bid, NT);
            for (int b = tid; b < 256; b += NT) {
                unsigned t = 0;
#pragma unroll
                for (int w = 0; w < NW; ++w) t += whist[w * 256 + b];
                h[b] = t;
            }
        } else {
            for (int i = tid; i < V; i += NT) {
                const uint32_t key = float_key(s[i]);
                if ((key & mask) == prefix) atomicAdd(&h[(key >> shift) & 0xFFu], 1u);
            }
        }
        named_sync(bid, NT);
        const int slot = 16 + 3 * (3 - pass);
        if (wid == 0) {
            // lane l holds digits 255 - 8l - k (k < 8), counted from the top digit down
            int cnt[8], tot = 0;
#pragma unroll
            for (int k = 0; k < 8; ++k) { cnt[k] = static_cast<int>(h[255 - 8 * lane - k]); tot += cnt[k]; }
            int incl = tot;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += v;
            }
            const int above = incl - tot;
            if (above < need && incl >= need) {
                int a = above;
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    if (a + cnt[k] >= need) {
                        ired[slot] = 255 - 8 * lane - k;
                        ired[slot + 1] = need - a;
                        ired[slot + 2] = cnt[k];
                        break;
                    }
                    a += cnt[k];
                }
            }
            // this buffer is used again two passes on
#pragma unroll
            for (int k = 0; k < 8; ++k) h[8 * lane + k] = 0u;
        }
        named_sync(bid, NT);
        need = ired[slot + 1];
        prefix |= static_cast<uint32_t>(ired[slot]) << shift;
        mask |= 0xFFu << shift;
        if (ired[slot + 2] == need && key_float(prefix) != 0.0f) break;
    }
    return key_float(prefix);
}

// kth_radix as a call: keeps the rarely taken radix path out of the caller's code
template <int NT>
__device__ __noinline__ float kth_radix_call(int V, int kth, const SampleScratch & S, int bid) {
    return kth_radix<NT>(V, kth, S, bid);
}

// Samples from S.s[0..V) (the raw logits on entry). Must be called by all NT threads (NT a
// multiple of 32, 320..1024: at least ten warps; barrier id `bid`); every thread returns the
// chosen id, the host oracle's bit for bit.
//
// Work plan, laid out to keep CTA barriers few (each costs the slowest warp's lag, and a frame
// runs the sampler on its critical path sixteen times):
//  1. modifications and temperature, block max; the barrier also ORs a NaN flag (1 barrier);
//  2. top-k threshold, the k-th largest value: a histogram of the values' distances below the
//     max in log-spaced bins (dist_bin; 1 barrier); every warp finds the bin where the count
//     from the top reaches k; the values of that bin are gathered (1 barrier) and every warp
//     finds the k-th largest among them by counting. A bin of more than 64 values, a
//     non-finite max or a NaN take the radix select of the keys (kth_radix) instead;
//  3. e = exp(v - max) over the candidates v >= threshold, and one ballot mask of nonzero e
//     per 32 consecutive ids (1 barrier);
//  4. the normaliser in the reference's 256-thread block_sum order by warps 0-7 (warp 7 also
//     draws the uniform) while the other warps compact the candidates in index order from the
//     masks, keeping the values and e of the first 64 (1 barrier);
//  5. top-p ranks by (value desc, index asc): for up to 64 candidates in warp 0, else by all
//     threads (1 more barrier); the sequential sums (top-p cut, renormaliser, draw) in warp 0,
//     values passed lane to lane by shuffles.
// OUTLINE: the radix path is a call rather than inlined. Which is faster depends on the
// caller: the single-stream frame program is faster with the call (its loop's code is
// smaller: one launch 2,063 -> 2,049 us), the batched one, which runs at its register limit,
// is slower with it (3.61 -> 3.80 ms: a call constrains the register allocation around it).
template <int NT, bool OUTLINE = false>
__device__ int sample_cta(int V, const SampleCfg & c, const SampleScratch & S, int bid) {
    constexpr int NW = NT / 32;
    static_assert(NT % 32 == 0 && NT >= 320 && NT <= 1024, "sampler thread count");
    constexpr int SMALL = 64;                                   // gathered bin / candidate list of the fast paths
    constexpr int RB_CNT = 48, RB_U = 50, RB_CHOSEN = 60, RB_N = 61;   // slots of red
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    float * s = S.s;
    float * e = S.e;
    int * ci = S.idx;
    float * red = S.red;
    int * ired = reinterpret_cast<int *>(S.red);
    unsigned * hist = S.hist;
    float * cv = reinterpret_cast<float *>(hist + 256);         // values of the first SMALL candidates
    float * ce = reinterpret_cast<float *>(hist + 256 + SMALL); // and their e
    // 1. codebook-0 modifications, temperature, max; the distance histogram and gather count cleared
    const bool greedy = c.temperature <= 0.f;
    const bool topk = !greedy && c.top_k > 0 && c.top_k < V;
    for (int i = tid; i < 256; i += NT) hist[i] = 0u;
    if (tid == 0) ired[RB_CNT] = 0;
    float lmax = -INFINITY;
    bool nan = false;
    for (int i = tid; i < V; i += NT) {
        float v = s[i];
        if (c.talker_mods) {
            if (i >= c.suppress_from && i != c.eos_id) v = -INFINITY;
            else if (i == c.eos_id && c.frame_index < c.min_frames) v = -INFINITY;
            else if (c.repetition_penalty > 0.f && c.seen[i]) v = (v > 0.f) ? __fdiv_rn(v, c.repetition_penalty) : __fmul_rn(v, c.repetition_penalty);
        }
        if (!greedy) v = __fdiv_rn(v, c.temperature);
        s[i] = v;
        lmax = fmaxf(lmax, v);
        nan = nan || v != v;
    }
    lmax = warp_max(lmax);
    if (lane == 0) red[wid] = lmax;
    const bool anynan = named_sync_or(bid, NT, nan);
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) mx = fmaxf(mx, red[w]);
    if (greedy) {
        // lowest index holding the maximum (index 0 when every value is -inf)
        int best = V;
        for (int i = tid; i < V; i += NT) if (s[i] == mx) { best = i; break; }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) best = min(best, __shfl_xor_sync(0xffffffffu, best, o));
        if (lane == 0) ired[32 + wid] = best;
        named_sync(bid, NT);
        int b = V;
#pragma unroll
        for (int w = 0; w < NW; ++w) b = min(b, ired[32 + w]);
        named_sync(bid, NT);
        return b >= V ? 0 : b;
    }
    // 2. the top-k threshold
    float threshold = -INFINITY;
    if (topk) {
        const int k = c.top_k;
        bool fast = !anynan && mx > -INFINITY && mx < INFINITY;
        int bstar = 0, needb = 0, cntb = 0;
        if (fast) {
            for (int i = tid; i < V; i += NT) atomicAdd(&hist[dist_bin(mx, s[i])], 1u);
            named_sync(bid, NT);
            // every warp: lane l holds bins 8l..8l+7; the bin where the count from bin 0 reaches k
            const uint4 h0 = reinterpret_cast<const uint4 *>(hist)[2 * lane], h1 = reinterpret_cast<const uint4 *>(hist)[2 * lane + 1];
            const int cnt[8] = {static_cast<int>(h0.x), static_cast<int>(h0.y), static_cast<int>(h0.z), static_cast<int>(h0.w),
                                static_cast<int>(h1.x), static_cast<int>(h1.y), static_cast<int>(h1.z), static_cast<int>(h1.w)};
            int tot = 0;
#pragma unroll
            for (int q = 0; q < 8; ++q) tot += cnt[q];
            int incl = tot;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += v;
            }
            const bool mine = incl - tot < k && incl >= k;
            int b_ = 0, n_ = 0, c_ = 0;
            if (mine) {
                int a = incl - tot;
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    if (a + cnt[q] >= k) { b_ = 8 * lane + q; n_ = k - a; c_ = cnt[q]; break; }
                    a += cnt[q];
                }
            }
            const int src = __ffs(__ballot_sync(0xffffffffu, mine)) - 1;
            bstar = __shfl_sync(0xffffffffu, b_, src);
            needb = __shfl_sync(0xffffffffu, n_, src);
            cntb = __shfl_sync(0xffffffffu, c_, src);
            if (cntb > SMALL) {
                fast = false;
                named_sync(bid, NT);   // every warp has read the histogram before kth_radix clears it
            }
        }
        if (fast) {
            // the values of bin bstar, then (every warp) the needb-th largest of them: the value
            // with fewer than needb values above it and at least needb at or above it
            float * list = reinterpret_cast<float *>(ci);
            for (int i = tid; i < V; i += NT) {
                const float v = s[i];
                if (dist_bin(mx, v) == bstar) list[atomicAdd(&ired[RB_CNT], 1)] = v;
            }
            named_sync(bid, NT);
            const float x0 = lane < cntb ? list[lane] : 0.f, x1 = lane + 32 < cntb ? list[lane + 32] : 0.f;
            int g0 = 0, e0 = 0, g1 = 0, e1 = 0;
#pragma unroll 4
            for (int m = 0; m < cntb; ++m) {
                const float y = list[m];
                g0 += y > x0 ? 1 : 0;
                e0 += y >= x0 ? 1 : 0;
                g1 += y > x1 ? 1 : 0;
                e1 += y >= x1 ? 1 : 0;
            }
            const unsigned b0 = __ballot_sync(0xffffffffu, lane < cntb && g0 < needb && needb <= e0);
            const unsigned b1 = __ballot_sync(0xffffffffu, lane + 32 < cntb && g1 < needb && needb <= e1);
            threshold = b0 ? __shfl_sync(0xffffffffu, x0, __ffs(b0) - 1) : __shfl_sync(0xffffffffu, x1, __ffs(b1) - 1);
        } else {
            threshold = OUTLINE ? kth_radix_call<NT>(V, k, S, bid) : kth_radix<NT>(V, k, S, bid);
        }
    }
    // 3. e over the candidates; one ballot mask of nonzero e per (round, warp): 32 consecutive ids
    const int R = (V + NT - 1) / NT;
    unsigned * masks = reinterpret_cast<unsigned *>(S.ord);   // [R][NW]
    for (int k = 0; k < R; ++k) {
        const int i = k * NT + tid;
        float ev = 0.f;
        if (i < V) {
            const float v = s[i];
            if (v >= threshold) ev = exp_spec(__fsub_rn(v, mx));
            e[i] = ev;
        }
        const unsigned m = __ballot_sync(0xffffffffu, ev != 0.f);
        if (lane == 0) masks[k * NW + wid] = m;
    }
    named_sync(bid, NT);
    // 4. normaliser (warps 0-7) and compaction (warps 8..NW-1, a contiguous share of the masks each)
    if (wid < 8) {
        float acc = 0.f;
        for (int i = tid; i < V; i += 256) acc = __fadd_rn(acc, e[i]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
        if (lane == 0) red[32 + wid] = acc;
        if (wid == 7 && lane == 0) red[RB_U] = draw_uniform(c);
    } else {
        constexpr int CW = NW - 8;
        const int M = R * NW;
        const int q0 = (M * (wid - 8)) / CW, q1 = (M * (wid - 7)) / CW;
        int before = 0;
        for (int q = lane; q < q0; q += 32) before += __popc(masks[q]);
        int run = static_cast<int>(__reduce_add_sync(0xffffffffu, static_cast<unsigned>(before)));
        for (int m0 = q0; m0 < q1; m0 += 32) {
            const int q = m0 + lane;
            const unsigned m = q < q1 ? masks[q] : 0u;
            const int cnt = __popc(m);
            int incl = cnt;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += v;
            }
            // mask q covers ids (q / NW) * NT + (q % NW) * 32 + bit
            const int first = (q / NW) * NT + (q % NW) * 32;
            int at = run + incl - cnt;
            for (unsigned bb = m; bb; bb &= bb - 1) {
                const int i = first + __ffs(bb) - 1;
                ci[at] = i;
                if (at < SMALL) {
                    cv[at] = s[i];
                    ce[at] = e[i];
                }
                ++at;
            }
            run += __shfl_sync(0xffffffffu, incl, 31);
        }
        if (wid == NW - 1 && lane == 0) ired[RB_N] = run;
    }
    named_sync(bid, NT);
    const int n = ired[RB_N];
    // 5. top-p order and the draw
    const bool nucleus = c.top_p > 0.f && c.top_p < 1.f;
    const bool small = n <= SMALL;
    int * ord = S.ord;   // top-p: candidate position of each rank (the masks are no longer needed)
    if (nucleus && !small) {
        // thread j reads the other candidates' values from shared memory (every thread of a step
        // reads the same element: a broadcast), eight independent loads per step
        for (int j = tid; j < n; j += NT) {
            const float vj = s[ci[j]];
            int r = 0, m = 0;
#pragma unroll 1
            for (; m + 8 <= n; m += 8) {
                float vm[8];
#pragma unroll
                for (int q = 0; q < 8; ++q) vm[q] = s[ci[m + q]];
#pragma unroll
                for (int q = 0; q < 8; ++q) r += (vm[q] > vj || (vm[q] == vj && m + q < j)) ? 1 : 0;
            }
#pragma unroll 1
            for (; m < n; ++m) {
                const float v = s[ci[m]];
                r += (v > vj || (v == vj && m < j)) ? 1 : 0;
            }
            ord[r] = j;
        }
        named_sync(bid, NT);
    }
    if (wid == 0) {
        float ssum = lane < 8 ? red[32 + lane] : 0.f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ssum = __fadd_rn(ssum, __shfl_xor_sync(0xffffffffu, ssum, o));
        const float inv = __fdiv_rn(1.0f, ssum);
        const float u = red[RB_U];
        const auto ev = [&](int j) { return small ? ce[j] : e[ci[j]]; };   // e of candidate position j
        if (nucleus && small) {
            // ranks in this warp: lane l takes positions l and l + 32
            const float x0 = lane < n ? cv[lane] : 0.f, x1 = lane + 32 < n ? cv[lane + 32] : 0.f;
            int r0 = 0, r1 = 0;
#pragma unroll 4
            for (int m = 0; m < n; ++m) {
                const float y = cv[m];
                r0 += (y > x0 || (y == x0 && m < lane)) ? 1 : 0;
                r1 += (y > x1 || (y == x1 && m < lane + 32)) ? 1 : 0;
            }
            if (lane < n) ord[r0] = lane;
            if (lane + 32 < n) ord[r1] = lane + 32;
            __syncwarp();
        }
        // Sequential sums, 32 terms per block: every lane gathers the block's 32 values by
        // shuffles (independent, so they overlap), then runs the same in-order __fadd_rn chain
        // over them straight through, keeping the running sum at its own position; a ballot
        // finds the first position past the target. The additions are the same, in the same
        // order, as one sequential loop, so the results are too.
        auto block_scan = [&](float acc, float v, float & mine) {
#pragma unroll 1
            for (int g = 0; g < 32; g += 8) {   // eight values gathered per group: few live registers
                float t[8];
#pragma unroll
                for (int q = 0; q < 8; ++q) t[q] = __shfl_sync(0xffffffffu, v, g + q);
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    acc = __fadd_rn(acc, t[q]);
                    if (g + q == lane) mine = acc;
                }
            }
            return acc;
        };
        int chosen;
        if (nucleus) {
            // the shortest prefix by rank whose cumulative probability reaches top_p: ranks <= Rk
            float cum = 0.f;
            int Rk = n - 1;
            for (int r0 = 0; r0 < n; r0 += 32) {
                const bool in = r0 + lane < n;
                const float p = in ? __fmul_rn(ev(ord[r0 + lane]), inv) : 0.f;
                float mine = 0.f;
                cum = block_scan(cum, p, mine);
                const unsigned hit = __ballot_sync(0xffffffffu, in && mine >= c.top_p);
                if (hit) {
                    Rk = r0 + __ffs(hit) - 1;
                    break;
                }
            }
            // keep flags by candidate position (the values in s are no longer needed)
            float * kept = s;
            for (int j = lane; j < n; j += 32) kept[j] = 0.f;
            __syncwarp();
            for (int r = lane; r <= Rk; r += 32) kept[ord[r]] = 1.f;
            __syncwarp();
            // renormalise over the kept candidates, in index order; adding the 0 of a dropped
            // candidate leaves a sum unchanged
            float ksum = 0.f;
            int last = V - 1;
            for (int j0 = 0; j0 < n; j0 += 32) {
                const int j = j0 + lane;
                const bool kp = j < n && kept[j] != 0.f;
                const int ii = j < n ? ci[j] : 0;
                const float evj = kp ? ev(j) : 0.f;
                const unsigned km = __ballot_sync(0xffffffffu, kp);
                float mine = 0.f;
                ksum = block_scan(ksum, evj, mine);
                if (km) last = __shfl_sync(0xffffffffu, ii, 31 - __clz(km));
            }
            const float kinv = __fdiv_rn(1.0f, ksum);
            chosen = last;
            float c2 = 0.f;
            for (int j0 = 0; j0 < n; j0 += 32) {
                const int j = j0 + lane;
                const bool kp = j < n && kept[j] != 0.f;
                const int ii = j < n ? ci[j] : 0;
                const float pv = kp ? __fmul_rn(ev(j), kinv) : 0.f;
                float mine = 0.f;
                c2 = block_scan(c2, pv, mine);
                const unsigned hit = __ballot_sync(0xffffffffu, kp && mine >= u);
                if (hit) {
                    chosen = __shfl_sync(0xffffffffu, ii, __ffs(hit) - 1);
                    break;
                }
            }
        } else {
            chosen = V - 1;
            float cum = 0.f;
            for (int j0 = 0; j0 < n; j0 += 32) {
                const int j = j0 + lane;
                const int ii = j < n ? ci[j] : 0;
                const float p = j < n ? __fmul_rn(ev(j), inv) : 0.f;
                float mine = 0.f;
                cum = block_scan(cum, p, mine);
                const unsigned hit = __ballot_sync(0xffffffffu, j < n && mine >= u);
                if (hit) {
                    chosen = __shfl_sync(0xffffffffu, ii, __ffs(hit) - 1);
                    break;
                }
            }
        }
        if (lane == 0) ired[RB_CHOSEN] = chosen;
    }
    named_sync(bid, NT);
    const int chosen = ired[RB_CHOSEN];
    named_sync(bid, NT);
    return chosen;
}

} // namespace navi::dev
