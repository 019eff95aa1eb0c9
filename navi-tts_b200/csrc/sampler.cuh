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
    float * s;        // [V] in: logits; out: modified, tempered values
    float * e;        // [V]
    int * idx;        // [V] candidate ids in index order
    int * ord;        // [V] candidates in value order (top-p)
    uint8_t * keep;   // [V]
    unsigned * hist;  // [256]
    float * red;      // [64]
};

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

// Samples from S.s[0..V) (the raw logits on entry). Must be called by all NT threads
// (NT a multiple of 32, >= 256; barrier id `bid`); every thread returns the chosen id.
template <int NT>
__device__ int sample_cta(int V, const SampleCfg & c, const SampleScratch & S, int bid) {
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    static_assert(NT % 32 == 0 && NT >= 256 && NT <= 1024, "sampler thread count");
    float * s = S.s;
    float * red = S.red;
    int * ired = reinterpret_cast<int *>(S.red);
    // 1. codebook-0 modifications, temperature
    const bool greedy = c.temperature <= 0.f;
    float lmax = -INFINITY;
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
    }
    lmax = warp_max(lmax);
    if (lane == 0) red[wid] = lmax;
    named_sync(bid, NT);
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < NT / 32; ++w) mx = fmaxf(mx, red[w]);
    named_sync(bid, NT);
    if (greedy) {
        // lowest index holding the maximum (index 0 when every value is -inf)
        int best = V;
        for (int i = tid; i < V; i += NT) if (s[i] == mx) { best = i; break; }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) best = min(best, __shfl_xor_sync(0xffffffffu, best, o));
        if (lane == 0) ired[wid] = best;
        named_sync(bid, NT);
        int b = V;
#pragma unroll
        for (int w = 0; w < NT / 32; ++w) b = min(b, ired[w]);
        named_sync(bid, NT);
        return b >= V ? 0 : b;
    }
    // 2. exact k-th largest key (4 passes of 8 bits), threshold
    float threshold = -INFINITY;
    if (c.top_k > 0 && c.top_k < V) {
        uint32_t prefix = 0, mask = 0;
        int need = c.top_k;
        for (int pass = 3; pass >= 0; --pass) {
            const int shift = pass * 8;
            if (tid < 256) S.hist[tid] = 0;
            named_sync(bid, NT);
            for (int i = tid; i < V; i += NT) {
                const uint32_t key = float_key(s[i]);
                if ((key & mask) == prefix) atomicAdd(&S.hist[(key >> shift) & 0xFFu], 1u);
            }
            named_sync(bid, NT);
            // threads 0..255: t owns digit 255 - t; inclusive scan of counts from the top digit down
            int cnt = 0, incl = 0;
            if (tid < 256) {
                cnt = static_cast<int>(S.hist[255 - tid]);
                incl = cnt;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int v = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= o) incl += v;
                }
                if (lane == 31) ired[wid] = incl;
            }
            named_sync(bid, NT);
            if (tid < 256) {
                int above = incl - cnt;
                for (int w = 0; w < wid; ++w) above += ired[w];
                if (above < need && above + cnt >= need) { ired[16] = 255 - tid; ired[17] = need - above; }
            }
            named_sync(bid, NT);
            need = ired[17];
            prefix |= static_cast<uint32_t>(ired[16]) << shift;
            mask |= 0xFFu << shift;
            named_sync(bid, NT);
        }
        threshold = key_float(prefix);
    }
    // 3. e_i over candidates
    for (int i = tid; i < V; i += NT) S.e[i] = (s[i] >= threshold) ? exp_spec(__fsub_rn(s[i], mx)) : 0.0f;
    named_sync(bid, NT);
    // 4. normaliser in the reference's 256-thread block_sum order
    if (tid < 256) {
        float acc = 0.f;
        for (int i = tid; i < V; i += 256) acc = __fadd_rn(acc, S.e[i]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
        if (lane == 0) red[32 + wid] = acc;
    }
    named_sync(bid, NT);
    if (wid == 0) {
        float v = lane < 8 ? red[32 + lane] : 0.f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (lane == 0) red[48] = v;
    }
    named_sync(bid, NT);
    const float ssum = red[48];
    const float inv = __fdiv_rn(1.0f, ssum);
    // 5. compact the nonzero e_i in index order
    int total = 0;
    for (int base = 0; base < V; base += NT) {
        const int i = base + tid;
        const bool nz = i < V && S.e[i] != 0.f;
        const unsigned m = __ballot_sync(0xffffffffu, nz);
        if (lane == 0) ired[wid] = __popc(m);
        named_sync(bid, NT);
        int before = total;
        for (int w = 0; w < wid; ++w) before += ired[w];
        if (nz) S.idx[before + __popc(m & ((1u << lane) - 1u))] = i;
        int t = 0;
#pragma unroll
        for (int w = 0; w < NT / 32; ++w) t += ired[w];
        total += t;
        named_sync(bid, NT);
    }
    const int n = total;
    const float u = draw_uniform(c);
    const bool nucleus = c.top_p > 0.f && c.top_p < 1.f;
    if (nucleus) {
        // rank of each candidate in (value desc, index asc) order
        for (int j = tid; j < n; j += NT) {
            const int ij = S.idx[j];
            const float vj = s[ij];
            int r = 0;
            for (int m = 0; m < n; ++m) {
                const int im = S.idx[m];
                const float vm = s[im];
                r += (vm > vj || (vm == vj && im < ij)) ? 1 : 0;
            }
            S.ord[r] = ij;
        }
        for (int i = tid; i < V; i += NT) S.keep[i] = 0;
        named_sync(bid, NT);
    }
    if (tid == 0) {
        int chosen;
        if (nucleus) {
            float cum = 0.f;
            for (int r = 0; r < n; ++r) {
                const int i = S.ord[r];
                cum = __fadd_rn(cum, __fmul_rn(S.e[i], inv));
                S.keep[i] = 1;
                if (cum >= c.top_p) break;
            }
            float ksum = 0.f;
            int last = V - 1;
            for (int j = 0; j < n; ++j) {
                const int i = S.idx[j];
                if (S.keep[i]) { ksum = __fadd_rn(ksum, S.e[i]); last = i; }
            }
            const float kinv = __fdiv_rn(1.0f, ksum);
            chosen = last;
            float c2 = 0.f;
            for (int j = 0; j < n; ++j) {
                const int i = S.idx[j];
                if (!S.keep[i]) continue;
                c2 = __fadd_rn(c2, __fmul_rn(S.e[i], kinv));
                if (c2 >= u) { chosen = i; break; }
            }
        } else {
            chosen = V - 1;
            float cum = 0.f;
            for (int j = 0; j < n; ++j) {
                const int i = S.idx[j];
                cum = __fadd_rn(cum, __fmul_rn(S.e[i], inv));
                if (cum >= u) { chosen = i; break; }
            }
        }
        ired[60] = chosen;
    }
    named_sync(bid, NT);
    const int chosen = ired[60];
    named_sync(bid, NT);
    return chosen;
}

} // namespace navi::dev
