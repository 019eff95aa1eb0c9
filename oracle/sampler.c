/* CPU oracle of the frame sampler -- TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg load
 * this library, and only as a checker; the product path never does.
 *
 * It restates, sequentially and in plain C, the sampling that the reference
 * frame kernel does on the device (model/qwen3tts/frame.hip):
 *   - the codebook-0 logit modifications, tl_modified_logit (frame.hip:413-419):
 *     ids >= suppress_from except EOS -> -inf; EOS -> -inf before min_frames;
 *     repetition penalty over seen ids (v > 0 ? v / p : v * p);
 *   - greedy argmax, lowest index on ties (block_argmax, frame.hip:178-203);
 *   - temperature, then the exact k-th largest by monotone float keys
 *     (float_key / block_kth_largest, frame.hip:212-256), candidates v >= threshold;
 *   - e_i = exp(v_i - max) for candidates, the normaliser summed in the order
 *     of the reference's 256-thread block_sum (runtime/device/kernel_util.h:20-34),
 *     and the multinomial walk over the nonzero e_i in index order
 *     (block_draw, frame.hip:263-296);
 *   - the PCG32 stream and its seeding (pcg32_next frame.hip:169-175, the
 *     per-draw state frame.hip:284-286) and the splitmix64 per-frame /
 *     per-codebook seeds (frame.hip:581-586, 658-659, 497).
 * Added by this build (not in the reference): top-p (nucleus) after top-k,
 * and a Philox4x32-10 stream (Salmon et al., SC'11) keyed by the request
 * seed with counter (frame index, codebook).
 *
 * exp is the one function both sides must agree on bit for bit, so it is
 * specified here rather than taken from a math library: Cody-Waite range
 * reduction x = n ln2 + r with ln2 split as the fdlibm hi/lo pair, a degree-7
 * Taylor polynomial for e^r evaluated by Horner's rule with fused
 * multiply-adds, and an exact power-of-two scaling with a single final
 * rounding.  Compiled with -ffp-contract=off so every other operation is one
 * IEEE-754 binary32 rounding.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static float pow2i(int k) { /* 2^k for k in [-126, 127] */
    union { uint32_t u; float f; } v;
    v.u = (uint32_t)(k + 127) << 23;
    return v.f;
}

float oracle_exp(float x) {
    if (x != x) return x;
    if (x > 0x1.62e43p+6f) return INFINITY;           /* 88.72283935546875: e^x overflows above */
    if (x < -0x1.9fe36ap+6f) return 0.0f;             /* -103.97208404541015625: e^x rounds to 0 below */
    const float n = rintf(x * 0x1.715476p+0f);        /* log2(e) */
    float r = fmaf(-n, 0x1.62e4p-1f, x);              /* ln2 hi (fdlibm split) */
    r = fmaf(-n, 0x1.7f7d1cp-20f, r);                 /* ln2 lo */
    float p = 0x1.a01a02p-13f;                        /* 1/5040 */
    p = fmaf(p, r, 0x1.6c16c2p-10f);                  /* 1/720 */
    p = fmaf(p, r, 0x1.111112p-7f);                   /* 1/120 */
    p = fmaf(p, r, 0x1.555556p-5f);                   /* 1/24 */
    p = fmaf(p, r, 0x1.555556p-3f);                   /* 1/6 */
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int ni = (int)n;
    if (ni > 127) { p = p * pow2i(127); ni -= 127; }
    else if (ni < -126) { p = p * pow2i(ni + 64); ni = -64; }
    return p * pow2i(ni);
}

uint64_t oracle_splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

/* PCG32 XSH-RR step with an explicit increment (the reference uses the default
 * increment 1442695040888963407). */
uint32_t oracle_pcg32_step(uint64_t * s, uint64_t inc) {
    const uint64_t old = *s;
    *s = old * 6364136223846793005ull + inc;
    const uint32_t xs = (uint32_t)(((old >> 18u) ^ old) >> 27u);
    const uint32_t rot = (uint32_t)(old >> 59u);
    return (xs >> rot) | (xs << ((0u - rot) & 31u));
}

void oracle_philox4x32_10(const uint32_t ctr_in[4], const uint32_t key_in[2], uint32_t out[4]) {
    uint32_t c0 = ctr_in[0], c1 = ctr_in[1], c2 = ctr_in[2], c3 = ctr_in[3];
    uint32_t k0 = key_in[0], k1 = key_in[1];
    for (int round = 0; round < 10; ++round) {
        const uint64_t p0 = (uint64_t)0xD2511F53u * c0, p1 = (uint64_t)0xCD9E8D57u * c2;
        const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0, hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
        c0 = hi1 ^ c1 ^ k0; c1 = lo1; c2 = hi0 ^ c3 ^ k1; c3 = lo0;
        k0 += 0x9E3779B9u; k1 += 0xBB67AE85u;
    }
    out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

/* Per-draw seeds of the reference's PCG mode. codebook 0 is the talker draw. */
uint64_t oracle_draw_seed(uint64_t seed, int frame_index, int codebook) {
    const uint64_t tl = oracle_splitmix64(seed ^ ((uint64_t)(int64_t)frame_index * 0xA24BAED4963EE407ull));
    if (codebook == 0) return tl;
    const uint64_t cp = oracle_splitmix64(tl ^ 0x9FB21C651E98DF25ull);
    return cp + (uint64_t)codebook * 0xD1B54A32D192ED03ull;
}

/* The uniform in [0, 1) a draw compares against: 24 high bits of the stream word. */
float oracle_uniform(int rng, uint64_t seed, int frame_index, int codebook) {
    uint32_t w;
    if (rng == 0) {
        uint64_t st = oracle_draw_seed(seed, frame_index, codebook) * 0x9E3779B97F4A7C15ull + 0xBF58476D1CE4E5B9ull + 1ull;
        (void)oracle_pcg32_step(&st, 1442695040888963407ull);
        (void)oracle_pcg32_step(&st, 1442695040888963407ull);
        (void)oracle_pcg32_step(&st, 1442695040888963407ull);
        w = oracle_pcg32_step(&st, 1442695040888963407ull);
    } else {
        const uint32_t ctr[4] = {(uint32_t)frame_index, (uint32_t)codebook, 0u, 0u};
        const uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
        uint32_t out[4];
        oracle_philox4x32_10(ctr, key, out);
        w = out[0];
    }
    return (float)(w >> 8) * (1.0f / 16777216.0f);
}

static uint32_t float_key(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
static float key_float(uint32_t k) {
    const uint32_t u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
    float f;
    memcpy(&f, &u, 4);
    return f;
}
static int cmp_u32_desc(const void * a, const void * b) {
    const uint32_t x = *(const uint32_t *)a, y = *(const uint32_t *)b;
    return x < y ? 1 : (x > y ? -1 : 0);
}

typedef struct {
    float temperature;         /* <= 0: greedy */
    int top_k;                 /* 0 or >= V: off */
    float top_p;               /* >= 1 or <= 0: off */
    int rng;                   /* 0 PCG (reference stream), 1 Philox */
    uint64_t seed;             /* the request seed */
    int frame_index;
    int codebook;              /* 0 talker, 1..15 code predictor */
    /* codebook-0 modifications (talker draw only) */
    int talker_mods;
    int suppress_from, eos_id, min_frames;
    float repetition_penalty;  /* <= 0: off */
    const uint8_t * seen;      /* [V] or null */
    /* 1: e_i with the C library's expf instead of oracle_exp -- only to compare with the
     * reference's own sampler compiled for the host (oracle/ref_frame_check.cpp), which
     * calls expf from the same library */
    int exp_libm;
} oracle_sample_args;

/* Writes the per-index working values into dbg_e (e_i, or NaN when unused) when
 * dbg_e is non-null, and the normaliser into *dbg_sum. Returns the chosen id. */
int oracle_sample(const float * logits, int V, const oracle_sample_args * a, float * dbg_e, float * dbg_sum) {
    float * s = (float *)malloc(sizeof(float) * (size_t)V);
    float * e = (float *)malloc(sizeof(float) * (size_t)V);
    for (int i = 0; i < V; ++i) {
        float v = logits[i];
        if (a->talker_mods) {
            if (i >= a->suppress_from && i != a->eos_id) v = -INFINITY;
            else if (i == a->eos_id && a->frame_index < a->min_frames) v = -INFINITY;
            else if (a->repetition_penalty > 0.f && a->seen && a->seen[i]) v = (v > 0.f) ? v / a->repetition_penalty : v * a->repetition_penalty;
        }
        s[i] = v;
    }
    int chosen = 0;
    if (a->temperature <= 0.f) {
        float bv = -INFINITY;
        for (int i = 0; i < V; ++i) if (s[i] > bv) { bv = s[i]; chosen = i; }
        if (dbg_sum) *dbg_sum = 0.f;
        if (dbg_e) for (int i = 0; i < V; ++i) dbg_e[i] = NAN;
        free(s); free(e);
        return chosen;
    }
    float mx = -INFINITY;
    for (int i = 0; i < V; ++i) { s[i] = s[i] / a->temperature; mx = fmaxf(mx, s[i]); }
    float threshold = -INFINITY;
    if (a->top_k > 0 && a->top_k < V) {
        uint32_t * keys = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)V);
        for (int i = 0; i < V; ++i) keys[i] = float_key(s[i]);
        qsort(keys, (size_t)V, sizeof(uint32_t), cmp_u32_desc);
        threshold = key_float(keys[a->top_k - 1]);
        free(keys);
    }
    for (int i = 0; i < V; ++i) e[i] = (s[i] >= threshold) ? (a->exp_libm ? expf(s[i] - mx) : oracle_exp(s[i] - mx)) : 0.0f;
    /* the normaliser, in the reference block_sum order for a 256-thread block */
    float part[256], wsum[8];
    for (int t = 0; t < 256; ++t) {
        float acc = 0.f;
        for (int i = t; i < V; i += 256) acc = acc + e[i];
        part[t] = acc;
    }
    for (int w = 0; w < 8; ++w) {
        float v[32];
        for (int l = 0; l < 32; ++l) v[l] = part[32 * w + l];
        for (int o = 16; o > 0; o >>= 1) {
            float nv[32];
            for (int l = 0; l < 32; ++l) nv[l] = v[l] + v[l ^ o];
            memcpy(v, nv, sizeof v);
        }
        wsum[w] = v[0];
    }
    {
        float v[32];
        for (int l = 0; l < 32; ++l) v[l] = l < 8 ? wsum[l] : 0.f;
        for (int o = 16; o > 0; o >>= 1) {
            float nv[32];
            for (int l = 0; l < 32; ++l) nv[l] = v[l] + v[l ^ o];
            memcpy(v, nv, sizeof v);
        }
        wsum[0] = v[0];
    }
    const float ssum = wsum[0];
    const float inv = 1.0f / ssum;
    if (dbg_sum) *dbg_sum = ssum;
    if (dbg_e) memcpy(dbg_e, e, sizeof(float) * (size_t)V);
    const float u = oracle_uniform(a->rng, a->seed, a->frame_index, a->codebook);
    if (a->top_p > 0.f && a->top_p < 1.f) {
        /* nucleus over the candidates: descending value, ties by lower index; keep the
         * shortest prefix whose cumulative probability reaches top_p */
        int n = 0;
        int * cand = (int *)malloc(sizeof(int) * (size_t)V);
        for (int i = 0; i < V; ++i) if (e[i] != 0.f) cand[n++] = i;
        int * order = (int *)malloc(sizeof(int) * (size_t)(n ? n : 1));
        for (int j = 0; j < n; ++j) {   /* rank of cand[j] */
            int r = 0;
            for (int m = 0; m < n; ++m) {
                const int a_i = cand[m], b_i = cand[j];
                if (s[a_i] > s[b_i] || (s[a_i] == s[b_i] && a_i < b_i)) ++r;
            }
            order[r] = cand[j];
        }
        uint8_t * keep = (uint8_t *)calloc((size_t)V, 1);
        float cum = 0.f;
        for (int r = 0; r < n; ++r) {
            cum = cum + e[order[r]] * inv;
            keep[order[r]] = 1;
            if (cum >= a->top_p) break;
        }
        float ksum = 0.f;
        int last = V - 1;
        for (int i = 0; i < V; ++i) if (keep[i]) { ksum = ksum + e[i]; last = i; }
        const float kinv = 1.0f / ksum;
        chosen = last;
        float c2 = 0.f;
        for (int i = 0; i < V; ++i) {
            if (!keep[i]) continue;
            c2 = c2 + e[i] * kinv;
            if (c2 >= u) { chosen = i; break; }
        }
        free(cand); free(order); free(keep);
    } else {
        chosen = V - 1;
        float cum = 0.f;
        for (int i = 0; i < V; ++i) {
            if (e[i] == 0.f) continue;
            cum = cum + e[i] * inv;
            if (cum >= u) { chosen = i; break; }
        }
    }
    free(s); free(e);
    return chosen;
}
