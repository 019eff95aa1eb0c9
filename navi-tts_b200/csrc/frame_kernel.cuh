// The persistent frame kernel: one cooperative launch per 12.5 Hz frame runs the
// talker decode step, samples codebook 0, runs the code predictor's 16 positions
// (sampling codebooks 1..15) and assembles the next frame's step embedding.
//
// What it computes is the reference's k_frame (model/qwen3tts/frame.hip:517-579);
// how it is organised is B200-specific:
//
//  * One CTA per SM (148), 11 consumer warps + 1 producer warp.
//  * The producer warp walks the same phase program as the consumers and streams
//    this CTA's slice of every weight matrix (rows [r0, r1) of the matrix; weights
//    never depend on activations) into a shared-memory ring with cp.async.bulk on
//    the TMA engine, one mbarrier per ring slot, running as many phases ahead as the
//    ring holds. HBM streaming therefore never waits on the phase dependencies.
//  * No grid barriers. Each phase's outputs travel between CTAs as 64-bit words
//    {value, tag} in L2 (tag = launch base + phase index); a consumer polls exactly
//    the words it needs until the tag matches. One L2 round trip per dependency
//    instead of a barrier plus a reload.
//  * q/k RMSNorm + RoPE + the KV store are fused into the attention phase. Talker
//    attention is split over KV position ranges (flash-decoding; each split CTA
//    streams its K/V rows through the ring like weights) with a fixed-order combine
//    by one CTA per query head; code-predictor attention (<= 16 positions) runs in one
//    CTA per KV head on K/V kept in shared memory.
//  * Sampling runs redundantly in every CTA (bit-identical inputs, deterministic
//    code), so the next phase starts without a barrier.
//  * Code-predictor positions 0 and 1 run as one 2-column pass over the weights.
//  * Every wait has a wall-clock deadline (%globaltimer); on expiry the CTA raises
//    the launch's abort word, every CTA unwinds, and the host reports a timeout.
#pragma once

#include "device.cuh"
#include "sampler.cuh"

#include <cuda_fp16.h>
#include <cstdint>

namespace navi::fk {

// 11 consumer warps + the producer = 12 warps, 3 on each of the SM's 4 schedulers, whose
// register files (16K registers each) then allow 168 registers a thread; a 13th warp would
// put 4 warps on one scheduler and cap every thread at 128, where this kernel spills.
constexpr int NCW = 11;                 // consumer warps
constexpr int NCT = NCW * 32;           // consumer threads
constexpr int NTHR = NCT + 32;          // + the producer warp
constexpr int BID = 1;                  // named barrier of the consumer threads
constexpr int MAX_TL = 32;              // talker layers
constexpr int MAX_CP = 8;               // code-predictor layers
constexpr int NCB = 16;                 // codebooks per frame
constexpr int NSLOT = 16;               // ring slots (mbarriers)
constexpr int MAX_SPLIT = 148;          // talker attention splits per KV head
constexpr int MAX_ATTN_CHUNK = 511;     // cached positions per talker attention split
constexpr int MAX_SEG = 5;              // weight segments per phase chunk
constexpr int MAX_GROUP = 4;            // q heads per KV head
constexpr int KHD = 128;                // head_dim the attention code is compiled for
constexpr int KGR = 2;                  // query heads per KV head the attention code is compiled for
constexpr uint32_t PIECE = 32768;       // bulk copies are issued in pieces of at most this
constexpr uint32_t CTRL_BYTES = 256;    // per-CTA control block in shared memory
constexpr int PROF_STRIDE = 4 * 4096 + 1;   // trace words per CTA: 4 stamps x phases, then the start
constexpr int MAX_B = 4;                // streams of one batched launch (each with its own KV cache and draws)
constexpr int MAXC = 4;                 // input columns of one GEMV phase (streams, or code-predictor positions)
constexpr int CP_SLOTS = 2;             // code-predictor K/V sets one CTA may keep (MAX_B * layers * KV heads / grid)
constexpr int KV_BOX = 32;              // cached positions per 2-D TMA box of a talker K or V cache
constexpr uint32_t TMAP_BYTES = 128;    // one CUtensorMap

enum Op : uint8_t { TQKV, TATTN, TO, TGU, TDOWN, THEAD, CQKV, CATTN, CO, CGU, CDOWN, CHEAD, FINAL, XOUT, SAMPLE };

// Talker QKV phase flag (Phase::pos): stage the layer input from Args::step_in instead of the
// previous layer's output (the first phase of a single-layer program).
constexpr uint8_t POS_STEP_IN = 1;

// op, input columns (batched programs: one per stream), layer, code-predictor position
// (SAMPLE: the codebook drawn)
struct Phase {
    uint8_t op, ncol, layer, pos;
};

struct LayerW {
    const float * ln1, * ln2, * qn, * kn;
    const __half * wqkv;   // [Q + 2 KV][H]: q, k, v rows adjacent
    const __half * wo;     // [H][Q]
    const __half * wg;     // [F][H]
    const __half * wu;     // [F][H]
    const __half * wd;     // [H][F]
};

struct ModelW {
    LayerW tl[MAX_TL];
    LayerW cp[MAX_CP];
    const float * tl_norm, * cp_norm;
    const __half * codec_head;        // [TV][H]
    const __half * tl_emb;            // [TV][H]
    const __half * cp_emb[NCB - 1];   // [CV][H]
    const __half * lm_head[NCB - 1];  // [CV][H]
};

struct Dims {
    int H, NH, NKV, HD, F, TV, CV, TL, CL;
    int Q, KV, QKV, GROUP;
    float eps_t, eps_c;
};

// Exchange words ({value, tag}) are indexed by input column c (a stream of a batched launch,
// or a code-predictor position of the single-stream pass over positions 0 and 1), and
// per-stream outputs by the stream's place s in the launch.
struct Work {
    uint64_t * x;        // [MAXC][H]   residual stream
    uint64_t * qkv;      // [MAXC][QKV]
    uint64_t * attn;     // [MAXC][Q]
    uint64_t * h;        // [MAXC][F]
    uint64_t * logits;   // [MAX_B][TV]
    uint64_t * clogits;  // [MAX_B][15][CV]
    uint64_t * part;     // [MAX_SPLIT * NH][HD + 2] talker attention partials (m, l, acc)
    uint64_t * hid_x;    // [MAX_B][H] batched: the talker's post-norm hidden, for code-predictor position 0
    uint64_t * code_x;   // [MAX_B][16] batched: the drawn codes
    int32_t * codes;     // [MAX_B][16]
    float * hidden;      // [MAX_B][H] talker post-norm hidden of the last talker step
    unsigned * ctl;      // [0] done tag, [1] failing phase, [2] abort tag, [3] failing CTA
};

struct Args {
    const Phase * prog;
    int nphase;
    const ModelW * mw;
    Dims d;
    Work w;
    uint32_t tag_base;
    int grid;          // CTAs of the launch
    int nb;            // streams of this launch (1: the single-stream program)
    // per stream s < nb
    int n_past[MAX_B];         // talker position
    int attn_split[MAX_B];     // talker attention splits of each KV head (<= attn_per)
    int attn_chunk[MAX_B];     // cached positions per split
    int attn_per;              // CTAs per (stream, KV head): CTA b < nb * NKV * attn_per takes stream
                               // (b / attn_per) / NKV, KV head (b / attn_per) % NKV, split b % attn_per
    const float * step_in[MAX_B];    // talker input row (frames >= 1)
    const float * trailing[MAX_B];   // [H]
    float * step_out[MAX_B];         // [H]
    uint8_t * seen[MAX_B];           // [TV] codebook-0 ids drawn so far this request
    __half * kc[MAX_B][MAX_TL];
    __half * vc[MAX_B][MAX_TL];
    // per stream: [MAX_TL][K, V] tensor maps of the KV cache ([max_pos][KV] f16, boxes of
    // KV_BOX positions x head_dim), in device memory, or null (row copies instead)
    const uint8_t * kvmap[MAX_B];
    float rope_t[MAX_B][128];        // talker position n_past: cos[HD/2], then sin[HD/2]
    uint64_t seed[MAX_B];
    int frame_index[MAX_B];
    uint64_t pcg_seed[MAX_B][NCB];
    // batched programs: phase indices whose tags the exchange words carry
    int thead_phase;                 // THEAD (hid_x)
    int sample_phase[NCB];           // SAMPLE of each codebook (code_x)
    // single stream, frame 0
    const float * hidden_in;   // the prefill's post-norm hidden
    const float * logits_in;   // the prefill's codec logits
    // batched frame 0 (the code predictor only): every stream's prefill hidden and logits
    const float * first_hidden[MAX_B];
    const float * first_logits[MAX_B];
    const float * inv_freq_t;  // [HD/2]
    const float * inv_freq_c;
    const float * rope_c;      // code predictor, positions 0..15: [NCB][HD] = cos[HD/2], sin[HD/2]
    // sampling (shared by the streams)
    float temp, top_p, rep;
    int top_k;
    float cp_temp, cp_top_p;
    int cp_top_k;
    int min_frames, rng;
    int eos_id, suppress_from;
    uint64_t timeout_ns;
    uint32_t poll_ns;          // pause between polls of exchange words that are not there yet (0: none)
    uint32_t ring_bytes;
    int xcols;                 // columns of the residual copy in shared memory (max(2, nb))
    int cp_slots;              // code-predictor K/V slots in shared memory (sets / grid, rounded up)
    int cp_keep_layers;        // code-predictor layers whose weights the producer asks L2 to keep
    uint32_t scratch_floats;
    uint32_t part_floats;
    uint32_t ysum_off;         // GEMV sums [2 * columns][rows] at part + ysum_off (after the per-warp partials)
    unsigned long long * prof;   // optional trace: [4 * nphase + 1] globaltimer stamps on CTA prof_cta,
    int prof_cta;                // or, prof_cta < 0, on every CTA b at prof + b * PROF_STRIDE
};

// ---- shared-memory layout (identical on host and device) ---------------------------------

struct SmemLayout {
    uint32_t bars, meta_off, meta_split, meta_end, ctrl, codes, xres, hid, part, scratch, cpkv, ring, total;
};

// The code predictor's K/V of one (stream, layer, KV head), kept in shared memory across the
// positions of a frame by the CTA that attends for it: [position][K, V][head_dim] f16.
__host__ __device__ inline uint32_t cpkv_bytes(const Dims & d) { return static_cast<uint32_t>(NCB) * 2 * d.HD * 2; }

// Code-predictor attention set i = (layer * nb + stream) * NKV + KV head lives on CTA i % G in
// its K/V slot i / G. A layer's nb * NKV sets are consecutive, so while nb * NKV <= G a CTA
// attends for at most one set per layer.
__host__ __device__ inline int cp_set(const Dims & d, int nb, int l, int s, int g) { return (l * nb + s) * d.NKV + g; }

__host__ __device__ inline uint32_t align_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

__host__ __device__ inline SmemLayout smem_layout(const Dims & d, uint32_t ring_bytes, uint32_t scratch_floats, uint32_t part_floats,
                                                  int xcols, int cp_slots) {
    SmemLayout L{};
    uint32_t o = 0;
    L.bars = o;     o += NSLOT * 8;
    L.meta_end = o; o += NSLOT * 8;
    L.meta_off = o; o += NSLOT * 4;
    L.meta_split = o; o += NSLOT * 4;
    L.ctrl = o;     o += CTRL_BYTES;
    L.codes = o;    o += MAX_B * NCB * 4;
    o = align_up(o, 16);
    L.xres = o;     o += static_cast<uint32_t>(xcols) * d.H * 4;
    L.hid = o;      o += d.H * 4;
    L.part = o;     o += align_up(part_floats * 4, 16);
    L.scratch = o;  o += align_up(scratch_floats * 4, 16);
    L.cpkv = o;     o += static_cast<uint32_t>(cp_slots) * align_up(cpkv_bytes(d), 16);
    o = align_up(o, 128);
    L.ring = o;     o += ring_bytes;
    L.total = o;
    return L;
}

// Rows [r0, r1) of an R-row matrix that CTA b of G owns.
// Frame weight matrices are re-laid out per CTA slice: the rows [r0, r1) of CTA b keep their
// bytes [r0 * K, r1 * K) (the same HBM range the producer streams) but inside the slice
// element (r, k) sits at ((k / 8) * (r1 - r0) + (r - r0)) * 8 + k % 8, so that in shared
// memory lane = row reads 16 consecutive bytes per 8-column chunk without bank conflicts.
__host__ __device__ inline void split_rows(int R, int b, int G, int & r0, int & r1) {
    r0 = static_cast<int>((static_cast<long long>(R) * b) / G);
    r1 = static_cast<int>((static_cast<long long>(R) * (b + 1)) / G);
}

// A run of `rows` copies of `bytes` each, from src, src + stride, ... (bytes and stride
// multiples of 16), packed back to back in the chunk.
struct Seg {
    const void * src;
    uint32_t bytes;
    uint32_t rows = 1;
    uint32_t stride = 0;
    uint32_t nr = 0;      // a weight slice [K/8][nr][8] f16 of nr rows (0: other data)
    // tensor segment (tmap non-null): `rows` boxes of `bytes` each, box r read by one 2-D TMA
    // load of tmap at element coordinates (tx, ty + r * KV_BOX)
    const void * tmap = nullptr;
    int tx = 0, ty = 0;
};

// Where a chunk may be cut when it does not fit before the end of the ring: at the start
// of any segment, and inside a weight slice at the first k-chunk of any consumer warp's
// K range (so every warp still reads one contiguous run). Returns the largest such logical
// offset <= room (0: the whole chunk starts over at the ring's start).
__host__ __device__ inline uint32_t chunk_split(const Seg * s, int ns, uint32_t room) {
    uint32_t best = 0, o = 0;
    for (int i = 0; i < ns; ++i) {
        if (o <= room) best = o;
        if (s[i].nr > 0 && s[i].rows == 1) {
            const uint32_t kstep = s[i].nr * 16u, nk = s[i].bytes / kstep;
            for (int w = 1; w < NCW; ++w) {
                const uint32_t at = o + (nk * static_cast<uint32_t>(w) / NCW) * kstep;
                if (at <= room && at > best) best = at;
            }
        }
        o += s[i].bytes * s[i].rows;
    }
    return best;
}

// This CTA's rows of every matrix shape the phases use (computed once per launch: the
// 64-bit divisions of split_rows stay off the per-phase path).
struct Rows {
    int qkv0, qkv1, h0, h1, f0, f1, tv0, tv1, cv0, cv1;
};
__host__ __device__ inline Rows cta_rows(const Dims & d, int b, int G) {
    Rows r;
    split_rows(d.QKV, b, G, r.qkv0, r.qkv1);
    split_rows(d.H, b, G, r.h0, r.h1);
    split_rows(d.F, b, G, r.f0, r.f1);
    split_rows(d.TV, b, G, r.tv0, r.tv1);
    split_rows(d.CV, b, G, r.cv0, r.cv1);
    return r;
}

// Talker attention role of CTA b: (stream, KV head, split) while b < nb * NKV * attn_per and
// the split holds positions (splits past attn_split[stream] have none but the last one's new row).
__host__ __device__ inline bool talker_attn_role(const Args & A, int b, int & stream, int & g, int & sp) {
    const int grp = b / A.attn_per;
    if (grp >= A.nb * A.d.NKV) return false;
    stream = grp / A.d.NKV;
    g = grp - stream * A.d.NKV;
    sp = b - grp * A.attn_per;
    return sp < A.attn_split[stream];
}

// Code-predictor attention role of CTA b for layer l (cp_set): its stream, KV head and K/V slot.
__host__ __device__ inline bool cp_attn_role(const Args & A, int b, int l, int & stream, int & g, int & slot) {
    const int G = A.grid;
    const int n = A.nb * A.d.NKV, first = cp_set(A.d, A.nb, l, 0, 0);
    // the set of layer l on CTA b: first <= i < first + n with i % G == b
    int i = first + ((b - first % G) % G + G) % G;
    if (i >= first + n) return false;
    stream = (i - first) / A.d.NKV;
    g = (i - first) - stream * A.d.NKV;
    slot = i / G;
    return slot < A.cp_slots;
}

// The bytes phase `ph` streams into CTA b's ring chunk, in order (up to MAX_SEG segments,
// each a multiple of 16 bytes): the phase's norm weights first, then its weight rows
// [r0, r1); for attention, the q/k norm weights, then (talker) this split's KV head slice
// [HD] of the K and of the V rows of its cached positions [r0, r1). Returns the number of
// segments (0: no chunk).
__host__ __device__ inline int phase_segments(const Args & A, const ModelW & W, const Phase & ph, int b, const Rows & R, Seg * s,
                                              int & r0, int & r1) {
    const Dims & d = A.d;
    const LayerW * L = nullptr;
    if (ph.op <= TDOWN) L = &W.tl[ph.layer];
    else if (ph.op >= CQKV && ph.op <= CDOWN) L = &W.cp[ph.layer];
    const uint32_t H4 = static_cast<uint32_t>(d.H) * 4, HD4 = static_cast<uint32_t>(d.HD) * 4;
    r0 = r1 = 0;
    switch (ph.op) {
        case TQKV: case CQKV:
            r0 = R.qkv0; r1 = R.qkv1;
            s[0] = {L->ln1, H4};
            s[1] = {L->wqkv + static_cast<size_t>(r0) * d.H, static_cast<uint32_t>((r1 - r0) * d.H * 2), 1, 0, static_cast<uint32_t>(r1 - r0)};
            return r1 > r0 ? 2 : 0;
        case TO: case CO:
            r0 = R.h0; r1 = R.h1;
            s[0] = {L->wo + static_cast<size_t>(r0) * d.Q, static_cast<uint32_t>((r1 - r0) * d.Q * 2), 1, 0, static_cast<uint32_t>(r1 - r0)};
            return r1 > r0 ? 1 : 0;
        case TGU: case CGU:
            r0 = R.f0; r1 = R.f1;
            s[0] = {L->ln2, H4};
            s[1] = {L->wg + static_cast<size_t>(r0) * d.H, static_cast<uint32_t>((r1 - r0) * d.H * 2), 1, 0, static_cast<uint32_t>(r1 - r0)};
            s[2] = {L->wu + static_cast<size_t>(r0) * d.H, static_cast<uint32_t>((r1 - r0) * d.H * 2), 1, 0, static_cast<uint32_t>(r1 - r0)};
            return r1 > r0 ? 3 : 0;
        case TDOWN: case CDOWN:
            r0 = R.h0; r1 = R.h1;
            s[0] = {L->wd + static_cast<size_t>(r0) * d.F, static_cast<uint32_t>((r1 - r0) * d.F * 2), 1, 0, static_cast<uint32_t>(r1 - r0)};
            return r1 > r0 ? 1 : 0;
        case THEAD:
            r0 = R.tv0; r1 = R.tv1;
            s[0] = {W.tl_norm, H4};
            s[1] = {W.codec_head + static_cast<size_t>(r0) * d.H, static_cast<uint32_t>((r1 - r0) * d.H * 2), 1, 0, static_cast<uint32_t>(r1 - r0)};
            return r1 > r0 ? 2 : 0;
        case CHEAD:
            r0 = R.cv0; r1 = R.cv1;
            s[0] = {W.cp_norm, H4};
            s[1] = {W.lm_head[ph.pos - 1] + static_cast<size_t>(r0) * d.H, static_cast<uint32_t>((r1 - r0) * d.H * 2), 1, 0,
                    static_cast<uint32_t>(r1 - r0)};
            return r1 > r0 ? 2 : 0;
        case TATTN: {
            int st_, g, sp;
            if (!talker_attn_role(A, b, st_, g, sp)) return 0;
            s[0] = {L->qn, HD4};
            s[1] = {L->kn, HD4};
            // cached positions [r0, r1) of this split, stream st_, KV head g
            r0 = min(sp * A.attn_chunk[st_], A.n_past[st_]);
            r1 = min(r0 + A.attn_chunk[st_], A.n_past[st_]);
            if (r1 <= r0) return 2;
            if (A.kvmap[st_]) {
                // per cache, boxed loads of KV head g's 256-byte slices of positions [r0, r0 + nbox * KV_BOX)
                // (positions past r1 are read and not used; past max_pos they read as zeros)
                const uint32_t nbox = static_cast<uint32_t>((r1 - r0 + KV_BOX - 1) / KV_BOX), bb = static_cast<uint32_t>(KV_BOX * d.HD * 2);
                const uint8_t * m = A.kvmap[st_] + static_cast<size_t>(ph.layer) * 2 * TMAP_BYTES;
                s[2] = {nullptr, bb, nbox, 0, 0, m, g * d.HD, r0};
                s[3] = {nullptr, bb, nbox, 0, 0, m + TMAP_BYTES, g * d.HD, r0};
                return 4;
            }
            const size_t off = static_cast<size_t>(r0) * d.KV + static_cast<size_t>(g) * d.HD;
            const uint32_t rows = static_cast<uint32_t>(r1 - r0), rb = static_cast<uint32_t>(d.HD) * 2, st = static_cast<uint32_t>(d.KV) * 2;
            s[2] = {A.kc[st_][ph.layer] + off, rb, rows, st};
            s[3] = {A.vc[st_][ph.layer] + off, rb, rows, st};
            return 4;
        }
        case CATTN: {
            int st_, g, slot;
            if (!cp_attn_role(A, b, ph.layer, st_, g, slot)) return 0;
            s[0] = {L->qn, HD4};
            s[1] = {L->kn, HD4};
            // the RoPE rows of the phase's positions (one per column; batched streams share one)
            s[2] = {A.rope_c + static_cast<size_t>(ph.pos) * d.HD, HD4 * static_cast<uint32_t>(A.nb > 1 ? 1 : ph.ncol)};
            return 3;
        }
        default:
            return 0;
    }
}

} // namespace navi::fk
