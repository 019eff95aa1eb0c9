// The persistent frame kernel: one cooperative launch per 12.5 Hz frame runs the
// talker decode step, samples codebook 0, runs the code predictor's 16 positions
// (sampling codebooks 1..15) and assembles the next frame's step embedding.
//
// What it computes is the reference's k_frame (model/qwen3tts/frame.hip:517-579);
// how it is organised is B200-specific:
//
//  * One CTA per SM (148), 16 consumer warps + 1 producer warp.
//  * The producer warp walks the same phase program as the consumers and streams
//    this CTA's slice of every weight matrix (rows [r0, r1) of the matrix; weights
//    never depend on activations) into a shared-memory ring with cp.async.bulk on
//    the TMA engine, one mbarrier per ring slot, running as many phases ahead as the
//    ring holds. HBM streaming therefore never waits on the phase dependencies.
//  * No grid barriers. Each phase's outputs travel between CTAs as 64-bit words
//    {value, tag} in L2 (tag = launch base + phase index); a consumer polls exactly
//    the words it needs until the tag matches. One L2 round trip per dependency
//    instead of a barrier plus a reload.
//  * q/k RMSNorm + RoPE + the KV store are fused into the attention phase; attention
//    is split over KV ranges (flash-decoding) with a fixed-order combine by the
//    split-0 CTA of each KV head.
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

constexpr int NCW = 16;                 // consumer warps
constexpr int NCT = NCW * 32;           // consumer threads
constexpr int NTHR = NCT + 32;          // + the producer warp
constexpr int BID = 1;                  // named barrier of the consumer threads
constexpr int MAX_TL = 32;              // talker layers
constexpr int MAX_CP = 8;               // code-predictor layers
constexpr int NCB = 16;                 // codebooks per frame
constexpr int NSLOT = 16;               // ring slots (mbarriers)
constexpr int MAX_SPLIT = 18;           // attention splits per KV head
constexpr int MAX_GROUP = 4;            // q heads per KV head
constexpr uint32_t PIECE = 32768;       // bulk copies are issued in pieces of at most this
constexpr uint32_t CTRL_BYTES = 256;    // per-CTA control block in shared memory

enum Op : uint8_t { TQKV, TATTN, TO, TGU, TDOWN, THEAD, CQKV, CATTN, CO, CGU, CDOWN, CHEAD, FINAL };

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

struct Work {
    uint64_t * x;        // [2][H]   residual stream (talker uses column 0)
    uint64_t * qkv;      // [2][QKV]
    uint64_t * attn;     // [2][Q]
    uint64_t * h;        // [2][F]
    uint64_t * logits;   // [TV]
    uint64_t * clogits;  // [15][CV]
    uint64_t * part;     // [NKV][MAX_SPLIT][2][GROUP][HD + 2]
    __half * ckc, * cvc; // [CL][16][KV]
    uint8_t * seen;      // [TV]
    int32_t * codes;     // [16]
    float * hidden;      // [H] talker post-norm hidden of the last talker step
    unsigned * ctl;      // [0] done tag, [1] failing phase, [2] abort tag, [3] failing CTA
};

struct Args {
    const Phase * prog;
    int nphase;
    const ModelW * mw;
    Dims d;
    Work w;
    uint32_t tag_base;
    int n_past;        // talker position
    int attn_split;    // talker attention splits per KV head
    const float * step_in;     // talker input row (frames >= 1)
    const float * hidden_in;   // frame 0: the prefill's post-norm hidden
    const float * logits_in;   // frame 0: the prefill's codec logits
    const float * trailing;    // [H]
    float * step_out;          // [H]
    __half * kc[MAX_TL];
    __half * vc[MAX_TL];
    const float * inv_freq_t;  // [HD/2]
    const float * inv_freq_c;
    // sampling
    float temp, top_p, rep;
    int top_k;
    float cp_temp, cp_top_p;
    int cp_top_k;
    int min_frames, rng;
    uint64_t seed;
    int frame_index;
    uint64_t pcg_seed[NCB];
    int eos_id, suppress_from;
    uint64_t timeout_ns;
    uint32_t ring_bytes;
    uint32_t scratch_floats;
    uint32_t part_floats;
    unsigned long long * prof;   // optional: [nphase] globaltimer at the end of each phase on CTA 0
};

// ---- shared-memory layout (identical on host and device) ---------------------------------

struct SmemLayout {
    uint32_t bars, meta_off, meta_end, ctrl, codes, xres, hid, part, scratch, ring, total;
};

__host__ __device__ inline uint32_t align_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

__host__ __device__ inline SmemLayout smem_layout(const Dims & d, uint32_t ring_bytes, uint32_t scratch_floats, uint32_t part_floats) {
    SmemLayout L{};
    uint32_t o = 0;
    L.bars = o;     o += NSLOT * 8;
    L.meta_end = o; o += NSLOT * 8;
    L.meta_off = o; o += NSLOT * 4;
    L.ctrl = o;     o += CTRL_BYTES;
    L.codes = o;    o += NCB * 4;
    o = align_up(o, 16);
    L.xres = o;     o += 2 * d.H * 4;
    L.hid = o;      o += d.H * 4;
    L.part = o;     o += align_up(part_floats * 4, 16);
    L.scratch = o;  o += align_up(scratch_floats * 4, 16);
    o = align_up(o, 128);
    L.ring = o;     o += ring_bytes;
    L.total = o;
    return L;
}

// Rows [r0, r1) of an R-row matrix that CTA b of G owns.
__host__ __device__ inline void split_rows(int R, int b, int G, int & r0, int & r1) {
    r0 = static_cast<int>((static_cast<long long>(R) * b) / G);
    r1 = static_cast<int>((static_cast<long long>(R) * (b + 1)) / G);
}

struct Seg {
    const void * src;
    uint32_t bytes;
};

// The weight bytes phase p needs on CTA b (0, 1 or 2 contiguous segments).
__host__ __device__ inline int phase_segments(const Args & A, const ModelW & W, const Phase & ph, int b, int G, Seg * s,
                                              int & r0, int & r1) {
    const Dims & d = A.d;
    const bool tl = ph.op <= THEAD;
    const LayerW * L = nullptr;
    if (ph.op <= TDOWN) L = &W.tl[ph.layer];
    else if (ph.op >= CQKV && ph.op <= CDOWN) L = &W.cp[ph.layer];
    (void) tl;
    r0 = r1 = 0;
    switch (ph.op) {
        case TQKV: case CQKV:
            split_rows(d.QKV, b, G, r0, r1);
            s[0] = {L->wqkv + static_cast<size_t>(r0) * d.H, static_cast<uint32_t>((r1 - r0) * d.H * 2)};
            return r1 > r0 ? 1 : 0;
        case TO: case CO:
            split_rows(d.H, b, G, r0, r1);
            s[0] = {L->wo + static_cast<size_t>(r0) * d.Q, static_cast<uint32_t>((r1 - r0) * d.Q * 2)};
            return r1 > r0 ? 1 : 0;
        case TGU: case CGU:
            split_rows(d.F, b, G, r0, r1);
            s[0] = {L->wg + static_cast<size_t>(r0) * d.H, static_cast<uint32_t>((r1 - r0) * d.H * 2)};
            s[1] = {L->wu + static_cast<size_t>(r0) * d.H, static_cast<uint32_t>((r1 - r0) * d.H * 2)};
            return r1 > r0 ? 2 : 0;
        case TDOWN: case CDOWN:
            split_rows(d.H, b, G, r0, r1);
            s[0] = {L->wd + static_cast<size_t>(r0) * d.F, static_cast<uint32_t>((r1 - r0) * d.F * 2)};
            return r1 > r0 ? 1 : 0;
        case THEAD:
            split_rows(d.TV, b, G, r0, r1);
            s[0] = {W.codec_head + static_cast<size_t>(r0) * d.H, static_cast<uint32_t>((r1 - r0) * d.H * 2)};
            return r1 > r0 ? 1 : 0;
        case CHEAD:
            split_rows(d.CV, b, G, r0, r1);
            s[0] = {W.lm_head[ph.pos - 1] + static_cast<size_t>(r0) * d.H, static_cast<uint32_t>((r1 - r0) * d.H * 2)};
            return r1 > r0 ? 1 : 0;
        default:
            return 0;
    }
}

} // namespace navi::fk
