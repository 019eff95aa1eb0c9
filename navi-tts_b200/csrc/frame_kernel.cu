// Device code of the persistent frame kernel (layout and phase program in frame_kernel.cuh).
#include "frame_kernel.cuh"

namespace navi::fk {

using namespace navi::dev;

struct Ctrl {
    volatile unsigned long long released;   // ring bytes the consumers have freed (monotonic)
    volatile int consumed;                  // chunks the consumers are done with
    volatile int abort;                     // this CTA is unwinding
    float red[2][NCW];                      // CTA reduction scratch
};

static_assert(sizeof(Ctrl) <= CTRL_BYTES, "control block outgrows its shared-memory slot");

struct Sm {
    uint64_t * bars;
    uint64_t * meta_end;
    uint32_t * meta_off;
    Ctrl * ctrl;
    int * codes;
    float * xres;
    float * hid;
    float * part;
    float * scratch;
    uint8_t * ring;
};

__device__ __forceinline__ Sm carve(char * base, const SmemLayout & L) {
    Sm s;
    s.bars = reinterpret_cast<uint64_t *>(base + L.bars);
    s.meta_end = reinterpret_cast<uint64_t *>(base + L.meta_end);
    s.meta_off = reinterpret_cast<uint32_t *>(base + L.meta_off);
    s.ctrl = reinterpret_cast<Ctrl *>(base + L.ctrl);
    s.codes = reinterpret_cast<int *>(base + L.codes);
    s.xres = reinterpret_cast<float *>(base + L.xres);
    s.hid = reinterpret_cast<float *>(base + L.hid);
    s.part = reinterpret_cast<float *>(base + L.part);
    s.scratch = reinterpret_cast<float *>(base + L.scratch);
    s.ring = reinterpret_cast<uint8_t *>(base + L.ring);
    return s;
}

// ---- abort handling -------------------------------------------------------------------------

__device__ __forceinline__ bool launch_aborted(const Args & A) { return ld_relaxed_u32(&A.w.ctl[2]) == A.tag_base; }

__device__ void raise_abort(const Args & A, Sm & S, int phase) {
    st_relaxed_u32(&A.w.ctl[1], static_cast<uint32_t>(phase));
    st_relaxed_u32(&A.w.ctl[3], blockIdx.x);
    __threadfence();
    st_relaxed_u32(&A.w.ctl[2], A.tag_base);
}

// Polls one exchange word until it carries `tag`. False when the launch is aborting.
__device__ __forceinline__ bool ll_get(const uint64_t * p, uint32_t tag, float & out, const Args & A, Sm & S, int phase) {
    uint64_t w = ll_load(p);
    if (static_cast<uint32_t>(w >> 32) == tag) { out = __uint_as_float(static_cast<uint32_t>(w)); return true; }
    const uint64_t t0 = globaltimer();
    uint32_t spins = 0;
    for (;;) {
        w = ll_load(p);
        if (static_cast<uint32_t>(w >> 32) == tag) { out = __uint_as_float(static_cast<uint32_t>(w)); return true; }
        if ((++spins & 31u) == 0) {
            if (S.ctrl->abort || launch_aborted(A)) return false;
            if (globaltimer() - t0 > A.timeout_ns) { raise_abort(A, S, phase); return false; }
        }
    }
}

// Consumer barrier that also decides, uniformly, whether any consumer thread failed.
// True when all succeeded. A failure is recorded for the producer warp.
__device__ __forceinline__ bool consumers_ok(Sm & S, bool ok) {
    const bool any_fail = named_sync_or(BID, NCT, !ok);
    if (any_fail && threadIdx.x == 0) S.ctrl->abort = 1;
    return !any_fail;
}

// n words -> dst (smem) by all consumer threads; ends with a (deciding) consumer barrier.
__device__ bool ll_vec(const uint64_t * src, int n, uint32_t tag, float * dst, const Args & A, Sm & S, int phase) {
    bool ok = true;
    for (int i = threadIdx.x; i < n && ok; i += NCT) {
        float v;
        ok = ll_get(src + i, tag, v, A, S, phase);
        dst[i] = v;
    }
    return consumers_ok(S, ok);
}

// ---- ring ------------------------------------------------------------------------------------

__device__ bool wait_chunk(const Args & A, Sm & S, int chunk, int phase) {
    const int slot = chunk % NSLOT;
    const uint32_t parity = static_cast<uint32_t>((chunk / NSLOT) & 1);
    bool ok = true;
    if (!mbar_try_wait(&S.bars[slot], parity)) {
        const uint64_t t0 = globaltimer();
        uint32_t spins = 0;
        while (!mbar_try_wait(&S.bars[slot], parity)) {
            if ((++spins & 15u) == 0) {
                if (S.ctrl->abort || launch_aborted(A)) { ok = false; break; }
                if (globaltimer() - t0 > A.timeout_ns) { raise_abort(A, S, phase); ok = false; break; }
            }
        }
    }
    return consumers_ok(S, ok);
}

__device__ __forceinline__ void release_chunk(Sm & S, int chunk) {
    // every consumer thread has passed a barrier after its last read of the chunk
    if (threadIdx.x == 0) {
        fence_proxy_async_smem();
        S.ctrl->released = S.meta_end[chunk % NSLOT];
        S.ctrl->consumed = chunk + 1;
    }
}

__device__ void prefetch_kv(const Args & A, const Phase & ph, int b) {
    const Dims & d = A.d;
    const int Sp = A.attn_split;
    if (b >= d.NKV * Sp) return;
    int a0, a1;
    split_rows(A.n_past + 1, b % Sp, Sp, a0, a1);
    a1 = min(a1, A.n_past);
    if (a1 <= a0) return;
    const size_t row = static_cast<size_t>(d.KV) * 2;
    const char * kp = reinterpret_cast<const char *>(A.kc[ph.layer]) + static_cast<size_t>(a0) * row;
    const char * vp = reinterpret_cast<const char *>(A.vc[ph.layer]) + static_cast<size_t>(a0) * row;
    const size_t bytes = static_cast<size_t>(a1 - a0) * row;
    for (size_t o = 0; o < bytes; o += 65536) {
        const uint32_t n = static_cast<uint32_t>(min(static_cast<size_t>(65536), bytes - o));
        bulk_prefetch_l2(kp + o, n);
        bulk_prefetch_l2(vp + o, n);
    }
}

__device__ void producer(const Args & A, Sm & S) {
    if ((threadIdx.x & 31) != 0) return;
    const ModelW & W = *A.mw;
    const int G = gridDim.x, b = blockIdx.x;
    const uint32_t RB = A.ring_bytes;
    uint64_t issued = 0;
    int chunk = 0;
    bool aborted = false;
    for (int p = 0; p < A.nphase && !aborted; ++p) {
        const Phase ph = A.prog[p];
        Seg seg[2];
        int r0, r1;
        const int ns = phase_segments(A, W, ph, b, G, seg, r0, r1);
        if (ns == 0) {
            if (ph.op == TATTN) prefetch_kv(A, ph, b);
            continue;
        }
        uint32_t total = 0;
        for (int i = 0; i < ns; ++i) total += seg[i].bytes;
        // The chunk takes virtual bytes [head, head + total) of the ring stream, contiguous in
        // shared memory (a chunk that would straddle the end starts the next lap). It may
        // only overwrite bytes whose data chunk the consumers have released; skipped tail
        // bytes hold no data, hence the min() with the end of the issued data.
        uint64_t head = issued;
        if (head % RB + total > RB) head += RB - head % RB;
        const uint64_t need = head + total > RB ? min(head + total - RB, issued) : 0;
        uint64_t t0 = 0;
        uint32_t spins = 0;
        while (S.ctrl->released < need || chunk - S.ctrl->consumed >= NSLOT) {
            if (S.ctrl->abort) { aborted = true; break; }
            if ((++spins & 63u) == 0) {
                const uint64_t now = globaltimer();
                if (t0 == 0) t0 = now;
                else if (now - t0 > 4 * A.timeout_ns) { raise_abort(A, S, p); S.ctrl->abort = 1; aborted = true; break; }
            }
            __nanosleep(64);
        }
        if (aborted) break;
        const int slot = chunk % NSLOT;
        S.meta_off[slot] = static_cast<uint32_t>(head % RB);
        issued = head + total;
        S.meta_end[slot] = issued;
        mbar_arrive_expect_tx(&S.bars[slot], total);
        uint32_t dst = static_cast<uint32_t>(head % RB);
        for (int i = 0; i < ns; ++i) {
            const char * src = static_cast<const char *>(seg[i].src);
            for (uint32_t o = 0; o < seg[i].bytes; o += PIECE) {
                const uint32_t n = min(PIECE, seg[i].bytes - o);
                bulk_g2s(S.ring + dst + o, src + o, n, &S.bars[slot]);
            }
            dst += seg[i].bytes;
        }
        ++chunk;
    }
    // Leave only when no copy into this CTA's shared memory is still in flight: on the
    // normal path the consumers have waited on every chunk; after an abort wait here.
    const uint64_t t0 = globaltimer();
    while (S.ctrl->consumed < chunk && !S.ctrl->abort) {
        __nanosleep(256);
        if (globaltimer() - t0 > 8 * A.timeout_ns) break;
    }
    for (int c = S.ctrl->consumed; c < chunk; ++c) {
        const uint64_t t1 = globaltimer();
        while (!mbar_try_wait(&S.bars[c % NSLOT], static_cast<uint32_t>((c / NSLOT) & 1))) {
            if (globaltimer() - t1 > 100000000ull) break;   // 100 ms: copies complete in microseconds
        }
    }
}

// ---- consumer building blocks ---------------------------------------------------------------------

// y-partials of rows [0, nrows) of a row-major f16 matrix in shared memory against NC input
// columns. Work item = 4 rows x 256 columns; lane covers columns {4l..4l+3} and {128+4l..}.
// part[(c * nrows + row) * nseg + seg]. Caller follows with a consumer barrier.
template <int NC>
__device__ void gemv_part(const __half * Ws, int nrows, int ncols, const float * xin, int xstride, float * part) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nseg = ncols >> 8, ngrp = (nrows + 3) >> 2, nitems = ngrp * nseg;
    for (int it = warp; it < nitems; it += NCW) {
        const int grp = it / nseg, seg = it - grp * nseg;
        const int col = seg * 256 + lane * 4;
        float4 xa[NC], xb[NC];
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            xa[c] = *reinterpret_cast<const float4 *>(xin + c * xstride + col);
            xb[c] = *reinterpret_cast<const float4 *>(xin + c * xstride + col + 128);
        }
        float acc[4][NC];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int row = grp * 4 + r;
            if (row < nrows) {
                const __half * wr = Ws + static_cast<size_t>(row) * ncols + col;
                const uint2 wa = *reinterpret_cast<const uint2 *>(wr);
                const uint2 wb = *reinterpret_cast<const uint2 *>(wr + 128);
#pragma unroll
                for (int c = 0; c < NC; ++c) acc[r][c] = dot4h(wa, xa[c]) + dot4h(wb, xb[c]);
            } else {
#pragma unroll
                for (int c = 0; c < NC; ++c) acc[r][c] = 0.f;
            }
        }
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int c = 0; c < NC; ++c) acc[r][c] = warp_sum(acc[r][c]);
        if (lane == 0) {
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const int row = grp * 4 + r;
                if (row < nrows)
#pragma unroll
                    for (int c = 0; c < NC; ++c) part[(c * nrows + row) * nseg + seg] = acc[r][c];
            }
        }
    }
}

__device__ __forceinline__ float part_sum(const float * part, int c, int row, int nrows, int nseg) {
    const float * p = part + (c * nrows + row) * nseg;
    float s = 0.f;
    for (int k = 0; k < nseg; ++k) s += p[k];
    return s;
}

__device__ __forceinline__ void run_gemv(int ncol, const __half * Ws, int nrows, int ncols, const float * xin, int xstride,
                                         float * part) {
    if (ncol == 2) gemv_part<2>(Ws, nrows, ncols, xin, xstride, part);
    else gemv_part<1>(Ws, nrows, ncols, xin, xstride, part);
}

// out[c] = x[c] * rsqrt(mean(x[c]^2) + eps) * w for c < ncol (x, out in shared memory).
__device__ void rmsnorm_cols(Sm & S, const float * x, int xstride, const float * w, float eps, int ncol, int n, float * out,
                             int ostride) {
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    float ss[2] = {0.f, 0.f};
#pragma unroll
    for (int c = 0; c < 2; ++c) {
        if (c >= ncol) continue;
        for (int i = tid; i < n; i += NCT) { const float v = x[c * xstride + i]; ss[c] += v * v; }
        ss[c] = warp_sum(ss[c]);
        if (lane == 0) S.ctrl->red[c][wid] = ss[c];
    }
    named_sync(BID, NCT);
    for (int c = 0; c < ncol; ++c) {
        float t = 0.f;
#pragma unroll
        for (int k = 0; k < NCW; ++k) t += S.ctrl->red[c][k];
        const float scale = rsqrtf(t / static_cast<float>(n) + eps);
        for (int i = tid; i < n; i += NCT) out[c * ostride + i] = x[c * xstride + i] * scale * __ldg(w + i);
    }
    named_sync(BID, NCT);
}

__device__ __forceinline__ void row_f16_to_smem(const __half * row, int n, float * dst) {
    for (int i = threadIdx.x; i < n; i += NCT) dst[i] = __half2float(row[i]);
}

__device__ SampleScratch sampler_scratch(Sm & S, int Vmax) {
    SampleScratch sc;
    float * base = S.scratch;
    sc.s = base;
    sc.e = base + Vmax;
    sc.idx = reinterpret_cast<int *>(base + 2 * Vmax);
    sc.ord = reinterpret_cast<int *>(base + 3 * Vmax);
    sc.keep = reinterpret_cast<uint8_t *>(base + 4 * Vmax);
    sc.hist = reinterpret_cast<unsigned *>(base + 4 * Vmax + (Vmax + 3) / 4);
    sc.red = base + 4 * Vmax + (Vmax + 3) / 4 + 256;
    return sc;
}

__device__ SampleCfg sample_cfg(const Args & A, int codebook) {
    SampleCfg c{};
    if (codebook == 0) {
        c.temperature = A.temp; c.top_k = A.top_k; c.top_p = A.top_p;
        c.talker_mods = 1;
        c.suppress_from = A.suppress_from; c.eos_id = A.eos_id; c.min_frames = A.min_frames;
        c.repetition_penalty = A.rep;
        c.seen = A.w.seen;
    } else {
        c.temperature = A.cp_temp; c.top_k = A.cp_top_k; c.top_p = A.cp_top_p;
        c.talker_mods = 0;
    }
    c.rng = A.rng; c.seed = A.seed; c.frame_index = A.frame_index; c.codebook = codebook;
    c.pcg_seed = A.pcg_seed[codebook];
    return c;
}

// ---- attention phase (q/k norm + RoPE + KV store + split-KV GQA attention) ----------------------------

__device__ bool attention_phase(const Args & A, Sm & S, const Phase & ph, bool talker, uint32_t tag, uint32_t ptag, int p) {
    const Dims & d = A.d;
    const ModelW & W = *A.mw;
    const int HD = d.HD, GR = d.GROUP, ncol = ph.ncol, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int Sp = talker ? A.attn_split : 1;
    const int b = blockIdx.x;
    if (b >= d.NKV * Sp) return true;
    const int g = b / Sp, s = b - g * Sp;
    const int pos = talker ? A.n_past : ph.pos;
    const LayerW & L = talker ? W.tl[ph.layer] : W.cp[ph.layer];
    const float eps = talker ? d.eps_t : d.eps_c;
    const float * inv_freq = talker ? A.inv_freq_t : A.inv_freq_c;
    __half * kc = talker ? A.kc[ph.layer] : A.w.ckc + static_cast<size_t>(ph.layer) * NCB * d.KV;
    __half * vc = talker ? A.vc[ph.layer] : A.w.cvc + static_cast<size_t>(ph.layer) * NCB * d.KV;
    float * qs = S.scratch;                        // [2][MAX_GROUP][HD]
    float * ks = qs + 2 * MAX_GROUP * HD;          // [2][HD]
    float * vs = ks + 2 * HD;                      // [2][HD]
    float * wst = vs + 2 * HD;                     // [NCW][2][MAX_GROUP][HD + 2]
    const int WST = HD + 2;
    // 1. this KV head's raw q (GROUP heads), k, v for each column
    {
        const int per = (GR + 2) * HD;
        bool ok = true;
        for (int i = tid; i < ncol * per && ok; i += NCT) {
            const int c = i / per, rem = i - c * per, j = rem / HD, e = rem - j * HD;
            const uint64_t * src = A.w.qkv + static_cast<size_t>(c) * d.QKV;
            int idx;
            float * dst;
            if (j < GR) { idx = (g * GR + j) * HD + e; dst = qs + (c * MAX_GROUP + j) * HD + e; }
            else if (j == GR) { idx = d.Q + g * HD + e; dst = ks + c * HD + e; }
            else { idx = d.Q + d.KV + g * HD + e; dst = vs + c * HD + e; }
            float v;
            ok = ll_get(src + idx, ptag, v, A, S, p);
            *dst = v;
        }
        if (!consumers_ok(S, ok)) return false;
    }
    // 2. per-head RMSNorm of q and k, RoPE at pos + c, f16 rounding of k and v
    {
        const int nvec = ncol * (GR + 1);
        const int EPL = HD / 32;   // elements per lane: lane + 32 t
        for (int v = warp; v < nvec; v += NCW) {
            const int c = v / (GR + 1), j = v - c * (GR + 1);
            float * vec = j < GR ? qs + (c * MAX_GROUP + j) * HD : ks + c * HD;
            const float * nw = j < GR ? L.qn : L.kn;
            float e[4];
            float ss = 0.f;
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                e[t] = t < EPL ? vec[lane + 32 * t] : 0.f;
                ss += e[t] * e[t];
            }
            ss = warp_sum(ss);
            const float scale = rsqrtf(ss / static_cast<float>(HD) + eps);
#pragma unroll
            for (int t = 0; t < 4; ++t) if (t < EPL) e[t] = e[t] * scale * __ldg(nw + lane + 32 * t);
            const float fpos = static_cast<float>(pos + c);
#pragma unroll
            for (int t = 0; t < 2; ++t) {
                if (t >= EPL / 2) continue;
                const int i = lane + 32 * t;   // pairs (i, i + HD/2)
                const float ang = fpos * __ldg(inv_freq + i);
                float sn, cs;
                sincosf(ang, &sn, &cs);
                const float x0 = e[t], x1 = (EPL == 4) ? e[t + 2] : e[t + 1];
                float r0 = x0 * cs - x1 * sn, r1 = x0 * sn + x1 * cs;
                if (j == GR) { r0 = f16_round(r0); r1 = f16_round(r1); }
                vec[i] = r0;
                vec[i + HD / 2] = r1;
            }
        }
        for (int i = tid; i < ncol * HD; i += NCT) vs[i] = f16_round(vs[i]);
        named_sync(BID, NCT);
    }
    // 3. the new positions' K/V rows (the split holding them)
    if (s == Sp - 1) {
        for (int i = tid; i < ncol * HD; i += NCT) {
            const int c = i / HD, e = i - c * HD;
            const size_t o = static_cast<size_t>(pos + c) * d.KV + g * HD + e;
            kc[o] = __float2half_rn(ks[i]);
            vc[o] = __float2half_rn(vs[i]);
        }
    }
    // 4. online-softmax attention over this split's positions, one position per warp per step
    int a0, a1;
    split_rows(pos + ncol, s, Sp, a0, a1);
    const float scale = rsqrtf(static_cast<float>(HD));
    {
        const int DPL = HD / 32;   // contiguous dims per lane
        float qreg[2][MAX_GROUP][4];
        float m[2][MAX_GROUP], l[2][MAX_GROUP], acc[2][MAX_GROUP][4];
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int j = 0; j < MAX_GROUP; ++j) {
                m[c][j] = -INFINITY; l[c][j] = 0.f;
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    acc[c][j][t] = 0.f;
                    qreg[c][j][t] = (c < ncol && j < GR && t < DPL) ? qs[(c * MAX_GROUP + j) * HD + lane * DPL + t] : 0.f;
                }
            }
        for (int jp = a0 + warp; jp < a1; jp += NCW) {
            float kv[4] = {0.f, 0.f, 0.f, 0.f}, vv[4] = {0.f, 0.f, 0.f, 0.f};
            if (jp < pos) {
                const __half * kr = kc + static_cast<size_t>(jp) * d.KV + g * HD + lane * DPL;
                const __half * vr = vc + static_cast<size_t>(jp) * d.KV + g * HD + lane * DPL;
                if (DPL == 4) {
                    const uint2 ku = talker ? __ldg(reinterpret_cast<const uint2 *>(kr)) : __ldcg(reinterpret_cast<const uint2 *>(kr));
                    const uint2 vu = talker ? __ldg(reinterpret_cast<const uint2 *>(vr)) : __ldcg(reinterpret_cast<const uint2 *>(vr));
                    const float2 k0 = __half22float2(*reinterpret_cast<const __half2 *>(&ku.x)), k1 = __half22float2(*reinterpret_cast<const __half2 *>(&ku.y));
                    const float2 v0 = __half22float2(*reinterpret_cast<const __half2 *>(&vu.x)), v1 = __half22float2(*reinterpret_cast<const __half2 *>(&vu.y));
                    kv[0] = k0.x; kv[1] = k0.y; kv[2] = k1.x; kv[3] = k1.y;
                    vv[0] = v0.x; vv[1] = v0.y; vv[2] = v1.x; vv[3] = v1.y;
                } else {
#pragma unroll
                    for (int t = 0; t < 4; ++t) {
                        if (t >= DPL) continue;
                        kv[t] = __half2float(__ushort_as_half(__ldcg(reinterpret_cast<const unsigned short *>(kr + t))));
                        vv[t] = __half2float(__ushort_as_half(__ldcg(reinterpret_cast<const unsigned short *>(vr + t))));
                    }
                }
            } else {
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    if (t >= DPL) continue;
                    kv[t] = ks[(jp - pos) * HD + lane * DPL + t];
                    vv[t] = vs[(jp - pos) * HD + lane * DPL + t];
                }
            }
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                if (c >= ncol || jp > pos + c) continue;
#pragma unroll
                for (int j = 0; j < MAX_GROUP; ++j) {
                    if (j >= GR) continue;
                    float dsum = 0.f;
#pragma unroll
                    for (int t = 0; t < 4; ++t) dsum += qreg[c][j][t] * kv[t];
                    const float sc = warp_sum(dsum) * scale;
                    const float mn = fmaxf(m[c][j], sc);
                    const float corr = expf(m[c][j] - mn), pe = expf(sc - mn);
                    l[c][j] = l[c][j] * corr + pe;
#pragma unroll
                    for (int t = 0; t < 4; ++t) acc[c][j][t] = acc[c][j][t] * corr + pe * vv[t];
                    m[c][j] = mn;
                }
            }
        }
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int j = 0; j < MAX_GROUP; ++j) {
                if (c >= ncol || j >= GR) continue;
                float * st = wst + ((warp * 2 + c) * GR + j) * WST;
                if (lane == 0) { st[0] = m[c][j]; st[1] = l[c][j]; }
#pragma unroll
                for (int t = 0; t < 4; ++t) if (t < DPL) st[2 + lane * DPL + t] = acc[c][j][t];
            }
        named_sync(BID, NCT);
    }
    // 5. combine the warps (fixed order) into this split's partial, or the final output
    {
        const int nout = ncol * GR * HD;
        uint64_t * part = A.w.part + static_cast<size_t>(g * MAX_SPLIT + s) * 2 * MAX_GROUP * WST;
        for (int i = tid; i < nout; i += NCT) {
            const int c = i / (GR * HD), rem = i - c * GR * HD, j = rem / HD, e = rem - j * HD;
            float M = -INFINITY;
            for (int w = 0; w < NCW; ++w) M = fmaxf(M, wst[((w * 2 + c) * GR + j) * WST]);
            float Ls = 0.f, As = 0.f;
            if (M != -INFINITY) {
                for (int w = 0; w < NCW; ++w) {
                    const float * st = wst + ((w * 2 + c) * GR + j) * WST;
                    if (st[0] == -INFINITY) continue;
                    const float f = expf(st[0] - M);
                    Ls += st[1] * f;
                    As += st[2 + e] * f;
                }
            }
            if (Sp == 1) {
                ll_store(A.w.attn + static_cast<size_t>(c) * d.Q + (g * GR + j) * HD + e, As / Ls, tag);
            } else {
                uint64_t * pp = part + (c * MAX_GROUP + j) * WST;
                if (e == 0) { ll_store(pp + 0, M, tag); ll_store(pp + 1, Ls, tag); }
                ll_store(pp + 2 + e, As, tag);
            }
        }
    }
    if (Sp > 1 && s == 0) {
        const int nout = ncol * GR * HD;
        bool ok = true;
        for (int i = tid; i < nout && ok; i += NCT) {
            const int c = i / (GR * HD), rem = i - c * GR * HD, j = rem / HD, e = rem - j * HD;
            float Ms[MAX_SPLIT], Lv[MAX_SPLIT], Av[MAX_SPLIT];
            float M = -INFINITY;
            for (int k = 0; k < Sp && ok; ++k) {
                const uint64_t * pp = A.w.part + (static_cast<size_t>(g * MAX_SPLIT + k) * 2 * MAX_GROUP + c * MAX_GROUP + j) * WST;
                ok = ll_get(pp + 0, tag, Ms[k], A, S, p) && ll_get(pp + 1, tag, Lv[k], A, S, p) && ll_get(pp + 2 + e, tag, Av[k], A, S, p);
                M = fmaxf(M, Ms[k]);
            }
            if (!ok) break;
            float Ls = 0.f, As = 0.f;
            for (int k = 0; k < Sp; ++k) {
                if (Ms[k] == -INFINITY) continue;
                const float f = expf(Ms[k] - M);
                Ls += Lv[k] * f;
                As += Av[k] * f;
            }
            ll_store(A.w.attn + static_cast<size_t>(c) * d.Q + (g * GR + j) * HD + e, As / Ls, tag);
        }
        if (!consumers_ok(S, ok)) return false;
    } else {
        named_sync(BID, NCT);
    }
    return true;
}

// ---- the consumer: the phase program ----------------------------------------------------------------

__device__ void consumer(const Args & A, Sm & S) {
    const Dims & d = A.d;
    const ModelW & W = *A.mw;
    const int G = gridDim.x, b = blockIdx.x, tid = threadIdx.x;
    const int XS = max(d.H, max(d.Q, d.F));   // xin column stride
    const int Vmax = max(d.TV, d.CV);
    float * xin = S.scratch;
    int chunk = 0;
    for (int p = 0; p < A.nphase; ++p) {
        const Phase ph = A.prog[p];
        const uint32_t tag = A.tag_base + static_cast<uint32_t>(p), ptag = tag - 1u;
        const bool talker = ph.op <= THEAD;
        const int ncol = ph.ncol;
        Seg seg[2];
        int r0, r1;
        const int ns = phase_segments(A, W, ph, b, G, seg, r0, r1);
        const int nr = r1 - r0;
        const LayerW * L = ph.op <= TDOWN ? &W.tl[ph.layer] : (ph.op >= CQKV && ph.op <= CDOWN ? &W.cp[ph.layer] : nullptr);
        const float eps = talker ? d.eps_t : d.eps_c;

        if (ph.op == TATTN || ph.op == CATTN) {
            if (!attention_phase(A, S, ph, talker, tag, ptag, p)) break;
            if (A.prof && b == 0 && tid == 0) A.prof[p] = globaltimer();
            continue;
        }

        // ---- prologue: this phase's inputs into shared memory
        bool ok = true;
        switch (ph.op) {
            case TQKV: case CQKV: {
                if (ph.layer == 0 && ph.op == TQKV) {
                    for (int i = tid; i < d.H; i += NCT) S.xres[i] = __ldcg(A.step_in + i);
                    named_sync(BID, NCT);
                } else if (ph.layer == 0 && ph.pos == 0) {
                    // code-predictor positions 0 and 1: sample codebook 0 first
                    const SampleScratch sc = sampler_scratch(S, Vmax);
                    if (A.logits_in) {
                        for (int i = tid; i < d.TV; i += NCT) sc.s[i] = __ldcg(A.logits_in + i);
                        named_sync(BID, NCT);
                    } else {
                        ok = ll_vec(A.w.logits, d.TV, ptag, sc.s, A, S, p);
                        if (!ok) break;
                    }
                    const int cb0 = sample_cta(d.TV, sample_cfg(A, 0), sc, BID);
                    if (tid == 0) S.codes[0] = cb0;
                    for (int i = tid; i < d.H; i += NCT) {
                        S.xres[i] = A.hidden_in ? __ldcg(A.hidden_in + i) : S.hid[i];
                        S.xres[d.H + i] = __half2float(W.tl_emb[static_cast<size_t>(cb0) * d.H + i]);
                    }
                    named_sync(BID, NCT);
                } else if (ph.layer == 0) {
                    const SampleScratch sc = sampler_scratch(S, Vmax);
                    ok = ll_vec(A.w.clogits + static_cast<size_t>(ph.pos - 2) * d.CV, d.CV, ptag, sc.s, A, S, p);
                    if (!ok) break;
                    const int code = sample_cta(d.CV, sample_cfg(A, ph.pos - 1), sc, BID);
                    if (tid == 0) S.codes[ph.pos - 1] = code;
                    row_f16_to_smem(W.cp_emb[ph.pos - 2] + static_cast<size_t>(code) * d.H, d.H, S.xres);
                    named_sync(BID, NCT);
                } else {
                    for (int c = 0; c < ncol && ok; ++c) ok = ll_vec(A.w.x + static_cast<size_t>(c) * d.H, d.H, ptag, S.xres + c * d.H, A, S, p);
                    if (!ok) break;
                }
                rmsnorm_cols(S, S.xres, d.H, L->ln1, eps, ncol, d.H, xin, XS);
                break;
            }
            case TO: case CO:
                for (int c = 0; c < ncol && ok; ++c) ok = ll_vec(A.w.attn + static_cast<size_t>(c) * d.Q, d.Q, ptag, xin + c * XS, A, S, p);
                break;
            case TGU: case CGU:
                for (int c = 0; c < ncol && ok; ++c) ok = ll_vec(A.w.x + static_cast<size_t>(c) * d.H, d.H, ptag, S.xres + c * d.H, A, S, p);
                if (ok) rmsnorm_cols(S, S.xres, d.H, L->ln2, eps, ncol, d.H, xin, XS);
                break;
            case TDOWN: case CDOWN:
                for (int c = 0; c < ncol && ok; ++c) ok = ll_vec(A.w.h + static_cast<size_t>(c) * d.F, d.F, ptag, xin + c * XS, A, S, p);
                break;
            case THEAD:
                ok = ll_vec(A.w.x, d.H, ptag, S.xres, A, S, p);
                if (!ok) break;
                rmsnorm_cols(S, S.xres, d.H, W.tl_norm, d.eps_t, 1, d.H, xin, XS);
                for (int i = tid; i < d.H; i += NCT) {
                    S.hid[i] = xin[i];
                    if (b == 0) A.w.hidden[i] = xin[i];
                }
                break;
            case CHEAD: {
                const int cc = ncol - 1;
                ok = ll_vec(A.w.x + static_cast<size_t>(cc) * d.H, d.H, ptag, S.xres, A, S, p);
                if (!ok) break;
                rmsnorm_cols(S, S.xres, d.H, W.cp_norm, d.eps_c, 1, d.H, xin, XS);
                break;
            }
            case FINAL: {
                const SampleScratch sc = sampler_scratch(S, Vmax);
                ok = ll_vec(A.w.clogits + static_cast<size_t>(NCB - 2) * d.CV, d.CV, ptag, sc.s, A, S, p);
                if (!ok) break;
                const int code = sample_cta(d.CV, sample_cfg(A, NCB - 1), sc, BID);
                if (tid == 0) S.codes[NCB - 1] = code;
                named_sync(BID, NCT);
                int e0, e1;
                split_rows(d.H, b, G, e0, e1);
                for (int i = e0 + tid; i < e1; i += NCT) {
                    float v = __half2float(W.tl_emb[static_cast<size_t>(S.codes[0]) * d.H + i]);
                    for (int cb = 0; cb < NCB - 1; ++cb)
                        v = __fadd_rn(v, __half2float(W.cp_emb[cb][static_cast<size_t>(S.codes[cb + 1]) * d.H + i]));
                    v = __fadd_rn(v, __ldcg(A.trailing + i));
                    A.step_out[i] = v;
                }
                if (b == 0 && tid < NCB) A.w.codes[tid] = S.codes[tid];
                if (b == 0 && tid == 0) {
                    if (S.codes[0] != A.eos_id) A.w.seen[S.codes[0]] = 1;
                    __threadfence();
                    st_relaxed_u32(&A.w.ctl[0], A.tag_base);
                }
                break;
            }
            default: break;
        }
        if (!ok) break;
        if (ns == 0) {
            if (A.prof && b == 0 && tid == 0) A.prof[p] = globaltimer();
            continue;
        }

        // ---- weights of this phase, then the dot products
        if (!wait_chunk(A, S, chunk, p)) break;
        const __half * Ws = reinterpret_cast<const __half *>(S.ring + S.meta_off[chunk % NSLOT]);
        int nrows = nr, ncols = d.H;
        if (ph.op == TO || ph.op == CO) ncols = d.Q;
        else if (ph.op == TDOWN || ph.op == CDOWN) ncols = d.F;
        else if (ph.op == TGU || ph.op == CGU) nrows = 2 * nr;
        const int gcol = (ph.op == THEAD || ph.op == CHEAD) ? 1 : ncol;
        const int nseg = ncols >> 8;
        run_gemv(gcol, Ws, nrows, ncols, xin, XS, S.part);
        named_sync(BID, NCT);
        release_chunk(S, chunk);
        ++chunk;

        // ---- epilogue: outputs to the exchange words
        const uint32_t t = tag;
        switch (ph.op) {
            case TQKV: case CQKV:
                for (int k = tid; k < ncol * nr; k += NCT) {
                    const int c = k / nr, r = k - c * nr;
                    ll_store(A.w.qkv + static_cast<size_t>(c) * d.QKV + r0 + r, part_sum(S.part, c, r, nrows, nseg), t);
                }
                break;
            case TO: case CO: case TDOWN: case CDOWN:
                for (int k = tid; k < ncol * nr; k += NCT) {
                    const int c = k / nr, r = k - c * nr;
                    const float x = S.xres[c * d.H + r0 + r] + part_sum(S.part, c, r, nrows, nseg);
                    ll_store(A.w.x + static_cast<size_t>(c) * d.H + r0 + r, x, t);
                }
                break;
            case TGU: case CGU:
                for (int k = tid; k < ncol * nr; k += NCT) {
                    const int c = k / nr, r = k - c * nr;
                    const float gv = part_sum(S.part, c, r, nrows, nseg), uv = part_sum(S.part, c, nr + r, nrows, nseg);
                    ll_store(A.w.h + static_cast<size_t>(c) * d.F + r0 + r, gv / (1.f + expf(-gv)) * uv, t);
                }
                break;
            case THEAD:
                for (int r = tid; r < nr; r += NCT) ll_store(A.w.logits + r0 + r, part_sum(S.part, 0, r, nrows, nseg), t);
                break;
            case CHEAD:
                for (int r = tid; r < nr; r += NCT)
                    ll_store(A.w.clogits + static_cast<size_t>(ph.pos - 1) * d.CV + r0 + r, part_sum(S.part, 0, r, nrows, nseg), t);
                break;
            default: break;
        }
        named_sync(BID, NCT);   // xres and the partials are rewritten by the next prologue
        if (A.prof && b == 0 && tid == 0) A.prof[p] = globaltimer();
    }
}

__global__ void __launch_bounds__(NTHR, 1) k_frame(const __grid_constant__ Args A) {
    extern __shared__ __align__(128) char smem[];
    const SmemLayout L = smem_layout(A.d, A.ring_bytes, A.scratch_floats, A.part_floats);
    Sm S = carve(smem, L);
    if (threadIdx.x == 0) {
        for (int i = 0; i < NSLOT; ++i) mbar_init(&S.bars[i], 1);
        S.ctrl->released = 0;
        S.ctrl->consumed = 0;
        S.ctrl->abort = 0;
        fence_mbar_init();
    }
    __syncthreads();
    if (A.prof && blockIdx.x == 0 && threadIdx.x == 0) A.prof[A.nphase] = globaltimer();
    if (threadIdx.x >= NCT) producer(A, S);
    else consumer(A, S);
}

// A standalone launch of the device sampler on given logits (one CTA), for parity tests.
__global__ void __launch_bounds__(NCT, 1) k_sample(const float * logits, int V, SampleCfg cfg, int * out) {
    extern __shared__ __align__(16) float sbuf[];
    SampleScratch sc;
    sc.s = sbuf;
    sc.e = sbuf + V;
    sc.idx = reinterpret_cast<int *>(sbuf + 2 * V);
    sc.ord = reinterpret_cast<int *>(sbuf + 3 * V);
    sc.keep = reinterpret_cast<uint8_t *>(sbuf + 4 * V);
    sc.hist = reinterpret_cast<unsigned *>(sbuf + 4 * V + (V + 3) / 4);
    sc.red = sbuf + 4 * V + (V + 3) / 4 + 256;
    for (int i = threadIdx.x; i < V; i += NCT) sc.s[i] = logits[i];
    named_sync(BID, NCT);
    const int c = sample_cta(V, cfg, sc, BID);
    if (threadIdx.x == 0) *out = c;
}

} // namespace navi::fk
