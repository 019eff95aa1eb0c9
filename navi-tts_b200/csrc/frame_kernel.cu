// Device code of the persistent frame kernel (layout and phase program in frame_kernel.cuh).
#include "frame_kernel.cuh"

namespace navi::fk {

using namespace navi::dev;

struct Ctrl {
    volatile unsigned long long released;   // ring bytes the consumers have freed (monotonic)
    volatile int consumed;                  // chunks the consumers are done with
    volatile int abort;                     // this CTA is unwinding
    float red[MAXC][NCW];                   // CTA reduction scratch
};

static_assert(sizeof(Ctrl) <= CTRL_BYTES, "control block outgrows its shared-memory slot");

struct Sm {
    uint64_t * bars;
    uint64_t * meta_end;
    uint32_t * meta_off;     // physical offset of the chunk's logical byte 0
    uint32_t * meta_split;   // logical offset where the chunk continues at the ring's start
    Ctrl * ctrl;
    int * codes;        // [MAX_B][NCB]
    float * xres;
    float * hid;
    float * part;
    float * scratch;
    __half * cpkv;
    uint8_t * ring;
};

__device__ __forceinline__ Sm carve(char * base, const SmemLayout & L) {
    Sm s;
    s.bars = reinterpret_cast<uint64_t *>(base + L.bars);
    s.meta_end = reinterpret_cast<uint64_t *>(base + L.meta_end);
    s.meta_off = reinterpret_cast<uint32_t *>(base + L.meta_off);
    s.meta_split = reinterpret_cast<uint32_t *>(base + L.meta_split);
    s.ctrl = reinterpret_cast<Ctrl *>(base + L.ctrl);
    s.codes = reinterpret_cast<int *>(base + L.codes);
    s.xres = reinterpret_cast<float *>(base + L.xres);
    s.hid = reinterpret_cast<float *>(base + L.hid);
    s.part = reinterpret_cast<float *>(base + L.part);
    s.scratch = reinterpret_cast<float *>(base + L.scratch);
    s.cpkv = reinterpret_cast<__half *>(base + L.cpkv);
    s.ring = reinterpret_cast<uint8_t *>(base + L.ring);
    return s;
}

// ---- abort handling -------------------------------------------------------------------------

__device__ __forceinline__ bool launch_aborted(const Args & A) { return ld_relaxed_u32(&A.w.ctl[2]) == A.tag_base; }

__device__ __noinline__ void raise_abort(const Args & A, int phase) {
    st_relaxed_u32(&A.w.ctl[1], static_cast<uint32_t>(phase));
    st_relaxed_u32(&A.w.ctl[3], blockIdx.x);
    __threadfence();
    st_relaxed_u32(&A.w.ctl[2], A.tag_base);
}

// Consumer barrier that also decides, uniformly, whether any consumer thread failed.
// True when all succeeded. A failure is recorded for the producer warp.
__device__ __forceinline__ bool consumers_ok(Sm & S, bool ok) {
    const bool any_fail = named_sync_or(BID, NCT, !ok);
    if (any_fail && threadIdx.x == 0) S.ctrl->abort = 1;
    return !any_fail;
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
                if (globaltimer() - t0 > A.timeout_ns) { raise_abort(A, phase); ok = false; break; }
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

// Address of logical byte x of ring chunk `chunk` (see the producer's cut).
__device__ __forceinline__ const uint8_t * chunk_at(const Sm & S, int chunk, uint32_t x) {
    const int slot = chunk % NSLOT;
    const uint32_t cut = S.meta_split[slot];
    return S.ring + (x < cut ? S.meta_off[slot] + x : x - cut);
}

// The producer warp streams every phase's slice into the ring, in phase order. All 32 lanes
// take the same ring decisions; lane 0 writes the slot's bookkeeping and arms its mbarrier
// with the chunk's byte count, then the chunk's rows are dealt to the lanes round-robin, so
// the many small row copies of an attention chunk (one per cached position) are issued 32 at
// a time instead of one after another.
__device__ void producer(const Args & A, Sm & S) {
    const int lane = threadIdx.x & 31;
    const ModelW & W = *A.mw;
    const int G = gridDim.x, b = blockIdx.x;
    const Rows R = cta_rows(A.d, b, G);
    const uint32_t RB = A.ring_bytes;
    uint64_t issued = 0;
    int chunk = 0;
    bool aborted = false;
    // code-predictor layers below cp_keep_layers are read 15 times a frame: keep them in L2;
    // everything else (talker weights, KV rows, heads) is read once and streams through
    const uint64_t keep = l2_policy_keep(), stream = l2_policy_stream();
    for (int p = 0; p < A.nphase && !aborted; ++p) {
        const Phase ph = A.prog[p];
        Seg seg[MAX_SEG];
        int r0, r1;
        const int ns = phase_segments(A, W, ph, b, R, seg, r0, r1);
        if (ns == 0) continue;
        uint32_t total = 0;
        for (int i = 0; i < ns; ++i) total += seg[i].bytes * seg[i].rows;
        // The chunk takes the next bytes of the ring stream. When it does not fit before the
        // ring's end it is cut once (chunk_split): its first part fills the end, the rest
        // continues at the ring's start, and the bytes between the cut point's offset and the
        // end stay unused. It may only overwrite bytes whose chunk the consumers have
        // released; unused bytes hold no data, hence the min() with the end of the issued data.
        // a chunk with boxed (tensor-map) loads starts on a 128-byte boundary, as those copies'
        // shared-memory destinations must (its segments are all multiples of 128 bytes); the
        // bytes skipped hold no data
        bool boxed = false;
        for (int i = 0; i < ns; ++i) boxed = boxed || seg[i].tmap != nullptr;
        const uint64_t head = boxed ? (issued + 127) / 128 * 128 : issued;
        const uint32_t pos = static_cast<uint32_t>(head % RB);
        uint32_t cut = total;
        uint64_t end = head + total;
        if (pos + total > RB) {
            cut = chunk_split(seg, ns, RB - pos);
            if (total - cut > pos) cut = 0;   // the rest would reach the first part: start over
            end = head + (RB - pos) + (total - cut);
        }
        const uint64_t need = end > RB ? min(end - RB, issued) : 0;
        uint64_t t0 = 0;
        uint32_t spins = 0;
        while (S.ctrl->released < need || chunk - S.ctrl->consumed >= NSLOT) {
            if (S.ctrl->abort) { aborted = true; break; }
            if ((++spins & 63u) == 0) {
                const uint64_t now = globaltimer();
                if (t0 == 0) t0 = now;
                else if (now - t0 > 4 * A.timeout_ns) { raise_abort(A, p); S.ctrl->abort = 1; aborted = true; break; }
            }
            __nanosleep(64);
        }
        aborted = __shfl_sync(0xffffffffu, aborted ? 1 : 0, 0) != 0;
        if (aborted) break;
        const int slot = chunk % NSLOT;
        const uint32_t moff = cut > 0 ? pos : 0u;
        if (lane == 0) {
            S.meta_off[slot] = moff;
            S.meta_split[slot] = cut;
            S.meta_end[slot] = end;
            mbar_arrive_expect_tx(&S.bars[slot], total);
        }
        issued = end;
        __syncwarp();
        const bool kept = ph.op >= CQKV && ph.op <= CDOWN && ph.layer < A.cp_keep_layers;
        const uint64_t pol = kept ? keep : stream;
        uint32_t lo = 0;   // logical offset of the segment's first byte
        uint32_t gr = 0;   // rows of the chunk before this segment: row gr + r goes to lane (gr + r) % 32
        for (int i = 0; i < ns; ++i) {
            if (seg[i].tmap) {
                // boxed loads (one per box, dealt to the lanes like rows)
                tensormap_acquire(seg[i].tmap);
                for (uint32_t r = (lane - gr % 32u + 32u) % 32u; r < seg[i].rows; r += 32) {
                    const uint32_t x = lo + r * seg[i].bytes;
                    tma_box_2d(S.ring + (x < cut ? moff + x : x - cut), seg[i].tmap, seg[i].tx, seg[i].ty + static_cast<int>(r) * KV_BOX,
                               &S.bars[slot]);
                }
                lo += seg[i].bytes * seg[i].rows;
                gr += seg[i].rows;
                continue;
            }
            for (uint32_t r = (lane - gr % 32u + 32u) % 32u; r < seg[i].rows; r += 32) {
                const char * src = static_cast<const char *>(seg[i].src) + static_cast<size_t>(r) * seg[i].stride;
                const uint32_t rl = lo + r * seg[i].bytes;
                for (uint32_t o = 0; o < seg[i].bytes;) {
                    // up to PIECE bytes, not across the cut
                    const uint32_t x = rl + o;
                    uint32_t n = min(PIECE, seg[i].bytes - o);
                    if (x < cut) n = min(n, cut - x);
                    const uint32_t phys = x < cut ? moff + x : x - cut;
                    bulk_g2s_hint(S.ring + phys, src + o, n, &S.bars[slot], pol);
                    o += n;
                }
            }
            lo += seg[i].bytes * seg[i].rows;
            gr += seg[i].rows;
        }
        ++chunk;
    }
    // Leave only when no copy into this CTA's shared memory is still in flight: on the
    // normal path the consumers have waited on every chunk; after an abort wait here.
    if (lane != 0) return;
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

__device__ __forceinline__ uint32_t tag_of(uint64_t w) { return static_cast<uint32_t>(w >> 32); }
__device__ __forceinline__ float val_of(uint64_t w) { return __uint_as_float(static_cast<uint32_t>(w)); }

// Fetches exchange words carrying `tag` into dst. The words are rows of `len` words (len
// even): `cols` column blocks (block c at src + c * csrc, its rows at dst + c * cdst), each
// with na rows at offa + r * stra and then nb rows at offb + r * strb (source offsets, even),
// written as consecutive rows of ldst floats. Thread t takes the word pairs 2t + 2*NCT*k of
// the packed order (block, row, word), issues up to 6 pair loads at once, then re-issues
// every stale pair together until all carry the tag: one L2 round trip per poll for all of
// a phase's inputs. Returns this thread's success (the caller decides with a barrier).
// ll_each() visits the same packed elements in the same thread, so a transform needs no
// barrier in between.
template <int MAXK = 4>
__device__ __noinline__ bool ll_fetch_plan(const uint64_t * src, int cols, int csrc, int cdst, int na, int offa, int stra, int nb, int offb,
                                           int strb, int len, int ldst, uint32_t tag, float * dst, const Args & A, Ctrl * ctrl, int phase) {
    const int rpc = na + nb, n = cols * rpc * len;
    for (int base = 2 * threadIdx.x; base < n; base += 2 * NCT * MAXK) {
        uint64_t w[MAXK][2];
        uint32_t at[MAXK], to[MAXK];
        unsigned pend = 0;
#pragma unroll
        for (int k = 0; k < MAXK; ++k) {
            const int i = base + 2 * NCT * k;
            at[k] = to[k] = 0;
            if (i < n) {
                const int R = i / len, e = i - R * len, c = R / rpc, rr = R - c * rpc;
                at[k] = static_cast<uint32_t>(c * csrc + (rr < na ? offa + rr * stra : offb + (rr - na) * strb) + e);
                to[k] = static_cast<uint32_t>(c * cdst + rr * ldst + e);
                ll_load2(src + at[k], w[k][0], w[k][1]);
                pend |= 1u << k;
            }
        }
        uint64_t t0 = 0;
        uint32_t spins = 0;
        for (;;) {
#pragma unroll
            for (int k = 0; k < MAXK; ++k) {
                if (((pend >> k) & 1u) && tag_of(w[k][0]) == tag && tag_of(w[k][1]) == tag) {
                    dst[to[k]] = val_of(w[k][0]);
                    dst[to[k] + 1] = val_of(w[k][1]);
                    pend &= ~(1u << k);
                }
            }
            if (!pend) break;
            if (t0 == 0) t0 = globaltimer();
            if (A.poll_ns) __nanosleep(A.poll_ns);
#pragma unroll
            for (int k = 0; k < MAXK; ++k)
                if ((pend >> k) & 1u) ll_load2(src + at[k], w[k][0], w[k][1]);
            ++spins;
            if ((spins & 3u) == 0 && globaltimer() - t0 > A.timeout_ns) { raise_abort(A, phase); return false; }
            if ((spins & 31u) == 0 && (ctrl->abort || launch_aborted(A))) return false;
        }
    }
    return true;
}

// Exchange words [0, n) (n even) into dst[0, n): ll_fetch_plan's single-run case without
// its index arithmetic (the common case: one input vector per phase), up to 6 pair loads per
// thread at once, so a 3,072-word vector (the down projections' input) takes one round.
__device__ __noinline__ bool ll_fetch(const uint64_t * src, int n, uint32_t tag, float * dst, const Args & A, Ctrl * ctrl, int phase) {
    constexpr int MAXK = 6;
    for (int base = 2 * threadIdx.x; base < n; base += 2 * NCT * MAXK) {
        uint64_t w[MAXK][2];
        unsigned pend = 0;
#pragma unroll
        for (int k = 0; k < MAXK; ++k) {
            const int i = base + 2 * NCT * k;
            if (i < n) {
                ll_load2(src + i, w[k][0], w[k][1]);
                pend |= 1u << k;
            }
        }
        uint64_t t0 = 0;
        uint32_t spins = 0;
        for (;;) {
#pragma unroll
            for (int k = 0; k < MAXK; ++k) {
                if (((pend >> k) & 1u) && tag_of(w[k][0]) == tag && tag_of(w[k][1]) == tag) {
                    const int i = base + 2 * NCT * k;
                    dst[i] = val_of(w[k][0]);
                    dst[i + 1] = val_of(w[k][1]);
                    pend &= ~(1u << k);
                }
            }
            if (!pend) break;
            if (t0 == 0) t0 = globaltimer();
            if (A.poll_ns) __nanosleep(A.poll_ns);
#pragma unroll
            for (int k = 0; k < MAXK; ++k)
                if ((pend >> k) & 1u) ll_load2(src + base + 2 * NCT * k, w[k][0], w[k][1]);
            ++spins;
            if ((spins & 3u) == 0 && globaltimer() - t0 > A.timeout_ns) { raise_abort(A, phase); return false; }
            if ((spins & 31u) == 0 && (ctrl->abort || launch_aborted(A))) return false;
        }
    }
    return true;
}

// `cols` runs of len words at src + c * len into dst + c * dstride (one column: ll_fetch).
template <bool WIDE = false>
__device__ __forceinline__ bool ll_fetch_cols(const uint64_t * src, int cols, int len, float * dst, int dstride, uint32_t tag, const Args & A,
                                              Ctrl * ctrl, int phase) {
    if (cols == 1) return ll_fetch(src, len, tag, dst, A, ctrl, phase);
    return ll_fetch_plan<WIDE ? 6 : 4>(src, cols, len, dstride, 1, 0, 0, 0, 0, 0, len, len, tag, dst, A, ctrl, phase);
}

// One exchange word into v once it carries `tag` (a polling thread of its own; the caller
// decides with a barrier).
__device__ __noinline__ bool ll_poll1(const uint64_t * src, uint32_t tag, float & v, const Args & A, Ctrl * ctrl, int phase) {
    uint64_t t0 = 0;
    for (uint32_t spins = 0;; ++spins) {
        const uint64_t w = ll_load1(src);
        if (tag_of(w) == tag) {
            v = val_of(w);
            return true;
        }
        if (t0 == 0) t0 = globaltimer();
        if ((spins & 3u) == 3u && globaltimer() - t0 > A.timeout_ns) { raise_abort(A, phase); return false; }
        if ((spins & 31u) == 31u && (ctrl->abort || launch_aborted(A))) return false;
    }
}

// Visits the packed indices i < n that ll_fetch_plan gave this thread.
template <class F>
__device__ __forceinline__ void ll_each(int n, F && fn) {
    for (int i = 2 * threadIdx.x; i < n; i += 2 * NCT) {
        fn(i);
        fn(i + 1);
    }
}

// Per-thread wait for ring chunk `chunk` (no barrier).
__device__ __forceinline__ bool wait_chunk_local(const Args & A, Sm & S, int chunk, int phase) {
    const int slot = chunk % NSLOT;
    const uint32_t parity = static_cast<uint32_t>((chunk / NSLOT) & 1);
    if (mbar_try_wait(&S.bars[slot], parity)) return true;
    const uint64_t t0 = globaltimer();
    uint32_t spins = 0;
    while (!mbar_try_wait(&S.bars[slot], parity)) {
        if ((++spins & 15u) == 0) {
            if (S.ctrl->abort || launch_aborted(A)) return false;
            if (globaltimer() - t0 > A.timeout_ns) { raise_abort(A, phase); return false; }
        }
    }
    return true;
}

// Dot products of the rows of a CTA slice ([K/8][nr][8] f16 in shared memory, see
// frame_kernel.cuh) with NC input columns xin (f32, stride xstride). PAIR: the slice is
// followed by a second one of the same shape (gate, then up) and unit u is the row pair.
// Lane (row, j) with row = lane % R2, j = lane / R2 (R2 = 32 / J rows per round, both powers
// of two, so the lane split is shifts and masks: the GPU has no integer divider and a runtime
// division costs tens of instructions) takes 8-column chunks of its warp's K range,
// j-interleaved, so the live lanes of a warp read consecutive 16-byte words; x chunks are
// broadcasts. Products accumulate on the packed fp32 pipe (dot8h2: even and odd products in
// two chains, 12-18 % faster than scalar FMAs with 2 or 4 columns, the same with one; every
// column is summed the same way whatever NC, so batched and single-stream frames agree).
// Per-warp sums are folded over j with shuffles, written to
// part[warp][value][row], and after a consumer barrier thread (value, row) adds the NCW warp
// sums in warp order into ys[(column * 2 + value) * nr + row] (gemv_owned's mapping).
template <int NC, bool PAIR>
__device__ __forceinline__ void gemv_slice(const Sm & S, int chunk, uint32_t woff, int nr, int K, const float * xin, int xstride, float * part,
                                           float * ys) {
    constexpr int NV = NC * (PAIR ? 2 : 1);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nk = K >> 3;
    // J lanes per row: the largest power of two with 2 * J * nr > 32 >= J * nr, i.e. at
    // least half of the lanes live; R2 = 32 / J row slots per round
    int lj = 0;
    while (lj < 5 && (2 << lj) * nr <= 32) ++lj;
    const int J = 1 << lj, lr = 5 - lj, R2 = 1 << lr;
    const int k0 = (nk * warp) / NCW, k1 = (nk * (warp + 1)) / NCW;   // NCW is a constant: no division
    const size_t cs = static_cast<size_t>(J) * nr * 8;                 // halves between a lane's chunks
    const int j = lane >> lr;
    // this warp's K range of the slice (and of the up slice after it), each contiguous in the ring
    const uint32_t kb = static_cast<uint32_t>(nr) * 16u;
    const __half * wa = reinterpret_cast<const __half *>(chunk_at(S, chunk, woff + static_cast<uint32_t>(k0) * kb));
    const __half * wb = PAIR ? reinterpret_cast<const __half *>(chunk_at(S, chunk, woff + static_cast<uint32_t>(nk + k0) * kb)) : wa;
    // rows beyond 32 lanes (small grids) are taken in rounds of R2. Every loop stays rolled:
    // this code runs with a cold instruction cache in every phase (the phases in between
    // evict it), and an unrolled body costs more in instruction fetch than it saves in
    // issue (measured 1,300-2,600 fewer cycles per call cold than a 4-way unrolled body).
#pragma unroll 1
    for (int rb = 0; rb < nr; rb += R2) {
        const int row = rb + (lane & (R2 - 1));
        const bool live = row < nr;
        float2 acc2[NV];   // even / odd products of each value, on the packed fp32 pipe
#pragma unroll
        for (int v = 0; v < NV; ++v) acc2[v] = make_float2(0.f, 0.f);
        if (live) {
            // this lane's chunks: k0 + j, k0 + j + J, ... < k1
            const __half * pw = wa + (static_cast<size_t>(j) * nr + row) * 8;
            const __half * pu = wb + (static_cast<size_t>(j) * nr + row) * 8;
            const float * px = xin + (k0 + j) * 8;
            const int cnt = (k0 + j < k1) ? (k1 - (k0 + j) + J - 1) >> lj : 0;
#pragma unroll 1
            for (int i = 0; i < cnt; ++i) {
                const uint4 ga = *reinterpret_cast<const uint4 *>(pw);
                uint4 gb = make_uint4(0, 0, 0, 0);
                if constexpr (PAIR) gb = *reinterpret_cast<const uint4 *>(pu);
#pragma unroll
                for (int c = 0; c < NC; ++c) {
                    const float4 xa = *reinterpret_cast<const float4 *>(px + c * xstride);
                    const float4 xb = *reinterpret_cast<const float4 *>(px + c * xstride + 4);
                    acc2[c * (PAIR ? 2 : 1)] = dot8h2(ga, xa, xb, acc2[c * (PAIR ? 2 : 1)]);
                    if constexpr (PAIR) acc2[c * 2 + 1] = dot8h2(gb, xa, xb, acc2[c * 2 + 1]);
                }
                pw += cs;
                pu += cs;
                px += J * 8;
            }
        }
        float acc[NV];
#pragma unroll
        for (int v = 0; v < NV; ++v) acc[v] = acc2[v].x + acc2[v].y;
        // fold the J lanes of each row (lanes row, row + R2, ...); dead lanes hold zeros
#pragma unroll 1
        for (int s = 16; s >= R2; s >>= 1)
#pragma unroll
            for (int v = 0; v < NV; ++v) acc[v] += __shfl_down_sync(0xffffffffu, acc[v], s);
        if (live && j == 0)
#pragma unroll
            for (int v = 0; v < NV; ++v) part[(warp * NV + v) * nr + row] = acc[v];
    }
    named_sync(BID, NCT);
    // column c is summed by the threads [c * TPC, (c + 1) * TPC), TPC a constant
    constexpr int TPC = NCT / NC;
    const int c = threadIdx.x / TPC;
    if (c < NC)
        for (int row = threadIdx.x - c * TPC; row < nr; row += TPC) {
            float y = 0.f, y2 = 0.f;
#pragma unroll
            for (int w = 0; w < NCW; ++w) {
                y += part[(w * NV + c * (PAIR ? 2 : 1)) * nr + row];
                if constexpr (PAIR) y2 += part[(w * NV + c * 2 + 1) * nr + row];
            }
            ys[2 * c * nr + row] = y;
            if constexpr (PAIR) ys[(2 * c + 1) * nr + row] = y2;
        }
}

// gemv_slice for nc input columns (2 or 4 in batched programs, 1 or 2 otherwise). The phase
// loop has one call site per shape (plain or gate/up pair), shared by every phase that streams
// a matrix; the phases differ only in the epilogue each applies to the sums afterwards
// (gemv_owned). So consecutive phases run the same GEMV instructions, which are then still in
// the SM's instruction cache, instead of each phase fetching its own copy.
template <bool PAIR, bool BATCHED>
__device__ __forceinline__ void gemv_sums(int nc, const Sm & S, int chunk, uint32_t woff, int nr, int K, const float * xin, int xstride,
                                          float * part, float * ys) {
    if constexpr (BATCHED) {
        if (nc == 4) gemv_slice<4, PAIR>(S, chunk, woff, nr, K, xin, xstride, part, ys);
        else gemv_slice<2, PAIR>(S, chunk, woff, nr, K, xin, xstride, part, ys);
    } else {
        if (nc == 2) gemv_slice<2, PAIR>(S, chunk, woff, nr, K, xin, xstride, part, ys);
        else gemv_slice<1, PAIR>(S, chunk, woff, nr, K, xin, xstride, part, ys);
    }
}

// The (row, column) sums of gemv_sums that this thread wrote (column c is owned by the threads
// [c * TPC, (c + 1) * TPC), TPC = NCT / nc), so its epilogue reads them without a barrier.
template <class F>
__device__ __forceinline__ void gemv_owned(int nc, int nr, F && f) {
    const int TPC = nc == 1 ? NCT : nc == 2 ? NCT / 2 : NCT / 4;
    const int tid = threadIdx.x;
    const int c = (tid >= TPC) + (tid >= 2 * TPC) + (tid >= 3 * TPC);
    if (c < nc)
        for (int row = tid - c * TPC; row < nr; row += TPC) f(row, c);
}

// Sums of squares of this thread's part of columns 0..ncol-1, folded per warp into the CTA
// scratch; the totals are read after the next consumer barrier (norm_scale).
__device__ __forceinline__ void norm_partial(Sm & S, const float (&ss)[MAXC], int ncol) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
    for (int c = 0; c < MAXC; ++c) {
        if (c >= ncol) break;
        const float t = warp_sum(ss[c]);
        if (lane == 0) S.ctrl->red[c][wid] = t;
    }
}
__device__ __forceinline__ float norm_scale(Sm & S, int c, int n, float eps) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < NCW; ++k) t += S.ctrl->red[c][k];
    return rsqrtf(t / static_cast<float>(n) + eps);
}

__device__ __forceinline__ void row_f16_to_smem(const __half * row, int n, float * dst) {
    for (int i = threadIdx.x; i < n; i += NCT) dst[i] = __half2float(row[i]);
}

__device__ SampleScratch sampler_scratch(Sm & S, int Vmax) { return sampler_layout(S.scratch, Vmax); }

// The draw of codebook `codebook` for stream s of the launch.
__device__ SampleCfg sample_cfg(const Args & A, int codebook, int s) {
    SampleCfg c{};
    if (codebook == 0) {
        c.temperature = A.temp; c.top_k = A.top_k; c.top_p = A.top_p;
        c.talker_mods = 1;
        c.suppress_from = A.suppress_from; c.eos_id = A.eos_id; c.min_frames = A.min_frames;
        c.repetition_penalty = A.rep;
        c.seen = A.seen[s];
    } else {
        c.temperature = A.cp_temp; c.top_k = A.cp_top_k; c.top_p = A.cp_top_p;
        c.talker_mods = 0;
    }
    c.rng = A.rng; c.seed = A.seed[s]; c.frame_index = A.frame_index[s]; c.codebook = codebook;
    c.pcg_seed = A.pcg_seed[s][codebook];
    return c;
}

// Trace stamp k (0..3) of phase p on the traced CTA: 0 inputs ready, 1 weights ready,
// 2 dot products done, 3 phase end (attention: 0 gathered, 1 normed, 2 attended, 3 combined).
__device__ __forceinline__ unsigned long long * prof_base(const Args & A) {
    if (!A.prof || threadIdx.x != 0) return nullptr;
    if (A.prof_cta < 0) return A.prof + static_cast<size_t>(blockIdx.x) * PROF_STRIDE;
    return blockIdx.x == A.prof_cta ? A.prof : nullptr;
}
__device__ __forceinline__ void stamp(const Args & A, int p, int k) {
    if (unsigned long long * pb = prof_base(A)) pb[4 * p + k] = globaltimer();
}

// ---- attention -------------------------------------------------------------------------------------

// Per-head RMSNorm + rotate-half RoPE of a head vector in shared memory, by one warp
// (frame.hip:312-346: norm before RoPE, pairs (i, i + hd/2)). cs holds this position's
// cos[hd/2] then sin[hd/2] (host-computed: f32 angle pos * inv_freq, cos/sin in double,
// rounded to f32). round16: store the result rounded to f16 (K, as the cache holds it).
__device__ __forceinline__ void warp_norm_rope(float * vec, const float * nw, const float * cs, int HD, float eps, bool round16) {
    const int lane = threadIdx.x & 31, EPL = HD / 32, H2 = HD / 2;
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
    for (int t = 0; t < 4; ++t) if (t < EPL) e[t] = e[t] * scale * nw[lane + 32 * t];
#pragma unroll
    for (int t = 0; t < 2; ++t) {
        if (t >= EPL / 2) continue;
        const int i = lane + 32 * t;
        const float c = cs[i], sn = cs[H2 + i];
        const float x0 = e[t], x1 = (EPL == 4) ? e[t + 2] : e[t + 1];
        float r0 = x0 * c - x1 * sn, r1 = x0 * sn + x1 * c;
        if (round16) { r0 = f16_round(r0); r1 = f16_round(r1); }
        vec[i] = r0;
        vec[i + H2] = r1;
    }
}

// Scaled scores q_j . K_t for the GR query heads j of `ngroups` groups (a KV head, or a
// code-predictor column) and positions t < n. Lane groups of LPI = HD/8 lanes take one
// (group, position) at a time, each lane 8 dims (one 16-byte K load); group g = stream %
// ngroups keeps its queries in registers and walks positions t0, t0 + per, ... four at a
// time, so the shuffle reductions of 4 x GR dots overlap. krow(g, t): K row (f16, HD);
// qbase(g): query of head j at + j * HD (f32); sc_at(g, t): score of head j at + j * jstride.
// Requires ngroups <= NCW * 32 / LPI. Every lane of a warp runs the same rounds.
template <class KRow, class QBase, class ScAt>
__device__ __forceinline__ void attn_scores(int ngroups, int n, int GR, int HD, float scale, int jstride, KRow && krow, QBase && qbase,
                                            ScAt && sc_at) {
    constexpr int B = 4;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int LPI = HD / 8, IPW = 32 / LPI, sub = lane / LPI, sl = lane % LPI;
    const int per = (NCW * IPW) / ngroups;
    const int hw = warp * IPW + sub, g = hw % ngroups, t0 = hw / ngroups;
    const bool live = hw < per * ngroups;
    float q[MAX_GROUP][8];
    const float * qb = qbase(g);
#pragma unroll
    for (int j = 0; j < MAX_GROUP; ++j) {
        if (j < GR && live) {
            const float4 a = *reinterpret_cast<const float4 *>(qb + j * HD + sl * 8);
            const float4 c = *reinterpret_cast<const float4 *>(qb + j * HD + sl * 8 + 4);
            q[j][0] = a.x; q[j][1] = a.y; q[j][2] = a.z; q[j][3] = a.w;
            q[j][4] = c.x; q[j][5] = c.y; q[j][6] = c.z; q[j][7] = c.w;
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) q[j][i] = 0.f;
        }
    }
    for (int k = 0; k * per < n; k += B) {
        float dots[B][MAX_GROUP];
#pragma unroll
        for (int bb = 0; bb < B; ++bb) {
            const int t = t0 + (k + bb) * per;
            float kf[8];
            if (live && t < n) {
                const uint4 kw = *reinterpret_cast<const uint4 *>(krow(g, t) + sl * 8);
                const float2 f0 = __half22float2(*reinterpret_cast<const __half2 *>(&kw.x));
                const float2 f1 = __half22float2(*reinterpret_cast<const __half2 *>(&kw.y));
                const float2 f2 = __half22float2(*reinterpret_cast<const __half2 *>(&kw.z));
                const float2 f3 = __half22float2(*reinterpret_cast<const __half2 *>(&kw.w));
                kf[0] = f0.x; kf[1] = f0.y; kf[2] = f1.x; kf[3] = f1.y; kf[4] = f2.x; kf[5] = f2.y; kf[6] = f3.x; kf[7] = f3.y;
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) kf[i] = 0.f;
            }
#pragma unroll
            for (int j = 0; j < MAX_GROUP; ++j) {
                float a = 0.f;
                if (j < GR)
#pragma unroll
                    for (int i = 0; i < 8; ++i) a = fmaf(q[j][i], kf[i], a);
                dots[bb][j] = a;
            }
        }
        for (int o = LPI / 2; o > 0; o >>= 1)
#pragma unroll
            for (int bb = 0; bb < B; ++bb)
#pragma unroll
                for (int j = 0; j < MAX_GROUP; ++j)
                    if (j < GR) dots[bb][j] += __shfl_xor_sync(0xffffffffu, dots[bb][j], o);
        if (sl == 0 && live) {
#pragma unroll
            for (int bb = 0; bb < B; ++bb) {
                const int t = t0 + (k + bb) * per;
                if (t < n) {
                    float * dst = sc_at(g, t);
#pragma unroll
                    for (int j = 0; j < MAX_GROUP; ++j) if (j < GR) dst[j * jstride] = dots[bb][j] * scale;
                }
            }
        }
    }
}

// Softmax rows: row r (< nrows) holds n_of(r) scores at sc + r * stride; they are replaced by
// e^(s - m), and ml[2r], ml[2r+1] get m and l = sum e^(s - m). One warp per row.
template <class NOf>
__device__ __forceinline__ void attn_softmax(float * sc, int stride, int nrows, NOf && n_of, float * ml) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int r = warp; r < nrows; r += NCW) {
        const int n = n_of(r);
        float * row = sc + r * stride;
        float m = -INFINITY;
        for (int t = lane; t < n; t += 32) m = fmaxf(m, row[t]);
        m = warp_max(m);
        float l = 0.f;
        for (int t = lane; t < n; t += 32) {
            const float e = expf(row[t] - m);
            row[t] = e;
            l += e;
        }
        l = warp_sum(l);
        if (lane == 0) { ml[2 * r] = m; ml[2 * r + 1] = l; }
    }
}

// sum over positions of p_j[t] * V_t for the GR heads j of each of `ngroups` groups: warp w
// takes group w % ngroups and the positions t = w / ngroups + k * (NCW / ngroups), lane e4
// dims [4 e4, 4 e4 + 4) (HD == 128) -- so a warp reads one contiguous V row slice per step.
// The per-warp sums go to pv[w][j][HD]; after a barrier, emit(g, j, e, sum) gets the total
// of every (g, j < GR, e < HD), summed over the warps of g in warp order. ngroups divides NCW.
template <class NOf, class PAt, class VRow, class Emit>
__device__ __forceinline__ void attn_pv(int ngroups, int GR, int HD, NOf && n_of, PAt && p_at, VRow && vrow, float * pv, Emit && emit) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int WPG = NCW / ngroups, g = warp % ngroups, tq = warp / ngroups, E4 = HD / 4;
    const int n = n_of(g);
    float acc[MAX_GROUP][4];
#pragma unroll
    for (int j = 0; j < MAX_GROUP; ++j)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[j][i] = 0.f;
    if (lane < E4) {
        for (int t = tq; t < n; t += WPG) {
            const uint2 vw = *reinterpret_cast<const uint2 *>(vrow(g, t) + lane * 4);
            const float2 v01 = __half22float2(*reinterpret_cast<const __half2 *>(&vw.x));
            const float2 v23 = __half22float2(*reinterpret_cast<const __half2 *>(&vw.y));
#pragma unroll
            for (int j = 0; j < MAX_GROUP; ++j) {
                if (j >= GR) continue;
                const float pt = p_at(g, j)[t];
                acc[j][0] = fmaf(pt, v01.x, acc[j][0]);
                acc[j][1] = fmaf(pt, v01.y, acc[j][1]);
                acc[j][2] = fmaf(pt, v23.x, acc[j][2]);
                acc[j][3] = fmaf(pt, v23.y, acc[j][3]);
            }
        }
#pragma unroll
        for (int j = 0; j < MAX_GROUP; ++j)
            if (j < GR) *reinterpret_cast<float4 *>(pv + (warp * MAX_GROUP + j) * HD + lane * 4) = make_float4(acc[j][0], acc[j][1], acc[j][2], acc[j][3]);
    }
    named_sync(BID, NCT);
    for (int u = threadIdx.x; u < ngroups * GR * HD; u += NCT) {
        const int e = u % HD, gj = u / HD, gg = gj / GR, j = gj - gg * GR;
        float sum = 0.f;
        for (int w = gg; w < NCW; w += ngroups) sum += pv[(w * MAX_GROUP + j) * HD + e];
        emit(gg, j, e, sum);
    }
}

// Talker attention at position n_past (frame.hip:350-385) of every stream of the launch,
// split over (stream, KV head) groups and cached positions: CTA b in group (s, g) with split
// sp < attn_split[s] (talker_attn_role) takes positions [sp * chunk, (sp + 1) * chunk) of
// stream s, streamed into its ring chunk as KV head g's 256-byte K and V row slices; the last
// split also takes the new position (and writes its K/V row of head g). Scores, softmax and P.V
// run as CTA-wide passes over the GR query heads of g. Partials (m, l, acc) go to the
// exchange words; CTA G - nb * NH + (s * NH + h) combines head h of stream s in split order.
// A single split writes the output directly.
template <bool BATCHED>
__device__ __forceinline__ bool talker_attention(const Args & A, Sm & S, const Phase & ph, int chunk, uint32_t tag, uint32_t ptag, int p) {
    const Dims & d = A.d;
    constexpr int HD = KHD, GR = KGR;
    const int NH = d.NH, tid = threadIdx.x;
    const int G = gridDim.x, b = blockIdx.x;
    const float scale = rsqrtf(static_cast<float>(HD));
    const uint32_t WST = HD + 2;
    int st, g, sp;
    const bool has = talker_attn_role(A, b, st, g, sp);
    if constexpr (!BATCHED) st = 0;
    if (has) {
        const int Sp = A.attn_split[st], pos = A.n_past[st], ch = A.attn_chunk[st];
        const int NPS = ch + 1;                            // score slots per head
        float * qs = S.scratch;                            // [GR][HD]
        float * ks = qs + GR * HD;                         // [HD] new position
        float * vs = ks + HD;                              // [HD]
        __half * kh = reinterpret_cast<__half *>(vs + HD); // new K/V row slice as f16 [2][HD]
        float * ml = vs + 2 * HD;                          // [GR][2]
        float * pv = ml + 2 * MAX_GROUP;                   // [NCW][MAX_GROUP][HD]
        float * sc = pv + NCW * MAX_GROUP * HD;            // [GR][NPS] scores, then e^(s - m)
        // chunk segments: q norm, k norm, K rows, V rows (the chunk is only ever cut between them)
        const int r0 = min(sp * ch, pos), r1 = min(r0 + ch, pos);
        const int nc = r1 - r0;
        const float * qn = reinterpret_cast<const float *>(chunk_at(S, chunk, 0));
        const float * kn = reinterpret_cast<const float *>(chunk_at(S, chunk, HD * 4));
        const __half * Kc = reinterpret_cast<const __half *>(chunk_at(S, chunk, 2 * HD * 4));
        // V follows K: nc rows, or whole boxes of KV_BOX rows when the rows came by tensor map
        const int krows = A.kvmap[st] ? (nc + KV_BOX - 1) / KV_BOX * KV_BOX : nc;
        const __half * Vc = reinterpret_cast<const __half *>(chunk_at(S, chunk, 2 * HD * 4 + krows * HD * 2));
        const bool last = sp == Sp - 1;
        const int n = nc + (last ? 1 : 0);
        // rows of HD words: the group's q heads, then (last split) k and v of head g, of column st
        const uint64_t * qkv = A.w.qkv + static_cast<size_t>(st) * d.QKV;
        const bool ok = ll_fetch_plan(qkv, 1, 0, 0, GR, g * GR * HD, HD, last ? 2 : 0, d.Q + g * HD, d.KV, HD, HD, ptag, qs, A, S.ctrl, p);
        if (!consumers_ok(S, ok)) return false;
        stamp(A, p, 0);
        const int warp = tid >> 5;
        if (warp < GR + (last ? 1 : 0))
            warp_norm_rope(warp < GR ? qs + warp * HD : ks, warp < GR ? qn : kn, A.rope_t[st], HD, d.eps_t, warp >= GR);
        named_sync(BID, NCT);
        if (last) {
            for (int i = tid; i < HD; i += NCT) {
                const __half kq = __float2half_rn(ks[i]), vq = __float2half_rn(vs[i]);
                kh[i] = kq;
                kh[HD + i] = vq;
                A.kc[st][ph.layer][static_cast<size_t>(pos) * d.KV + g * HD + i] = kq;
                A.vc[st][ph.layer][static_cast<size_t>(pos) * d.KV + g * HD + i] = vq;
            }
            named_sync(BID, NCT);
        }
        stamp(A, p, 1);
        attn_scores(1, n, GR, HD, scale, NPS, [&](int, int t) { return t < nc ? Kc + static_cast<size_t>(t) * HD : kh; },
                    [&](int) { return static_cast<const float *>(qs); }, [&](int, int t) { return sc + t; });
        named_sync(BID, NCT);
        attn_softmax(sc, NPS, GR, [&](int) { return n; }, ml);
        named_sync(BID, NCT);
        attn_pv(1, GR, HD, [&](int) { return n; }, [&](int, int j) { return static_cast<const float *>(sc + j * NPS); },
                [&](int, int t) { return t < nc ? Vc + static_cast<size_t>(t) * HD : kh + HD; }, pv,
                [&](int, int j, int e, float sum) {
                    const int h = g * GR + j;
                    if (Sp == 1) {
                        ll_store(A.w.attn + static_cast<size_t>(st) * d.Q + h * HD + e, sum / ml[2 * j + 1], tag);
                    } else {
                        uint64_t * pp = A.w.part + (static_cast<size_t>(st * NH + h) * A.attn_per + sp) * WST;
                        ll_store(pp + 2 + e, sum, tag);
                        if (e == 0) { ll_store(pp, ml[2 * j], tag); ll_store(pp + 1, ml[2 * j + 1], tag); }
                    }
                });
        stamp(A, p, 2);
    }
    // combine: CTA G - nb * NH + (s * NH + h) reduces head h of stream s over its splits, in split order
    const int ch_ = b - (G - (BATCHED ? A.nb : 1) * NH);
    if (ch_ >= 0) {
        const int cs = BATCHED ? ch_ / NH : 0, h = ch_ - cs * NH, Sp = A.attn_split[cs];
        if (Sp > 1) {
            named_sync(BID, NCT);                   // this CTA's own split (if any) is done with its scratch
            float * pb = S.scratch;                 // [Sp][WST]: m, l, acc[HD] of every split
            const bool ok = ll_fetch_plan(A.w.part + static_cast<size_t>(cs * NH + h) * A.attn_per * WST, Sp, WST, WST, 1, 0, 0, 0, 0, 0,
                                          WST, WST, tag, pb, A, S.ctrl, p);
            if (!consumers_ok(S, ok)) return false;
            if (tid < HD) {
                float M = -INFINITY;
                for (int k = 0; k < Sp; ++k) M = fmaxf(M, pb[k * WST]);
                float L = 0.f, num = 0.f;
                for (int k = 0; k < Sp; ++k) {
                    const float wk = expf(pb[k * WST] - M);
                    L += pb[k * WST + 1] * wk;
                    num += pb[k * WST + 2 + tid] * wk;
                }
                ll_store(A.w.attn + static_cast<size_t>(cs) * d.Q + h * HD + tid, num / L, tag);
            }
            named_sync(BID, NCT);
        }
    }
    return true;
}

// Code-predictor attention (frame.hip:555-575: its own KV, positions 0..15, reset every
// frame). Single stream: positions pos..pos+ncol-1 (the pass over positions 0 and 1 has two
// columns). Batched: position pos of every stream, column c = stream c. The CTA of set
// (layer, stream, KV head g) (cp_attn_role) keeps that K/V in shared memory slot across the
// frame's positions.
template <bool BATCHED>
__device__ __forceinline__ bool cp_attention(const Args & A, Sm & S, const Phase & ph, int chunk, uint32_t tag, uint32_t ptag, int p) {
    const Dims & d = A.d;
    constexpr int HD = KHD, GR = KGR;
    const int tid = threadIdx.x;
    int st, g, slot;
    if (!cp_attn_role(A, blockIdx.x, ph.layer, st, g, slot)) return true;
    constexpr bool batched = BATCHED;
    const int ncol = batched ? 1 : ph.ncol, pos = ph.pos, col0 = batched ? st : 0;
    const float * qn = reinterpret_cast<const float *>(chunk_at(S, chunk, 0));
    const float * kn = reinterpret_cast<const float *>(chunk_at(S, chunk, HD * 4));
    const float * rc = reinterpret_cast<const float *>(chunk_at(S, chunk, 2 * HD * 4));   // RoPE rows of the columns
    __half * kv = S.cpkv + static_cast<size_t>(slot) * (cpkv_bytes(d) / 2);   // [pos][K,V][HD] of the set
    float * qkv = S.scratch;                // [2][GR + 2][HD]: per column the q heads, k, v
    const auto qof = [&](int c) { return qkv + c * (GR + 2) * HD; };
    const auto kof = [&](int c) { return qkv + (c * (GR + 2) + GR) * HD; };
    const auto vof = [&](int c) { return qkv + (c * (GR + 2) + GR + 1) * HD; };
    // per column: the group's q heads, then k and v of head g (rows of HD words)
    const bool ok = ll_fetch_plan(A.w.qkv + static_cast<size_t>(col0) * d.QKV, ncol, d.QKV, (GR + 2) * HD, GR, g * GR * HD, HD, 2,
                                  d.Q + g * HD, d.KV, HD, HD, ptag, qkv, A, S.ctrl, p);
    if (!consumers_ok(S, ok)) return false;
    stamp(A, p, 0);
    // norm + RoPE of the q heads and k, one warp per vector; the warp of column c's k also
    // writes k (f16, after RoPE) and v into the group's cache rows
    const int lane = tid & 31;
    for (int v = tid >> 5; v < ncol * (GR + 1); v += NCW) {
        const int c = v / (GR + 1), j = v - c * (GR + 1);
        warp_norm_rope(j < GR ? qof(c) + j * HD : kof(c), j < GR ? qn : kn, rc + c * HD, HD, d.eps_c, j == GR);
        if (j == GR) {
            __syncwarp();
            for (int e = lane; e < HD; e += 32) {
                kv[(static_cast<size_t>(pos + c) * 2 + 0) * HD + e] = __float2half_rn(kof(c)[e]);
                kv[(static_cast<size_t>(pos + c) * 2 + 1) * HD + e] = __float2half_rn(vof(c)[e]);
            }
        }
    }
    named_sync(BID, NCT);
    stamp(A, p, 1);
    // one warp per (column c, query head j) attends over positions 0..pos+c (<= NCB) with no
    // CTA barrier: lanes t and t + 16 take the two halves of position t's dot product
    // (16-byte loads rotated by t, so the 16 rows do not hit one bank), softmax in 16-lane
    // halves by shuffles, then lane l sums dims 4l..4l+3 of P.V.
    const int w = tid >> 5;
    if (w < ncol * GR) {
        const int c = w / GR, j = w - c * GR;
        const int n = pos + c + 1;
        const float * q = qof(c) + j * HD;
        const int t = lane & 15, hh = lane >> 4;
        float dot = 0.f;
        if (t < n) {
            const __half * kr = kv + static_cast<size_t>(t) * 2 * HD + hh * (HD / 2);
            const float * qh = q + hh * (HD / 2);
#pragma unroll
            for (int i = 0; i < HD / 2; i += 8) {
                const int o = (i + 8 * t) & (HD / 2 - 1);
                const uint4 kk = *reinterpret_cast<const uint4 *>(kr + o);
                const float4 qa = *reinterpret_cast<const float4 *>(qh + o), qb = *reinterpret_cast<const float4 *>(qh + o + 4);
                dot += dot8h(kk, qa, qb);
            }
        }
        dot += __shfl_xor_sync(0xffffffffu, dot, 16);
        const float sc = t < n ? dot * rsqrtf(static_cast<float>(HD)) : -INFINITY;
        float m = sc;
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        const float ev = t < n ? expf(sc - m) : 0.f;
        float z = ev;
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
        for (int tt = 0; tt < n; ++tt) {
            const float pt = __shfl_sync(0xffffffffu, ev, tt);
            const uint2 vv = *reinterpret_cast<const uint2 *>(kv + (static_cast<size_t>(tt) * 2 + 1) * HD + lane * 4);
            const float2 v01 = __half22float2(*reinterpret_cast<const __half2 *>(&vv.x));
            const float2 v23 = __half22float2(*reinterpret_cast<const __half2 *>(&vv.y));
            acc[0] = fmaf(pt, v01.x, acc[0]);
            acc[1] = fmaf(pt, v01.y, acc[1]);
            acc[2] = fmaf(pt, v23.x, acc[2]);
            acc[3] = fmaf(pt, v23.y, acc[3]);
        }
        const float inv = 1.f / z;
#pragma unroll
        for (int e = 0; e < 4; ++e)
            ll_store(A.w.attn + static_cast<size_t>(col0 + c) * d.Q + (g * GR + j) * HD + lane * 4 + e, acc[e] * inv, tag);
    }
    stamp(A, p, 2);
    named_sync(BID, NCT);
    return true;
}

// ---- the consumer: the phase program ----------------------------------------------------------------

// The phase program, compiled twice: for the single-stream programs (BATCHED false: at most
// two input columns) and for the batched ones (2 or 4 streams), so that each runs only the
// code of its own shape (the phases run with a cold instruction cache).
template <bool BATCHED>
__device__ void consumer(const Args & A, Sm & S) {
    const Dims & d = A.d;
    const ModelW & W = *A.mw;
    const int G = gridDim.x, b = blockIdx.x, tid = threadIdx.x;
    const int XS = max(d.H, max(d.Q, d.F));   // xin column stride
    const int Vmax = max(d.TV, d.CV);
    float * xin = S.scratch;
    const Rows R = cta_rows(d, b, G);
    int chunk = 0;
    for (int p = 0; p < A.nphase; ++p) {
        const Phase ph = A.prog[p];
        const uint32_t tag = A.tag_base + static_cast<uint32_t>(p), ptag = tag - 1u;
        const int ncol = ph.ncol;
        Seg seg[MAX_SEG];
        int r0, r1;
        const int ns = phase_segments(A, W, ph, b, R, seg, r0, r1);
        const int nr = r1 - r0;

        // single stream: every draw (codebook 0 before code-predictor position 0, codebook
        // pos - 1 before position pos, codebook 15 in FINAL) runs at this one place, so the
        // sampler's code is shared by the sixteen draws of a frame
        int drawn = 0;
        const __half * etab = nullptr;   // the embedding table the draw's id indexes next (loaded before the draw)
        if (!BATCHED && (ph.op == FINAL || (ph.op == CQKV && ph.layer == 0))) {
            const int cb = ph.op == FINAL ? NCB - 1 : ph.pos == 0 ? 0 : ph.pos - 1;
            const int V = cb == 0 ? d.TV : d.CV;
            const SampleScratch sc = sampler_scratch(S, Vmax);
            etab = cb == 0 ? W.tl_emb : W.cp_emb[cb - 1];
            bool okl = true;
            if (cb == 0 && A.logits_in) {
                for (int i0 = 0; i0 < d.TV; i0 += 4 * NCT) {
                    float v[4];
#pragma unroll
                    for (int k = 0; k < 4; ++k) v[k] = i0 + tid + k * NCT < d.TV ? __ldcg(A.logits_in + i0 + tid + k * NCT) : 0.f;
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        if (i0 + tid + k * NCT < d.TV) sc.s[i0 + tid + k * NCT] = v[k];
                }
            } else {
                okl = ll_fetch(cb == 0 ? A.w.logits : A.w.clogits + static_cast<size_t>(cb - 1) * d.CV, V, ptag, sc.s, A, S.ctrl, p);
            }
            if (!consumers_ok(S, okl)) break;
            if (ph.op == FINAL) stamp(A, p, 0);
            drawn = sample_cta<NCT, true>(V, sample_cfg(A, cb, 0), sc, BID);
            if (tid == 0) S.codes[cb] = drawn;
        }

        if (ph.op == TATTN || ph.op == CATTN) {
            if (ns > 0 && !wait_chunk(A, S, chunk, p)) break;
            const bool ok = ph.op == TATTN ? talker_attention<BATCHED>(A, S, ph, chunk, tag, ptag, p) : cp_attention<BATCHED>(A, S, ph, chunk, tag, ptag, p);
            if (!ok) break;
            if (ns > 0) {
                named_sync(BID, NCT);
                release_chunk(S, chunk);
                ++chunk;
            }
            stamp(A, p, 3);
            continue;
        }

        if (!BATCHED && ph.op == XOUT) {
            // single-layer program: the residual stream after the layer, this CTA's rows as f32
            const bool ok = ll_fetch(A.w.x, d.H, ptag, S.xres, A, S.ctrl, p);
            if (!consumers_ok(S, ok)) break;
            for (int i = R.h0 + tid; i < R.h1; i += NCT) A.step_out[0][i] = S.xres[i];
            if (b == 0 && tid == 0) {
                __threadfence();
                st_relaxed_u32(&A.w.ctl[0], A.tag_base);
            }
            named_sync(BID, NCT);
            stamp(A, p, 3);
            continue;
        }

        if (BATCHED && ph.op == SAMPLE) {
            // batched: CTA s draws codebook ph.pos of stream s from its logits (the phase
            // before) and publishes the code; the other CTAs go on
            const int st = b, cb = ph.pos;
            if (st < A.nb) {
                const SampleScratch sc = sampler_scratch(S, Vmax);
                const int V = cb == 0 ? d.TV : d.CV;
                const uint64_t * src = cb == 0 ? A.w.logits + static_cast<size_t>(st) * d.TV
                                               : A.w.clogits + (static_cast<size_t>(st) * (NCB - 1) + cb - 1) * d.CV;
                bool ok = true;
                if (cb == 0 && A.first_logits[st]) {
                    // batched frame 0: the stream's prefill logits
                    for (int i0 = 0; i0 < V; i0 += 4 * NCT) {
                        float v[4];
#pragma unroll
                        for (int k = 0; k < 4; ++k) v[k] = i0 + tid + k * NCT < V ? __ldcg(A.first_logits[st] + i0 + tid + k * NCT) : 0.f;
#pragma unroll
                        for (int k = 0; k < 4; ++k)
                            if (i0 + tid + k * NCT < V) sc.s[i0 + tid + k * NCT] = v[k];
                    }
                } else {
                    ok = ll_fetch(src, V, ptag, sc.s, A, S.ctrl, p);
                }
                if (!consumers_ok(S, ok)) break;
                stamp(A, p, 0);
                const int code = sample_cta<NCT>(V, sample_cfg(A, cb, st), sc, BID);
                if (tid == 0) ll_store(A.w.code_x + st * NCB + cb, static_cast<float>(code), tag);
            }
            stamp(A, p, 3);
            continue;
        }

        if (BATCHED && ph.op == FINAL) {
            // batched: every stream's 16 codes (words of the SAMPLE phases) -> step embeddings
            bool ok = true;
            if (tid < A.nb * NCB) {
                float v = 0.f;
                ok = ll_poll1(A.w.code_x + tid, A.tag_base + static_cast<uint32_t>(A.sample_phase[tid % NCB]), v, A, S.ctrl, p);
                S.codes[tid] = static_cast<int>(v);
            }
            if (!consumers_ok(S, ok)) break;
            stamp(A, p, 0);
            for (int st = 0; st < A.nb; ++st) {
                const int * cd = S.codes + st * NCB;
                for (int i = R.h0 + tid; i < R.h1; i += NCT) {
                    float v = __half2float(W.tl_emb[static_cast<size_t>(cd[0]) * d.H + i]);
                    for (int cb = 0; cb < NCB - 1; ++cb)
                        v = __fadd_rn(v, __half2float(W.cp_emb[cb][static_cast<size_t>(cd[cb + 1]) * d.H + i]));
                    v = __fadd_rn(v, __ldcg(A.trailing[st] + i));
                    A.step_out[st][i] = v;
                }
            }
            if (b == 0 && tid < A.nb * NCB) A.w.codes[tid] = S.codes[tid];
            if (b == 0 && tid < A.nb && S.codes[tid * NCB] != A.eos_id) A.seen[tid][S.codes[tid * NCB]] = 1;
            named_sync(BID, NCT);
            if (b == 0 && tid == 0) {
                __threadfence();
                st_relaxed_u32(&A.w.ctl[0], A.tag_base);
            }
            stamp(A, p, 3);
            continue;
        }

        if (!BATCHED && ph.op == FINAL) {
            // codebook 15 was drawn above
            named_sync(BID, NCT);
            for (int i = R.h0 + tid; i < R.h1; i += NCT) {
                float v = __half2float(W.tl_emb[static_cast<size_t>(S.codes[0]) * d.H + i]);
                for (int cb = 0; cb < NCB - 1; ++cb)
                    v = __fadd_rn(v, __half2float(W.cp_emb[cb][static_cast<size_t>(S.codes[cb + 1]) * d.H + i]));
                v = __fadd_rn(v, __ldcg(A.trailing[0] + i));
                A.step_out[0][i] = v;
            }
            if (b == 0 && tid < NCB) A.w.codes[tid] = S.codes[tid];
            if (b == 0 && tid == 0) {
                if (S.codes[0] != A.eos_id) A.seen[0][S.codes[0]] = 1;
                __threadfence();
                st_relaxed_u32(&A.w.ctl[0], A.tag_base);
            }
            stamp(A, p, 3);
            continue;
        }

        // ---- GEMV phases: chunk [norm weights][rows], inputs staged with the norm weights,
        // one barrier, dot products with the epilogue in the lanes that hold the sums
        const bool has_norm = ph.op == TQKV || ph.op == CQKV || ph.op == TGU || ph.op == CGU || ph.op == THEAD || ph.op == CHEAD;
        bool ok = ns > 0 ? wait_chunk_local(A, S, chunk, p) : true;
        stamp(A, p, 1);
        const float * nw = reinterpret_cast<const float *>(chunk_at(S, chunk, 0));
        const uint32_t woff = has_norm ? d.H * 4 : 0;     // the weight slice follows the norm weights
        const auto at = [&](uint32_t x) { return chunk_at(S, chunk, x); };
        float ss0 = 0.f, ss1 = 0.f, ss2 = 0.f, ss3 = 0.f;   // sums of squares of this thread's inputs, per column
        int nnorm = 0;                                      // columns whose norm scale is needed
        constexpr bool batched = BATCHED;
        auto stage = [&](int c, int i, float v) {
            S.xres[c * d.H + i] = v;
            xin[c * XS + i] = v * nw[i];
            const float q = v * v;
            if constexpr (BATCHED) {
                if (c == 0) ss0 += q;
                else if (c == 1) ss1 += q;
                else if (c == 2) ss2 += q;
                else ss3 += q;
            } else {
                if (c == 0) ss0 += q;
                else ss1 += q;
            }
        };
        // columns c < nc of H inputs read from global memory by load(c, i): each thread issues
        // its loads of a round before its first shared-memory store, so they are in flight
        // together instead of one after another
        auto stage_loaded = [&](int nc, auto && load) {
            constexpr int MC = BATCHED ? 4 : 2;
            for (int i0 = 0; i0 < d.H; i0 += 3 * NCT) {
                float v[MC][3];
#pragma unroll
                for (int c = 0; c < MC; ++c)
#pragma unroll
                    for (int k = 0; k < 3; ++k) {
                        const int i = i0 + tid + k * NCT;
                        v[c][k] = (c < nc && i < d.H) ? load(c, i) : 0.f;
                    }
#pragma unroll
                for (int c = 0; c < MC; ++c)
#pragma unroll
                    for (int k = 0; k < 3; ++k) {
                        const int i = i0 + tid + k * NCT;
                        if (c < nc && i < d.H) stage(c, i, v[c][k]);
                    }
            }
        };
        // after ll_fetch_cols of nc columns into xres: the same thread stages its elements
        auto stage_fetched = [&](int nc) {
            ll_each(nc * d.H, [&](int i) {
                int c = i >= d.H ? 1 : 0;
                if constexpr (BATCHED) c += (i >= 2 * d.H ? 1 : 0) + (i >= 3 * d.H ? 1 : 0);
                stage(c, i - c * d.H, S.xres[i]);
            });
        };
        switch (ph.op) {
            case TQKV: case CQKV: {
                nnorm = ncol;
                if (ph.op == TQKV && (ph.layer == 0 || ph.pos == POS_STEP_IN)) {
                    if (ok) stage_loaded(ncol, [&](int c, int i) { return __ldcg(A.step_in[c] + i); });
                } else if (batched && ph.layer == 0 && ph.pos == 0 && A.first_hidden[0]) {
                    // batched frame 0, position 0: every stream's prefill hidden
                    if (ok) stage_loaded(ncol, [&](int c, int i) { return __ldcg(A.first_hidden[c] + i); });
                } else if (batched && ph.layer == 0 && ph.pos == 0) {
                    // batched position 0: every stream's post-norm talker hidden
                    if (ok) {
                        ok = ll_fetch_cols<BATCHED>(A.w.hid_x, ncol, d.H, S.xres, d.H, A.tag_base + static_cast<uint32_t>(A.thead_phase), A, S.ctrl, p);
                        if (ok) stage_fetched(ncol);
                    }
                } else if (batched && ph.layer == 0) {
                    // batched position pos: the embedding rows of every stream's code pos - 1
                    bool okc = true;
                    const int cb = ph.pos - 1;
                    if (tid < ncol) {
                        float v = 0.f;
                        okc = ll_poll1(A.w.code_x + tid * NCB + cb, A.tag_base + static_cast<uint32_t>(A.sample_phase[cb]), v, A, S.ctrl, p);
                        S.codes[tid * NCB + cb] = static_cast<int>(v);
                    }
                    if (!consumers_ok(S, okc && ok)) { ok = false; break; }
                    const __half * tab = cb == 0 ? W.tl_emb : W.cp_emb[cb - 1];
                    stage_loaded(ncol, [&](int c, int i) { return __half2float(tab[static_cast<size_t>(S.codes[c * NCB + cb]) * d.H + i]); });
                } else if (!batched && ph.layer == 0 && ph.pos == 0) {
                    // code-predictor positions 0 and 1: the hidden and codebook 0's embedding
                    if (ok) {
                        const __half * row = etab + static_cast<size_t>(drawn) * d.H;   // codebook 0's row
                        stage_loaded(2, [&](int c, int i) {
                            return c == 0 ? (A.hidden_in ? __ldcg(A.hidden_in + i) : S.hid[i]) : __half2float(row[i]);
                        });
                    }
                } else if (!batched && ph.layer == 0) {
                    // position pos: the embedding of codebook pos - 1's draw
                    const __half * row = etab + static_cast<size_t>(drawn) * d.H;   // cp_emb[pos - 2]
                    if (ok) stage_loaded(1, [&](int, int i) { return __half2float(row[i]); });
                } else if (ok) {
                    ok = ll_fetch_cols<BATCHED>(A.w.x, ncol, d.H, S.xres, d.H, ptag, A, S.ctrl, p);
                    if (ok) stage_fetched(ncol);
                }
                break;
            }
            case TGU: case CGU:
                nnorm = ncol;
                if (ok) {
                    ok = ll_fetch_cols<BATCHED>(A.w.x, ncol, d.H, S.xres, d.H, ptag, A, S.ctrl, p);
                    if (ok) stage_fetched(ncol);
                }
                break;
            case TO: case CO:
                if (ok) ok = ll_fetch_cols<BATCHED>(A.w.attn, ncol, d.Q, xin, XS, ptag, A, S.ctrl, p);
                break;
            case TDOWN: case CDOWN:
                if (ok) ok = ll_fetch_cols<BATCHED>(A.w.h, ncol, d.F, xin, XS, ptag, A, S.ctrl, p);
                break;
            case THEAD:
                nnorm = ncol;
                if (ok) ok = ll_fetch_cols<BATCHED>(A.w.x, ncol, d.H, S.xres, d.H, ptag, A, S.ctrl, p);
                if (ok) stage_fetched(ncol);
                break;
            case CHEAD:
                if (batched) {
                    nnorm = ncol;
                    if (ok) ok = ll_fetch_cols<BATCHED>(A.w.x, ncol, d.H, S.xres, d.H, ptag, A, S.ctrl, p);
                    if (ok) stage_fetched(ncol);
                } else {
                    // the single-stream pass's last column is this position
                    nnorm = 1;
                    ok = ok && ll_fetch(A.w.x + static_cast<size_t>(ncol - 1) * d.H, d.H, ptag, S.xres, A, S.ctrl, p);
                    if (ok) stage_fetched(1);
                }
                break;
            default: break;
        }
        {
            const float ss[MAXC] = {ss0, ss1, ss2, ss3};
            norm_partial(S, ss, nnorm);
        }
        if (!consumers_ok(S, ok)) break;
        stamp(A, p, 0);
        const float eps = (ph.op <= THEAD) ? d.eps_t : d.eps_c;
        const float sc0 = nnorm > 0 ? norm_scale(S, 0, d.H, eps) : 1.f;
        const float sc1 = nnorm > 1 ? norm_scale(S, 1, d.H, eps) : 1.f;
        const float sc2 = BATCHED && nnorm > 2 ? norm_scale(S, 2, d.H, eps) : 1.f;
        const float sc3 = BATCHED && nnorm > 3 ? norm_scale(S, 3, d.H, eps) : 1.f;
        const auto scale_of = [&](int c) {
            if constexpr (BATCHED) return c == 0 ? sc0 : c == 1 ? sc1 : c == 2 ? sc2 : sc3;
            else return c == 0 ? sc0 : sc1;
        };
        const int gcol = (ph.op == CHEAD && !batched) ? 1 : ncol;
        const uint32_t t = tag;
        if (ph.op == THEAD)
            for (int c = 0; c < ncol; ++c) {
                const float s = scale_of(c);
                for (int i = tid; i < d.H; i += NCT) {
                    const float hv = xin[c * XS + i] * s;
                    if (!batched) S.hid[i] = hv;
                    else if (i >= R.h0 && i < R.h1) ll_store(A.w.hid_x + static_cast<size_t>(c) * d.H + i, hv, t);
                    if (b == 0) A.w.hidden[static_cast<size_t>(c) * d.H + i] = hv;
                }
            }
        // the sums (one GEMV call site per shape), then this phase's epilogue on the rows this thread owns
        float * ys = S.part + A.ysum_off;
        {
            const int K = (ph.op == TDOWN || ph.op == CDOWN) ? d.F : (ph.op == TO || ph.op == CO) ? d.Q : d.H;
            if (ph.op == TGU || ph.op == CGU) gemv_sums<true, BATCHED>(gcol, S, chunk, woff, nr, K, xin, XS, S.part, ys);
            else gemv_sums<false, BATCHED>(gcol, S, chunk, woff, nr, K, xin, XS, S.part, ys);
        }
        const auto y_of = [&](int u, int c) { return ys[2 * c * nr + u]; };
        switch (ph.op) {
            case TQKV: case CQKV:
                gemv_owned(gcol, nr, [&](int u, int c) { ll_store(A.w.qkv + static_cast<size_t>(c) * d.QKV + r0 + u, y_of(u, c) * scale_of(c), t); });
                break;
            case TO: case CO: case TDOWN: case CDOWN:
                gemv_owned(gcol, nr, [&](int u, int c) {
                    ll_store(A.w.x + static_cast<size_t>(c) * d.H + r0 + u, S.xres[c * d.H + r0 + u] + y_of(u, c), t);
                });
                break;
            case TGU: case CGU:
                gemv_owned(gcol, nr, [&](int u, int c) {
                    const float s = scale_of(c);
                    const float g = y_of(u, c) * s, up = ys[(2 * c + 1) * nr + u] * s;
                    ll_store(A.w.h + static_cast<size_t>(c) * d.F + r0 + u, g / (1.f + expf(-g)) * up, t);
                });
                break;
            case THEAD:
                gemv_owned(gcol, nr, [&](int u, int c) { ll_store(A.w.logits + static_cast<size_t>(c) * d.TV + r0 + u, y_of(u, c) * scale_of(c), t); });
                break;
            case CHEAD:
                gemv_owned(gcol, nr, [&](int u, int c) {
                    ll_store(A.w.clogits + (static_cast<size_t>(c) * (NCB - 1) + ph.pos - 1) * d.CV + r0 + u, y_of(u, c) * scale_of(c), t);
                });
                break;
            default: break;
        }
        stamp(A, p, 2);
        named_sync(BID, NCT);   // the chunk, xin and xres are reused from here on
        if (ns > 0) {
            release_chunk(S, chunk);
            ++chunk;
        }
        stamp(A, p, 3);
    }
}

// One launch of a phase program: BATCHED selects the consumer compiled for 2 or 4 streams.
// The two shapes are separate kernels, so each gets its own register allocation and code: the
// batched program's wider fetches do not cost the single-stream frame registers.
template <bool BATCHED>
__device__ __forceinline__ void frame_main(const Args & A) {
    extern __shared__ __align__(128) char smem[];
    const SmemLayout L = smem_layout(A.d, A.ring_bytes, A.scratch_floats, A.part_floats, A.xcols, A.cp_slots);
    Sm S = carve(smem, L);
    if (threadIdx.x == 0) {
        for (int i = 0; i < NSLOT; ++i) mbar_init(&S.bars[i], 1);
        S.ctrl->released = 0;
        S.ctrl->consumed = 0;
        S.ctrl->abort = 0;
        fence_mbar_init();
    }
    __syncthreads();
    if (unsigned long long * pb = prof_base(A)) pb[4 * A.nphase] = globaltimer();
    if (threadIdx.x >= NCT) producer(A, S);
    else consumer<BATCHED>(A, S);
}

// Single-stream programs (a frame, frame 0, one talker layer).
__global__ void __launch_bounds__(NTHR, 1) k_frame(const __grid_constant__ Args A) { frame_main<false>(A); }
// Batched programs: 2 or 4 streams, one weight pass.
__global__ void __launch_bounds__(NTHR, 1) k_frame_batch(const __grid_constant__ Args A) { frame_main<true>(A); }

// A standalone launch of the device sampler on given logits (one CTA), for parity tests.
__global__ void __launch_bounds__(NCT, 1) k_sample(const float * logits, int V, SampleCfg cfg, int * out) {
    extern __shared__ __align__(16) float sbuf[];
    const SampleScratch sc = sampler_layout(sbuf, V);
    for (int i = threadIdx.x; i < V; i += NCT) sc.s[i] = logits[i];
    named_sync(BID, NCT);
    const int c = sample_cta<NCT>(V, cfg, sc, BID);
    if (threadIdx.x == 0) *out = c;
}

} // namespace navi::fk
