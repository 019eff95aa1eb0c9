"""Host-side model of the frame kernel's weight ring (producer warp vs consumer warps).

The producer streams each phase's weight slice into a shared-memory ring; a chunk that
would straddle the ring's end starts the next lap, and it may only overwrite bytes whose
data chunk the consumers have released (the rule in navi-tts_b200/csrc/frame_kernel.cu,
producer()).  This test replays that rule over the full-size phase program for several
CTAs and ring sizes and checks that the stream never deadlocks and never overwrites
unreleased data -- a property the GPU can only show by timing out.
"""
import pytest

from navi_b200 import model_spec

NSLOT = 16


NCW = 11   # consumer warps: weight slices may be cut at the first k-chunk of a warp's K range


def phase_chunks(cfg, b, G, n_past=512):
    """Chunks per phase on CTA b of G (phases without a chunk dropped), program order, as
    lists of segments (bytes, rows of a weight slice or 0): norm weights ride with QKV /
    gate-up / heads; talker attention carries q/k norms and its KV head's slice of the
    split's K and V rows (Frame::Impl::attn_plan's splits); the code predictor's attention
    CTA for (KV head, layer) carries q/k norms."""
    tl, cp = cfg.talker, cfg.cp
    H, Q, KV, F, HD = tl.hidden, tl.n_head * tl.head_dim, tl.n_kv_head * tl.head_dim, tl.ff, tl.head_dim
    QKV = Q + 2 * KV

    def rows(R):
        return (R * (b + 1)) // G - (R * b) // G
    NKV = tl.n_kv_head
    per_head = max(1, min(148, G // NKV))
    split = min(per_head, max(1, -(-n_past // 8)))
    chunk = max(1, -(-n_past // split))
    split = max(1, -(-n_past // chunk))
    sp = b % split
    r0 = min(sp * chunk, n_past)
    r1 = min(r0 + chunk, n_past)
    nc = r1 - r0
    tattn = [(HD * 4, 0), (HD * 4, 0)] + ([(nc * HD * 2, 0), (nc * HD * 2, 0)] if nc else []) if b < NKV * split else []
    cattn_layers = {l for l in range(cp.n_layer) if l * NKV <= b < (l + 1) * NKV}   # CTA l * NKV + g

    def mat(R, K):
        n = rows(R)
        return [(n * K * 2, n)] if n else []
    qkv = [(H * 4, 0)] + mat(QKV, H) if rows(QKV) else []
    o = mat(H, Q)
    gu = [(H * 4, 0)] + mat(F, H) + mat(F, H) if rows(F) else []
    down = mat(H, F)
    out = []
    for _ in range(tl.n_layer):
        out += [qkv, tattn, o, gu, down]
    out.append([(H * 4, 0)] + mat(tl.vocab, H) if rows(tl.vocab) else [])
    for _pass in range(15):
        for l in range(cp.n_layer):
            out += [qkv, [(HD * 4, 0), (HD * 4, 0)] if l in cattn_layers else [], o, gu, down]
        out.append([(H * 4, 0)] + mat(cp.vocab, H) if rows(cp.vocab) else [])
    return [c for c in out if c]


def chunk_split(segs, room):
    """The largest allowed cut offset <= room (frame_kernel.cuh, chunk_split)."""
    best, o = 0, 0
    for nbytes, nr in segs:
        if o <= room:
            best = o
        if nr:
            kstep = nr * 16
            nk = nbytes // kstep
            for w in range(1, NCW):
                at = o + (nk * w // NCW) * kstep
                if best < at <= room:
                    best = at
        o += nbytes
    return best


def place(segs, issued, RB):
    """(cut, virtual end, physical pieces) of the next chunk (the producer's placement)."""
    total = sum(n for n, _ in segs)
    pos = issued % RB
    cut, end = total, issued + total
    if pos + total > RB:
        cut = chunk_split(segs, RB - pos)
        if total - cut > pos:
            cut = 0
        end = issued + (RB - pos) + (total - cut)
    pieces = []
    if cut > 0:
        pieces.append((pos, pos + cut))
    if total > cut:
        pieces.append((0, total - cut))
    return cut, end, pieces


def simulate(chunks, RB):
    """Producer issues greedily under the ring rule; consumer frees one chunk per step.
    Returns the number of chunks consumed (== len(chunks) unless the stream stalls) and
    the lookahead of every chunk (chunks still unconsumed ahead of it when it was issued)."""
    issued, released, consumed = 0, 0, 0
    meta = {}
    nxt = 0
    live = {}   # chunk -> physical pieces of issued, unreleased chunks
    ahead = []
    while consumed < len(chunks):
        progressed = False
        while nxt < len(chunks):
            cut, end, pieces = place(chunks[nxt], issued, RB)
            need = min(end - RB, issued) if end > RB else 0
            if released < need or nxt - consumed >= NSLOT:
                break
            # the physical bytes of the new pieces must not hold unreleased data, nor overlap
            for a0, a1 in pieces:
                assert 0 <= a0 < a1 <= RB
                for c, qs in live.items():
                    for q0, q1 in qs:
                        assert not (a0 < q1 and q0 < a1), ("overwrites live data", nxt, c)
            if len(pieces) == 2:
                assert pieces[1][1] <= pieces[0][0]
            meta[nxt] = end
            live[nxt] = pieces
            ahead.append(nxt - consumed)
            issued = end
            nxt += 1
            progressed = True
        if consumed < nxt:
            released = meta[consumed]
            del live[consumed]
            consumed += 1
            progressed = True
        assert progressed
    return consumed, ahead


@pytest.mark.parametrize("G", [148, 132, 100])
@pytest.mark.parametrize("ring_kb", [100, 120, 160])
@pytest.mark.parametrize("n_past", [0, 64, 512, 2048])
def test_ring_never_stalls_full_size(G, ring_kb, n_past):
    cfg = model_spec.full_config(1024)
    RB = ring_kb * 1024
    for b in (0, 1, G // 2, G - 1):
        chunks = phase_chunks(cfg, b, G, n_past)
        if max(sum(n for n, _ in c) for c in chunks) > RB:
            continue   # Frame::create refuses such a ring
        done, _ = simulate(chunks, RB)
        assert done == len(chunks), (b, G, ring_kb)


def test_cut_chunks_keep_the_producer_ahead():
    """At the full-size ring (about 150 KB) cutting chunks at the ring's end lets the
    producer issue nearly every chunk while an earlier one is still being consumed."""
    cfg = model_spec.full_config(1024)
    for b in (0, 60, 147):
        chunks = phase_chunks(cfg, b, 148, 512)
        done, ahead = simulate(chunks, 150 * 1024)
        assert done == len(chunks)
        assert sum(1 for a in ahead if a <= 0) <= 4, (b, sum(1 for a in ahead if a <= 0))

