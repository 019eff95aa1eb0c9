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


def phase_chunks(cfg, b, G, n_past=512):
    """Chunk bytes per phase on CTA b of G (phases without a chunk dropped), program order:
    norm weights ride with QKV / gate-up / heads; talker attention carries q/k norms and
    its KV head's slice of the split's K and V rows (Frame::Impl::attn_plan's splits)."""
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
    tattn = (2 * HD * 4 + 2 * (r1 - r0) * HD * 2) if b < NKV * split else 0
    cattn_layers = {l for l in range(cp.n_layer) if l * NKV <= b < (l + 1) * NKV}   # CTA l * NKV + g
    qkv, o, gu, down = H * 4 + rows(QKV) * H * 2, rows(H) * Q * 2, H * 4 + 2 * rows(F) * H * 2, rows(H) * F * 2
    out = []
    for _ in range(tl.n_layer):
        out += [qkv, tattn, o, gu, down]
    out.append(H * 4 + rows(tl.vocab) * H * 2)
    for _pass in range(15):
        for l in range(cp.n_layer):
            out += [qkv, 2 * HD * 4 if l in cattn_layers else 0, o, gu, down]
        out.append(H * 4 + rows(cp.vocab) * H * 2)
    return [c for c in out if c > 0]


def simulate(chunks, RB):
    """Producer issues greedily under the ring rule; consumer frees one chunk per step.
    Returns the number of chunks consumed (== len(chunks) unless the stream stalls)."""
    issued, released, consumed = 0, 0, 0
    meta = {}
    nxt = 0
    live = []   # (virtual start, virtual end) of issued, unreleased chunks
    while consumed < len(chunks):
        progressed = False
        while nxt < len(chunks):
            total = chunks[nxt]
            head = issued
            if head % RB + total > RB:
                head += RB - head % RB
            need = min(head + total - RB, issued) if head + total > RB else 0
            if released < need or nxt - consumed >= NSLOT:
                break
            # the physical bytes [head % RB, +total) must not hold unreleased data
            p0, p1 = head % RB, head % RB + total
            for s, e in live:
                q0, q1 = s % RB, s % RB + (e - s)
                assert not (p0 < q1 and q0 < p1), ("overwrites live data", nxt, s, e, head)
            meta[nxt] = head + total
            live.append((head, head + total))
            issued = head + total
            nxt += 1
            progressed = True
        if consumed < nxt:
            released = meta[consumed]
            live.pop(0)
            consumed += 1
            progressed = True
        if not progressed:
            break
    return consumed


@pytest.mark.parametrize("G", [148, 132, 100])
@pytest.mark.parametrize("ring_kb", [100, 120, 160])
@pytest.mark.parametrize("n_past", [0, 64, 512, 2048])
def test_ring_never_stalls_full_size(G, ring_kb, n_past):
    cfg = model_spec.full_config(1024)
    RB = ring_kb * 1024
    for b in (0, 1, G // 2, G - 1):
        chunks = phase_chunks(cfg, b, G, n_past)
        if max(chunks) > RB:
            continue   # Frame::create refuses such a ring
        assert simulate(chunks, RB) == len(chunks), (b, G, ring_kb)

