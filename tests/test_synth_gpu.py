"""The per-utterance loop (reference model/qwen3tts/graph.cpp:52-111) through the C ABI:
navi_graph_synth_ids against the same loop written out over the talker and frame entry points
(prompt, prefill, run_first on the prefill's hidden and logits, run at KV position
n_prefill + i - 1 with the i-th trailing row, tts_pad after them), bit for bit; seeded
repeatability; and the stop rules (EOS or max_frames)."""
import numpy as np
import pytest

from navi_b200 import capi, engine
from oracle import model as om

pytestmark = pytest.mark.gpu


def _ids(cfg, n_text, seed):
    rng = np.random.default_rng(seed)
    nl = 198 % cfg.text_vocab
    return [cfg.im_start_id, cfg.assistant_id, nl] + rng.integers(0, cfg.text_vocab, n_text).tolist() + \
        [cfg.im_end_id, nl, cfg.im_start_id, cfg.assistant_id, nl]


def _manual_loop(dev, w, ids, language, spk, s, seed, max_frames):
    tal = engine.Talker(dev, w, max_prompt_tokens=256, max_positions=256 + max_frames + 1)
    frame = engine.Frame(dev, w)
    pr = tal.build_prompt(ids, language, spk)
    tal.prefill(pr)
    kv = tal.kv()
    H = w.params.talker.hidden
    frame.reset()
    out = []
    for i in range(max_frames):
        trailing = pr.trailing + 4 * H * i if i < pr.n_trailing else pr.tts_pad
        r = frame.run_first(tal.d_hidden(), tal.d_logits(), trailing, s, seed, 0) if i == 0 else \
            frame.run(kv, pr.n_prefill + i - 1, trailing, s, seed, i)
        assert r.ok, r.error
        if r.eos:
            break
        out.append(r.codes)
    return np.array(out, np.int32).reshape(-1, 16)


def test_graph_matches_the_loop_written_out(small_navi):
    W = om.Weights.from_navi(small_navi)
    dev = engine.Device(0)
    w = engine.Weights(dev, small_navi)
    g = engine.Graph(dev, w, max_prompt_tokens=256, max_frames=64)
    ids = _ids(W.cfg, 9, seed=3)
    spk = np.random.default_rng(2).standard_normal(W.tl.hidden).astype(np.float32)
    s = engine.Sampling(top_p=0.9, cp_top_p=0.9)
    codes, st = g.synth_ids(ids, "english", spk, s, 11, 14)
    want = _manual_loop(dev, w, ids, "english", spk, s, 11, 14)
    assert codes.shape == want.shape and np.array_equal(codes, want)
    assert st.n_frames == len(codes) and st.n_tokens == 9
    assert (st.eos == 1) != (st.hit_cap == 1)
    assert st.hit_cap == 0 or st.n_frames == 14
    assert st.prefill_ms > 0 and st.frames_ms > 0 and st.total_ms >= st.prefill_ms
    # codes are ids of the codebooks: codebook 0 below the talker vocabulary, the others below the cp vocabulary
    if len(codes):
        assert codes[:, 0].max() < W.tl.vocab and codes[:, 1:].max() < W.cp.vocab


def test_graph_is_seeded(small_navi):
    W = om.Weights.from_navi(small_navi)
    dev = engine.Device(0)
    w = engine.Weights(dev, small_navi)
    g = engine.Graph(dev, w, max_prompt_tokens=256, max_frames=32)
    ids = _ids(W.cfg, 6, seed=8)
    spk = np.random.default_rng(4).standard_normal(W.tl.hidden).astype(np.float32)
    s = engine.Sampling()
    a, _ = g.synth_ids(ids, "auto", spk, s, 5, 10)
    b, _ = g.synth_ids(ids, "auto", spk, s, 5, 10)
    c, _ = g.synth_ids(ids, "auto", spk, s, 6, 10)
    assert np.array_equal(a, b)
    assert not np.array_equal(a, c)


def test_graph_streams_pcm_of_its_codes(small_navi):
    """Graph::synth with audio (graph.cpp:73-108): the frames are vocoded in a first batch of
    first_batch frames, then batches of vocoder_batch, then the remainder; the PCM equals one
    vocoder pass over the same codes (batching never changes it), and the codes equal the
    codes-only loop's."""
    W = om.Weights.from_navi(small_navi)
    dev = engine.Device(0)
    w = engine.Weights(dev, small_navi)
    g = engine.Graph(dev, w, max_prompt_tokens=256, max_frames=64, vocoder_chunk=8)
    ids = _ids(W.cfg, 7, seed=5)
    spk = np.random.default_rng(6).standard_normal(W.tl.hidden).astype(np.float32)
    s = engine.Sampling(top_p=0.9, cp_top_p=0.9, min_frames=40)
    seen = []
    codes, pcm, st, sizes = g.synth(ids, "english", spk, s, 21, 23, first_batch=3, vocoder_batch=8,
                                    on_pcm=lambda a: seen.append(a.size))
    want_codes, _ = g.synth_ids(ids, "english", spk, s, 21, 23)
    assert np.array_equal(codes, want_codes)
    assert st.n_frames == 23 and st.hit_cap == 1
    spf = W.cfg.samples_per_frame
    assert sizes == seen == [3 * spf, 8 * spf, 8 * spf, 4 * spf]
    voc = engine.Vocoder(dev, w, max_chunk_frames=32)
    want = voc.decode(codes)
    assert pcm.shape == want.shape
    np.testing.assert_allclose(pcm, want, rtol=0, atol=1e-5)
    assert np.abs(pcm).max() <= 1.0
    assert st.vocoder_ms > 0 and 0 < st.ttfc_ms <= st.ttfa_ms <= st.total_ms
    assert st.audio_s == pytest.approx(23 * spf / W.cfg.sample_rate)
    assert st.rtf == pytest.approx(st.total_ms / 1000.0 / st.audio_s)
    # the vocoder's chunk caps the batch; first_batch 0 = vocoder_batch
    _, pcm2, _, sizes2 = g.synth(ids, "english", spk, s, 21, 23, first_batch=0, vocoder_batch=100)
    assert sizes2 == [8 * spf, 8 * spf, 7 * spf]
    np.testing.assert_allclose(pcm2, want, rtol=0, atol=1e-5)
    g.close()
    voc.close()


def test_graph_without_vocoder_refuses_pcm(small_navi):
    W = om.Weights.from_navi(small_navi)
    dev = engine.Device(0)
    w = engine.Weights(dev, small_navi)
    g = engine.Graph(dev, w, max_prompt_tokens=256, max_frames=16, vocoder_chunk=0)
    ids = _ids(W.cfg, 5, seed=1)
    spk = np.zeros(W.tl.hidden, np.float32)
    codes, st = g.synth_ids(ids, "english", spk, engine.Sampling(), 1, 4)
    assert st.ttfa_ms == 0 and st.vocoder_ms == 0
    with pytest.raises(capi.NaviError):
        g.synth(ids, "english", spk, engine.Sampling(), 1, 4)
    g.close()


def test_graph_rejects_bad_requests_and_stays_usable(small_navi):
    """Graph::synth's argument checks (graph.cpp:60-64: empty text; KV cache too small for the
    prompt plus max_frames) fail with a status and leave the graph usable for the next
    request, whose codes equal a fresh graph's."""
    W = om.Weights.from_navi(small_navi)
    dev = engine.Device(0)
    w = engine.Weights(dev, small_navi)
    g = engine.Graph(dev, w, max_prompt_tokens=64, max_frames=8, vocoder_chunk=4)
    spk = np.random.default_rng(3).standard_normal(W.tl.hidden).astype(np.float32)
    s = engine.Sampling(top_p=0.9, cp_top_p=0.9)
    empty = _ids(W.cfg, 0, seed=1)            # the template alone: no text
    with pytest.raises(capi.NaviError) as e:
        g.synth_ids(empty, "english", spk, s, 1, 4)
    assert e.value.status == capi.NAVI_E_ARG
    ids = _ids(W.cfg, 5, seed=2)
    with pytest.raises(capi.NaviError) as e:      # the prompt + 80 frames > the 64 + 8 + 1 positions
        g.synth(ids, "english", spk, s, 1, 80, first_batch=2, vocoder_batch=4)
    assert e.value.status == capi.NAVI_E_KV_FULL
    codes, pcm, st, _ = g.synth(ids, "english", spk, s, 9, 6, first_batch=2, vocoder_batch=4)
    fresh = engine.Graph(dev, w, max_prompt_tokens=64, max_frames=8, vocoder_chunk=4)
    codes2, pcm2, _, _ = fresh.synth(ids, "english", spk, s, 9, 6, first_batch=2, vocoder_batch=4)
    assert np.array_equal(codes, codes2) and np.array_equal(pcm, pcm2)
    g.close()
    fresh.close()


@pytest.mark.parametrize("n", [3, 4])
def test_synth_batch_matches_single_streams(small_navi, n):
    """Graph::synth_batch of n utterances (different texts, speakers, seeds and frame caps; 3
    streams run as launches of 2 + 1) against Graph::synth of each alone: the same codes and
    the same PCM, sample for sample (at these KV lengths the batched attention splits equal
    the single-stream ones, so every float sum is the same), and per-stream stats."""
    W = om.Weights.from_navi(small_navi)
    dev = engine.Device(0)
    w = engine.Weights(dev, small_navi)
    g = engine.Graph(dev, w, max_prompt_tokens=64, max_frames=24, vocoder_chunk=8, max_streams=4)
    one = engine.Graph(dev, w, max_prompt_tokens=64, max_frames=24, vocoder_chunk=8)
    s = engine.Sampling(top_p=0.9, cp_top_p=0.9, min_frames=24)
    reqs = []
    for i in range(n):
        ids = _ids(W.cfg, 5 + 3 * i, seed=20 + i)
        spk = np.random.default_rng(30 + i).standard_normal(W.tl.hidden).astype(np.float32)
        reqs.append((ids, spk, 500 + i, 12 + 3 * i))
    out = g.synth_batch(reqs, "english", s, first_batch=4, vocoder_batch=8)
    for i, (ids, spk, seed, mf) in enumerate(reqs):
        codes, pcm, st = out[i]
        c1, p1, s1, _ = one.synth(ids, "english", spk, s, seed, mf, first_batch=4, vocoder_batch=8)
        assert np.array_equal(codes, c1), i
        assert pcm.shape == p1.shape and np.array_equal(pcm, p1), i
        assert st.n_frames == s1.n_frames == mf and st.hit_cap == 1
        assert st.ttfa_ms > 0 and st.vocoder_ms > 0 and st.total_ms >= st.ttfa_ms


def test_synth_batch_rejects_more_streams_than_created(small_navi):
    W = om.Weights.from_navi(small_navi)
    dev = engine.Device(0)
    w = engine.Weights(dev, small_navi)
    g = engine.Graph(dev, w, max_prompt_tokens=64, max_frames=8, vocoder_chunk=0, max_streams=2)
    spk = np.zeros(W.tl.hidden, np.float32)
    r = (_ids(W.cfg, 4, 1), spk, 1, 4)
    with pytest.raises(capi.NaviError) as e:
        g.synth_batch([r, r, r], "english", engine.Sampling(), audio=False)
    assert e.value.status == capi.NAVI_E_ARG
    codes = g.synth_batch([r, r], "english", engine.Sampling(), audio=False)
    assert all(c.shape == (4, 16) for c, _, _ in codes)
