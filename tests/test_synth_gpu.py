"""The per-utterance loop (reference model/qwen3tts/graph.cpp:52-111) through the C ABI:
navi_graph_synth_ids against the same loop written out over the talker and frame entry points
(prompt, prefill, run_first on the prefill's hidden and logits, run at KV position
n_prefill + i - 1 with the i-th trailing row, tts_pad after them), bit for bit; seeded
repeatability; and the stop rules (EOS or max_frames)."""
import numpy as np
import pytest

from navi_b200 import engine
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
