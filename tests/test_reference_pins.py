"""The oracle against the reference engine's own frame code, on the CPU.

oracle/_ref/ref_frame_check is model/qwen3tts/frame.hip of the reference compiled for the host
against this repository's stand-in for the HIP runtime (oracle/hipsim: one thread block as
256 cooperative fibers, wave32 shuffles and ballots, block barriers), driven through the
reference's own Frame::Impl::launch. It therefore runs the reference's integer work exactly
(the splitmix64 seed chain, frame.hip:581-586, 658-659, 497; the radix k-th largest,
225-256; the draw walk and PCG32, 169-175, 263-296) and its float work in its own order, with
the host C library's expf / powf / sincosf in place of the GPU's.

Pins:
- the per-draw seeds of oracle_draw_seed (and of the device sampler, which shares the chain)
  equal the reference's for any request seed and frame index;
- oracle_sample with the C library's expf (the only difference between the two on the same
  logits) picks the reference's tl_sample / cp_sample id bit for bit, including greedy ties,
  -inf logits, suppression, the EOS gate and the repetition penalty;
- a whole reference frame (talker step, code predictor, sampling, step embedding) on the small
  model agrees with oracle.talker_step / code_predictor / step_embedding, and its codes are
  the oracle sampler's on the reference's own logits.
The golden file tests/golden/ref_frame_small.npz (tests/golden/make_ref_golden.py) holds one
reference frame and a set of reference draws, so the last two checks also run where the
reference tree is absent.
"""
import os
from dataclasses import replace

import numpy as np
import pytest
import torch

from navi_b200 import model_spec
from oracle import model as om
from oracle import ref_frame as rf

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
needs_ref = pytest.mark.skipif(not rf.available(), reason="oracle/_ref/ref_frame_check is built by build() from the reference tree")


def full_vocab_config():
    """The small model with the benchmark vocabularies (talker 3072, code predictor 2048) and
    the control ids that go with them (suppression from 2048, EOS 2050)."""
    c = model_spec.small_config()
    return replace(c, name="synthetic-small-full-vocab", talker=replace(c.talker, vocab=3072), cp=replace(c.cp, vocab=2048),
                   codec_pad_id=2048, codec_bos_id=2049, codec_eos_id=2050, codec_think_id=2054, codec_nothink_id=2055,
                   codec_think_bos_id=2056, codec_think_eos_id=2057, languages=(("english", 2050), ("german", 2053)))


@pytest.fixture(scope="module")
def vocab_navi(tmp_path_factory):
    path = tmp_path_factory.mktemp("navi") / "full_vocab.navi"
    model_spec.write_synthetic(path, full_vocab_config())
    return str(path)


@needs_ref
def test_seed_chain_matches_reference(small_navi):
    rng = np.random.default_rng(11)
    pairs = [(int(rng.integers(0, 2**63)) * 2 + int(rng.integers(2)), int(rng.integers(-5, 100000))) for _ in range(300)]
    pairs += [(0, 0), (2**64 - 1, -1), (1, 2**31 - 1)]
    ref = rf.seeds(small_navi, pairs)
    L = om.sampler_lib()
    for (seed, fi), (ts, cs) in zip(pairs, ref):
        assert L.oracle_draw_seed(seed, fi, 0) == ts
        for cb in (1, 7, 15):   # cp_sample's per-position seed, frame.hip:497
            assert L.oracle_draw_seed(seed, fi, cb) == (cs + cb * 0xD1B54A32D192ED03) % 2**64


def _sampler_cases(TV, CV, eos, rng):
    out = []
    for kind in ("normal", "ties", "neginf", "peaked"):
        for cb in (0, 1, 9, 15):
            V = TV if cb == 0 else CV
            x = rng.standard_normal(V).astype(np.float32) * 3
            if kind == "ties":
                x = np.round(x)
            elif kind == "neginf":
                x[rng.random(V) < 0.7] = -np.inf
            elif kind == "peaked":
                x[rng.integers(V)] += 40.0
            for temp, k, rep, fi in ((0.9, 50, 1.05, 5), (1.3, 0, 1.05, 1), (0.7, 1, 0.0, 7), (0.9, V, 1.05, 0), (0.0, 50, 1.05, 3),
                                     (1.0, 7, 1.3, 2)):
                seen = (rng.random(TV) < 0.05).astype(np.uint8)
                if cb == 0 and kind == "peaked":
                    x[eos] = x.max() + 1.0   # EOS on top: gated before min_frames, else drawn
                s = rf.RefSampling(temperature=temp, top_k=k, repetition_penalty=rep, cp_temperature=temp, cp_top_k=k, min_frames=2)
                out.append((s, int(rng.integers(1 << 62)), fi, cb, x.copy(), seen))
    return out


@needs_ref
@pytest.mark.parametrize("which", ["small", "full_vocab"])
def test_sampler_matches_reference_code(small_navi, vocab_navi, which):
    navi = small_navi if which == "small" else vocab_navi
    c = model_spec.small_config() if which == "small" else full_vocab_config()
    TV, CV, eos = c.talker.vocab, c.cp.vocab, c.codec_eos_id
    cases = _sampler_cases(TV, CV, eos, np.random.default_rng(5 if which == "small" else 6))
    ref = rf.sample(navi, cases)
    for (s, seed, fi, cb, x, seen), want in zip(cases, ref):
        os_ = om.Sampling(temperature=s.temperature, top_k=s.top_k, top_p=1.0, repetition_penalty=s.repetition_penalty,
                          cp_temperature=s.cp_temperature, cp_top_k=s.cp_top_k, cp_top_p=1.0, min_frames=s.min_frames, rng=0)
        mods = (TV - 1024, eos, seen) if cb == 0 else None
        got = om.sample(x, cb, os_, seed, fi, talker_mods=mods, exp_libm=True)
        assert got == want, (which, cb, s, fi, got, want)


def _frame_inputs(W, n_past, seed):
    tl = W.tl
    kvd = tl.n_kv_head * tl.head_dim
    g = torch.Generator().manual_seed(seed)
    kv = [(torch.randn(n_past + 1, kvd, generator=g).half(), torch.randn(n_past + 1, kvd, generator=g).half())
          for _ in range(tl.n_layer)]
    step, trailing = torch.randn(tl.hidden, generator=g), torch.randn(tl.hidden, generator=g)
    seen = (torch.rand(tl.vocab, generator=g) < 0.03).numpy().astype(np.uint8)
    return kv, step, trailing, seen


def check_frame(W, r, kv, n_past, step, trailing, seen, seed, fi, hidden=None, logits=None):
    """The oracle on the reference frame's inputs (and, for the draws, on its logits)."""
    tl = W.tl
    s = om.Sampling(rng=0)
    if hidden is None:
        kvd = tl.n_kv_head * tl.head_dim
        kv_o = [(torch.cat([k.float(), torch.zeros(2, kvd)]), torch.cat([v.float(), torch.zeros(2, kvd)])) for k, v in kv]
        hid_o, lg_o = om.talker_step(W, step, kv_o, n_past)
        assert om.rel_l2(r.hidden, hid_o) < 1e-5, om.rel_l2(r.hidden, hid_o)
        assert om.rel_l2(r.logits, lg_o) < 1e-5, om.rel_l2(r.logits, lg_o)
        for l in range(tl.n_layer):   # the new K/V rows: one f16 rounding of the same value
            assert om.rel_l2(np.asarray(r.k_rows[l], np.float32), kv_o[l][0][n_past]) < 1e-3
            assert om.rel_l2(np.asarray(r.v_rows[l], np.float32), kv_o[l][1][n_past]) < 1e-3
    else:
        assert np.array_equal(r.hidden, hidden) and np.array_equal(r.logits, logits)
    cb0 = om.sample(r.logits, 0, s, seed, fi, talker_mods=(tl.vocab - 1024, W.cfg.codec_eos_id, seen), exp_libm=True)
    assert r.codes[0] == cb0
    _, clo = om.code_predictor(W, torch.from_numpy(np.asarray(r.hidden)), r.codes[0], s, seed, fi, teacher_codes=r.codes)
    for k in range(15):
        assert om.rel_l2(r.clogits[k], clo[k]) < 1e-4, (k, om.rel_l2(r.clogits[k], clo[k]))
        assert r.codes[k + 1] == om.sample(r.clogits[k], k + 1, s, seed, fi, exp_libm=True), k
    assert om.rel_l2(r.step_out, om.step_embedding(W, r.codes, torch.as_tensor(trailing))) < 1e-6
    want_seen = seen.copy()
    if r.codes[0] != W.cfg.codec_eos_id:
        want_seen[r.codes[0]] = 1
    assert np.array_equal(r.seen, want_seen)


@needs_ref
@pytest.mark.parametrize("n_past", [0, 10, 37])
def test_frame_matches_reference_code(small_navi, n_past):
    W = om.Weights.from_navi(small_navi)
    tl = W.tl
    kv, step, trailing, seen = _frame_inputs(W, n_past, seed=n_past + 100)
    dims = (tl.hidden, tl.vocab, W.cp.vocab, tl.n_layer, tl.n_kv_head * tl.head_dim)
    r = rf.frame(small_navi, dims, rf.RefSampling(), 42 + n_past, 3, seen, trailing.numpy(), step_in=step.numpy(),
                 kv=[(k.numpy(), v.numpy()) for k, v in kv], n_past=n_past)
    assert r.ok
    check_frame(W, r, kv, n_past, step, trailing.numpy(), seen, 42 + n_past, 3)


@needs_ref
def test_first_frame_matches_reference_code(small_navi):
    W = om.Weights.from_navi(small_navi)
    tl = W.tl
    g = torch.Generator().manual_seed(9)
    hidden, logits, trailing = torch.randn(tl.hidden, generator=g), torch.randn(tl.vocab, generator=g) * 3, torch.randn(tl.hidden, generator=g)
    seen = np.zeros(tl.vocab, np.uint8)
    dims = (tl.hidden, tl.vocab, W.cp.vocab, tl.n_layer, tl.n_kv_head * tl.head_dim)
    r = rf.frame(small_navi, dims, rf.RefSampling(), 7, 0, seen, trailing.numpy(), hidden=hidden.numpy(), logits=logits.numpy())
    assert r.ok
    check_frame(W, r, None, 0, None, trailing.numpy(), seen, 7, 0, hidden=hidden.numpy(), logits=logits.numpy())


def test_oracle_reproduces_reference_golden(small_navi):
    """The committed reference outputs (no reference tree needed)."""
    g = np.load(os.path.join(GOLDEN, "ref_frame_small.npz"))
    W = om.Weights.from_navi(small_navi)
    tl = W.tl
    n_past = int(g["n_past"])
    kv, step, trailing, seen = _frame_inputs(W, n_past, seed=int(g["input_seed"]))
    r = rf.RefFrame(True, g["codes"].tolist(), 0, 0, g["hidden"], g["logits"], g["clogits"], g["step_out"], g["seen"],
                    list(g["k_rows"]), list(g["v_rows"]))
    check_frame(W, r, kv, n_past, step, trailing.numpy(), seen, int(g["seed"]), int(g["frame_index"]))
    s = om.Sampling(rng=0)
    for i in range(len(g["draw_ids"])):
        cb, fi, seed, temp, k = (int(g["draw_meta"][i][j]) for j in range(5))
        os_ = om.Sampling(temperature=temp / 1000, top_k=k, top_p=1.0, cp_temperature=temp / 1000, cp_top_k=k, cp_top_p=1.0, rng=0)
        x = g["draw_logits"][i][: (tl.vocab if cb == 0 else W.cp.vocab)]
        mods = (tl.vocab - 1024, W.cfg.codec_eos_id, g["draw_seen"][i]) if cb == 0 else None
        assert om.sample(x, cb, os_, seed, fi, talker_mods=mods, exp_libm=True) == int(g["draw_ids"][i]), i
    L = om.sampler_lib()
    for seed, fi, ts, cs in g["seeds"].tolist():
        assert L.oracle_draw_seed(int(seed), int(fi), 0) == int(ts)
        assert L.oracle_draw_seed(int(seed), int(fi), 4) == (int(cs) + 4 * 0xD1B54A32D192ED03) % 2**64
