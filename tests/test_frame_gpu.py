"""Parity of the B200 frame path with the CPU oracle, through the C ABI.

Gates (the north star's): sampled codes bit-exact given identical logits (the
GPU's own logits fed to the oracle sampler); talker hidden / codec logits and
code-predictor logits within rel-L2 1e-2 of the fp32 oracle on the same weights
and inputs (observed ~1e-5); plus the reference's own frame gates
(tests/test_frame.cpp:50-123): run-to-run bit identity for a seed, a different
seed differs, and a device wait forced past its deadline fails the frame cleanly
without poisoning the next one.
"""
import numpy as np
import pytest
import torch

from navi_b200 import capi, engine
from oracle import model as om

from frame_harness import Setup, dev_f32, oracle_sampling

pytestmark = pytest.mark.gpu

REL_L2 = 1e-2      # the north star's gate for hidden states and logits
REL_L2_TIGHT = 2e-4


def _check_codes(S, codes, logits, clogits, s, seed, fi, seen):
    """Every code must be the oracle sampler's draw on the GPU's own logits."""
    cfg = S.W.cfg
    want0 = om.sample(logits, 0, oracle_sampling(s), seed, fi, talker_mods=(S.TV - 1024, cfg.codec_eos_id, seen))
    assert codes[0] == want0, (codes[0], want0)
    for k in range(1, 16):
        want = om.sample(clogits[k - 1], k, oracle_sampling(s), seed, fi)
        assert codes[k] == want, (k, codes[k], want)


@pytest.mark.parametrize("rng", [capi.NAVI_RNG_PCG, capi.NAVI_RNG_PHILOX])
def test_run_first_matches_oracle(small_navi, rng):
    S = Setup(small_navi)
    torch.manual_seed(1)
    hidden = torch.randn(S.H)
    logits = torch.randn(S.TV) * 3
    trailing = torch.randn(S.H)
    hd, ld, td = hidden.cuda(), logits.cuda(), trailing.cuda()
    s = engine.Sampling(top_p=0.9, cp_top_p=0.9, rng=rng)
    S.frame.reset()
    r = S.frame.run_first(hd.data_ptr(), ld.data_ptr(), td.data_ptr(), s, 7, 0)
    assert r.ok, r.error
    _, _, clg = S.frame.inspect()
    _check_codes(S, r.codes, logits.numpy(), clg, s, 7, 0, np.zeros(S.TV, np.uint8))
    # code-predictor logits, teacher-forced with the GPU's codes
    _, clo = om.code_predictor(S.W, hidden, r.codes[0], oracle_sampling(s), 7, 0, teacher_codes=r.codes)
    for k in range(15):
        assert om.rel_l2(clg[k], clo[k]) < REL_L2_TIGHT, (k, om.rel_l2(clg[k], clo[k]))
    # next step embedding
    want = om.step_embedding(S.W, r.codes, trailing)
    assert om.rel_l2(S.step_out(), want) < 1e-6


@pytest.mark.parametrize("n_past", [1, 40, 200])
def test_run_matches_oracle(small_navi, n_past):
    S = Setup(small_navi, max_pos=256)
    S.fill_kv(n_past, seed=n_past)
    kv_o = S.oracle_kv()
    torch.manual_seed(2)
    step_in = torch.randn(S.H)
    trailing = torch.randn(S.H)
    sd, td = step_in.cuda(), trailing.cuda()
    s = engine.Sampling(top_p=0.9, cp_top_p=0.9)
    S.frame.reset()
    S.frame.set_step_in(sd.data_ptr())
    r = S.frame.run(S.kv, n_past, td.data_ptr(), s, 11, 5)
    assert r.ok, r.error
    assert S.kv.n_used == n_past + 1
    hid, lg, clg = S.frame.inspect()
    hid_o, lg_o = om.talker_step(S.W, step_in, kv_o, n_past)
    assert om.rel_l2(hid, hid_o) < REL_L2_TIGHT, om.rel_l2(hid, hid_o)
    assert om.rel_l2(lg, lg_o) < REL_L2_TIGHT, om.rel_l2(lg, lg_o)
    # the new KV row of every layer (f16, post-RoPE K)
    for l in range(S.n_layer):
        assert om.rel_l2(S.k[l][n_past].float().cpu(), kv_o[l][0][n_past]) < 1e-3
        assert om.rel_l2(S.v[l][n_past].float().cpu(), kv_o[l][1][n_past]) < 1e-3
        assert torch.equal(S.k[l][:n_past].float().cpu(), kv_o[l][0][:n_past])   # older rows untouched
    _check_codes(S, r.codes, lg, clg, s, 11, 5, np.zeros(S.TV, np.uint8))
    _, clo = om.code_predictor(S.W, torch.from_numpy(hid), r.codes[0], oracle_sampling(s), 11, 5, teacher_codes=r.codes)
    for k in range(15):
        assert om.rel_l2(clg[k], clo[k]) < REL_L2_TIGHT
    assert om.rel_l2(S.step_out(), om.step_embedding(S.W, r.codes, trailing)) < 1e-6


def test_frame_loop_bit_identical_and_seeded(small_navi):
    """Frames chained on the device's own step embeddings: same seed twice is bit-identical,
    another seed differs, and the repetition set carries across frames (reference gates,
    tests/test_frame.cpp:72-96)."""
    S = Setup(small_navi, max_pos=128)
    torch.manual_seed(3)
    hidden, logits = torch.randn(S.H).cuda(), (torch.randn(S.TV) * 3).cuda()
    trailing = torch.randn(8, S.H).cuda()
    s = engine.Sampling()

    def run(seed):
        S.fill_kv(10, seed=99)
        S.frame.reset()
        out = []
        r = S.frame.run_first(hidden.data_ptr(), logits.data_ptr(), trailing[0].data_ptr(), s, seed, 0)
        assert r.ok, r.error
        out.append(r.codes)
        for i in range(1, 6):
            r = S.frame.run(S.kv, 10 + i - 1, trailing[i].data_ptr(), s, seed, i)
            assert r.ok, r.error
            out.append(r.codes)
        return out

    a, b, c = run(2), run(2), run(3)
    assert a == b
    assert a != c


def test_deadline_timeout_fails_cleanly(small_navi):
    """A 1 us deadline makes the first cross-CTA wait give up: the frame fails with
    NAVI_E_TIMEOUT, promptly, and a normal frame afterwards still works."""
    import time
    S = Setup(small_navi)
    tight = engine.Frame(S.dev, S.w, deadline_us=1)
    hidden, logits, trailing = torch.randn(S.H).cuda(), torch.randn(S.TV).cuda(), torch.randn(S.H).cuda()
    t0 = time.time()
    r = tight.run_first(hidden.data_ptr(), logits.data_ptr(), trailing.data_ptr(), engine.Sampling(), 0, 0)
    assert not r.ok and r.status == capi.NAVI_E_TIMEOUT, (r.ok, r.status, r.error)
    assert time.time() - t0 < 2.0
    tight.close()
    S.frame.reset()
    r = S.frame.run_first(hidden.data_ptr(), logits.data_ptr(), trailing.data_ptr(), engine.Sampling(), 0, 0)
    assert r.ok, r.error


def test_kv_full_is_reported(small_navi):
    S = Setup(small_navi, max_pos=16)
    trailing = torch.randn(S.H).cuda()
    r = S.frame.run(S.kv, 16, trailing.data_ptr(), engine.Sampling(), 0, 1)
    assert not r.ok and r.status == capi.NAVI_E_KV_FULL


@pytest.mark.parametrize("n_past", [64, 512, 2048])   # 2048: several 8-position steps per warp
def test_full_size_frame_matches_oracle(full_navi, n_past):
    """configs[1]+[2] shapes: 28-layer talker at KV length n_past, 5-layer code predictor."""
    S = Setup(full_navi, max_pos=2049)
    S.fill_kv(n_past, seed=7)
    kv_o = S.oracle_kv()
    torch.manual_seed(4)
    step_in, trailing = torch.randn(S.H), torch.randn(S.H)
    sd, td = step_in.cuda(), trailing.cuda()
    s = engine.Sampling(top_p=0.9, cp_top_p=0.9, rng=capi.NAVI_RNG_PHILOX)
    S.frame.reset()
    S.frame.set_step_in(sd.data_ptr())
    r = S.frame.run(S.kv, n_past, td.data_ptr(), s, 99, 3)
    assert r.ok, r.error
    hid, lg, clg = S.frame.inspect()
    hid_o, lg_o = om.talker_step(S.W, step_in, kv_o, n_past)
    assert om.rel_l2(hid, hid_o) < REL_L2_TIGHT, om.rel_l2(hid, hid_o)
    assert om.rel_l2(lg, lg_o) < REL_L2_TIGHT, om.rel_l2(lg, lg_o)
    _check_codes(S, r.codes, lg, clg, s, 99, 3, np.zeros(S.TV, np.uint8))
    _, clo = om.code_predictor(S.W, torch.from_numpy(hid), r.codes[0], oracle_sampling(s), 99, 3, teacher_codes=r.codes)
    worst = max(om.rel_l2(clg[k], clo[k]) for k in range(15))
    assert worst < REL_L2_TIGHT, worst
    assert om.rel_l2(S.step_out(), om.step_embedding(S.W, r.codes, trailing)) < 1e-6
