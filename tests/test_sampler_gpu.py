"""The device sampler against the C oracle, bit for bit, on the same logits.

Covers the reference's sampling semantics (model/qwen3tts/frame.hip:413-500) and
this build's additions: greedy with ties and all -inf, exact top-k with ties at the
threshold, top-p boundaries, temperature, codebook-0 suppression / EOS gating /
repetition penalty, both RNG streams, and the vocab sizes of the benchmark configs.
The value kinds also drive each path of the device's top-k selection: the distance
histogram with one bin to resolve (normal, peaked), the radix select for a crowded bin
(ties, flat) or a k-th value beyond the bins (wide, neginf), and top-p orders over more
than 64 candidates (top-k 200 or off).
"""
import numpy as np
import pytest
import torch

from navi_b200 import capi, engine
from oracle import model as om

pytestmark = pytest.mark.gpu


def _cases():
    rng = np.random.default_rng(5)
    out = []
    for V in (3072, 2048, 1536, 512):
        for kind in ("normal", "ties", "neginf", "peaked", "wide", "flat"):
            x = rng.standard_normal(V).astype(np.float32) * 3
            if kind == "ties":
                x = np.round(x)                       # many exact ties, including at the top-k threshold
            elif kind == "neginf":
                x[rng.random(V) < 0.7] = -np.inf
            elif kind == "peaked":
                x[rng.integers(V)] += 40.0            # one dominant id: most e_i underflow to 0
            elif kind == "wide":
                x *= 12.0                             # the k-th largest lies beyond the distance bins
            elif kind == "flat":
                x = np.full(V, 0.25, np.float32)      # every value in one bin and tied
                x[rng.integers(V, size=5)] = 1.5
            for temp, k, p in ((0.9, 50, 1.0), (0.9, 50, 0.9), (1.3, 0, 0.5), (0.7, 1, 1.0), (0.9, V, 0.01),
                               (0.0, 50, 1.0), (1.0, 7, 0.999), (0.8, 200, 0.95)):
                for rs in (capi.NAVI_RNG_PCG, capi.NAVI_RNG_PHILOX):
                    out.append((V, kind, temp, k, p, rs, int(rng.integers(1 << 62)), int(rng.integers(200)), x))
    return out


CASES = _cases()


@pytest.fixture(scope="module")
def dev():
    return engine.Device(0)


@pytest.mark.parametrize("i", range(len(CASES)))
def test_code_predictor_draw_bit_exact(dev, i):
    V, kind, temp, k, p, rs, seed, fi, x = CASES[i]
    s = engine.Sampling(cp_temperature=temp, cp_top_k=k, cp_top_p=p, rng=rs)
    d = torch.from_numpy(x).cuda()
    cb = 1 + i % 15
    got = engine.sample_logits(dev, d.data_ptr(), V, s, seed, fi, cb)
    want = om.sample(x, cb, om.Sampling(cp_temperature=temp, cp_top_k=k, cp_top_p=p, rng=rs), seed, fi)
    assert got == want, (kind, V, temp, k, p, rs, got, want)


@pytest.mark.parametrize("fi", [0, 1, 2, 9])
@pytest.mark.parametrize("rs", [capi.NAVI_RNG_PCG, capi.NAVI_RNG_PHILOX])
def test_codebook0_draw_with_modifications(dev, fi, rs):
    V, eos = 3072, 2050
    rng = np.random.default_rng(fi + 10 * rs)
    for trial in range(12):
        x = (rng.standard_normal(V) * 4).astype(np.float32)
        x[eos] = 30.0 if trial % 3 == 0 else x[eos]          # EOS wins only once min_frames has passed
        seen = (rng.random(V) < 0.05).astype(np.uint8)
        temp = [0.0, 0.9, 1.1][trial % 3]
        s = engine.Sampling(temperature=temp, top_k=50, top_p=[1.0, 0.9][trial % 2], repetition_penalty=1.05,
                            min_frames=2, rng=rs)
        d, sd = torch.from_numpy(x).cuda(), torch.from_numpy(seen).cuda()
        seed = int(rng.integers(1 << 62))
        got = engine.sample_logits(dev, d.data_ptr(), V, s, seed, fi, 0, V - 1024, eos, sd.data_ptr())
        want = om.sample(x, 0, om.Sampling(temperature=temp, top_k=50, top_p=s.top_p, repetition_penalty=1.05,
                                           min_frames=2, rng=rs), seed, fi, talker_mods=(V - 1024, eos, seen))
        assert got == want, (trial, got, want)
        if fi < 2:
            assert got != eos
        assert got < V - 1024 or got == eos


def test_device_draws_match_golden_fixture(dev):
    """The device sampler returns the committed ids of tests/golden/sampler_golden.json (the
    sampler specification's draws, fixed when the fixture was written)."""
    import json
    import os
    import sys
    golden = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
    sys.path.insert(0, golden)
    from make_golden import case_logits, case_seen
    with open(os.path.join(golden, "sampler_golden.json")) as f:
        cases = json.load(f)["cases"]
    for c in cases:
        V, cb = c["V"], c["codebook"]
        s = engine.Sampling(temperature=c["temperature"], top_k=c["top_k"], top_p=c["top_p"], cp_temperature=c["temperature"],
                            cp_top_k=c["top_k"], cp_top_p=c["top_p"], rng=c["rng"])
        d = torch.from_numpy(case_logits(c)).cuda()
        if cb == 0:
            sd = torch.from_numpy(case_seen(c)).cuda()
            got = engine.sample_logits(dev, d.data_ptr(), V, s, c["seed"], c["frame_index"], 0, V - 1024, V - 1022, sd.data_ptr())
        else:
            got = engine.sample_logits(dev, d.data_ptr(), V, s, c["seed"], c["frame_index"], cb)
        assert got == c["id"], c
