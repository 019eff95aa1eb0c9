"""navi_sample_logits_static (the sampler entry point that allocates nothing) against
navi_sample_logits on the same device logits, through the C ABI.

Each case makes two calls in a row of the static entry point, so the second one runs on
scratch left over from the first; both must return the id navi_sample_logits returns
(sampled ids are integers: the tolerance is equality).  Above the vocabulary the allocating
entry point stages in shared memory, the static one is checked against the C oracle
sampler instead, bit for bit.  The file name sorts last so the module also runs after every
other test in one process; it passes on its own as well.
"""
import numpy as np
import pytest
import torch

from navi_b200 import capi, engine
from oracle import model as om

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    d = engine.Device(0)
    yield d
    d.close()


def _cases():
    out = []
    for rng in (capi.NAVI_RNG_PCG, capi.NAVI_RNG_PHILOX):
        for cb, V in ((0, 3072), (3, 2048), (15, 2048)):
            for top_p in (1.0, 0.9):
                out.append((rng, cb, V, top_p))
    return out


@pytest.mark.parametrize("rng,codebook,vocab,top_p", _cases())
def test_static_matches_allocating_sampler(dev, rng, codebook, vocab, top_p):
    g = torch.Generator().manual_seed(1000 * codebook + vocab + int(top_p * 10) + rng)
    logits = (torch.randn(vocab, generator=g) * 3).cuda()
    seen = torch.zeros(vocab, dtype=torch.uint8)
    seen[torch.randint(0, vocab, (40,), generator=g)] = 1
    seen = seen.cuda()
    s = engine.Sampling(top_p=top_p, cp_top_p=top_p, rng=rng)
    for seed, fi in ((5, 3), (6, 4)):
        args = (logits.data_ptr(), vocab, s, seed, fi, codebook)
        kw = dict(suppress_from=vocab - 1024, eos_id=vocab - 1022, d_seen=seen.data_ptr()) if codebook == 0 else {}
        want = engine.sample_logits(dev, *args, **kw)
        got1 = engine.sample_logits_static(dev, *args, **kw)
        got2 = engine.sample_logits_static(dev, *args, **kw)
        assert got1 == want and got2 == want, (got1, got2, want)


def test_static_greedy_and_max_vocab(dev):
    """Greedy draw at the largest vocabulary the scratch holds (beyond what the allocating
    entry point's shared-memory staging takes): the argmax, lowest index on ties."""
    V = capi.NAVI_SAMPLE_STATIC_MAX_VOCAB
    x = np.random.default_rng(7).standard_normal(V).astype(np.float32)
    x[[123, 30000]] = 50.0
    d = torch.from_numpy(x).cuda()
    s = engine.Sampling(temperature=0.0, cp_temperature=0.0)
    assert engine.sample_logits_static(dev, d.data_ptr(), V, s, 1, 0, 2) == 123
    assert engine.sample_logits_static(dev, d.data_ptr(), V, s, 1, 0, 2) == 123


def test_static_rejects_vocab_beyond_limit(dev):
    V = capi.NAVI_SAMPLE_STATIC_MAX_VOCAB + 1
    d = torch.zeros(V, device="cuda")
    with pytest.raises(capi.NaviError) as e:
        engine.sample_logits_static(dev, d.data_ptr(), V, engine.Sampling(), 1, 0, 1)
    assert e.value.status == capi.NAVI_E_ARG
    assert "32768" in str(e.value)


@pytest.mark.parametrize("vocab", [20011, capi.NAVI_SAMPLE_STATIC_MAX_VOCAB])
@pytest.mark.parametrize("rng", [capi.NAVI_RNG_PCG, capi.NAVI_RNG_PHILOX])
def test_static_sampled_at_large_vocab_matches_oracle(dev, vocab, rng):
    """Top-k 50 / top-p 0.9 / T 0.9 draws (the radix select over global scratch) at a
    vocabulary near 20,000 and at the limit, against the C oracle on the same logits; two
    calls in a row each time, and no device memory taken by either."""
    x = (np.random.default_rng(vocab + rng).standard_normal(vocab) * 3).astype(np.float32)
    d = torch.from_numpy(x).cuda()
    s = engine.Sampling(cp_temperature=0.9, cp_top_k=50, cp_top_p=0.9, rng=rng)
    os_ = om.Sampling(cp_temperature=0.9, cp_top_k=50, cp_top_p=0.9, rng=rng)
    engine.sample_logits_static(dev, d.data_ptr(), vocab, s, 1, 0, 1)   # set-up call (symbol address)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for seed, fi, cb in ((11, 0, 1), (12, 7, 9), (13, 199, 15)):
        want = om.sample(x, cb, os_, seed, fi)
        got1 = engine.sample_logits_static(dev, d.data_ptr(), vocab, s, seed, fi, cb)
        got2 = engine.sample_logits_static(dev, d.data_ptr(), vocab, s, seed, fi, cb)
        assert got1 == want and got2 == want, (vocab, rng, seed, got1, got2, want)
    assert torch.cuda.mem_get_info()[0] == free0
