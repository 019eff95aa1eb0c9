"""The vocoder oracle (oracle/vocoder.py) against the reference engine's own vocoder, on the CPU.

oracle/_ref/ref_vocoder_check is the reference's model/qwen3tts/vocoder.hip + kernels.h
(its kernel launches rewritten for the host emulator by oracle/hip_to_host.py) compiled
against the host stand-in for the HIP runtime (oracle/hipsim), and used as the reference's
tests/test_vocoder.cpp uses it: DeviceWeights::upload of the decoder tensors it does not own,
Vocoder::create, decode. Its stage hook (vocoder.hip:181-185) gives every intermediate of
decode_chunk (vocoder.hip:261-343), so the oracle's stage graph -- RVQ, pre_conv, the
sliding-window transformer, the ConvNeXt upsamplers, the decoder blocks with SnakeBeta
residual units, the output conv and clamp -- is checked stage by stage against the
reference's own, and chunked decoding against the reference's chunking. Float results
differ only by the host's expf / sinf in place of the GPU's __expf / __sinf (tolerance
rel-L2 1e-5; observed about 1e-7). tests/golden/ref_vocoder_small.npz holds the reference's
PCM so the end-to-end check also runs where the reference tree is absent.
"""
import os

import numpy as np
import pytest

from oracle import model as om
from oracle import ref_frame as rf
from oracle import vocoder as ov

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
needs_ref = pytest.mark.skipif(not rf.vocoder_available(), reason="oracle/_ref/ref_vocoder_check is built by build() from the reference tree")

# reference stage name -> the oracle's name for the same activation
STAGES = {"rvq": "rvq", "pre_conv": "pre_conv", "layer0": "layer0", "layer1": "layer1", "pre_transformer": "pre_transformer",
          "up0_cnx": "up0", "up1_cnx": "up1", "dec0": "dec0", "dec1_b4": "dec1", "dec2_b4": "dec2", "dec3_b4": "dec3",
          "dec4_b4": "dec4"}


def codes_of(W, n, seed):
    return np.random.default_rng(seed).integers(0, W.cfg.vq_codebook_size, (n, W.cfg.vq_n_q)).astype(np.int32)


@needs_ref
def test_vocoder_stages_match_reference_code(small_navi):
    W = om.Weights.from_navi(small_navi)
    codes = codes_of(W, 6, 1)
    pcm, got = rf.vocoder_decode(small_navi, codes, max_chunk=8, stages=True)
    want = {}
    ref = ov.Vocoder(W).decode_chunk(codes, want).numpy()
    for rname, oname in STAGES.items():
        assert got[rname].shape == tuple(want[oname].shape), rname
        assert om.rel_l2(got[rname], want[oname].numpy()) < 1e-5, (rname, om.rel_l2(got[rname], want[oname].numpy()))
    assert pcm.shape == ref.shape == (6 * W.cfg.samples_per_frame,)
    assert om.rel_l2(pcm, ref) < 1e-5, om.rel_l2(pcm, ref)
    assert np.abs(pcm).max() <= 1.0


@needs_ref
def test_vocoder_chunking_matches_reference_code(small_navi):
    """7 frames in chunks of 3 (3 + 3 + 1): conv histories, the ConvNeXt depthwise history and
    the attention window carried across chunks, as the reference carries them."""
    W = om.Weights.from_navi(small_navi)
    codes = codes_of(W, 7, 2)
    pcm, _ = rf.vocoder_decode(small_navi, codes, max_chunk=3)
    ref = ov.Vocoder(W).decode(codes, 7, 3).numpy()
    assert om.rel_l2(pcm, ref) < 1e-5, om.rel_l2(pcm, ref)


def test_vocoder_oracle_reproduces_reference_golden(small_navi):
    g = np.load(os.path.join(GOLDEN, "ref_vocoder_small.npz"))
    W = om.Weights.from_navi(small_navi)
    ref = ov.Vocoder(W).decode(g["codes"], len(g["codes"]), int(g["max_chunk"])).numpy()
    assert om.rel_l2(g["pcm"], ref) < 1e-5, om.rel_l2(g["pcm"], ref)
