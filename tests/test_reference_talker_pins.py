"""The talker prompt and prefill oracle (oracle.model.build_prompt / prefill) against the
reference engine's own talker.hip run on the host emulator, on the CPU.

oracle/_ref/ref_talker_check is the reference's model/qwen3tts/talker.hip + kernels.h (kernel
launches rewritten for the host by oracle/hip_to_host.py) on the host stand-in for the HIP
runtime (oracle/hipsim), used as the reference's Graph uses it: DeviceWeights::upload with
Talker::fused_groups, Talker::create, build_prompt (talker.hip:283-352), prefill (355-399).
Checked: the prefill, trailing and tts_pad rows (row layout of the prompt, text projection,
codec and speaker rows) within rel-L2 1e-6; the last row's post-norm hidden and codec logits
within 1e-4 and every KV row within 1e-4 (the reference forms RoPE angles with f32 powf /
sincosf, the oracle in double; observed about 7e-6 and 2e-5). The golden file
tests/golden/ref_talker_small.npz keeps the reference's outputs for where the tree is absent.
"""
import os

import numpy as np
import pytest
import torch

from oracle import model as om
from oracle import ref_frame as rf

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
needs_ref = pytest.mark.skipif(not rf.talker_available(), reason="oracle/_ref/ref_talker_check is built by build() from the reference tree")


def prompt_ids(c, n_text, seed):
    rng = np.random.default_rng(seed)
    nl = 198 % c.text_vocab
    return [c.im_start_id, c.assistant_id, nl] + rng.integers(0, c.text_vocab, n_text).tolist() + [c.im_end_id, nl, c.im_start_id,
                                                                                                  c.assistant_id, nl]


def check(W, ids, language, spk, ref):
    pre, trail, pad, hid, lg, kv = ref
    tl = W.tl
    pre_o, trail_o, pad_o = om.build_prompt(W, ids, language, torch.from_numpy(spk))
    assert pre.shape == tuple(pre_o.shape) and trail.shape == tuple(trail_o.shape)
    assert om.rel_l2(pre, pre_o) < 1e-6 and om.rel_l2(trail, trail_o) < 1e-6 and om.rel_l2(pad, pad_o) < 1e-6
    T, kvd = pre_o.shape[0], tl.n_kv_head * tl.head_dim
    kv_o = [(torch.zeros(T, kvd), torch.zeros(T, kvd)) for _ in range(tl.n_layer)]
    hid_o, lg_o = om.prefill(W, pre_o, kv_o)
    assert om.rel_l2(hid, hid_o) < 1e-4, om.rel_l2(hid, hid_o)
    assert om.rel_l2(lg, lg_o) < 1e-4, om.rel_l2(lg, lg_o)
    for l in range(tl.n_layer):
        assert om.rel_l2(kv[l][0].astype(np.float32), kv_o[l][0]) < 1e-4, (l, "k")
        assert om.rel_l2(kv[l][1].astype(np.float32), kv_o[l][1]) < 1e-4, (l, "v")


@needs_ref
@pytest.mark.parametrize("language,n_text", [("english", 23), ("auto", 5), ("german", 60)])
def test_prompt_and_prefill_match_reference_code(small_navi, language, n_text):
    W = om.Weights.from_navi(small_navi)
    tl = W.tl
    ids = prompt_ids(W.cfg, n_text, n_text)
    spk = np.random.default_rng(n_text + 1).standard_normal(tl.hidden).astype(np.float32)
    ref = rf.talker_prefill(small_navi, ids, language, spk, (tl.hidden, tl.vocab, tl.n_layer, tl.n_kv_head * tl.head_dim))
    check(W, ids, language, spk, ref)


def test_prefill_oracle_reproduces_reference_golden(small_navi):
    g = np.load(os.path.join(GOLDEN, "ref_talker_small.npz"))
    W = om.Weights.from_navi(small_navi)
    kv = [(g["k"][l], g["v"][l]) for l in range(W.tl.n_layer)]
    check(W, g["ids"].tolist(), str(g["language"]), g["speaker"], (g["prefill"], g["trailing"], g["tts_pad"], g["hidden"], g["logits"], kv))
