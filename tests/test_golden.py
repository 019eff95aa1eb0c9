"""The committed golden fixtures (tests/golden/, written by tests/golden/make_golden.py).

- the reference's own .navi reader accepted the seeded small model and read these
  hyperparameters; this build's writer and reader must agree with it;
- transformers' Qwen3DecoderLayer outputs on seeded inputs; the oracle's decoder layer must
  reproduce them;
- the sampler specification's draws on seeded logits; the C oracle must reproduce them (the
  device sampler is held to the same ids in tests/test_sampler_gpu.py).
"""
import json
import os

import numpy as np
import pytest
import torch

from navi_b200 import model_spec
from navi_b200.navi_file import NaviFile
from oracle import model as om

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load(name):
    with open(os.path.join(GOLDEN, name)) as f:
        return json.load(f)


def test_navi_header_agrees_with_reference_reader(small_navi):
    ref = _load("navi_ref_small.json")
    assert ref["ok"] and ref["missing"] == 0 and ref["shape_mismatch"] == 0 and ref["unused"] == 0
    f = NaviFile.open(small_navi)
    c = model_spec.config_from_kv(f.kv)
    t, cp = c.talker, c.cp
    assert [t.hidden, t.n_layer, t.n_head, t.n_kv_head, t.head_dim, t.ff, t.vocab] == ref["talker"]
    assert [cp.hidden, cp.n_layer, cp.n_head, cp.n_kv_head, cp.head_dim, cp.ff, cp.vocab] == ref["cp"]
    assert c.codec_eos_id == ref["codec_eos"] and c.decoder_dim == ref["decoder_dim"]
    assert np.float32(t.eps) == np.float32(ref["rms_eps"]) and t.rope_theta == ref["rope_theta"]
    assert f.data_offset == ref["data_offset"] and len(f.tensors) == ref["n_tensors"]


@pytest.mark.parametrize("component", ["talker", "cp"])
def test_oracle_layer_reproduces_transformers_fixture(small_navi, component):
    g = np.load(os.path.join(GOLDEN, "decoder_layer_small.npz"))
    W = om.Weights.from_navi(small_navi)
    d = W.tl if component == "talker" else W.cp
    x = torch.from_numpy(g[f"{component}_x"])
    kv = d.n_kv_head * d.head_dim
    kc, vc = torch.zeros(16, kv), torch.zeros(16, kv)
    ours = om.decoder_layer(W, component, 1, x, kc, vc, 0, kv_round=False)
    assert om.rel_l2(ours, torch.from_numpy(g[f"{component}_y"])) < 2e-6


def test_oracle_sampler_reproduces_fixture():
    import sys
    sys.path.insert(0, GOLDEN)
    from make_golden import case_draw
    for c in _load("sampler_golden.json")["cases"]:
        assert case_draw(c) == c["id"], c
