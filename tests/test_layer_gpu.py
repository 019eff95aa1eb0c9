"""one talker decoder layer, one decode step at batch 1, through the C ABI
(navi_frame_run_layer) against the CPU oracle's decoder layer (the reference's layer phases,
model/qwen3tts/frame.hip:300-402): hidden 1024, 16 / 8 heads x 128, SwiGLU 3072, q/k
RMSNorm, RoPE theta 1e6, GQA over a KV cache of 256 positions. Weights f16 N(0, 0.02) from
seed 0 (norm weights 1 + N(0, 0.02)); input hidden N(0, 1) f32; cache N(0, 1) f16.

Tolerance: rel-L2 2e-4 on the layer output (the north star's gate is 1e-2), 1e-3 on the new
f16 K/V row (one f16 rounding); the cached rows must be left untouched."""
import numpy as np
import pytest
import torch

from frame_harness import Setup
from navi_b200 import capi
from oracle import model as om

pytestmark = pytest.mark.gpu

REL = 2e-4


@pytest.mark.parametrize("n_past", [256, 0, 1, 37, 1000])
def test_single_layer_matches_oracle(layer_navi, n_past):
    S = Setup(layer_navi, max_pos=1024)
    S.fill_kv(n_past, seed=11)
    before = [(S.k[0][:n_past].clone(), S.v[0][:n_past].clone())]
    kc, vc = S.oracle_kv()[0]
    x = torch.randn(S.H, generator=torch.Generator().manual_seed(n_past + 1))
    xd, out = x.cuda(), torch.zeros(S.H, device="cuda")
    r = S.frame.run_layer(0, xd.data_ptr(), S.kv, n_past, out.data_ptr())
    assert r.ok, r.error
    want = om.decoder_layer(S.W, "talker", 0, x.reshape(1, -1), kc, vc, n_past)[0]
    got = out.cpu()
    assert om.rel_l2(got, want) < REL, om.rel_l2(got, want)
    assert om.rel_l2(S.k[0][n_past].float().cpu(), kc[n_past]) < 1e-3
    assert om.rel_l2(S.v[0][n_past].float().cpu(), vc[n_past]) < 1e-3
    assert torch.equal(S.k[0][:n_past], before[0][0]) and torch.equal(S.v[0][:n_past], before[0][1])
    # a second step at the next position reads the row this one wrote
    r = S.frame.run_layer(0, out.data_ptr(), S.kv, n_past + 1, xd.data_ptr())
    assert r.ok, r.error
    want2 = om.decoder_layer(S.W, "talker", 0, want.reshape(1, -1), kc, vc, n_past + 1)[0]
    assert om.rel_l2(xd.cpu(), want2) < REL


def test_layer_step_rejects_bad_arguments(layer_navi):
    S = Setup(layer_navi, max_pos=64)
    x, out = torch.zeros(S.H, device="cuda"), torch.zeros(S.H, device="cuda")
    r = S.frame.run_layer(1, x.data_ptr(), S.kv, 3, out.data_ptr())
    assert not r.ok and r.status == capi.NAVI_E_ARG
    r = S.frame.run_layer(0, x.data_ptr(), S.kv, 64, out.data_ptr())
    assert not r.ok and r.status == capi.NAVI_E_KV_FULL
