"""Pins of the vocoder oracle (oracle/vocoder.py) against independent torch formulations,
on the CPU: the causal transposed-conv phase form against torch's ConvTranspose1d, the
causal conv with history against a left-padded Conv1d, the sliding-window attention
against dense masked attention, and chunked decoding against one-shot decoding."""
import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import model as om
from oracle import vocoder as ov


@pytest.fixture(scope="module")
def W(small_navi):
    return om.Weights.from_navi(small_navi)


def test_transposed_phases_equal_conv_transpose1d():
    """out[i s + p] = b + sum_m x[i - m] W[:, :, p + m s] (vocoder.hip:373-385) is
    ConvTranspose1d(stride s, k = 2 s) with the (k - s) trailing samples trimmed."""
    g = torch.Generator().manual_seed(0)
    for s, kk in ((2, 1), (5, 2), (8, 2), (3, 2)):
        Cin, Cout, T = 12, 10, 9
        w = torch.randn(Cin, Cout, kk * s, generator=g)
        b = torch.randn(Cout, generator=g)
        x = torch.randn(T, Cin, generator=g)
        v = ov.Vocoder.__new__(ov.Vocoder)
        v.hist = {}
        got = v.trans_conv("t", x, w, b, s)
        ref = F.conv_transpose1d(x.T.unsqueeze(0), w, b, stride=s)[0].T[:T * s]
        assert torch.allclose(got, ref, atol=1e-5, rtol=1e-5)


def test_causal_conv_with_history_equals_padded_conv():
    """Chunks with carried history reproduce one causal (left zero-padded) Conv1d."""
    g = torch.Generator().manual_seed(1)
    for K, dil in ((7, 1), (7, 3), (7, 9), (3, 1), (1, 1)):
        Cin, Cout, T = 6, 5, 40
        w = torch.randn(Cout, Cin, K, generator=g)
        b = torch.randn(Cout, generator=g)
        x = torch.randn(T, Cin, generator=g)
        ref = F.conv1d(F.pad(x.T.unsqueeze(0), ((K - 1) * dil, 0)), w, b, dilation=dil)[0].T
        v = ov.Vocoder.__new__(ov.Vocoder)
        v.hist = {}
        parts = [v.conv("c", x[a:b2], w, b, dil) for a, b2 in ((0, 3), (3, 4), (4, 25), (25, 40))]
        assert torch.allclose(torch.cat(parts), ref, atol=1e-5, rtol=1e-5)


def test_sliding_window_attention_equals_dense_masked(W):
    """The pre-transformer attention over keys (pos - window, pos] equals dense attention
    with the band mask, across chunk boundaries."""
    c = W.cfg
    v = ov.Vocoder(W)
    T = 3 * c.sliding_window
    x = torch.randn(T, c.vocoder.hidden, generator=torch.Generator().manual_seed(2))
    outs = []
    for a in range(0, T, 5):
        outs.append(v.attention_layer(0, x[a:a + 5]))
        v.pos0 += min(5, T - a)
    got = torch.cat(outs)
    # dense restatement
    p = f"{ov.DEC}pre_transformer.layers.0."
    nh, hd = c.vocoder.n_head, c.vocoder.head_dim
    n = om.rmsnorm(x, W[p + "input_layernorm.weight"], c.vocoder.eps)
    q = (n @ W[p + "self_attn.q_proj.weight"].T).view(T, nh, hd)
    k = (n @ W[p + "self_attn.k_proj.weight"].T).view(T, nh, hd)
    val = (n @ W[p + "self_attn.v_proj.weight"].T).view(T, nh, hd)
    inv = om.rope_inv_freq(hd, c.vocoder.rope_theta)
    q = torch.stack([om.rope(q[t], t, inv) for t in range(T)])
    k = torch.stack([om.rope(k[t], t, inv) for t in range(T)])
    i = torch.arange(T)
    mask = (i[None, :] <= i[:, None]) & (i[None, :] > i[:, None] - c.sliding_window)
    s = torch.einsum("thd,shd->hts", q, k) / math.sqrt(hd)
    s = s.masked_fill(~mask, float("-inf"))
    att = torch.einsum("hts,shd->thd", torch.softmax(s, -1), val).reshape(T, -1)
    y = x + (att @ W[p + "self_attn.o_proj.weight"].T) * W[p + "self_attn_layer_scale.scale"]
    n2 = om.rmsnorm(y, W[p + "post_attention_layernorm.weight"], c.vocoder.eps)
    a = om.silu(n2 @ W[p + "mlp.gate_proj.weight"].T) * (n2 @ W[p + "mlp.up_proj.weight"].T)
    ref = y + (a @ W[p + "mlp.down_proj.weight"].T) * W[p + "mlp_layer_scale.scale"]
    assert om.rel_l2(got.numpy(), ref.numpy()) < 1e-5


def test_chunked_decoding_equals_one_shot(W):
    c = W.cfg
    codes = torch.from_numpy(np.random.default_rng(3).integers(0, c.vq_codebook_size, (11, c.vq_n_q)))
    v = ov.Vocoder(W)
    one = v.decode(codes, 11, 11)
    v.reset()
    chunked = v.decode(codes, 11, 3)
    assert one.shape == (11 * c.samples_per_frame,)
    assert (one - chunked).abs().max() <= 1e-6
    assert one.abs().max() <= 1.0
