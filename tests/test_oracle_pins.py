"""Pins the CPU oracle before it is trusted as the checker.

- The decoder layer (q/k RMSNorm, rotate-half RoPE, GQA, SwiGLU, residuals) against
  transformers' Qwen3DecoderLayer, the layer the reference's PyTorch model builds
  its talker and code predictor from (qwen-tts 0.1.1 on transformers 4.57.3,
  tools/uv.lock:1935-1936, 2687-2688; transformers here is 5.5, whose Qwen3 layer
  computes the same function).
- The sampler's exact exp against double-precision exp (<= 1 ulp), and its RNG
  building blocks against published known answers: splitmix64 from seed 0,
  Philox4x32-10 (Random123 known-answer vectors), and PCG32 XSH-RR (the pcg32
  reference demo stream, seed 42 / sequence 54).
"""
import ctypes
import math

import numpy as np
import pytest
import torch

from oracle import model as om


def _qwen3_layer_reference(W, component, l, x, pos0):
    from transformers import Qwen3Config
    from transformers.models.qwen3.modeling_qwen3 import Qwen3DecoderLayer, Qwen3RotaryEmbedding
    d = W.tl if component == "talker" else W.cp
    cfg = Qwen3Config(hidden_size=d.hidden, intermediate_size=d.ff, num_attention_heads=d.n_head,
                      num_key_value_heads=d.n_kv_head, head_dim=d.head_dim, rms_norm_eps=d.eps,
                      rope_theta=d.rope_theta, num_hidden_layers=1, vocab_size=8, attention_bias=False,
                      max_position_embeddings=4096)
    cfg._attn_implementation = "eager"
    layer = Qwen3DecoderLayer(cfg, 0).eval()
    p = om.layer_prefix(component, l)
    sd = {k[len(p):]: v for k, v in W.t.items() if k.startswith(p)}
    layer.load_state_dict(sd)
    T = x.shape[0]
    rot = Qwen3RotaryEmbedding(cfg)
    pos = torch.arange(pos0, pos0 + T).unsqueeze(0)
    cos, sin = rot(x.unsqueeze(0), pos)
    mask = torch.full((T, T), float("-inf")).triu(1).view(1, 1, T, T)
    with torch.no_grad():
        return layer(x.unsqueeze(0), attention_mask=mask, position_ids=pos, position_embeddings=(cos, sin))[0]


@pytest.mark.parametrize("component", ["talker", "cp"])
def test_decoder_layer_matches_transformers_qwen3(small_navi, component):
    W = om.Weights.from_navi(small_navi)
    d = W.tl if component == "talker" else W.cp
    torch.manual_seed(0)
    x = torch.randn(5, d.hidden)
    kv = d.n_kv_head * d.head_dim
    kc, vc = torch.zeros(16, kv), torch.zeros(16, kv)
    ours = om.decoder_layer(W, component, 1, x, kc, vc, 0, kv_round=False)
    ref = _qwen3_layer_reference(W, component, 1, x, 0)
    assert om.rel_l2(ours, ref) < 2e-6, om.rel_l2(ours, ref)
    # one-row-at-a-time decode with a cache equals the causal prefill
    kc2, vc2 = torch.zeros(16, kv), torch.zeros(16, kv)
    rows = [om.decoder_layer(W, component, 1, x[t:t + 1], kc2, vc2, t, kv_round=False)[0] for t in range(5)]
    assert om.rel_l2(torch.stack(rows), ref) < 2e-6


def test_exact_exp_within_one_ulp():
    lib = om.sampler_lib()
    xs = np.concatenate([np.linspace(-103.9, 88.7, 40001), -np.abs(np.random.default_rng(1).standard_normal(20000)) * 30])
    worst = 0.0
    for x in xs.astype(np.float32):
        ref = math.exp(float(x))
        if ref < 1.1754944e-38:
            continue
        y = lib.oracle_exp(float(x))
        worst = max(worst, abs(y - ref) / float(np.spacing(np.float32(ref))))
    assert worst <= 1.0, worst
    assert lib.oracle_exp(-200.0) == 0.0 and lib.oracle_exp(float("-inf")) == 0.0 and lib.oracle_exp(0.0) == 1.0


def test_rng_known_answers():
    lib = om.sampler_lib()
    lib.oracle_splitmix64.restype = ctypes.c_uint64
    lib.oracle_splitmix64.argtypes = [ctypes.c_uint64]
    assert lib.oracle_splitmix64(0) == 0xE220A8397B1DCDAF
    lib.oracle_philox4x32_10.argtypes = [ctypes.POINTER(ctypes.c_uint32)] * 3

    def philox(c, k):
        C, K, O = (ctypes.c_uint32 * 4)(*c), (ctypes.c_uint32 * 2)(*k), (ctypes.c_uint32 * 4)()
        lib.oracle_philox4x32_10(C, K, O)
        return list(O)
    assert philox([0, 0, 0, 0], [0, 0]) == [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]
    assert philox([0xFFFFFFFF] * 4, [0xFFFFFFFF] * 2) == [0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]
    assert philox([0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344], [0xA4093822, 0x299F31D0]) == \
        [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]
    lib.oracle_pcg32_step.restype = ctypes.c_uint32
    lib.oracle_pcg32_step.argtypes = [ctypes.POINTER(ctypes.c_uint64), ctypes.c_uint64]
    st, inc = ctypes.c_uint64(0), (54 << 1) | 1
    lib.oracle_pcg32_step(ctypes.byref(st), inc)
    st.value = (st.value + 42) % 2**64
    lib.oracle_pcg32_step(ctypes.byref(st), inc)
    got = [lib.oracle_pcg32_step(ctypes.byref(st), inc) for _ in range(6)]
    assert got == [0xA15C02B7, 0x7B47F409, 0xBA1D3330, 0x83D2F293, 0xBFA4784B, 0xCBED606E]
