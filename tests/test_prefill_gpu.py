"""The talker prompt and prefill (reference model/qwen3tts/talker.hip:283-399) on the GPU
against the CPU oracle, through the C ABI: prompt rows, trailing rows and tts_pad; the last
row's post-norm hidden and codec logits; every KV row the prefill writes. Then the first
frames decode from the talker's own cache and outputs.

Tolerance: rel-L2 2e-4 on hidden / logits / prompt rows (the north star's gate is 1e-2), 1e-3
on the f16 KV rows (one f16 rounding each)."""
import numpy as np
import pytest
import torch

from navi_b200 import engine
from oracle import model as om

pytestmark = pytest.mark.gpu

REL = 2e-4


def _ids(cfg, n_text, seed):
    rng = np.random.default_rng(seed)
    head = [cfg.im_start_id, cfg.assistant_id, 198 % cfg.text_vocab]
    text = rng.integers(0, cfg.text_vocab, n_text).tolist()
    tail = [cfg.im_end_id, 198 % cfg.text_vocab, cfg.im_start_id, cfg.assistant_id, 198 % cfg.text_vocab]
    return head + text + tail


def _to_numpy(ptr, n):
    torch.cuda.synchronize()
    t = torch.empty(n, dtype=torch.float32, device="cuda")
    _copy(t.data_ptr(), ptr, n * 4)
    return t.cpu().numpy()


def _copy(dst, src, nbytes):
    import ctypes
    if _copy.lib is None:
        _copy.lib = ctypes.CDLL("libcudart.so.12")
    lib = _copy.lib
    lib.cudaMemcpy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]
    assert lib.cudaMemcpy(ctypes.c_void_p(dst), ctypes.c_void_p(src), nbytes, 3) == 0   # device to device


_copy.lib = None


def _check_prompt(W, tal, ids, language, spk):
    H = W.tl.hidden
    pr = tal.build_prompt(ids, language, spk)
    pre_o, trail_o, pad_o = om.build_prompt(W, ids, language, torch.from_numpy(spk))
    assert pr.n_prefill == pre_o.shape[0] and pr.n_trailing == trail_o.shape[0]
    pre = _to_numpy(pr.prefill, pr.n_prefill * H).reshape(-1, H)
    trail = _to_numpy(pr.trailing, pr.n_trailing * H).reshape(-1, H)
    pad = _to_numpy(pr.tts_pad, H)
    assert om.rel_l2(pre, pre_o) < REL, om.rel_l2(pre, pre_o)
    assert om.rel_l2(trail, trail_o) < REL, om.rel_l2(trail, trail_o)
    assert om.rel_l2(pad, pad_o) < REL
    return pr, pre_o


def _check_prefill(W, tal, pr, pre_o):
    H, L = W.tl.hidden, W.tl.n_layer
    kvd = W.tl.n_kv_head * W.tl.head_dim
    T = pr.n_prefill
    kv_o = [(torch.zeros(T, kvd), torch.zeros(T, kvd)) for _ in range(L)]
    hid_o, lg_o = om.prefill(W, pre_o, kv_o)
    tal.prefill(pr)
    hid = _to_numpy(tal.d_hidden(), H)
    lg = _to_numpy(tal.d_logits(), W.tl.vocab)
    assert om.rel_l2(hid, hid_o) < REL, om.rel_l2(hid, hid_o)
    assert om.rel_l2(lg, lg_o) < REL, om.rel_l2(lg, lg_o)
    kv = tal.kv()
    assert kv.n_used == T
    import ctypes
    tk = torch.empty(T * kvd, dtype=torch.float16, device="cuda")
    for l in range(L):
        _copy(tk.data_ptr(), ctypes.cast(kv.s.k[l], ctypes.c_void_p).value, T * kvd * 2)
        k = tk.cpu().numpy().copy()
        _copy(tk.data_ptr(), ctypes.cast(kv.s.v[l], ctypes.c_void_p).value, T * kvd * 2)
        v = tk.cpu().numpy().copy()
        assert om.rel_l2(k.astype(np.float32), kv_o[l][0].reshape(-1)) < 1e-3, (l, "k")
        assert om.rel_l2(v.astype(np.float32), kv_o[l][1].reshape(-1)) < 1e-3, (l, "v")
    return hid, lg


@pytest.mark.parametrize("language", ["english", "auto"])
def test_small_prompt_and_prefill(small_navi, language):
    W = om.Weights.from_navi(small_navi)
    dev = engine.Device(0)
    w = engine.Weights(dev, small_navi)
    tal = engine.Talker(dev, w, max_prompt_tokens=256, max_positions=512)
    ids = _ids(W.cfg, 23, seed=4)
    spk = np.random.default_rng(5).standard_normal(W.tl.hidden).astype(np.float32)
    pr, pre_o = _check_prompt(W, tal, ids, language, spk)
    _check_prefill(W, tal, pr, pre_o)


def test_small_prefill_then_frames(small_navi):
    """Frame 0 from the talker's hidden and logits, frames 1.. from its KV cache (the loop of
    Graph::synth, graph.cpp:78-92)."""
    W = om.Weights.from_navi(small_navi)
    dev = engine.Device(0)
    w = engine.Weights(dev, small_navi)
    tal = engine.Talker(dev, w, max_prompt_tokens=256, max_positions=512)
    frame = engine.Frame(dev, w)
    ids = _ids(W.cfg, 12, seed=9)
    spk = np.random.default_rng(1).standard_normal(W.tl.hidden).astype(np.float32)
    pr = tal.build_prompt(ids, "english", spk)
    tal.prefill(pr)
    kv = tal.kv()
    frame.reset()
    H = W.tl.hidden
    r = frame.run_first(tal.d_hidden(), tal.d_logits(), pr.trailing, engine.Sampling(), 7, 0)
    assert r.ok, r.error
    for i in range(1, 6):
        trailing = pr.trailing + 4 * H * i if i < pr.n_trailing else pr.tts_pad
        r = frame.run(kv, pr.n_prefill + i - 1, trailing, engine.Sampling(), 7, i)
        assert r.ok, r.error
        assert kv.n_used == pr.n_prefill + i


@pytest.mark.parametrize("n_text", [40, 200])
def test_full_size_prompt_and_prefill(full_navi, n_text):
    """configs[4]'s talker: full-size weights (text vocabulary 151936 x 2048), a 40-token text
    and configs[4]'s 200-token text (208 prefill rows)."""
    W = om.Weights.from_navi(full_navi)
    dev = engine.Device(0)
    w = engine.Weights(dev, full_navi)
    tal = engine.Talker(dev, w, max_prompt_tokens=256, max_positions=2048)
    ids = _ids(W.cfg, n_text, seed=2)
    spk = (np.random.default_rng(3).standard_normal(W.tl.hidden) * 0.05).astype(np.float32)
    pr, pre_o = _check_prompt(W, tal, ids, "english", spk)
    _check_prefill(W, tal, pr, pre_o)


@pytest.mark.parametrize("T", [208, 1100])
def test_full_size_long_prefill(full_navi, T):
    """The 28-layer prefill over T arbitrary rows (T = 208: the row count of configs[4]'s
    200-token prompt if it were prefilled whole; T = 1100: past the 1024 keys the reference's
    prefill attention holds, talker.hip:86): last row's hidden and logits, every layer's T K/V
    rows, against the oracle. The rows go in through navi_talker_prefill's prompt pointer."""
    import ctypes
    from navi_b200 import capi
    W = om.Weights.from_navi(full_navi)
    dev = engine.Device(0)
    w = engine.Weights(dev, full_navi)
    tal = engine.Talker(dev, w, max_prompt_tokens=T, max_positions=T + 16)
    rows = torch.randn(T, W.tl.hidden, generator=torch.Generator().manual_seed(T)) * 0.5
    d_rows = rows.cuda()
    pr = capi.Prompt(d_rows.data_ptr(), d_rows.data_ptr(), d_rows.data_ptr(), T, 0)
    _check_prefill(W, tal, pr, rows)
