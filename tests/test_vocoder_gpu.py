"""The vocoder on the GPU (reference: model/qwen3tts/vocoder.hip, kernels.h:72-242).

1. The implicit-GEMM conv primitive (navi_conv1d) against a float64 torch evaluation of
   the same sum, over the shapes and options the decoder uses and their edges: taps 1/2/3/7,
   dilation 1/3/9, history rows, transposed-conv phases, Snake / SiLU-gate prologues,
   GELU / residual / scaled-residual epilogues, channel counts that are not multiples of
   the 128 x 64 tile, row counts that are not multiples of the row tile, split-K shapes.
   Tolerance rel-L2 1e-5: activations enter the tensor cores as f16 hi + lo halves
   (about 22 bits), weights are exact f16, accumulation f32.
2. The whole decoder against the CPU oracle (oracle/vocoder.py) stage by stage, small and
   benchmark-size models. Tolerance rel-L2 1e-3 per stage and on the PCM (the north star's
   gate for hidden states is 1e-2).
3. Chunked decoding equals one-shot decoding (max |diff| <= 1e-5, the reference's own
   gate, test_vocoder.cpp:104-107), state carries across calls, reset() restarts.
"""
import numpy as np
import pytest
import torch

from navi_b200 import capi, engine
from oracle import model as om
from oracle import vocoder as ov

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    return engine.Device(0)


def _snake(x, a, b):
    s = torch.sin(x * a)
    return x + s * s * b


def _ref_conv(w, x, Cin, K, dil, hist, pro, sa, sb, epi, bias, resid, scale, P):
    """float64 restatement: w f16 numpy ([Cout][Cin][K], or [Cin][Cout][K*P] when P > 1)."""
    W = torch.from_numpy(w.astype(np.float64))
    X = torch.from_numpy(x.astype(np.float64))
    T = X.shape[0]
    H = (K - 1) * dil
    if pro == engine.PRO_SILU_GATE:
        g, u = X[:, :Cin], X[:, Cin:2 * Cin]
        xin = g / (1 + torch.exp(-g)) * u
    else:
        xin = X[:, :Cin]
    hz = torch.zeros(H, Cin, dtype=torch.float64) if hist is None else torch.from_numpy(hist.astype(np.float64))
    full = torch.cat([hz, xin], 0)
    if pro == engine.PRO_SNAKE:
        full = _snake(full, torch.from_numpy(sa.astype(np.float64)), torch.from_numpy(sb.astype(np.float64)))
    if P == 1:
        Cout = W.shape[0]
        y = torch.zeros(T, Cout, dtype=torch.float64)
        for j in range(K):
            y += full[j * dil:j * dil + T] @ W[:, :, j].T
    else:
        Cb = W.shape[1]
        y = torch.zeros(T, P, Cb, dtype=torch.float64)
        for p in range(P):
            for m in range(K):
                y[:, p] += full[H - m:H - m + T] @ W[:, :, p + m * P]
        y = y.reshape(T * P, Cb)
    if bias is not None:
        y = y + torch.from_numpy(bias.astype(np.float64))
    if epi == engine.EPI_GELU:
        y = 0.5 * y * (1 + torch.erf(y / np.sqrt(2.0)))
    elif epi == engine.EPI_RESIDUAL:
        y = y + torch.from_numpy(resid.astype(np.float64))
    elif epi == engine.EPI_SCALE_RESIDUAL:
        y = y * torch.from_numpy(scale.astype(np.float64)) + torch.from_numpy(resid.astype(np.float64))
    elif epi == engine.EPI_SILU:
        y = y / (1 + torch.exp(-y))
    return y.numpy()


# (Cout, Cin, K, dil, T, hist, pro, epi, trans_stride)
CONV_CASES = [
    (64, 64, 7, 1, 100, True, engine.PRO_SNAKE, engine.EPI_NONE, 0),          # Cout < 128, one channel block
    (256, 512, 7, 9, 300, True, engine.PRO_SNAKE, engine.EPI_NONE, 0),        # dilation 9, several row tiles
    (256, 256, 7, 3, 1000, True, engine.PRO_SNAKE, engine.EPI_NONE, 0),       # row-heavy, dilation 3
    (1024, 1024, 7, 1, 64, True, engine.PRO_NONE, engine.EPI_NONE, 0),        # dec0: split-K
    (512, 1024, 1, 1, 16, False, engine.PRO_NONE, engine.EPI_SCALE_RESIDUAL, 0),
    (512, 1024, 1, 1, 16, False, engine.PRO_SILU_GATE, engine.EPI_SCALE_RESIDUAL, 0),
    (4096, 1024, 1, 1, 32, False, engine.PRO_NONE, engine.EPI_GELU, 0),
    (200, 136, 3, 1, 37, True, engine.PRO_NONE, engine.EPI_NONE, 0),          # ragged channels and rows
    (64, 64, 1, 1, 1000, False, engine.PRO_SNAKE, engine.EPI_RESIDUAL, 0),
    (128, 64, 7, 1, 1, True, engine.PRO_SNAKE, engine.EPI_NONE, 0),           # one row: history only
    (256, 512, 2, 1, 40, True, engine.PRO_SNAKE, engine.EPI_NONE, 5),         # transposed, k = 2s
    (128, 128, 1, 1, 9, False, engine.PRO_NONE, engine.EPI_NONE, 2),          # transposed, k = s
    (64, 128, 2, 1, 300, True, engine.PRO_SNAKE, engine.EPI_NONE, 3),
]


# K == 1 layers with the weight read in place by TMA (128B-swizzled tiles), as the prefill
# uses them: (Cout, Cin, T, prologue, epilogue)
TMA_CASES = [
    (3072, 1024, 10, engine.PRO_NONE, engine.EPI_NONE),               # prefill QKV, 10-row prompt
    (1024, 2048, 200, engine.PRO_NONE, engine.EPI_RESIDUAL),          # O projection + residual, 200 rows
    (6144, 1024, 37, engine.PRO_NONE, engine.EPI_NONE),               # gate/up
    (1024, 3072, 200, engine.PRO_SILU_GATE, engine.EPI_RESIDUAL),     # down: SiLU gate prologue + residual
    (2048, 2048, 64, engine.PRO_NONE, engine.EPI_SILU),               # text projection fc1 (bias + SiLU)
    (200, 136, 5, engine.PRO_NONE, engine.EPI_SILU),                  # ragged: TMA zero fill past Cout / Cin
    (64, 64, 1000, engine.PRO_SNAKE, engine.EPI_RESIDUAL),            # one channel tile: weights resident
    (3072, 1024, 1, engine.PRO_NONE, engine.EPI_NONE),                # one row (the codec head)
]


@pytest.mark.parametrize("case", range(len(TMA_CASES)))
def test_conv_primitive_rowmajor_tma_weights(dev, case):
    Cout, Cin, T, pro, epi = TMA_CASES[case]
    _conv_case(dev, Cout, Cin, 1, 1, T, False, pro, epi, 0, 300 + case, rowmajor=True)


@pytest.mark.parametrize("case", range(len(CONV_CASES)))
def test_conv_primitive_matches_float64(dev, case):
    Cout, Cin, K, dil, T, use_hist, pro, epi, P = CONV_CASES[case]
    _conv_case(dev, Cout, Cin, K, dil, T, use_hist, pro, epi, P, 100 + case)


def _conv_case(dev, Cout, Cin, K, dil, T, use_hist, pro, epi, P, seed, rowmajor=False):
    rng = np.random.default_rng(seed)
    H = (K - 1) * dil
    if P:
        w = (rng.standard_normal((Cin, Cout, K * P)) * 0.05).astype(np.float16)
    else:
        w = (rng.standard_normal((Cout, Cin, K)) * 0.05).astype(np.float16)
    xs = 2 * Cin if pro == engine.PRO_SILU_GATE else Cin
    x = rng.standard_normal((T, xs)).astype(np.float32)
    hist = rng.standard_normal((H, Cin)).astype(np.float32) if (use_hist and H) else None
    sa = np.exp(rng.standard_normal(Cin).astype(np.float32) * 0.3)
    sb = (1.0 / (np.exp(rng.standard_normal(Cin).astype(np.float32) * 0.3) + 1e-9)).astype(np.float32)
    Pn = max(P, 1)
    bias = (rng.standard_normal(Cout) * 0.1).astype(np.float32)
    Ctot = Cout
    resid = rng.standard_normal((T, Ctot)).astype(np.float32) if epi in (engine.EPI_RESIDUAL, engine.EPI_SCALE_RESIDUAL) else None
    scale = (rng.standard_normal(Ctot) * 0.5).astype(np.float32) if epi == engine.EPI_SCALE_RESIDUAL else None
    want = _ref_conv(w, x, Cin, K, dil, hist, pro, sa, sb, epi, bias, resid, scale, Pn)

    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    dw = torch.from_numpy(np.ascontiguousarray(w).view(np.int16)).cuda()
    dx, dsa, dsb, db = d(x), d(sa), d(sb), d(bias)
    dh = d(hist) if hist is not None else None
    dy = d(resid.copy()) if resid is not None else torch.full((T * Pn, Cout), float("nan"), device="cuda")
    dsc = d(scale) if scale is not None else None
    engine.conv1d(dev, dw.data_ptr(), Cout, Cin, K, dx.data_ptr(), T, dy.data_ptr(), dil=dil, trans_stride=P, x_stride=xs,
                  hist_ptr=dh.data_ptr() if dh is not None else 0, pro=pro, snake_a=dsa.data_ptr(), snake_b=dsb.data_ptr(), epi=epi,
                  bias=db.data_ptr(), resid=dy.data_ptr() if resid is not None else 0, scale=dsc.data_ptr() if dsc is not None else 0,
                  rowmajor=rowmajor)
    got = dy.cpu().numpy().astype(np.float64)
    assert np.isfinite(got).all()
    err = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert err < 1e-5, err


def test_conv_primitive_rejects_bad_shapes(dev):
    x = torch.zeros(16, 12, device="cuda")
    w = torch.zeros(64 * 12, dtype=torch.int16, device="cuda")
    y = torch.zeros(16, 64, device="cuda")
    with pytest.raises(capi.NaviError) as e:
        engine.conv1d(dev, w.data_ptr(), 64, 12, 1, x.data_ptr(), 16, y.data_ptr())
    assert e.value.status == capi.NAVI_E_SHAPE


# ---- the decoder against the oracle --------------------------------------------------------

def _codes(cfg, n, seed):
    return np.random.default_rng(seed).integers(0, cfg.vq_codebook_size, (n, cfg.vq_n_q)).astype(np.int32)


def _stage_capture(voc):
    got = {}

    def hook(name, ptr, rows, cols):
        t = torch.empty(rows * cols, dtype=torch.float32, device="cuda")
        import ctypes
        lib = ctypes.CDLL("libcudart.so.12")
        lib.cudaMemcpy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]
        assert lib.cudaMemcpy(ctypes.c_void_p(t.data_ptr()), ctypes.c_void_p(ptr), rows * cols * 4, 3) == 0
        got[name] = t.cpu().numpy().reshape(rows, cols)
    voc.set_stage_hook(hook)
    return got


def _check_stages(got, want, tol):
    names = [k for k in want if k in got]
    assert {"rvq", "pre_conv", "pre_transformer", "up0", "up1", "dec0", "dec1", "dec4"} <= set(names), names
    worst = {}
    for k in names:
        w = want[k].numpy()
        assert got[k].shape == w.shape, (k, got[k].shape, w.shape)
        worst[k] = om.rel_l2(got[k], w)
    bad = {k: v for k, v in worst.items() if not v < tol}
    assert not bad, bad
    return worst


@pytest.fixture(scope="module")
def small(dev, small_navi):
    w = engine.Weights(dev, small_navi)
    return w, om.Weights.from_navi(small_navi)


def test_small_decoder_stages_match_oracle(dev, small):
    w, W = small
    voc = engine.Vocoder(dev, w, max_chunk_frames=8)
    got = _stage_capture(voc)
    codes = _codes(W.cfg, 6, 1)
    pcm = voc.decode(codes)
    o = ov.Vocoder(W)
    want = {}
    ref = o.decode_chunk(codes, want).numpy()
    assert pcm.shape == ref.shape == (6 * W.cfg.samples_per_frame,)
    _check_stages(got, want, 1e-3)
    assert om.rel_l2(pcm, ref) < 1e-3
    assert np.abs(pcm).max() <= 1.0


def test_small_chunked_equals_one_shot_and_oracle(dev, small):
    w, W = small
    codes = _codes(W.cfg, 13, 2)
    one = engine.Vocoder(dev, w, max_chunk_frames=16).decode(codes)
    v4 = engine.Vocoder(dev, w, max_chunk_frames=4)
    chunked = v4.decode(codes)                                   # chunks 4, 4, 4, 1
    assert np.abs(chunked - one).max() <= 1e-5
    # state carries across calls, and reset() starts a new utterance
    v4.reset()
    parts = np.concatenate([v4.decode(codes[:5]), v4.decode(codes[5:6]), v4.decode(codes[6:])])
    assert np.abs(parts - one).max() <= 1e-5
    v4.reset()
    again = v4.decode(codes)
    assert np.array_equal(again, chunked)
    ref = ov.Vocoder(W).decode(torch.from_numpy(codes.astype(np.int64)), 13, 3).numpy()
    assert om.rel_l2(one, ref) < 1e-3


def test_rejects_bad_codes_and_small_buffer(dev, small):
    w, W = small
    voc = engine.Vocoder(dev, w, max_chunk_frames=4)
    codes = _codes(W.cfg, 2, 3)
    bad = codes.copy()
    bad[1, 5] = W.cfg.vq_codebook_size
    with pytest.raises(capi.NaviError) as e:
        voc.decode(bad)
    assert e.value.status == capi.NAVI_E_ARG
    import ctypes
    out = np.empty(10, np.float32)
    st = capi.lib().navi_vocoder_decode(voc.h, codes.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), 2,
                                        out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), out.size)
    assert st == capi.NAVI_E_ARG
    assert voc.decode(codes[:0]).size == 0


def test_full_size_decoder_matches_oracle(dev, full_navi):
    """configs[3] shapes (decoder_dim 1024): 4 frames one-shot, then 16 more in chunks of 16."""
    w = engine.Weights(dev, full_navi)
    W = om.Weights.from_navi(full_navi)
    voc = engine.Vocoder(dev, w, max_chunk_frames=16)
    got = _stage_capture(voc)
    o = ov.Vocoder(W)
    codes = _codes(W.cfg, 20, 4)
    want = {}
    ref0 = o.decode_chunk(codes[:4], want).numpy()
    pcm0 = voc.decode(codes[:4])
    worst = _check_stages(got, want, 1e-3)
    assert om.rel_l2(pcm0, ref0) < 1e-3, worst
    voc.set_stage_hook(None)
    ref1 = o.decode_chunk(codes[4:]).numpy()
    pcm1 = voc.decode(codes[4:])
    assert om.rel_l2(pcm1, ref1) < 1e-3
    assert pcm1.shape == (16 * 1920,)
