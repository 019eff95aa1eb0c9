"""CPU oracle of the navi-tts frame path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg import
this module, and only as the checker (or, for bench, as the timed CPU
baseline); the product path never does.

A plain PyTorch fp32 (CPU) restatement of the reference engine's per-frame math
(model/qwen3tts/frame.hip) on f16-rounded weights upcast to f32, so the oracle
and the device kernels see identical weights:

  decoder layer    frame.hip:300-305 (RMSNorm eps, QKV), 312-346 (per-head q/k
                   RMSNorm before rotate-half RoPE, theta = pos * theta0^(-2t/hd),
                   K stored post-RoPE, K and V rounded to f16 in the cache),
                   350-385 (GQA, scale 1/sqrt(hd), softmax over 0..pos),
                   388-402 (silu(gate) * up), 539-549 (residual adds)
  talker step      frame.hip:536-550 (x = step_in, 28 layers, final norm,
                   codec_head); hidden_out is the post-final-norm hidden
  code predictor   frame.hip:555-575 (16 positions: 0 = talker hidden,
                   1 = talker codec_embedding[cb0], p >= 2 = cp codec_embedding
                   [p-2][code p-1]; lm_head[p-1] on position p gives code p;
                   its own KV, positions 0..15, reset every frame)
  step embedding   frame.hip:504-513 (codec_embedding[cb0] + sum of the 15 cp
                   code embeddings + the trailing text row)
  sampling         oracle/sampler.c (bit-exact restatement, via ctypes)

M-RoPE at batch one reduces to plain RoPE (docs/model.md:48-53).  The
reference's PyTorch model (qwen-tts 0.1.1 on transformers 4.57.3,
tools/uv.lock:1935-1936, 2687-2688) is not available here; tests pin this
module's decoder layer against transformers' Qwen3DecoderLayer instead, which
is the layer qwen-tts builds the talker from.
"""
from __future__ import annotations

import ctypes
import math
import os
from dataclasses import dataclass

import numpy as np
import torch

_HERE = os.path.dirname(os.path.abspath(__file__))


# --- primitives -------------------------------------------------------------------------

def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """y = x * rsqrt(mean(x^2) + eps) * w over the last dim (frame.hip:107-114)."""
    return x * torch.rsqrt((x * x).mean(-1, keepdim=True) + eps) * w


def rope_inv_freq(head_dim: int, theta: float) -> torch.Tensor:
    """theta^(-2t/hd) for t < hd/2, computed in double and rounded to f32."""
    t = torch.arange(head_dim // 2, dtype=torch.float64)
    return (1.0 / (theta ** (2.0 * t / head_dim))).to(torch.float32)


def rope(x: torch.Tensor, pos: int, inv_freq: torch.Tensor) -> torch.Tensor:
    """Rotate-half RoPE of x[..., hd] at integer position pos (pairs i and i + hd/2)."""
    half = x.shape[-1] // 2
    ang = torch.tensor(float(pos), dtype=torch.float32) * inv_freq
    c, s = torch.cos(ang.double()).float(), torch.sin(ang.double()).float()
    x0, x1 = x[..., :half], x[..., half:]
    return torch.cat([x0 * c - x1 * s, x0 * s + x1 * c], dim=-1)


def silu(x: torch.Tensor) -> torch.Tensor:
    return x / (1.0 + torch.exp(-x))


def f16r(x: torch.Tensor) -> torch.Tensor:
    """Round to f16 and back (the KV cache storage)."""
    return x.half().float()


# --- weights ----------------------------------------------------------------------------

@dataclass
class Dims:
    hidden: int
    n_layer: int
    n_head: int
    n_kv_head: int
    head_dim: int
    ff: int
    vocab: int
    eps: float
    rope_theta: float


class Weights:
    """name -> f32 torch tensor (f16 values upcast), plus the hyperparameters."""

    def __init__(self, tensors: dict, cfg) -> None:
        self.t = {k: (v if isinstance(v, torch.Tensor) else torch.from_numpy(np.asarray(v, dtype=np.float32)))
                  for k, v in tensors.items()}
        self.cfg = cfg
        tl, cp = cfg.talker, cfg.cp
        self.tl = Dims(tl.hidden, tl.n_layer, tl.n_head, tl.n_kv_head, tl.head_dim, tl.ff, tl.vocab, tl.eps, tl.rope_theta)
        self.cp = Dims(cp.hidden, cp.n_layer, cp.n_head, cp.n_kv_head, cp.head_dim, cp.ff, cp.vocab, cp.eps, cp.rope_theta)

    def __getitem__(self, k):
        return self.t[k]

    @staticmethod
    def from_navi(path: str) -> "Weights":
        import sys
        sys.path.insert(0, os.path.join(os.path.dirname(_HERE), "navi-tts_b200"))
        from navi_b200 import model_spec
        from navi_b200.navi_file import NaviFile
        f = NaviFile.open(path)
        cfg = model_spec.config_from_kv(f.kv)
        tensors = {t.name: torch.from_numpy(np.array(f.array(t), dtype=np.float32)) for t in f.tensors if t.dtype != 4}
        return Weights(tensors, cfg)


def layer_prefix(component: str, l: int) -> str:
    return ("talker.model" if component == "talker" else "talker.code_predictor.model") + f".layers.{l}."


# --- decoder layer (one or more positions, appended to a KV cache) ----------------------------

def decoder_layer(W: Weights, component: str, l: int, x: torch.Tensor, kcache: torch.Tensor,
                  vcache: torch.Tensor, pos0: int, kv_round: bool = True) -> torch.Tensor:
    """Runs rows x[T, H] at positions pos0..pos0+T-1 through layer l, causally.
    kcache/vcache: [max_pos, n_kv*hd] f32 tensors holding f16-rounded values; rows
    pos0..pos0+T-1 are written (post-RoPE K). kv_round=False keeps K/V in f32 (used only
    to pin this layer against a full-precision reference implementation)."""
    d = W.tl if component == "talker" else W.cp
    p = layer_prefix(component, l)
    T = x.shape[0]
    inv = rope_inv_freq(d.head_dim, d.rope_theta)
    h = rmsnorm(x, W[p + "input_layernorm.weight"], d.eps)
    q = (h @ W[p + "self_attn.q_proj.weight"].T).view(T, d.n_head, d.head_dim)
    k = (h @ W[p + "self_attn.k_proj.weight"].T).view(T, d.n_kv_head, d.head_dim)
    v = (h @ W[p + "self_attn.v_proj.weight"].T).view(T, d.n_kv_head, d.head_dim)
    q = rmsnorm(q, W[p + "self_attn.q_norm.weight"], d.eps)
    k = rmsnorm(k, W[p + "self_attn.k_norm.weight"], d.eps)
    q = torch.stack([rope(q[t], pos0 + t, inv) for t in range(T)])
    k = torch.stack([rope(k[t], pos0 + t, inv) for t in range(T)])
    kv = d.n_kv_head * d.head_dim
    rnd = f16r if kv_round else (lambda t: t)
    kcache[pos0:pos0 + T] = rnd(k.reshape(T, kv))
    vcache[pos0:pos0 + T] = rnd(v.reshape(T, kv))
    K = kcache[:pos0 + T].view(-1, d.n_kv_head, d.head_dim)
    V = vcache[:pos0 + T].view(-1, d.n_kv_head, d.head_dim)
    group = d.n_head // d.n_kv_head
    scale = 1.0 / math.sqrt(d.head_dim)
    out = torch.empty(T, d.n_head, d.head_dim)
    n = pos0 + T
    causal = torch.arange(n)[None, :] > (pos0 + torch.arange(T))[:, None]   # key j hidden from row t when j > pos0 + t
    for hh in range(d.n_head):
        g = hh // group
        s = (q[:, hh] @ K[:n, g].T) * scale
        s = s.masked_fill(causal, float("-inf"))
        out[:, hh] = torch.softmax(s, dim=1) @ V[:n, g]
    x = x + out.reshape(T, -1) @ W[p + "self_attn.o_proj.weight"].T
    h2 = rmsnorm(x, W[p + "post_attention_layernorm.weight"], d.eps)
    a = silu(h2 @ W[p + "mlp.gate_proj.weight"].T) * (h2 @ W[p + "mlp.up_proj.weight"].T)
    return x + a @ W[p + "mlp.down_proj.weight"].T


def talker_step(W: Weights, step_in: torch.Tensor, kv: list, n_past: int):
    """One talker decode step (frame.hip:536-550). kv: per layer (kcache, vcache).
    Returns (post-norm hidden [H], codec logits [V])."""
    x = step_in.reshape(1, -1).clone()
    for l in range(W.tl.n_layer):
        x = decoder_layer(W, "talker", l, x, kv[l][0], kv[l][1], n_past)
    hidden = rmsnorm(x[0], W["talker.model.norm.weight"], W.tl.eps)
    logits = W["talker.codec_head.weight"] @ hidden
    return hidden, logits


# --- prompt and prefill ----------------------------------------------------------------------

def build_prompt(W: Weights, ids, language: str, speaker: torch.Tensor):
    """The talker prompt of the reference (talker.hip:283-352): text rows are the role header
    ids[0:3], the text ids[3:-5], then tts_bos / tts_eos / tts_pad, each a text_embedding row
    through text_projection (fc1 + bias, SiLU, fc2 + bias). Codec rows: the think block
    (nothink, think_bos, think_eos; or think, think_bos, language, think_eos), codec_pad,
    codec_bos. Prefill rows: the 3 header rows; tts_pad + each think row; tts_pad + speaker;
    tts_bos + codec_pad; first text row + codec_bos. Trailing rows: the other text rows,
    then tts_eos. Returns (prefill [n, H], trailing [m, H], tts_pad [H])."""
    c = W.cfg
    ids = [int(i) for i in ids]
    n_text = len(ids) - 8
    assert n_text >= 1, "prompt ids too short"
    tids = ids[:3] + ids[3:3 + n_text] + [c.tts_bos_id, c.tts_eos_id, c.tts_pad_id]
    i_bos, i_eos, i_pad = len(tids) - 3, len(tids) - 2, len(tids) - 1
    rows = W["talker.model.text_embedding.weight"][torch.tensor(tids)]
    h = silu(rows @ W["talker.text_projection.linear_fc1.weight"].T + W["talker.text_projection.linear_fc1.bias"])
    proj = h @ W["talker.text_projection.linear_fc2.weight"].T + W["talker.text_projection.linear_fc2.bias"]
    langs = dict(c.languages)
    if not language or language == "auto":
        cids = [c.codec_nothink_id, c.codec_think_bos_id, c.codec_think_eos_id]
    else:
        cids = [c.codec_think_id, c.codec_think_bos_id, langs[language], c.codec_think_eos_id]
    n_think = len(cids)
    cids += [c.codec_pad_id, c.codec_bos_id]
    codec = W["talker.model.codec_embedding.weight"][torch.tensor(cids)]
    pre = [proj[0], proj[1], proj[2]]
    pre += [proj[i_pad] + codec[r] for r in range(n_think)]
    pre += [proj[i_pad] + speaker, proj[i_bos] + codec[n_think], proj[3] + codec[n_think + 1]]
    trailing = [proj[3 + r] for r in range(1, n_text)] + [proj[i_eos]]
    return torch.stack(pre), torch.stack(trailing), proj[i_pad].clone()


def prefill(W: Weights, rows: torch.Tensor, kv: list):
    """The talker prefill (talker.hip:355-399): rows [T, H] at positions 0..T-1 through all
    layers, causally, filling kv (per layer (kcache, vcache), f16-rounded, K after RoPE).
    Returns (post-norm hidden of the last row [H], its codec logits [V])."""
    x = rows.clone()
    for l in range(W.tl.n_layer):
        x = decoder_layer(W, "talker", l, x, kv[l][0], kv[l][1], 0)
    hidden = rmsnorm(x[-1], W["talker.model.norm.weight"], W.tl.eps)
    return hidden, W["talker.codec_head.weight"] @ hidden


# --- sampling (bit-exact C restatement) -----------------------------------------------------

class _SampleArgs(ctypes.Structure):
    _fields_ = [("temperature", ctypes.c_float), ("top_k", ctypes.c_int), ("top_p", ctypes.c_float),
                ("rng", ctypes.c_int), ("seed", ctypes.c_uint64), ("frame_index", ctypes.c_int),
                ("codebook", ctypes.c_int), ("talker_mods", ctypes.c_int), ("suppress_from", ctypes.c_int),
                ("eos_id", ctypes.c_int), ("min_frames", ctypes.c_int), ("repetition_penalty", ctypes.c_float),
                ("seen", ctypes.c_void_p), ("exp_libm", ctypes.c_int)]


_lib = None


def sampler_lib():
    global _lib
    if _lib is None:
        path = os.path.join(_HERE, "_build", "liboracle_sampler.so")
        if not os.path.exists(path):
            raise RuntimeError(f"{path} is missing: run `make -C oracle` (or __graft_entry__.build())")
        _lib = ctypes.CDLL(path)
        _lib.oracle_sample.restype = ctypes.c_int
        _lib.oracle_sample.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(_SampleArgs), ctypes.c_void_p,
                                       ctypes.c_void_p]
        _lib.oracle_exp.restype = ctypes.c_float
        _lib.oracle_exp.argtypes = [ctypes.c_float]
        _lib.oracle_uniform.restype = ctypes.c_float
        _lib.oracle_uniform.argtypes = [ctypes.c_int, ctypes.c_uint64, ctypes.c_int, ctypes.c_int]
        _lib.oracle_draw_seed.restype = ctypes.c_uint64
        _lib.oracle_draw_seed.argtypes = [ctypes.c_uint64, ctypes.c_int, ctypes.c_int]
    return _lib


@dataclass
class Sampling:
    """Mirrors navi::qwen3tts::Sampling (frame.h:24-31) plus top-p and the RNG choice."""
    temperature: float = 0.9
    top_k: int = 50
    top_p: float = 1.0
    repetition_penalty: float = 1.05
    cp_temperature: float = 0.9
    cp_top_k: int = 50
    cp_top_p: float = 1.0
    min_frames: int = 2
    rng: int = 0          # 0 PCG (the reference's stream), 1 Philox


def sample(logits, codebook: int, s: Sampling, seed: int, frame_index: int, *, talker_mods=None, exp_libm: bool = False) -> int:
    """codebook 0: the talker draw (talker_mods = (suppress_from, eos_id, seen u8[V]));
    codebooks 1..15: the code-predictor draws. exp_libm: take e_i from the C library's expf
    (to compare with the reference's own sampler run on the host), not the specified exp."""
    lg = np.ascontiguousarray(np.asarray(logits, dtype=np.float32))
    a = _SampleArgs()
    if codebook == 0:
        a.temperature, a.top_k, a.top_p = s.temperature, s.top_k, s.top_p
    else:
        a.temperature, a.top_k, a.top_p = s.cp_temperature, s.cp_top_k, s.cp_top_p
    a.rng, a.seed, a.frame_index, a.codebook = s.rng, seed & (2**64 - 1), frame_index, codebook
    a.exp_libm = 1 if exp_libm else 0
    seen = None
    if talker_mods is not None:
        sup, eos, seen_arr = talker_mods
        seen = np.ascontiguousarray(np.asarray(seen_arr, dtype=np.uint8))
        a.talker_mods, a.suppress_from, a.eos_id, a.min_frames = 1, sup, eos, s.min_frames
        a.repetition_penalty = s.repetition_penalty
        a.seen = seen.ctypes.data
    return int(sampler_lib().oracle_sample(lg.ctypes.data, lg.shape[0], ctypes.byref(a), None, None))


# --- code predictor + whole frame ---------------------------------------------------------

@dataclass
class FrameOut:
    codes: list              # 16 ints
    hidden: torch.Tensor     # talker post-norm hidden [H]
    logits: torch.Tensor     # talker codec logits [V]
    clogits: torch.Tensor    # [15, cp vocab]
    step_out: torch.Tensor   # next frame's step embedding [H]


def code_predictor(W: Weights, hidden: torch.Tensor, cb0: int, s: Sampling, seed: int, frame_index: int,
                   teacher_codes=None):
    """Positions 0..15 of the code predictor (frame.hip:555-575). Returns (codes[1..15], clogits[15, V]).
    With teacher_codes, codes[1..15] are taken from it instead of sampled (logits still computed)."""
    d = W.cp
    kv_dim = d.n_kv_head * d.head_dim
    kc = [torch.zeros(16, kv_dim) for _ in range(d.n_layer)]
    vc = [torch.zeros(16, kv_dim) for _ in range(d.n_layer)]
    codes = [cb0]
    clogits = torch.zeros(15, d.vocab)
    for pos in range(16):
        if pos == 0:
            x = hidden.reshape(1, -1).clone()
        elif pos == 1:
            x = W["talker.model.codec_embedding.weight"][cb0].reshape(1, -1).clone()
        else:
            x = W[f"talker.code_predictor.model.codec_embedding.{pos - 2}.weight"][codes[pos - 1]].reshape(1, -1).clone()
        for l in range(d.n_layer):
            x = decoder_layer(W, "cp", l, x, kc[l], vc[l], pos)
        if pos >= 1:
            hn = rmsnorm(x[0], W["talker.code_predictor.model.norm.weight"], d.eps)
            lg = W[f"talker.code_predictor.lm_head.{pos - 1}.weight"] @ hn
            clogits[pos - 1] = lg
            if teacher_codes is not None:
                codes.append(int(teacher_codes[pos]))
            else:
                codes.append(sample(lg, pos, s, seed, frame_index))
    return codes[1:], clogits


def step_embedding(W: Weights, codes, trailing: torch.Tensor) -> torch.Tensor:
    v = W["talker.model.codec_embedding.weight"][codes[0]].clone()
    for cb in range(15):
        v = v + W[f"talker.code_predictor.model.codec_embedding.{cb}.weight"][codes[1 + cb]]
    return v + trailing


def frame(W: Weights, *, step_in=None, kv=None, n_past=None, hidden=None, logits=None, trailing=None,
          s: Sampling = None, seed: int = 0, frame_index: int = 0, seen=None, teacher_codes=None) -> FrameOut:
    """One frame. Talker step from (step_in, kv, n_past), or, for frame 0, the prefill's
    (hidden, logits) as run_first does.  seen: u8[V] repetition set, updated in place."""
    s = s or Sampling()
    if hidden is None:
        hidden, logits = talker_step(W, step_in, kv, n_past)
    V = W.tl.vocab
    if seen is None:
        seen = np.zeros(V, dtype=np.uint8)
    cfg = W.cfg
    if teacher_codes is not None:
        cb0 = int(teacher_codes[0])
    else:
        cb0 = sample(logits, 0, s, seed, frame_index, talker_mods=(V - 1024, cfg.codec_eos_id, seen))
    if cb0 != cfg.codec_eos_id:
        seen[cb0] = 1
    rest, clogits = code_predictor(W, hidden, cb0, s, seed, frame_index, teacher_codes)
    codes = [cb0] + rest
    return FrameOut(codes, hidden, logits, clogits, step_embedding(W, codes, trailing))


def rel_l2(a, b) -> float:
    a = torch.as_tensor(np.asarray(a, dtype=np.float64))
    b = torch.as_tensor(np.asarray(b, dtype=np.float64))
    return float(torch.linalg.vector_norm(a - b) / max(float(torch.linalg.vector_norm(b)), 1e-30))
