"""Driver of oracle/_ref/ref_frame_check -- TEST INFRASTRUCTURE ONLY.

ref_frame_check is the reference engine's own frame code (model/qwen3tts/frame.hip) compiled
for the CPU against the host stand-in for the HIP runtime in oracle/hipsim (built by
`make -C oracle REF=<reference tree>`). These helpers write its binary requests and read its
responses: whole frames (Frame::run / run_first on a one-block grid), the per-frame seeds of
Frame::Impl::launch, and the reference samplers tl_sample / cp_sample on given logits.
Only tests use it, as a checker.
"""
from __future__ import annotations

import os
import struct
import subprocess
import tempfile
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
BIN = os.path.join(HERE, "_ref", "ref_frame_check")


def available() -> bool:
    return os.path.exists(BIN)


@dataclass
class RefSampling:
    """The reference's Sampling (frame.h:24-31): no top-p, PCG stream only."""
    temperature: float = 0.9
    top_k: int = 50
    repetition_penalty: float = 1.05
    cp_temperature: float = 0.9
    cp_top_k: int = 50
    min_frames: int = 2

    def pack(self) -> bytes:
        return struct.pack("<fiffii", self.temperature, self.top_k, self.repetition_penalty, self.cp_temperature,
                           self.cp_top_k, self.min_frames)


def _call(req: bytes, timeout: int = 900) -> bytes:
    with tempfile.TemporaryDirectory() as td:
        a, b = os.path.join(td, "req.bin"), os.path.join(td, "resp.bin")
        with open(a, "wb") as f:
            f.write(req)
        r = subprocess.run([BIN, a, b], capture_output=True, text=True, timeout=timeout)
        if r.returncode != 0:
            raise RuntimeError(f"ref_frame_check failed ({r.returncode}): {r.stderr.strip()}")
        with open(b, "rb") as f:
            return f.read()


def _head(mode: int, navi: str) -> bytes:
    p = navi.encode()
    return struct.pack("<ii", mode, len(p)) + p


def seeds(navi: str, pairs):
    """[(talker_seed, cp_seed)] that Frame::Impl::launch derives for each (seed, frame_index)."""
    req = _head(2, navi) + struct.pack("<i", len(pairs)) + b"".join(struct.pack("<Qi", s & (2**64 - 1), f) for s, f in pairs)
    out = _call(req)
    v = np.frombuffer(out, dtype=np.uint64).reshape(-1, 2)
    return [(int(a), int(b)) for a, b in v]


def sample(navi: str, cases):
    """cases: (RefSampling, seed, frame_index, codebook, logits f32[V], seen u8[talker vocab]);
    returns the ids tl_sample (codebook 0) / cp_sample pick."""
    req = [_head(3, navi), struct.pack("<i", len(cases))]
    for s, seed, fi, cb, logits, seen in cases:
        req += [s.pack(), struct.pack("<Qii", seed & (2**64 - 1), fi, cb), np.ascontiguousarray(logits, np.float32).tobytes(),
                np.ascontiguousarray(seen, np.uint8).tobytes()]
    return np.frombuffer(_call(b"".join(req)), dtype=np.int32).tolist()


@dataclass
class RefFrame:
    ok: bool
    codes: list
    talker_seed: int
    cp_seed: int
    hidden: np.ndarray
    logits: np.ndarray
    clogits: np.ndarray
    step_out: np.ndarray
    seen: np.ndarray
    k_rows: list = None     # per layer: the K row written at n_past (f16)
    v_rows: list = None


def frame(navi: str, dims, s: RefSampling, seed: int, frame_index: int, seen, trailing, *, step_in=None, kv=None, n_past=None,
          hidden=None, logits=None) -> RefFrame:
    """One frame of the reference k_frame: Frame::run (step_in, kv = per layer (K, V) f16
    [n_past + 1, kv_dim], n_past) or Frame::run_first (hidden, logits). dims: (H, TV, CV,
    n_layer, kv_dim)."""
    H, TV, CV, NL, KVD = dims
    mode = 1 if hidden is not None else 0
    req = [_head(mode, navi), s.pack(), struct.pack("<Qi", seed & (2**64 - 1), frame_index),
           np.ascontiguousarray(seen, np.uint8).tobytes(), np.ascontiguousarray(trailing, np.float32).tobytes()]
    if mode == 0:
        req.append(struct.pack("<i", n_past))
        req.append(np.ascontiguousarray(step_in, np.float32).tobytes())
        for k, v in kv:
            req.append(np.ascontiguousarray(k[:n_past + 1], np.float16).tobytes())
            req.append(np.ascontiguousarray(v[:n_past + 1], np.float16).tobytes())
    else:
        req += [np.ascontiguousarray(hidden, np.float32).tobytes(), np.ascontiguousarray(logits, np.float32).tobytes()]
    out = _call(b"".join(req))
    o = 0

    def take(dtype, n):
        nonlocal o
        a = np.frombuffer(out, dtype=dtype, count=n, offset=o)
        o += a.nbytes
        return a.copy()

    ok = bool(take(np.int32, 1)[0])
    codes = take(np.int32, 16).tolist()
    ts, cs = (int(x) for x in take(np.uint64, 2))
    r = RefFrame(ok, codes, ts, cs, take(np.float32, H), take(np.float32, TV), take(np.float32, 15 * CV).reshape(15, CV),
                 take(np.float32, H), take(np.uint8, TV))
    if mode == 0:
        r.k_rows, r.v_rows = [], []
        for _ in range(NL):
            r.k_rows.append(take(np.float16, KVD))
            r.v_rows.append(take(np.float16, KVD))
    return r


VOC_BIN = os.path.join(HERE, "_ref", "ref_vocoder_check")


def vocoder_available() -> bool:
    return os.path.exists(VOC_BIN)


def vocoder_decode(navi: str, codes, max_chunk: int = 32, stages: bool = False):
    """The reference's Vocoder::decode (oracle/_ref/ref_vocoder_check) of codes [n][16]:
    PCM f32 [n * samples_per_frame] and, with stages=True, {name: [rows, cols]} of every
    stage of the first chunk (the reference's stage hook)."""
    with tempfile.TemporaryDirectory() as td:
        cpath, ppath, sdir = os.path.join(td, "codes.bin"), os.path.join(td, "pcm.bin"), os.path.join(td, "stages")
        np.ascontiguousarray(codes, np.int32).tofile(cpath)
        args = [VOC_BIN, navi, cpath, ppath, str(max_chunk)]
        if stages:
            os.mkdir(sdir)
            args.append(sdir)
        r = subprocess.run(args, capture_output=True, text=True, timeout=1800)
        if r.returncode != 0:
            raise RuntimeError(f"ref_vocoder_check failed ({r.returncode}): {r.stderr.strip()}")
        pcm = np.fromfile(ppath, np.float32)
        out = {}
        if stages:
            for f in os.listdir(sdir):
                if f.endswith(".f32"):
                    name = f[:-4]
                    rows, cols = map(int, open(os.path.join(sdir, name + ".shape")).read().split())
                    out[name] = np.fromfile(os.path.join(sdir, f), np.float32).reshape(rows, cols)
        return pcm, out


TALKER_BIN = os.path.join(HERE, "_ref", "ref_talker_check")


def talker_available() -> bool:
    return os.path.exists(TALKER_BIN)


def talker_prefill(navi: str, ids, language: str, speaker, dims):
    """The reference's Talker::build_prompt + prefill (oracle/_ref/ref_talker_check).
    dims = (H, V, n_layer, kv_dim). Returns (prefill rows, trailing rows, tts_pad, hidden,
    logits, [(K rows, V rows) f16 per layer])."""
    H, V, NL, KVD = dims
    lang = (language or "").encode()
    req = struct.pack("<i", len(ids)) + np.asarray(ids, np.int32).tobytes() + struct.pack("<i", len(lang)) + lang
    req += np.ascontiguousarray(speaker, np.float32).tobytes()
    with tempfile.TemporaryDirectory() as td:
        a, b = os.path.join(td, "req.bin"), os.path.join(td, "out.bin")
        with open(a, "wb") as f:
            f.write(req)
        r = subprocess.run([TALKER_BIN, navi, a, b], capture_output=True, text=True, timeout=1800)
        if r.returncode != 0:
            raise RuntimeError(f"ref_talker_check failed ({r.returncode}): {r.stderr.strip()}")
        out = open(b, "rb").read()
    n_pre, n_tr = struct.unpack_from("<ii", out, 0)
    o = 8

    def take(dtype, n):
        nonlocal o
        x = np.frombuffer(out, dtype=dtype, count=n, offset=o)
        o += x.nbytes
        return x.copy()

    pre = take(np.float32, n_pre * H).reshape(n_pre, H)
    trail = take(np.float32, n_tr * H).reshape(n_tr, H)
    pad, hid, lg = take(np.float32, H), take(np.float32, H), take(np.float32, V)
    kv = [(take(np.float16, n_pre * KVD).reshape(n_pre, KVD), take(np.float16, n_pre * KVD).reshape(n_pre, KVD)) for _ in range(NL)]
    return pre, trail, pad, hid, lg, kv
