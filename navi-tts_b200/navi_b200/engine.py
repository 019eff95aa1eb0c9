"""Python mirror of the reference engine's classes over the C ABI.

Device      <- navi::Device        (runtime/device/device.h:43-66)
Weights     <- NaviFile + DeviceWeights + Params (runtime/weights/*, model/qwen3tts/params.h)
KvCache     <- navi::qwen3tts::KvCache (model/qwen3tts/talker.h:20-24)
Frame       <- navi::qwen3tts::Frame   (model/qwen3tts/frame.h:46-71)

Same method names and argument meaning; failures raise NaviError carrying the
C status code (the reference throws navi::Error at setup and returns
FrameResult{ok=false} on the request path; Frame.run here returns the result
with ok=False and status set, and raises only on setup/argument errors).
"""
from __future__ import annotations

import ctypes
from ctypes import byref, c_int, c_int32, c_uint16, c_void_p, POINTER
from dataclasses import dataclass, field

from . import capi
from .capi import check, lib


@dataclass
class Sampling:
    """navi::qwen3tts::Sampling (frame.h:24-31) plus top-p and the RNG stream."""
    temperature: float = 0.9
    top_k: int = 50
    top_p: float = 1.0
    repetition_penalty: float = 1.05
    cp_temperature: float = 0.9
    cp_top_k: int = 50
    cp_top_p: float = 1.0
    min_frames: int = 2
    rng: int = capi.NAVI_RNG_PCG

    def c(self) -> capi.Sampling:
        return capi.Sampling(self.temperature, self.top_k, self.top_p, self.repetition_penalty, self.cp_temperature,
                             self.cp_top_k, self.cp_top_p, self.min_frames, self.rng)


@dataclass
class FrameResult:
    ok: bool
    eos: bool
    codes: list
    us: float
    status: int
    error: str = ""


def _open(*owners) -> bool:
    """True while every owner handle (device, weights) is still open. A handle is destroyed
    only then: after its device is closed the native destroy would touch freed resources
    (garbage collection of a reference cycle may finalise the device first), so such a
    handle is dropped and the process's teardown releases its memory."""
    return all(getattr(o, "h", None) for o in owners if o is not None)


class Device:
    def __init__(self, ordinal: int = 0):
        h = c_void_p()
        check(lib().navi_device_open(ordinal, byref(h)))
        self.h = h
        info = capi.DeviceInfo()
        check(lib().navi_device_get_info(self.h, byref(info)))
        self.info = info

    @staticmethod
    def count() -> int:
        n = c_int(0)
        check(lib().navi_device_count(byref(n)))
        return n.value

    @property
    def stream(self) -> int:
        return lib().navi_device_stream(self.h)

    def close(self):
        if self.h:
            lib().navi_device_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Weights:
    def __init__(self, dev: Device, path: str):
        h = c_void_p()
        check(lib().navi_weights_upload(dev.h, str(path).encode(), byref(h)))
        self.h = h
        self.dev = dev
        p = capi.Params()
        check(lib().navi_weights_get_params(self.h, byref(p)))
        self.params = p

    def tensor(self, name: str) -> int:
        return lib().navi_weights_tensor(self.h, name.encode(), None, None, None) or 0

    @property
    def nbytes(self) -> int:
        return lib().navi_weights_bytes(self.h)

    def close(self):
        if self.h:
            if _open(self.dev):
                lib().navi_weights_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class KvCache:
    """Per layer [max_pos][kv_dim] f16 device buffers. Either allocated by the library
    (from_device) or wrapping caller-owned device tensors (wrap), e.g. torch tensors."""

    def __init__(self):
        self._owned = None
        self._keep = None
        self.s = None

    @staticmethod
    def create(dev: Device, n_layer: int, max_pos: int, kv_dim: int) -> "KvCache":
        kv = KvCache()
        ptr = POINTER(capi.KV)()
        check(lib().navi_kv_create(dev.h, n_layer, max_pos, kv_dim, byref(ptr)))
        kv._owned = ptr
        kv.s = ptr.contents
        kv.dev = dev
        return kv

    @staticmethod
    def wrap(k_ptrs, v_ptrs, max_pos: int, kv_dim: int, n_used: int = 0, keepalive=None) -> "KvCache":
        kv = KvCache()
        n = len(k_ptrs)
        ka = (POINTER(c_uint16) * n)(*[ctypes.cast(c_void_p(p), POINTER(c_uint16)) for p in k_ptrs])
        va = (POINTER(c_uint16) * n)(*[ctypes.cast(c_void_p(p), POINTER(c_uint16)) for p in v_ptrs])
        kv.s = capi.KV(n, max_pos, kv_dim, n_used, ka, va)
        kv._keep = (ka, va, keepalive)
        return kv

    def ptr(self):
        return self._owned if self._owned is not None else byref(self.s)

    @property
    def n_used(self) -> int:
        return self.s.n_used

    def close(self):
        if self._owned is not None:
            if _open(getattr(self, "dev", None)):
                lib().navi_kv_destroy(self._owned)
            self._owned = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Talker:
    """navi::qwen3tts::Talker (talker.h:34-67): prompt rows and the prefill that fills its KV cache."""

    def __init__(self, dev: Device, w: Weights, max_prompt_tokens: int = 1024, max_positions: int = 4096):
        h = c_void_p()
        check(lib().navi_talker_create(dev.h, w.h, max_prompt_tokens, max_positions, byref(h)))
        self.h, self.dev, self.w = h, dev, w
        self.prompt = None

    def build_prompt(self, ids, language: str, speaker) -> capi.Prompt:
        import numpy as np
        ids = np.ascontiguousarray(np.asarray(ids, dtype=np.int32))
        spk = np.ascontiguousarray(np.asarray(speaker, dtype=np.float32))
        pr = capi.Prompt()
        check(lib().navi_talker_build_prompt(self.h, ids.ctypes.data_as(POINTER(c_int32)), len(ids),
                                             (language or "").encode(), spk.ctypes.data_as(POINTER(ctypes.c_float)), byref(pr)))
        self.prompt = pr
        return pr

    def prefill(self, pr: capi.Prompt = None) -> None:
        check(lib().navi_talker_prefill(self.h, byref(pr or self.prompt)))

    def kv(self) -> "KvCache":
        kv = KvCache()
        kv.s = capi.KV()
        check(lib().navi_talker_kv(self.h, byref(kv.s)))
        kv._keep = (self,)
        return kv

    def d_hidden(self) -> int:
        return lib().navi_talker_hidden(self.h)

    def d_logits(self) -> int:
        return lib().navi_talker_logits(self.h)

    def last_ms(self) -> float:
        return lib().navi_talker_last_ms(self.h)

    def close(self):
        if self.h:
            if _open(self.dev, self.w):
                lib().navi_talker_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Graph:
    """navi::qwen3tts::Graph (graph.h:43-79) from token ids: prompt, prefill, the frame loop and,
    with vocoder_chunk > 0, the streaming vocoder."""

    def __init__(self, dev: Device, w: Weights, max_prompt_tokens: int = 1024, max_frames: int = 2048, deadline_us: int = 0,
                 vocoder_chunk: int = 32, max_streams: int = 1):
        h = c_void_p()
        opts = capi.FrameOpts(1, deadline_us)
        if max_streams == 1:
            check(lib().navi_graph_create(dev.h, w.h, byref(opts), max_prompt_tokens, max_frames, vocoder_chunk, byref(h)))
        else:
            check(lib().navi_graph_create_streams(dev.h, w.h, byref(opts), max_prompt_tokens, max_frames, vocoder_chunk, max_streams,
                                                  byref(h)))
        self.h, self.dev, self.w = h, dev, w
        self.max_streams = max_streams

    def synth_batch(self, requests, language: str, s: Sampling, first_batch: int = 4, vocoder_batch: int = 16, audio: bool = True):
        """Graph::synth_batch: requests = [(ids, speaker, seed, max_frames)], up to max_streams.
        Returns per stream (codes [n_frames, 16], PCM f32 (empty without audio), stats)."""
        import numpy as np
        n = len(requests)
        keep, reqs = [], (capi.SynthRequest * n)()
        codes = []
        for i, (ids, spk, seed, mf) in enumerate(requests):
            ids = np.ascontiguousarray(np.asarray(ids, dtype=np.int32))
            spk = np.ascontiguousarray(np.asarray(spk, dtype=np.float32))
            c = np.zeros((mf, 16), np.int32)
            keep += [ids, spk]
            codes.append(c)
            reqs[i] = capi.SynthRequest(ids.ctypes.data_as(POINTER(c_int32)), len(ids), (language or "").encode(),
                                        spk.ctypes.data_as(POINTER(ctypes.c_float)), seed, mf, c.ctypes.data_as(POINTER(c_int32)), mf)
        chunks = [[] for _ in range(n)]

        def take(stream, ptr, k, _user):
            chunks[stream].append(np.ctypeslib.as_array(ptr, shape=(k,)).copy())

        fn = capi.STREAM_PCM_FN(take) if audio else capi.STREAM_PCM_FN()
        stats = (capi.SynthStats * n)()
        check(lib().navi_graph_synth_batch(self.h, n, reqs, byref(s.c()), first_batch, vocoder_batch, fn, None, stats))
        out = []
        for i in range(n):
            pcm = np.concatenate(chunks[i]) if chunks[i] else np.zeros(0, np.float32)
            out.append((codes[i][:stats[i].n_frames], pcm, stats[i]))
        return out

    def synth_ids(self, ids, language: str, speaker, s: Sampling, seed: int, max_frames: int):
        """(codes [n_frames, 16] int32, stats) of one utterance, without the vocoder."""
        import numpy as np
        ids = np.ascontiguousarray(np.asarray(ids, dtype=np.int32))
        spk = np.ascontiguousarray(np.asarray(speaker, dtype=np.float32))
        codes = np.zeros((max_frames, 16), np.int32)
        st = capi.SynthStats()
        check(lib().navi_graph_synth_ids(self.h, ids.ctypes.data_as(POINTER(c_int32)), len(ids), (language or "").encode(),
                                         spk.ctypes.data_as(POINTER(ctypes.c_float)), byref(s.c()), seed, max_frames,
                                         codes.ctypes.data_as(POINTER(c_int32)), max_frames, byref(st)))
        return codes[:st.n_frames], st

    def synth(self, ids, language: str, speaker, s: Sampling, seed: int, max_frames: int, first_batch: int = 4,
              vocoder_batch: int = 16, on_pcm=None):
        """Graph::synth (graph.cpp:52-111): (codes [n_frames, 16], PCM [n_frames * 1920] f32, stats,
        the sample count of every vocoder batch). on_pcm(np.ndarray), if given, sees each batch
        as it is produced."""
        import numpy as np
        ids = np.ascontiguousarray(np.asarray(ids, dtype=np.int32))
        spk = np.ascontiguousarray(np.asarray(speaker, dtype=np.float32))
        codes = np.zeros((max_frames, 16), np.int32)
        chunks = []

        def take(ptr, n, _user):
            a = np.ctypeslib.as_array(ptr, shape=(n,)).copy()
            chunks.append(a)
            if on_pcm is not None:
                on_pcm(a)

        fn = capi.PCM_FN(take)
        st = capi.SynthStats()
        check(lib().navi_graph_synth(self.h, ids.ctypes.data_as(POINTER(c_int32)), len(ids), (language or "").encode(),
                                     spk.ctypes.data_as(POINTER(ctypes.c_float)), byref(s.c()), seed, max_frames, first_batch,
                                     vocoder_batch, codes.ctypes.data_as(POINTER(c_int32)), max_frames, fn, None, byref(st)))
        pcm = np.concatenate(chunks) if chunks else np.zeros(0, np.float32)
        return codes[:st.n_frames], pcm, st, [len(c) for c in chunks]

    def close(self):
        if self.h:
            if _open(self.dev, self.w):
                lib().navi_graph_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Vocoder:
    """navi::qwen3tts::Vocoder (vocoder.h:27-55): codes [T][n_q] -> PCM [T * samples_per_frame]."""

    def __init__(self, dev: Device, w: Weights, max_chunk_frames: int = 32, max_frames: int = 4096):
        h = c_void_p()
        check(lib().navi_vocoder_create(dev.h, w.h, max_chunk_frames, max_frames, byref(h)))
        self.h, self.dev, self.w = h, dev, w
        self.n_q = w.params.vq_n_q
        self._hook = None

    @property
    def samples_per_frame(self) -> int:
        return lib().navi_vocoder_samples_per_frame(self.h)

    @property
    def max_chunk_frames(self) -> int:
        return lib().navi_vocoder_max_chunk_frames(self.h)

    @property
    def last_ms(self) -> float:
        return lib().navi_vocoder_last_ms(self.h)

    def reset(self) -> None:
        check(lib().navi_vocoder_reset(self.h))

    def decode(self, codes, n_frames: int | None = None):
        """float32 numpy PCM of the frames (decoder state carries over between calls)."""
        import numpy as np
        codes = np.ascontiguousarray(np.asarray(codes, dtype=np.int32).reshape(-1, self.n_q))
        n = codes.shape[0] if n_frames is None else n_frames
        out = np.empty(max(n, 0) * self.samples_per_frame, np.float32)
        check(lib().navi_vocoder_decode(self.h, codes.ctypes.data_as(POINTER(c_int32)), n,
                                        out.ctypes.data_as(POINTER(ctypes.c_float)), out.size))
        return out

    def set_stage_hook(self, fn) -> None:
        """fn(name: str, device_ptr: int, rows: int, cols: int) after each stage; None removes it."""
        if fn is None:
            self._hook = None
            check(lib().navi_vocoder_set_stage_hook(self.h, capi.STAGE_FN(), None))
            return
        self._hook = capi.STAGE_FN(lambda _u, name, d, r, c: fn(name.decode(), d, r, c))
        check(lib().navi_vocoder_set_stage_hook(self.h, self._hook, None))

    def close(self):
        if self.h:
            if _open(self.dev, self.w):
                lib().navi_vocoder_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


PRO_NONE, PRO_SNAKE, PRO_SILU_GATE = 0, 1, 2
EPI_NONE, EPI_GELU, EPI_RESIDUAL, EPI_SCALE_RESIDUAL, EPI_SILU = 0, 1, 2, 3, 4


def conv1d(dev: Device, w_ptr: int, Cout: int, Cin: int, K: int, x_ptr: int, T: int, y_ptr: int, *, dil: int = 1,
           trans_stride: int = 0, x_stride: int | None = None, hist_ptr: int = 0, pro: int = PRO_NONE, snake_a: int = 0,
           snake_b: int = 0, epi: int = EPI_NONE, bias: int = 0, resid: int = 0, scale: int = 0, y_stride: int | None = None,
           rowmajor: bool = False) -> None:
    """navi_conv1d on device pointers (the implicit-GEMM conv primitive)."""
    P = trans_stride if trans_stride > 0 else 1
    a = capi.ConvArgs(w_ptr, Cout, Cin, K, dil, trans_stride, x_ptr, Cin if x_stride is None else x_stride, T, hist_ptr or None,
                      pro, snake_a or None, snake_b or None, epi, bias or None, resid or None, scale or None, y_ptr,
                      Cout * P if y_stride is None else y_stride, 1 if rowmajor else 0)
    check(lib().navi_conv1d(dev.h, byref(a)))


def _result(r: capi.FrameResult, st: int) -> FrameResult:
    err = "" if st == capi.NAVI_OK else lib().navi_last_error().decode(errors="replace")
    return FrameResult(bool(r.ok), bool(r.eos), list(r.codes), r.us, r.status if st == capi.NAVI_OK else st, err)


class Frame:
    """The persistent frame kernel: talker step -> cb0 sample -> 15 code-predictor steps."""

    def __init__(self, dev: Device, w: Weights, deadline_us: int = 0, blocks_per_mp: int = 1):
        h = c_void_p()
        opts = capi.FrameOpts(blocks_per_mp, deadline_us)
        check(lib().navi_frame_create(dev.h, w.h, byref(opts), byref(h)))
        self.h, self.dev, self.w = h, dev, w

    def reset(self):
        check(lib().navi_frame_reset(self.h))

    def run_first(self, d_hidden: int, d_logits: int, d_trailing: int, s: Sampling, seed: int, frame_index: int) -> FrameResult:
        r = capi.FrameResult()
        st = lib().navi_frame_run_first(self.h, c_void_p(d_hidden), c_void_p(d_logits), c_void_p(d_trailing), byref(s.c()),
                                        seed, frame_index, byref(r))
        return _result(r, st)

    def run(self, kv: KvCache, n_past: int, d_trailing: int, s: Sampling, seed: int, frame_index: int) -> FrameResult:
        r = capi.FrameResult()
        st = lib().navi_frame_run(self.h, kv.ptr(), n_past, c_void_p(d_trailing), byref(s.c()), seed, frame_index, byref(r))
        return _result(r, st)

    def reset_slot(self, slot: int) -> None:
        check(lib().navi_frame_reset_slot(self.h, slot))

    def run_first_slot(self, slot: int, d_hidden: int, d_logits: int, d_trailing: int, s: Sampling, seed: int,
                       frame_index: int) -> FrameResult:
        r = capi.FrameResult()
        st = lib().navi_frame_run_first_slot(self.h, slot, c_void_p(d_hidden), c_void_p(d_logits), c_void_p(d_trailing), byref(s.c()),
                                             seed, frame_index, byref(r))
        return _result(r, st)

    def _batch_args(self, slots, kvs, n_past, d_trailing, seeds, frame_index):
        nb = len(slots)
        return (nb, (c_int * nb)(*slots), (ctypes.POINTER(capi.KV) * nb)(*[ctypes.pointer(k.s) for k in kvs]), (c_int * nb)(*n_past),
                (c_void_p * nb)(*d_trailing), (ctypes.c_uint64 * nb)(*seeds), (c_int * nb)(*frame_index))

    def run_batch(self, slots, kvs, n_past, d_trailing, s: Sampling, seeds, frame_index) -> list:
        """One frame of len(slots) streams (1, 2 or 4) in one launch; a FrameResult per stream."""
        nb, sl, kp, npst, tr, sd, fi = self._batch_args(slots, kvs, n_past, d_trailing, seeds, frame_index)
        res = (capi.FrameResult * nb)()
        st = lib().navi_frame_run_batch(self.h, nb, sl, kp, npst, tr, byref(s.c()), sd, fi, res)
        return [_result(res[i], st) for i in range(nb)]

    def run_first_batch(self, slots, d_hidden, d_logits, d_trailing, s: Sampling, seeds, frame_index) -> list:
        """Frame 0 of len(slots) streams (2 or 4) in one launch, each from its prefill's hidden and
        logits (device pointers); a FrameResult per stream."""
        nb = len(slots)
        res = (capi.FrameResult * nb)()
        st = lib().navi_frame_run_first_batch(self.h, nb, (c_int * nb)(*slots), (c_void_p * nb)(*d_hidden), (c_void_p * nb)(*d_logits),
                                              (c_void_p * nb)(*d_trailing), byref(s.c()), (ctypes.c_uint64 * nb)(*seeds),
                                              (c_int * nb)(*frame_index), res)
        return [_result(res[i], st) for i in range(nb)]

    def enqueue_batch(self, slots, kvs, n_past, d_trailing, s: Sampling, seeds, frame_index) -> None:
        nb, sl, kp, npst, tr, sd, fi = self._batch_args(slots, kvs, n_past, d_trailing, seeds, frame_index)
        check(lib().navi_frame_enqueue_batch(self.h, nb, sl, kp, npst, tr, byref(s.c()), sd, fi))

    def collect_batch(self, nb: int) -> list:
        res = (capi.FrameResult * nb)()
        st = lib().navi_frame_collect_batch(self.h, nb, res)
        return [_result(res[i], st) for i in range(nb)]

    def d_step_out_slot(self, slot: int) -> int:
        return lib().navi_frame_step_out_slot(self.h, slot)

    def set_step_in_slot(self, slot: int, d_step: int) -> None:
        check(lib().navi_frame_set_step_in_slot(self.h, slot, c_void_p(d_step)))

    def inspect_stream(self, index: int):
        """(hidden [H], logits [TV], clogits [15, CV]) of stream `index` of the last launch."""
        import numpy as np
        p = self.w.params
        hid = np.zeros(p.talker.hidden, np.float32)
        lg = np.zeros(p.talker.vocab, np.float32)
        clg = np.zeros((15, p.cp.vocab), np.float32)
        check(lib().navi_frame_inspect_stream(self.h, index, hid.ctypes.data, lg.ctypes.data, clg.ctypes.data))
        return hid, lg, clg

    def run_layer(self, layer: int, d_x: int, kv: KvCache, n_past: int, d_out: int) -> FrameResult:
        """One talker decoder layer alone at position n_past: d_x -> d_out, f32 [hidden]."""
        r = capi.FrameResult()
        st = lib().navi_frame_run_layer(self.h, layer, c_void_p(d_x), kv.ptr(), n_past, c_void_p(d_out), byref(r))
        return _result(r, st)

    def enqueue(self, kv: KvCache, n_past: int, d_trailing: int, s: Sampling, seed: int, frame_index: int) -> None:
        check(lib().navi_frame_enqueue(self.h, kv.ptr(), n_past, c_void_p(d_trailing), byref(s.c()), seed, frame_index))

    def collect(self) -> FrameResult:
        r = capi.FrameResult()
        st = lib().navi_frame_collect(self.h, byref(r))
        return _result(r, st)

    def d_step_out(self) -> int:
        return lib().navi_frame_step_out(self.h)

    def set_step_in(self, d_step: int) -> None:
        check(lib().navi_frame_set_step_in(self.h, c_void_p(d_step)))

    def grid_blocks(self) -> int:
        return lib().navi_frame_grid_blocks(self.h)

    def inspect(self):
        """(hidden [H], logits [TV], clogits [15, CV]) of the last frame, as numpy arrays."""
        import numpy as np
        p = self.w.params
        hid = np.zeros(p.talker.hidden, np.float32)
        lg = np.zeros(p.talker.vocab, np.float32)
        clg = np.zeros((15, p.cp.vocab), np.float32)
        check(lib().navi_frame_inspect(self.h, hid.ctypes.data, lg.ctypes.data, clg.ctypes.data))
        return hid, lg, clg

    def set_profile(self, on: bool = True, cta: int = 0) -> None:
        check(lib().navi_frame_set_profile(self.h, 1 if on else 0, cta))

    def profile_raw(self):
        """Stamps of the last launch on the traced CTA: (start_ns, array [phases, 4] in ns)."""
        import numpy as np
        buf = (ctypes.c_uint64 * (4 * 4096 + 1))()
        n = c_int(0)
        check(lib().navi_frame_profile(self.h, buf, 4 * 4096 + 1, byref(n)))
        a = np.array(buf[:n.value], dtype=np.float64)
        return a[0], a[1:].reshape(-1, 4)

    def profile_all(self):
        """Stamps of the last launch on every CTA (after set_profile(True, -1)):
        (start_ns [G], array [G, phases, 4] in ns)."""
        import numpy as np
        G = self.grid_blocks()
        cap = G * (4 * 4096 + 1)
        buf = (ctypes.c_uint64 * cap)()
        n = c_int(0)
        check(lib().navi_frame_profile(self.h, buf, cap, byref(n)))
        a = np.array(buf[:n.value], dtype=np.float64).reshape(G, -1)
        return a[:, 0], a[:, 1:].reshape(G, -1, 4)

    def profile(self):
        """Per-phase durations (us) of the last launch on the traced CTA."""
        import numpy as np
        t0, st = self.profile_raw()
        ends = np.concatenate([[t0], st[:, 3]])
        return np.diff(ends) / 1000.0

    def close(self):
        if self.h:
            if _open(self.dev, self.w):
                lib().navi_frame_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def sample_logits(dev: Device, d_logits: int, vocab: int, s: Sampling, seed: int, frame_index: int, codebook: int,
                  suppress_from: int = 0, eos_id: int = -1, d_seen: int = 0) -> int:
    out = c_int32(-1)
    check(lib().navi_sample_logits(dev.h, c_void_p(d_logits), vocab, byref(s.c()), seed, frame_index, codebook, suppress_from,
                                   eos_id, c_void_p(d_seen) if d_seen else None, byref(out)))
    return out.value


def sample_logits_static(dev: Device, d_logits: int, vocab: int, s: Sampling, seed: int, frame_index: int, codebook: int,
                         suppress_from: int = 0, eos_id: int = -1, d_seen: int = 0) -> int:
    """sample_logits without any device allocation (static scratch of the library,
    vocab <= NAVI_SAMPLE_STATIC_MAX_VOCAB)."""
    out = c_int32(-1)
    check(lib().navi_sample_logits_static(dev.h, c_void_p(d_logits), vocab, byref(s.c()), seed, frame_index, codebook,
                                          suppress_from, eos_id, c_void_p(d_seen) if d_seen else None, byref(out)))
    return out.value
