"""HTTP front end over the engine (the reference's runtime/server/server.cpp, runtime/voices/store.cpp):
the OpenAI speech dialect and the XTTS dialect, streaming as a chunked WAV / raw s16le body or as
server-sent events, Prometheus `/metrics`, a persistent voice store, one worker thread that owns
the GPU and runs one request at a time.

    python -m navi_b200.serve --model model.navi --voices VOICES_DIR [--port 8080] [--xtts-port 8020]

What differs from the reference:

* cloning a voice from a reference WAV needs the speaker encoder, which this build does not
  have: `POST /v1/audio/voices` (and the XTTS clone routes) take the speaker embedding itself
  (an `embedding` part holding little-endian f32 or a .npy file) and answer 501 for a WAV
  alone. Voices stored by the reference (`<id>/embedding.f32`) load unchanged;
* a client that stops reading a stream stops receiving it, but the utterance runs to its end
  (the engine's PCM callback cannot cancel a request);
* `stream_batch_size` maps to the vocoder batch of `Graph::synth` as in the reference; the
  first batch is 4 frames.

Everything else (routes, request fields and their defaults and limits, error bodies, voice
resolution, XTTS seeds, metric names) follows the reference.
"""
from __future__ import annotations

import argparse
import base64
import hashlib
import io
import json
import os
import queue
import re
import struct
import sys
import threading
import time
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass, field
from datetime import datetime, timezone
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer
from pathlib import Path
from urllib.parse import parse_qs, unquote, urlsplit

import numpy as np

# language codes the OpenAI dialect accepts besides the model's own language names (server.cpp:278-281)
LANG_CODES = {"en": "english", "zh": "chinese", "de": "german", "it": "italian", "pt": "portuguese", "es": "spanish",
              "ja": "japanese", "ko": "korean", "fr": "french", "ru": "russian"}
STREAM_FIRST_BATCH = 4     # frames of the first vocoder batch of a stream
STREAM_BATCH = 16          # default frames per later batch (`stream_batch_size`)
WAV_STREAMING = 0xFFFFFFFF


# ---- audio ---------------------------------------------------------------------------------------

def to_s16(pcm: np.ndarray) -> np.ndarray:
    """f32 PCM -> int16: clamped to [-1, 1], times 32767 in f32, rounded to nearest even (wav.cpp:13-22)."""
    v = np.clip(np.asarray(pcm, dtype=np.float32), np.float32(-1.0), np.float32(1.0)) * np.float32(32767.0)
    return np.rint(v).astype(np.int16)


def wav_header(rate: int, n_samples: int | None) -> bytes:
    """44-byte RIFF/WAVE header of 16-bit mono PCM; n_samples None: the streaming form with both
    sizes 0xFFFFFFFF."""
    data = WAV_STREAMING if n_samples is None else 2 * n_samples
    riff = WAV_STREAMING if n_samples is None else 36 + data
    return struct.pack("<4sI4s4sIHHIIHH4sI", b"RIFF", riff, b"WAVE", b"fmt ", 16, 1, 1, rate, 2 * rate, 2, 16, b"data", data)


def wav_bytes(s16: np.ndarray, rate: int) -> bytes:
    return wav_header(rate, len(s16)) + np.asarray(s16, dtype="<i2").tobytes()


# ---- voices ----------------------------------------------------------------------------------------

def voice_id_for(name: str) -> str:
    """The store id of a registered name: characters other than [A-Za-z0-9_.-] become '_',
    leading dots are dropped, at most 128 characters, "unnamed" when nothing is left
    (store.cpp:133-142)."""
    out = "".join(c if (c.isascii() and (c.isalnum() or c in "_-.")) else "_" for c in name.encode("utf-8").decode("latin-1"))
    out = out.lstrip(".")[:128]
    return out or "unnamed"


@dataclass(frozen=True)
class Voice:
    id: str
    name: str
    embedding: np.ndarray
    ref_text: str = ""
    model: str = ""
    sample_sha256: str = ""
    created: str = ""
    sample_seconds: float = 0.0


class VoiceStore:
    """One directory per voice under `root`: voice.json (name, ref_text, model, sample_sha256,
    dim, created), embedding.f32 (little-endian f32) and, when registered from audio,
    sample.wav -- the reference's layout (store.h:9-12), so either engine reads the other's
    voices. Thread-safe; a voice object is immutable, so a request keeps the one it resolved."""

    def __init__(self, root, dim: int):
        self.root = Path(root)
        self.dim = dim
        self._lock = threading.Lock()
        self._voices: dict[str, Voice] = {}
        self.root.mkdir(parents=True, exist_ok=True)
        for d in sorted(p for p in self.root.iterdir() if p.is_dir()):
            try:
                meta = json.loads((d / "voice.json").read_text("utf-8"))
                emb = np.fromfile(d / "embedding.f32", dtype="<f4")
            except (OSError, ValueError) as e:
                print(f"voices: skipping {d.name}: {e}", file=sys.stderr)
                continue
            if dim > 0 and emb.size != dim:
                print(f"voices: skipping {d.name}: embedding has {emb.size} floats, the model wants {dim}", file=sys.stderr)
                continue
            self._voices[d.name] = Voice(d.name, meta.get("name", d.name), emb.astype(np.float32), meta.get("ref_text", ""),
                                         meta.get("model", ""), meta.get("sample_sha256", ""), meta.get("created", ""),
                                         float(meta.get("sample_seconds", 0.0)))

    def __len__(self) -> int:
        with self._lock:
            return len(self._voices)

    def ids(self) -> list[str]:
        with self._lock:
            return sorted(self._voices)

    def find(self, vid: str) -> Voice | None:
        with self._lock:
            return self._voices.get(vid)

    def put(self, name: str, embedding, ref_text: str = "", model: str = "", sample: bytes = b"") -> tuple[Voice, str]:
        """Adds or replaces the voice `name`; returns (voice, "created" | "replaced" | "exists")."""
        emb = np.ascontiguousarray(np.asarray(embedding, dtype=np.float32).reshape(-1))
        if self.dim > 0 and emb.size != self.dim:
            raise ValueError(f"embedding has {emb.size} floats, the model wants {self.dim}")
        if not np.all(np.isfinite(emb)):
            raise ValueError("embedding holds non-finite values")
        vid = voice_id_for(name)
        sha = hashlib.sha256(sample if sample else emb.astype("<f4").tobytes()).hexdigest()
        with self._lock:
            old = self._voices.get(vid)
            if old is not None and old.sample_sha256 == sha:
                return old, "exists"
            v = Voice(vid, name, emb, ref_text, model, sha, datetime.now(timezone.utc).strftime("%Y-%m-%dT%H:%M:%SZ"))
            d = self.root / vid
            d.mkdir(parents=True, exist_ok=True)
            # payloads first, the manifest last: a voice exists once voice.json does
            _write_atomic(d / "embedding.f32", emb.astype("<f4").tobytes())
            if sample:
                _write_atomic(d / "sample.wav", sample)
            meta = dict(name=name, ref_text=ref_text, model=model, sample_sha256=sha, dim=int(emb.size), created=v.created)
            _write_atomic(d / "voice.json", json.dumps(meta, indent=2).encode())
            self._voices[vid] = v
            return v, "replaced" if old is not None else "created"

    def remove(self, vid: str) -> bool:
        with self._lock:
            if vid not in self._voices:
                return False
            del self._voices[vid]
            d = self.root / vid
            for f in ("voice.json", "embedding.f32", "sample.wav"):
                try:
                    (d / f).unlink()
                except FileNotFoundError:
                    pass
            try:
                d.rmdir()
            except OSError:
                pass
            return True


def _write_atomic(path: Path, data: bytes) -> None:
    tmp = path.with_name(path.name + ".tmp")
    with open(tmp, "wb") as f:
        f.write(data)
        f.flush()
        os.fsync(f.fileno())
    os.replace(tmp, path)


# ---- metrics -------------------------------------------------------------------------------------

class Metrics:
    """Counters and histograms in the Prometheus text format (server.cpp:173-280): requests by
    outcome, errors by kind, frames, audio seconds, time to first audio and real-time factor."""

    TTFA_BUCKETS = (0.05, 0.1, 0.2, 0.3, 0.5, 0.75, 1.0, 2.0, 5.0)
    RTF_BUCKETS = (0.05, 0.1, 0.2, 0.3, 0.5, 0.75, 1.0, 1.5, 2.0)

    def __init__(self):
        self._lock = threading.Lock()
        self.requests_total = 0
        self.requests_processing = 0
        self.errors: dict[str, int] = {}
        self.frames_total = 0
        self.audio_seconds_total = 0.0
        self.generate_seconds_total = 0.0
        self.eos_total = 0
        self.cap_total = 0
        self.clones_total = 0
        self.ttfa = [0] * (len(self.TTFA_BUCKETS) + 1)
        self.ttfa_sum = 0.0
        self.rtf = [0] * (len(self.RTF_BUCKETS) + 1)
        self.rtf_sum = 0.0

    def error(self, kind: str) -> None:
        with self._lock:
            self.errors[kind] = self.errors.get(kind, 0) + 1

    def processing(self, delta: int) -> None:
        with self._lock:
            self.requests_processing += delta

    @staticmethod
    def _observe(counts, buckets, v):
        for i, b in enumerate(buckets):
            if v <= b:
                counts[i] += 1
        counts[-1] += 1

    def observe(self, st: dict) -> None:
        with self._lock:
            self.requests_total += 1
            self.frames_total += st["frames"]
            self.audio_seconds_total += st["audio_seconds"]
            self.generate_seconds_total += st["total_ms"] / 1e3
            if st["eos"]:
                self.eos_total += 1
            else:
                self.cap_total += 1
            self._observe(self.ttfa, self.TTFA_BUCKETS, st["ttfa_ms"] / 1e3)
            self.ttfa_sum += st["ttfa_ms"] / 1e3
            self._observe(self.rtf, self.RTF_BUCKETS, st["rtf"])
            self.rtf_sum += st["rtf"]

    def render(self, model: str, n_voices: int) -> str:
        with self._lock:
            lab = f'model="{model}"'
            out = [
                "# HELP navi_tts_requests_total Speech requests completed.", "# TYPE navi_tts_requests_total counter",
                f"navi_tts_requests_total{{{lab}}} {self.requests_total}",
                "# HELP navi_tts_requests_processing Speech requests queued or running.", "# TYPE navi_tts_requests_processing gauge",
                f"navi_tts_requests_processing{{{lab}}} {self.requests_processing}",
                "# HELP navi_tts_errors_total Failed requests by stage.", "# TYPE navi_tts_errors_total counter",
            ]
            for kind in sorted(self.errors):
                out.append(f'navi_tts_errors_total{{{lab},kind="{kind}"}} {self.errors[kind]}')
            out += [
                "# TYPE navi_tts_frames_total counter", f"navi_tts_frames_total{{{lab}}} {self.frames_total}",
                "# TYPE navi_tts_audio_seconds_total counter", f"navi_tts_audio_seconds_total{{{lab}}} {self.audio_seconds_total:.6f}",
                "# TYPE navi_tts_generate_seconds_total counter",
                f"navi_tts_generate_seconds_total{{{lab}}} {self.generate_seconds_total:.6f}",
                "# TYPE navi_tts_stop_total counter", f'navi_tts_stop_total{{{lab},reason="eos"}} {self.eos_total}',
                f'navi_tts_stop_total{{{lab},reason="cap"}} {self.cap_total}',
                "# TYPE navi_tts_voice_clones_total counter", f"navi_tts_voice_clones_total{{{lab}}} {self.clones_total}",
                "# TYPE navi_tts_voices gauge", f"navi_tts_voices{{{lab}}} {n_voices}",
            ]
            for name, counts, buckets, total in (("navi_tts_ttfa_seconds", self.ttfa, self.TTFA_BUCKETS, self.ttfa_sum),
                                                  ("navi_tts_rtf", self.rtf, self.RTF_BUCKETS, self.rtf_sum)):
                out.append(f"# TYPE {name} histogram")
                for b, c in zip(buckets, counts):
                    out.append(f'{name}_bucket{{{lab},le="{b}"}} {c}')
                out.append(f'{name}_bucket{{{lab},le="+Inf"}} {counts[-1]}')
                out.append(f"{name}_sum{{{lab}}} {total:.6f}")
                out.append(f"{name}_count{{{lab}}} {counts[-1]}")
            return "\n".join(out) + "\n"


# ---- the engine behind the service ---------------------------------------------------------------

@dataclass
class SpeechRequest:
    """What both dialects reduce to (server.cpp:360-398): the validated fields of one utterance."""
    text: str
    voice: Voice
    voice_id: str
    language: str = ""
    seed: int = 0
    max_frames: int = 600
    temperature: float = 0.9
    top_k: int = 50
    repetition_penalty: float = 1.05
    first_batch: int = STREAM_FIRST_BATCH
    vocoder_batch: int = 0


class GraphEngine:
    """The engine a service drives: tokenizer + navi_graph_synth on one device. Every method is
    called from the service's single worker thread."""

    def __init__(self, model: str, ordinal: int = 0, max_frames: int = 4096, deadline_us: int = 0):
        from . import engine
        from .navi_file import NaviFile
        from .tokenizer import Tokenizer
        self._engine = engine
        self.dev = engine.Device(ordinal)
        self.w = engine.Weights(self.dev, model)
        self.p = self.w.params
        kv = NaviFile.open(model).kv
        self.languages = {k[len("talker.language."):]: v for k, v in kv.items() if k.startswith("talker.language.")}
        self.tokenizer = Tokenizer.from_navi(model)
        self.graph = engine.Graph(self.dev, self.w, max_frames=max_frames, deadline_us=deadline_us)
        self.sample_rate = self.p.sample_rate
        self.samples_per_frame = self.p.codec_upsample
        self.speaker_dim = self.p.talker.hidden
        self.defaults = dict(temperature=self.p.temperature, top_k=self.p.top_k, repetition_penalty=self.p.repetition_penalty)

    def synth(self, r: SpeechRequest, on_pcm) -> dict:
        """Runs one utterance; on_pcm(np.ndarray f32) sees each vocoder batch. Returns its stats."""
        ids = self.tokenizer.prompt_ids(r.text)
        s = self._engine.Sampling(temperature=r.temperature, top_k=r.top_k, repetition_penalty=r.repetition_penalty,
                                  cp_temperature=self.p.cp_temperature, cp_top_k=self.p.cp_top_k)
        # batch sizes 0: the vocoder's largest chunk (the PCM is the same for any batching)
        _, _, st, _ = self.graph.synth(ids, r.language, r.voice.embedding, s, r.seed, r.max_frames, r.first_batch, r.vocoder_batch,
                                       on_pcm=on_pcm)
        return dict(tokens=st.n_tokens, frames=st.n_frames, eos=bool(st.eos), audio_seconds=st.audio_s, prefill_ms=st.prefill_ms,
                    frames_ms=st.frames_ms, vocoder_ms=st.vocoder_ms, ttfa_ms=st.ttfa_ms, total_ms=st.total_ms, rtf=st.rtf)


# ---- the service: validation, the worker, streaming ------------------------------------------------

class HttpError(Exception):
    def __init__(self, status: int, message: str, kind: str = "invalid_request_error"):
        super().__init__(message)
        self.status, self.message, self.kind = status, message, kind


class PcmQueue:
    """Bounded queue of s16 batches between the worker and one streaming response
    (server.cpp:100-160). The worker blocks while the client is behind; after the client
    leaves, batches are dropped."""

    def __init__(self, depth: int = 64):
        self._q: queue.Queue = queue.Queue(maxsize=depth)
        self._first = threading.Event()
        self.aborted = False
        self.error = ""
        self.pushed = 0

    def push(self, s16: np.ndarray) -> None:
        self.pushed += 1
        self._first.set()
        while not self.aborted:
            try:
                self._q.put(s16, timeout=0.5)
                return
            except queue.Full:
                continue

    def finish(self, error: str = "") -> None:
        self.error = error
        self._first.set()
        while not self.aborted:
            try:
                self._q.put(None, timeout=0.5)
                return
            except queue.Full:
                continue

    def wait_first(self) -> bool:
        """True once a batch is queued; False when the request ended without audio."""
        self._first.wait()
        return self.pushed > 0

    def pop(self):
        return self._q.get()

    def abort(self) -> None:
        self.aborted = True


class Service:
    """Everything the handlers share: the engine (driven by one worker thread), the voice store,
    the metrics and the options (server.h:17-28)."""

    def __init__(self, engine, store: VoiceStore, model_id: str, default_voice: str = "", max_input_chars: int = 4096,
                 max_audio_tokens: int = 600, xtts_fallback_male: str = "default", xtts_fallback_female: str = "default",
                 verbose: bool = False):
        self.engine, self.store, self.model_id = engine, store, model_id
        self.default_voice, self.max_input_chars, self.max_audio_tokens = default_voice, max_input_chars, max_audio_tokens
        self.xtts_fallback_male, self.xtts_fallback_female, self.verbose = xtts_fallback_male, xtts_fallback_female, verbose
        self.metrics = Metrics()
        self.worker = ThreadPoolExecutor(max_workers=1, thread_name_prefix="navi-gpu")
        self._rng = np.random.default_rng()
        self._rng_lock = threading.Lock()

    def random_seed(self) -> int:
        with self._rng_lock:
            return int(self._rng.integers(0, 1 << 63))

    def resolve_voice(self, vid: str) -> Voice | None:
        """"default" (or empty) -> the configured default, else voice_1, else the first id."""
        if vid and vid != "default":
            return self.store.find(vid)
        if self.default_voice:
            return self.store.find(self.default_voice)
        v = self.store.find("voice_1")
        if v is not None:
            return v
        ids = self.store.ids()
        return self.store.find(ids[0]) if ids else None

    def resolve_language(self, lang: str) -> str:
        """"" for auto; the model's language name for a name or a code it knows (server.cpp:283-292)."""
        if not lang or lang == "auto":
            return ""
        s = lang.lower()
        if s in self.engine.languages:
            return s
        if s in LANG_CODES and LANG_CODES[s] in self.engine.languages:
            return LANG_CODES[s]
        raise HttpError(400, f"unknown language '{lang}'")

    def prepare(self, text: str, voice_id: str, language: str) -> SpeechRequest:
        try:
            if not text:
                raise HttpError(400, "'input' is empty")
            if len(text.encode("utf-8")) > self.max_input_chars:
                raise HttpError(400, f"'input' exceeds {self.max_input_chars} characters")
            lang = self.resolve_language(language)
            voice = self.resolve_voice(voice_id)
            if voice is None:
                raise HttpError(400, "no voices registered: POST /v1/audio/voices a speaker embedding first" if len(self.store) == 0
                                else f"unknown voice '{voice_id}'")
        except HttpError:
            self.metrics.error("request")
            raise
        d = self.engine.defaults
        return SpeechRequest(text=text, voice=voice, voice_id=voice_id, language=lang, max_frames=self.max_audio_tokens,
                             temperature=d["temperature"], top_k=d["top_k"], repetition_penalty=d["repetition_penalty"])

    def speak(self, r: SpeechRequest) -> tuple[np.ndarray, dict]:
        """The whole utterance on the worker: (s16 PCM, stats). Vocoder batches of the largest size."""
        r.first_batch = r.vocoder_batch = 0
        chunks = []
        self.metrics.processing(1)
        try:
            st = self.worker.submit(self.engine.synth, r, lambda pcm: chunks.append(to_s16(pcm))).result()
        except Exception:
            self.metrics.error("generate")
            raise
        finally:
            self.metrics.processing(-1)
        self.metrics.observe(st)
        self.log(r, st)
        return (np.concatenate(chunks) if chunks else np.zeros(0, np.int16)), st

    def speak_stream(self, r: SpeechRequest) -> tuple[PcmQueue, dict]:
        """Queues the utterance on the worker; its batches arrive in the returned queue, its
        stats in the dict once the queue is finished."""
        q, st = PcmQueue(), {}
        self.metrics.processing(1)

        def job():
            err = ""
            try:
                st.update(self.engine.synth(r, lambda pcm: q.push(to_s16(pcm))))
            except Exception as e:   # the request fails, the service goes on
                err = str(e) or type(e).__name__
            q.finish(err)
            self.metrics.processing(-1)
            if err:
                self.metrics.error("stream" if q.aborted else "generate")
            else:
                self.metrics.observe(st)
                self.log(r, st)

        self.worker.submit(job)
        return q, st

    def log(self, r: SpeechRequest, st: dict) -> None:
        if self.verbose:
            print(f"speech {r.voice_id} seed {r.seed}: {st['tokens']} tokens, {st['frames']} frames ({'eos' if st['eos'] else 'cap'}), "
                  f"prefill {st['prefill_ms']:.1f} frames {st['frames_ms']:.1f} vocoder {st['vocoder_ms']:.1f} | "
                  f"{st['audio_seconds']:.2f} s audio in {st['total_ms']:.0f} ms, RTF {st['rtf']:.3f}", file=sys.stderr)

    def register(self, name: str, embedding: np.ndarray, ref_text: str = "") -> tuple[Voice, str]:
        v, status = self.store.put(name, embedding, ref_text, self.model_id)
        if status != "exists":
            with self.metrics._lock:
                self.metrics.clones_total += 1
        return v, status

    @staticmethod
    def stable_seed(speaker: str) -> int:
        """XTTS: one fixed seed per speaker name, the first 32 bits of its SHA-256 (server.cpp:665-668)."""
        return int(hashlib.sha256(speaker.encode("utf-8")).hexdigest()[:8], 16)

    def resolve_xtts_speaker(self, speaker: str) -> tuple[Voice | None, str]:
        if speaker:
            used = voice_id_for(speaker)
            v = self.store.find(used)
            if v is not None:
                return v, used
        used = self.xtts_fallback_male if speaker.lower().startswith("male") else self.xtts_fallback_female
        return self.resolve_voice(used), used


# ---- HTTP --------------------------------------------------------------------------------------------

def parse_multipart(body: bytes, content_type: str) -> tuple[dict[str, str], dict[str, tuple[str, bytes]]]:
    """multipart/form-data -> (fields, files {name: (filename, bytes)})."""
    m = re.search(r'boundary="?([^";]+)"?', content_type)
    if not m:
        raise HttpError(400, "multipart body without a boundary")
    sep = b"--" + m.group(1).encode()
    fields, files = {}, {}
    for part in body.split(sep)[1:]:
        if part.startswith(b"--"):
            break
        part = part[2:] if part.startswith(b"\r\n") else part
        head, _, data = part.partition(b"\r\n\r\n")
        data = data[:-2] if data.endswith(b"\r\n") else data
        disp = next((h for h in head.decode("utf-8", "replace").split("\r\n") if h.lower().startswith("content-disposition")), "")
        name = re.search(r'\bname="([^"]*)"', disp)
        fname = re.search(r'\bfilename="([^"]*)"', disp)
        if not name:
            continue
        if fname or name.group(1) == "embedding":   # an embedding is bytes even without a file name
            files[name.group(1)] = (fname.group(1) if fname else "", data)
        else:
            fields[name.group(1)] = data.decode("utf-8", "replace")
    return fields, files


def embedding_of(data: bytes) -> np.ndarray:
    """A speaker embedding upload: a .npy file or raw little-endian f32."""
    if data[:6] == b"\x93NUMPY":
        return np.load(io.BytesIO(data), allow_pickle=False).astype(np.float32).reshape(-1)
    if len(data) % 4:
        raise HttpError(400, "embedding: expected a .npy file or little-endian f32 bytes")
    return np.frombuffer(data, dtype="<f4").astype(np.float32)


def is_riff(b: bytes) -> bool:
    return len(b) >= 12 and b[:4] == b"RIFF"


XTTS_OK_ROUTES = ("/", "/docs", "/get_folders", "/get_models_list", "/sample", "/get_tts_settings")
XTTS_TTS_ROUTES = ("/tts_to_audio", "/tts_to_audio/", "/tts_stream", "/tts_stream/", "/tts_to_file", "/tts_to_file/")
XTTS_CLONE_ROUTES = ("/create_and_store_latents", "/create_and_store_latents/", "/clone_speaker", "/set_speaker", "/upload_speaker")
NO_ENCODER = "cloning from audio needs the speaker encoder, which this engine does not include: send the speaker embedding as an 'embedding' part"


def make_handler(svc: Service):
    class Handler(BaseHTTPRequestHandler):
        protocol_version = "HTTP/1.1"
        server_version = "navi-b200"

        def log_message(self, fmt, *args):
            if svc.verbose:
                super().log_message(fmt, *args)

        # -- plumbing
        def _body(self) -> bytes:
            n = int(self.headers.get("Content-Length") or 0)
            if n > (64 << 20):
                raise HttpError(413, "request body too large")
            return self.rfile.read(n) if n > 0 else b""

        def _send(self, status: int, body: bytes, ctype: str, headers=()):
            self.send_response(status)
            self.send_header("Content-Type", ctype)
            self.send_header("Content-Length", str(len(body)))
            for k, v in headers:
                self.send_header(k, v)
            self.end_headers()
            self.wfile.write(body)

        def _json(self, obj, status: int = 200):
            self._send(status, json.dumps(obj).encode(), "application/json")

        def _error(self, e: HttpError, xtts: bool = False):
            body = {"error": e.message} if xtts else {"error": {"message": e.message, "type": e.kind}}
            self._json(body, e.status)

        def _chunk(self, data: bytes) -> bool:
            try:
                self.wfile.write(b"%x\r\n%s\r\n" % (len(data), data))
                self.wfile.flush()
                return True
            except OSError:
                return False

        def _route(self):
            u = urlsplit(self.path)
            return unquote(u.path), {k: v[-1] for k, v in parse_qs(u.query).items()}

        # -- verbs
        def do_GET(self):
            path, _ = self._route()
            if path == "/metrics":
                return self._send(200, svc.metrics.render(svc.model_id, len(svc.store)).encode(), "text/plain; version=0.0.4")
            if path == "/health" or path in XTTS_OK_ROUTES:
                return self._json({"status": "ok", "model": svc.model_id, "voices": len(svc.store)})
            if path == "/v1/models":
                return self._json({"object": "list", "data": [{"id": svc.model_id, "object": "model", "owned_by": "navi-tts"}]})
            if path == "/v1/audio/languages":
                langs = [{"code": c, "name": n, "id": svc.engine.languages[n]} for c, n in sorted(LANG_CODES.items())
                         if n in svc.engine.languages]
                return self._json({"languages": langs})
            if path == "/languages":
                return self._json([c for c, n in sorted(LANG_CODES.items()) if n in svc.engine.languages])
            if path == "/v1/audio/voices":
                ids = (["default"] if svc.resolve_voice("default") is not None else []) + svc.store.ids()
                return self._json({svc.model_id: ids})
            if path == "/speakers":
                return self._json(svc.store.ids())
            if path == "/speakers_list":
                return self._json({i: {"speaker_name": i} for i in svc.store.ids()})
            self._error(HttpError(404, f"no route GET {path}"))

        def do_DELETE(self):
            path, _ = self._route()
            m = re.fullmatch(r"/v1/audio/voices/(.+)", path)
            if not m:
                return self._error(HttpError(404, f"no route DELETE {path}"))
            if not svc.store.remove(m.group(1)):
                return self._error(HttpError(404, "no such voice"))
            self._json({"deleted": True})

        def do_POST(self):
            path, query = self._route()
            xtts = path in XTTS_TTS_ROUTES or path in XTTS_CLONE_ROUTES
            try:
                body = self._body()
                if path == "/v1/audio/speech":
                    return self._speech(body)
                if path == "/v1/audio/voices":
                    return self._register(body, query, xtts=False)
                if path in XTTS_TTS_ROUTES:
                    return self._xtts_tts(body, query)
                if path in XTTS_CLONE_ROUTES:
                    return self._register(body, query, xtts=True)
                raise HttpError(404, f"no route POST {path}")
            except HttpError as e:
                self._error(e, xtts)
            except Exception as e:   # an engine failure: the request fails, the server goes on
                self._error(HttpError(500, str(e) or type(e).__name__, "engine_error"), xtts)

        # -- OpenAI dialect
        def _speech(self, raw: bytes):
            try:
                body = json.loads(raw or b"null")
            except ValueError:
                raise HttpError(400, "invalid JSON")
            if not isinstance(body, dict) or not isinstance(body.get("input"), str):
                raise HttpError(400, "'input' is required")
            r = svc.prepare(body["input"], str(body.get("voice", "default")), str(body.get("language", "en")))

            def num(key, default, kind):
                v = body.get(key, default)
                if isinstance(v, bool) or not isinstance(v, (int, float)):
                    raise HttpError(400, f"'{key}' must be a number")
                return kind(v)

            r.seed = num("seed", 0, int) if "seed" in body else svc.random_seed()
            r.max_frames = num("max_audio_tokens", svc.max_audio_tokens, int)
            if not 1 <= r.max_frames <= 4096:
                raise HttpError(400, "'max_audio_tokens' out of range")
            r.temperature = num("temperature", r.temperature, float)
            r.top_k = num("top_k", r.top_k, int)
            r.repetition_penalty = num("repetition_penalty", r.repetition_penalty, float)
            fmt = body.get("response_format", "wav")
            if fmt not in ("wav", "pcm"):
                raise HttpError(400, "'response_format' must be wav or pcm")
            stream = body.get("stream_format", "")
            rate = svc.engine.sample_rate
            if stream in ("audio", "sse"):
                # batching changes when the PCM arrives, not the PCM: a small first batch for the
                # time to first audio, then bigger ones for the vocoder's sake
                r.vocoder_batch = num("stream_batch_size", STREAM_BATCH, int)
                if not 1 <= r.vocoder_batch <= 64:
                    raise HttpError(400, "'stream_batch_size' out of range (1-64)")
                r.first_batch = min(STREAM_FIRST_BATCH, r.vocoder_batch)
                return self._stream(r, stream == "sse", fmt == "pcm", rate)
            if stream:
                raise HttpError(400, "'stream_format' must be audio or sse")
            s16, _ = svc.speak(r)   # whole body: the vocoder's largest batch is the cheapest
            if fmt == "pcm":
                return self._send(200, s16.astype("<i2").tobytes(), "audio/pcm")
            self._send(200, wav_bytes(s16, rate), "audio/wav")

        def _stream(self, r: SpeechRequest, sse: bool, raw_pcm: bool, rate: int):
            """Chunked response; the headers go out with the first batch (or the failure), so an
            early error is still an HTTP status and the headers' arrival is the time to first audio."""
            q, st = svc.speak_stream(r)
            if not q.wait_first():
                raise HttpError(500, q.error or "no audio produced", "engine_error")
            self.send_response(200)
            self.send_header("Content-Type", "text/event-stream" if sse else "audio/pcm" if raw_pcm else "audio/wav")
            self.send_header("Transfer-Encoding", "chunked")
            if sse:
                self.send_header("Cache-Control", "no-cache")
            self.end_headers()
            ok = True
            if not sse and not raw_pcm:
                ok = self._chunk(wav_header(rate, None))
            while ok:
                batch = q.pop()
                if batch is None:
                    break
                if sse:
                    ev = {"type": "speech.audio.delta", "audio": base64.b64encode(batch.astype("<i2").tobytes()).decode()}
                    ok = self._chunk(f"data: {json.dumps(ev)}\n\n".encode())
                else:
                    ok = self._chunk(batch.astype("<i2").tobytes())
            if not ok:
                q.abort()
                self.close_connection = True
                return
            if sse:
                if q.error:
                    ev = {"type": "error", "error": q.error}
                else:
                    ev = {"type": "speech.audio.done",
                          "usage": {"input_tokens": st["tokens"], "output_tokens": st["frames"],
                                    "total_tokens": st["tokens"] + st["frames"]},
                          "navi": {"frames": st["frames"], "eos": st["eos"], "audio_seconds": st["audio_seconds"],
                                   "prefill_ms": st["prefill_ms"], "frames_ms": st["frames_ms"], "vocoder_ms": st["vocoder_ms"],
                                   "ttfa_ms": st["ttfa_ms"], "total_ms": st["total_ms"], "rtf": st["rtf"]}}
                self._chunk(f"data: {json.dumps(ev)}\n\n".encode())
            self._chunk(b"")

        def _register(self, raw: bytes, query: dict, xtts: bool):
            ctype = self.headers.get("Content-Type", "")
            fields, files = parse_multipart(raw, ctype) if ctype.startswith("multipart/") else ({}, {})
            keys = ("speaker_name", "name", "speaker", "voice_name") if xtts else ("name",)
            name = next((fields.get(k) or query.get(k) for k in keys if fields.get(k) or query.get(k)), "")
            ref_text = next((fields[k] for k in ("ref_text", "text") if k in fields), "")
            emb = files.get("embedding")
            audio = next((f for k, f in files.items() if k != "embedding" and is_riff(f[1])), None)
            if emb is None:
                if audio is not None or is_riff(raw):
                    raise HttpError(501, NO_ENCODER, "not_implemented")
                raise HttpError(400, "need a speaker name and an 'embedding' part" if xtts else
                                "multipart field 'embedding' (little-endian f32 or .npy) is required")
            if not name:
                if xtts:
                    raise HttpError(400, "need a speaker embedding and a speaker name")
                name = emb[0] or "voice"
            try:
                v, status = svc.register(name, embedding_of(emb[1]), ref_text)
            except ValueError as e:
                svc.metrics.error("clone")
                raise HttpError(400, str(e))
            if xtts:
                return self._json({"status": "ok", "speaker_name": name, "name": name, "voice_id": v.id, "latents": v.id,
                                   "message": status})
            self._json({"id": v.id, "name": v.name, "status": status})

        # -- XTTS dialect: {text, speaker_wav (the speaker's name), language} -> audio/wav
        def _xtts_tts(self, raw: bytes, query: dict):
            ctype = self.headers.get("Content-Type", "")
            body = None
            try:
                body = json.loads(raw) if raw else None
            except ValueError:
                pass
            fields = parse_multipart(raw, ctype)[0] if ctype.startswith("multipart/") else {}
            if ctype.startswith("application/x-www-form-urlencoded"):
                fields = {k: v[-1] for k, v in parse_qs(raw.decode("utf-8", "replace")).items()}

            def field(*keys):
                for k in keys:
                    if isinstance(body, dict) and isinstance(body.get(k), str):
                        return body[k]
                    if k in fields:
                        return fields[k]
                    if k in query:
                        return query[k]
                return ""

            text = field("text", "input")
            speaker = field("speaker_wav", "speaker", "speaker_name", "voice")
            language = (field("language") or "en").split("-")[0]
            if not text.strip():
                raise HttpError(400, "empty text")
            voice, used = svc.resolve_xtts_speaker(speaker)
            if voice is None:
                raise HttpError(400, f"no voice for speaker '{speaker}' and no fallback registered")
            r = svc.prepare(text, used, language)
            r.seed = Service.stable_seed(speaker or used)
            s16, _ = svc.speak(r)
            self._send(200, wav_bytes(s16, svc.engine.sample_rate), "audio/wav")

    return Handler


def serve(svc: Service, host: str = "127.0.0.1", port: int = 8080, xtts_port: int = 0):
    """Listening servers on port (and xtts_port) over svc; returns them, already serving on
    background threads."""
    servers = []
    for p in [port] + ([xtts_port] if xtts_port else []):
        s = ThreadingHTTPServer((host, p), make_handler(svc))
        s.daemon_threads = True
        threading.Thread(target=s.serve_forever, daemon=True).start()
        servers.append(s)
    return servers


def warm_up(svc: Service) -> None:
    """One short utterance before listening, so the first real request runs at steady state
    (server.cpp:771-793)."""
    ids = svc.store.ids()
    spk = svc.store.find(ids[0]).embedding if ids else np.zeros(svc.engine.speaker_dim, np.float32)
    d = svc.engine.defaults
    r = SpeechRequest(text="Warm up.", voice=Voice("warmup", "warmup", spk), voice_id="warmup", max_frames=16,
                      temperature=d["temperature"], top_k=d["top_k"], repetition_penalty=d["repetition_penalty"])
    t0 = time.perf_counter()
    st = svc.worker.submit(svc.engine.synth, r, lambda pcm: None).result()
    if svc.verbose:
        print(f"warm-up: {st['frames']} frames in {(time.perf_counter() - t0) * 1e3:.0f} ms", file=sys.stderr)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="navi-b200 HTTP server (OpenAI and XTTS speech dialects)")
    ap.add_argument("--model", required=True)
    ap.add_argument("--voices", default="voices")
    ap.add_argument("--default-voice", default="")
    ap.add_argument("--model-id", default="")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8080)
    ap.add_argument("--xtts-port", type=int, default=0)
    ap.add_argument("--xtts-fallback-male", default="default")
    ap.add_argument("--xtts-fallback-female", default="default")
    ap.add_argument("--max-frames", type=int, default=600)
    ap.add_argument("--device", type=int, default=0)
    ap.add_argument("--no-warmup", action="store_true")
    ap.add_argument("-V", "--verbose", action="store_true")
    a = ap.parse_args(argv)
    eng = GraphEngine(a.model, a.device)
    model_id = a.model_id or Path(a.model).stem
    store = VoiceStore(a.voices, eng.speaker_dim)
    svc = Service(eng, store, model_id, a.default_voice, max_audio_tokens=a.max_frames, xtts_fallback_male=a.xtts_fallback_male,
                  xtts_fallback_female=a.xtts_fallback_female, verbose=a.verbose)
    if not a.no_warmup:
        warm_up(svc)
    servers = serve(svc, a.host, a.port, a.xtts_port)
    print(f"navi-b200 serving {model_id} on http://{a.host}:{a.port}"
          f"{f' and :{a.xtts_port} (xtts)' if a.xtts_port else ''}, {len(store)} voice(s) in {store.root}", file=sys.stderr)
    try:
        threading.Event().wait()
    except KeyboardInterrupt:
        pass
    for s in servers:
        s.shutdown()
    return 0


if __name__ == "__main__":
    sys.exit(main())
