"""The HTTP front end (navi_b200.serve, the reference's runtime/server/server.cpp and
runtime/voices/store.cpp) on the CPU, over a fake engine that makes deterministic PCM: routes
of both dialects, request validation and its error bodies, whole-body and streamed audio
(chunked WAV, raw s16le, server-sent events), the voice store and its on-disk layout, voice
resolution and XTTS fallbacks and seeds, metrics, and an engine failure that the server
survives. The same server over the real engine is tested on the GPU in test_serve_gpu.py.
"""
import base64
import hashlib
import http.client
import io
import json
import struct

import numpy as np
import pytest

from navi_b200 import serve

SPF = 240


class FakeEngine:
    """Frames of a ramp whose slope is the seed: frame f of the utterance holds SPF samples."""

    def __init__(self):
        self.languages = {"english": 2050, "chinese": 2055, "german": 2053}
        self.sample_rate = 24000
        self.speaker_dim = 8
        self.defaults = dict(temperature=0.9, top_k=50, repetition_penalty=1.05)
        self.requests = []
        self.fail_next = False

    def pcm(self, r):
        n = min(r.max_frames, 3 + len(r.text) % 5)
        t = np.arange(n * SPF, dtype=np.float32)
        return (np.sin(t * 1e-3 * (1 + r.seed % 7)) * 0.5 + r.voice.embedding[0] * 0.1).astype(np.float32), n

    def synth(self, r, on_pcm):
        self.requests.append(r)
        if self.fail_next:
            self.fail_next = False
            raise RuntimeError("device wait timed out")
        pcm, n = self.pcm(r)
        step = r.vocoder_batch if r.vocoder_batch > 0 else 64
        f0 = r.first_batch if r.first_batch > 0 else step
        at = 0
        while at < n:
            k = min(f0 if at == 0 else step, n - at)
            on_pcm(pcm[at * SPF:(at + k) * SPF])
            at += k
        return dict(tokens=len(r.text) + 8, frames=n, eos=n < r.max_frames, audio_seconds=n * SPF / 24000, prefill_ms=1.0,
                    frames_ms=2.0 * n, vocoder_ms=0.5, ttfa_ms=4.0, total_ms=10.0, rtf=0.1)


@pytest.fixture
def server(tmp_path):
    eng = FakeEngine()
    store = serve.VoiceStore(tmp_path / "voices", eng.speaker_dim)
    store.put("voice_1", np.full(8, 0.5, np.float32))
    store.put("femaleeventoned", np.full(8, -0.5, np.float32))
    svc = serve.Service(eng, store, "navi-test")
    (srv,) = serve.serve(svc, "127.0.0.1", 0)
    yield svc, eng, srv.server_address[1]
    srv.shutdown()
    svc.worker.shutdown()


def req(port, method, path, body=None, headers=None):
    c = http.client.HTTPConnection("127.0.0.1", port, timeout=30)
    if isinstance(body, (dict, list)):
        body = json.dumps(body).encode()
        headers = {"Content-Type": "application/json", **(headers or {})}
    c.request(method, path, body=body, headers=headers or {})
    r = c.getresponse()
    data = r.read()
    c.close()
    return r.status, dict(r.getheaders()), data


def multipart(fields=None, files=None):
    b = "----navitestboundary"
    out = io.BytesIO()
    for k, v in (fields or {}).items():
        out.write(f'--{b}\r\nContent-Disposition: form-data; name="{k}"\r\n\r\n{v}\r\n'.encode())
    for k, (fn, data) in (files or {}).items():
        out.write(f'--{b}\r\nContent-Disposition: form-data; name="{k}"; filename="{fn}"\r\n'
                  f"Content-Type: application/octet-stream\r\n\r\n".encode() + data + b"\r\n")
    out.write(f"--{b}--\r\n".encode())
    return out.getvalue(), {"Content-Type": f"multipart/form-data; boundary={b}"}


def wav_pcm(data):
    assert data[:4] == b"RIFF" and data[8:16] == b"WAVEfmt "
    ch, rate = struct.unpack("<HI", data[22:28])
    assert (ch, rate) == (1, 24000)
    return np.frombuffer(data[44:], dtype="<i2")


def test_info_routes(server):
    svc, eng, port = server
    assert json.loads(req(port, "GET", "/health")[2]) == {"status": "ok", "model": "navi-test", "voices": 2}
    assert json.loads(req(port, "GET", "/v1/models")[2])["data"][0]["id"] == "navi-test"
    langs = json.loads(req(port, "GET", "/v1/audio/languages")[2])["languages"]
    assert {(l["code"], l["name"], l["id"]) for l in langs} == {("en", "english", 2050), ("zh", "chinese", 2055), ("de", "german", 2053)}
    assert json.loads(req(port, "GET", "/v1/audio/voices")[2]) == {"navi-test": ["default", "femaleeventoned", "voice_1"]}
    assert json.loads(req(port, "GET", "/speakers")[2]) == ["femaleeventoned", "voice_1"]
    assert json.loads(req(port, "GET", "/languages")[2]) == ["de", "en", "zh"]
    for p in serve.XTTS_OK_ROUTES:
        assert req(port, "GET", p)[0] == 200
    st, _, body = req(port, "GET", "/nope")
    assert st == 404 and json.loads(body)["error"]["type"] == "invalid_request_error"


def test_speech_wav_and_pcm(server):
    svc, eng, port = server
    st, h, body = req(port, "POST", "/v1/audio/speech", {"input": "Hello there.", "voice": "voice_1", "seed": 3})
    assert st == 200 and h["Content-Type"] == "audio/wav"
    r = eng.requests[-1]
    assert (r.seed, r.voice.id, r.language, r.max_frames, r.first_batch, r.vocoder_batch) == (3, "voice_1", "english", 600, 0, 0)
    pcm, _ = eng.pcm(r)
    assert np.array_equal(wav_pcm(body), serve.to_s16(pcm))
    st, h, raw = req(port, "POST", "/v1/audio/speech", {"input": "Hello there.", "voice": "voice_1", "seed": 3, "response_format": "pcm"})
    assert st == 200 and h["Content-Type"] == "audio/pcm" and raw == body[44:]
    # defaults: voice_1 for "default", a random seed, the model's sampling
    req(port, "POST", "/v1/audio/speech", {"input": "Hi", "temperature": 0.7, "top_k": 20, "language": "zh"})
    r = eng.requests[-1]
    assert r.voice.id == "voice_1" and (r.temperature, r.top_k, r.repetition_penalty, r.language) == (0.7, 20, 1.05, "chinese")


@pytest.mark.parametrize("body, msg", [
    ({"voice": "voice_1"}, "'input' is required"),
    ({"input": ""}, "'input' is empty"),
    ({"input": "x" * 4097}, "exceeds 4096"),
    ({"input": "hi", "language": "xx"}, "unknown language 'xx'"),
    ({"input": "hi", "voice": "nobody"}, "unknown voice 'nobody'"),
    ({"input": "hi", "max_audio_tokens": 0}, "'max_audio_tokens' out of range"),
    ({"input": "hi", "max_audio_tokens": 5000}, "'max_audio_tokens' out of range"),
    ({"input": "hi", "response_format": "mp3"}, "'response_format' must be wav or pcm"),
    ({"input": "hi", "stream_format": "ws"}, "'stream_format' must be audio or sse"),
    ({"input": "hi", "stream_format": "sse", "stream_batch_size": 65}, "out of range (1-64)"),
    ({"input": "hi", "top_k": "many"}, "'top_k' must be a number"),
])
def test_speech_validation(server, body, msg):
    svc, eng, port = server
    st, _, data = req(port, "POST", "/v1/audio/speech", body)
    err = json.loads(data)["error"]
    assert st == 400 and msg in err["message"] and err["type"] == "invalid_request_error"
    assert req(port, "POST", "/v1/audio/speech", b"{not json", {"Content-Type": "application/json"})[0] == 400


def test_stream_audio_equals_whole_body(server):
    svc, eng, port = server
    body = {"input": "Streaming text!", "voice": "voice_1", "seed": 9}
    whole = req(port, "POST", "/v1/audio/speech", body)[2]
    st, h, streamed = req(port, "POST", "/v1/audio/speech", {**body, "stream_format": "audio", "stream_batch_size": 2})
    assert st == 200 and h["Transfer-Encoding"] == "chunked"
    assert struct.unpack("<I", streamed[4:8])[0] == 0xFFFFFFFF and struct.unpack("<I", streamed[40:44])[0] == 0xFFFFFFFF
    assert streamed[44:] == whole[44:]
    assert (eng.requests[-1].first_batch, eng.requests[-1].vocoder_batch) == (2, 2)
    st, h, raw = req(port, "POST", "/v1/audio/speech", {**body, "stream_format": "audio", "response_format": "pcm"})
    assert h["Content-Type"] == "audio/pcm" and raw == whole[44:]


def test_stream_sse(server):
    svc, eng, port = server
    body = {"input": "Events", "voice": "femaleeventoned", "seed": 5, "stream_format": "sse"}
    st, h, data = req(port, "POST", "/v1/audio/speech", body)
    assert st == 200 and h["Content-Type"] == "text/event-stream"
    events = [json.loads(e[len("data: "):]) for e in data.decode().split("\n\n") if e]
    deltas = [e for e in events if e["type"] == "speech.audio.delta"]
    pcm = np.concatenate([np.frombuffer(base64.b64decode(e["audio"]), "<i2") for e in deltas])
    assert np.array_equal(pcm, serve.to_s16(eng.pcm(eng.requests[-1])[0]))
    done = events[-1]
    assert done["type"] == "speech.audio.done" and done["navi"]["frames"] == len(pcm) // SPF
    assert done["usage"]["total_tokens"] == done["usage"]["input_tokens"] + done["usage"]["output_tokens"]


def test_engine_failure_then_recovery(server):
    svc, eng, port = server
    eng.fail_next = True
    st, _, data = req(port, "POST", "/v1/audio/speech", {"input": "boom"})
    assert st == 500 and json.loads(data)["error"] == {"message": "device wait timed out", "type": "engine_error"}
    eng.fail_next = True
    st, _, data = req(port, "POST", "/v1/audio/speech", {"input": "boom", "stream_format": "sse"})
    assert st == 500 and "timed out" in json.loads(data)["error"]["message"]
    assert req(port, "POST", "/v1/audio/speech", {"input": "fine"})[0] == 200
    m = req(port, "GET", "/metrics")[2].decode()
    assert 'navi_tts_errors_total{model="navi-test",kind="generate"} 2' in m
    assert 'navi_tts_requests_total{model="navi-test"} 1' in m and 'navi_tts_requests_processing{model="navi-test"} 0' in m


def test_voice_register_replace_delete(server, tmp_path):
    svc, eng, port = server
    emb = np.linspace(-1, 1, 8).astype(np.float32)
    npy = io.BytesIO()
    np.save(npy, emb)
    body, h = multipart({"name": "Lydia the Housecarl"}, {"embedding": ("lydia.npy", npy.getvalue())})
    st, _, data = req(port, "POST", "/v1/audio/voices", body, h)
    assert st == 200 and json.loads(data) == {"id": "Lydia_the_Housecarl", "name": "Lydia the Housecarl", "status": "created"}
    assert json.loads(req(port, "POST", "/v1/audio/voices", body, h)[2])["status"] == "exists"
    body2, h2 = multipart({"name": "Lydia the Housecarl"}, {"embedding": ("raw.f32", (emb * 2).astype("<f4").tobytes())})
    assert json.loads(req(port, "POST", "/v1/audio/voices", body2, h2)[2])["status"] == "replaced"
    d = tmp_path / "voices" / "Lydia_the_Housecarl"
    assert np.array_equal(np.fromfile(d / "embedding.f32", "<f4"), emb * 2)
    meta = json.loads((d / "voice.json").read_text())
    assert meta["dim"] == 8 and meta["model"] == "navi-test" and meta["name"] == "Lydia the Housecarl"
    # reloaded from disk
    again = serve.VoiceStore(tmp_path / "voices", 8)
    assert np.array_equal(again.find("Lydia_the_Housecarl").embedding, emb * 2)
    # a WAV without an embedding needs the speaker encoder
    wav = serve.wav_bytes(np.zeros(2400, np.int16), 24000)
    body3, h3 = multipart({"name": "x"}, {"audio_sample": ("x.wav", wav)})
    st, _, data = req(port, "POST", "/v1/audio/voices", body3, h3)
    assert st == 501 and "speaker encoder" in json.loads(data)["error"]["message"]
    body4, h4 = multipart({"name": "bad"}, {"embedding": ("e.f32", np.zeros(3, "<f4").tobytes())})
    assert req(port, "POST", "/v1/audio/voices", body4, h4)[0] == 400
    assert req(port, "DELETE", "/v1/audio/voices/Lydia_the_Housecarl")[0] == 200
    assert req(port, "DELETE", "/v1/audio/voices/Lydia_the_Housecarl")[0] == 404
    assert not d.exists()


def test_voice_ids():
    assert serve.voice_id_for("voice 1") == "voice_1"
    assert serve.voice_id_for("../../etc") == "_.._etc"
    assert serve.voice_id_for("...") == "unnamed"
    assert serve.voice_id_for("Grüße") == "Gr____e"   # one "_" per byte of a multi-byte character
    assert len(serve.voice_id_for("a" * 300)) == 128


def test_xtts_dialect(server):
    svc, eng, port = server
    st, h, body = req(port, "POST", "/tts_to_audio/", {"text": "Greetings.", "speaker_wav": "femaleeventoned", "language": "en-US"})
    assert st == 200 and h["Content-Type"] == "audio/wav"
    r = eng.requests[-1]
    assert r.voice.id == "femaleeventoned" and r.language == "english"
    assert r.seed == int(hashlib.sha256(b"femaleeventoned").hexdigest()[:8], 16)
    # unknown speaker: the fallback by its male/female prefix ("default" -> voice_1), seed still by its name
    req(port, "POST", "/tts_stream", {"text": "Hm.", "speaker_wav": "malenord"})
    r = eng.requests[-1]
    assert r.voice.id == "voice_1" and r.seed == serve.Service.stable_seed("malenord")
    # form fields
    body, hh = multipart({"text": "Form.", "speaker_wav": "voice_1"})
    assert req(port, "POST", "/tts_to_file", body, hh)[0] == 200 and eng.requests[-1].text == "Form."
    st, _, data = req(port, "POST", "/tts_to_audio", {"text": "  ", "speaker_wav": "voice_1"})
    assert st == 400 and json.loads(data) == {"error": "empty text"}
    # clone under a name from an embedding; a WAV alone needs the encoder
    emb = np.ones(8, "<f4").tobytes()
    body, hh = multipart({"speaker_name": "maleguard"}, {"embedding": ("e.f32", emb)})
    st, _, data = req(port, "POST", "/clone_speaker", body, hh)
    assert st == 200 and json.loads(data)["voice_id"] == "maleguard"
    st, _, data = req(port, "POST", "/upload_speaker?speaker_name=x", serve.wav_bytes(np.zeros(100, np.int16), 24000),
                      {"Content-Type": "audio/wav"})
    assert st == 501


def test_wav_helpers():
    pcm = np.array([0.0, 0.5, -0.5, 1.5, -2.0, 1 / 65534], np.float32)
    s = serve.to_s16(pcm)
    assert s.tolist() == [0, 16384, -16384, 32767, -32767, 0]   # 16383.5 rounds to even; half an lsb to 0
    w = serve.wav_bytes(s, 24000)
    assert len(w) == 44 + 12 and struct.unpack("<I", w[4:8])[0] == 36 + 12 and struct.unpack("<I", w[40:44])[0] == 12
