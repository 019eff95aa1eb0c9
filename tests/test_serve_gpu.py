"""The HTTP front end (navi_b200.serve) over the real engine on the small synthetic model: the
audio of `POST /v1/audio/speech` (whole body, and streamed as a chunked WAV and as server-sent
events) is the PCM of Graph::synth for the tokenizer's prompt ids, the voice's embedding, the
request's seed and the model's sampling defaults, sample for sample; the XTTS route answers
with its speaker's fixed seed; metrics count the requests."""
import base64
import json

import numpy as np
import pytest

from navi_b200 import engine, serve
from test_serve import req

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def live(small_navi, tmp_path_factory):
    eng = serve.GraphEngine(str(small_navi), max_frames=64)
    store = serve.VoiceStore(tmp_path_factory.mktemp("voices"), eng.speaker_dim)
    rng = np.random.default_rng(4)
    store.put("voice_1", rng.standard_normal(eng.speaker_dim).astype(np.float32) * 0.1)
    svc = serve.Service(eng, store, "navi-small", max_audio_tokens=12)
    serve.warm_up(svc)
    (srv,) = serve.serve(svc, "127.0.0.1", 0)
    yield svc, eng, srv.server_address[1]
    srv.shutdown()
    svc.worker.shutdown()


def _direct(svc, eng, text, seed, max_frames):
    """Graph::synth with what the server derives from the request, on the server's worker."""
    v = svc.store.find("voice_1")
    s = engine.Sampling(temperature=eng.p.temperature, top_k=eng.p.top_k, repetition_penalty=eng.p.repetition_penalty,
                        cp_temperature=eng.p.cp_temperature, cp_top_k=eng.p.cp_top_k)
    ids = eng.tokenizer.prompt_ids(text)
    lang = next(iter(eng.languages))
    _, pcm, st, _ = svc.worker.submit(eng.graph.synth, ids, lang, v.embedding, s, seed, max_frames).result()
    return serve.to_s16(pcm), st, lang


def test_speech_matches_graph_synth(live):
    svc, eng, port = live
    text = "Hello there, general."
    pcm, st, lang = _direct(svc, eng, text, 77, 12)
    assert st.n_frames > 0 and len(pcm) == st.n_frames * eng.samples_per_frame
    code, h, body = req(port, "POST", "/v1/audio/speech", {"input": text, "voice": "voice_1", "seed": 77, "language": lang})
    assert code == 200 and h["Content-Type"] == "audio/wav"
    assert np.array_equal(np.frombuffer(body[44:], "<i2"), pcm)
    code, h, streamed = req(port, "POST", "/v1/audio/speech", {"input": text, "voice": "voice_1", "seed": 77, "language": lang,
                                                              "stream_format": "audio", "stream_batch_size": 3})
    assert code == 200 and streamed[44:] == body[44:]
    code, h, sse = req(port, "POST", "/v1/audio/speech", {"input": text, "voice": "voice_1", "seed": 77, "language": lang,
                                                         "stream_format": "sse"})
    events = [json.loads(e[len("data: "):]) for e in sse.decode().split("\n\n") if e]
    got = np.concatenate([np.frombuffer(base64.b64decode(e["audio"]), "<i2") for e in events if e["type"] == "speech.audio.delta"])
    assert np.array_equal(got, pcm) and events[-1]["type"] == "speech.audio.done" and events[-1]["navi"]["frames"] == st.n_frames


def test_xtts_seed_and_metrics(live):
    svc, eng, port = live
    text = "Greetings, traveller."
    code, _, body = req(port, "POST", "/tts_to_audio/", {"text": text, "speaker_wav": "voice_1",
                                                        "language": next(iter(eng.languages))})
    assert code == 200
    pcm, _, _ = _direct(svc, eng, text, serve.Service.stable_seed("voice_1"), 12)
    assert np.array_equal(np.frombuffer(body[44:], "<i2"), pcm)
    m = req(port, "GET", "/metrics")[2].decode()
    assert 'navi_tts_requests_total{model="navi-small"}' in m and "navi_tts_ttfa_seconds_count" in m
