"""The command-line front (navi-tts_b200/cli/navi_b200_cli.cpp, mirroring the reference's
runtime/cli/main.cpp:59-72, 247-279 without the tokenizer): argument handling on the CPU, and
on a GPU `synth` against Graph.synth through the Python bindings (same ids, speaker, seed and
the model's generation defaults), sample for sample in the 16-bit WAV."""
import os
import struct
import subprocess

import numpy as np
import pytest

from navi_b200 import capi, engine

CLI = os.path.join(os.path.dirname(capi.LIB_PATH), "navi-b200")


def _run(*args):
    return subprocess.run([CLI, *args], capture_output=True, text=True, timeout=600)


def test_cli_usage_and_argument_errors():
    assert os.path.exists(CLI), "build() makes the CLI next to the library"
    r = _run("--help")
    assert r.returncode == 2 and "synth --model FILE" in r.stderr and "info" in r.stderr
    r = _run("synth", "--model", "x.navi")
    assert r.returncode == 2 and "synth needs --model" in r.stderr
    r = _run("synth", "--bogus")
    assert r.returncode == 2 and "unknown option --bogus" in r.stderr
    r = _run("frobnicate")
    assert r.returncode == 2


def _read_wav(path):
    b = open(path, "rb").read()
    assert b[:4] == b"RIFF" and b[8:16] == b"WAVEfmt "
    fmt, ch, rate, brate, align, bits = struct.unpack("<HHIIHH", b[20:36])
    assert (fmt, ch, align, bits) == (1, 1, 2, 16) and brate == 2 * rate
    assert b[36:40] == b"data"
    n = struct.unpack("<I", b[40:44])[0]
    assert struct.unpack("<I", b[4:8])[0] == 36 + n and len(b) == 44 + n
    return rate, np.frombuffer(b[44:], dtype="<i2")


@pytest.mark.gpu
def test_cli_synth_matches_graph(small_navi, tmp_path):
    from oracle import model as om
    W = om.Weights.from_navi(small_navi)
    cfg = W.cfg
    rng = np.random.default_rng(12)
    ids = [cfg.im_start_id, cfg.assistant_id, 198 % cfg.text_vocab] + rng.integers(0, cfg.text_vocab, 7).tolist() + \
        [cfg.im_end_id, 198 % cfg.text_vocab, cfg.im_start_id, cfg.assistant_id, 198 % cfg.text_vocab]
    spk = rng.standard_normal(W.tl.hidden).astype(np.float32)
    np.save(tmp_path / "spk.npy", spk)
    (tmp_path / "ids.txt").write_text(" ".join(map(str, ids)))
    out = tmp_path / "out.wav"
    r = _run("synth", "--model", small_navi, "--ids-file", str(tmp_path / "ids.txt"), "--speaker", str(tmp_path / "spk.npy"),
             "--out", str(out), "--seed", "9", "--max-frames", "20", "--batch", "8")
    assert r.returncode == 0, r.stderr
    assert "frames" in r.stderr and "RTF" in r.stderr
    rate, s16 = _read_wav(out)
    dev = engine.Device(0)
    w = engine.Weights(dev, small_navi)
    p = w.params
    assert rate == p.sample_rate
    g = engine.Graph(dev, w, max_prompt_tokens=len(ids) + 16, max_frames=20, vocoder_chunk=8)
    s = engine.Sampling(temperature=p.temperature, top_k=p.top_k, top_p=p.top_p, repetition_penalty=p.repetition_penalty,
                        cp_temperature=p.cp_temperature, cp_top_k=p.cp_top_k, cp_top_p=p.cp_top_p, min_frames=2,
                        rng=capi.NAVI_RNG_PCG)
    codes, pcm, st, _ = g.synth(ids, "english", spk, s, 9, 20, first_batch=4, vocoder_batch=8)
    want = np.rint(np.clip(pcm, -1.0, 1.0).astype(np.float32) * np.float32(32767.0)).astype(np.int16)   # lrintf of the f32 product
    assert s16.shape == want.shape and s16.shape[0] == st.n_frames * p.codec_upsample
    assert np.array_equal(s16, want)
    # the raw float32 speaker form gives the same audio
    spk.tofile(tmp_path / "spk.f32")
    out2 = tmp_path / "out2.wav"
    r = _run("synth", "--model", small_navi, "--ids", ",".join(map(str, ids)), "--speaker", str(tmp_path / "spk.f32"),
             "--out", str(out2), "--seed", "9", "--max-frames", "20", "--batch", "8")
    assert r.returncode == 0, r.stderr
    assert np.array_equal(_read_wav(out2)[1], s16)
    g.close()


def test_cli_bench_argument_errors(small_navi):
    r = _run("bench")
    assert r.returncode == 2 and "bench needs --model" in r.stderr
    r = _run("bench", "--model", small_navi)      # the small model's text vocabulary has no default prompt
    assert r.returncode == 2 and "needs --ids" in r.stderr
    r = _run("bench", "--repeats")
    assert r.returncode == 2 and "--repeats needs a value" in r.stderr


@pytest.mark.gpu
def test_cli_bench_line(small_navi, tmp_path):
    """`bench` (runtime/bench/bench.cpp:98-155): one JSON line per repeat with the reference's
    BenchResult fields; the WAV digest is the SHA-256 of the WAV it makes (also written with
    --out X.wav), and that WAV is `synth`'s for the same ids, speaker, seed and batching."""
    import hashlib
    import json
    from oracle import model as om
    W = om.Weights.from_navi(small_navi)
    cfg = W.cfg
    rng = np.random.default_rng(3)
    ids = [cfg.im_start_id, cfg.assistant_id, 198 % cfg.text_vocab] + rng.integers(0, cfg.text_vocab, 6).tolist() + \
        [cfg.im_end_id, 198 % cfg.text_vocab, cfg.im_start_id, cfg.assistant_id, 198 % cfg.text_vocab]
    idarg = ",".join(map(str, ids))
    out = tmp_path / "b.wav"
    r = _run("bench", "--model", small_navi, "--ids", idarg, "--seed", "5", "--max-frames", "12", "--repeats", "2",
             "--warmup", "1", "--out", str(out))
    assert r.returncode == 0, r.stderr
    lines = [json.loads(x) for x in r.stdout.strip().splitlines()]
    assert len(lines) == 2
    keys = {"ts", "git", "gfx", "device", "multiprocessors", "model", "weight_bytes", "load_map_ms", "load_upload_ms", "upload_gbps",
            "prefill_ms", "frame_ms", "talker_ms", "cp_ms", "vocoder_ms_per_frame", "ttfa_ms", "rtf", "n_frames", "wav_sha256", "text",
            "seed"}
    for j in lines:
        assert keys <= set(j), keys - set(j)
        assert j["n_frames"] <= 12 and j["frame_ms"] > 0 and j["weight_bytes"] > 0 and j["talker_ms"] is None and j["seed"] == 5
    assert lines[0]["wav_sha256"] == lines[1]["wav_sha256"] == hashlib.sha256(out.read_bytes()).hexdigest()
    np.zeros(W.tl.hidden, np.float32).tofile(tmp_path / "zero.f32")
    syn = tmp_path / "s.wav"
    r = _run("synth", "--model", small_navi, "--ids", idarg, "--speaker", str(tmp_path / "zero.f32"), "--out", str(syn), "--seed", "5",
             "--max-frames", "12", "--first-batch", "4", "--batch", "16")
    assert r.returncode == 0, r.stderr
    assert syn.read_bytes() == out.read_bytes()
    jl = tmp_path / "results.jsonl"
    r = _run("bench", "--model", small_navi, "--ids", idarg, "--seed", "5", "--max-frames", "4", "--out", str(jl))
    assert r.returncode == 0 and "appended to" in r.stderr
    assert len(jl.read_text().splitlines()) == 1
