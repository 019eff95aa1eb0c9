"""The checkpoint converter (navi_b200.convert, the reference's tools/convert.py:150-315) on a
synthetic HF Qwen3-TTS directory, on the CPU.

The directory is built from the small synthetic model: config.json / generation_config.json /
speech_tokenizer/config.json carrying its hyperparameters in the HF layout, model.safetensors
with the talker and speaker-encoder tensors (some stored as bf16), the codec's tensors without
their `codec.` prefix in speech_tokenizer/model.safetensors with each codebook split into the
EMA pair (embedding_sum, cluster_usage), `initialized` flags and an encoder tensor that must be
dropped. The converted file must pass the C++ reader and the reference's tensor-table check
(navi_model_probe), read back the same hyperparameters, hold every tensor at the target dtype
(1-D in f32), and hold the codebooks baked back to embedding_sum / cluster_usage.
"""
import ctypes
import json

import numpy as np
import pytest
import torch
from safetensors.torch import save_file

from navi_b200 import capi, convert, model_spec
from navi_b200.navi_file import F16, F32, U8, NaviFile


def _transformer(t, vocab=True):
    d = dict(hidden_size=t.hidden, num_hidden_layers=t.n_layer, num_attention_heads=t.n_head, num_key_value_heads=t.n_kv_head,
             head_dim=t.head_dim, intermediate_size=t.ff, rms_norm_eps=t.eps, rope_theta=t.rope_theta,
             max_position_embeddings=t.max_pos, hidden_act="silu", attention_bias=False)
    if vocab and t.vocab:
        d["vocab_size"] = t.vocab
    return d


def make_hf_dir(root, c, synth_navi):
    """An HF-layout checkpoint of config c whose tensors are synth_navi's."""
    (root / "speech_tokenizer").mkdir(parents=True)
    talker = _transformer(c.talker)
    talker.update(text_hidden_size=c.text_hidden, text_vocab_size=c.text_vocab, num_code_groups=c.n_code_groups,
                  position_id_per_seconds=13, codec_bos_id=c.codec_bos_id, codec_eos_token_id=c.codec_eos_id,
                  codec_pad_id=c.codec_pad_id, codec_think_id=c.codec_think_id, codec_nothink_id=c.codec_nothink_id,
                  codec_think_bos_id=c.codec_think_bos_id, codec_think_eos_id=c.codec_think_eos_id,
                  rope_scaling={"mrope_section": [24, 20, 20], "interleaved": True},
                  codec_language_id=dict(c.languages), spk_id={"voice_a": 3000},
                  code_predictor_config={**_transformer(c.cp), "num_code_groups": c.n_code_groups})
    cfg = dict(model_type="qwen3_tts", tts_model_type="base", tts_model_size="0b6", tokenizer_type="qwen",
               im_start_token_id=c.im_start_id, im_end_token_id=c.im_end_id, assistant_token_id=c.assistant_id,
               tts_bos_token_id=c.tts_bos_id, tts_eos_token_id=c.tts_eos_id, tts_pad_token_id=c.tts_pad_id,
               talker_config=talker, speaker_encoder_config={"enc_dim": c.spk_dim, "sample_rate": c.sample_rate})
    dec = _transformer(c.vocoder, vocab=False)
    dec.update(latent_dim=c.vq_latent, codebook_dim=c.vq_codebook_dim, codebook_size=c.vq_codebook_size,
               decoder_dim=c.decoder_dim, num_quantizers=c.vq_n_q, num_semantic_quantizers=c.vq_n_semantic,
               sliding_window=c.sliding_window, upsample_rates=list(c.upsample_rates),
               upsampling_ratios=list(c.upsampling_ratios))
    codec = dict(input_sample_rate=c.sample_rate, output_sample_rate=c.sample_rate, decode_upsample_rate=c.samples_per_frame,
                 encode_downsample_rate=c.samples_per_frame, encoder_valid_num_quantizers=c.vq_n_q, decoder_config=dec,
                 encoder_config={"hidden_size": 8})
    gen = {f"subtalker_{k}" if sub else k: v for sub in (False, True)
           for k, v in dict(temperature=0.9, top_k=50, top_p=1.0).items()}
    gen.update(repetition_penalty=1.05, do_sample=True)
    (root / "config.json").write_text(json.dumps(cfg))
    (root / "speech_tokenizer" / "config.json").write_text(json.dumps(codec))
    (root / "generation_config.json").write_text(json.dumps(gen))
    for f, text in (("vocab.json", '{"a": 0}'), ("merges.txt", "#version: 0.2\n"), ("tokenizer_config.json", "{}")):
        (root / f).write_text(text)
    src = NaviFile.open(synth_navi)
    main, cod = {}, {}
    rng = np.random.default_rng(0)
    for t in src.tensors:
        if t.dtype == U8:
            continue
        a = torch.from_numpy(np.array(src.array(t), dtype=np.float32))
        if t.name.startswith("codec."):
            name = t.name[len("codec."):]
            if name.endswith("._codebook.codebook"):
                stem = name[:-len(".codebook")]
                usage = torch.from_numpy(2.0 ** rng.integers(0, 4, a.shape[0]).astype(np.float32))
                cod[stem + ".embedding_sum"] = a * usage[:, None]
                cod[stem + ".cluster_usage"] = usage
                cod[stem + ".initialized"] = torch.ones(1)
            else:
                cod[name] = a
        else:
            main[t.name] = a.to(torch.bfloat16) if t.name.startswith("talker.code_predictor.lm_head.") else a
    cod["encoder.downsample.conv.weight"] = torch.zeros(4, 4, 2)
    save_file(main, str(root / "model.safetensors"))
    save_file(cod, str(root / "speech_tokenizer" / "model.safetensors"))
    return src


def _probe(path):
    L = capi.lib()
    n = [ctypes.c_int(-1) for _ in range(4)]
    p = capi.Params()
    st = L.navi_model_probe(str(path).encode(), ctypes.byref(p), *[ctypes.byref(x) for x in n])
    return st, p, [x.value for x in n], L.navi_last_error().decode()


def test_convert_synthetic_checkpoint(small_navi, tmp_path):
    c = model_spec.small_config()
    hf = tmp_path / "Qwen3-TTS-synthetic"
    src = make_hf_dir(hf, c, small_navi)
    out = tmp_path / "converted.navi"
    rep = convert.convert(hf, out)
    assert rep.tensors > 0 and not rep.f16_overflow
    st, p, (nt, miss, bad, unused), err = _probe(out)
    assert st == capi.NAVI_OK and (miss, bad) == (0, 0), err
    f = NaviFile.open(out)
    for key in ("talker.hidden_size", "talker.num_hidden_layers", "talker.codec_eos_token_id", "cp.vocab_size", "text.tts_pad_id",
                "codec.decoder.decoder_dim", "codec.decoder.upsample_rates", "codec.decode_upsample_rate", "gen.top_k",
                "gen.subtalker_temperature", "talker.language.english", "speaker.enc_dim"):
        assert f.kv[key] == src.kv[key], key
    assert f.kv["talker.speaker.voice_a"] == 3000 and f.kv["general.has_codec_encoder"] == 0
    assert f.kv["talker.mrope_section"] == [24, 20, 20] and f.kv["speaker.mel.n_fft"] == 1024
    names = {t.name for t in f.tensors}
    assert not any(n.startswith("codec.encoder.") or n.endswith("initialized") or "embedding_sum" in n for n in names)
    assert {"tokenizer.vocab.json", "tokenizer.merges.txt", "tokenizer.config.json"} <= names
    for t in src.tensors:
        if t.dtype == U8:
            continue
        got = f.find(t.name)
        assert got is not None, t.name
        assert got.dtype == (F16 if len(t.dims) >= 2 else F32) and got.dims == t.dims, t.name
        want = np.array(src.array(t), dtype=np.float32)
        if t.name.startswith("talker.code_predictor.lm_head."):     # stored as bf16 in the checkpoint
            want = torch.from_numpy(want).to(torch.bfloat16).float().numpy()
        want = want.astype(np.float16 if len(t.dims) >= 2 else np.float32)
        assert np.array_equal(f.array(got), want), t.name


def test_convert_keeps_f32_and_the_encoder_on_request(small_navi, tmp_path):
    c = model_spec.small_config()
    hf = tmp_path / "ckpt"
    make_hf_dir(hf, c, small_navi)
    out = tmp_path / "f32.navi"
    convert.convert(hf, out, dtype="f32", with_encoder=True)
    f = NaviFile.open(out)
    assert f.find("talker.codec_head.weight").dtype == F32
    assert f.find("codec.encoder.downsample.conv.weight") is not None
    assert f.kv["general.has_codec_encoder"] == 1 and f.kv["codec.encoder.hidden_size"] == 8


def test_convert_command_line(small_navi, tmp_path, capsys):
    hf = tmp_path / "ckpt"
    make_hf_dir(hf, model_spec.small_config(), small_navi)
    assert convert.main([str(hf), str(tmp_path / "cli.navi"), "--codec-dtype", "f32"]) == 0
    f = NaviFile.open(tmp_path / "cli.navi")
    assert f.find("codec.decoder.pre_conv.conv.weight").dtype == F32 and f.find("talker.codec_head.weight").dtype == F16
    assert "wrote" in capsys.readouterr().err
    with pytest.raises(FileNotFoundError):
        convert.convert(tmp_path / "missing", tmp_path / "x.navi")
