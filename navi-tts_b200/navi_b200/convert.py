"""HF Qwen3-TTS checkpoint directory -> `.navi` v1 (the reference's tools/convert.py:150-315).

    python -m navi_b200.convert MODEL_DIR OUT.navi [--dtype f16|f32] [--codec-dtype f16|f32] [--with-encoder]

MODEL_DIR is the released layout: config.json, generation_config.json, model.safetensors,
vocab.json, merges.txt, tokenizer_config.json, and speech_tokenizer/{config.json,
model.safetensors}. The output is what the reference's converter writes, so either engine
loads it:

* hyperparameters under general.* / text.* / talker.* / cp.* / speaker.* / codec.* / gen.*,
  with the key names the reference's reader expects (model/qwen3tts/params.cpp:59-130);
* every tensor of model.safetensors under its own name, and every tensor of the codec's
  under `codec.` + its name, except the codec encoder (unless --with-encoder) and the
  `initialized` bookkeeping flags;
* each EMA codebook pair (embedding_sum, cluster_usage) baked into one
  `...codebook` = embedding_sum / max(cluster_usage, 1e-5), as the codec decodes it;
* tensors of two or more dims in the target dtype, one-dimensional ones (norms, biases,
  snake alpha / beta, layer scales) in f32;
* the tokenizer files as U8 tensors tokenizer.vocab.json / .merges.txt / .config.json.

bf16 checkpoints are read without torch: a bf16 value is the high half of an f32.
"""
from __future__ import annotations

import argparse
import json
import struct
import sys
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

from .navi_file import F16, F32, U8, NaviBuilder

# safetensors dtype name -> (numpy dtype of the stored bytes, widening to f32 or None)
_ST_DTYPES = {
    "F32": (np.float32, None),
    "F16": (np.float16, None),
    "BF16": (np.uint16, lambda u: (u.astype(np.uint32) << 16).view(np.float32)),
    "F64": (np.float64, None),
    "I64": (np.int64, None),
    "I32": (np.int32, None),
    "BOOL": (np.bool_, None),
    "U8": (np.uint8, None),
}

_TARGETS = {"f16": F16, "f32": F32}


class SafetensorsFile:
    """The tensors of one .safetensors file: an 8-byte little-endian header length, a JSON
    table of {name: {dtype, shape, data_offsets}}, then the data; read through a memory map."""

    def __init__(self, path: Path):
        self.path = Path(path)
        raw = np.memmap(self.path, dtype=np.uint8, mode="r")
        (hlen,) = struct.unpack("<Q", bytes(raw[:8]))
        table = json.loads(bytes(raw[8:8 + hlen]).decode("utf-8"))
        table.pop("__metadata__", None)
        self._table = table
        self._data = raw[8 + hlen:]

    def names(self) -> list[str]:
        return list(self._table)

    def array(self, name: str) -> np.ndarray:
        e = self._table[name]
        if e["dtype"] not in _ST_DTYPES:
            raise ValueError(f"{self.path}: tensor {name!r} has dtype {e['dtype']}, which this converter does not read")
        store, widen = _ST_DTYPES[e["dtype"]]
        lo, hi = e["data_offsets"]
        a = self._data[lo:hi].view(store).reshape(e["shape"])
        return widen(a) if widen else a


# hyperparameters copied from a config section when present: talker / code predictor / codec decoder
_TRANSFORMER = ("hidden_size", "num_hidden_layers", "num_attention_heads", "num_key_value_heads", "head_dim",
                "intermediate_size", "rms_norm_eps", "rope_theta", "vocab_size", "max_position_embeddings", "hidden_act",
                "attention_bias")
_TALKER_EXTRA = ("text_hidden_size", "text_vocab_size", "num_code_groups", "position_id_per_seconds", "codec_bos_id",
                 "codec_eos_token_id", "codec_pad_id", "codec_think_id", "codec_nothink_id", "codec_think_bos_id",
                 "codec_think_eos_id")
_DECODER_EXTRA = ("latent_dim", "codebook_dim", "codebook_size", "decoder_dim", "num_quantizers", "num_semantic_quantizers",
                  "semantic_codebook_size", "sliding_window", "vector_quantization_hidden_dimension",
                  "layer_scale_initial_scale", "upsample_rates", "upsampling_ratios")
_ENCODER_KEYS = ("hidden_size", "num_hidden_layers", "num_attention_heads", "num_key_value_heads", "head_dim",
                 "intermediate_size", "norm_eps", "rope_theta", "max_position_embeddings", "hidden_act", "codebook_dim",
                 "codebook_size", "num_quantizers", "num_semantic_quantizers", "num_filters", "kernel_size", "last_kernel_size",
                 "residual_kernel_size", "compress", "dilation_growth_rate", "num_residual_layers", "sliding_window",
                 "upsampling_ratios", "upsample_groups", "vector_quantization_hidden_dimension", "layer_scale_initial_scale",
                 "use_causal_conv", "pad_mode", "trim_right_ratio", "sampling_rate")
_GEN_KEYS = ("temperature", "top_k", "top_p", "repetition_penalty", "do_sample", "subtalker_temperature", "subtalker_top_k",
             "subtalker_top_p", "subtalker_dosample")
# the speaker encoder's defaults (its config class) and the mel front end of its embedding extraction, which
# config.json does not carry
_SPEAKER_DEFAULTS = dict(mel_dim=128, enc_channels=[512, 512, 512, 512, 1536], enc_kernel_sizes=[5, 3, 3, 3, 1],
                         enc_dilations=[1, 2, 3, 4, 1], enc_attention_channels=128, enc_res2net_scale=8, enc_se_channels=128,
                         enc_dim=192, sample_rate=24000)
_SPEAKER_MEL = dict(n_fft=1024, num_mels=128, hop_size=256, win_size=1024, fmin=0, fmax=12000)


def hyperparameters(model_dir: Path, dtype: str, codec_dtype: str, with_encoder: bool) -> list[tuple[str, object]]:
    """The (key, value) pairs of a converted file, in the order they are written."""
    d = Path(model_dir)
    cfg = json.loads((d / "config.json").read_text())
    codec = json.loads((d / "speech_tokenizer" / "config.json").read_text())
    gen = json.loads((d / "generation_config.json").read_text())
    talker = cfg["talker_config"]
    cp = talker["code_predictor_config"]
    out: list[tuple[str, object]] = []

    def section(prefix: str, src: dict, keys) -> None:
        out.extend((f"{prefix}.{k}", src[k]) for k in keys if src.get(k) is not None)

    out += [("general.arch", "qwen3-tts"), ("general.name", d.name), ("general.model_type", cfg["model_type"]),
            ("general.tts_model_type", cfg["tts_model_type"]), ("general.tts_model_size", cfg["tts_model_size"]),
            ("general.tokenizer_type", cfg["tokenizer_type"]), ("general.dtype", dtype), ("general.codec_dtype", codec_dtype),
            ("general.converter", "navi-b200 convert (.navi format v1)"), ("general.has_codec_encoder", with_encoder)]
    for role in ("im_start", "im_end", "assistant", "tts_bos", "tts_eos", "tts_pad"):
        out.append((f"text.{role}_id", cfg[f"{role}_token_id"]))
    section("talker", talker, _TRANSFORMER + _TALKER_EXTRA)
    rope = talker.get("rope_scaling") or {}
    out += [("talker.mrope_section", rope.get("mrope_section")), ("talker.mrope_interleaved", bool(rope.get("interleaved", False)))]
    out += [(f"talker.language.{k}", v) for k, v in talker["codec_language_id"].items()]
    out += [(f"talker.speaker.{k}", v) for k, v in talker.get("spk_id", {}).items()]
    section("cp", cp, _TRANSFORMER + ("num_code_groups",))
    spk = {**_SPEAKER_DEFAULTS, **cfg["speaker_encoder_config"]}
    out += [(f"speaker.{k}", v) for k, v in spk.items()]
    out += [(f"speaker.mel.{k}", v) for k, v in _SPEAKER_MEL.items()]
    for k in ("input_sample_rate", "output_sample_rate", "decode_upsample_rate", "encode_downsample_rate",
              "encoder_valid_num_quantizers"):
        out.append((f"codec.{k}", codec[k]))
    section("codec.decoder", codec["decoder_config"], _TRANSFORMER + _DECODER_EXTRA)
    if with_encoder:
        section("codec.encoder", codec["encoder_config"], _ENCODER_KEYS)
    section("gen", gen, _GEN_KEYS)
    return out


@dataclass
class Report:
    tensors: int = 0
    weight_bytes: int = 0
    f16_overflow: dict = field(default_factory=dict)   # name -> values beyond the f16 range


def _put(b: NaviBuilder, rep: Report, name: str, a: np.ndarray, target: int) -> None:
    code = target if a.ndim >= 2 else F32
    a = np.asarray(a, dtype=np.float32)
    if code == F16:
        big = int(np.count_nonzero(np.abs(a[np.isfinite(a)]) > 65504.0))
        if big:
            rep.f16_overflow[name] = big
    b.put_tensor(name, code, a)
    rep.tensors += 1
    rep.weight_bytes += a.size * (2 if code == F16 else 4)


_CODEBOOK_PARTS = ("embedding_sum", "embed_sum", "cluster_usage")


def convert(model_dir, out, dtype: str = "f16", codec_dtype: str | None = None, with_encoder: bool = False) -> Report:
    d = Path(model_dir)
    codec_dtype = codec_dtype or dtype
    b = NaviBuilder()
    for k, v in hyperparameters(d, dtype, codec_dtype, with_encoder):
        b.set_kv(k, v)
    for fname, tname in (("vocab.json", "vocab.json"), ("merges.txt", "merges.txt"), ("tokenizer_config.json", "config.json")):
        b.put_tensor(f"tokenizer.{tname}", U8, np.frombuffer((d / fname).read_bytes(), dtype=np.uint8))
    rep = Report()
    main = SafetensorsFile(d / "model.safetensors")
    b.set_kv("general.source.main", "model.safetensors")
    for name in main.names():
        _put(b, rep, name, main.array(name), _TARGETS[dtype])
    codec = SafetensorsFile(d / "speech_tokenizer" / "model.safetensors")
    b.set_kv("general.source.codec", "speech_tokenizer/model.safetensors")
    books: dict[str, dict[str, np.ndarray]] = {}
    for name in codec.names():
        stem, leaf = name.rsplit(".", 1) if "." in name else ("", name)
        if (name.startswith("encoder.") and not with_encoder) or leaf == "initialized":
            continue
        if leaf in _CODEBOOK_PARTS:
            books.setdefault(stem, {})[leaf] = np.asarray(codec.array(name), dtype=np.float32)
            continue
        _put(b, rep, "codec." + name, codec.array(name), _TARGETS[codec_dtype])
    for stem, parts in books.items():
        total = parts.get("embedding_sum", parts.get("embed_sum"))
        usage = parts["cluster_usage"]
        _put(b, rep, f"codec.{stem}.codebook", total / np.maximum(usage, np.float32(1e-5))[:, None], _TARGETS[codec_dtype])
    b.save(out)
    return rep


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="HF Qwen3-TTS checkpoint -> .navi")
    ap.add_argument("model_dir", type=Path)
    ap.add_argument("out", type=Path)
    ap.add_argument("--dtype", choices=sorted(_TARGETS), default="f16")
    ap.add_argument("--codec-dtype", choices=sorted(_TARGETS), default=None)
    ap.add_argument("--with-encoder", action="store_true")
    a = ap.parse_args(argv)
    rep = convert(a.model_dir, a.out, a.dtype, a.codec_dtype, a.with_encoder)
    print(f"wrote {a.out}: {rep.tensors} tensors, {rep.weight_bytes / 1e9:.3f} GB of weights", file=sys.stderr)
    if rep.f16_overflow:
        print(f"warning: values beyond the f16 range in {len(rep.f16_overflow)} tensors: {list(rep.f16_overflow)[:8]}", file=sys.stderr)
    return 0


if __name__ == "__main__":
    sys.exit(main())
