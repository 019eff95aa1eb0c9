"""Qwen3-TTS-12Hz hyperparameters, the tensor table, and seeded synthetic weights.

`kv_entries` writes the keys the reference engine reads
(model/qwen3tts/params.cpp:59-130); `tensor_table` lists every tensor with the
shapes of model/qwen3tts/params.cpp:132-284 (expected_tensors), in an order
that keeps q/k/v and gate/up adjacent so the device arena can treat each group
as one matrix (the reference's Talker::fused_groups, talker.hip:190-198).

Synthetic weights: every tensor of two or more dims is N(0, 0.02) rounded to
f16 (tools/convert.py:257-268 stores >=2-D as f16, 1-D as f32).  One-dimensional
norm weights are 1 + N(0, 0.02) so activations keep unit scale; every other 1-D
tensor (biases, snake alpha/beta, layer scales, gamma) is N(0, 0.02).  Each
tensor draws from its own numpy PCG64 stream keyed by (component seed, crc32 of
its name); the component seeds follow the benchmark configs: talker 1, code
predictor 2, codec 3, everything else 4.
"""
from __future__ import annotations

import json

import zlib
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass, field, replace
from pathlib import Path

import numpy as np

from .navi_file import F16, F32, U8, NaviBuilder


@dataclass(frozen=True)
class Transformer:
    hidden: int
    n_layer: int
    n_head: int
    n_kv_head: int
    head_dim: int
    ff: int
    eps: float
    rope_theta: float
    vocab: int
    max_pos: int


@dataclass(frozen=True)
class ModelConfig:
    name: str
    talker: Transformer
    cp: Transformer
    vocoder: Transformer
    text_vocab: int
    text_hidden: int
    n_code_groups: int = 16
    # text-side special ids
    im_start_id: int = 151644
    im_end_id: int = 151645
    assistant_id: int = 77091
    tts_pad_id: int = 151671
    tts_bos_id: int = 151672
    tts_eos_id: int = 151673
    # codec-side control ids (offsets from the first id past the 2048 acoustic codes)
    codec_pad_id: int = 2048
    codec_bos_id: int = 2049
    codec_eos_id: int = 2050
    codec_think_id: int = 2054
    codec_nothink_id: int = 2055
    codec_think_bos_id: int = 2056
    codec_think_eos_id: int = 2057
    languages: tuple = (("chinese", 2055), ("english", 2050), ("german", 2053), ("spanish", 2054),
                        ("japanese", 2058), ("korean", 2064), ("french", 2061))
    # speaker encoder (out of scope for compute; its tensors are written so the table validates)
    spk_dim: int = 1024
    # codec decoder
    vq_latent: int = 1024
    vq_codebook_dim: int = 512
    vq_codebook_size: int = 2048
    vq_n_q: int = 16
    vq_n_semantic: int = 1
    decoder_dim: int = 1536
    sliding_window: int = 72
    upsample_rates: tuple = (8, 5, 4, 3)
    upsampling_ratios: tuple = (2, 2)
    sample_rate: int = 24000
    # generation defaults (generation_config.json)
    gen: dict = field(default_factory=lambda: dict(temperature=0.9, top_k=50, top_p=1.0, repetition_penalty=1.05,
                                                   subtalker_temperature=0.9, subtalker_top_k=50, subtalker_top_p=1.0))

    @property
    def samples_per_frame(self) -> int:
        n = 1
        for r in self.upsample_rates + self.upsampling_ratios:
            n *= r
        return n


def full_config(decoder_dim: int = 1024) -> ModelConfig:
    """The shapes every benchmark config uses (hidden 1024, 16/8 heads x 128, ff 3072,
    talker 28 layers / vocab 3072, code predictor 5 layers / vocab 2048).
    decoder_dim 1024 is configs[3]; the released model has 1536."""
    tl = Transformer(1024, 28, 16, 8, 128, 3072, 1e-6, 1e6, 3072, 32768)
    cp = Transformer(1024, 5, 16, 8, 128, 3072, 1e-6, 1e6, 2048, 65536)
    voc = Transformer(512, 8, 16, 16, 64, 1024, 1e-5, 1e4, 0, 8000)
    return ModelConfig(name=f"synthetic-qwen3-tts-12hz-0.6b-d{decoder_dim}", talker=tl, cp=cp, vocoder=voc,
                       text_vocab=151936, text_hidden=2048, decoder_dim=decoder_dim)


def layer_config() -> ModelConfig:
    """configs[0]'s model: the benchmark shapes with a single talker layer (the layer under
    test). Written with seed_offset=-1 (LAYER_SEED_OFFSET) its talker weights draw from seed 0.
    The text embedding, unused by a decode layer, is cut to 4096 rows to keep the file small."""
    c = full_config(1024)
    return replace(c, name="synthetic-qwen3-tts-one-layer", talker=replace(c.talker, n_layer=1), text_vocab=4096)


LAYER_SEED_OFFSET = -1   # component seed 1 (talker) - 1 = configs[0]'s seed 0


def small_config() -> ModelConfig:
    """A reduced model for tests that the CPU oracle finishes in seconds.
    Keeps head_dim 128, 16 codebooks and the 1920x upsampling chain; shrinks widths and depth."""
    tl = Transformer(256, 2, 4, 2, 128, 512, 1e-6, 1e6, 1536, 4096)
    cp = Transformer(256, 2, 4, 2, 128, 512, 1e-6, 1e6, 512, 4096)
    voc = Transformer(64, 2, 4, 4, 16, 128, 1e-5, 1e4, 0, 8000)
    base = 1536 - 1024   # first control id past the acoustic codes (suppression starts there)
    return ModelConfig(name="synthetic-qwen3-tts-small", talker=tl, cp=cp, vocoder=voc,
                       text_vocab=1000, text_hidden=256, im_start_id=990, im_end_id=991, assistant_id=700,
                       tts_pad_id=995, tts_bos_id=996, tts_eos_id=997,
                       codec_pad_id=base, codec_bos_id=base + 1, codec_eos_id=base + 2, codec_think_id=base + 6,
                       codec_nothink_id=base + 7, codec_think_bos_id=base + 8, codec_think_eos_id=base + 9,
                       languages=(("english", base + 2), ("german", base + 5)),
                       spk_dim=256, vq_latent=128, vq_codebook_dim=64, vq_codebook_size=512, decoder_dim=128,
                       sliding_window=8)


# --- KV section -----------------------------------------------------------------------

def _transformer_kv(w: NaviBuilder, ns: str, t: Transformer) -> None:
    w.set_kv(f"{ns}.hidden_size", t.hidden)
    w.set_kv(f"{ns}.num_hidden_layers", t.n_layer)
    w.set_kv(f"{ns}.num_attention_heads", t.n_head)
    w.set_kv(f"{ns}.num_key_value_heads", t.n_kv_head)
    w.set_kv(f"{ns}.head_dim", t.head_dim)
    w.set_kv(f"{ns}.intermediate_size", t.ff)
    w.set_kv(f"{ns}.rms_norm_eps", float(t.eps))
    w.set_kv(f"{ns}.rope_theta", float(t.rope_theta))
    if t.vocab:
        w.set_kv(f"{ns}.vocab_size", t.vocab)
    w.set_kv(f"{ns}.max_position_embeddings", t.max_pos)


def kv_entries(w: NaviBuilder, c: ModelConfig) -> None:
    w.set_kv("general.arch", "qwen3-tts")
    w.set_kv("general.name", c.name)
    w.set_kv("general.dtype", "f16")
    w.set_kv("general.codec_dtype", "f16")
    w.set_kv("general.converter", "navi-b200 synthetic (random-init, seeded)")
    w.set_kv("general.has_codec_encoder", 0)
    for k in ("im_start_id", "im_end_id", "assistant_id", "tts_bos_id", "tts_eos_id", "tts_pad_id"):
        w.set_kv("text." + k, getattr(c, k))
    _transformer_kv(w, "talker", c.talker)
    w.set_kv("talker.text_hidden_size", c.text_hidden)
    w.set_kv("talker.text_vocab_size", c.text_vocab)
    w.set_kv("talker.num_code_groups", c.n_code_groups)
    w.set_kv("talker.position_id_per_seconds", 13)
    for k, key in (("codec_bos_id", "codec_bos_id"), ("codec_eos_id", "codec_eos_token_id"),
                   ("codec_pad_id", "codec_pad_id"), ("codec_think_id", "codec_think_id"),
                   ("codec_nothink_id", "codec_nothink_id"), ("codec_think_bos_id", "codec_think_bos_id"),
                   ("codec_think_eos_id", "codec_think_eos_id")):
        w.set_kv("talker." + key, getattr(c, k))
    w.set_kv("talker.mrope_section", [24, 20, 20])
    w.set_kv("talker.mrope_interleaved", 1)
    for name, lid in c.languages:
        w.set_kv(f"talker.language.{name}", lid)
    _transformer_kv(w, "cp", c.cp)
    w.set_kv("cp.num_code_groups", c.n_code_groups)
    w.set_kv("speaker.enc_dim", c.spk_dim)
    w.set_kv("speaker.sample_rate", c.sample_rate)
    for k, v in dict(n_fft=1024, num_mels=128, hop_size=256, win_size=1024, fmin=0, fmax=12000).items():
        w.set_kv(f"speaker.mel.{k}", v)
    w.set_kv("codec.input_sample_rate", c.sample_rate)
    w.set_kv("codec.output_sample_rate", c.sample_rate)
    w.set_kv("codec.decode_upsample_rate", c.samples_per_frame)
    w.set_kv("codec.encode_downsample_rate", c.samples_per_frame)
    _transformer_kv(w, "codec.decoder", c.vocoder)
    for k, v in dict(latent_dim=c.vq_latent, codebook_dim=c.vq_codebook_dim, codebook_size=c.vq_codebook_size,
                     decoder_dim=c.decoder_dim, num_quantizers=c.vq_n_q,
                     num_semantic_quantizers=c.vq_n_semantic, sliding_window=c.sliding_window).items():
        w.set_kv(f"codec.decoder.{k}", v)
    w.set_kv("codec.decoder.upsample_rates", list(c.upsample_rates))
    w.set_kv("codec.decoder.upsampling_ratios", list(c.upsampling_ratios))
    for k, v in c.gen.items():
        w.set_kv(f"gen.{k}", v)


# --- tensor table ---------------------------------------------------------------------

def _decoder_layers(prefix: str, t: Transformer, qk_norm: bool):
    H, Q, K, F, D = t.hidden, t.n_head * t.head_dim, t.n_kv_head * t.head_dim, t.ff, t.head_dim
    out = []
    for l in range(t.n_layer):
        p = f"{prefix}.layers.{l}."
        out += [(p + "input_layernorm.weight", (H,)), (p + "post_attention_layernorm.weight", (H,)),
                (p + "self_attn.q_proj.weight", (Q, H)), (p + "self_attn.k_proj.weight", (K, H)),
                (p + "self_attn.v_proj.weight", (K, H)), (p + "self_attn.o_proj.weight", (H, Q))]
        if qk_norm:
            out += [(p + "self_attn.q_norm.weight", (D,)), (p + "self_attn.k_norm.weight", (D,))]
        out += [(p + "mlp.gate_proj.weight", (F, H)), (p + "mlp.up_proj.weight", (F, H)),
                (p + "mlp.down_proj.weight", (H, F))]
    return out


def tensor_table(c: ModelConfig):
    """[(name, shape)] for every weight tensor, in file order."""
    H, TH, TV, CV, PV, G = c.talker.hidden, c.text_hidden, c.text_vocab, c.talker.vocab, c.cp.vocab, c.n_code_groups
    out = [("talker.model.text_embedding.weight", (TV, TH)),
           ("talker.text_projection.linear_fc1.weight", (TH, TH)),
           ("talker.text_projection.linear_fc1.bias", (TH,)),
           ("talker.text_projection.linear_fc2.weight", (H, TH)),
           ("talker.text_projection.linear_fc2.bias", (H,)),
           ("talker.model.codec_embedding.weight", (CV, H))]
    out += _decoder_layers("talker.model", c.talker, True)
    out += [("talker.model.norm.weight", (H,)), ("talker.codec_head.weight", (CV, H))]
    CH = c.cp.hidden
    for i in range(G - 1):
        out.append((f"talker.code_predictor.model.codec_embedding.{i}.weight", (PV, CH)))
    for i in range(G - 1):
        out.append((f"talker.code_predictor.lm_head.{i}.weight", (PV, CH)))
    out += _decoder_layers("talker.code_predictor.model", c.cp, True)
    out.append(("talker.code_predictor.model.norm.weight", (CH,)))
    # speaker encoder (ECAPA-TDNN), shapes as the released checkpoint ships them
    C, R, SE, MFA, ASP = 512, 64, 128, 1536, 128
    out += [("speaker_encoder.blocks.0.conv.weight", (C, 128, 5)), ("speaker_encoder.blocks.0.conv.bias", (C,))]
    for b in range(1, 4):
        bp = f"speaker_encoder.blocks.{b}."
        out += [(bp + "tdnn1.conv.weight", (C, C, 1)), (bp + "tdnn1.conv.bias", (C,))]
        for r in range(7):
            rp = f"{bp}res2net_block.blocks.{r}.conv."
            out += [(rp + "weight", (R, R, 3)), (rp + "bias", (R,))]
        out += [(bp + "tdnn2.conv.weight", (C, C, 1)), (bp + "tdnn2.conv.bias", (C,)),
                (bp + "se_block.conv1.weight", (SE, C, 1)), (bp + "se_block.conv1.bias", (SE,)),
                (bp + "se_block.conv2.weight", (C, SE, 1)), (bp + "se_block.conv2.bias", (C,))]
    out += [("speaker_encoder.mfa.conv.weight", (MFA, MFA, 1)), ("speaker_encoder.mfa.conv.bias", (MFA,)),
            ("speaker_encoder.asp.tdnn.conv.weight", (ASP, 3 * MFA, 1)), ("speaker_encoder.asp.tdnn.conv.bias", (ASP,)),
            ("speaker_encoder.asp.conv.weight", (MFA, ASP, 1)), ("speaker_encoder.asp.conv.bias", (MFA,)),
            ("speaker_encoder.fc.weight", (c.spk_dim, 2 * MFA, 1)), ("speaker_encoder.fc.bias", (c.spk_dim,))]
    # codec decoder
    L, CD, CS, NQ, NS, DD = c.vq_latent, c.vq_codebook_dim, c.vq_codebook_size, c.vq_n_q, c.vq_n_semantic, c.decoder_dim
    VQ = CD // 2
    q = "codec.decoder.quantizer."
    out += [(q + "rvq_first.input_proj.weight", (VQ, CD, 1)), (q + "rvq_first.output_proj.weight", (CD, VQ, 1))]
    for i in range(NS):
        out.append((f"{q}rvq_first.vq.layers.{i}._codebook.codebook", (CS, VQ)))
    out += [(q + "rvq_rest.input_proj.weight", (VQ, CD, 1)), (q + "rvq_rest.output_proj.weight", (CD, VQ, 1))]
    for i in range(NQ - NS):
        out.append((f"{q}rvq_rest.vq.layers.{i}._codebook.codebook", (CS, VQ)))
    out += [("codec.decoder.pre_conv.conv.weight", (L, CD, 3)), ("codec.decoder.pre_conv.conv.bias", (L,))]
    VH = c.vocoder.hidden
    pt = "codec.decoder.pre_transformer."
    out += [(pt + "input_proj.weight", (VH, L)), (pt + "input_proj.bias", (VH,))]
    out += _decoder_layers("codec.decoder.pre_transformer", c.vocoder, False)
    for l in range(c.vocoder.n_layer):
        lp = f"{pt}layers.{l}."
        out += [(lp + "self_attn_layer_scale.scale", (VH,)), (lp + "mlp_layer_scale.scale", (VH,))]
    out += [(pt + "norm.weight", (VH,)), (pt + "output_proj.weight", (L, VH)), (pt + "output_proj.bias", (L,))]
    for u, r in enumerate(c.upsampling_ratios):
        up = f"codec.decoder.upsample.{u}."
        out += [(up + "0.conv.weight", (L, L, r)), (up + "0.conv.bias", (L,)),
                (up + "1.dwconv.conv.weight", (L, 1, 7)), (up + "1.dwconv.conv.bias", (L,)),
                (up + "1.norm.weight", (L,)), (up + "1.norm.bias", (L,)),
                (up + "1.pwconv1.weight", (4 * L, L)), (up + "1.pwconv1.bias", (4 * L,)),
                (up + "1.pwconv2.weight", (L, 4 * L)), (up + "1.pwconv2.bias", (L,)), (up + "1.gamma", (L,))]
    out += [("codec.decoder.decoder.0.conv.weight", (DD, L, 7)), ("codec.decoder.decoder.0.conv.bias", (DD,))]
    width = DD
    for i, rate in enumerate(c.upsample_rates):
        bp = f"codec.decoder.decoder.{i + 1}.block."
        ow = width // 2
        out += [(bp + "0.alpha", (width,)), (bp + "0.beta", (width,)),
                (bp + "1.conv.weight", (width, ow, 2 * rate)), (bp + "1.conv.bias", (ow,))]
        for r in range(3):
            rp = f"{bp}{2 + r}."
            out += [(rp + "act1.alpha", (ow,)), (rp + "act1.beta", (ow,)),
                    (rp + "conv1.conv.weight", (ow, ow, 7)), (rp + "conv1.conv.bias", (ow,)),
                    (rp + "act2.alpha", (ow,)), (rp + "act2.beta", (ow,)),
                    (rp + "conv2.conv.weight", (ow, ow, 1)), (rp + "conv2.conv.bias", (ow,))]
        width = ow
    n = len(c.upsample_rates)
    out += [(f"codec.decoder.decoder.{n + 1}.alpha", (width,)), (f"codec.decoder.decoder.{n + 1}.beta", (width,)),
            (f"codec.decoder.decoder.{n + 2}.conv.weight", (1, width, 7)), (f"codec.decoder.decoder.{n + 2}.conv.bias", (1,))]
    return out


def component_seed(name: str) -> int:
    if name.startswith("talker.code_predictor."):
        return 2
    if name.startswith("talker."):
        return 1
    if name.startswith("codec."):
        return 3
    return 4


def _is_norm_weight(name: str) -> bool:
    return name.endswith("norm.weight") or name.endswith("layernorm.weight")


CHUNK_ELEMS = 1 << 22   # tensors are drawn in row chunks of about this many elements, one stream per chunk


def _chunks(shape: tuple):
    rows = shape[0]
    per_row = int(np.prod(shape[1:])) if len(shape) > 1 else 1
    step = max(1, CHUNK_ELEMS // max(per_row, 1))
    return [(r, min(rows, r + step)) for r in range(0, rows, step)]


def _draw(name: str, shape: tuple, r0: int, r1: int, ci: int, seed_offset: int, out: np.ndarray) -> None:
    rng = np.random.Generator(np.random.PCG64(np.random.SeedSequence(
        [component_seed(name) + seed_offset, zlib.crc32(name.encode()), ci])))
    a = rng.standard_normal(size=(r1 - r0,) + tuple(shape[1:]), dtype=np.float32)
    a *= np.float32(0.02)
    out[r0:r1] = a


def synth_tensor(name: str, shape: tuple, seed_offset: int = 0, pool=None) -> np.ndarray:
    """The seeded value of one synthetic tensor (f16 for >=2-D, f32 for 1-D).
    Row chunk i of a tensor draws from PCG64(SeedSequence([component seed, crc32(name), i]))."""
    out = np.empty(shape, dtype=np.float16 if len(shape) >= 2 else np.float32)
    jobs = [(ci, r0, r1) for ci, (r0, r1) in enumerate(_chunks(shape))]
    run = lambda j: _draw(name, shape, j[1], j[2], j[0], seed_offset, out)
    list(pool.map(run, jobs)) if pool is not None and len(jobs) > 1 else [run(j) for j in jobs]
    if len(shape) == 1 and _is_norm_weight(name):
        out += np.float32(1.0)
    return out


def synthetic_tokenizer(c: ModelConfig) -> tuple[str, str, str]:
    """Tokenizer files of a synthetic model: a byte-level vocabulary (ids 0..255, one per byte,
    no merges) with the chat tokens as added tokens at the model's ids ("assistant" one of
    them, so the prompt template has the 3-id header and 5-id trailer the talker expects)."""
    from .tokenizer import BYTE_TO_CHAR
    vocab = {BYTE_TO_CHAR[b]: b for b in range(256)}
    added = {c.im_start_id: "<|im_start|>", c.im_end_id: "<|im_end|>", c.assistant_id: "assistant", c.tts_pad_id: "<|tts_pad|>",
             c.tts_bos_id: "<|tts_text_bos|>", c.tts_eos_id: "<|tts_text_eod|>"}
    cfg = {"added_tokens_decoder": {str(i): {"content": t, "lstrip": False, "rstrip": False, "single_word": False,
                                             "normalized": False, "special": t.startswith("<|")} for i, t in sorted(added.items())}}
    return json.dumps(vocab, ensure_ascii=False), "#version: 0.2\n", json.dumps(cfg)


def write_synthetic(path: str | Path, c: ModelConfig, seed_offset: int = 0, threads: int = 8,
                    include: callable = None) -> int:
    """Writes a complete `.navi` for config `c` with seeded random weights.
    `include(name)` can drop tensors (they are then absent from the table)."""
    w = NaviBuilder()
    kv_entries(w, c)
    for tname, text in zip(("tokenizer.vocab.json", "tokenizer.merges.txt", "tokenizer.config.json"), synthetic_tokenizer(c)):
        w.put_tensor(tname, U8, np.frombuffer(text.encode("utf-8"), dtype=np.uint8))
    table = [(n, s) for n, s in tensor_table(c) if include is None or include(n)]
    with ThreadPoolExecutor(max_workers=threads) as ex:
        arrays = [synth_tensor(n, s, seed_offset, ex) for n, s in table]
    for (name, shape), arr in zip(table, arrays):
        w.put_tensor(name, F16 if len(shape) >= 2 else F32, arr)
    return w.save(path)


def load_weights(path: str | Path) -> dict:
    """name -> float32 numpy array (f16 values upcast) for every non-U8 tensor."""
    from .navi_file import NaviFile
    f = NaviFile.open(path)
    out = {}
    for t in f.tensors:
        if t.dtype == U8:
            continue
        out[t.name] = np.asarray(f.array(t), dtype=np.float32)
    return out


def config_from_kv(kv: dict) -> ModelConfig:
    """Rebuilds the ModelConfig a `.navi` KV section describes."""
    def tr(ns, vocab_default=0):
        return Transformer(kv[f"{ns}.hidden_size"], kv[f"{ns}.num_hidden_layers"], kv[f"{ns}.num_attention_heads"],
                           kv[f"{ns}.num_key_value_heads"], kv[f"{ns}.head_dim"], kv[f"{ns}.intermediate_size"],
                           float(kv[f"{ns}.rms_norm_eps"]), float(kv[f"{ns}.rope_theta"]),
                           kv.get(f"{ns}.vocab_size", vocab_default), kv.get(f"{ns}.max_position_embeddings", 0))
    langs = tuple((k[len("talker.language."):], v) for k, v in kv.items() if k.startswith("talker.language."))
    gen = {k[4:]: v for k, v in kv.items() if k.startswith("gen.")}
    return ModelConfig(
        name=kv["general.name"], talker=tr("talker"), cp=tr("cp"), vocoder=tr("codec.decoder"),
        text_vocab=kv["talker.text_vocab_size"], text_hidden=kv["talker.text_hidden_size"],
        n_code_groups=kv["talker.num_code_groups"], im_start_id=kv["text.im_start_id"], im_end_id=kv["text.im_end_id"],
        assistant_id=kv["text.assistant_id"], tts_pad_id=kv["text.tts_pad_id"], tts_bos_id=kv["text.tts_bos_id"],
        tts_eos_id=kv["text.tts_eos_id"], codec_pad_id=kv["talker.codec_pad_id"], codec_bos_id=kv["talker.codec_bos_id"],
        codec_eos_id=kv["talker.codec_eos_token_id"], codec_think_id=kv["talker.codec_think_id"],
        codec_nothink_id=kv["talker.codec_nothink_id"], codec_think_bos_id=kv["talker.codec_think_bos_id"],
        codec_think_eos_id=kv["talker.codec_think_eos_id"], languages=langs, spk_dim=kv["speaker.enc_dim"],
        vq_latent=kv["codec.decoder.latent_dim"], vq_codebook_dim=kv["codec.decoder.codebook_dim"],
        vq_codebook_size=kv["codec.decoder.codebook_size"], vq_n_q=kv["codec.decoder.num_quantizers"],
        vq_n_semantic=kv["codec.decoder.num_semantic_quantizers"], decoder_dim=kv["codec.decoder.decoder_dim"],
        sliding_window=kv.get("codec.decoder.sliding_window", 0),
        upsample_rates=tuple(kv["codec.decoder.upsample_rates"]),
        upsampling_ratios=tuple(kv["codec.decoder.upsampling_ratios"]),
        sample_rate=kv["codec.output_sample_rate"], gen=gen)


def with_decoder_dim(c: ModelConfig, d: int) -> ModelConfig:
    return replace(c, decoder_dim=d, name=c.name.rsplit("-d", 1)[0] + f"-d{d}")
