"""ctypes binding of include/navi_b200.h (the C ABI of libnavi_b200.so).

This is the stub a Python host binds; the same signatures serve cgo / JNI / N-API
hosts.  Loading fails loudly when the library is missing: there is no fallback.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char, c_char_p, c_double, c_float, c_int, c_int32, c_size_t, c_uint8, c_uint16, c_uint64, c_void_p

# NAVI_B200_LIB overrides the library path (e.g. a variant build); the default is the in-tree build.
LIB_PATH = os.environ.get("NAVI_B200_LIB") or os.path.join(os.path.dirname(os.path.abspath(__file__)), "libnavi_b200.so")

NAVI_OK, NAVI_E_ARG, NAVI_E_CUDA, NAVI_E_FORMAT, NAVI_E_TIMEOUT, NAVI_E_KV_FULL, NAVI_E_LAUNCH, NAVI_E_SHAPE, NAVI_E_NOMEM = range(9)
NAVI_FRAME_SLOTS = 4
NAVI_RNG_PCG, NAVI_RNG_PHILOX = 0, 1
NAVI_SAMPLE_STATIC_MAX_VOCAB = 32768


class DeviceInfo(ctypes.Structure):
    _fields_ = [("ordinal", c_int), ("name", c_char * 128), ("cc_major", c_int), ("cc_minor", c_int),
                ("multiprocessors", c_int), ("cooperative_launch", c_int), ("smem_per_block_optin", c_size_t),
                ("l2_bytes", c_size_t), ("vram_total", c_size_t), ("vram_free", c_size_t)]


class TransformerParams(ctypes.Structure):
    _fields_ = [("hidden", c_int), ("n_layer", c_int), ("n_head", c_int), ("n_kv_head", c_int), ("head_dim", c_int),
                ("ff", c_int), ("vocab", c_int), ("max_pos", c_int), ("rms_eps", c_float), ("rope_theta", c_double)]


class Params(ctypes.Structure):
    _fields_ = [("talker", TransformerParams), ("cp", TransformerParams), ("vocoder", TransformerParams),
                ("text_vocab", c_int), ("text_hidden", c_int), ("n_code_groups", c_int),
                ("tts_bos_id", c_int), ("tts_eos_id", c_int), ("tts_pad_id", c_int),
                ("codec_bos_id", c_int), ("codec_eos_id", c_int), ("codec_pad_id", c_int),
                ("codec_think_id", c_int), ("codec_nothink_id", c_int), ("codec_think_bos_id", c_int),
                ("codec_think_eos_id", c_int), ("vq_latent", c_int), ("vq_codebook_dim", c_int),
                ("vq_codebook_size", c_int), ("vq_n_q", c_int), ("vq_n_semantic", c_int), ("decoder_dim", c_int),
                ("sliding_window", c_int), ("upsample_rates", c_int * 4), ("upsampling_ratios", c_int * 2),
                ("codec_upsample", c_int), ("sample_rate", c_int), ("temperature", c_float), ("top_p", c_float),
                ("repetition_penalty", c_float), ("cp_temperature", c_float), ("cp_top_p", c_float),
                ("top_k", c_int), ("cp_top_k", c_int)]


class KV(ctypes.Structure):
    _fields_ = [("n_layer", c_int), ("max_pos", c_int), ("kv_dim", c_int), ("n_used", c_int),
                ("k", POINTER(POINTER(c_uint16))), ("v", POINTER(POINTER(c_uint16)))]


class Sampling(ctypes.Structure):
    _fields_ = [("temperature", c_float), ("top_k", c_int), ("top_p", c_float), ("repetition_penalty", c_float),
                ("cp_temperature", c_float), ("cp_top_k", c_int), ("cp_top_p", c_float), ("min_frames", c_int),
                ("rng", c_int)]


class Prompt(ctypes.Structure):
    _fields_ = [("prefill", c_void_p), ("trailing", c_void_p), ("tts_pad", c_void_p), ("n_prefill", c_int), ("n_trailing", c_int)]


class SynthStats(ctypes.Structure):
    _fields_ = [("n_tokens", c_int), ("n_frames", c_int), ("hit_cap", c_int), ("eos", c_int), ("prefill_ms", c_double),
                ("frames_ms", c_double), ("total_ms", c_double), ("ttfc_ms", c_double), ("vocoder_ms", c_double),
                ("ttfa_ms", c_double), ("audio_s", c_double), ("rtf", c_double)]


class ConvArgs(ctypes.Structure):
    _fields_ = [("w", c_void_p), ("Cout", c_int), ("Cin", c_int), ("K", c_int), ("dil", c_int), ("trans_stride", c_int),
                ("x", c_void_p), ("x_stride", c_int), ("T", c_int), ("hist", c_void_p), ("pro", c_int), ("snake_a", c_void_p),
                ("snake_b", c_void_p), ("epi", c_int), ("bias", c_void_p), ("resid", c_void_p), ("scale", c_void_p),
                ("y", c_void_p), ("y_stride", c_int), ("rowmajor", c_int)]


class SynthRequest(ctypes.Structure):
    _fields_ = [("ids", POINTER(c_int32)), ("n_ids", c_int), ("language", c_char_p), ("speaker", POINTER(c_float)), ("seed", c_uint64),
                ("max_frames", c_int), ("codes", POINTER(c_int32)), ("codes_cap", c_int)]


STREAM_PCM_FN = ctypes.CFUNCTYPE(None, c_int, POINTER(c_float), c_int, c_void_p)
STAGE_FN = ctypes.CFUNCTYPE(None, c_void_p, c_char_p, c_void_p, c_int, c_int)
PCM_FN = ctypes.CFUNCTYPE(None, POINTER(c_float), c_int, c_void_p)


class FrameOpts(ctypes.Structure):
    _fields_ = [("blocks_per_mp", c_int), ("deadline_us", c_uint64)]


class FrameResult(ctypes.Structure):
    _fields_ = [("ok", c_int), ("eos", c_int), ("codes", c_int32 * 16), ("us", c_double), ("status", c_int)]


# (name, restype, argtypes) of every exported function, in header order
SIGNATURES = [
    ("navi_version", c_char_p, []),
    ("navi_last_error", c_char_p, []),
    ("navi_device_count", c_int, [POINTER(c_int)]),
    ("navi_device_open", c_int, [c_int, POINTER(c_void_p)]),
    ("navi_device_get_info", c_int, [c_void_p, POINTER(DeviceInfo)]),
    ("navi_device_stream", c_void_p, [c_void_p]),
    ("navi_device_close", None, [c_void_p]),
    ("navi_weights_upload", c_int, [c_void_p, c_char_p, POINTER(c_void_p)]),
    ("navi_weights_get_params", c_int, [c_void_p, POINTER(Params)]),
    ("navi_model_probe", c_int, [c_char_p, POINTER(Params), POINTER(c_int), POINTER(c_int), POINTER(c_int), POINTER(c_int)]),
    ("navi_weights_tensor", c_void_p, [c_void_p, c_char_p, POINTER(c_int), POINTER(c_int), POINTER(c_uint64)]),
    ("navi_weights_bytes", c_uint64, [c_void_p]),
    ("navi_weights_free", None, [c_void_p]),
    ("navi_kv_create", c_int, [c_void_p, c_int, c_int, c_int, POINTER(POINTER(KV))]),
    ("navi_kv_destroy", None, [POINTER(KV)]),
    ("navi_talker_create", c_int, [c_void_p, c_void_p, c_int, c_int, POINTER(c_void_p)]),
    ("navi_talker_build_prompt", c_int, [c_void_p, POINTER(c_int32), c_int, c_char_p, POINTER(c_float), POINTER(Prompt)]),
    ("navi_talker_prefill", c_int, [c_void_p, POINTER(Prompt)]),
    ("navi_talker_kv", c_int, [c_void_p, POINTER(KV)]),
    ("navi_talker_hidden", c_void_p, [c_void_p]),
    ("navi_talker_logits", c_void_p, [c_void_p]),
    ("navi_talker_last_ms", c_double, [c_void_p]),
    ("navi_talker_destroy", None, [c_void_p]),
    ("navi_frame_create", c_int, [c_void_p, c_void_p, POINTER(FrameOpts), POINTER(c_void_p)]),
    ("navi_frame_reset", c_int, [c_void_p]),
    ("navi_frame_run_first", c_int, [c_void_p, c_void_p, c_void_p, c_void_p, POINTER(Sampling), c_uint64, c_int,
                                     POINTER(FrameResult)]),
    ("navi_frame_run", c_int, [c_void_p, POINTER(KV), c_int, c_void_p, POINTER(Sampling), c_uint64, c_int,
                               POINTER(FrameResult)]),
    ("navi_frame_run_layer", c_int, [c_void_p, c_int, c_void_p, POINTER(KV), c_int, c_void_p, POINTER(FrameResult)]),
    ("navi_frame_enqueue", c_int, [c_void_p, POINTER(KV), c_int, c_void_p, POINTER(Sampling), c_uint64, c_int]),
    ("navi_frame_collect", c_int, [c_void_p, POINTER(FrameResult)]),
    ("navi_frame_step_out", c_void_p, [c_void_p]),
    ("navi_frame_set_step_in", c_int, [c_void_p, c_void_p]),
    ("navi_frame_grid_blocks", c_int, [c_void_p]),
    ("navi_frame_reset_slot", c_int, [c_void_p, c_int]),
    ("navi_frame_run_first_slot", c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, POINTER(Sampling), c_uint64, c_int,
                                          POINTER(FrameResult)]),
    ("navi_frame_run_batch", c_int, [c_void_p, c_int, POINTER(c_int), POINTER(POINTER(KV)), POINTER(c_int), POINTER(c_void_p),
                                     POINTER(Sampling), POINTER(c_uint64), POINTER(c_int), POINTER(FrameResult)]),
    ("navi_frame_run_first_batch", c_int, [c_void_p, c_int, POINTER(c_int), POINTER(c_void_p), POINTER(c_void_p), POINTER(c_void_p),
                                           POINTER(Sampling), POINTER(c_uint64), POINTER(c_int), POINTER(FrameResult)]),
    ("navi_frame_enqueue_batch", c_int, [c_void_p, c_int, POINTER(c_int), POINTER(POINTER(KV)), POINTER(c_int), POINTER(c_void_p),
                                         POINTER(Sampling), POINTER(c_uint64), POINTER(c_int)]),
    ("navi_frame_collect_batch", c_int, [c_void_p, c_int, POINTER(FrameResult)]),
    ("navi_frame_step_out_slot", c_void_p, [c_void_p, c_int]),
    ("navi_frame_set_step_in_slot", c_int, [c_void_p, c_int, c_void_p]),
    ("navi_frame_inspect_stream", c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p]),
    ("navi_frame_destroy", None, [c_void_p]),
    ("navi_graph_create", c_int, [c_void_p, c_void_p, POINTER(FrameOpts), c_int, c_int, c_int, POINTER(c_void_p)]),
    ("navi_graph_synth_ids", c_int, [c_void_p, POINTER(c_int32), c_int, c_char_p, POINTER(c_float), POINTER(Sampling), c_uint64,
                                     c_int, POINTER(c_int32), c_int, POINTER(SynthStats)]),
    ("navi_graph_synth", c_int, [c_void_p, POINTER(c_int32), c_int, c_char_p, POINTER(c_float), POINTER(Sampling), c_uint64, c_int,
                                 c_int, c_int, POINTER(c_int32), c_int, PCM_FN, c_void_p, POINTER(SynthStats)]),
    ("navi_graph_destroy", None, [c_void_p]),
    ("navi_graph_create_streams", c_int, [c_void_p, c_void_p, POINTER(FrameOpts), c_int, c_int, c_int, c_int, POINTER(c_void_p)]),
    ("navi_graph_synth_batch", c_int, [c_void_p, c_int, POINTER(SynthRequest), POINTER(Sampling), c_int, c_int, STREAM_PCM_FN, c_void_p,
                                       POINTER(SynthStats)]),
    ("navi_vocoder_create", c_int, [c_void_p, c_void_p, c_int, c_int, POINTER(c_void_p)]),
    ("navi_vocoder_reset", c_int, [c_void_p]),
    ("navi_vocoder_decode", c_int, [c_void_p, POINTER(c_int32), c_int, POINTER(c_float), ctypes.c_size_t]),
    ("navi_vocoder_samples_per_frame", c_int, [c_void_p]),
    ("navi_vocoder_max_chunk_frames", c_int, [c_void_p]),
    ("navi_vocoder_last_ms", c_double, [c_void_p]),
    ("navi_vocoder_set_stage_hook", c_int, [c_void_p, STAGE_FN, c_void_p]),
    ("navi_vocoder_destroy", None, [c_void_p]),
    ("navi_conv1d", c_int, [c_void_p, POINTER(ConvArgs)]),
    ("navi_frame_inspect", c_int, [c_void_p, c_void_p, c_void_p, c_void_p]),
    ("navi_frame_set_profile", c_int, [c_void_p, c_int, c_int]),
    ("navi_frame_profile", c_int, [c_void_p, POINTER(c_uint64), c_int, POINTER(c_int)]),
    ("navi_sample_logits", c_int, [c_void_p, c_void_p, c_int, POINTER(Sampling), c_uint64, c_int, c_int, c_int, c_int,
                                   c_void_p, POINTER(c_int32)]),
    ("navi_sample_logits_static", c_int, [c_void_p, c_void_p, c_int, POINTER(Sampling), c_uint64, c_int, c_int, c_int,
                                          c_int, c_void_p, POINTER(c_int32)]),
]

_lib = None


def lib():
    """The loaded library with typed prototypes. Raises if the library is missing."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with __graft_entry__.build() "
                               "(there is no CPU fallback for the navi-b200 path)")
        L = ctypes.CDLL(LIB_PATH)
        for name, res, args in SIGNATURES:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


class NaviError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"[status {status}] {msg}")
        self.status = status


def check(status: int) -> None:
    if status != NAVI_OK:
        raise NaviError(status, lib().navi_last_error().decode(errors="replace"))
