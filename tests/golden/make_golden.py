"""Writes the committed golden fixtures of this directory. Run from the repository root:

    python tests/golden/make_golden.py

- navi_ref_small.json: what the reference engine's own .navi reader and tensor table
  (runtime/weights/navi_file.cpp, model/qwen3tts/params.cpp, compiled into oracle/_ref by
  oracle/Makefile from the reference sources) make of the seeded small synthetic model
  that navi_b200.model_spec writes: the reference accepts the file, and its hyperparameters
  are the ones recorded. Needs oracle/_ref/navi_ref_check (built only where the reference
  tree is present).
- decoder_layer_small.npz: one talker and one code-predictor decoder layer of that model,
  evaluated by transformers' Qwen3DecoderLayer (fp32, eager) on seeded inputs: an
  implementation independent of the oracle.
- sampler_golden.json: the draws of the sampler specification (oracle/sampler.c) on seeded
  logits across temperature / top-k / top-p / RNG / codebook-0 modifications; the device
  sampler must return the same ids.
"""
import json
import os
import subprocess
import sys
import tempfile

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "navi-tts_b200"))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

from navi_b200 import model_spec  # noqa: E402
from oracle import model as om  # noqa: E402


def sampler_cases():
    """(name, V, rng, codebook, temperature, top_k, top_p, seed, frame_index, logits seed)"""
    out = []
    k = 0
    for V in (2048, 3072):
        for rng in (0, 1):
            for cb in (0, 5):
                for (temp, top_k, top_p) in ((0.9, 50, 1.0), (0.9, 50, 0.9), (0.7, 20, 0.8), (1.0, 0, 0.95), (0.0, 50, 1.0)):
                    out.append(dict(V=V, rng=rng, codebook=cb, temperature=temp, top_k=top_k, top_p=top_p,
                                    seed=1000 + k, frame_index=k % 7, logits_seed=k))
                    k += 1
    return out


def case_logits(c):
    return (np.random.default_rng(c["logits_seed"]).standard_normal(c["V"]) * 3.0).astype(np.float32)


def case_seen(c):
    seen = np.zeros(c["V"], np.uint8)
    seen[np.random.default_rng(c["logits_seed"] + 7).integers(0, c["V"], 40)] = 1
    return seen


def case_sampling(c):
    return om.Sampling(temperature=c["temperature"], top_k=c["top_k"], top_p=c["top_p"], cp_temperature=c["temperature"],
                       cp_top_k=c["top_k"], cp_top_p=c["top_p"], rng=c["rng"])


def case_draw(c):
    lg = case_logits(c)
    mods = (c["V"] - 1024, c["V"] - 1022, case_seen(c)) if c["codebook"] == 0 else None
    return om.sample(lg, c["codebook"], case_sampling(c), c["seed"], c["frame_index"], talker_mods=mods)


def main():
    with tempfile.TemporaryDirectory() as td:
        path = os.path.join(td, "small.navi")
        model_spec.write_synthetic(path, model_spec.small_config())
        ref = os.path.join(ROOT, "oracle", "_ref", "navi_ref_check")
        if os.path.exists(ref):
            r = subprocess.run([ref, path], capture_output=True, text=True)
            j = json.loads(r.stdout)
            j["generator"] = "model_spec.write_synthetic(small_config()) read by the reference's NaviFile + validate"
            with open(os.path.join(HERE, "navi_ref_small.json"), "w") as f:
                json.dump(j, f, indent=1)
        else:
            print("oracle/_ref/navi_ref_check missing: navi_ref_small.json left as it is")
        # decoder layers by transformers
        from test_oracle_pins import _qwen3_layer_reference
        W = om.Weights.from_navi(path)
        arrays = {}
        for comp in ("talker", "cp"):
            d = W.tl if comp == "talker" else W.cp
            x = torch.from_numpy(np.random.default_rng(11).standard_normal((5, d.hidden)).astype(np.float32))
            y = _qwen3_layer_reference(W, comp, 1, x, 0)
            arrays[f"{comp}_x"] = x.numpy()
            arrays[f"{comp}_y"] = y.numpy()
        np.savez_compressed(os.path.join(HERE, "decoder_layer_small.npz"), **arrays)
    cases = sampler_cases()
    for c in cases:
        c["id"] = case_draw(c)
    with open(os.path.join(HERE, "sampler_golden.json"), "w") as f:
        json.dump({"logits": "np.random.default_rng(logits_seed).standard_normal(V) * 3, as f32",
                   "seen": "codebook 0: u8[V], ones at np.random.default_rng(logits_seed + 7).integers(0, V, 40)",
                   "mods": "codebook 0: suppress_from V - 1024, eos V - 1022, min_frames 2, repetition_penalty 1.05",
                   "cases": cases}, f, indent=1)
    print("wrote", os.listdir(HERE))


if __name__ == "__main__":
    main()
