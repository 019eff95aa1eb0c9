"""Writes tests/golden/ref_frame_small.npz, ref_vocoder_small.npz, ref_talker_small.npz: outputs of the reference
engine's own frame code, vocoder and talker (oracle/_ref/ref_*_check, built from
the reference sources by `make -C oracle REF=...`) on the seeded small synthetic model -- one
frame at KV 10, a set of sampler draws, a set of per-frame seeds, and the PCM of 7 frames
decoded in chunks of 3, and a talker prompt + prefill -- so tests/test_reference_*pins.py can
pin the oracle where the reference tree is absent.

    python tests/golden/make_ref_golden.py
"""
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [os.path.join(ROOT, "navi-tts_b200"), ROOT, os.path.dirname(HERE)]

from navi_b200 import model_spec  # noqa: E402
from oracle import model as om  # noqa: E402
from oracle import ref_frame as rf  # noqa: E402
from test_reference_pins import _frame_inputs  # noqa: E402


def main():
    with tempfile.TemporaryDirectory() as td:
        navi = os.path.join(td, "small.navi")
        model_spec.write_synthetic(navi, model_spec.small_config())
        W = om.Weights.from_navi(navi)
        tl = W.tl
        n_past, input_seed, seed, fi = 10, 110, 1234, 3
        kv, step, trailing, seen = _frame_inputs(W, n_past, seed=input_seed)
        dims = (tl.hidden, tl.vocab, W.cp.vocab, tl.n_layer, tl.n_kv_head * tl.head_dim)
        r = rf.frame(navi, dims, rf.RefSampling(), seed, fi, seen, trailing.numpy(), step_in=step.numpy(),
                     kv=[(k.numpy(), v.numpy()) for k, v in kv], n_past=n_past)
        assert r.ok
        rng = np.random.default_rng(21)
        cases, meta, logits, seens = [], [], [], []
        for i in range(24):
            cb = i % 4 * 5 % 16
            V = tl.vocab if cb == 0 else W.cp.vocab
            x = np.full(tl.vocab, np.nan, np.float32)
            x[:V] = rng.standard_normal(V).astype(np.float32) * 3
            temp, k = (900, 50) if i % 3 else (1300, 7)
            sn = (rng.random(tl.vocab) < 0.05).astype(np.uint8)
            s = rf.RefSampling(temperature=temp / 1000, top_k=k, cp_temperature=temp / 1000, cp_top_k=k)
            sd = int(rng.integers(1 << 40))
            cases.append((s, sd, i, cb, x[:V], sn))
            meta.append((cb, i, sd, temp, k))
            logits.append(x)
            seens.append(sn)
        ids = rf.sample(navi, cases)
        pairs = [(int(rng.integers(1 << 62)), int(rng.integers(-3, 5000))) for _ in range(16)]
        sds = rf.seeds(navi, pairs)
        np.savez_compressed(os.path.join(HERE, "ref_frame_small.npz"), n_past=n_past, input_seed=input_seed, seed=seed,
                            frame_index=fi, codes=np.array(r.codes, np.int32), hidden=r.hidden, logits=r.logits,
                            clogits=r.clogits, step_out=r.step_out, seen=r.seen, k_rows=np.stack(r.k_rows),
                            v_rows=np.stack(r.v_rows), draw_ids=np.array(ids, np.int32), draw_meta=np.array(meta, np.int64),
                            draw_logits=np.stack(logits), draw_seen=np.stack(seens),
                            seeds=np.array([(p[0], p[1], s[0], s[1]) for p, s in zip(pairs, sds)], np.uint64))
        print("wrote ref_frame_small.npz; codes", r.codes)
        vc = np.random.default_rng(31).integers(0, W.cfg.vq_codebook_size, (7, W.cfg.vq_n_q)).astype(np.int32)
        pcm, _ = rf.vocoder_decode(navi, vc, max_chunk=3)
        np.savez_compressed(os.path.join(HERE, "ref_vocoder_small.npz"), codes=vc, max_chunk=3, pcm=pcm)
        print("wrote ref_vocoder_small.npz;", pcm.size, "samples")
        from test_reference_talker_pins import prompt_ids
        ids = prompt_ids(W.cfg, 23, 23)
        spk = np.random.default_rng(24).standard_normal(tl.hidden).astype(np.float32)
        pre, trail, pad, hid, lg, kv = rf.talker_prefill(navi, ids, "english", spk, (tl.hidden, tl.vocab, tl.n_layer, tl.n_kv_head * tl.head_dim))
        np.savez_compressed(os.path.join(HERE, "ref_talker_small.npz"), ids=np.array(ids, np.int32), language="english", speaker=spk,
                            prefill=pre, trailing=trail, tts_pad=pad, hidden=hid, logits=lg, k=np.stack([k for k, _ in kv]),
                            v=np.stack([v for _, v in kv]))
        print("wrote ref_talker_small.npz;", pre.shape[0], "prefill rows")


if __name__ == "__main__":
    main()
