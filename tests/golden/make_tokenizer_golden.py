"""Writes tests/golden/ref_tokenizer_small.json: a small byte-level BPE vocabulary (trained with
the tokenizers library on a synthetic multilingual corpus plus the case strings; NFC, the Qwen2
pre-tokenizer pattern, ByteLevel, the chat special tokens added) and, for every case string,
the ids and decoded bytes of the reference engine's own tokenizer (oracle/_ref/ref_tokenizer_check,
built from the reference sources by `make -C oracle REF=...`) and the ids of HF tokenizers.

The case strings are the reference's tests/reference/tokenizer_cases.json keys (its tokenizer
gate, whose ids need the released vocabulary) plus the strings of tests/test_tokenizer.py.

    python tests/golden/make_tokenizer_golden.py <reference tree>
"""
import json
import os
import subprocess
import sys
import tempfile

from tokenizers import Regex, Tokenizer as HFTokenizer, models, normalizers, pre_tokenizers, trainers

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [os.path.join(ROOT, "navi-tts_b200"), os.path.dirname(HERE)]

from navi_b200.tokenizer import PRETOKENIZE  # noqa: E402
from test_tokenizer import CASES, CORPUS, SPECIAL  # noqa: E402


def train(corpus):
    hf = HFTokenizer(models.BPE())
    hf.normalizer = normalizers.NFC()
    hf.pre_tokenizer = pre_tokenizers.Sequence([pre_tokenizers.Split(Regex(PRETOKENIZE.pattern), behavior="isolated"),
                                                pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=False)])
    trainer = trainers.BpeTrainer(vocab_size=1200, initial_alphabet=pre_tokenizers.ByteLevel.alphabet(), show_progress=False)
    hf.train_from_iterator(corpus, trainer)
    hf.add_special_tokens(SPECIAL)
    return hf


def main(ref):
    with open(os.path.join(ref, "tests", "reference", "tokenizer_cases.json"), encoding="utf-8") as f:
        ref_cases = list(json.load(f))
    cases = ref_cases + [c for c in CASES if c not in ref_cases]
    hf = train(CORPUS + cases)
    with tempfile.TemporaryDirectory() as td:
        hf.model.save(td)
        added = {str(i): {"content": t.content, "lstrip": False, "rstrip": False, "single_word": False,
                          "normalized": False, "special": True} for i, t in hf.get_added_tokens_decoder().items()}
        files = {"vocab_json": open(os.path.join(td, "vocab.json"), encoding="utf-8").read(),
                 "merges_txt": open(os.path.join(td, "merges.txt"), encoding="utf-8").read(),
                 "config_json": json.dumps({"added_tokens_decoder": added})}
        paths = []
        for k in ("vocab_json", "merges_txt", "config_json"):
            paths.append(os.path.join(td, k))
            with open(paths[-1], "w", encoding="utf-8") as f:
                f.write(files[k])
        paths.append(os.path.join(td, "cases.json"))
        with open(paths[-1], "w", encoding="utf-8") as f:
            json.dump(cases, f)
        out = subprocess.run([os.path.join(ROOT, "oracle", "_ref", "ref_tokenizer_check"), *paths], check=True,
                             capture_output=True, text=True).stdout.splitlines()
    assert len(out) == len(cases)
    rows = []
    for text, line in zip(cases, out):
        ids, hexs = line.split("\t")
        rows.append({"text": text, "ref_ids": [int(x) for x in ids.split()], "ref_decoded_hex": hexs,
                     "hf_ids": hf.encode(text).ids})
    doc = {"about": "reference tokenizer (model/qwen3tts/tokenizer.cpp) outputs on a synthetic vocabulary",
           **files, "cases": rows}
    with open(os.path.join(HERE, "ref_tokenizer_small.json"), "w", encoding="utf-8") as f:
        json.dump(doc, f, ensure_ascii=False, indent=0)
    same = sum(r["ref_ids"] == r["hf_ids"] for r in rows)
    print(f"{len(rows)} cases, reference == HF tokenizers on {same}")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("NAVI_REFERENCE", ""))
