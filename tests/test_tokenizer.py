"""The text tokenizer (navi_b200.tokenizer: the reference's model/qwen3tts/tokenizer.cpp and
runtime/text/bpe.cpp) against HF tokenizers' own implementation of the same pipeline, on the
CPU: a byte-level BPE trained with the tokenizers library on a synthetic multilingual corpus,
with NFC, the Qwen2 pre-tokenizer pattern (Split, isolated) + ByteLevel without its own regex,
and the chat special tokens as added tokens -- the components of Qwen2TokenizerFast. The ids
must be equal on every test string (scripts, digits, punctuation runs, white space and
newlines, combining marks that NFC composes, emoji, special tokens inside the text), and
decoding must give the NFC text back. The reference's own tokenizer gate (tests/reference/
tokenizer_cases.json) needs the released vocabulary; its strings are pinned instead on a
committed synthetic vocabulary against the reference tokenizer's own outputs
(tests/golden/ref_tokenizer_small.json).
"""
import json
import unicodedata

import pytest
from tokenizers import Regex, Tokenizer as HFTokenizer, models, normalizers, pre_tokenizers, trainers

from navi_b200.tokenizer import PRETOKENIZE, Tokenizer

SPECIAL = ["<|im_start|>", "<|im_end|>", "<|tts_pad|>", "<|tts_text_bos|>", "<|tts_text_eod|>"]

CORPUS = [
    "The quick brown fox jumps over the lazy dog, and the bench text stays fixed.",
    "Hello there! It's 2026-12-02, 10:45am; numbers like 3.14159 and 1,000,000 stay digit by digit.",
    "Grüße aus München: Straße, Mädchen, Öl. Ça va? Où est l'été? Ñandú, año, niño.",
    "Привет, как дела? Это тест токенизатора. Ελληνικά γράμματα και αριθμοί 123.",
    "中文分词测试：今天天气很好，我们去公园散步吧。日本語のテキストも少し、カタカナとひらがな。",
    "한국어 문장도 있습니다. العربية نص قصير. עברית טקסט קצר. हिन्दी वाक्य भी।",
    "Tabs\tand  double  spaces\n\nnew lines\r\nwindows lines, trailing   \n   leading spaces",
    "Emoji 😀🎉👍🏽 and symbols © ® ™ § ¶ — – … « » “quotes” ‘single’ <tags> {braces} [x] /path/to/file",
    "camelCase PascalCase snake_case SCREAMING_CASE mixedUPPERlower ABCdef DEFghi",
    "é ä ô combining marks compose under NFC; ﬁ ligature stays; Å and Å",
] * 3


@pytest.fixture(scope="module")
def pair(tmp_path_factory):
    d = tmp_path_factory.mktemp("tok")
    hf = HFTokenizer(models.BPE())
    hf.normalizer = normalizers.NFC()
    hf.pre_tokenizer = pre_tokenizers.Sequence([pre_tokenizers.Split(Regex(PRETOKENIZE.pattern), behavior="isolated"),
                                                pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=False)])
    trainer = trainers.BpeTrainer(vocab_size=900, initial_alphabet=pre_tokenizers.ByteLevel.alphabet(), show_progress=False)
    hf.train_from_iterator(CORPUS, trainer)
    hf.add_special_tokens(SPECIAL)
    hf.model.save(str(d))
    added = {str(i): {"content": t.content, "lstrip": False, "rstrip": False, "single_word": False, "normalized": False,
                      "special": True} for i, t in hf.get_added_tokens_decoder().items()}
    (d / "tokenizer_config.json").write_text(json.dumps({"added_tokens_decoder": added}))
    return hf, Tokenizer.from_dir(d), d


CASES = [
    "Hello world", "  leading and trailing  ", "a\n\nb\r\n\r\nc", "x  \n  y", "trailing space ", "   ",
    "1234567890", "v1.2.3-rc4", "$12.50/kg", "e-mail: someone@example.com", "C++ / C# / F#",
    "Grüße, Straße", "Café au lait", "Ça va?", "ǅemal", "Привет мир", "中文分词测试", "日本語テキスト",
    "한국어", "مرحبا", "😀👍🏽🎉", "©®™", "...!!!???", "''\"\"", "it's they're we've I'm you'll he'd",
    "<|im_start|>assistant\nHello there.<|im_end|>\n<|im_start|>assistant\n",
    "before<|tts_pad|>after<|tts_pad|><|tts_pad|>", "<|im_end|>", "a\tb\tc", "CamelCaseWord ABCdef", "mixedUPPERlower",
    "new\nline/slash\n/", "tab\t\n", " nbsp em-space　ideographic", "Å vs Å", "ﬁre",
]


@pytest.mark.parametrize("text", CASES + CORPUS[:10])
def test_ids_match_hf_tokenizers(pair, text):
    hf, ours, _ = pair
    assert ours.encode(text) == hf.encode(text).ids, text


def test_decode_round_trip(pair):
    _, ours, _ = pair
    for text in CASES:
        assert ours.decode(ours.encode(text)) == unicodedata.normalize("NFC", text)


def test_prompt_template_and_navi(pair, tmp_path):
    hf, ours, d = pair
    ids = ours.prompt_ids("Hello there.")
    assert ids[0] == ours.added["<|im_start|>"] and ids.count(ours.added["<|im_end|>"]) == 1
    assert ids == hf.encode("<|im_start|>assistant\nHello there.<|im_end|>\n<|im_start|>assistant\n").ids
    # the same files as the tokenizer.* tensors of a .navi
    import numpy as np
    from navi_b200.navi_file import U8, NaviBuilder
    b = NaviBuilder()
    for f, t in (("vocab.json", "vocab.json"), ("merges.txt", "merges.txt"), ("tokenizer_config.json", "config.json")):
        b.put_tensor(f"tokenizer.{t}", U8, np.frombuffer((d / f).read_bytes(), dtype=np.uint8))
    b.save(tmp_path / "tok.navi")
    assert Tokenizer.from_navi(tmp_path / "tok.navi").encode("Grüße, Straße 42") == ours.encode("Grüße, Straße 42")


def _golden():
    import os
    with open(os.path.join(os.path.dirname(__file__), "golden", "ref_tokenizer_small.json"), encoding="utf-8") as f:
        return json.load(f)


def test_reference_tokenizer_pins():
    """The reference engine's own tokenizer (its tokenizer gate's strings and ours) on a committed
    synthetic vocabulary, from tests/golden/make_tokenizer_golden.py: ids and decoded bytes equal."""
    g = _golden()
    tok = Tokenizer(g["vocab_json"], g["merges_txt"], g["config_json"])
    assert len(g["cases"]) >= 80
    for c in g["cases"]:
        ids = tok.encode(c["text"])
        assert ids == c["ref_ids"] == c["hf_ids"], c["text"]
        assert tok.decode(ids).encode("utf-8").hex() == c["ref_decoded_hex"], c["text"]


def test_command_line(pair, tmp_path, capsys):
    import numpy as np
    from navi_b200 import tokenizer as tk
    from navi_b200.navi_file import U8, NaviBuilder
    _, ours, d = pair
    b = NaviBuilder()
    for f, t in (("vocab.json", "vocab.json"), ("merges.txt", "merges.txt"), ("tokenizer_config.json", "config.json")):
        b.put_tensor(f"tokenizer.{t}", U8, np.frombuffer((d / f).read_bytes(), dtype=np.uint8))
    b.save(tmp_path / "m.navi")
    assert tk.main(["--model", str(tmp_path / "m.navi"), "Hello there."]) == 0
    assert [int(x) for x in capsys.readouterr().out.split()] == ours.prompt_ids("Hello there.")
    assert tk.main(["--model", str(tmp_path / "m.navi"), "--raw", "Hello"]) == 0
    assert [int(x) for x in capsys.readouterr().out.split()] == ours.encode("Hello")
