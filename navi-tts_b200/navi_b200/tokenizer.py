"""The Qwen3 text tokenizer (the reference's model/qwen3tts/tokenizer.{h,cpp} and
runtime/text/bpe.{h,cpp}): added-token splitting, NFC, the Qwen2 fast pre-tokenizer pattern,
byte-level BPE, from the tokenizer files a `.navi` carries (tokenizer.vocab.json /
tokenizer.merges.txt / tokenizer.config.json) or from an HF model directory.

    tok = Tokenizer.from_navi("model.navi")
    ids = tok.prompt_ids("Hello there.")   # <|im_start|>assistant\\n{text}<|im_end|>\\n<|im_start|>assistant\\n

Steps, in the order HF's Qwen2TokenizerFast applies them:

1. added tokens (tokenizer_config.json's added_tokens_decoder) are cut out of the raw text,
   leftmost first and, at one position, longest first; they map to their ids directly;
2. every other segment is NFC-normalised;
3. the segment is split by the pre-tokenizer pattern (ordered alternatives, each backtracking
   as a PCRE engine does; text no alternative matches is a piece of its own):
       [^\\r\\n\\p{L}\\p{N}]?[A]*[B]+ | [^\\r\\n\\p{L}\\p{N}]?[A]+[B]* | \\p{N}
       |  ?[^\\s\\p{L}\\p{N}]+[\\r\\n/]* | \\s*[\\r\\n]+ | \\s+(?!\\S) | \\s+
   with A = [\\p{Lu}\\p{Lt}\\p{Lm}\\p{Lo}\\p{M}] and B = [\\p{Ll}\\p{Lm}\\p{Lo}\\p{M}];
4. each piece's UTF-8 bytes are written in the GPT-2 byte-to-unicode alphabet and merged by
   BPE: repeatedly the adjacent pair of lowest merge rank (leftmost on equal rank), until no
   pair has a rank; the resulting symbols are vocabulary entries.
"""
from __future__ import annotations

import json
import unicodedata
from functools import lru_cache
from pathlib import Path

import regex

_A = r"\p{Lu}\p{Lt}\p{Lm}\p{Lo}\p{M}"
_B = r"\p{Ll}\p{Lm}\p{Lo}\p{M}"
PRETOKENIZE = regex.compile(
    rf"[^\r\n\p{{L}}\p{{N}}]?[{_A}]*[{_B}]+|[^\r\n\p{{L}}\p{{N}}]?[{_A}]+[{_B}]*|\p{{N}}"
    r"| ?[^\s\p{L}\p{N}]+[\r\n/]*|\s*[\r\n]+|\s+(?!\S)|\s+")


def _byte_alphabet() -> tuple[dict[int, str], dict[str, int]]:
    """GPT-2's reversible byte <-> code point map: printable Latin-1 bytes stand for
    themselves, the other 68 bytes take code points 256, 257, ... in byte order."""
    keep = set(range(ord("!"), ord("~") + 1)) | set(range(0xA1, 0xAD)) | set(range(0xAE, 0x100))
    fwd, extra = {}, 0
    for b in range(256):
        if b in keep:
            fwd[b] = chr(b)
        else:
            fwd[b] = chr(256 + extra)
            extra += 1
    return fwd, {v: k for k, v in fwd.items()}


BYTE_TO_CHAR, CHAR_TO_BYTE = _byte_alphabet()


class Tokenizer:
    def __init__(self, vocab_json: str, merges_txt: str, config_json: str):
        self.vocab: dict[str, int] = json.loads(vocab_json)
        self.id_to_token = {i: t for t, i in self.vocab.items()}
        self.ranks: dict[tuple[str, str], int] = {}
        for line in merges_txt.splitlines():
            if not line or line.startswith("#version"):
                continue
            a, b = line.split(" ")
            self.ranks.setdefault((a, b), len(self.ranks))
        cfg = json.loads(config_json) if config_json.strip() else {}
        self.added: dict[str, int] = {}
        for sid, tok in (cfg.get("added_tokens_decoder") or {}).items():
            if any(tok.get(k) for k in ("lstrip", "rstrip", "single_word")):
                raise ValueError(f"added token {tok['content']!r}: lstrip / rstrip / single_word are not supported")
            self.added[tok["content"]] = int(sid)
        self.id_to_added = {i: t for t, i in self.added.items()}
        # longest first, so that at one position the longest added token wins
        self._added_by_len = sorted(self.added, key=len, reverse=True)
        self._bpe = lru_cache(maxsize=65536)(self._bpe_uncached)

    @staticmethod
    def from_navi(path) -> "Tokenizer":
        from .navi_file import NaviFile
        f = NaviFile.open(path)
        text = lambda n: bytes(f.array(n)).decode("utf-8")
        return Tokenizer(text("tokenizer.vocab.json"), text("tokenizer.merges.txt"), text("tokenizer.config.json"))

    @staticmethod
    def from_dir(model_dir) -> "Tokenizer":
        d = Path(model_dir)
        return Tokenizer((d / "vocab.json").read_text("utf-8"), (d / "merges.txt").read_text("utf-8"),
                         (d / "tokenizer_config.json").read_text("utf-8"))

    def __len__(self) -> int:
        return max(max(self.vocab.values(), default=-1), max(self.added.values(), default=-1)) + 1

    # --- encoding -------------------------------------------------------------------------

    def _split_added(self, text: str):
        """(segment, added id or None) in order: added tokens cut out, leftmost first."""
        out, i, start = [], 0, 0
        while i < len(text):
            hit = next((a for a in self._added_by_len if text.startswith(a, i)), None)
            if hit is None:
                i += 1
                continue
            if i > start:
                out.append((text[start:i], None))
            out.append((hit, self.added[hit]))
            i += len(hit)
            start = i
        if start < len(text):
            out.append((text[start:], None))
        return out

    def _bpe_uncached(self, piece: str) -> tuple[int, ...]:
        word = [BYTE_TO_CHAR[b] for b in piece.encode("utf-8")]
        while len(word) > 1:
            best, at = None, -1
            for j in range(len(word) - 1):
                r = self.ranks.get((word[j], word[j + 1]))
                if r is not None and (best is None or r < best):
                    best, at = r, j
            if best is None:
                break
            word[at:at + 2] = [word[at] + word[at + 1]]
        try:
            return tuple(self.vocab[w] for w in word)
        except KeyError as e:
            raise ValueError(f"symbol {e.args[0]!r} of {piece!r} is not in the vocabulary") from None

    @staticmethod
    def pretokenize(text: str) -> list[str]:
        """The pattern's matches in order; text between matches (if any) is a piece of its own."""
        pieces, i = [], 0
        for m in PRETOKENIZE.finditer(text):
            if m.start() > i:
                pieces.append(text[i:m.start()])
            pieces.append(m.group())
            i = m.end()
        if i < len(text):
            pieces.append(text[i:])
        return pieces

    def encode(self, text: str) -> list[int]:
        ids: list[int] = []
        for seg, aid in self._split_added(text):
            if aid is not None:
                ids.append(aid)
                continue
            for piece in self.pretokenize(unicodedata.normalize("NFC", seg)):
                ids.extend(self._bpe(piece))
        return ids

    def decode(self, ids) -> str:
        out, buf = [], bytearray()
        for i in ids:
            if i in self.id_to_added:
                out.append(buf.decode("utf-8", errors="replace"))
                buf = bytearray()
                out.append(self.id_to_added[i])
            else:
                buf.extend(CHAR_TO_BYTE[c] for c in self.id_to_token[i])
        out.append(buf.decode("utf-8", errors="replace"))
        return "".join(out)

    def prompt_ids(self, text: str) -> list[int]:
        """The talker's prompt template (talker.h:44-46): "<|im_start|>assistant\\n{text}<|im_end|>\\n
        <|im_start|>assistant\\n", tokenised -- the ids navi_talker_build_prompt and
        navi_graph_synth take."""
        return self.encode(f"<|im_start|>assistant\n{text}<|im_end|>\n<|im_start|>assistant\n")


def main(argv=None) -> int:
    """python -m navi_b200.tokenizer --model model.navi [--raw] TEXT: prints the prompt's ids
    (the `--ids-file` of `navi-b200 synth`), or with --raw the ids of TEXT alone."""
    import argparse
    import sys
    ap = argparse.ArgumentParser(description="Qwen3 text tokenizer of a .navi")
    ap.add_argument("--model", required=True)
    ap.add_argument("--raw", action="store_true", help="tokenise TEXT without the prompt template")
    ap.add_argument("text")
    a = ap.parse_args(argv)
    tok = Tokenizer.from_navi(a.model)
    ids = tok.encode(a.text) if a.raw else tok.prompt_ids(a.text)
    sys.stdout.write(" ".join(map(str, ids)) + "\n")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
