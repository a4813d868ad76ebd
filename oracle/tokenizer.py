"""Oracle for the tokenizer: a plain-Python restatement of the reference's
tokenizer::Tokenizer (src/lib/tokenizer/tokenizer.cpp).  TEST INFRASTRUCTURE
ONLY -- tests import it as the checker of inference_b200's C++ tokenizer.

Step by step, as the reference does it:

* added tokens split the text first, by an alternation of their strings
  (make_special_token_regex / split_special_tokens, tokenizer.cpp:64-87,
  used by tokenize :217-235); a piece equal to an added token maps to its id;
* other pieces: NFC (normalize_nfc, :103-118, ICU), then the pre-tokenizer
  pattern of the file (:53-62, :120-124; Boost.Regex over ICU), byte-level
  symbols per byte (:126-134, alphabet :182-193), BPE by rescanning for the
  lowest-ranked adjacent pair and merging its first occurrence (:136-169),
  vocabulary lookup (:89-101);
* decode (:237-265): added tokens verbatim, other tokens' characters back to
  bytes.

The pattern engine here is the ``regex`` module with the reference engine's
meaning of ``\\s`` written out: Boost's ICU traits match ``\\s`` with
``u_isspace`` -- general category Z plus TAB..CR, U+001C..U+001F and U+0085 --
where ``regex`` (and Hugging Face ``tokenizers``) use the White_Space
property, which lacks U+001C..U+001F.  Ill-formed UTF-8 becomes U+FFFD per
maximal subpart, as ICU's conversion does (Python's "replace" handler follows
the same rule).

Parity pin: the reference's known-answer tests (testing/tests/tokenizer.cpp:
"Hello world", a CJK + emoji string, and three added tokens, with their ids)
on the reference's own tokenizer.json resource; and agreement with Hugging
Face ``tokenizers`` on the same file for text without U+001C..U+001F.
"""
from __future__ import annotations

import json
import os
import unicodedata

import regex

# u_isspace as set members (for use inside a character class)
_ICU_SPACE = r"\t-\r\x1c-\x20\x85\p{Z}"


def icu_pattern(pattern: str) -> str:
    """The file's pattern with \\s / \\S given the reference engine's meaning."""
    out, i, in_class = [], 0, False
    while i < len(pattern):
        c = pattern[i]
        if c == "\\" and i + 1 < len(pattern):
            nxt = pattern[i + 1]
            if nxt == "s":
                out.append(_ICU_SPACE if in_class else f"[{_ICU_SPACE}]")
            elif nxt == "S":
                if in_class:
                    raise ValueError("\\S inside a character class is not handled")
                out.append(f"[^{_ICU_SPACE}]")
            else:
                out.append(pattern[i:i + 2])
            i += 2
            continue
        if c == "[" and not in_class:
            in_class = True
        elif c == "]" and in_class:
            in_class = False
        out.append(c)
        i += 1
    return "".join(out)


def byte_to_symbol() -> list[str]:
    """byte_to_codepoint_table (tokenizer.cpp:182-193)."""
    table, nxt = [], 0x100
    for b in range(256):
        keep = 0x21 <= b <= 0x7E or 0xA1 <= b <= 0xAC or 0xAE <= b <= 0xFF
        table.append(chr(b) if keep else chr(nxt))
        if not keep:
            nxt += 1
    return table


class OracleTokenizer:
    def __init__(self, path: str):
        if os.path.isdir(path):
            path = os.path.join(path, "tokenizer.json")
        with open(path, encoding="utf-8") as f:
            j = json.load(f)
        self.vocab = dict(j["model"]["vocab"])
        self.id_to_word = {v: k for k, v in self.vocab.items()}
        self.merges = {}
        for rank, m in enumerate(j["model"]["merges"]):
            left, right = (m if isinstance(m, list) else m.split(" ", 1))
            self.merges.setdefault((left, right), rank)
        self.special = {a["content"]: a["id"] for a in j["added_tokens"]}
        self.special_by_id = {v: k for k, v in self.special.items()}
        self.pattern_text = j["pre_tokenizer"]["pretokenizers"][0]["pattern"]["Regex"]
        self.pattern = regex.compile(icu_pattern(self.pattern_text))
        self.special_re = regex.compile("|".join(regex.escape(s) for s in self.special))
        self.b2s = byte_to_symbol()
        self.s2b = {s: b for b, s in enumerate(self.b2s)}

    # ---- tokenize
    def merge_bpe(self, symbols: list[str]) -> list[str]:
        while len(symbols) > 1:
            best = None
            for i in range(len(symbols) - 1):
                r = self.merges.get((symbols[i], symbols[i + 1]))
                if r is not None and (best is None or r < best[0]):
                    best = (r, i)
            if best is None:
                break
            i = best[1]
            symbols = symbols[:i] + [symbols[i] + symbols[i + 1]] + symbols[i + 2:]
        return symbols

    def tokenize_text(self, text: str) -> list[int]:
        ids = []
        for m in self.pattern.finditer(unicodedata.normalize("NFC", text)):
            symbols = [self.b2s[b] for b in m.group(0).encode("utf-8")]
            ids.extend(self.vocab[s] for s in self.merge_bpe(symbols))
        return ids

    def tokenize(self, text: str | bytes) -> list[int]:
        if isinstance(text, bytes):
            text = text.decode("utf-8", errors="replace")
        ids, pos = [], 0
        for m in self.special_re.finditer(text) if self.special else ():
            if m.start() > pos:
                ids.extend(self.tokenize_text(text[pos:m.start()]))
            ids.append(self.special[m.group(0)])
            pos = m.end()
        if pos < len(text):
            ids.extend(self.tokenize_text(text[pos:]))
        return ids

    # ---- decode
    def decode_bytes(self, ids) -> bytes:
        out = bytearray()
        for t in ids:
            t = int(t)
            if t in self.special_by_id:
                out += self.special_by_id[t].encode("utf-8")
                continue
            for ch in self.id_to_word[t]:
                out.append(self.s2b[ch])
        return bytes(out)


def chat_template(prompt: str) -> str:
    """Model::apply_chat_template (src/lib/model/qwen3/qwen3.hpp:97-103)."""
    return f"<|im_start|>user\n{prompt}<|im_end|>\n<|im_start|>assistant\n<think>\n\n</think>"
