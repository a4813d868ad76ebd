"""Seeded text for the tokenizer tests and fixtures: words, numbers, white
space of every kind the pre-tokenizer pattern tells apart, punctuation,
contractions (any case), CJK, emoji sequences, precomposed and decomposed
accents (NFC), Hangul jamo, and Qwen3's added tokens."""
from __future__ import annotations

import random
import unicodedata

# The pre-tokenizer pattern of Qwen2 / Qwen3 tokenizer.json files.
QWEN2_PATTERN = (r"(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}| ?[^\s\p{L}\p{N}]+[\r\n]*|"
                 r"\s*[\r\n]+|\s+(?!\S)|\s+")

# Qwen3's added tokens, ids 151643.. in this order.
QWEN3_ADDED_TOKENS = [
    "<|endoftext|>", "<|im_start|>", "<|im_end|>", "<|object_ref_start|>", "<|object_ref_end|>", "<|box_start|>",
    "<|box_end|>", "<|quad_start|>", "<|quad_end|>", "<|vision_start|>", "<|vision_end|>", "<|vision_pad|>",
    "<|image_pad|>", "<|video_pad|>", "<tool_call>", "</tool_call>", "<|fim_prefix|>", "<|fim_middle|>",
    "<|fim_suffix|>", "<|fim_pad|>", "<|repo_name|>", "<|file_sep|>", "<tool_response>", "</tool_response>",
    "<think>", "</think>",
]

_WORDS = ["the", "of", "and", "token", "decode", "page", "Hello", "World", "GPU", "cache", "naïve", "café",
          "Straße", "über", "Ωmega", "данные", "مرحبا", "שלום", "नमस्ते", "สวัสดี"]
_POOLS = [
    list("abcdefghijklmnopqrstuvwxyzABCDEFGHIJKLMNOPQRSTUVWXYZ"),
    list("0123456789"),
    list(" " * 8 + "\n\r\t"),
    list("!\"#$%&'()*+,-./:;<=>?@[\\]^_`{|}~"),
    ["'s", "'t", "'re", "'ve", "'m", "'ll", "'d", "'S", "'LL", "'Re", "'ſ"],
    [chr(c) for c in range(0x4E00, 0x4E80)],
    ["\U0001F600", "\U0001F480", "\U0001F44D\U0001F3FD", "\U0001F1FA\U0001F1F8", "\U0001F468‍\U0001F469"],
    ["é", "Å", "각", "Ạ̇", "क़", "ȫ"],
    ["\x1c", "\x1d", "\x1e", "\x1f", "\x85", "\xa0", "　", " ", " ", "​", "\xad"],
    ["¹", "²", "½", "Ⅻ", "٣", "०"],
    _WORDS,
]


def random_text(rng: random.Random, max_len: int, specials: bool = True) -> str:
    out = []
    for _ in range(rng.randint(0, max_len)):
        r = rng.random()
        if r < 0.04:
            cp = rng.randrange(0x20, 0x30000)
            if unicodedata.category(chr(cp)) not in ("Cn", "Cs", "Co"):
                out.append(chr(cp))
        elif r < 0.08 and specials:
            out.append(rng.choice(QWEN3_ADDED_TOKENS))
        elif r < 0.3:
            out.append(rng.choice(["", " "]) + rng.choice(_WORDS))
        else:
            out.append(rng.choice(rng.choice(_POOLS)))
    return "".join(out)


def random_bytes(rng: random.Random, max_len: int) -> bytes:
    """Bytes with ill-formed UTF-8 among them: truncated and overlong
    sequences, surrogates, stray continuation bytes, bytes C0, C1, F5..FF."""
    parts = [b"a", b" ", b"\n", "é".encode(), "€".encode(), "\U0001F600".encode(), b"\xc3", b"\xe2\x82",
             b"\xf0\x9f\x98", b"\xed\xa0\x80", b"\xc0\xaf", b"\xe0\x80\xaf", b"\xf4\x90\x80\x80", b"\x80", b"\xbf",
             b"\xf5", b"\xff"]
    return b"".join(rng.choice(parts) for _ in range(rng.randint(0, max_len)))
