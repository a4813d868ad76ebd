"""Tokenizer parity (CPU): the library's C++ tokenizer (csrc/tokenizer.cpp,
through the C ABI) against the oracle (oracle/tokenizer.py, the restatement of
the reference's tokenizer.cpp) and the committed fixtures.

* the reference's own known-answer tests (testing/tests/tokenizer.cpp:13-30:
  ids and decode round trip) on its tokenizer.json resource, when present;
* committed golden cases (tests/golden/tokenizer_cases.json, made by the
  oracle) on the committed synthetic tokenizer and on the Qwen3 file;
* seeded random text and bytes against the oracle, live;
* Hugging Face ``tokenizers`` on the same files, where its white-space class
  and Unicode data agree with the reference's engine;
* error behaviour of the loader, encode and decode.
"""
from __future__ import annotations

import json
import os
import random
import unicodedata

import numpy as np
import pytest

from tokenizer_inputs import random_bytes, random_text

GOLD = os.path.join(os.path.dirname(__file__), "golden")
SYNTH = os.path.join(GOLD, "tokenizer_synth.json")


def _qwen3_path():
    from oracle.build_ref import reference_dir

    p = os.path.join(reference_dir(), "testing", "tests", "resources", "tokenizer.json")
    return p if os.path.exists(p) else None


@pytest.fixture(scope="module")
def cases():
    with open(os.path.join(GOLD, "tokenizer_cases.json")) as f:
        return json.load(f)


@pytest.fixture(scope="module", params=["synthetic", "qwen3"])
def pair(request):
    """(name, library tokenizer, oracle tokenizer) for one tokenizer.json."""
    from inference_b200 import Tokenizer
    from oracle.tokenizer import OracleTokenizer

    path = SYNTH if request.param == "synthetic" else _qwen3_path()
    if path is None:
        pytest.skip("the reference's tokenizer.json resource is not present")
    t = Tokenizer(path)
    yield request.param, t, OracleTokenizer(path)
    t.close()


def test_reference_known_answers():
    """testing/tests/tokenizer.cpp: ids and exact decode, library and oracle."""
    from inference_b200 import Tokenizer
    from oracle.tokenizer import OracleTokenizer

    path = _qwen3_path()
    if path is None:
        pytest.skip("the reference's tokenizer.json resource is not present")
    kats = [("Hello world", [9707, 1879]), ("曹尼玛💀", [102263, 99685, 101382, 146571]),
            ("<|endoftext|><tool_response></tool_response>", [151643, 151665, 151666])]
    o = OracleTokenizer(path)
    with Tokenizer(os.path.dirname(path)) as t:  # a model directory, as Tokenizer(model_path)
        for text, ids in kats:
            assert list(t.tokenize(text)) == ids
            assert t.decode(ids) == text
            assert o.tokenize(text) == ids
            assert o.decode_bytes(ids).decode() == text


def test_golden_cases(pair, cases):
    name, t, o = pair
    for hexed, ids in cases[name]:
        b = bytes.fromhex(hexed)
        assert list(t.tokenize(b)) == ids, (b, list(t.tokenize(b)), ids)
        assert o.tokenize(b) == ids  # the oracle still gives what it gave when the fixture was made


def test_random_text_matches_oracle(pair):
    name, t, o = pair
    rng = random.Random(101)
    for _ in range(1500):
        s = random_text(rng, 60)
        ids = list(t.tokenize(s))
        assert ids == o.tokenize(s), repr(s)
        # decode gives back the NFC form of the text, byte for byte
        assert t.decode_bytes(ids) == unicodedata.normalize("NFC", s).encode(), repr(s)


def test_random_bytes_match_oracle(pair):
    """Ill-formed UTF-8: U+FFFD per maximal subpart, as the reference's ICU conversion."""
    name, t, o = pair
    rng = random.Random(102)
    for _ in range(1500):
        b = random_bytes(rng, 30)
        assert list(t.tokenize(b)) == o.tokenize(b), b
    ids = t.tokenize(b"a\xffb")
    assert t.decode_bytes(ids) == "a�b".encode()


def test_pre_tokenizer_edges(pair):
    """Cases each alternative of the pattern decides: contractions in any case
    (and long s), a space before letters / punctuation, runs of spaces before
    a word and at the end, CR/LF runs, digits one by one, and U+001C..U+001F,
    which the reference's engine counts as white space."""
    name, t, o = pair
    edge = ["don't", "DON'T", "we'LL", "it'ſ", "'s", "''s", " hello", "  hello", "hello  ", "a \n\n b", "\r\n\r\n",
            " \t\n x", "12345", "x1y2", "a\x1cb", "a \x1f b", "\x1c\x1d", "!!!\n\n", " !!", "　x", "a\u0085b",
            "é", "각", "", " ", "\n", "<|im_start|>user\nhi<|im_end|>", "<|im_end|><|im_end|>"]
    for s in edge:
        assert list(t.tokenize(s)) == o.tokenize(s), repr(s)


def test_long_pieces(pair):
    """BPE over long pre-tokenizer splits (a heap here, a rescan per merge in
    the oracle): same ids."""
    name, t, o = pair
    for s in ["a" * 700, " " * 700 + "x", "一" * 300, "ab" * 300, "9" * 200, "!" * 500]:
        assert list(t.tokenize(s)) == o.tokenize(s)


def test_hf_tokenizers_agree(pair):
    """Hugging Face tokenizers on the same file: the same ids on text without
    U+001C..U+001F (white space to the reference's engine, not to HF's) and
    without combining marks whose combining class differs across Unicode
    versions."""
    tokenizers = pytest.importorskip("tokenizers")
    name, t, o = pair
    hf = tokenizers.Tokenizer.from_file(SYNTH if name == "synthetic" else _qwen3_path())
    rng = random.Random(103)
    for _ in range(1500):
        s = "".join(c for c in random_text(rng, 60) if c not in "\x1c\x1d\x1e\x1f" and not unicodedata.combining(c))
        assert list(t.tokenize(s)) == hf.encode(s, add_special_tokens=False).ids, repr(s)


def test_chat_template():
    from inference_b200 import apply_chat_template
    from oracle.tokenizer import chat_template

    for p in ["", "hi", "曹尼玛💀", "a\nb<|im_end|>"]:
        assert apply_chat_template(p) == chat_template(p).encode()


def test_encode_decode_buffers_and_errors(tmp_path):
    import ctypes as C

    from inference_b200 import Q3Error, Tokenizer
    from inference_b200._lib import lib

    with pytest.raises(Q3Error):
        Tokenizer(str(tmp_path / "missing.json"))
    # a pre-tokenizer other than the Qwen2 pattern is refused
    with open(SYNTH, encoding="utf-8") as f:
        j = json.load(f)
    j["pre_tokenizer"]["pretokenizers"][0]["pattern"]["Regex"] = r"\w+|\s+"
    bad = tmp_path / "tokenizer.json"
    bad.write_text(json.dumps(j), encoding="utf-8")
    with pytest.raises(Q3Error, match="UNSUPPORTED"):
        Tokenizer(str(tmp_path))
    with Tokenizer(SYNTH) as t:
        with pytest.raises(Q3Error):
            t.decode([10 ** 6])  # not in the vocabulary
        # a too small ids buffer is refused, with the count reported
        n = C.c_size_t()
        out = np.zeros(1, np.uint32)
        text = "hello world, hello".encode()
        assert lib().q3_tokenizer_encode(t.handle, text, len(text), out.ctypes.data, 1, C.byref(n)) == 1
        assert n.value == len(t.tokenize(text))
        assert list(t.tokenize("")) == []
        assert t.decode([]) == ""


@pytest.mark.parametrize("where", ["vocab", "added"])
@pytest.mark.parametrize("bad_id", [-1, 1.5, 2 ** 24, 1e300, "7"])
def test_hostile_ids_are_rejected(tmp_path, where, bad_id):
    """Vocabulary and added-token ids must be integers in [0, 2^24): anything
    else is Q3_ERR_INVALID, never a huge allocation or an undefined cast."""
    from inference_b200 import Q3Error, Tokenizer

    with open(SYNTH, encoding="utf-8") as f:
        j = json.load(f)
    if where == "vocab":
        word = next(iter(j["model"]["vocab"]))
        j["model"]["vocab"][word] = bad_id
    else:
        j["added_tokens"].append({"id": bad_id, "content": "<|hostile|>", "special": True})
    (tmp_path / "tokenizer.json").write_text(json.dumps(j), encoding="utf-8")
    with pytest.raises(Q3Error, match="INVALID"):
        Tokenizer(str(tmp_path))
