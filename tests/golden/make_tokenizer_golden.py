"""Writes the tokenizer fixtures under tests/golden/:

* tokenizer_synth.json -- a small byte-level BPE tokenizer in the layout of a
  Qwen3 tokenizer.json (NFC normaliser; Split by the Qwen2 pattern, then
  ByteLevel without its own regex; Qwen3's 26 added tokens after the
  vocabulary, 2048 ids in all), trained with Hugging Face ``tokenizers`` on seeded synthetic
  text.  It travels with the repository, so tokenizer tests and the GPU
  generate-text test need no checkpoint.
* tokenizer_cases.json -- seeded inputs (hex bytes, ill-formed UTF-8 among
  them) and the ids the oracle (oracle/tokenizer.py, the restatement of the
  reference's tokenizer) gives on the synthetic tokenizer and, when the
  reference's own tokenizer.json resource is present, on that file ("qwen3",
  with the reference's three known-answer cases first).

    python tests/golden/make_tokenizer_golden.py [--reference-dir DIR]
"""
from __future__ import annotations

import argparse
import json
import os
import random
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, HERE)

from oracle.build_ref import reference_dir  # noqa: E402
from oracle.tokenizer import OracleTokenizer  # noqa: E402
from tokenizer_inputs import QWEN2_PATTERN, QWEN3_ADDED_TOKENS, random_bytes, random_text  # noqa: E402

SYNTH = os.path.join(HERE, "tokenizer_synth.json")
CASES = os.path.join(HERE, "tokenizer_cases.json")
REFERENCE_KATS = [  # testing/tests/tokenizer.cpp:13-26
    ("Hello world", [9707, 1879]),
    ("曹尼玛💀", [102263, 99685, 101382, 146571]),
    ("<|endoftext|><tool_response></tool_response>", [151643, 151665, 151666]),
]


def train_synthetic(vocab_size: int = 2022) -> None:
    from tokenizers import Regex, Tokenizer, decoders, models, normalizers, pre_tokenizers, trainers

    tok = Tokenizer(models.BPE())
    tok.normalizer = normalizers.NFC()
    tok.pre_tokenizer = pre_tokenizers.Sequence([
        pre_tokenizers.Split(Regex(QWEN2_PATTERN), behavior="isolated", invert=False),
        pre_tokenizers.ByteLevel(add_prefix_space=False, trim_offsets=False, use_regex=False),
    ])
    tok.decoder = decoders.ByteLevel(add_prefix_space=False, trim_offsets=False, use_regex=False)
    trainer = trainers.BpeTrainer(vocab_size=vocab_size, initial_alphabet=pre_tokenizers.ByteLevel.alphabet(),
                                  show_progress=False)
    rng = random.Random(2024)
    corpus = [random_text(rng, 200, specials=False) for _ in range(4000)]
    tok.train_from_iterator(corpus, trainer)
    tok.add_tokens([t for t in QWEN3_ADDED_TOKENS])
    tok.save(SYNTH)
    # the layout the loaders read: model.vocab / merges, pre_tokenizer.pretokenizers[0].pattern.Regex
    with open(SYNTH, encoding="utf-8") as f:
        j = json.load(f)
    assert j["pre_tokenizer"]["pretokenizers"][0]["pattern"]["Regex"] == QWEN2_PATTERN
    with open(SYNTH, "w", encoding="utf-8") as f:
        json.dump(j, f, ensure_ascii=False, separators=(",", ":"))


def cases_for(path: str, n: int, seed: int, kats=()) -> list:
    o = OracleTokenizer(path)
    rng = random.Random(seed)
    out = [[s.encode().hex(), ids] for s, ids in kats]
    for s, ids in kats:
        assert o.tokenize(s) == ids, (s, o.tokenize(s), ids)
    for k in range(n):
        b = random_bytes(rng, 24) if k % 5 == 4 else random_text(rng, 40).encode()
        out.append([b.hex(), o.tokenize(b)])
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-dir", default=reference_dir())
    ap.add_argument("--retrain", action="store_true", help="retrain tokenizer_synth.json")
    a = ap.parse_args(argv)
    if a.retrain or not os.path.exists(SYNTH):
        train_synthetic()
    doc = {"synthetic": cases_for(SYNTH, 300, 11)}
    real = os.path.join(a.reference_dir, "testing", "tests", "resources", "tokenizer.json")
    if os.path.exists(real):
        doc["qwen3"] = cases_for(real, 300, 12, REFERENCE_KATS)
    with open(CASES, "w") as f:
        json.dump(doc, f, separators=(",", ":"))
    print({k: len(v) for k, v in doc.items()}, os.path.getsize(SYNTH), os.path.getsize(CASES))
    return 0


if __name__ == "__main__":
    sys.exit(main())
