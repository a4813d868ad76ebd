"""Text generation on the GPU -- Generator::generate on text
(src/lib/inference/generator.cpp:37-63) through q3_engine_generate_text --
against the same steps taken one at a time: the oracle tokenizer's ids of the
chat-templated prompt (oracle/tokenizer.py), the engine's greedy ids
(q3_engine_generate with EOS stopping), and the oracle's decode of them.
A 2-layer Qwen3 with random weights over the committed synthetic tokenizer
(2048 ids, as many as the model's vocabulary)."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
SYNTH = os.path.join(os.path.dirname(__file__), "golden", "tokenizer_synth.json")
PROMPTS = ["Hello world", "曹尼玛💀 and naïve café", "<think>x</think> 12 + 30 = ?", ""]


def _engine(eos, capacity=160):
    from inference_b200 import Engine, Qwen3Config

    cfg = Qwen3Config("qwen3-tok", hidden=1024, inter=3072, layers=2, q_heads=16, kv_heads=8, vocab=2048, tied=True,
                      eos=eos)
    e = Engine(cfg, capacity=capacity)
    e.init_synthetic(0)
    return e


def test_generate_text_matches_steps():
    from inference_b200 import Tokenizer
    from oracle.tokenizer import OracleTokenizer, chat_template

    o = OracleTokenizer(SYNTH)
    im_end = o.special["<|im_end|>"]
    with Tokenizer(SYNTH) as t, _engine(im_end) as e:
        for p in PROMPTS:
            ids = o.tokenize(chat_template(p))
            assert list(t.tokenize(chat_template(p))) == ids
            gen = e.generate(np.array(ids, np.uint32), max_new=e.capacity, stop_at_eos=True)
            assert e.generate_text(t, p) == o.decode_bytes(gen)


def test_generate_text_stops_before_eos():
    """EOS ends the response and is not part of it (generator.cpp:52-54): the
    EOS id is set to a token the model is known to produce."""
    from inference_b200 import Tokenizer
    from oracle.tokenizer import OracleTokenizer, chat_template

    o = OracleTokenizer(SYNTH)
    ids = np.array(o.tokenize(chat_template(PROMPTS[0])), np.uint32)
    with _engine(eos=5000) as e:  # an id outside the vocabulary: never produced
        free = e.generate(ids, max_new=e.capacity, stop_at_eos=True)
    assert len(free) == 160 - len(ids)  # ran to the full cache
    stop = int(free[6])
    first = int(np.argmax(free == stop))
    with Tokenizer(SYNTH) as t, _engine(eos=stop) as e:
        assert e.generate_text(t, PROMPTS[0]) == o.decode_bytes(free[:first])


def test_generate_text_prompt_too_long():
    """A templated prompt of >= capacity tokens is refused (the reference's
    std::length_error, generator.cpp:42-44)."""
    from inference_b200 import Q3Error, Tokenizer

    with Tokenizer(SYNTH) as t, _engine(eos=5000, capacity=32) as e:
        with pytest.raises(Q3Error, match="does not fit"):
            e.generate_text(t, "word " * 40)
