"""Tokenizer and text generation: handles on the library's host C++ tokenizer
(csrc/tokenizer.cpp) -- the reference's tokenizer::Tokenizer
(src/lib/tokenizer/tokenizer.hpp:35-66) and Generator::generate on text
(src/lib/inference/generator.cpp:37-63)."""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import check, lib


class Tokenizer:
    """Byte-level BPE of a Qwen3 ``tokenizer.json`` (a file, or the model
    directory holding it, as ``Tokenizer(model_path)``, tokenizer.cpp:205-215)."""

    def __init__(self, path: str):
        h = C.c_void_p()
        check(lib().q3_tokenizer_load(str(path).encode(), C.byref(h)))
        self._h = h

    def close(self):
        if self._h:
            lib().q3_tokenizer_destroy(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._h

    def tokenize(self, text: str | bytes) -> np.ndarray:
        """Tokenizer::tokenize (tokenizer.cpp:217-235): uint32 ids."""
        b = text.encode() if isinstance(text, str) else bytes(text)
        n = C.c_size_t()
        check(lib().q3_tokenizer_encode(self._h, b, len(b), None, 0, C.byref(n)))
        out = np.zeros(n.value, np.uint32)
        check(lib().q3_tokenizer_encode(self._h, b, len(b), out.ctypes.data, out.size, C.byref(n)))
        return out

    def decode_bytes(self, ids) -> bytes:
        """Tokenizer::decode (tokenizer.cpp:237-265) as bytes: a token may end
        inside a multi-byte character."""
        a = np.ascontiguousarray(np.asarray(ids, np.uint32))
        need = C.c_size_t()
        check(lib().q3_tokenizer_decode(self._h, a.ctypes.data, a.size, None, 0, C.byref(need)))
        buf = C.create_string_buffer(need.value)
        check(lib().q3_tokenizer_decode(self._h, a.ctypes.data, a.size, buf, need.value, C.byref(need)))
        return buf.raw[: need.value - 1]

    def decode(self, ids) -> str:
        return self.decode_bytes(ids).decode(errors="replace")


def apply_chat_template(prompt: str | bytes) -> bytes:
    """Model::apply_chat_template (src/lib/model/qwen3/qwen3.hpp:97-103)."""
    b = prompt.encode() if isinstance(prompt, str) else bytes(prompt)
    need = C.c_size_t()
    check(lib().q3_chat_template(b, len(b), None, 0, C.byref(need)))
    buf = C.create_string_buffer(need.value)
    check(lib().q3_chat_template(b, len(b), buf, need.value, C.byref(need)))
    return buf.raw[: need.value - 1]


def generate_text(engine, tokenizer: Tokenizer, prompt: str | bytes) -> bytes:
    """Generator::generate (generator.cpp:37-63): the response to `prompt`
    (chat template applied), greedy until EOS or a full KV cache, as bytes."""
    b = prompt.encode() if isinstance(prompt, str) else bytes(prompt)
    out, n = C.c_void_p(), C.c_size_t()
    check(lib().q3_engine_generate_text(engine.h, tokenizer.handle, b, len(b), C.byref(out), C.byref(n)))
    try:
        return C.string_at(out, n.value)
    finally:
        lib().q3_string_free(out)
