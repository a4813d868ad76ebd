"""Hugging Face safetensors checkpoints (q3_safetensors_list, q3_engine_load_safetensors).

A checkpoint is a ``.safetensors`` file, a sharded checkpoint's
``model.safetensors.index.json``, or a directory holding either.  Loading goes
through :meth:`Engine.load_safetensors`; :func:`safetensors_list` reads the
headers only (no GPU).
"""
from __future__ import annotations

import ctypes as C
import os

from ._lib import check, lib


def safetensors_list(path) -> list[dict]:
    """Every tensor of the checkpoint: name, dtype, shape, file, absolute data offset, bytes."""
    need = C.c_size_t()
    p = os.fsencode(path)
    check(lib().q3_safetensors_list(p, None, 0, C.byref(need)))
    buf = C.create_string_buffer(need.value)
    check(lib().q3_safetensors_list(p, buf, need.value, C.byref(need)))
    out = []
    for line in buf.value.decode().splitlines():
        name, dtype, shape, file, offset, nbytes = line.split("\t")
        out.append({"name": name, "dtype": dtype, "shape": tuple(int(d) for d in shape.split("x") if d),
                    "file": file, "offset": int(offset), "bytes": int(nbytes)})
    return out
