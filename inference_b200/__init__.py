"""B200 (sm_100a) Qwen3 batch-1 decode: hand-written CUDA kernels behind a
C ABI (include/q3_sm100a.h, libq3_sm100a.so), with thin Python handles.

* :class:`Engine` -- Model + paged KV cache + greedy loop on one GPU / TP rank.
* :class:`B200Backend` -- the reference Backend operator interface, op by op.
* :func:`safetensors_list` / :meth:`Engine.load_safetensors` -- Hugging Face checkpoints.
* :class:`Batch` -- batched decode of several sequences on one engine.
* :class:`Tokenizer` / :func:`generate_text` -- tokenizer.json BPE and Generator::generate on text.
"""
from ._lib import Q3Error, lib  # noqa: F401
from .checkpoint import safetensors_list  # noqa: F401
from .backend import B200Backend, RopeCache, fill_normal, prompt_ids, rope_tables  # noqa: F401
from .config import MODELS, QWEN3_0P6B, QWEN3_4B, QWEN3_8B, QWEN3_32B, WORKLOADS, Qwen3Config  # noqa: F401
from .engine import Engine  # noqa: F401
from .batch import Batch  # noqa: F401
from .tokenizer import Tokenizer, apply_chat_template, generate_text  # noqa: F401
