"""Oracle for the Qwen3 batch-1 decode path.  TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline and
reference legs may import this package.  The product (``inference_b200``)
never does.

* :class:`Oracle` wraps ``libq3_oracle.so``, the C restatement in q3_oracle.c.
* :class:`RefLib` wraps ``_ref/libref_cpu.so`` / ``_ref/libref_cuda.so``: the
  reference's own backends and model, compiled from its sources by
  ``build_ref.py``.
"""
from .oracle import Oracle, RefLib, ModelConfig, CONFIGS, bf16_to_f32, f32_to_bf16  # noqa: F401
