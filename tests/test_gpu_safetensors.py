"""Checkpoint loading on the GPU: a sharded Hugging Face checkpoint holding
the engine's synthetic weights loads into an engine that then produces
bit-identical logits to one initialised in place; incomplete checkpoints
are rejected."""
import json

import numpy as np
import pytest

from st_util import hf_tensors, write_sharded

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("weights", ["bf16", "fp8"])
@pytest.mark.parametrize("tied", [True, False])
def test_loaded_checkpoint_matches_synthetic_weights(tmp_path, oracle, tied, weights):
    """FP8 engines quantize what they load exactly as what they generate."""
    from inference_b200 import Engine, Qwen3Config, prompt_ids

    H, I, L, QH, KVH, V = 1024, 3072, 2, 16, 8, 8192
    qc = Qwen3Config("qwen3-tiny", hidden=H, inter=I, layers=L, q_heads=QH, kv_heads=KVH, vocab=V, tied=tied)
    write_sharded(tmp_path, hf_tensors(oracle, H, I, L, QH, KVH, V, tied), 3)
    ids = prompt_ids(6, vocab=V)
    logits = []
    for load in (False, True):
        with Engine(qc, capacity=64, weights=weights) as e:
            if load:
                n = e.load_safetensors(tmp_path)
                assert n == 2 + (0 if tied else 1) + 11 * L
            else:
                e.init_synthetic(0)
            e.set_tokens(ids)
            out = []
            for _ in ids:
                e.step(1)
                e.sync()
                out.append(e.logits())
            logits.append(np.stack(out))
    np.testing.assert_array_equal(logits[0], logits[1])


def test_incomplete_checkpoint_is_rejected(tmp_path, oracle):
    from inference_b200 import Engine, Q3Error, Qwen3Config

    H, I, L, QH, KVH, V = 1024, 3072, 2, 16, 8, 8192
    qc = Qwen3Config("qwen3-tiny", hidden=H, inter=I, layers=L, q_heads=QH, kv_heads=KVH, vocab=V, tied=True)
    ts = hf_tensors(oracle, H, I, L, QH, KVH, V, True)
    del ts["model.layers.1.mlp.down_proj.weight"]
    write_sharded(tmp_path, ts, 2)
    with Engine(qc, capacity=64) as e:
        with pytest.raises(Q3Error) as ex:
            e.load_safetensors(tmp_path)
        assert "model.layers.1.mlp.down_proj.weight" in str(ex.value)
    idx = json.loads((tmp_path / "model.safetensors.index.json").read_text())
    assert "model.layers.1.mlp.down_proj.weight" not in idx["weight_map"]
