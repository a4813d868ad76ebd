"""Writes safetensors files for the tests (the format: 8-byte little-endian
header length, JSON header, data; offsets relative to the data)."""
import json
import struct

import numpy as np

DTYPES = {np.dtype(np.uint16): "BF16", np.dtype(np.float32): "F32", np.dtype(np.int64): "I64"}


def write_safetensors(path, tensors, metadata=None, header_patch=None):
    """tensors: name -> numpy array (uint16 arrays are BF16 bits)."""
    header, blobs, off = {}, [], 0
    for name, arr in tensors.items():
        arr = np.ascontiguousarray(arr)
        b = arr.tobytes()
        header[name] = {"dtype": DTYPES[arr.dtype], "shape": list(arr.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    if metadata is not None:
        header["__metadata__"] = metadata
    if header_patch:
        header_patch(header)
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def write_sharded(directory, tensors, n_shards):
    """model-0000k-of-0000n.safetensors + model.safetensors.index.json."""
    names = list(tensors)
    weight_map = {}
    for k in range(n_shards):
        fname = f"model-{k + 1:05d}-of-{n_shards:05d}.safetensors"
        part = {n: tensors[n] for n in names[k::n_shards]}
        write_safetensors(f"{directory}/{fname}", part, metadata={"format": "pt"})
        weight_map.update({n: fname for n in part})
    with open(f"{directory}/model.safetensors.index.json", "w") as f:
        json.dump({"metadata": {"total_size": sum(t.nbytes for t in tensors.values())}, "weight_map": weight_map}, f)


def hf_tensors(oracle, hidden, inter, layers, q_heads, kv_heads, vocab, tied, seed=0):
    """The engine's synthetic weights (q3_engine_init_synthetic tensor ids) under Hugging Face names."""
    one = lambda n: np.full(n, 0x3F80, np.uint16)  # BF16 1.0
    qf, kf = q_heads * 128, kv_heads * 128
    t = {"model.embed_tokens.weight": oracle.normal(seed, 1, vocab, hidden), "model.norm.weight": one(hidden)}
    if not tied:
        t["lm_head.weight"] = oracle.normal(seed, 2, vocab, hidden)
    for l in range(layers):
        b, p = 16 + 16 * l, f"model.layers.{l}."
        t[p + "self_attn.q_proj.weight"] = oracle.normal(seed, b + 0, qf, hidden)
        t[p + "self_attn.k_proj.weight"] = oracle.normal(seed, b + 1, kf, hidden)
        t[p + "self_attn.v_proj.weight"] = oracle.normal(seed, b + 2, kf, hidden)
        t[p + "self_attn.o_proj.weight"] = oracle.normal(seed, b + 3, hidden, qf)
        t[p + "mlp.gate_proj.weight"] = oracle.normal(seed, b + 4, inter, hidden)
        t[p + "mlp.up_proj.weight"] = oracle.normal(seed, b + 5, inter, hidden)
        t[p + "mlp.down_proj.weight"] = oracle.normal(seed, b + 6, hidden, inter)
        t[p + "input_layernorm.weight"] = one(hidden)
        t[p + "post_attention_layernorm.weight"] = one(hidden)
        t[p + "self_attn.q_norm.weight"] = one(128)
        t[p + "self_attn.k_norm.weight"] = one(128)
    return t
