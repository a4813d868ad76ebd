"""Checkpoint headers (q3_safetensors_list): single files, sharded
checkpoints through their index, directories, and rejection of malformed
files -- host code, no GPU."""
import os
import struct

import numpy as np
import pytest

from st_util import write_safetensors, write_sharded


def _tensors():
    rng = np.random.default_rng(3)
    return {
        "model.embed_tokens.weight": rng.integers(0, 65535, (16, 8), dtype=np.uint16),
        "model.norm.weight": rng.integers(0, 65535, (8,), dtype=np.uint16),
        "extra.f32": rng.standard_normal((3, 5)).astype(np.float32),
    }


def test_single_file_listing_and_offsets(tmp_path):
    from inference_b200 import safetensors_list

    ts = _tensors()
    p = tmp_path / "model.safetensors"
    write_safetensors(p, ts, metadata={"format": "pt"})
    got = {t["name"]: t for t in safetensors_list(p)}
    assert set(got) == set(ts)
    raw = p.read_bytes()
    for name, arr in ts.items():
        t = got[name]
        assert t["shape"] == arr.shape and t["bytes"] == arr.nbytes
        assert t["dtype"] == ("F32" if arr.dtype == np.float32 else "BF16")
        assert raw[t["offset"]:t["offset"] + t["bytes"]] == arr.tobytes()
    # a directory holding model.safetensors lists the same
    assert {t["name"] for t in safetensors_list(tmp_path)} == set(ts)


def test_sharded_checkpoint_through_index_and_directory(tmp_path):
    from inference_b200 import safetensors_list

    ts = _tensors()
    write_sharded(tmp_path, ts, 2)
    by_index = safetensors_list(tmp_path / "model.safetensors.index.json")
    by_dir = safetensors_list(tmp_path)
    assert {t["name"] for t in by_index} == {t["name"] for t in by_dir} == set(ts)
    assert {os.path.basename(t["file"]) for t in by_index} == {"model-00001-of-00002.safetensors",
                                                               "model-00002-of-00002.safetensors"}
    for t in by_index:
        with open(t["file"], "rb") as f:
            f.seek(t["offset"])
            assert f.read(t["bytes"]) == ts[t["name"]].tobytes()


def _expect_error(path, fragment):
    from inference_b200 import Q3Error, safetensors_list

    with pytest.raises(Q3Error) as ex:
        safetensors_list(path)
    assert fragment in str(ex.value), str(ex.value)


def test_malformed_files_are_rejected(tmp_path):
    ts = _tensors()
    # header length beyond the file
    p = tmp_path / "big.safetensors"
    write_safetensors(p, ts)
    raw = bytearray(p.read_bytes())
    raw[:8] = struct.pack("<Q", len(raw) * 4)
    p.write_bytes(bytes(raw))
    _expect_error(p, "header length")
    # data offsets past the end of the data
    p = tmp_path / "range.safetensors"
    write_safetensors(p, ts, header_patch=lambda h: h["model.norm.weight"].update(data_offsets=[0, 10 ** 9]))
    _expect_error(p, "out of range")
    # shape inconsistent with the byte count
    p = tmp_path / "shape.safetensors"
    write_safetensors(p, ts, header_patch=lambda h: h["model.norm.weight"].update(shape=[9]))
    _expect_error(p, "inconsistent")
    # broken JSON
    p = tmp_path / "json.safetensors"
    write_safetensors(p, ts)
    raw = bytearray(p.read_bytes())
    raw[8] = ord("[")
    p.write_bytes(bytes(raw))
    _expect_error(p, "header JSON")
    # truncated file
    p = tmp_path / "short.safetensors"
    p.write_bytes(b"\x01\x02")
    _expect_error(p, "header length")
    # an index that names a tensor its shard does not hold
    d = tmp_path / "idx"
    d.mkdir()
    write_sharded(d, ts, 2)
    import json

    idx = json.loads((d / "model.safetensors.index.json").read_text())
    idx["weight_map"]["ghost.weight"] = "model-00001-of-00002.safetensors"
    (d / "model.safetensors.index.json").write_text(json.dumps(idx))
    _expect_error(d, "ghost.weight")
    # nothing to load
    _expect_error(tmp_path / "nowhere", "cannot open")


def test_hostile_header_numbers_are_rejected(tmp_path):
    """Shapes whose element count wraps 64 bits, data offsets that are not
    numbers, and fractional or >= 2^53 numbers are rejected, not converted."""
    ts = _tensors()
    # 2^33 x 2^31 BF16 elements: the element count wraps to 0 in uint64, matching empty offsets
    p = tmp_path / "wrap.safetensors"
    write_safetensors(p, ts, header_patch=lambda h: h["model.norm.weight"].update(shape=[2 ** 33, 2 ** 31],
                                                                               data_offsets=[0, 0]))
    _expect_error(p, "overflows")
    # data offsets given as strings
    p = tmp_path / "strings.safetensors"
    write_safetensors(p, ts, header_patch=lambda h: h["model.norm.weight"].update(data_offsets=["0", "16"]))
    _expect_error(p, "not non-negative integers")
    # a fractional offset and one at 2^53 (no exact uint64 conversion is defined for them)
    p = tmp_path / "frac.safetensors"
    write_safetensors(p, ts, header_patch=lambda h: h["model.norm.weight"].update(data_offsets=[0.5, 16.5]))
    _expect_error(p, "not non-negative integers")
    p = tmp_path / "huge.safetensors"
    write_safetensors(p, ts, header_patch=lambda h: h["model.norm.weight"].update(data_offsets=[2 ** 53, 2 ** 53 + 16]))
    _expect_error(p, "not non-negative integers")
    # a fractional or negative dimension
    p = tmp_path / "dimfrac.safetensors"
    write_safetensors(p, ts, header_patch=lambda h: h["model.norm.weight"].update(shape=[7.5]))
    _expect_error(p, "bad shape")
