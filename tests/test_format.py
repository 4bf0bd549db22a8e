"""The .circuit format: byte compatibility with the reference writer and
validation of malformed files (reference circuit_rag/storage/format.py)."""
import filecmp
import json
import os
import struct

import numpy as np
import pytest
import torch

from circuit_rag import CircuitIndex, build_circuit_index
from circuit_rag.storage.format import (DATA_START, CircuitFormatError, load_circuit_index, read_header,
                                        save_circuit_index)

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.mark.parametrize("name", ["ref_small.circuit", "ref_d384.circuit"])
@pytest.mark.parametrize("use_mmap", [True, False])
def test_reference_file_round_trips_byte_for_byte(tmp_path, name, use_mmap):
    src = os.path.join(GOLDEN, name)
    idx = load_circuit_index(src, device="cpu", use_mmap=use_mmap)
    out = tmp_path / name
    nbytes = idx.save(str(out))
    assert nbytes == os.path.getsize(out)
    assert filecmp.cmp(src, out, shallow=False)


def test_offsets_are_12_mod_64():
    meta = read_header(os.path.join(GOLDEN, "ref_small.circuit"))
    offs = [v["offset"] for v in meta["tensor_meta"].values()]
    assert offs[0] == DATA_START == 8204
    assert all(o % 64 == 12 for o in offs)


def test_builder_index_round_trip(tmp_path):
    rng = np.random.default_rng(0)
    X = rng.normal(size=(600, 16)).astype(np.float32)
    X /= np.linalg.norm(X, axis=1, keepdims=True)
    idx = build_circuit_index(X, num_roots=4, children_per_root=3, rank=5, device="cpu")
    p = tmp_path / "b.circuit"
    idx.save(str(p))
    back = CircuitIndex.load(str(p), device="cpu")
    for name in ("root_centers", "root_radii", "bases", "child_intervals_l", "child_intervals_u", "child_radii",
                 "child_parent_ids", "leaf_offsets", "leaf_sizes", "leaf_vectors", "original_ids"):
        assert torch.equal(getattr(idx, name), getattr(back, name)), name
    assert (back.dim, back.rank, back.num_roots, back.num_total_children, back.N) == (16, 5, 4, 12, 600)


def _corrupt(tmp_path, mutate):
    src = os.path.join(GOLDEN, "ref_small.circuit")
    data = bytearray(open(src, "rb").read())
    data = mutate(data)
    p = tmp_path / "bad.circuit"
    p.write_bytes(bytes(data))
    return str(p)


def _with_header(data, fn):
    hlen = struct.unpack("<I", data[8:12])[0]
    meta = json.loads(bytes(data[12:12 + hlen]).decode().rstrip("\x00"))
    fn(meta)
    h = json.dumps(meta).encode()
    data[12:12 + hlen] = h + b"\x00" * (hlen - len(h))
    return data


@pytest.mark.parametrize("mutate,msg", [
    (lambda d: b"NOTCIRC1" + d[8:], "not a valid"),
    (lambda d: d[:10], "truncated"),
    (lambda d: d[:12] + b"{not json" + d[21:], "JSON"),
    (lambda d: _with_header(d, lambda m: m.pop("rank")), "lacks rank"),
    (lambda d: _with_header(d, lambda m: m["tensor_meta"]["bases"].update(shape=[1, 2, 3])), "shape"),
    (lambda d: _with_header(d, lambda m: m["tensor_meta"]["leaf_sizes"].update(dtype="float32")), "dtype"),
    (lambda d: _with_header(d, lambda m: m["tensor_meta"]["original_ids"].update(offset=10 ** 9)), "outside"),
    (lambda d: d[:-5000], "outside"),
])
def test_malformed_files_are_rejected(tmp_path, mutate, msg):
    p = _corrupt(tmp_path, mutate)
    with pytest.raises(CircuitFormatError, match=msg):
        load_circuit_index(p, device="cpu")


def test_missing_file():
    with pytest.raises(FileNotFoundError):
        load_circuit_index("/nonexistent/x.circuit", device="cpu")
