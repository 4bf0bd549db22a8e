"""The ``.circuit`` single-file index format, read and written byte for byte as
the reference does (reference circuit_rag/storage/format.py:11-142):

    bytes 0..7      magic ``CIRCUIT1``
    bytes 8..11     uint32 little endian header length (always 8192)
    bytes 12..8203  JSON header (``json.dumps`` default separators), zero padded
    bytes 8204..    11 tensors in TENSOR_ORDER, each padded to a multiple of 64
                    bytes; ``offset`` in the header is absolute, ``nbytes``
                    unpadded.

Because data starts at byte 8204, every tensor offset is 12 (mod 64): tensor
data in the file is only 4-byte aligned.  The loader therefore never hands an
mmap view to device code directly; it copies to the device (aligned) or, on
the CPU, returns views that are only used by numpy / torch on the host.

Differences from the reference loader: the header and every tensor's dtype,
shape, offset and size are validated before any data is touched (the
reference trusts them), and ``device`` accepts any torch device string.
"""
import json
import mmap
import os
import struct
from typing import Any, Dict, Optional

import numpy as np
import torch

MAGIC_HEADER = b"CIRCUIT1"
HEADER_BLOCK = 8192
DATA_START = 8 + 4 + HEADER_BLOCK

# (name, dtype) in file order -- reference format.py:18-30
TENSOR_ORDER = (
    ("root_centers", "float32"),
    ("root_radii", "float32"),
    ("bases", "float32"),
    ("child_intervals_l", "float32"),
    ("child_intervals_u", "float32"),
    ("child_radii", "float32"),
    ("child_parent_ids", "int32"),
    ("leaf_offsets", "int32"),
    ("leaf_sizes", "int32"),
    ("leaf_vectors", "float32"),
    ("original_ids", "int32"),
)


class CircuitFormatError(ValueError):
    """The file is not a valid .circuit index."""


def _expected_shapes(meta: Dict[str, Any]) -> Dict[str, tuple]:
    d, r, R, C, N = (int(meta[k]) for k in ("dim", "rank", "num_roots", "num_total_children", "N"))
    return {
        "root_centers": (R, d),
        "root_radii": (R,),
        "bases": (R, d, r),
        "child_intervals_l": (C, r),
        "child_intervals_u": (C, r),
        "child_radii": (C,),
        "child_parent_ids": (C,),
        "leaf_offsets": (C,),
        "leaf_sizes": (C,),
        "leaf_vectors": (N, d),
        "original_ids": (N,),
    }


def _to_numpy(t: torch.Tensor, dtype: str) -> np.ndarray:
    a = t.detach().cpu().contiguous().numpy()
    want = np.dtype(dtype)
    if a.dtype != want:
        a = a.astype(want)
    return a


def save_circuit_index(index, filepath: str) -> int:
    """Write ``index`` to ``filepath``; returns the file size in bytes
    (reference format.py:13-80, identical bytes for identical tensors)."""
    arrays = [(name, _to_numpy(getattr(index, name), dt), dt) for name, dt in TENSOR_ORDER]
    meta: Dict[str, Any] = {
        "version": 1,
        "dim": int(index.dim),
        "rank": int(index.rank),
        "num_roots": int(index.num_roots),
        "num_total_children": int(index.num_total_children),
        "N": int(index.N),
        "tensor_meta": {},
    }
    offset = DATA_START
    for name, arr, dt in arrays:
        meta["tensor_meta"][name] = {"dtype": dt, "shape": list(arr.shape), "offset": offset, "nbytes": arr.nbytes}
        offset += (arr.nbytes + 63) & ~63
    header = json.dumps(meta).encode("utf-8")
    if len(header) > HEADER_BLOCK:
        raise CircuitFormatError("header too large to fit in 8 KB")
    os.makedirs(os.path.dirname(os.path.abspath(filepath)), exist_ok=True)
    with open(filepath, "wb") as f:
        f.write(MAGIC_HEADER)
        f.write(struct.pack("<I", HEADER_BLOCK))
        f.write(header)
        f.write(b"\x00" * (DATA_START - f.tell()))
        for _, arr, _ in arrays:
            f.write(arr.tobytes())
            pad = ((arr.nbytes + 63) & ~63) - arr.nbytes
            if pad:
                f.write(b"\x00" * pad)
    return offset


def read_header(filepath: str) -> Dict[str, Any]:
    """Parse and validate the header of a .circuit file (no tensor data read)."""
    if not os.path.exists(filepath):
        raise FileNotFoundError(f"File {filepath} does not exist.")
    size = os.path.getsize(filepath)
    with open(filepath, "rb") as f:
        magic = f.read(8)
        if magic != MAGIC_HEADER:
            raise CircuitFormatError(f"File {filepath} is not a valid CircuitIndex file.")
        raw = f.read(4)
        if len(raw) != 4:
            raise CircuitFormatError("truncated header length")
        header_len = struct.unpack("<I", raw)[0]
        if 12 + header_len > size:
            raise CircuitFormatError("header length exceeds file size")
        header = f.read(header_len)
    try:
        meta = json.loads(header.decode("utf-8").rstrip("\x00"))
    except (UnicodeDecodeError, json.JSONDecodeError) as e:
        raise CircuitFormatError(f"header is not valid JSON: {e}") from e
    for key in ("dim", "rank", "num_roots", "num_total_children", "N", "tensor_meta"):
        if key not in meta:
            raise CircuitFormatError(f"header lacks {key}")
    shapes = _expected_shapes(meta)
    for name, dt in TENSOR_ORDER:
        info = meta["tensor_meta"].get(name)
        if info is None:
            raise CircuitFormatError(f"tensor_meta lacks {name}")
        if info.get("dtype") != dt:
            raise CircuitFormatError(f"unexpected dtype for {name}: {info.get('dtype')}")
        if tuple(info.get("shape", ())) != shapes[name]:
            raise CircuitFormatError(f"shape mismatch for {name}: {info.get('shape')} != {list(shapes[name])}")
        nbytes = int(np.prod(shapes[name], dtype=np.int64)) * 4
        if int(info.get("nbytes", -1)) != nbytes:
            raise CircuitFormatError(f"nbytes mismatch for {name}")
        off = int(info.get("offset", -1))
        if off < 12 + header_len or off + nbytes > size:
            raise CircuitFormatError(f"tensor data outside the file for {name}")
    return meta


def check_child_tables(parent, offsets, sizes, num_roots: int, n: int) -> None:
    """The child-table checks the native loader makes before it uses the tables
    as indices (csrc/index.cpp, build_host_tables): no negative size; every
    non-empty child has a parent in [0, num_roots) and a row range inside
    [0, n); the ranges are disjoint and cover all n rows.  Empty children may
    carry any parent id and offset (the reference builder leaves them 0)."""
    parent = np.asarray(parent, dtype=np.int64)
    offsets = np.asarray(offsets, dtype=np.int64)
    sizes = np.asarray(sizes, dtype=np.int64)
    if (sizes < 0).any():
        raise CircuitFormatError("leaf_sizes has a negative entry")
    live = sizes > 0
    p, o, z = parent[live], offsets[live], sizes[live]
    if ((p < 0) | (p >= num_roots)).any():
        raise CircuitFormatError("child_parent_ids out of range for a non-empty child")
    if ((o < 0) | (o + z > n)).any():
        raise CircuitFormatError("leaf_offsets/leaf_sizes reach outside leaf_vectors")
    order = np.argsort(o, kind="stable")
    o, z = o[order], z[order]
    if len(o) > 1 and (o[:-1] + z[:-1] > o[1:]).any():
        raise CircuitFormatError("child leaf ranges overlap")
    if int(z.sum()) != int(n):
        raise CircuitFormatError(f"children do not cover all N leaf rows ({int(z.sum())} of {int(n)})")


def load_circuit_index(filepath: str, device: str = "cuda", use_mmap: bool = True):
    """Load a .circuit file (reference format.py:82-142).  With ``use_mmap`` the
    tensors are zero-copy views of a private (copy-on-write) mapping until they
    are moved to ``device``."""
    from circuit_rag.hierarchy.build import CircuitIndex

    meta = read_header(filepath)
    tensors = {}
    if use_mmap:
        with open(filepath, "rb") as f:
            mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_COPY)
        for name, dt in TENSOR_ORDER:
            info = meta["tensor_meta"][name]
            arr = np.ndarray(buffer=mm, dtype=np.dtype(dt), offset=int(info["offset"]), shape=tuple(info["shape"]))
            tensors[name] = torch.from_numpy(arr)
    else:
        with open(filepath, "rb") as f:
            for name, dt in TENSOR_ORDER:
                info = meta["tensor_meta"][name]
                f.seek(int(info["offset"]))
                data = f.read(int(info["nbytes"]))
                arr = np.frombuffer(data, dtype=np.dtype(dt)).reshape(tuple(info["shape"]))
                tensors[name] = torch.from_numpy(arr.copy())
    check_child_tables(tensors["child_parent_ids"].numpy(), tensors["leaf_offsets"].numpy(),
                       tensors["leaf_sizes"].numpy(), int(meta["num_roots"]), int(meta["N"]))
    return CircuitIndex(
        root_centers=tensors["root_centers"],
        root_radii=tensors["root_radii"],
        bases=tensors["bases"],
        child_intervals_l=tensors["child_intervals_l"],
        child_intervals_u=tensors["child_intervals_u"],
        child_radii=tensors["child_radii"],
        child_parent_ids=tensors["child_parent_ids"],
        leaf_offsets=tensors["leaf_offsets"],
        leaf_sizes=tensors["leaf_sizes"],
        leaf_vectors=tensors["leaf_vectors"],
        original_ids=tensors["original_ids"],
        dim=int(meta["dim"]),
        rank=int(meta["rank"]),
        device=device,
    )
