"""Child process of tests/test_loader_fuzz.py: feeds corrupted .circuit files to
the native loaders (circuit_load_index, circuit_load_shard) and prints one
JSON summary line.  It runs in its own process so that a crash in a loader
shows up as a failed test instead of ending the test session."""
import ctypes
import json
import os
import struct
import sys

import numpy as np

HEADER_FIELDS = ("version", "dim", "rank", "num_roots", "num_total_children", "N")
CHILD_TABLES = ("child_parent_ids", "leaf_offsets", "leaf_sizes")


def _paths(root):
    for p in (os.path.join(root, "circuit-rag_b200"), root):
        if p not in sys.path:
            sys.path.insert(0, p)


def _header(data):
    hl = struct.unpack("<I", data[8:12])[0]
    return hl, json.loads(data[12:12 + hl].decode().rstrip("\x00 "))


def _with_header(data, hl, meta):
    text = json.dumps(meta).encode()
    if len(text) > hl:
        return None
    return data[:12] + text + b" " * (hl - len(text)) + data[12 + hl:]


def mutants(data, rng, n):
    """Yield (kind, bytes) corrupted copies of a valid .circuit file."""
    hl, meta = _header(data)
    tm = meta["tensor_meta"]
    nasty = [-1, -2 ** 31, 0, 1, 2 ** 31 - 1, 2 ** 31, 2 ** 40, 65, 7]
    for j in range(n):
        kind = j % 6
        b = bytearray(data)
        if kind == 0:  # one entry of a child table gets an out-of-range or random value
            name = CHILD_TABLES[int(rng.integers(0, 3))]
            e = tm[name]
            cnt = e["nbytes"] // 4
            i = int(rng.integers(0, cnt))
            R, N = meta["num_roots"], meta["N"]
            v = int(rng.choice([-1, -2 ** 31, R, R + 3, N, N + 1, N - 1, 2 ** 31 - 1,
                                int(rng.integers(0, max(N, 1)))]))
            struct.pack_into("<i", b, e["offset"] + 4 * i, v)
            yield f"child:{name}[{i}]={v}", bytes(b)
        elif kind == 1:  # a header integer
            m = json.loads(json.dumps(meta))
            key = HEADER_FIELDS[int(rng.integers(0, len(HEADER_FIELDS)))]
            m[key] = int(rng.choice(nasty + [meta[key] + 1, meta[key] - 1, meta[key] * 2]))
            out = _with_header(data, hl, m)
            if out is not None:
                yield f"header:{key}={m[key]}", out
        elif kind == 2:  # a tensor_meta shape, offset or nbytes
            m = json.loads(json.dumps(meta))
            name = list(tm)[int(rng.integers(0, len(tm)))]
            field = ["shape", "offset", "nbytes"][int(rng.integers(0, 3))]
            if field == "shape":
                shp = list(m["tensor_meta"][name]["shape"])
                shp[int(rng.integers(0, len(shp)))] = int(rng.choice(nasty))
                m["tensor_meta"][name]["shape"] = shp
            else:
                m["tensor_meta"][name][field] = int(rng.choice(nasty + [len(data), len(data) - 4]))
            out = _with_header(data, hl, m)
            if out is not None:
                yield f"meta:{name}.{field}", out
        elif kind == 3:  # random bytes in the header text
            for _ in range(int(rng.integers(1, 4))):
                b[12 + int(rng.integers(0, hl))] = int(rng.integers(0, 256))
            yield "header-bytes", bytes(b)
        elif kind == 4:  # truncated
            yield "truncated", bytes(b[:int(rng.integers(0, len(data)))])
        else:  # the header length word
            struct.pack_into("<I", b, 8, int(rng.choice([0, 1, 13, hl - 1, hl + 1, len(data), 2 ** 32 - 1])))
            yield "header-length", bytes(b)


def main(root, src, tmpdir, n, seed):
    _paths(root)
    from circuit_rag import _native

    L = _native.lib()
    data = open(src, "rb").read()
    rng = np.random.default_rng(seed)
    path = os.path.join(tmpdir, "fuzz.circuit")
    tried = rejected = loaded = 0
    unexplained = []
    for kind, blob in mutants(data, rng, n):
        with open(path, "wb") as f:
            f.write(blob)
        for shard in (False, True):
            tried += 1
            if shard:
                world = int(rng.integers(1, 4))
                h = L.circuit_load_shard(path.encode(), int(rng.integers(0, world)), world, 0, ctypes.c_double(1.05))
            else:
                h = L.circuit_load_index(path.encode(), 0)
            if h:
                loaded += 1
                L.circuit_destroy_index(h)
            else:
                rejected += 1
                if not _native.last_error():
                    unexplained.append(kind)
    print(json.dumps({"tried": tried, "rejected": rejected, "loaded": loaded, "unexplained": unexplained[:10]}))


if __name__ == "__main__":
    main(sys.argv[1], sys.argv[2], sys.argv[3], int(sys.argv[4]), int(sys.argv[5]))
