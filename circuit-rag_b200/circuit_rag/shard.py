"""Multi-GPU exact search: the corpus sharded by root cluster, one process per GPU.

* ``plan_shard_parts`` assigns roots to ranks largest first and cuts a root
  too large for its rank between children (Zipf-sized clusters make whole-root
  plans unbalanced); ``plan_shards`` is the whole-root plan.
* ``load_shard`` reads a .circuit file and keeps only the parts one rank owns:
  their centres, bases, children and leaf rows (read as byte ranges of the
  file, never the whole corpus) with their global original ids.  The native
  loader circuit_load_shard does the same without Python.
* ``ShardedSearcher.search`` runs the local exact search on the rank's GPU,
  all-gathers the k (score, id) candidates of every rank (NCCL over
  NVLink/NVSwitch; gloo works for CPU tests) and merges them on the device
  (``circuit_merge_topk``).  Every rank returns the identical global top-k.

Exactness: each shard's top-k contains every global top-k row it holds, so the
merge of all shard lists is the global top-k (same (score desc, id asc) order).
"""
import ctypes
import datetime
import mmap
from typing import Callable, Dict, Optional, Sequence, Tuple

import numpy as np
import torch

from circuit_rag import _native
from circuit_rag.hierarchy.build import CircuitIndex
from circuit_rag.storage.format import TENSOR_ORDER, check_child_tables, read_header


def plan_shards(root_rows: Sequence[int], world: int) -> np.ndarray:
    """root -> rank by longest-processing-time on leaf rows, whole roots only
    (circuit_plan_shards)."""
    rows = np.ascontiguousarray(root_rows, dtype=np.int64)
    out = np.empty(len(rows), dtype=np.int32)
    _native.check(_native.lib().circuit_plan_shards(rows.ctypes.data, len(rows), int(world), out.ctypes.data, None),
                  "plan_shards")
    return out


def plan_shard_parts(atom_rows: Sequence[int], root_atom_ptr: Sequence[int], world: int,
                     max_imbalance: float = 1.05) -> Dict[str, np.ndarray]:
    """Shard plan that cuts oversized roots between atoms (circuit_plan_shard_parts).
    Root p's rows are the atoms atom_rows[root_atom_ptr[p]:root_atom_ptr[p+1]]
    (its children in leaf order, or blocks of rows).  Returns arrays part_root,
    part_atom_begin, part_atom_end, part_rank (ordered by rank, root, first
    atom) and rank_rows."""
    atoms = np.ascontiguousarray(atom_rows, dtype=np.int64)
    ptr = np.ascontiguousarray(root_atom_ptr, dtype=np.int64)
    R = len(ptr) - 1
    cap = R + 2 * int(world) + 8
    while True:
        pr = np.empty(cap, np.int32)
        pb = np.empty(cap, np.int64)
        pe = np.empty(cap, np.int64)
        rk = np.empty(cap, np.int32)
        npart = ctypes.c_int(0)
        rr = np.empty(int(world), np.int64)
        rc = _native.lib().circuit_plan_shard_parts(atoms.ctypes.data, ptr.ctypes.data, R, int(world),
                                                    float(max_imbalance), pr.ctypes.data, pb.ctypes.data,
                                                    pe.ctypes.data, rk.ctypes.data, cap, ctypes.byref(npart),
                                                    rr.ctypes.data)
        if rc == 0:
            m = npart.value
            return {"part_root": pr[:m], "part_atom_begin": pb[:m], "part_atom_end": pe[:m], "part_rank": rk[:m],
                    "rank_rows": rr}
        if npart.value <= cap:
            _native.check(rc, "plan_shard_parts")
        cap = npart.value


def _root_children(parent: np.ndarray, offsets: np.ndarray, sizes: np.ndarray, num_roots: int):
    """CSR of each root's non-empty children in leaf order: (ptr [R+1], children)."""
    live = np.nonzero(sizes > 0)[0]
    order = live[np.lexsort((offsets[live], parent[live]))]
    counts = np.bincount(parent[order], minlength=num_roots)
    ptr = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
    return ptr, order


def load_shard(filepath: str, rank: int, world: int, device: str = "cuda",
               max_imbalance: float = 1.05) -> CircuitIndex:
    """The part of a .circuit index that `rank` of `world` owns.  The plan
    (plan_shard_parts over each root's children in leaf order) places whole
    roots where they fit and cuts a root too large for
    ``max_imbalance`` x the mean shard between children: each part becomes a
    root of the shard with the original centre, radius and basis, and keeps a
    contiguous range of its children.  Only the owned parts' byte ranges of the
    file are read; original ids stay global."""
    meta = read_header(filepath)
    R, C, D, r = (int(meta[k]) for k in ("num_roots", "num_total_children", "dim", "rank"))
    with open(filepath, "rb") as f:
        mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
    try:
        def arr(name):
            info = meta["tensor_meta"][name]
            return np.ndarray(buffer=mm, dtype=np.dtype(info["dtype"]), offset=int(info["offset"]),
                              shape=tuple(info["shape"]))

        parent, offsets, sizes = (arr(n).copy() for n in ("child_parent_ids", "leaf_offsets", "leaf_sizes"))
        check_child_tables(parent, offsets, sizes, R, int(meta["N"]))
        ptr, kids_all = _root_children(parent, offsets, sizes, R)
        plan = plan_shard_parts(sizes[kids_all].astype(np.int64), ptr, world, max_imbalance)
        own = np.nonzero(plan["part_rank"] == rank)[0]
        roots = plan["part_root"][own]
        kids = [kids_all[int(a):int(b)] for a, b in zip(plan["part_atom_begin"][own], plan["part_atom_end"][own])]
        cpr = max([len(k) for k in kids] + [1])
        Rs, Cs = len(roots), max(1, len(roots)) * cpr
        n_rows = int(sum(int(sizes[k].sum()) for k in kids))
        leaf_src, ids_src = arr("leaf_vectors"), arr("original_ids")
        leaf = np.empty((n_rows, D), np.float32)
        ids = np.empty(n_rows, np.int32)
        cl, cu, crad = arr("child_intervals_l"), arr("child_intervals_u"), arr("child_radii")
        new = {
            "child_intervals_l": np.zeros((Cs, r), np.float32), "child_intervals_u": np.zeros((Cs, r), np.float32),
            "child_radii": np.zeros(Cs, np.float32), "child_parent_ids": np.zeros(Cs, np.int32),
            "leaf_offsets": np.zeros(Cs, np.int32), "leaf_sizes": np.zeros(Cs, np.int32),
        }
        cur = 0
        for i, ks in enumerate(kids):
            for j, c in enumerate(ks):
                g = i * cpr + j
                o, n = int(offsets[c]), int(sizes[c])
                leaf[cur:cur + n] = leaf_src[o:o + n]
                ids[cur:cur + n] = ids_src[o:o + n]
                new["child_intervals_l"][g] = cl[c]
                new["child_intervals_u"][g] = cu[c]
                new["child_radii"][g] = crad[c]
                new["child_parent_ids"][g] = i
                new["leaf_offsets"][g] = cur
                new["leaf_sizes"][g] = n
                cur += n
            for j in range(len(ks), cpr):
                new["child_parent_ids"][i * cpr + j] = i
        centers, radii, bases = arr("root_centers")[roots].copy(), arr("root_radii")[roots].copy(), \
            arr("bases")[roots].copy()
    finally:
        mm.close()
    if Rs == 0:
        raise ValueError(f"rank {rank} owns no rows (world {world} > non-empty children)")
    idx = CircuitIndex(root_centers=centers, root_radii=radii, bases=bases, leaf_vectors=leaf, original_ids=ids,
                       dim=D, rank=r, device=device, **new)
    idx.shard_info = {"rank": rank, "world": world, "part_root": roots.tolist(), "rows": n_rows,
                      "rank_rows": plan["rank_rows"].tolist(), "parts_total": int(len(plan["part_root"])),
                      "roots": R}
    return idx


def _aligned(q: torch.Tensor) -> torch.Tensor:
    q = q.to(torch.float32).contiguous()
    return q if q.data_ptr() % 16 == 0 else q.clone()


def merge_topk(scores: torch.Tensor, ids: torch.Tensor, k: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """Global top-k of gathered candidates on the device (circuit_merge_topk)."""
    scores = scores.to(torch.float32).contiguous()
    ids = ids.to(torch.int32).contiguous()
    out_s = torch.empty(k, dtype=torch.float32, device=scores.device)
    out_i = torch.empty(k, dtype=torch.int32, device=scores.device)
    rc = _native.lib().circuit_merge_topk(scores.data_ptr(), ids.data_ptr(), scores.numel(), int(k), out_s.data_ptr(),
                                          out_i.data_ptr(), torch.cuda.current_stream(scores.device).cuda_stream)
    _native.check(rc, "merge_topk")
    return out_s, out_i


def merge_topk_batch(scores: torch.Tensor, ids: torch.Tensor, k: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """Per-query global top-k of gathered batch results on the device
    (circuit_merge_topk_batch): scores / ids [world, B, k_in] -> [B, k]."""
    world, B, k_in = scores.shape
    scores = scores.to(torch.float32).contiguous()
    ids = ids.to(torch.int32).contiguous()
    out_s = torch.empty(B, k, dtype=torch.float32, device=scores.device)
    out_i = torch.empty(B, k, dtype=torch.int32, device=scores.device)
    rc = _native.lib().circuit_merge_topk_batch(scores.data_ptr(), ids.data_ptr(), B, world, k_in, int(k),
                                                out_s.data_ptr(), out_i.data_ptr(),
                                                torch.cuda.current_stream(scores.device).cuda_stream)
    _native.check(rc, "merge_topk_batch")
    return out_s, out_i


def merge_topk_batch_host(scores: torch.Tensor, ids: torch.Tensor, k: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """The batched merge on host tensors (used with the gloo backend)."""
    world, B, k_in = scores.shape
    out_s = torch.empty(B, k)
    out_i = torch.empty(B, k, dtype=torch.int32)
    for q in range(B):
        out_s[q], out_i[q] = merge_topk_host(scores[:, q].reshape(-1), ids[:, q].reshape(-1), k)
    return out_s, out_i


def merge_topk_host(scores: torch.Tensor, ids: torch.Tensor, k: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """The same merge on host tensors (used with the gloo backend)."""
    s = scores.double().numpy()
    i = ids.numpy().astype(np.int64)
    live = i >= 0
    s, i = s[live], i[live]
    order = np.lexsort((i, -s))[:k]
    out_s = torch.full((k,), float("-inf"))
    out_i = torch.full((k,), -1, dtype=torch.int32)
    out_s[:len(order)] = torch.from_numpy(s[order]).float()
    out_i[:len(order)] = torch.from_numpy(i[order]).int()
    return out_s, out_i


class SharedThreshold:
    """The running threshold shared by the ranks of a process group that search
    the same query on their shards (circuit_search_finish_shared_async): every
    rank owns one 64-bit word on its GPU; the words' CUDA IPC handles are
    all-gathered and every rank opens the others', so each rank's main scan
    raises every word with the k-th best scores it finds and prunes with the
    largest one carrying the query's tag.  The tag is a counter advanced by
    finish(), identical on every rank as long as every rank searches the same
    queries in the same order.  Construction is collective."""

    def __init__(self, device: torch.device, group=None):
        import torch.distributed as dist

        self.dist, self.group = dist, group
        world, rank = dist.get_world_size(group), dist.get_rank(group)
        lib = _native.lib()
        self.word = torch.zeros(1, dtype=torch.int64, device=device)
        handle = (ctypes.c_ubyte * 64)()
        offset = ctypes.c_int64()
        _native.check(lib.circuit_ipc_export(self.word.data_ptr(), handle, ctypes.byref(offset)), "ipc export")
        mine = torch.tensor(list(bytes(handle)) + list(int(offset.value).to_bytes(8, "little", signed=True)),
                            dtype=torch.uint8, device=device)
        every = torch.empty(world * 72, dtype=torch.uint8, device=device)
        dist.all_gather_into_tensor(every, mine, group=group)
        every = every.cpu().numpy().reshape(world, 72)
        self.imported, peers = [], []
        for r in range(world):
            if r == rank:
                continue
            ptr = ctypes.c_void_p()
            _native.check(lib.circuit_ipc_import(every[r, :64].tobytes(), device.index, ctypes.byref(ptr)),
                          "ipc import")
            self.imported.append(ptr.value)
            peers.append(ptr.value + int.from_bytes(every[r, 64:].tobytes(), "little", signed=True))
        self.peers = torch.tensor(peers or [0], dtype=torch.int64, device=device)
        self.n_peers = len(peers)
        self.tag = 0
        dist.barrier(group=group)  # every rank's peers are open before any scan writes to them

    def finish(self, index, query, k, T, scores, ids, stream):
        """circuit_search_finish_shared_async for the next query (advances the tag)."""
        self.tag = ((self.tag + 1) & 0xFFFFFFFF) or 1
        rc = _native.lib().circuit_search_finish_shared_async(
            index.native_handle(), _aligned(query).data_ptr(), int(k), T.data_ptr() if T is not None else None,
            self.word.data_ptr(), self.peers.data_ptr(), self.n_peers, self.tag, scores.data_ptr(), ids.data_ptr(),
            None, stream, None, None)
        _native.check(rc, "circuit_search_finish_shared_async")

    def close(self):
        self.dist.barrier(group=self.group)
        for p in self.imported:
            _native.lib().circuit_ipc_close(p)
        self.imported = []


class ShardedSearcher:
    """Exact top-k over a corpus sharded across the ranks of a process group."""

    def __init__(self, index: Optional[CircuitIndex], group=None,
                 local_search: Optional[Callable] = None, merge: Optional[Callable] = None):
        import torch.distributed as dist

        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.index = index
        self._local = local_search or self._native_local
        self._merge = merge or merge_topk
        self._shared = None  # SharedThreshold (enable_shared_threshold)

    def enable_shared_threshold(self):
        """Share the running threshold of a search between the ranks while their
        scans run (circuit_search_finish_shared_async; see SharedThreshold).
        Collective; used by search(..., exchange_threshold=True)."""
        self._shared = SharedThreshold(self.index.leaf_vectors.device, self.group)

    def close_shared_threshold(self):
        """Collective: no rank may still be searching."""
        if self._shared is not None:
            self._shared.close()
            self._shared = None

    def _native_local(self, query: torch.Tensor, k: int, min_hierarchy_n: int):
        from circuit_rag.search import circuit_search

        s, i, _ = circuit_search(query, self.index, k=min(k, self.index.N), min_hierarchy_n=min_hierarchy_n)
        if len(i) < k:  # a shard smaller than k: pad with empty slots
            s = torch.cat([s, s.new_full((k - len(s),), float("-inf"))])
            i = torch.cat([i, i.new_full((k - len(i),), -1)])
        return s, i

    def search(self, query: torch.Tensor, k: int = 10, min_hierarchy_n: int = 10000,
               exchange_threshold: bool = False, local_seed: Optional[Callable] = None,
               local_finish: Optional[Callable] = None, seed_allreduce: bool = True):
        """Global exact top-k of one query.  With exchange_threshold, every rank
        first computes its shard's seed threshold, one all-reduce (MAX) makes
        the largest of them every rank's pruning threshold (it never exceeds
        the global k-th best score), then each rank finishes its search.
        seed_allreduce=False (needs enable_shared_threshold) skips that
        all-reduce: each rank starts from its own seed and the ranks exchange
        thresholds only through the shared running threshold while their scans
        run, so the bounds and the scan follow the seed on the GPU without
        waiting for the other ranks."""
        if exchange_threshold:
            if not seed_allreduce and self._shared is None and local_finish is None:
                raise ValueError("seed_allreduce=False exchanges thresholds only through the shared running "
                                 "threshold: call enable_shared_threshold() first")
            T = (local_seed or self._native_seed)(query, k)
            if seed_allreduce:
                self.dist.all_reduce(T, op=self.dist.ReduceOp.MAX, group=self.group)
            s, i = (local_finish or self._native_finish)(query, k, T)
        else:
            s, i = self._local(query, k, min_hierarchy_n)
        gs = s.new_empty(self.world * k)
        gi = i.new_empty(self.world * k)
        self.dist.all_gather_into_tensor(gs, s.contiguous(), group=self.group)
        self.dist.all_gather_into_tensor(gi, i.contiguous(), group=self.group)
        return self._merge(gs, gi, k)

    def _native_seed(self, query: torch.Tensor, k: int) -> torch.Tensor:
        T = torch.empty(1, dtype=torch.float32, device=query.device)
        rc = _native.lib().circuit_search_seed_async(self.index.native_handle(), _aligned(query).data_ptr(), int(k),
                                                     T.data_ptr(), torch.cuda.current_stream(query.device).cuda_stream)
        _native.check(rc, "circuit_search_seed_async")
        return T

    def _native_finish(self, query: torch.Tensor, k: int, T: torch.Tensor):
        s = torch.empty(k, dtype=torch.float32, device=query.device)
        i = torch.empty(k, dtype=torch.int32, device=query.device)
        st = torch.cuda.current_stream(query.device).cuda_stream
        if self._shared is not None:
            self._shared.finish(self.index, query, k, T, s, i, st)
            return s, i
        rc = _native.lib().circuit_search_finish_async(self.index.native_handle(), _aligned(query).data_ptr(), int(k),
                                                       T.data_ptr(), s.data_ptr(), i.data_ptr(), None, st, None,
                                                       None)
        _native.check(rc, "circuit_search_finish_async")
        return s, i

    def search_batch(self, queries: torch.Tensor, k: int = 10, local_batch: Optional[Callable] = None,
                     merge_batch: Optional[Callable] = None):
        """Exact top-k of a batch [B, dim]: each rank runs the batched search on
        its shard, one all-gather of [B, k] scores and ids, per-query merge."""
        local = local_batch or self._native_local_batch
        s, i = local(queries, k)
        B = queries.shape[0]
        gs = s.new_empty((self.world * B, k))
        gi = i.new_empty((self.world * B, k))
        self.dist.all_gather_into_tensor(gs, s.contiguous(), group=self.group)
        self.dist.all_gather_into_tensor(gi, i.contiguous(), group=self.group)
        return (merge_batch or merge_topk_batch)(gs.view(self.world, B, k), gi.view(self.world, B, k), k)

    def _native_local_batch(self, queries: torch.Tensor, k: int):
        from circuit_rag.search import circuit_search_batch

        s, i = circuit_search_batch(queries, self.index, k=min(k, self.index.N))
        if i.shape[1] < k:
            s = torch.cat([s, s.new_full((s.shape[0], k - s.shape[1]), float("-inf"))], dim=1)
            i = torch.cat([i, i.new_full((i.shape[0], k - i.shape[1]), -1)], dim=1)
        return s, i


def init_process_group(backend: str = "nccl", timeout_s: float = 120.0):
    """One process per GPU (torchrun env vars); a short timeout turns a lost rank
    into an error on the survivors' next collective instead of a hang."""
    import os

    import torch.distributed as dist

    if backend == "nccl":
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s),
                                device_id=torch.device("cuda", local))
    else:
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s))
    return dist.get_rank(), dist.get_world_size()
