"""CircuitIndex (index container + device workspace + CUDA-graph replay) and the
index builder.

Container: reference circuit_rag/hierarchy/build.py:7-131.  The index tensors
keep the reference names, shapes and dtypes (float32 / int32), so a
``.circuit`` file written by either side loads in the other.  When the index
lives on a CUDA device it owns a native handle (libcircuit.so) that borrows the
tensors' device memory and holds the search workspace; searches never copy the
index.

Builder: reference build.py:133-387.  Same hierarchy (k-means roots; per-root
rank-r PCA basis, orthonormalised by QR; per-root k-means children; per-child
coordinate boxes in the root basis and residual radii; root-major,
child-contiguous leaf layout), built with torch on CPU or GPU.  Unlike the
reference, every certificate (root radius, box, residual radius) is computed
in float64 from the float32 data and basis and rounded outward to float32, then
widened by the reference's 1e-5 slack, so the stored bounds hold for the exact
projections of the stored float32 vectors.  Builder outputs are not bitwise
the reference's (different k-means), only structurally identical.
"""
from typing import Optional

import numpy as np
import torch

from circuit_rag import _native

MAX_RANK = _native.CIRCUIT_MAX_RANK


def _default_device() -> str:
    return "cuda" if torch.cuda.is_available() else "cpu"


class CircuitIndex:
    _FLOAT = ("root_centers", "root_radii", "bases", "child_intervals_l", "child_intervals_u", "child_radii",
              "leaf_vectors")
    _INT = ("child_parent_ids", "leaf_offsets", "leaf_sizes", "original_ids")

    def __init__(self, root_centers, root_radii, bases, child_intervals_l, child_intervals_u, child_radii,
                 child_parent_ids, leaf_offsets, leaf_sizes, leaf_vectors, original_ids, dim, rank,
                 device: Optional[str] = None):
        if device is None:
            device = _default_device()
        if str(device).startswith("cuda") and not torch.cuda.is_available():
            device = "cpu"  # storage only; searches require a CUDA device
        self.device = device
        given = dict(root_centers=root_centers, root_radii=root_radii, bases=bases,
                     child_intervals_l=child_intervals_l, child_intervals_u=child_intervals_u,
                     child_radii=child_radii, child_parent_ids=child_parent_ids, leaf_offsets=leaf_offsets,
                     leaf_sizes=leaf_sizes, leaf_vectors=leaf_vectors, original_ids=original_ids)
        for name, t in given.items():
            t = torch.as_tensor(t)
            dt = torch.float32 if name in self._FLOAT else torch.int32
            setattr(self, name, t.to(device=device, dtype=dt).contiguous())
        self.dim = int(dim)
        self.rank = int(rank)
        self.num_roots = self.root_centers.shape[0]
        self.num_total_children = self.child_radii.shape[0]
        self.N = self.leaf_vectors.shape[0]
        self._cuda_graphs = {}
        self._handle = None
        self._ws = {}

    # ------------------------------------------------------------------ native handle
    @property
    def is_cuda(self) -> bool:
        return self.leaf_vectors.is_cuda

    def native_handle(self):
        """The libcircuit handle over this index's device tensors (created on first use)."""
        if self._handle is None:
            if not self.is_cuda:
                raise RuntimeError("circuit-b200 searches run on a CUDA device; build or load the index with "
                                   "device='cuda'")
            lib = _native.lib()
            dev = self.leaf_vectors.device.index or 0
            with torch.cuda.device(dev):
                torch.cuda.current_stream().synchronize()
                h = lib.circuit_index_from_device(
                    dev, self.dim, self.rank, self.num_roots, self.num_total_children, self.N,
                    self.root_centers.data_ptr(), self.root_radii.data_ptr(), self.bases.data_ptr(),
                    self.child_intervals_l.data_ptr(), self.child_intervals_u.data_ptr(),
                    self.child_radii.data_ptr(), self.child_parent_ids.data_ptr(), self.leaf_offsets.data_ptr(),
                    self.leaf_sizes.data_ptr(), self.leaf_vectors.data_ptr(), self.original_ids.data_ptr())
            if not h:
                raise _native.NativeLibraryError(f"circuit_index_from_device failed: {_native.last_error()}")
            self._handle = h
        return self._handle

    def close(self) -> None:
        """Release the native handle (the tensors stay valid)."""
        self._cuda_graphs = {}
        if self._handle is not None:
            _native.lib().circuit_destroy_index(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ------------------------------------------------------------------ workspaces
    def _init_workspace(self):
        """Reference build.py:35-49: the ws_* tensors used by the op-level
        ``circuit_cuda.hierarchical_search``.  The fused search does not need
        them; they are allocated on first access."""
        for name in ("ws_survivor_mask", "ws_vector_scores"):
            getattr(self, name)

    _WS_SPECS = {
        "ws_survivor_mask": ("R", torch.int32),
        "ws_survivor_indices": ("R", torch.int32),
        "ws_num_survivors": ("1", torch.int32),
        "ws_root_dot_products": ("R", torch.float32),
        "ws_projected_queries": ("Rr", torch.float32),
        "ws_perp_norms": ("R", torch.float32),
        "ws_child_survivor_mask": ("C", torch.int32),
        "ws_child_survivor_indices": ("C", torch.int32),
        "ws_num_child_survivors": ("1", torch.int32),
        "ws_vector_scores": ("N", torch.float32),
    }

    def __getattr__(self, name):
        spec = CircuitIndex._WS_SPECS.get(name)
        if spec is None:
            raise AttributeError(name)
        ws = self.__dict__.setdefault("_ws", {})
        if name not in ws:
            shape = {"R": (self.num_roots,), "1": (1,), "Rr": (self.num_roots, self.rank),
                     "C": (self.num_total_children,), "N": (self.N,)}[spec[0]]
            fill = -1e9 if name == "ws_vector_scores" else 0
            ws[name] = torch.full(shape, fill, dtype=spec[1], device=self.leaf_vectors.device)
        return ws[name]

    # ------------------------------------------------------------------ incremental growth
    def append(self, X_new, ids_new=None) -> None:
        """Add rows without rebuilding the hierarchy.

        Each new row joins the root with the largest inner product with its
        centre (the builder's assignment rule); the root's radius is widened
        if needed, and every touched root gets one new child whose box and
        residual radius are computed from the new rows against the root's
        stored float32 basis, in float64 with outward rounding (the builder's
        certificate rules, so pruning stays exact).  Rows and children are
        then laid out root-major again, so every root's rows stay contiguous.
        ``ids_new`` defaults to N, N + 1, ...  Costs one gather of the leaf rows;
        the native handle, workspaces and captured graphs are rebuilt on the
        next search."""
        Xn = torch.as_tensor(np.ascontiguousarray(X_new, dtype=np.float32) if isinstance(X_new, np.ndarray)
                             else X_new).to(device=self.leaf_vectors.device, dtype=torch.float32).contiguous()
        if Xn.ndim != 2 or Xn.shape[1] != self.dim:
            raise ValueError("X_new must have shape [n, index.dim]")
        n_new = Xn.shape[0]
        if n_new == 0:
            return
        dev = self.leaf_vectors.device
        if ids_new is None:
            ids_new = torch.arange(self.N, self.N + n_new, dtype=torch.int32, device=dev)
        ids_new = torch.as_tensor(ids_new).to(device=dev, dtype=torch.int32).reshape(-1)
        if ids_new.numel() != n_new:
            raise ValueError("ids_new must have one id per new row")
        labels = _assign(Xn, self.root_centers)
        touched = torch.unique(labels).tolist()
        C0, r = self.num_total_children, self.rank
        new_l, new_u, new_rho, new_parent, new_rows = [], [], [], [], []
        radii = self.root_radii.clone()
        for p in touched:
            sel = torch.nonzero(labels == p).flatten()
            d = Xn[sel].double() - self.root_centers[p].double()
            rad = d.norm(dim=1).max() + _EPS
            radii[p] = torch.maximum(radii[p], _round_up_f32(rad.reshape(1))[0])
            Q64 = self.bases[p].double()
            z = d @ Q64
            new_l.append(_round_down_f32(z.min(dim=0).values - _EPS))
            new_u.append(_round_up_f32(z.max(dim=0).values + _EPS))
            res = d - z @ Q64.T
            new_rho.append(_round_up_f32((res.norm(dim=1).max() + _EPS).reshape(1))[0])
            new_parent.append(p)
            new_rows.append(sel)
        # children of both kinds, root-major: each root's old children (in leaf
        # order), then its new child; empty children keep their records
        parent = torch.cat([self.child_parent_ids.long(), torch.tensor(new_parent, device=dev)])
        sizes = torch.cat([self.leaf_sizes.long(), torch.tensor([len(x) for x in new_rows], device=dev)])
        offs = torch.cat([self.leaf_offsets.long(), torch.full((len(new_rows),), self.N, device=dev)])
        is_new = torch.cat([torch.zeros(C0, dtype=torch.long, device=dev),
                            torch.ones(len(new_rows), dtype=torch.long, device=dev)])
        key = (parent * 2 + is_new) * (self.N + n_new + 1) + offs
        order = torch.argsort(key, stable=True)
        # gather map over the source [old leaf rows ; new rows]
        new_src = torch.cat([x + self.N for x in new_rows]) if new_rows else torch.empty(0, dtype=torch.long,
                                                                                        device=dev)
        starts = torch.cat([self.leaf_offsets.long(), torch.cumsum(torch.tensor([0] + [len(x) for x in new_rows][:-1],
                                                                                 device=dev), 0) + self.N])
        pieces = []
        for g in order.tolist():
            m = int(sizes[g])
            if m == 0:
                continue
            if g < C0:
                pieces.append(torch.arange(int(starts[g]), int(starts[g]) + m, device=dev))
            else:
                b = int(starts[g]) - self.N
                pieces.append(new_src[b:b + m])
        gather = torch.cat(pieces)
        src_rows = torch.cat([self.leaf_vectors, Xn])
        src_ids = torch.cat([self.original_ids, ids_new])
        sizes_o = sizes[order]
        offs_o = torch.cumsum(sizes_o, 0) - sizes_o
        l_all = torch.cat([self.child_intervals_l] + ([torch.stack(new_l)] if new_l else []))[order]
        u_all = torch.cat([self.child_intervals_u] + ([torch.stack(new_u)] if new_u else []))[order]
        rho_all = torch.cat([self.child_radii] + ([torch.stack(new_rho)] if new_rho else []))[order]
        self.close()
        self.__dict__["_ws"] = {}
        self.root_radii = radii.contiguous()
        self.child_intervals_l = l_all.contiguous()
        self.child_intervals_u = u_all.contiguous()
        self.child_radii = rho_all.contiguous()
        self.child_parent_ids = parent[order].to(torch.int32).contiguous()
        self.leaf_offsets = offs_o.to(torch.int32).contiguous()
        self.leaf_sizes = sizes_o.to(torch.int32).contiguous()
        self.leaf_vectors = src_rows[gather].contiguous()
        self.original_ids = src_ids[gather].contiguous()
        self.num_total_children = self.child_radii.shape[0]
        self.N = self.leaf_vectors.shape[0]

    # ------------------------------------------------------------------ CUDA graphs
    def warmup_cuda_graph(self, k: int = 10):
        """Capture one search (pruning on) into a CUDA graph on static buffers
        (reference build.py:51-106 captured it with pruning off)."""
        from circuit_rag.search import _launch

        if not self.is_cuda:
            return
        k_actual = min(k, self.N)
        h = self.native_handle()
        static_query = torch.zeros(self.dim, dtype=torch.float32, device=self.leaf_vectors.device)
        static_vals = torch.empty(k_actual, dtype=torch.float32, device=static_query.device)
        static_ids = torch.empty(k_actual, dtype=torch.int32, device=static_query.device)
        s = torch.cuda.Stream(device=static_query.device)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(3):
                _launch(h, static_query, k_actual, 10001, static_vals, static_ids, None, s)
        torch.cuda.current_stream().wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            _launch(h, static_query, k_actual, 10001, static_vals, static_ids, None, s)
        self._cuda_graphs[k] = {"graph": graph, "stream": s, "static_query": static_query,
                                "static_top_vals": static_vals, "static_top_ids": static_ids}

    def has_cuda_graph(self, k: int = 10) -> bool:
        return k in self._cuda_graphs

    def search_graph(self, query: torch.Tensor, k: int = 10):
        """Replay the captured search (reference build.py:111-118)."""
        if not self.has_cuda_graph(k):
            self.warmup_cuda_graph(k)
        g = self._cuda_graphs[k]
        g["static_query"].copy_(query)
        g["graph"].replay()
        return g["static_top_vals"], g["static_top_ids"].clone()

    # ------------------------------------------------------------------ persistence
    def save(self, filepath: str) -> int:
        """Write this index to a .circuit file (reference build.py:120-123)."""
        from circuit_rag.storage.format import save_circuit_index

        return save_circuit_index(self, filepath)

    @classmethod
    def load(cls, filepath: str, device: Optional[str] = None, use_mmap: bool = True) -> "CircuitIndex":
        """Load a .circuit file (reference build.py:125-131)."""
        from circuit_rag.storage.format import load_circuit_index

        if device is None:
            device = _default_device()
        return load_circuit_index(filepath, device=device, use_mmap=use_mmap)


# ====================================================================== builder
_EPS = 1e-5  # the reference's certificate slack (build.py:188, :223-227)


def _round_up_f32(x: torch.Tensor) -> torch.Tensor:
    """float64 -> float32 rounded towards +inf."""
    f = x.to(torch.float32)
    low = f.to(torch.float64) < x
    return torch.where(low, torch.nextafter(f, torch.full_like(f, float("inf"))), f)


def _round_down_f32(x: torch.Tensor) -> torch.Tensor:
    f = x.to(torch.float32)
    high = f.to(torch.float64) > x
    return torch.where(high, torch.nextafter(f, torch.full_like(f, float("-inf"))), f)


def _assign(X: torch.Tensor, centers: torch.Tensor, chunk: int = 1 << 16) -> torch.Tensor:
    """argmax_j <x, c_j> per row (reference build.py:153-154), in row chunks."""
    out = torch.empty(X.shape[0], dtype=torch.long, device=X.device)
    ct = centers.T.contiguous()
    for s in range(0, X.shape[0], chunk):
        out[s:s + chunk] = torch.argmax(X[s:s + chunk] @ ct, dim=1)
    return out


def _kmeans(X: torch.Tensor, k: int, iters: int, gen: torch.Generator) -> torch.Tensor:
    """Lloyd iterations with max-inner-product assignment (reference build.py:150-161)."""
    n = X.shape[0]
    init = torch.randperm(n, generator=gen, device="cpu")[:k].to(X.device)
    centers = X[init].clone()
    for _ in range(iters):
        labels = _assign(X, centers)
        sums = torch.zeros_like(centers).index_add_(0, labels, X)
        counts = torch.bincount(labels, minlength=k).to(X.dtype)
        nz = counts > 0
        centers[nz] = sums[nz] / counts[nz, None]
    return centers


def build_circuit_index(X, num_roots: int = 128, children_per_root: int = 16, rank: int = 8,
                        random_state: int = 42, device: Optional[str] = None) -> CircuitIndex:
    """Build the two-level hierarchy (reference build.py:256-275 signature).
    ``rank`` may be up to 64 (the reference rejects rank > 32, build.py:266-267)."""
    if rank > MAX_RANK:
        raise ValueError(f"rank must be <= {MAX_RANK}")
    if rank < 1:
        raise ValueError("rank must be >= 1")
    if device is None:
        device = _default_device()
    if str(device).startswith("cuda") and not torch.cuda.is_available():
        device = "cpu"
    Xt = torch.as_tensor(np.ascontiguousarray(X, dtype=np.float32) if isinstance(X, np.ndarray) else X)
    Xt = Xt.to(device=device, dtype=torch.float32).contiguous()
    N, D = Xt.shape
    if N < num_roots:
        raise ValueError("corpus smaller than num_roots")
    gen = torch.Generator(device="cpu")
    gen.manual_seed(random_state)

    root_centers = _kmeans(Xt, num_roots, 8, gen)
    root_labels = _assign(Xt, root_centers)
    order = torch.argsort(root_labels, stable=True)
    counts = torch.bincount(root_labels, minlength=num_roots).cpu().tolist()

    C = num_roots * children_per_root
    f32 = dict(dtype=torch.float32, device=device)
    root_radii = torch.zeros(num_roots, **f32)
    bases = torch.zeros((num_roots, D, rank), **f32)
    child_l = torch.zeros((C, rank), **f32)
    child_u = torch.zeros((C, rank), **f32)
    child_radii = torch.zeros(C, **f32)
    child_parent = torch.zeros(C, dtype=torch.int32, device=device)
    leaf_offsets = torch.zeros(C, dtype=torch.int32, device=device)
    leaf_sizes = torch.zeros(C, dtype=torch.int32, device=device)
    ordered_rows = []
    cursor = 0
    start = 0
    for p in range(num_roots):
        n_p = counts[p]
        if n_p == 0:
            continue
        idx = order[start:start + n_p]
        start += n_p
        vecs = Xt[idx]
        c = root_centers[p]
        diffs64 = vecs.double() - c.double()
        root_radii[p] = _round_up_f32(diffs64.norm(dim=1).max() + _EPS)
        actual = min(rank, n_p, D)
        Vfull = torch.zeros((D, rank), dtype=torch.float64, device=device)
        if n_p > 1:
            _, _, Vh = torch.linalg.svd(diffs64, full_matrices=False)
            Vfull[:, :actual] = Vh[:actual].T
        else:
            Vfull[:, :actual] = torch.eye(D, dtype=torch.float64, device=device)[:, :actual]
        Q, _ = torch.linalg.qr(Vfull)
        Q32 = Q.to(torch.float32)
        bases[p] = Q32
        Q64 = Q32.double()  # certificates are computed for the stored float32 basis
        k_c = min(children_per_root, n_p)
        if k_c > 1:
            cc = _kmeans(vecs, k_c, 5, gen)
            clabels = _assign(vecs, cc)
        else:
            clabels = torch.zeros(n_p, dtype=torch.long, device=device)
        corder = torch.argsort(clabels, stable=True)
        ccounts = torch.bincount(clabels, minlength=k_c).cpu().tolist()
        cs = 0
        for ci in range(k_c):
            g = p * children_per_root + ci
            child_parent[g] = p
            m = ccounts[ci]
            if m == 0:
                continue
            sub = corder[cs:cs + m]
            cs += m
            cd = diffs64[sub]
            z = cd @ Q64
            child_l[g] = _round_down_f32(z.min(dim=0).values - _EPS)
            child_u[g] = _round_up_f32(z.max(dim=0).values + _EPS)
            res = cd - z @ Q64.T
            child_radii[g] = _round_up_f32(res.norm(dim=1).max() + _EPS)
            leaf_offsets[g] = cursor
            leaf_sizes[g] = m
            ordered_rows.append(idx[sub])
            cursor += m
    ordered = torch.cat(ordered_rows)
    return CircuitIndex(
        root_centers=root_centers, root_radii=root_radii, bases=bases, child_intervals_l=child_l,
        child_intervals_u=child_u, child_radii=child_radii, child_parent_ids=child_parent,
        leaf_offsets=leaf_offsets, leaf_sizes=leaf_sizes, leaf_vectors=Xt[ordered],
        original_ids=ordered.to(torch.int32), dim=D, rank=rank, device=device)


def _eig_basis(gram: torch.Tensor, rank: int) -> torch.Tensor:
    """Top-`rank` eigenvectors of a float64 Gram matrix, orthonormalised by QR
    and rounded to float32 (the PCA basis of reference build.py:190-195)."""
    D = gram.shape[0]
    evals, evecs = torch.linalg.eigh(gram)
    V = torch.zeros((D, rank), dtype=torch.float64, device=gram.device)
    take = min(rank, D)
    V[:, :take] = evecs[:, -take:].flip(1)
    Q, _ = torch.linalg.qr(V)
    return Q.to(torch.float32)


def _part_hierarchy(leaf, orig, part_off, part_root, centers, children_per_root, rank, random_state, device,
                    sub=1 << 17):
    """Children and certificates of each part (a root, or a contiguous slice of
    a root's rows) laid out in leaf[part_off[j]:part_off[j+1]]: the PCA basis
    of the part's rows (top eigenvectors of the float64 Gram matrix of x - c,
    QR, float32), k-means children (generator seeded by (random_state, root,
    first row of the part), so a part's children do not depend on which rank
    builds it), rows reordered child-contiguous in place, and the float64
    certificates of build_circuit_index.  Returns the per-part / per-child arrays."""
    P = len(part_root)
    dim = leaf.shape[1]
    C = P * children_per_root
    f32 = dict(dtype=torch.float32, device=device)
    out = dict(root_centers=torch.zeros((P, dim), **f32), root_radii=torch.zeros(P, **f32),
               bases=torch.zeros((P, dim, rank), **f32), child_intervals_l=torch.zeros((C, rank), **f32),
               child_intervals_u=torch.zeros((C, rank), **f32), child_radii=torch.zeros(C, **f32),
               child_parent_ids=torch.zeros(C, dtype=torch.int32, device=device),
               leaf_offsets=torch.zeros(C, dtype=torch.int32, device=device),
               leaf_sizes=torch.zeros(C, dtype=torch.int32, device=device))
    for j in range(P):
        o_p, n_p = int(part_off[j]), int(part_off[j + 1] - part_off[j])
        for ci in range(children_per_root):
            out["child_parent_ids"][j * children_per_root + ci] = j
        c32 = centers[int(part_root[j])]
        out["root_centers"][j] = c32
        if n_p == 0:
            continue
        c64 = c32.double()
        gram = torch.zeros((dim, dim), dtype=torch.float64, device=device)
        rad = torch.zeros((), dtype=torch.float64, device=device)
        for a in range(o_p, o_p + n_p, sub):
            d = leaf[a:min(o_p + n_p, a + sub)].double() - c64
            gram += d.T @ d
            rad = torch.maximum(rad, d.norm(dim=1).max())
        out["root_radii"][j] = _round_up_f32(rad + _EPS)
        Q32 = _eig_basis(gram, rank)
        out["bases"][j] = Q32
        Q64 = Q32.double()
        k_c = min(children_per_root, n_p)
        if k_c > 1:
            gen = torch.Generator(device="cpu")
            gen.manual_seed((random_state * 1_000_003 + int(part_root[j]) * 7919 + int(orig[o_p]) * 31) % (2 ** 62))
            cc = _kmeans(leaf[o_p:o_p + min(n_p, 1 << 16)], k_c, 5, gen)
            clab = torch.cat([_assign(leaf[a:min(o_p + n_p, a + sub)], cc) for a in range(o_p, o_p + n_p, sub)])
        else:
            clab = torch.zeros(n_p, dtype=torch.long, device=device)
        perm = torch.argsort(clab, stable=True)
        leaf[o_p:o_p + n_p] = leaf[o_p:o_p + n_p][perm]
        orig[o_p:o_p + n_p] = orig[o_p:o_p + n_p][perm]
        ccounts = torch.bincount(clab, minlength=k_c).tolist()
        cs = o_p
        for ci in range(k_c):
            g = j * children_per_root + ci
            m = ccounts[ci]
            if m == 0:
                continue
            lo = torch.full((rank,), float("inf"), dtype=torch.float64, device=device)
            hi = torch.full((rank,), float("-inf"), dtype=torch.float64, device=device)
            rr = torch.zeros((), dtype=torch.float64, device=device)
            for a in range(cs, cs + m, sub):
                d = leaf[a:min(cs + m, a + sub)].double() - c64
                z = d @ Q64
                lo = torch.minimum(lo, z.min(dim=0).values)
                hi = torch.maximum(hi, z.max(dim=0).values)
                rr = torch.maximum(rr, (d - z @ Q64.T).norm(dim=1).max())
            out["child_intervals_l"][g] = _round_down_f32(lo - _EPS)
            out["child_intervals_u"][g] = _round_up_f32(hi + _EPS)
            out["child_radii"][g] = _round_up_f32(rr + _EPS)
            out["leaf_offsets"][g] = cs
            out["leaf_sizes"][g] = m
            cs += m
    return out


def build_circuit_index_streaming(rows_fn, n: int, dim: int, num_roots: int, children_per_root: int, rank: int,
                                  random_state: int = 42, device: str = "cuda", chunk: int = 1 << 18,
                                  sample: int = 1 << 19, shard_rank: int = 0, world: int = 1, group=None,
                                  max_imbalance: float = 1.05, block_rows: int = 64) -> CircuitIndex:
    """Build an index over a corpus too large to hold twice, or this rank's
    shard of it: ``rows_fn(start, stop)`` must return rows [start, stop)
    deterministically (as the seeded generators of circuit_rag.synthetic do).

    1. Root centres: k-means on the first ``sample`` rows (rank 0; broadcast
       to the other ranks).
    2. Root of every row (max inner product): each rank labels its 1/world of
       the rows and the labels are all-gathered, so every rank sees the same
       assignment.
    3. Shard plan (circuit_plan_shard_parts over blocks of ``block_rows`` rows
       of each root, in row order): whole roots, largest first, to the
       least-loaded rank; a root that does not fit within ``max_imbalance`` x
       the mean shard is cut into contiguous row ranges (parts), each becoming a
       root of its rank's index with the same centre.  world = 1: one part per
       root, the whole corpus.
    4. Second generation pass: every rank scatters the rows of its parts
       straight into their part-major slots.
    5. Per part: PCA basis, k-means children, certificates in float64
       (exact for the stored float32 data, as in build_circuit_index).

    The returned index holds this rank's parts only; ``original_ids`` are
    global row numbers; ``shard_info`` records the plan."""
    if not 1 <= rank <= MAX_RANK:
        raise ValueError(f"rank must be in [1, {MAX_RANK}]")
    if world > 1:
        import torch.distributed as dist
    gen = torch.Generator(device="cpu")
    gen.manual_seed(random_state)
    allow = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True  # assignments only pick clusters; certificates are fp64
    try:
        # 1. root centres
        if shard_rank == 0:
            S = rows_fn(0, min(sample, n)).to(device)
            centers = _kmeans(S, num_roots, 8, gen)
            del S
        else:
            centers = torch.empty((num_roots, dim), dtype=torch.float32, device=device)
        if world > 1:
            dist.broadcast(centers, 0, group=group)
        # 2. labels: this rank's slice, then all-gathered
        per = (n + world - 1) // world
        lo_r, hi_r = min(n, shard_rank * per), min(n, (shard_rank + 1) * per)
        mine = torch.full((per,), -1, dtype=torch.int32, device=device)
        for s in range(lo_r, hi_r, chunk):
            e = min(hi_r, s + chunk)
            mine[s - lo_r:e - lo_r] = _assign(rows_fn(s, e).to(device), centers).to(torch.int32)
        if world > 1:
            labels = torch.empty(per * world, dtype=torch.int32, device=device)
            dist.all_gather_into_tensor(labels, mine, group=group)
            labels = labels[:n]
        else:
            labels = mine[:n]
        del mine
        counts = torch.bincount(labels.long(), minlength=num_roots)
        root_start = torch.cumsum(counts, 0) - counts
        # 3. plan over blocks of rows of each root (host, identical on every rank)
        from circuit_rag.shard import plan_shard_parts

        counts_h = counts.cpu().numpy().astype(np.int64)
        nblk = (counts_h + block_rows - 1) // block_rows
        atom_ptr = np.concatenate([[0], np.cumsum(nblk)]).astype(np.int64)
        atom_rows = np.full(int(atom_ptr[-1]), block_rows, dtype=np.int64)
        last = atom_ptr[1:] - 1
        has = nblk > 0
        atom_rows[last[has]] = counts_h[has] - (nblk[has] - 1) * block_rows
        plan = plan_shard_parts(atom_rows, atom_ptr, world, max_imbalance)
        own = np.nonzero(plan["part_rank"] == shard_rank)[0]
        part_root = plan["part_root"][own]
        # rows of part j: positions [r0, r1) among its root's rows (row order)
        r0 = (plan["part_atom_begin"][own] - atom_ptr[part_root]) * block_rows
        r1 = np.minimum((plan["part_atom_end"][own] - atom_ptr[part_root]) * block_rows, counts_h[part_root])
        part_off = np.concatenate([[0], np.cumsum(r1 - r0)]).astype(np.int64)
        n_own = int(part_off[-1])
        # 4. slot of every owned row: the rows of root p in row order are
        # order[root_start[p] : root_start[p] + counts[p]]
        order = torch.argsort(labels, stable=True)
        del labels
        slot = torch.full((n,), -1, dtype=torch.int64, device=device)
        for j in range(len(own)):
            a = int(root_start[int(part_root[j])]) + int(r0[j])
            b = a + int(r1[j] - r0[j])
            slot[order[a:b]] = torch.arange(int(part_off[j]), int(part_off[j + 1]), device=device)
        del order
        leaf = torch.empty((n_own, dim), dtype=torch.float32, device=device)
        orig = torch.empty(n_own, dtype=torch.int32, device=device)
        for s in range(0, n, chunk):
            e = min(n, s + chunk)
            sl = slot[s:e]
            keep = torch.nonzero(sl >= 0).flatten()
            if keep.numel() == 0:
                continue
            X = rows_fn(s, e).to(device)
            leaf[sl[keep]] = X[keep]
            orig[sl[keep]] = (keep + s).to(torch.int32)
        del slot
        # 5. per part: basis, children, certificates
        arrays = _part_hierarchy(leaf, orig, part_off, part_root, centers, children_per_root, rank, random_state,
                                 device)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = allow
    idx = CircuitIndex(leaf_vectors=leaf, original_ids=orig, dim=dim, rank=rank, device=device, **arrays)
    idx.shard_info = {"rank": shard_rank, "world": world, "part_root": part_root.tolist(),
                      "rows": n_own, "rank_rows": plan["rank_rows"].tolist(),
                      "parts_total": int(len(plan["part_root"])), "roots": num_roots}
    return idx
