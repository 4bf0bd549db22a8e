"""Seeded synthetic corpora and queries for the benchmark workloads.

Deterministic per row chunk: rows [i*CHUNK, (i+1)*CHUNK) are always drawn as a
whole from a generator seeded by (seed, i), so any row range (a shard, a CPU
subset) can be regenerated without producing the rest, with identical values.  Values depend on the device the
generator runs on (torch's CPU and CUDA generators differ); tests that compare
devices generate once and copy.

Workloads (N x D, float32, unit norm):
  clustered : n_centers centres uniform on the sphere; x = c + sigma * N(0, I),
              renormalised; cluster sizes equal (row i -> centre i % n_centers)
              or Zipf(s) (inverse CDF of a per-row uniform).
  spread    : per-dimension std proportional to i^-0.5 (i = 1..D), the noise
              rescaled to norm 0.6, plus a shared mean direction of norm 0.6,
              renormalised (mean pairwise cosine about 0.5).
  mixed     : half clustered (Zipf), half spread, interleaved by row parity.
  reftest   : the reference's exactness-test corpus (tests/test_exact.py:9-14):
              n_centers Gaussian (non-unit) centres, random labels, sigma = 0.3
              per dimension, renormalised; numpy generators seeded 0 (corpus)
              and 1 (query row indices, tests/test_exact.py:19); queries are
              corpus rows, as in that test.
"""
from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch

CHUNK = 1 << 16  # rows per generator chunk; a chunk is always drawn whole


def _gen(seed: int, chunk: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed((seed * 1_000_003 + chunk * 7919 + 17) % (2 ** 63 - 1))
    return g


def sphere(n: int, dim: int, seed: int, device="cpu") -> torch.Tensor:
    g = _gen(seed, 0, device)
    c = torch.randn(n, dim, generator=g, device=device)
    return c / c.norm(dim=1, keepdim=True)


def zipf_cdf(n_centers: int, s: float, device="cpu") -> torch.Tensor:
    w = torch.arange(1, n_centers + 1, dtype=torch.float64, device=device).pow(-s)
    return torch.cumsum(w / w.sum(), 0)


def _chunks(start: int, stop: int):
    c = start // CHUNK
    while c * CHUNK < stop:
        lo, hi = max(start, c * CHUNK), min(stop, (c + 1) * CHUNK)
        yield c, lo, hi
        c += 1


def clustered(start: int, stop: int, dim: int, centers: torch.Tensor, sigma: float, seed: int,
              zipf_s: Optional[float] = None, device="cpu") -> torch.Tensor:
    """Rows [start, stop) of a clustered corpus around ``centers``."""
    out = torch.empty(stop - start, dim, device=device)
    cdf = zipf_cdf(centers.shape[0], zipf_s, device) if zipf_s else None
    for c, lo, hi in _chunks(start, stop):
        g = _gen(seed, c, device)
        full = CHUNK
        noise = torch.randn(full, dim, generator=g, device=device)
        u = torch.rand(full, generator=g, device=device, dtype=torch.float64)
        rows = torch.arange(c * CHUNK, c * CHUNK + full, device=device)
        if cdf is None:
            lab = rows % centers.shape[0]
        else:
            lab = torch.searchsorted(cdf, u).clamp_(max=centers.shape[0] - 1)
        x = centers[lab] + sigma * noise
        x = x / x.norm(dim=1, keepdim=True)
        out[lo - start:hi - start] = x[lo - c * CHUNK:hi - c * CHUNK]
    return out


def spread(start: int, stop: int, dim: int, seed: int, device="cpu") -> torch.Tensor:
    """Rows [start, stop) of the anisotropic spread corpus."""
    out = torch.empty(stop - start, dim, device=device)
    std = torch.arange(1, dim + 1, dtype=torch.float32, device=device).pow(-0.5)
    mean = sphere(1, dim, seed + 999, device)[0] * 0.6
    for c, lo, hi in _chunks(start, stop):
        g = _gen(seed, c, device)
        full = CHUNK
        z = torch.randn(full, dim, generator=g, device=device) * std
        z = z * (0.6 / z.norm(dim=1, keepdim=True))
        x = z + mean
        x = x / x.norm(dim=1, keepdim=True)
        out[lo - start:hi - start] = x[lo - c * CHUNK:hi - c * CHUNK]
    return out


def reftest(n: int, dim: int, n_centers: int, sigma: float, seed: int) -> torch.Tensor:
    """The whole reftest corpus (float32, unit rows, on the CPU)."""
    rng = np.random.default_rng(seed)
    centers = rng.normal(size=(n_centers, dim))
    x = centers[rng.integers(0, n_centers, n)] + sigma * rng.normal(size=(n, dim))
    return torch.from_numpy((x / np.linalg.norm(x, axis=1, keepdims=True)).astype(np.float32))


@dataclass(frozen=True)
class Workload:
    name: str
    n: int
    dim: int
    num_roots: int
    children_per_root: int
    rank: int
    k: int
    queries: int
    kind: str              # clustered | spread | mixed
    n_centers: int = 0
    sigma: float = 0.0
    zipf_s: Optional[float] = None
    seed: int = 0

    def corpus(self, start: int = 0, stop: Optional[int] = None, device="cpu") -> torch.Tensor:
        stop = self.n if stop is None else stop
        return self._rows(start, stop, self.seed, device)

    def query_batch(self, n: Optional[int] = None, device="cpu") -> torch.Tensor:
        """Queries drawn from the same law as the corpus (independent rows)."""
        n = self.queries if n is None else n
        if self.kind == "reftest":
            rows = np.random.default_rng(self.seed + 1).integers(0, self.n, n)
            return self.corpus(device="cpu")[torch.from_numpy(rows)].to(device)
        return self._rows(0, n, self.seed + 1, device)

    def _rows(self, start, stop, seed, device):
        if self.kind == "reftest":
            return reftest(self.n, self.dim, self.n_centers, self.sigma, seed)[start:stop].to(device)
        if self.kind == "spread":
            return spread(start, stop, self.dim, seed, device)
        centers = sphere(self.n_centers, self.dim, self.seed + 101, device)
        if self.kind == "clustered":
            return clustered(start, stop, self.dim, centers, self.sigma, seed, self.zipf_s, device)
        # mixed: even rows clustered, odd rows spread (half from each population)
        a = clustered(start, stop, self.dim, centers, self.sigma, seed, self.zipf_s, device)
        b = spread(start, stop, self.dim, seed + 55, device)
        rows = torch.arange(start, stop, device=device)
        return torch.where((rows % 2 == 0)[:, None], a, b)


WORKLOADS = {
    "clustered-50k": Workload("clustered-50k", 50_000, 128, 64, 16, 8, 10, 25, "clustered", 64, 0.05),
    # the reference's own exactness test (tests/test_exact.py:9-19): 40K x 128, R = 32 x 8, rank 8
    "reftest-40k": Workload("reftest-40k", 40_000, 128, 32, 8, 8, 10, 25, "reftest", 64, 0.3),
    # the clustered-50k law at 4M rows (2 GB): too large to stream whole while the bounds are computed
    "clustered-4m": Workload("clustered-4m", 4_000_000, 128, 64, 16, 8, 10, 25, "clustered", 64, 0.05),
    "spread-5k": Workload("spread-5k", 5_183, 384, 64, 16, 8, 10, 300, "spread"),
    "spread-200k": Workload("spread-200k", 200_000, 384, 128, 16, 8, 10, 1000, "spread"),
    "zipf-10m": Workload("zipf-10m", 10_000_000, 384, 256, 32, 16, 100, 1024, "clustered", 4096, 0.08, 1.1),
    "mixed-100m": Workload("mixed-100m", 100_000_000, 384, 1024, 32, 32, 10, 4096, "mixed", 16384, 0.1, 1.1),
}
