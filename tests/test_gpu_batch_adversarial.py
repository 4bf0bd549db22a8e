"""Adversarial parity test of the batched path's tf32 error band.

The batched scan filters rows with tf32 tensor-core scores and keeps every row
within band = 2 eps of the running k-th best, with
eps = (2^-9 + 2^-20 + 2 D 2^-23 + gamma_D) ||q|| max||x|| (1 % padding); the
kept rows are rescored exactly in fp32.  These inputs push the tf32 error
towards that bound and crowd the top-k boundary:

* every query and most rows have their 13 low mantissa bits set, the bits the
  tensor cores drop (maximal truncation, coherent when a row is aligned with
  the query);
* rows that are exact in tf32 (low bits clear) are interleaved with them around
  the k-th best, so the running threshold comes from rows without error while
  rows of the true top-k carry the largest underestimate;
* near-duplicates of the k-th row one ulp apart in one component;
* both signs, D in {384, 2048}, k in {10, 100}, and a second regime with row
  norms spread over 1e-3 .. 1e3 (the largest rows hold the top-k).

Every query must equal circuit_search bit for bit and pass the oracle rule.
The test also measures the operand-truncation error the band has to cover
(tf32 operands emulated by clearing the 13 low mantissa bits, products summed
in float64) relative to ||q|| max||x||, and checks it against the band's
first term."""
import math

import numpy as np
import pytest
import torch

from circuit_rag import build_circuit_index, circuit_search, circuit_search_batch
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"
U = 2.0 ** -24


def _set_low_bits(t):
    return (t.contiguous().view(torch.int32) | 0x1FFF).view(torch.float32)


def _clear_low_bits(t):
    return (t.contiguous().view(torch.int32) & ~0x1FFF).view(torch.float32)


def _unit(n, d, g):
    x = torch.randn(n, d, generator=g, dtype=torch.float64)
    return x / x.norm(dim=1, keepdim=True)


def _planted(Q, per_query, d, g, width, norm):
    """Rows at cosines within `width` of 0.9 to each query, half with maximal
    truncation, half exact in tf32, scaled to `norm`."""
    out = []
    for q in Q.double():
        qh = q / q.norm()
        r = _unit(per_query, d, g)
        r = r - (r @ qh)[:, None] * qh[None, :]
        r = r / r.norm(dim=1, keepdim=True)
        c = 0.9 + width * (torch.rand(per_query, generator=g, dtype=torch.float64) - 0.5)
        x = (c[:, None] * qh[None, :] + torch.sqrt(1 - c * c)[:, None] * r) * norm
        x = x.float()
        half = per_query // 2
        out.append(_set_low_bits(x[:half]))
        out.append(_clear_low_bits(x[half:]))
    return torch.cat(out)


def _near_duplicates(X, Q, k):
    """For each query, copies of its k-th best row with the last mantissa bit of
    one component flipped (scores one ulp apart or tied)."""
    exact = Q.double() @ X.double().T
    kth_rows = torch.topk(exact, k, dim=1).indices[:, -1]
    dups = []
    for r in kth_rows.tolist():
        base = X[r].clone()
        for j in range(4):
            y = base.clone().view(torch.int32)
            y[j] ^= 1
            dups.append(y.view(torch.float32))
    return torch.stack(dups)


def _measured_error(X, Q):
    """max over (query, row) of |tf32 - exact| / (||q|| max||x||) with tf32
    operands emulated by truncation and the products summed in float64."""
    exact = Q.double() @ X.double().T
    scale = Q.double().norm(dim=1)[:, None] * X.double().norm(dim=1).max()
    emul = _clear_low_bits(Q).double() @ _clear_low_bits(X).double().T
    return float(((emul - exact).abs() / scale).max())


def _check(X, Q, k, index):
    scores, ids = circuit_search_batch(Q, index, k)
    exact = (Q.double() @ X.double().T).cpu().numpy()
    for b in range(Q.shape[0]):
        oracle.check_topk(exact[b], k, scores[b].cpu().numpy(), ids[b].cpu().numpy())
        s1, i1, _ = circuit_search(Q[b], index, k)
        assert torch.equal(scores[b], s1), (b, scores[b], s1)
        assert torch.equal(ids[b], i1), (b, ids[b], i1)


@pytest.mark.parametrize("dim", [384, 2048])
@pytest.mark.parametrize("k", [10, 100])
def test_tf32_band_unit_rows_crowded_boundary(dim, k):
    """Unit-norm rows (max||x|| = 1, the tightest band), signed queries of
    norms 0.1 .. 1, 4k planted rows per query around cosine 0.9."""
    g = torch.Generator().manual_seed(1000 * dim + k)
    nq = 12
    Q = _unit(nq, dim, g) * (10.0 ** (torch.rand(nq, 1, generator=g, dtype=torch.float64) - 1))
    Q = _set_low_bits(Q.float())
    Q[nq // 2:] = -Q[nq // 2:]
    # the band in score units is about 2 eps ~ 2^-8 ||q||: crowd the planted rows into a window of that width
    width = 4.0 * (2.0 ** -9 + 2 * dim * 2.0 ** -23)
    P = _planted(Q, 4 * k, dim, g, width, 1.0)
    B = _set_low_bits(_unit(3000, dim, g).float())
    X = torch.cat([P, B])
    X = torch.cat([X, _near_duplicates(X, Q, k)]).to(DEV)
    Qd = Q.to(DEV)
    index = build_circuit_index(X, num_roots=8, children_per_root=4, rank=8, device=DEV)
    _check(X, Qd, k, index)
    emul = _measured_error(X, Qd)
    bound = 2.0 ** -9 + 2.0 ** -20
    print(f"\n[tf32 band] D={dim} k={k} unit rows: max |tf32 - exact| / (||q|| max||x||) with truncated "
          f"operands {emul:.3e}; band's truncation term {bound:.3e}, "
          f"full eps/(||q|| max||x||) {bound + 2 * dim * 2.0 ** -23 + dim * U / (1 - dim * U):.3e}")
    assert emul <= bound


@pytest.mark.parametrize("dim", [384, 2048])
def test_tf32_band_norms_spread(dim):
    """Row norms 10^U(-3, 3); the top-k is held by planted rows of norm 1e3
    (the largest), queries of norm 1e-3 keep scores near 1."""
    g = torch.Generator().manual_seed(7 * dim)
    k, nq = 10, 12
    Q = _set_low_bits((_unit(nq, dim, g) * 1e-3).float())
    Q[::2] = -Q[::2]
    width = 4.0 * (2.0 ** -9 + 2 * dim * 2.0 ** -23)
    P = _planted(Q, 4 * k, dim, g, width, 1e3)
    n_bg = 4000
    B = _unit(n_bg, dim, g) * (10.0 ** (torch.rand(n_bg, 1, generator=g, dtype=torch.float64) * 6 - 3))
    B = _set_low_bits(B.float())
    X = torch.cat([P, B])
    X = torch.cat([X, _near_duplicates(X, Q, k)]).to(DEV)
    Qd = Q.to(DEV)
    index = build_circuit_index(X, num_roots=8, children_per_root=4, rank=8, device=DEV)
    _check(X, Qd, k, index)
    emul = _measured_error(X, Qd)
    bound = 2.0 ** -9 + 2.0 ** -20
    print(f"\n[tf32 band] D={dim} k={k} norms 1e-3..1e3: max |tf32 - exact| / (||q|| max||x||) with truncated "
          f"operands {emul:.3e}; band's truncation term {bound:.3e}")
    assert emul <= bound
    assert math.isfinite(emul)
