"""Diagonal-offset SELL views (no column array) against the explicit SELL
layout of the same matrix: same entries, same ascending-column summation
order, so SpMV results and whole solves must agree bit for bit."""
import pytest
import torch

import torch_sla_b200 as T
from torch_sla_b200 import problems as P
from torch_sla_b200._csr import DeviceCSR, spmv
from torch_sla_b200.backends import pytorch_backend as PB

pytestmark = pytest.mark.gpu


def _matrix(kind):
    if kind == "p3d":
        return P.poisson_3d_7pt((20, 17, 33))
    if kind == "p2d":
        return P.poisson_2d_5pt(40)
    if kind == "cd":
        return P.convdiff_3d_upwind(13)
    v, r, c = P.stencil27_rows((40, 40, 40), 0, 40, seed=4)
    return v, r, c, (64000, 64000)


@pytest.mark.parametrize("kind,width", [("p3d", 7), ("p2d", 5), ("cd", 7), ("s27", 27)])
@pytest.mark.parametrize("dtype", [torch.float64, torch.float32])
def test_diag_view_spmv_bitwise(dev, kind, width, dtype):
    v, r, c, sh = _matrix(kind)
    csr = DeviceCSR(v.to(dtype).to(dev), r.to(dev), c.to(dev), sh)
    d = csr.sell(diagonal=True)
    e = csr.sell(diagonal=False)
    assert d.diagonal_offsets and d.uniform_width == width and d.col is None
    assert not e.diagonal_offsets
    x = P.rhs_normal(sh[0], 5, dtype).to(dev)
    assert torch.equal(spmv(d, x, sh[0]), spmv(e, x, sh[0]))


def test_diag_view_row_subset_bounded_columns(dev):
    """A view of interior rows whose columns stay below n_cols (the shard
    interior case): rows with a column >= n_cols are left out."""
    v, r, c, sh = P.poisson_3d_7pt((10, 24, 24))  # 24 x 24 layers (padding ~5 %)
    csr = DeviceCSR(v.to(dev), r.to(dev), c.to(dev), sh)
    n_cols = 576 * 7  # first 7 z-layers
    rows = torch.arange(0, 576 * 6, dtype=torch.int32, device=dev)  # never reach layer 7
    d = csr.sell(row_ids=rows, n_cols=n_cols)
    e = csr.sell(row_ids=rows, diagonal=False)
    assert d.diagonal_offsets
    x = P.rhs_normal(sh[0], 2).to(dev)
    yd = torch.zeros(sh[0], dtype=torch.float64, device=dev)
    ye = torch.zeros_like(yd)
    from torch_sla_b200 import _lib as L
    for s, y in ((d, yd), (e, ye)):
        L.check("sla_spmv", L.lib().sla_spmv(L.SLA_F64, s.ref(), L.ptr(x), L.ptr(y),
                                             L.stream_handle(dev)))
    assert torch.equal(yd, ye)


def test_scattered_pattern_keeps_explicit_columns(dev):
    g = torch.Generator().manual_seed(9)
    n, nnz = 500, 6000
    r = torch.randint(0, n, (nnz,), generator=g)
    c = torch.randint(0, n, (nnz,), generator=g)
    v = torch.randn(nnz, generator=g, dtype=torch.float64)
    csr = DeviceCSR(v.to(dev), r.to(dev), c.to(dev), (n, n))
    assert not csr.sell().diagonal_offsets


@pytest.mark.parametrize("flags", [1, 2])  # streamed, persistent
@pytest.mark.parametrize("kind", ["p3d", "p2d", "s27"])
def test_diag_view_pcg_bitwise(dev, kind, flags):
    v, r, c, sh = _matrix(kind)
    b = P.rhs_normal(sh[0], 7).to(dev)
    out = []
    for diagonal in (True, False):
        A = PB.CachedSparseMatrix(v.to(dev), r.to(dev), c.to(dev), sh)
        A.csr._sell = A.csr.sell(diagonal=diagonal)
        assert A.sell().diagonal_offsets == diagonal
        M = PB.get_preconditioner(A, "jacobi")
        x, info = PB._pcg_core(A, b, None, M.dinv, 0.0, 1e-10, 5000, flags=flags)
        out.append((x, info.iterations))
    assert out[0][1] == out[1][1]
    assert torch.equal(out[0][0], out[1][0])


def test_diag_view_bicgstab_bitwise(dev):
    v, r, c, sh = _matrix("cd")
    b = P.rhs_uniform01(sh[0], 3).to(dev)
    out = []
    for diagonal in (True, False):
        A = PB.CachedSparseMatrix(v.to(dev), r.to(dev), c.to(dev), sh)
        A.csr._sell = A.csr.sell(diagonal=diagonal)
        M = PB.get_preconditioner(A, "jacobi")
        x, info = PB._bicgstab_core(A, b, None, M.dinv, 0.0, 1e-8, 5000)
        out.append((x, info.iterations))
    assert out[0][1] == out[1][1]
    assert torch.equal(out[0][0], out[1][0])


def test_diag_view_multi_rhs_matches_csr(dev):
    """Multi-RHS CG on the diagonal-offset view (columns computed) against
    the CSR kernels: same iterations per column, same X up to zero signs."""
    v, r, c, sh = P.poisson_3d_7pt(14)
    g = torch.Generator().manual_seed(8)
    B = torch.randn(sh[0], 16, generator=g, dtype=torch.float64).to(dev)
    out = []
    for diagonal in (True, False):
        A = PB.CachedSparseMatrix(v.to(dev), r.to(dev), c.to(dev), sh)
        A.csr._sell = A.csr.sell(diagonal=diagonal)
        res = PB.batched_pcg_solve(A, B, atol=0.0, rtol=1e-10,
                                   preconditioner=PB.get_preconditioner(A, "jacobi"))
        out.append(res)
    assert torch.equal(out[0].num_iters, out[1].num_iters)
    assert float((out[0].X - out[1].X).abs().max()) == 0.0


def test_diag_view_batched_matches_csr(dev, monkeypatch):
    """Batched same-pattern CG with values in the diagonal-offset order
    against the CSR kernels: same iterations, same X up to zero signs."""
    from torch_sla_b200._csr import DeviceCSR as DC
    vb, r, c, sh, bb = P.diffusion_2d_batched(8, 40, seed=2)
    args = (vb.to(dev), r.to(dev), c.to(dev), sh, bb.to(dev))
    X_diag, info_diag = PB.batched_cg_same_pattern_info(*args, atol=0.0, rtol=1e-10)
    assert DC(None, r.to(dev), c.to(dev), sh, keep_map=True,
              dtype=torch.float64).diag_pattern() is not None
    monkeypatch.setattr(DC, "diag_pattern", lambda self: None)
    X_csr, info_csr = PB.batched_cg_same_pattern_info(*args, atol=0.0, rtol=1e-10)
    assert info_diag.iterations == info_csr.iterations
    assert float((X_diag - X_csr).abs().max()) == 0.0
