"""Edge cases of the device path against the oracle: zero right-hand side,
maxiter 0, a 1 x 1 system, rows without entries, duplicate COO entries,
rectangular and empty SpMV, a last slice with a single row."""
import warnings

import pytest
import torch

from oracle import krylov as K
import torch_sla_b200 as T
from torch_sla_b200 import problems as P
from torch_sla_b200.backends import pytorch_backend as PB

pytestmark = pytest.mark.gpu


def cu(*ts, dev):
    return [t.to(dev) for t in ts]


def test_zero_rhs(dev):
    """b = 0: with atol > 0 the start-of-iteration test stops at iteration 0
    with x = 0; with atol = 0 the reference divides 0 by 0, reports maxiter
    iterations and returns NaN -- the device path does the same (it stops
    early on the non-finite residual but reports maxiter)."""
    v, r, c, sh = P.poisson_3d_7pt(9)
    b = torch.zeros(sh[0], dtype=torch.float64)
    xo, ito, _, _ = K.pcg(v, r, c, sh, b, atol=1e-10, rtol=1e-8)
    res = T.pcg_solve_fused(*cu(v, r, c, dev=dev), sh, b.to(dev), atol=1e-10, rtol=1e-8)
    assert ito == 0 and res.num_iters == 0 and res.converged
    assert torch.equal(res.x.cpu(), xo)
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        xo, ito, _, conv = K.pcg(v, r, c, sh, b, atol=0.0, rtol=1e-8, maxiter=300)
        res = T.pcg_solve_fused(*cu(v, r, c, dev=dev), sh, b.to(dev), atol=0.0, rtol=1e-8,
                                maxiter=300)
    assert ito == 300 and res.num_iters == 300 and not conv and not res.converged
    assert bool(torch.isnan(xo).all()) and bool(torch.isnan(res.x).all())


def test_maxiter_zero_returns_start(dev):
    v, r, c, sh = P.poisson_2d_5pt(12)
    b = P.rhs_normal(sh[0], 2)
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        res = T.pcg_solve_fused(*cu(v, r, c, dev=dev), sh, b.to(dev), atol=0.0, rtol=1e-8,
                                maxiter=0)
    assert res.num_iters == 0 and not res.converged
    assert torch.count_nonzero(res.x) == 0


def test_one_by_one_system(dev):
    v = torch.tensor([4.0], dtype=torch.float64)
    r = torch.tensor([0])
    c = torch.tensor([0])
    b = torch.tensor([2.0], dtype=torch.float64)
    xo, ito, _, _ = K.pcg(v, r, c, (1, 1), b, atol=0.0, rtol=1e-12)
    res = T.pcg_solve_fused(*cu(v, r, c, dev=dev), (1, 1), b.to(dev), atol=0.0, rtol=1e-12)
    assert res.num_iters == ito and torch.equal(res.x.cpu(), xo)


def test_duplicates_summed_and_empty_rows_in_spmv(dev):
    g = torch.Generator().manual_seed(11)
    n = 70  # rows 0..69, rows 60..69 without entries; last slice holds 6 rows
    r = torch.randint(0, 60, (900,), generator=g)
    c = torch.randint(0, n, (900,), generator=g)
    r = torch.cat([r, r[:100]])  # exact duplicates
    c = torch.cat([c, c[:100]])
    v = torch.randn(r.numel(), generator=g, dtype=torch.float64)
    x = torch.randn(n, generator=g, dtype=torch.float64)
    y = T.SparseTensor(*cu(v, r, c, dev=dev), (n, n)) @ x.to(dev)
    yo = K.spmv(v, r, c, (n, n), x)
    assert float((y.cpu() - yo).abs().max() / yo.abs().max()) < 1e-13
    assert torch.count_nonzero(y[60:]) == 0


def test_rectangular_and_empty_spmv(dev):
    g = torch.Generator().manual_seed(12)
    r = torch.randint(0, 33, (400,), generator=g)
    c = torch.randint(0, 1000, (400,), generator=g)
    v = torch.randn(400, generator=g, dtype=torch.float64)
    x = torch.randn(1000, generator=g, dtype=torch.float64)
    y = T.SparseTensor(*cu(v, r, c, dev=dev), (33, 1000)) @ x.to(dev)
    yo = K.spmv(v, r, c, (33, 1000), x)
    assert y.shape == (33,)
    assert float((y.cpu() - yo).abs().max() / yo.abs().max()) < 1e-13
    e = torch.zeros(0, dtype=torch.int64)
    y0 = T.SparseTensor(torch.zeros(0, dtype=torch.float64, device=dev), e.to(dev), e.to(dev),
                        (5, 5)) @ torch.ones(5, dtype=torch.float64, device=dev)
    assert torch.count_nonzero(y0) == 0


def test_single_row_last_slice_pcg(dev):
    """n = 32k + 1: the last SELL slice holds one real row."""
    v, r, c, sh = P.poisson_2d_5pt(33)  # 1089 = 34 * 32 + 1
    b = P.rhs_normal(sh[0], 4)
    xo, ito, _, _ = K.pcg(v, r, c, sh, b, atol=0.0, rtol=1e-10)
    A = PB.CachedSparseMatrix(*cu(v, r, c, dev=dev), sh)
    M = PB.get_preconditioner(A, "jacobi")
    for flags in (1, 2):  # streamed, persistent
        x, info = PB._pcg_core(A, b.to(dev), None, M.dinv, 0.0, 1e-10, 5000, flags=flags)
        assert abs(info.iterations - ito) <= 1
        assert float((x.cpu() - xo).norm() / xo.norm()) < 1e-8
