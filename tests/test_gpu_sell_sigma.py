"""SELL-32-sigma views for irregular row lengths.

torch-sla's CSR SpMV serves any pattern (pytorch_backend.py:154-161). With
SELL-32 in row order, a slice is padded to its longest row, which costs
several times the stored entries when row lengths are skewed; sorting rows
by length inside windows of sigma rows (sla_sell_sigma_order) groups rows of
similar length. These tests use a seeded matrix with power-law row lengths
(problems.powerlaw_coo) and check: the device order against a host sort, the
SpMV on sorted and unsorted views (bitwise equal: every row is summed in the
same ascending-column order) and against the oracle (1e-13 fp64, 1e-5 fp32),
and the CG, BiCGStab and mixed-precision CG solvers on the sorted view
against the oracle (iterations within +-3 %)."""
import math
import warnings

import pytest
import torch

from oracle import krylov as K
import torch_sla_b200 as T
from torch_sla_b200 import _lib as L
from torch_sla_b200 import problems as P
from torch_sla_b200._csr import DeviceCSR, spmv
from torch_sla_b200.backends import pytorch_backend as PB

pytestmark = pytest.mark.gpu


def rel(a, b):
    a = a.detach().double().cpu()
    b = b.detach().double().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-300))


def iters_close(got, want):
    return abs(got - want) <= max(1, math.ceil(0.03 * want))


def host_order(rowptr, sigma):
    """Rows sorted by decreasing length inside windows of sigma, equal
    lengths in ascending order (a stable host sort), each full window
    rotated by (window index mod sigma/32) slices of 32 rows."""
    lens = (rowptr[1:] - rowptr[:-1]).long()
    n = lens.numel()
    out = []
    for w, w0 in enumerate(range(0, n, sigma)):
        seg = lens[w0:w0 + sigma]
        idx = torch.sort(-seg, stable=True).indices
        if seg.numel() == sigma:
            idx = torch.roll(idx, (w % (sigma // 32)) * 32)
        out.append(idx + w0)
    return torch.cat(out).to(torch.int32)


@pytest.mark.parametrize("n,sigma", [(50_000, 1024), (50_001, 32), (9_000, 4096)])
def test_sigma_order_matches_host_sort(dev, n, sigma):
    v, r, c, sh = P.powerlaw_coo(n, avg=12.0, seed=7, device=dev)
    csr = DeviceCSR(v, r, c, sh)
    got = csr.sigma_order(sigma).cpu()
    assert torch.equal(got, host_order(csr.rowptr.cpu(), sigma))


@pytest.mark.parametrize("dtype", [torch.float64, torch.float32])
def test_powerlaw_spmv_on_sigma_views(dev, dtype):
    n = 60_000
    v, r, c, sh = P.powerlaw_coo(n, avg=16.0, seed=5, dtype=dtype)
    x = P.rhs_normal(n, 1, dtype)
    y_ref = K.spmv(v, r, c, sh, x)
    csr = DeviceCSR(v.to(dev), r.to(dev), c.to(dev), sh)
    plain = csr.sell(sigma=1)
    auto = csr.sell()
    assert plain.sigma == 1 and auto.sigma > 1
    # the sorted view pads far less (power-law rows: several x in row order)
    assert auto.padded_nnz < 0.5 * plain.padded_nnz, (auto.padded_nnz, plain.padded_nnz)
    xd = x.to(dev)
    y1 = spmv(plain, xd, n)
    for sigma in (32, 1024, 4096):
        ys = spmv(csr.sell(sigma=sigma), xd, n)
        assert torch.equal(ys, y1), sigma
    assert torch.equal(spmv(auto, xd, n), y1)
    assert rel(y1, y_ref) <= (1e-13 if dtype == torch.float64 else 1e-5)


def test_stencil_explicit_view_keeps_row_order(dev):
    v, r, c, sh = P.poisson_3d_7pt(24, device=dev)
    assert DeviceCSR(v, r, c, sh).sell(diagonal=False).sigma == 1


@pytest.mark.parametrize("flags", [L.SLA_PCG_STREAMED, L.SLA_PCG_PERSISTENT])
def test_powerlaw_cg_on_sigma_view(dev, flags):
    n = 40_000
    v, r, c, sh = P.powerlaw_coo(n, avg=10.0, seed=3, spd=True)
    b = P.rhs_normal(n, 2)
    xo, ito, _, conv = K.pcg(v, r, c, sh, b, atol=0.0, rtol=1e-10, precond="jacobi")
    assert conv
    A = PB.CachedSparseMatrix(v.to(dev), r.to(dev), c.to(dev), sh)
    M = PB.get_preconditioner(A, "jacobi")
    bd = b.to(dev)
    sorted_view = A.csr.sell()
    assert sorted_view.sigma > 1
    xs, info_s = PB._pcg_core(A, bd, None, M.dinv, 0.0, 1e-10, 10000, flags, sell=sorted_view)
    xp, info_p = PB._pcg_core(A, bd, None, M.dinv, 0.0, 1e-10, 10000, flags,
                              sell=A.csr.sell(sigma=1))
    assert iters_close(info_s.iterations, ito), (info_s.iterations, ito)
    assert iters_close(info_p.iterations, ito), (info_p.iterations, ito)
    assert rel(xs, xo) < 1e-8 and rel(xp, xo) < 1e-8
    St = T.SparseTensor(v.to(dev), r.to(dev), c.to(dev), sh)
    assert float((bd - St @ xs).norm() / bd.norm()) < 2e-10


def test_powerlaw_bicgstab_on_sigma_view(dev):
    n = 40_000
    v, r, c, sh = P.powerlaw_coo(n, avg=10.0, seed=4)
    b = P.rhs_uniform01(n, 3)
    xo, ito, _ = K.pbicgstab(v, r, c, sh, b, atol=0.0, rtol=1e-9, precond="jacobi")[:3]
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        x, it, _ = T.pbicgstab_solve(v.to(dev), r.to(dev), c.to(dev), sh, b.to(dev), atol=0.0,
                                     rtol=1e-9, preconditioner="jacobi")
    # strongly diagonally dominant: a few tens of iterations, little room
    # for the summation order of the dots to move the count
    assert iters_close(it, ito), (it, ito)
    bd = b.to(dev)
    St = T.SparseTensor(v.to(dev), r.to(dev), c.to(dev), sh)
    assert float((bd - St @ x).norm() / bd.norm()) < 2e-9
    assert rel(x, xo) < 1e-8


def test_powerlaw_mixed_precision_on_sigma_view(dev):
    n = 40_000
    v, r, c, sh = P.powerlaw_coo(n, avg=10.0, seed=3, spd=True, dtype=torch.float32)
    b = P.rhs_normal(n, 2, torch.float32)
    xo, ito, _, conv, _ = K.pcg_mixed(v, r, c, sh, b, atol=0.0, rtol=1e-9, precond="jacobi")
    assert conv
    x = T.pytorch_solve(v.to(dev), r.to(dev), c.to(dev), sh, b.to(dev), method="cg", atol=0.0,
                        rtol=1e-9, preconditioner="jacobi", mixed_precision=True)
    it = PB.last_solve_info()["iterations"]
    assert abs(it - ito) <= 2, (it, ito)
    assert rel(x, xo) < 1e-6


@pytest.mark.parametrize("dtype", [torch.float64, torch.float32])
def test_powerlaw_hybrid_matvec(dev, dtype):
    """DeviceCSR.matvec on a power-law pattern: rows above the long-row
    threshold are summed by the warp-per-row CSR pass (lane-strided, then a
    fixed butterfly), the others by the SELL-32-sigma view. Short rows are
    bitwise those of the row-order view; every row agrees with the oracle
    (1e-13 fp64, 1e-5 fp32)."""
    n = 60_000
    v, r, c, sh = P.powerlaw_coo(n, avg=16.0, seed=5, dtype=dtype)
    x = P.rhs_normal(n, 1, dtype)
    y_ref = K.spmv(v, r, c, sh, x)
    csr = DeviceCSR(v.to(dev), r.to(dev), c.to(dev), sh)
    view = csr.spmv_view()
    assert view.long_rows is not None and 0 < view.long_rows.numel() < n // 10
    xd = x.to(dev)
    y = csr.matvec(xd)
    y1 = spmv(csr.sell(sigma=1), xd, n)
    short = torch.ones(n, dtype=torch.bool, device=dev)
    short[view.long_rows.long()] = False
    assert torch.equal(y[short], y1[short])
    assert rel(y, y_ref) <= (1e-13 if dtype == torch.float64 else 1e-5)
    # repeated calls are bitwise identical (fixed summation orders)
    assert torch.equal(csr.matvec(xd), y)
