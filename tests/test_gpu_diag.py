"""Diagonal-offset SELL views (no column array) against the explicit SELL
layout of the same matrix: same entries, same ascending-column summation
order, so SpMV results and whole solves must agree bit for bit."""
import pytest
import torch

import torch_sla_b200 as T
from oracle import krylov as K
from torch_sla_b200 import _lib as L
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


@pytest.mark.parametrize("grid", [(2, 5, 5), (20, 17, 33), (96, 96, 96)])
def test_fp32_spmv_views_across_sizes(dev, grid):
    """float32 SpMV on the diagonal-offset and explicit views of 7-point
    grids with 2, 351 and 27648 slices (fewer slices than warps, and several
    per warp with a ragged last step): the two views agree bit for bit and
    with the oracle within 1e-5."""
    v, r, c, sh = P.poisson_3d_7pt(grid)
    v = v.to(torch.float32)
    n = sh[0]
    x = P.rhs_normal(n, 9, torch.float32)
    y_ref = K.spmv(v, r, c, sh, x)
    csr = DeviceCSR(v.to(dev), r.to(dev), c.to(dev), sh)
    xd = x.to(dev)
    yd = spmv(csr.sell(diagonal=True), xd, n)
    ye = spmv(csr.sell(diagonal=False), xd, n)
    assert torch.equal(yd, ye)
    yr = yd.double().cpu()
    assert float((yr - y_ref.double()).abs().max() / y_ref.double().abs().max()) < 1e-5


@pytest.mark.parametrize("dtype,r0", [(torch.float64, 0), (torch.float32, 0),
                                      (torch.float32, 5)])
def test_diag_view_row_subset_bounded_columns(dev, dtype, r0):
    """A view of interior rows whose columns stay below n_cols (the shard
    interior case): rows with a column >= n_cols are left out. A run of rows
    starting at an odd row (row_base 5) puts the float32 two-rows-per-lane
    kernel's row pairs and gathers off 8-byte alignment."""
    v, r, c, sh = P.poisson_3d_7pt((10, 24, 24))  # 24 x 24 layers (padding ~5 %)
    csr = DeviceCSR(v.to(dtype).to(dev), r.to(dev), c.to(dev), sh)
    n_cols = 576 * 7  # first 7 z-layers
    rows = torch.arange(r0, 576 * 6, dtype=torch.int32, device=dev)  # never reach layer 7
    d = csr.sell(row_ids=rows, n_cols=n_cols)
    e = csr.sell(row_ids=rows, diagonal=False)
    assert d.diagonal_offsets and d.row_ids is None and d.row_base == r0
    x = P.rhs_normal(sh[0], 2, dtype).to(dev)
    yd = torch.zeros(sh[0], dtype=dtype, device=dev)
    ye = torch.zeros_like(yd)
    from torch_sla_b200 import _lib as L
    code = L.SLA_F64 if dtype == torch.float64 else L.SLA_F32
    for s, y in ((d, yd), (e, ye)):
        L.check("sla_spmv", L.lib().sla_spmv(code, s.ref(), L.ptr(x), L.ptr(y),
                                             L.stream_handle(dev)))
    assert torch.equal(yd, ye)
    assert float(yd[:r0].abs().sum()) == 0  # rows outside the view untouched


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


@pytest.mark.parametrize("grid", [(20, 17, 33), (16, 10, 7)])
def test_float32_pcg_two_rows_per_lane_views(dev, grid):
    """float32 PCG and mixed-precision PCG on 7-point grids whose slice
    count is odd (351 and 35: the last slice pair of the
    two-rows-per-lane K_A has one slice): the diagonal-offset and explicit
    views share the row-to-thread mapping, so the iterates agree bit for
    bit; the float32 solve stays within 1e-4 of the float64 solution and
    the mixed-precision one within 1e-6 of the oracle's mixed-precision
    PCG."""
    v, r, c, sh = P.poisson_3d_7pt(grid)
    b = P.rhs_normal(sh[0], 8)
    out, mixed = [], []
    for diagonal in (True, False):
        A = PB.CachedSparseMatrix(v.float().to(dev), r.to(dev), c.to(dev), sh)
        A.csr._sell = A.csr.sell(diagonal=diagonal)
        assert A.sell().diagonal_offsets == diagonal
        M = PB.get_preconditioner(A, "jacobi")
        x, info = PB._pcg_core(A, b.float().to(dev), None, M.dinv, 0.0, 1e-6, 5000,
                               flags=L.SLA_PCG_STREAMED)
        out.append((x, info.iterations))
        res = PB.pcg_solve_mixed_precision(A, b.float().to(dev), atol=0.0, rtol=1e-9,
                                           preconditioner=PB.Float32Preconditioner(M))
        mixed.append((res.x, res.num_iters))
    assert out[0][1] == out[1][1] and torch.equal(out[0][0], out[1][0])
    assert mixed[0][1] == mixed[1][1] and torch.equal(mixed[0][0], mixed[1][0])
    xo = K.pcg(v, r, c, sh, b, atol=0.0, rtol=1e-10, precond="jacobi")[0]
    e = float((out[0][0].double().cpu() - xo).abs().max() / xo.abs().max())
    assert e < 1e-4, e
    xm = K.pcg_mixed(v.float(), r, c, sh, b.float(), atol=0.0, rtol=1e-9, precond="jacobi")[0]
    em = float((mixed[0][0].cpu() - xm).abs().max() / xm.abs().max())
    assert em < 1e-6, em


def test_float32_two_rows_per_lane_permuted_view(dev):
    """A float32 7-point matrix on an explicit view of all rows in a seeded
    random order (row ids, uniform width 7): the two-rows-per-lane SpMV and
    K_A read each lane's rows through the row ids (no pair loads across
    non-adjacent rows). The SpMV gives the row-order view's sums bit for
    bit; float32 PCG on it reaches the same solution within float32
    rounding."""
    v, r, c, sh = P.poisson_3d_7pt((20, 17, 33))
    v = v.float()
    n = sh[0]
    csr = DeviceCSR(v.to(dev), r.to(dev), c.to(dev), sh)
    plain = csr.sell(diagonal=False, sigma=1)
    perm = torch.randperm(n, generator=torch.Generator().manual_seed(21)).to(torch.int32)
    shuf = csr.sell(row_ids=perm.to(dev), diagonal=False)
    assert shuf.row_ids is not None and shuf.uniform_width == 7 and plain.uniform_width == 7
    x = P.rhs_normal(n, 4, torch.float32).to(dev)
    assert torch.equal(spmv(shuf, x, n), spmv(plain, x, n))
    A = PB.CachedSparseMatrix(v.to(dev), r.to(dev), c.to(dev), sh)
    M = PB.get_preconditioner(A, "jacobi")
    b = P.rhs_normal(n, 5, torch.float32).to(dev)
    xs, info_s = PB._pcg_core(A, b, None, M.dinv, 0.0, 1e-6, 5000, L.SLA_PCG_STREAMED, sell=shuf)
    xp, info_p = PB._pcg_core(A, b, None, M.dinv, 0.0, 1e-6, 5000, L.SLA_PCG_STREAMED,
                              sell=plain)
    assert abs(info_s.iterations - info_p.iterations) <= 1
    assert float((xs - xp).abs().max() / xp.abs().max()) < 1e-4


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


@pytest.mark.parametrize("kind,dtype,k", [
    ("p3d", torch.float64, 16), ("p3d", torch.float64, 2), ("p3d", torch.float32, 16),
    ("p3d_big", torch.float64, 16), ("p3d_big", torch.float32, 64),
    ("p2d", torch.float64, 16), ("p2d", torch.float32, 4),
])
def test_staged_tile_multi_rhs_matches_csr(dev, kind, dtype, k):
    """Multi-RHS CG on 7-point (offsets -a,-b,-1,0,1,b,a) and 5-point
    (-b,-1,0,1,b) diagonal views runs the SpMM over P tiles staged in shared
    memory by bulk copies. Against the CSR kernels (gathers straight from
    global memory): same rows per thread and summation orders, so the same
    iterations per column and the same X. Shapes cover a partial last tile
    (20 x 17 x 33 = 11220 rows), several tiles per block with both staging
    buffers cycling (48^3), 2 to 64 columns (512 to 16 rows per tile) and
    both precisions."""
    if kind == "p3d":
        v, r, c, sh = P.poisson_3d_7pt((20, 17, 33))
    elif kind == "p3d_big":
        v, r, c, sh = P.poisson_3d_7pt(48)
    else:
        v, r, c, sh = P.poisson_2d_5pt(75)
    v = v.to(dtype)
    g = torch.Generator().manual_seed(11)
    B = torch.randn(sh[0], k, generator=g, dtype=torch.float64).to(dtype).to(dev)
    rtol = 1e-10 if dtype == torch.float64 else 1e-5
    out = []
    for diagonal in (True, False):
        A = PB.CachedSparseMatrix(v.to(dev), r.to(dev), c.to(dev), sh)
        A.csr._sell = A.csr.sell(diagonal=diagonal)
        assert A.csr._sell.diagonal_offsets == diagonal
        res = PB.batched_pcg_solve(A, B, atol=0.0, rtol=rtol,
                                   preconditioner=PB.get_preconditioner(A, "jacobi"))
        out.append(res)
    assert bool(out[0].converged.all())
    assert torch.equal(out[0].num_iters, out[1].num_iters)
    assert float((out[0].X - out[1].X).abs().max()) == 0.0
    St = T.SparseTensor(v.to(dev), r.to(dev), c.to(dev), sh)
    R = B.double() - torch.stack([(St @ out[0].X[:, j]).double() for j in range(k)], 1)
    # float32: the true residual sits above the recursive one by the float32
    # rounding of the updates
    tol = 2 * rtol if dtype == torch.float64 else 20 * rtol
    assert float((R.norm(dim=0) / B.double().norm(dim=0)).max()) < tol


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
