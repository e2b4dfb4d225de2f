"""GPU parity of the B200 kernels against the oracle and the reference
fixtures. Tolerances: SpMV 1e-13 relative (fp64) / 1e-5 (fp32); solves reach
the reference's stopping test with an iteration count within +-3%;
gradients within 1e-8 relative."""
import math
import warnings

import pytest
import torch

from conftest import case_inputs
from oracle import krylov as K
import torch_sla_b200 as T
from torch_sla_b200 import _lib as L
from torch_sla_b200 import problems as P
from torch_sla_b200._csr import DeviceCSR
from torch_sla_b200.backends import pytorch_backend as PB

pytestmark = pytest.mark.gpu


def rel(a, b):
    a = a.detach().double().cpu()
    b = b.detach().double().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-300))


def iters_close(got, want):
    return abs(got - want) <= max(1, math.ceil(0.03 * want))


def cu(*ts, dev):
    return [t.to(dev) for t in ts]


# ------------------------------------------------------------- CSR build
@pytest.mark.parametrize("n,nnz,long_row", [(300, 3000, 0), (64, 4000, 40), (10, 9000, 6000)])
def test_csr_build_matches_torch(dev, n, nnz, long_row):
    g = torch.Generator().manual_seed(n + nnz)
    r = torch.randint(0, n, (nnz,), generator=g)
    c = torch.randint(0, n, (nnz,), generator=g)
    if long_row:
        r[: long_row] = 3
    v = torch.randn(nnz, generator=g, dtype=torch.float64)
    ref = K.csr(v, r, c, (n, n))
    csr = DeviceCSR(*cu(v, r, c, dev=dev), (n, n))
    assert torch.equal(csr.rowptr.cpu().long(), ref.crow_indices())
    assert torch.equal(csr.colind.cpu().long(), ref.col_indices())
    assert rel(csr.vals, ref.values()) < 1e-14


@pytest.mark.parametrize("case", ["sorted", "sorted_gaps", "one_swap", "duplicate", "bad_index"])
def test_csr_build_sorted_input(dev, case):
    """COO whose (row, col) keys strictly increase takes the copy-through
    path; the same entries with one adjacent pair swapped, or with one
    duplicate, take the sort/merge path. Both must give torch's CSR, the
    identity maps (src_index[t] = t, seg_ptr[e] = e) on the sorted path, and
    an index outside the shape is refused on either."""
    g = torch.Generator().manual_seed(17)
    n = 500
    dense = torch.rand(n, n, generator=g) < 0.02
    if case == "sorted_gaps":
        dense[:7] = False       # empty leading rows
        dense[200:260] = False  # an empty run in the middle
        dense[-5:] = False      # empty trailing rows
    r, c = dense.nonzero(as_tuple=True)  # row-major: strictly increasing keys
    v = torch.randn(r.numel(), generator=g, dtype=torch.float64)
    if case == "one_swap":
        r, c, v = r.clone(), c.clone(), v.clone()
        r[[10, 11]], c[[10, 11]], v[[10, 11]] = r[[11, 10]], c[[11, 10]], v[[11, 10]]
    elif case == "duplicate":
        r, c = torch.cat([r, r[5:6]]), torch.cat([c, c[5:6]])
        v = torch.cat([v, torch.tensor([0.25], dtype=torch.float64)])
    elif case == "bad_index":
        c = c.clone()
        c[-1] = n
        with pytest.raises(ValueError):
            DeviceCSR(*cu(v, r, c, dev=dev), (n, n))
        return
    ref = K.csr(v, r, c, (n, n))
    csr = DeviceCSR(*cu(v, r, c, dev=dev), (n, n), keep_map=True)
    assert torch.equal(csr.rowptr.cpu().long(), ref.crow_indices())
    assert torch.equal(csr.colind.cpu().long(), ref.col_indices())
    assert rel(csr.vals, ref.values()) < 1e-15
    if case in ("sorted", "sorted_gaps"):
        m = r.numel()
        assert torch.equal(csr.src_index.cpu(), torch.arange(m))
        assert torch.equal(csr.seg_ptr.cpu().long(), torch.arange(m + 1))


def test_csr_build_rejects_bad_index(dev):
    r = torch.tensor([0, 1, 5], device=dev)
    c = torch.tensor([0, 1, 1], device=dev)
    v = torch.ones(3, dtype=torch.float64, device=dev)
    with pytest.raises(ValueError):
        DeviceCSR(v, r, c, (3, 3))


def test_cpu_tensors_raise_no_fallback():
    v, r, c, sh = P.poisson_2d_5pt(8)
    with pytest.raises(RuntimeError, match="GPU"):
        T.pytorch_solve(v, r, c, sh, torch.ones(64, dtype=torch.float64))


# ------------------------------------------------------------------- SpMV
def test_spmv_golden_fp64_fp32(dev, golden):
    case = golden["spmv_rand50"]
    A = T.SparseTensor(*cu(case["val"], case["row"], case["col"], dev=dev), case["shape"])
    assert rel(A @ case["x"].to(dev), case["y"]) < 1e-13
    Af = T.SparseTensor(*cu(case["val"].float(), case["row"], case["col"], dev=dev), case["shape"])
    assert rel(Af @ case["x"].float().to(dev), case["y_f32"]) < 1e-5


@pytest.mark.parametrize("gen", ["p3d", "s27", "cd"])
@pytest.mark.parametrize("dtype", [torch.float64, torch.float32])
def test_spmv_vs_oracle(dev, gen, dtype):
    if gen == "p3d":
        v, r, c, sh = P.poisson_3d_7pt((20, 17, 33))
    elif gen == "s27":
        v, r, c = P.stencil27_rows((9, 8, 7), 0, 9)
        sh = (504, 504)
    else:
        v, r, c, sh = P.convdiff_3d_upwind(13)
    x = P.rhs_normal(sh[0], 3)
    y_ref = K.spmv(v.to(dtype), r, c, sh, x.to(dtype))
    y = T.SparseTensor(*cu(v.to(dtype), r, c, dev=dev), sh) @ x.to(dtype).to(dev)
    assert rel(y, y_ref) < (1e-13 if dtype == torch.float64 else 1e-5)


def test_spmv_full_256cube_stencil_identity(dev):
    """7-point 256^3 SpMV against the stencil written with shifted views."""
    m = 256
    v, r, c, sh = P.poisson_3d_7pt(m, device=dev)
    x = P.rhs_normal(sh[0], 1).to(dev)
    y = T.SparseTensor(v, r, c, sh) @ x
    X = x.view(m, m, m)
    Y = 6 * X
    Y[1:] -= X[:-1]; Y[:-1] -= X[1:]
    Y[:, 1:] -= X[:, :-1]; Y[:, :-1] -= X[:, 1:]
    Y[:, :, 1:] -= X[:, :, :-1]; Y[:, :, :-1] -= X[:, :, 1:]
    assert rel(y, Y.reshape(-1)) < 1e-13


def test_spmv_autograd(dev):
    v, r, c, sh = P.convdiff_3d_upwind(5)
    x = P.rhs_normal(sh[0], 2)
    vv = v.clone().to(dev).requires_grad_(True)
    xx = x.clone().to(dev).requires_grad_(True)
    y = T.SparseTensor(vv, r.to(dev), c.to(dev), sh) @ xx
    (y * y).sum().backward()
    vr = v.clone().requires_grad_(True)
    xr = x.clone().requires_grad_(True)
    yr = torch.zeros(sh[0], dtype=torch.float64).index_add(0, r, vr * xr[c])
    (yr * yr).sum().backward()
    assert rel(xx.grad, xr.grad) < 1e-13
    assert rel(vv.grad, vr.grad) < 1e-13


# -------------------------------------------------------------------- PCG
PCG_CASES = ["pcg_2d32_none", "pcg_3d16_jacobi", "pcg_3d16_jacobi_f32", "pcg_2d16_x0",
             "pcg_2d32_maxiter"]


@pytest.mark.parametrize("flags", [L.SLA_PCG_STREAMED, L.SLA_PCG_PERSISTENT, L.SLA_PCG_CLUSTER])
@pytest.mark.parametrize("name", PCG_CASES)
def test_pcg_matches_reference(dev, golden, name, flags):
    case = golden[name]
    v, r, c, sh = case_inputs(case)
    kw = dict(case["kw"])
    pc = kw.pop("preconditioner")
    A = PB.CachedSparseMatrix(*cu(v, r, c, dev=dev), sh)
    M = PB.get_preconditioner(A, pc)
    x0 = kw.pop("x0", None)
    x, info = PB._pcg_core(A, case["b"].to(dev), None if x0 is None else x0.to(dev), M.dinv,
                           kw["atol"], kw["rtol"], kw["maxiter"], flags)
    assert iters_close(info.iterations, case["iters"]), (info.iterations, case["iters"])
    assert (info.status == 0) == case["converged"]
    tol = 1e-4 if v.dtype == torch.float32 else 1e-7
    if case["converged"]:
        assert rel(x, case["x"]) < tol
    else:
        assert info.iterations == case["iters"] and rel(x, case["x"]) < 1e-10


def test_pcg_config1_full_size_persistent(dev, golden):
    ref = golden["pcg_2d256_none"]
    v, r, c, sh = P.poisson_2d_5pt(256, device=dev)
    b = P.rhs_uniform_pm1(sh[0], 0).to(dev)
    res = T.pcg_solve_fused(v, r, c, sh, b, atol=0.0, rtol=1e-10, maxiter=10000,
                            preconditioner="none")
    assert res.converged and iters_close(res.num_iters, ref["iters"])
    assert float(res.x.sum()) == pytest.approx(ref["x_sum"], rel=1e-7)
    true_res = (b - T.SparseTensor(v, r, c, sh) @ res.x).norm() / b.norm()
    assert float(true_res) < 2e-10


@pytest.mark.parametrize("flags", [L.SLA_PCG_CLUSTER, L.SLA_PCG_PERSISTENT])
def test_pcg_config1_full_size_small_system_kernels(dev, golden, flags):
    """The 2-D 256^2 system (plain CG, rtol 1e-10) on the thread-block-cluster
    kernel (values, search direction and partial sums in distributed shared
    memory) and on the cooperative-grid kernel."""
    ref = golden["pcg_2d256_none"]
    v, r, c, sh = P.poisson_2d_5pt(256, device=dev)
    b = P.rhs_uniform_pm1(sh[0], 0).to(dev)
    A = PB.CachedSparseMatrix(v, r, c, sh)
    x, info = PB._pcg_core(A, b, None, None, 0.0, 1e-10, 10000, flags)
    assert info.status == 0 and iters_close(info.iterations, ref["iters"]), info.iterations
    assert float(x.sum()) == pytest.approx(ref["x_sum"], rel=1e-7)
    true_res = (b - T.SparseTensor(v, r, c, sh) @ x).norm() / b.norm()
    assert float(true_res) < 2e-10
    x2, _ = PB._pcg_core(A, b, None, None, 0.0, 1e-10, 10000, flags)
    assert torch.equal(x, x2)  # deterministic: fixed summation order


@pytest.mark.parametrize("m", [100, 200, 203])
def test_pcg_cluster_partial_last_tile(dev, m):
    """n = m^2 not a multiple of the cluster's 16 x 32-row tiling: the last
    CTA holds row slots past n, which rows near n reach through their local
    gathers (with a zero value). Repeated solves, after kernels that leave
    other data in shared memory, must match the streamed path."""
    v, r, c, sh = P.poisson_2d_5pt(m, device=dev)
    b = P.rhs_uniform_pm1(sh[0], 0).to(dev)
    A = PB.CachedSparseMatrix(v, r, c, sh)
    xs, info_s = PB._pcg_core(A, b, None, None, 0.0, 1e-10, 10000, L.SLA_PCG_STREAMED)
    for _ in range(3):
        y = T.SparseTensor(v, r, c, sh) @ b  # other kernels in between
        xc, info_c = PB._pcg_core(A, b, None, None, 0.0, 1e-10, 10000, L.SLA_PCG_CLUSTER)
        assert info_c.status == 0 and iters_close(info_c.iterations, info_s.iterations)
        assert rel(xc, xs) < 1e-8 and bool(torch.isfinite(y).all())


def test_pcg_cluster_refuses_systems_that_do_not_fit(dev):
    """More rows than one cluster holds in shared memory: SLA_ERR_UNSUPPORTED
    with the cluster flag (AUTO then runs the cooperative-grid kernel)."""
    v, r, c, sh = P.poisson_3d_7pt(48, device=dev)  # 110,592 rows, 7 diagonals
    A = PB.CachedSparseMatrix(v, r, c, sh)
    b = P.rhs_normal(sh[0], 1).to(dev)
    with pytest.raises(L.SlaError) as e:
        PB._pcg_core(A, b, None, None, 0.0, 1e-8, 100, L.SLA_PCG_CLUSTER)
    assert e.value.status == L.SLA_ERR_UNSUPPORTED


def test_pcg_deterministic(dev):
    v, r, c, sh = P.poisson_3d_7pt(40, device=dev)
    b = P.rhs_normal(sh[0], 1).to(dev)
    A = PB.CachedSparseMatrix(v, r, c, sh)
    M = PB.get_preconditioner(A, "jacobi")
    xs = [PB._pcg_core(A, b, None, M.dinv, 0.0, 1e-8, 5000, L.SLA_PCG_STREAMED)[0] for _ in range(3)]
    assert torch.equal(xs[0], xs[1]) and torch.equal(xs[0], xs[2])


def test_pcg_nonconvergence_warns(dev):
    v, r, c, sh = P.poisson_2d_5pt(32, device=dev)
    b = P.rhs_uniform_pm1(sh[0], 0).to(dev)
    with pytest.warns(UserWarning, match="did not converge"):
        res = T.pcg_solve_fused(v, r, c, sh, b, atol=0.0, rtol=1e-10, maxiter=7)
    assert res.num_iters == 7 and not res.converged


# --------------------------------------------------------------- BiCGStab
@pytest.mark.parametrize("name", ["bicg_cd3d10_jacobi", "bicg_ad2d12_none", "bicg_ad2d12_maxiter"])
def test_bicgstab_matches_reference(dev, golden, name):
    case = golden[name]
    v, r, c, sh = case_inputs(case)
    kw = dict(case["kw"])
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        x, it, res = T.pbicgstab_solve(*cu(v, r, c, dev=dev), sh, case["b"].to(dev), **kw)
    assert iters_close(it, case["iters"]), (it, case["iters"])
    assert rel(x, case["x"]) < (1e-7 if it < kw["maxiter"] else 1e-10)


def rounding_envelope(fn, *args, seeds=4, **kw):
    """Iteration counts of the oracle under its own summation order and under
    `seeds` permuted summation orders of every inner product: BiCGStab's
    count moves by several iterations with the rounding of the dots alone
    (convdiff 24^3: 63..70 around the reference's 67)."""
    import oracle.krylov as KK
    counts = [fn(*args, **kw)[1]]
    orig = KK.torch.vdot
    n = args[4].numel()
    for s in range(seeds):
        perm = torch.randperm(n, generator=torch.Generator().manual_seed(s))
        KK.torch.vdot = lambda a, b, perm=perm: (a[perm] * b[perm]).sum()
        try:
            counts.append(fn(*args, **kw)[1])
        finally:
            KK.torch.vdot = orig
    return min(counts), max(counts), counts[0]


def test_bicgstab_vs_oracle_larger(dev):
    v, r, c, sh = P.convdiff_3d_upwind(24)
    b = P.rhs_uniform01(sh[0], 3)
    lo, hi, ito = rounding_envelope(K.pbicgstab, v, r, c, sh, b, atol=0.0, rtol=1e-8,
                                    precond="jacobi")
    xo = K.pbicgstab(v, r, c, sh, b, atol=0.0, rtol=1e-8, precond="jacobi")[0]
    x, it, res = T.pbicgstab_solve(*cu(v, r, c, dev=dev), sh, b.to(dev), atol=0.0, rtol=1e-8,
                                   preconditioner="jacobi")
    assert math.floor(0.97 * lo) <= it <= math.ceil(1.03 * hi), (it, lo, hi, ito)
    # both stop at ||r|| < 1e-8 ||b||; the true residual confirms it
    A = T.SparseTensor(*cu(v, r, c, dev=dev), sh)
    bd = b.to(dev)
    assert float((bd - A @ x).norm() / bd.norm()) < 2e-8
    assert rel(x, xo) < 1e-6


def test_bicgstab_guess_float32_and_views(dev):
    """K3 stores q = p - omega v for the next K1 (rounded as the reference's
    p - omega * v), so the first iteration must see q = 0 whatever x0 is.
    With an initial guess: iterations within the oracle's rounding envelope
    and the true residual at rtol. float32: the true residual at the float32
    floor. The diagonal-offset and explicit views of the matrix give the same
    iterates bit for bit (same sums, same orders)."""
    v, r, c, sh = P.convdiff_3d_upwind(16)
    b = P.rhs_uniform01(sh[0], 5)
    x0 = 0.1 * P.rhs_normal(sh[0], 6)
    lo, hi, _ = rounding_envelope(K.pbicgstab, v, r, c, sh, b, x0=x0, atol=0.0, rtol=1e-9,
                                  precond="jacobi")
    x, it, _ = T.pbicgstab_solve(*cu(v, r, c, dev=dev), sh, b.to(dev), x0=x0.to(dev), atol=0.0,
                                 rtol=1e-9, preconditioner="jacobi")
    assert math.floor(0.97 * lo) <= it <= math.ceil(1.03 * hi), (it, lo, hi)
    A = T.SparseTensor(*cu(v, r, c, dev=dev), sh)
    bd = b.to(dev)
    assert float((bd - A @ x).norm() / bd.norm()) < 2e-9
    # float32
    xf, itf, _ = T.pbicgstab_solve(*cu(v.float(), r, c, dev=dev), sh, b.float().to(dev),
                                   atol=0.0, rtol=1e-5, preconditioner="jacobi")
    Af = T.SparseTensor(*cu(v, r, c, dev=dev), sh)
    assert xf.dtype == torch.float32
    assert float((bd - Af @ xf.double()).norm() / bd.norm()) < 1e-4
    # both views, bit for bit
    out = []
    for diagonal in (True, False):
        Am = PB.CachedSparseMatrix(*cu(v, r, c, dev=dev), sh)
        Am.csr._sell = Am.csr.sell(diagonal=diagonal)
        M = PB.get_preconditioner(Am, "jacobi", method="bicgstab")
        out.append(PB._bicgstab_core(Am, bd, None, M.dinv, 0.0, 1e-9, 10000))
    assert out[0][1].iterations == out[1][1].iterations
    assert torch.equal(out[0][0], out[1][0])


# ---------------------------------------------------------------- batched
def test_batched_cg_matches_reference(dev, golden):
    case = golden["batched_d2d12"]
    vb, r, c, sh, bb = case_inputs(case)
    X = T.batched_cg_same_pattern(*cu(vb, r, c, dev=dev), sh, bb.to(dev), atol=0.0, rtol=1e-8)
    assert rel(X, case["X_rtol1e-8"]) < 1e-9
    Xo, ito = K.batched_cg_same_pattern(vb, r, c, sh, bb, atol=0.0, rtol=1e-8)
    assert iters_close(PB.last_solve_info()["iterations"], ito)


def test_batched_autograd_matches_reference(dev, golden):
    case = golden["batched_d2d12"]
    vb, r, c, sh, bb = case_inputs(case)
    vg = vb.to(dev).requires_grad_(True)
    bg = bb.to(dev).requires_grad_(True)
    U = T.spsolve_batch_same_layout(vg, r.to(dev), c.to(dev), sh, bg, method="cg", atol=1e-10)
    (U * U).sum().backward()
    assert rel(U, case["U_autograd"]) < 1e-8
    assert rel(vg.grad, case["grad_val"]) < 1e-8
    assert rel(bg.grad, case["grad_b"]) < 1e-8


# ---------------------------------------------------------------- adjoint
@pytest.mark.parametrize("name", ["adj_cg_3d8", "adj_bicg_cd6"])
def test_adjoint_gradients_match_reference(dev, golden, name):
    case = golden[name]
    v, r, c, sh = case_inputs(case)
    vg = v.to(dev).requires_grad_(True)
    bg = case["b"].to(dev).requires_grad_(True)
    x = T.spsolve(vg, r.to(dev), c.to(dev), sh, bg, backend="pytorch", method=case["method"])
    (x * x).sum().backward()
    assert rel(x, case["x"]) < 1e-8
    assert rel(vg.grad, case["grad_val"]) < 1e-8
    assert rel(bg.grad, case["grad_b"]) < 1e-8


def test_sparse_tensor_solve_auto(dev, golden):
    case = golden["st_solve_2d10"]
    v, r, c, sh = case_inputs(case)
    x = T.SparseTensor(*cu(v, r, c, dev=dev), sh).solve(case["b"].to(dev))
    assert rel(x, case["x"]) < 1e-8


# ------------------------------------------------------------ multi-RHS CG
def test_multi_rhs_cg_matches_reference(dev, golden):
    case = golden["mrhs_2d24"]
    v, r, c, sh = case_inputs(case)
    vd, rd, cd = cu(v, r, c, dev=dev)
    B = case["B"].to(dev)
    X = T.pytorch_solve(vd, rd, cd, sh, B, method="cg", atol=1e-12, rtol=1e-9,
                        preconditioner="none")
    assert X.shape == B.shape and rel(X, case["X_none"]) < 1e-9
    A = PB.CachedSparseMatrix(vd, rd, cd, sh)
    res = PB.batched_pcg_solve(A, B, atol=1e-12, rtol=1e-9,
                               preconditioner=PB.get_preconditioner(A, "none"))
    assert torch.equal(res.num_iters.cpu(), case["iters_none"]) and bool(res.converged.all())
    Xj = T.pytorch_solve(vd, rd, cd, sh, B, method="cg", atol=1e-12, rtol=1e-9,
                         preconditioner="jacobi")
    assert rel(Xj, case["X_jacobi"]) < 1e-9


def test_multi_rhs_cg_guess_and_single_column(dev):
    v, r, c, sh = P.poisson_3d_7pt(12)
    g = torch.Generator().manual_seed(3)
    B = torch.randn(sh[0], 3, generator=g, dtype=torch.float64)
    X0 = torch.randn(sh[0], 3, generator=g, dtype=torch.float64)
    d = 1.0 / K.diagonal(v, r, c, sh[0])
    Xo, ito, _, _ = K.batched_pcg(v, r, c, sh, B, X0=X0, atol=0.0, rtol=1e-10, dinv=d)
    A = PB.CachedSparseMatrix(*cu(v, r, c, dev=dev), sh)
    res = PB.batched_pcg_solve(A, B.to(dev), X0=X0.to(dev), atol=0.0, rtol=1e-10,
                               preconditioner=PB.get_preconditioner(A, "jacobi"))
    assert torch.equal(res.num_iters.cpu(), ito) and rel(res.X, Xo) < 1e-9
    x1 = T.pytorch_solve(*cu(v, r, c, dev=dev), sh, B[:, :1].to(dev), method="cg", atol=0.0,
                         rtol=1e-10, preconditioner="jacobi")
    assert x1.shape == (sh[0], 1) and rel(x1[:, 0], Xo[:, 0]) < 1e-8


# ------------------------------------------------------------------- fp32
def test_pcg_fp32_matches_oracle(dev):
    """fp32 Jacobi PCG (the fp32 variant of the 3-D 7-point config) against
    the oracle run in fp32 with the same ops."""
    v, r, c, sh = P.poisson_3d_7pt(20)
    b = P.rhs_normal(sh[0], 1).float()
    xo, ito, _, _ = K.pcg(v.float(), r, c, sh, b, atol=0.0, rtol=1e-5, precond="jacobi")
    A = PB.CachedSparseMatrix(*cu(v.float(), r, c, dev=dev), sh)
    assert A.sell().diagonal_offsets
    res = PB.pcg_solve_optimized(A, b.to(dev), atol=0.0, rtol=1e-5,
                                 preconditioner=PB.get_preconditioner(A, "jacobi"))
    assert res.x.dtype == torch.float32 and res.converged
    assert iters_close(res.num_iters, ito), (res.num_iters, ito)
    assert rel(res.x, xo) < 1e-4
