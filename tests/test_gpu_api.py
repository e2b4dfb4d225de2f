"""torch-sla's legacy and helper entries of the pytorch backend (pcg_solve,
cg_solve, bicgstab_solve, batched_cg_solve, sparse_matvec,
extract_diagonal) on the device, against the reference's own outputs."""
import warnings

import pytest
import torch

from conftest import case_inputs
from oracle import krylov as K
from torch_sla_b200.backends import pytorch_backend as PB

pytestmark = pytest.mark.gpu


def cu(*ts, dev):
    return [t.to(dev) for t in ts]


def rel(a, b):
    a = a.detach().cpu().to(torch.float64)
    b = b.detach().cpu().to(torch.float64)
    return float((a - b).norm() / b.norm())


@pytest.mark.parametrize("fn", [PB.pcg_solve, PB.cg_solve])
def test_legacy_pcg_entries(dev, golden, fn):
    case = golden["pcg_3d16_jacobi"]
    v, r, c, sh = case_inputs(case)
    kw = {k: w for k, w in case["kw"].items() if k != "preconditioner"}
    x, it, res = fn(*cu(v, r, c, dev=dev), sh, case["b"].to(dev), **kw)
    assert isinstance(it, int) and isinstance(res, float)
    assert abs(it - case["iters"]) <= max(1, round(0.03 * case["iters"]))
    assert rel(x, case["x"]) < 1e-7


def test_legacy_bicgstab_entry(dev, golden):
    case = golden["bicg_cd3d10_jacobi"]
    v, r, c, sh = case_inputs(case)
    kw = {k: w for k, w in case["kw"].items() if k != "preconditioner"}
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        x, it, res = PB.bicgstab_solve(*cu(v, r, c, dev=dev), sh, case["b"].to(dev), **kw)
    vd = v.to(dev)
    Ax = PB.sparse_matvec(vd, r.to(dev), c.to(dev), sh, x)
    b = case["b"].to(dev)
    assert float((b - Ax).norm() / b.norm()) < 2e-8
    assert rel(x, case["x"]) < 1e-6


def test_batched_cg_solve_matches_reference(dev, golden):
    """batched_cg_solve(..., 'jacobi'): 1/diag with inf -> 1, column by column."""
    case = golden["mrhs_2d24"]
    v, r, c, sh = case_inputs(case)
    res = PB.batched_cg_solve(*cu(v, r, c, dev=dev), sh, case["B"].to(dev), atol=1e-12,
                              rtol=1e-9)
    assert torch.equal(res.num_iters.cpu().to(torch.int64),
                       case["iters_jacobi"].to(torch.int64))
    assert rel(res.X, case["X_jacobi"]) < 1e-9 and bool(res.converged.all())
    res_n = PB.batched_cg_solve(*cu(v, r, c, dev=dev), sh, case["B"].to(dev), atol=1e-12,
                                rtol=1e-9, preconditioner="none")
    assert torch.equal(res_n.num_iters.cpu().to(torch.int64),
                       case["iters_none"].to(torch.int64))


def test_sparse_matvec_and_extract_diagonal(dev, golden):
    case = golden["spmv_rand50"]
    v, r, c, sh = case["val"], case["row"], case["col"], case["shape"]
    y = PB.sparse_matvec(*cu(v, r, c, dev=dev), sh, case["x"].to(dev))
    assert rel(y, case["y"]) < 1e-13
    # values follow x's dtype, as in the reference
    yf = PB.sparse_matvec(*cu(v, r, c, dev=dev), sh, case["x"].float().to(dev))
    assert yf.dtype == torch.float32 and rel(yf, case["y_f32"]) < 1e-5
    d = PB.extract_diagonal(*cu(v, r, c, dev=dev), sh)
    do = K.diagonal(v, r, c, sh[0])
    assert d.shape == (50,) and float((d.cpu() - do).abs().max()) <= 1e-15 * float(do.abs().max())
    dr = PB.extract_diagonal(*cu(v[r < 30], r[r < 30], c[r < 30], dev=dev), (30, 50))
    assert dr.shape == (30,)
