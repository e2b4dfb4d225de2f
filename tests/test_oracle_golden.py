"""Pin the oracle against outputs of the reference itself (tests/golden/),
so the oracle can stand in for torch-sla in the GPU parity tests."""
import numpy as np
import pytest
import torch

from conftest import case_inputs
from oracle import krylov as K
from oracle import partition as OP
from torch_sla_b200 import problems as P


def test_generators_match_reference_grid_coo(golden):
    for key, dims, diag in (("grid2d_8", (8, 8), 4.0), ("grid3d_456", (4, 5, 6), 6.0)):
        g = golden[key]
        v, r, c = P.grid_coo(dims, diag, P.axis_edges(len(dims), -1.0))
        assert torch.equal(v, g["val"]) and torch.equal(r, g["row"]) and torch.equal(c, g["col"])


@pytest.mark.parametrize("name", ["pcg_2d32_none", "pcg_3d16_jacobi", "pcg_3d16_jacobi_f32",
                                  "pcg_2d16_x0", "pcg_2d32_maxiter"])
def test_oracle_pcg_matches_reference(golden, name):
    case = golden[name]
    v, r, c, sh = case_inputs(case)
    kw = dict(case["kw"])
    pc = kw.pop("preconditioner")
    x, it, res, conv = K.pcg(v, r, c, sh, case["b"], precond=pc, **kw)
    assert it == case["iters"]
    assert conv == case["converged"]
    assert torch.equal(x, case["x"])
    assert res == pytest.approx(case["residual"], rel=1e-12)


def test_oracle_pcg_config1_full_size(golden):
    case = golden["pcg_2d256_none"]
    v, r, c, sh = P.poisson_2d_5pt(256)
    b = P.rhs_uniform_pm1(sh[0], 0)
    x, it, res, conv = K.pcg(v, r, c, sh, b, atol=0.0, rtol=1e-10, maxiter=10000, precond="none")
    assert it == case["iters"] == 868
    assert float(x.sum()) == pytest.approx(case["x_sum"], rel=1e-12)


MIXED = ["mixed_3d12_jacobi", "mixed_3d12_default", "mixed_2d20_none", "mixed_2d20_x0",
         "mixed_2d20_maxiter", "mixed_indef_2d10", "mixed_indef_2d12"]


@pytest.mark.parametrize("name", MIXED)
def test_oracle_mixed_pcg_matches_reference(golden, name):
    """pcg_solve_mixed_precision / pytorch_solve(mixed_precision=True)."""
    case = golden[name]
    v, r, c, sh = case_inputs(case)
    pc = case["precond"] or "default"
    x, it, res, conv, pap = K.pcg_mixed(v, r, c, sh, case["b"], precond=pc, **case["kw"])
    assert it == case["iters"]
    assert conv == case["converged"]
    assert x.dtype == torch.float64 and torch.equal(x, case["x"])
    assert res == pytest.approx(case["residual"], rel=1e-12)
    assert (pap is not None) == name.startswith("mixed_indef")
    if case["x_pytorch_solve"] is not None:
        assert torch.equal(case["x_pytorch_solve"], case["x"])


def test_oracle_mixed_adjoint_matches_reference(golden):
    """spsolve(float32, mixed_precision=True) forward and adjoint."""
    case = golden["mixed_adj_3d6"]
    v, r, c, sh = case_inputs(case)
    x = K.pcg_mixed(v, r, c, sh, case["b"], atol=1e-10, rtol=1e-10, maxiter=10000)[0]
    u = x.to(torch.float32)
    assert torch.equal(u, case["x"])
    gval, gb = K.adjoint(v, r, c, sh, u, 2 * u, method="cg", mixed_precision=True)
    assert gb.dtype == torch.float32 and torch.equal(gb, case["grad_b"])
    assert torch.equal(gval, case["grad_val"])


@pytest.mark.parametrize("name", ["bicg_cd3d10_jacobi", "bicg_ad2d12_none", "bicg_ad2d12_maxiter"])
def test_oracle_bicgstab_matches_reference(golden, name):
    case = golden[name]
    v, r, c, sh = case_inputs(case)
    kw = dict(case["kw"])
    pc = kw.pop("preconditioner")
    x, it, res, how = K.pbicgstab(v, r, c, sh, case["b"], precond=pc, **kw)
    assert it == case["iters"]
    assert torch.equal(x, case["x"])


def test_oracle_batched_matches_reference(golden):
    case = golden["batched_d2d12"]
    vb, r, c, sh, bb = case_inputs(case)
    X, it = K.batched_cg_same_pattern(vb, r, c, sh, bb, atol=0.0, rtol=1e-8, maxiter=10000)
    assert torch.equal(X, case["X_rtol1e-8"])
    U, _ = K.batched_cg_same_pattern(vb, r, c, sh, bb, atol=1e-10, rtol=1e-6, maxiter=10000)
    assert torch.equal(U, case["U_autograd"])
    gval, gb = K.batched_adjoint(vb, r, c, sh, U, 2 * U, atol=1e-10, rtol=1e-6)
    torch.testing.assert_close(gval, case["grad_val"], rtol=0, atol=0)
    torch.testing.assert_close(gb, case["grad_b"], rtol=0, atol=0)


@pytest.mark.parametrize("name", ["adj_cg_3d8", "adj_bicg_cd6"])
def test_oracle_adjoint_matches_reference(golden, name):
    case = golden[name]
    v, r, c, sh = case_inputs(case)
    fn = K.pcg if case["method"] == "cg" else K.pbicgstab
    x = fn(v, r, c, sh, case["b"], atol=1e-10, rtol=1e-10, maxiter=10000, precond="jacobi")[0]
    assert torch.equal(x, case["x"])
    gval, gb = K.adjoint(v, r, c, sh, x, 2 * x, method=case["method"])
    torch.testing.assert_close(gb, case["grad_b"], rtol=1e-14, atol=0)
    torch.testing.assert_close(gval, case["grad_val"], rtol=1e-14, atol=0)


def test_oracle_spmv_matches_reference(golden):
    case = golden["spmv_rand50"]
    y = K.spmv(case["val"], case["row"], case["col"], case["shape"], case["x"])
    torch.testing.assert_close(y, case["y"], rtol=1e-13, atol=1e-13)


def test_oracle_st_solve_auto_agrees(golden):
    # on CPU the reference's backend='auto' picks a direct solve; the
    # iterative answer agrees to the solver tolerance
    case = golden["st_solve_2d10"]
    v, r, c, sh = case_inputs(case)
    x = K.pbicgstab(v, r, c, sh, case["b"], atol=1e-10, rtol=1e-10, precond="jacobi")[0]
    torch.testing.assert_close(x, case["x"], rtol=1e-8, atol=1e-10)


@pytest.mark.parametrize("name", ["p2d16_P3", "p3d8_P4", "p27_654_P2", "pcd5_P3"])
def test_oracle_partition_maps_bit_exact(golden, name):
    case = golden["partitions"][name]
    _, r, c, _ = case_inputs(case)
    ids = OP.partition_simple(case["n"], case["P"])
    assert np.array_equal(ids, case["ids"].numpy())
    for pid, ref in enumerate(case["ranks"]):
        got = OP.build_partition(r.numpy(), c.numpy(), case["n"], ids, pid)
        for key in ("owned_nodes", "halo_nodes", "local_nodes", "global_to_local"):
            assert np.array_equal(got[key], ref[key].numpy()), key
        assert got["neighbor_partitions"] == ref["neighbor_partitions"]
        for q in ref["neighbor_partitions"]:
            assert np.array_equal(got["send_indices"][q], ref["send_indices"][q].numpy())
            assert np.array_equal(got["recv_indices"][q], ref["recv_indices"][q].numpy())


@pytest.mark.parametrize("name", ["cg_2d16", "cg_3d8_none", "bicg_cd8", "cg_27_654"])
def test_oracle_shard_solvers_match_reference(golden_shard, name):
    case = golden_shard[name]
    v, r, c, sh = case_inputs(case)
    fn = K.cg_shard if case["method"] == "cg" else K.bicgstab_shard
    x, it = fn(v, r, c, sh, case["b"], atol=case["atol"], rtol=case["rtol"], maxiter=2000,
               precond=case["precond"])
    assert it == case["iters"]
    # the reference sums each dot product per rank before the allreduce
    torch.testing.assert_close(x, case["x"], rtol=1e-9, atol=1e-12)


def test_oracle_multi_rhs_matches_reference(golden):
    case = golden["mrhs_2d24"]
    v, r, c, sh = case_inputs(case)
    X, it, _, conv = K.batched_pcg(v, r, c, sh, case["B"], atol=1e-12, rtol=1e-9)
    assert torch.equal(X, case["X_none"]) and torch.equal(it, case["iters_none"]) and conv.all()
    d = 1.0 / K.diagonal(v, r, c, sh[0])
    d = torch.where(torch.isinf(d), torch.ones_like(d), d)
    Xj, itj, _, _ = K.batched_pcg(v, r, c, sh, case["B"], atol=1e-12, rtol=1e-9, dinv=d)
    assert torch.equal(Xj, case["X_jacobi"]) and torch.equal(itj, case["iters_jacobi"])
