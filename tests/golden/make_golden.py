"""Generate the golden fixtures of the parity tests by running torch-sla itself.

Run where the reference source tree is importable:

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py <torch-sla source tree>

(the tree may also come from the TORCH_SLA_REF environment variable).

It writes tests/golden/golden.pt (single-process solvers, SpMV, adjoints,
partition maps) and tests/golden/golden_shard.pt (the reference's
DSparseTensor shard CG/BiCGStab under a 2-rank gloo group). Inputs come from
torch_sla_b200.problems or the reference's own generators; every fixture
stores its inputs, so tests never need the reference at run time.
"""
from __future__ import annotations

import os
import sys
import warnings

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from torch_sla_b200 import problems as P  # noqa: E402


def _ref(path):
    sys.path.insert(0, path)
    import torch_sla  # noqa: F401
    return torch_sla


def coo(v, r, c, shape):
    return {"val": v.clone(), "row": r.clone(), "col": c.clone(), "shape": tuple(shape)}


def gen(name, *args, **kw):
    """Inputs rebuilt by torch_sla_b200.problems.<name>(*args, **kw) in the tests."""
    return {"gen": (name, args, kw)}


def single(ref_path):
    torch_sla = _ref(ref_path)
    from torch_sla.backends import pytorch_backend as PB
    from torch_sla.datasets import problems as RP
    from torch_sla.linear_solve import spsolve
    from torch_sla.batch_solve import spsolve_batch_same_layout
    from torch_sla.sparse_tensor import SparseTensor
    from torch_sla.partition import build_partition, partition_simple

    out = {}
    # generator equivalence: the reference's _grid_coo on small grids
    v, r, c = RP._grid_coo((8, 8), 4.0, RP._axis_edges(2, -1.0))
    out["grid2d_8"] = coo(v, r, c, (64, 64))
    v, r, c = RP._grid_coo((4, 5, 6), 6.0, RP._axis_edges(3, -1.0))
    out["grid3d_456"] = coo(v, r, c, (120, 120))

    def pcg_case(name, spec, v, r, c, shape, b, **kw):
        res = PB.pcg_solve_fused(v, r, c, shape, b, **kw)
        out[name] = {**spec, "b": b.clone(), "kw": dict(kw), "x": res.x.clone(),
                     "iters": int(res.num_iters), "residual": float(res.residual),
                     "converged": bool(res.converged)}

    v, r, c, sh = P.poisson_2d_5pt(32)
    b = P.rhs_uniform_pm1(sh[0], 0)
    pcg_case("pcg_2d32_none", gen("poisson_2d_5pt", 32), v, r, c, sh, b, atol=0.0, rtol=1e-10, maxiter=10000,
             preconditioner="none")
    v, r, c, sh = P.poisson_2d_5pt(256)
    b = P.rhs_uniform_pm1(sh[0], 0)
    res = PB.pcg_solve_fused(v, r, c, sh, b, atol=0.0, rtol=1e-10, maxiter=10000,
                             preconditioner="none")
    out["pcg_2d256_none"] = {"m": 256, "seed": 0, "iters": int(res.num_iters),
                             "residual": float(res.residual), "x_sum": float(res.x.sum()),
                             "x_norm": float(res.x.norm())}
    v, r, c, sh = P.poisson_3d_7pt(16)
    b = P.rhs_normal(sh[0], 1)
    pcg_case("pcg_3d16_jacobi", gen("poisson_3d_7pt", 16), v, r, c, sh, b, atol=0.0, rtol=1e-8, maxiter=10000,
             preconditioner="jacobi")
    pcg_case("pcg_3d16_jacobi_f32", gen("poisson_3d_7pt", 16, dtype=torch.float32), v.float(),
             r, c, sh, b.float(), atol=0.0, rtol=1e-5,
             maxiter=10000, preconditioner="jacobi")
    v, r, c, sh = P.poisson_2d_5pt(16)
    b = P.rhs_normal(sh[0], 4)
    x0 = P.rhs_normal(sh[0], 5)
    pcg_case("pcg_2d16_x0", gen("poisson_2d_5pt", 16), v, r, c, sh, b, x0=x0, atol=1e-12, rtol=1e-9, maxiter=10000,
             preconditioner="jacobi")
    v, r, c, sh = P.poisson_2d_5pt(32)
    b = P.rhs_uniform_pm1(sh[0], 0)
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        pcg_case("pcg_2d32_maxiter", gen("poisson_2d_5pt", 32), v, r, c, sh, b, atol=0.0, rtol=1e-10, maxiter=10,
                 preconditioner="jacobi")

    def bicg_case(name, spec, v, r, c, shape, b, **kw):
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")
            x, it, resid = PB.pbicgstab_solve(v, r, c, shape, b, **kw)
        out[name] = {**spec, "b": b.clone(), "kw": dict(kw), "x": x.clone(),
                     "iters": int(it), "residual": float(resid)}

    v, r, c, sh = P.convdiff_3d_upwind(10)
    b = P.rhs_uniform01(sh[0], 3)
    bicg_case("bicg_cd3d10_jacobi", gen("convdiff_3d_upwind", 10), v, r, c, sh, b, atol=0.0, rtol=1e-8, maxiter=10000,
              preconditioner="jacobi")
    prob = RP.advection_diffusion_2d(m=12, peclet=20.0)
    b = P.rhs_uniform01(prob.shape[0], 7)
    spec = coo(prob.val, prob.row, prob.col, prob.shape)
    bicg_case("bicg_ad2d12_none", spec, prob.val, prob.row, prob.col, prob.shape, b, atol=1e-12,
              rtol=1e-9, maxiter=10000, preconditioner="none")
    bicg_case("bicg_ad2d12_maxiter", spec, prob.val, prob.row, prob.col, prob.shape, b, atol=0.0,
              rtol=1e-12, maxiter=5, preconditioner="jacobi")

    # mixed-precision PCG: pytorch_solve(float32, mixed_precision=True) and
    # pcg_solve_mixed_precision with its own float64 Jacobi default
    def mixed_case(name, spec, v, r, c, shape, b, precond, **kw):
        A = PB.CachedSparseMatrix(v, r, c, shape)
        if precond is None:
            M_f64 = None
        else:
            M = PB.get_preconditioner(A, precond)
            M_f64 = lambda t, _M=M: _M(t.to(torch.float32)).to(torch.float64)  # noqa: E731
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")
            res = PB.pcg_solve_mixed_precision(A, b, preconditioner=M_f64, **kw)
            x_ps = (PB.pytorch_solve(v, r, c, shape, b, method="cg", preconditioner=precond,
                                     mixed_precision=True, **kw) if precond else None)
        out[name] = {**spec, "b": b.clone(), "kw": dict(kw), "precond": precond,
                     "x": res.x.clone(), "iters": int(res.num_iters),
                     "residual": float(res.residual), "converged": bool(res.converged),
                     "x_pytorch_solve": None if x_ps is None else x_ps.clone()}

    v, r, c, sh = P.poisson_3d_7pt(12)
    b = P.rhs_normal(sh[0], 1).float()
    mixed_case("mixed_3d12_jacobi", gen("poisson_3d_7pt", 12, dtype=torch.float32), v.float(),
               r, c, sh, b, "jacobi", atol=0.0, rtol=1e-8, maxiter=10000)
    mixed_case("mixed_3d12_default", gen("poisson_3d_7pt", 12, dtype=torch.float32), v.float(),
               r, c, sh, b, None, atol=0.0, rtol=1e-8, maxiter=10000)
    v, r, c, sh = P.poisson_2d_5pt(20)
    b = P.rhs_uniform_pm1(sh[0], 0).float()
    mixed_case("mixed_2d20_none", gen("poisson_2d_5pt", 20, dtype=torch.float32), v.float(),
               r, c, sh, b, "none", atol=1e-12, rtol=1e-9, maxiter=10000)
    x0 = P.rhs_normal(sh[0], 5)
    mixed_case("mixed_2d20_x0", gen("poisson_2d_5pt", 20, dtype=torch.float32), v.float(),
               r, c, sh, b, "jacobi", x0=x0, atol=0.0, rtol=1e-9, maxiter=10000)
    mixed_case("mixed_2d20_maxiter", gen("poisson_2d_5pt", 20, dtype=torch.float32), v.float(),
               r, c, sh, b, "jacobi", atol=0.0, rtol=1e-9, maxiter=7)
    # indefinite (Laplacian - shift*I, one negative eigenvalue): p'Ap <= 0
    # stops the solve after an even (10) and an odd (9) number of iterations
    for m, shift, seed in ((10, 0.3, 1), (12, 0.2, 0)):
        v, r, c, sh = P.poisson_2d_5pt(m)
        vi = v.float().clone()
        vi[r == c] -= shift
        mixed_case(f"mixed_indef_2d{m}", coo(vi, r, c, sh), vi, r, c, sh,
                   P.rhs_normal(sh[0], seed).float(), "jacobi", atol=0.0, rtol=1e-9, maxiter=500)
    v, r, c, sh = P.poisson_3d_7pt(6)
    vg = v.float().clone().requires_grad_(True)
    bg = P.rhs_normal(sh[0], 3).float().requires_grad_(True)
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        x = spsolve(vg, r, c, sh, bg, backend="pytorch", method="cg", mixed_precision=True)
    (x * x).sum().backward()
    out["mixed_adj_3d6"] = {**gen("poisson_3d_7pt", 6, dtype=torch.float32),
                            "b": bg.detach().clone(), "x": x.detach().clone(),
                            "grad_val": vg.grad.clone(), "grad_b": bg.grad.clone()}

    # multi-RHS CG: pytorch_solve with a 2-D b ('none' -- its 'jacobi' closure
    # does not broadcast over columns) and batched_cg_solve's column Jacobi
    v, r, c, sh = P.poisson_2d_5pt(24)
    g = torch.Generator().manual_seed(12)
    Bm = torch.randn(sh[0], 5, generator=g, dtype=torch.float64)
    Xm = PB.pytorch_solve(v, r, c, sh, Bm, method="cg", atol=1e-12, rtol=1e-9,
                          preconditioner="none")
    Am = PB.CachedSparseMatrix(v, r, c, sh)
    res_n = PB.batched_pcg_solve(Am, Bm, atol=1e-12, rtol=1e-9,
                                 preconditioner=PB.get_preconditioner(Am, "none"))
    res_j = PB.batched_cg_solve(v, r, c, sh, Bm, atol=1e-12, rtol=1e-9, preconditioner="jacobi")
    out["mrhs_2d24"] = {**gen("poisson_2d_5pt", 24), "B": Bm, "X_none": Xm.clone(),
                        "iters_none": res_n.num_iters.clone(), "X_jacobi": res_j.X.clone(),
                        "iters_jacobi": res_j.num_iters.clone()}

    # batched same-pattern CG (forward at rtol 1e-8; autograd path at its 1e-6)
    vb, r, c, sh, bb = P.diffusion_2d_batched(3, 12, seed=2)
    X = PB.batched_cg_same_pattern(vb, r, c, sh, bb, atol=0.0, rtol=1e-8, maxiter=10000)
    vbg = vb.clone().requires_grad_(True)
    bbg = bb.clone().requires_grad_(True)
    U = spsolve_batch_same_layout(vbg, r, c, sh, bbg, method="cg", atol=1e-10, maxiter=10000)
    (U * U).sum().backward()
    out["batched_d2d12"] = {**gen("diffusion_2d_batched", 3, 12, seed=2), "X_rtol1e-8": X.clone(),
                            "U_autograd": U.detach().clone(), "grad_val": vbg.grad.clone(),
                            "grad_b": bbg.grad.clone()}

    # adjoint through spsolve (pytorch backend forces rtol = 1e-10)
    def adj_case(name, spec, v, r, c, shape, b, method):
        vg = v.clone().requires_grad_(True)
        bg = b.clone().requires_grad_(True)
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")
            x = spsolve(vg, r, c, shape, bg, backend="pytorch", method=method)
        (x * x).sum().backward()
        out[name] = {**spec, "b": b.clone(), "method": method,
                     "x": x.detach().clone(), "grad_val": vg.grad.clone(),
                     "grad_b": bg.grad.clone()}

    v, r, c, sh = P.poisson_3d_7pt(8)
    adj_case("adj_cg_3d8", gen("poisson_3d_7pt", 8), v, r, c, sh, P.rhs_normal(sh[0], 1), "cg")
    v, r, c, sh = P.convdiff_3d_upwind(6)
    adj_case("adj_bicg_cd6", gen("convdiff_3d_upwind", 6), v, r, c, sh, P.rhs_uniform01(sh[0], 3), "bicgstab")

    # SparseTensor @ x on a random COO with duplicate entries
    g = torch.Generator().manual_seed(11)
    n, nnz = 50, 400
    r = torch.randint(0, n, (nnz,), generator=g)
    c = torch.randint(0, n, (nnz,), generator=g)
    v = torch.randn(nnz, generator=g, dtype=torch.float64)
    x = torch.randn(n, generator=g, dtype=torch.float64)
    A = SparseTensor(v, r, c, (n, n))
    Af = SparseTensor(v.float(), r, c, (n, n))
    out["spmv_rand50"] = {**coo(v, r, c, (n, n)), "x": x, "y": (A @ x).clone(),
                          "y_f32": (Af @ x.float()).clone()}

    # SparseTensor.solve with method='auto' (Gershgorin rejects Poisson -> bicgstab)
    v, r, c, sh = P.poisson_2d_5pt(10)
    b = P.rhs_normal(sh[0], 9)
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        xs = SparseTensor(v, r, c, sh).solve(b)
    out["st_solve_2d10"] = {**gen("poisson_2d_5pt", 10), "b": b, "x": xs.clone()}

    # partition maps
    parts = {}

    def part_case(name, spec, r, c, n, P_):
        ids = partition_simple(n, P_)
        ranks = []
        for pid in range(P_):
            pt = build_partition(r, c, n, ids, pid)
            ranks.append({
                "owned_nodes": pt.owned_nodes.clone(), "halo_nodes": pt.halo_nodes.clone(),
                "local_nodes": pt.local_nodes.clone(),
                "neighbor_partitions": [int(q) for q in pt.neighbor_partitions],
                "send_indices": {int(k): t.clone() for k, t in pt.send_indices.items()},
                "recv_indices": {int(k): t.clone() for k, t in pt.recv_indices.items()},
                "global_to_local": pt.global_to_local.clone(),
            })
        parts[name] = {**spec, "n": n, "P": P_,
                       "ids": ids.clone(), "ranks": ranks}

    v, r, c, sh = P.poisson_2d_5pt(16)
    part_case("p2d16_P3", gen("poisson_2d_5pt", 16), r, c, sh[0], 3)
    v, r, c, sh = P.poisson_3d_7pt(8)
    part_case("p3d8_P4", gen("poisson_3d_7pt", 8), r, c, sh[0], 4)
    dims = (6, 5, 4)
    v, r, c = P.stencil27_rows(dims, 0, dims[0], seed=4)
    part_case("p27_654_P2", gen("stencil27_rows", dims, 0, dims[0], seed=4), r, c, 120, 2)
    v, r, c, sh = P.convdiff_3d_upwind(5)
    part_case("pcd5_P3", gen("convdiff_3d_upwind", 5), r, c, sh[0], 3)
    out["partitions"] = parts
    return out


# ------------------------------------------------------------ shard solves
def _shard_worker(rank, world, port, ref_path, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        _ref(ref_path)
        from torch.distributed.device_mesh import init_device_mesh
        from torch_sla import DSparseTensor, SparseTensor, solve, SolverConfig
        mesh = init_device_mesh("cpu", (world,))
        res = {}
        cases = [
            ("cg_2d16", gen("poisson_2d_5pt", 16), P.poisson_2d_5pt(16), P.rhs_normal(256, 0), "cg", "jacobi", 1e-12, 1e-10),
            ("cg_3d8_none", gen("poisson_3d_7pt", 8), P.poisson_3d_7pt(8), P.rhs_normal(512, 1), "cg", None, 0.0, 1e-8),
            ("bicg_cd8", gen("convdiff_3d_upwind", 8), P.convdiff_3d_upwind(8), P.rhs_uniform01(512, 3), "bicgstab", "jacobi",
             0.0, 1e-8),
        ]
        dims = (6, 5, 4)
        v27, r27, c27 = P.stencil27_rows(dims, 0, dims[0], seed=4)
        cases.append(("cg_27_654", gen("stencil27_rows", dims, 0, dims[0], seed=4),
                      (v27, r27, c27, (120, 120)), P.rhs_normal(120, 4), "cg",
                      "jacobi", 0.0, 1e-8))
        for name, spec, (v, r, c, sh), b, method, pc, atol, rtol in cases:
            A = SparseTensor(v, r, c, sh)
            D = DSparseTensor.partition(A, mesh, partition_method="simple")
            calls = [0]
            inner = D._shard_matvec

            def counted(x, _inner=inner, _calls=calls):
                _calls[0] += 1
                return _inner(x)

            D._shard_matvec = counted
            b_dt = D.scatter(b)
            with SolverConfig(method=method, atol=atol, rtol=rtol, maxiter=2000,
                              preconditioner=pc):
                x_dt = solve(D, b_dt)
            x = x_dt.full_tensor()
            m = calls[0]
            if method == "cg":
                iters = m - 1
            else:
                iters = m // 2 if m % 2 == 0 else (m - 1) // 2
            res[name] = {**spec, "shape": sh, "b": b, "method": method, "precond": pc,
                         "atol": atol, "rtol": rtol, "x": x.clone(), "iters": iters}
        if rank == 0:
            torch.save(res, out_path)
    finally:
        dist.destroy_process_group()


def shard(ref_path, out_path, world=2, port=29631):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_shard_worker, args=(r, world, port, ref_path, out_path))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
        assert p.exitcode == 0, f"shard worker exited with {p.exitcode}"


if __name__ == "__main__":
    ref_path = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("TORCH_SLA_REF")
    if not ref_path:
        sys.exit("usage: make_golden.py <torch-sla source tree> (or set TORCH_SLA_REF)")
    torch.save(single(ref_path), os.path.join(HERE, "golden.pt"))
    shard(ref_path, os.path.join(HERE, "golden_shard.pt"))
    print("wrote", os.listdir(HERE))
