"""Host-side logic on CPU: partition maps (bit-exact with the oracle and the
reference fixtures), the owned-rows partition builder, the 2-rank gloo
scatter/gather plumbing, SolverConfig, argument checks and the rule that
compute on CPU tensors raises instead of falling back."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import case_inputs
from oracle import partition as OP
import torch_sla_b200 as T
from torch_sla_b200 import partition as PP
from torch_sla_b200 import problems as P


def _same_partition(got, ref):
    assert torch.equal(got.owned_nodes, torch.as_tensor(np.asarray(ref["owned_nodes"])))
    assert torch.equal(got.halo_nodes, torch.as_tensor(np.asarray(ref["halo_nodes"])))
    assert torch.equal(got.global_to_local, torch.as_tensor(np.asarray(ref["global_to_local"])))
    assert got.neighbor_partitions == list(ref["neighbor_partitions"])
    for q in got.neighbor_partitions:
        assert torch.equal(got.send_indices[q], torch.as_tensor(np.asarray(ref["send_indices"][q])))
        assert torch.equal(got.recv_indices[q], torch.as_tensor(np.asarray(ref["recv_indices"][q])))


@pytest.mark.parametrize("name", ["p2d16_P3", "p3d8_P4", "p27_654_P2", "pcd5_P3"])
def test_partition_matches_reference_fixture(golden, name):
    case = golden["partitions"][name]
    _, r, c, _ = case_inputs(case)
    ids = PP.partition_simple(case["n"], case["P"])
    assert torch.equal(ids, case["ids"])
    for pid, ref in enumerate(case["ranks"]):
        _same_partition(PP.build_partition(r, c, case["n"], ids, pid),
                        {k: (v.numpy() if torch.is_tensor(v) else
                             ({q: t.numpy() for q, t in v.items()} if isinstance(v, dict) else v))
                         for k, v in ref.items()})


@pytest.mark.parametrize("dims,P_", [((6, 5, 4), 2), ((7, 6, 5), 3), ((8, 4, 4), 4)])
@pytest.mark.parametrize("kind", ["7pt", "27pt"])
def test_partition_from_owned_rows_equals_global_build(dims, P_, kind):
    n = dims[0] * dims[1] * dims[2]
    if kind == "7pt":
        _, r, c, _ = P.poisson_3d_7pt(dims)
    else:
        _, r, c = P.stencil27_rows(dims, 0, dims[0])
    ids = PP.partition_simple(n, P_)
    for pid in range(P_):
        full = PP.build_partition(r, c, n, ids, pid)
        lo, hi = PP.simple_range(n, P_, pid)
        keep = (r >= lo) & (r < hi)
        local = PP.build_partition_from_rows(r[keep], c[keep], lo, hi, n, P_, pid)
        ref = OP.build_partition(r.numpy(), c.numpy(), n, ids.numpy(), pid)
        _same_partition(full, ref)
        _same_partition(local, ref)


def test_slab_rows_generators_match_global_matrices():
    dims = (5, 4, 3)
    v, r, c, sh = P.poisson_3d_7pt(dims)
    A = torch.sparse_coo_tensor(torch.stack([r, c]), v, sh).coalesce()
    parts = [P.poisson_3d_7pt_rows(dims, z0, 1) for z0 in range(5)]
    B = torch.sparse_coo_tensor(torch.stack([torch.cat([p[1] for p in parts]),
                                             torch.cat([p[2] for p in parts])]),
                                torch.cat([p[0] for p in parts]), sh).coalesce()
    assert torch.equal(A.indices(), B.indices()) and torch.equal(A.values(), B.values())
    v27, r27, c27 = P.stencil27_rows(dims, 0, 5)
    S = torch.sparse_coo_tensor(torch.stack([r27, c27]), v27, sh).coalesce().to_dense()
    assert torch.equal(S, S.T)  # symmetrised edge values
    off = S - torch.diag(torch.diag(S))
    assert torch.allclose(torch.diag(S), off.abs().sum(1) + 0.01)
    halves = [P.stencil27_rows(dims, z0, 1) for z0 in range(5)]
    S2 = torch.sparse_coo_tensor(torch.stack([torch.cat([h[1] for h in halves]),
                                              torch.cat([h[2] for h in halves])]),
                                 torch.cat([h[0] for h in halves]), sh).coalesce().to_dense()
    assert torch.equal(S, S2)


def test_extract_partition_matches_oracle():
    v, r, c, sh = P.convdiff_3d_upwind(5)
    ids = PP.partition_simple(sh[0], 3)
    A = T.SparseTensor(v, r, c, sh)
    for pid in range(3):
        part = PP.build_partition(r, c, sh[0], ids, pid)
        loc = A.extract_partition(part)
        ov, orow, ocol = OP.extract_partition(v.numpy(), r.numpy(), c.numpy(),
                                              OP.build_partition(r.numpy(), c.numpy(), sh[0],
                                                                 ids.numpy(), pid))
        assert np.array_equal(loc.values.numpy(), ov)
        assert np.array_equal(loc.row_indices.numpy(), orow)
        assert np.array_equal(loc.col_indices.numpy(), ocol)


def test_solver_config_scopes():
    from torch_sla_b200.solve import _active_defaults
    assert _active_defaults() == {}
    with T.SolverConfig(method="cg", atol=1e-8):
        with T.SolverConfig(atol=1e-12, maxiter=5):
            assert _active_defaults() == {"method": "cg", "atol": 1e-12, "maxiter": 5}
        assert _active_defaults() == {"method": "cg", "atol": 1e-8}
    assert _active_defaults() == {}


def test_package_exposes_distributed_names_lazily():
    """torch_sla.DSparseTensor / torch_sla.Partition are top-level names in
    the reference (torch_sla/__init__.py); here they load on first access."""
    from torch_sla_b200.distributed import DSparseTensor
    assert T.DSparseTensor is DSparseTensor
    assert T.Partition is PP.Partition
    assert T.distributed.__name__ == "torch_sla_b200.distributed"
    assert not hasattr(T, "no_such_name")


def test_mixed_precision_preconditioner_modes():
    """pcg_solve_mixed_precision's z = M r rule for each preconditioner form
    (pytorch_backend.py:1211-1216, 2281-2283) maps to one kernel mode."""
    from torch_sla_b200 import _lib as L
    from torch_sla_b200.backends import pytorch_backend as PB

    class FakeMixed:  # stands in for MixedPrecisionMatrix (no device here)
        def jacobi_inverse64(self):
            return "dinv64"

    def jacobi(dtype):
        M = PB.JacobiPreconditioner.__new__(PB.JacobiPreconditioner)
        M.dinv = torch.ones(3, dtype=dtype)
        return M

    Am = FakeMixed()
    assert PB._mixed_mode(None, Am) == (L.SLA_MIXED_M_F64_JACOBI, "dinv64")
    mode, d = PB._mixed_mode(PB.Float32Preconditioner(jacobi(torch.float32)), Am)
    assert mode == L.SLA_MIXED_M_F32_JACOBI and d.dtype == torch.float32
    assert PB._mixed_mode(PB.Float32Preconditioner(PB.IdentityPreconditioner()), Am) == (
        L.SLA_MIXED_M_F32_NONE, None)
    assert PB._mixed_mode(PB.IdentityPreconditioner(), Am) == (L.SLA_MIXED_M_F64_NONE, None)
    mode, d = PB._mixed_mode(jacobi(torch.float32), Am)  # dinv * r promotes to float64
    assert mode == L.SLA_MIXED_M_F64_JACOBI and d.dtype == torch.float64
    with pytest.raises(NotImplementedError):
        PB._mixed_mode(lambda r: r, Am)
    # the float32 wrapper rounds r before the preconditioner and widens after
    r = torch.tensor([1.0 + 2.0 ** -40, -3.0], dtype=torch.float64)
    z = PB.Float32Preconditioner(PB.IdentityPreconditioner())(r)
    assert z.dtype == torch.float64 and z[0] == 1.0 and z[1] == -3.0


def test_compute_on_cpu_tensors_raises():
    v, r, c, sh = P.poisson_2d_5pt(6)
    b = torch.ones(36, dtype=torch.float64)
    with pytest.raises(RuntimeError, match="GPU"):
        T.spsolve(v, r, c, sh, b, backend="pytorch", method="cg")
    with pytest.raises(RuntimeError, match="GPU"):
        T.SparseTensor(v, r, c, sh) @ b
    with pytest.raises(RuntimeError, match="GPU"):
        T.batched_cg_same_pattern(v.unsqueeze(0), r, c, sh, b.unsqueeze(0))


def test_spsolve_argument_checks_match_reference():
    v, r, c, sh = P.poisson_2d_5pt(4)
    with pytest.raises(AssertionError, match="b and shape\\[0\\] must have same size"):
        T.spsolve(v, r, c, sh, torch.ones(5, dtype=torch.float64))
    with pytest.raises(AssertionError, match="val and b must have same dtype"):
        T.spsolve(v, r, c, sh, torch.ones(16, dtype=torch.float32))
    with pytest.raises(ValueError, match="Unknown backend"):
        T.spsolve(v, r, c, sh, torch.ones(16, dtype=torch.float64), backend="cudss")
    with pytest.raises(ValueError, match="not supported by backend"):
        T.spsolve(v, r, c, sh, torch.ones(16, dtype=torch.float64), backend="pytorch", method="lu")


def test_halo_symmetry_check_detects_mismatch():
    from torch_sla_b200.distributed.core import check_halo_symmetry

    class Plan:  # what check_halo_symmetry reads
        neighbors, send_counts, recv_counts = [1], [3], [3]
    check_halo_symmetry(Plan())  # single process: nothing to compare


# ------------------------------------------------------------- gloo, 2 ranks
def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_worker(rank, world, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from torch.distributed.device_mesh import init_device_mesh
        from torch_sla_b200.distributed import DSparseTensor
        from torch_sla_b200.distributed.core import check_halo_symmetry
        mesh = init_device_mesh("cpu", (world,))
        v, r, c = P.stencil27_rows((6, 5, 4), 0, 6)
        A = T.SparseTensor(v, r, c, (120, 120))
        D = DSparseTensor.partition(A, mesh, partition_method="simple")
        b = P.rhs_normal(120, 4)
        b_dt = D.scatter(b)
        full = b_dt.full_tensor()
        lo, hi = PP.simple_range(120, world, rank)
        keep = (r >= lo) & (r < hi)
        D2 = DSparseTensor.from_owned_rows(v[keep], r[keep], c[keep], (120, 120), mesh=mesh)
        same = (D2.partition_info.neighbor_partitions == D.partition_info.neighbor_partitions
                and torch.equal(D2.partition_info.halo_nodes, D.partition_info.halo_nodes))
        p = D.partition_info

        class Plan:
            neighbors = sorted(p.neighbor_partitions)
            send_counts = [int(p.send_indices[q].numel()) for q in neighbors]
            recv_counts = [int(p.recv_indices[q].numel()) for q in neighbors]
        check_halo_symmetry(Plan())
        err = None
        try:
            D @ b_dt
        except RuntimeError as e:
            err = str(e)
        torch.save({"full_ok": torch.equal(full, b), "same": same, "err": err,
                    "norm": float((2 * b_dt - b_dt).norm())}, os.path.join(out_dir, f"r{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks_partition_scatter_gather(tmp_path):
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_gloo_worker, args=(rk, world, port, str(tmp_path)))
             for rk in range(world)]
    for p_ in procs:
        p_.start()
    for p_ in procs:
        p_.join(timeout=240)
        assert p_.exitcode == 0
    b = P.rhs_normal(120, 4)
    for rk in range(world):
        res = torch.load(tmp_path / f"r{rk}.pt")
        assert res["full_ok"] and res["same"]
        assert res["err"] is not None and "GPU" in res["err"]  # no CPU fallback
        assert res["norm"] == pytest.approx(float(b.norm()), rel=1e-14)


def test_patch_install_into_reference():
    from conftest import torch_sla_path
    ref = torch_sla_path()
    if ref is None:
        pytest.skip("torch-sla not found (set TORCH_SLA_REF or install it into baseline/_ref)")
    import subprocess
    import sys
    code = (
        "import sys; sys.path.insert(0, %r); sys.path.insert(0, %r)\n"
        "import torch, torch_sla, torch_sla_b200.patch as pt\n"
        "done = pt.install(torch_sla)\n"
        "import torch_sla.linear_solve as ls, torch_sla.backends.pytorch_backend as pb\n"
        "assert ls.pytorch_solve is pb.pytorch_solve and hasattr(pb.pytorch_solve, '__wrapped_b200__')\n"
        "from torch_sla_b200 import problems as P\n"
        "v, r, c, sh = P.poisson_2d_5pt(8)\n"
        "x = torch_sla.spsolve(v, r, c, sh, torch.ones(64, dtype=torch.float64), backend='pytorch', method='cg')\n"
        "A = torch.sparse_coo_tensor(torch.stack([r, c]), v, sh).to_dense()\n"
        "assert torch.allclose(A @ x, torch.ones(64, dtype=torch.float64), atol=1e-8)\n"
        "print(len(done))\n") % (ref, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, cwd="/tmp",
                         env={**os.environ, "PYTHONDONTWRITEBYTECODE": "1"}, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    assert int(out.stdout.strip().splitlines()[-1]) >= 8


SIG_SCRIPT = r"""
import importlib, inspect, json, sys
sys.path.insert(0, sys.argv[1])
names = json.loads(sys.argv[2])
out = {}
for mod, fns in names.items():
    m = importlib.import_module(mod)
    for f in fns:
        obj = m
        for part in f.split("."):
            obj = getattr(obj, part)
        sig = inspect.signature(obj)
        out[mod + "." + f] = [(p.name, repr(p.default) if p.default is not inspect._empty else None,
                               str(p.kind)) for p in sig.parameters.values()]
print(json.dumps(out))
"""

PUBLIC = {
    "backends.pytorch_backend": ["pcg_solve_optimized", "pcg_solve_fused", "pbicgstab_solve",
                                 "pytorch_solve", "batched_cg_same_pattern", "batched_pcg_solve",
                                 "batched_cg_solve", "get_preconditioner",
                                 "pcg_solve_mixed_precision", "pcg_solve", "cg_solve",
                                 "bicgstab_solve", "sparse_matvec", "extract_diagonal"],
    "linear_solve": ["spsolve"],
    "batch_solve": ["spsolve_batch_same_layout"],
    "distributed.solve": ["cg_shard", "bicgstab_shard", "make_preconditioner"],
    "distributed.matvec": ["halo_exchange", "shard_matvec", "shard_rmatvec",
                           "reverse_halo_exchange"],
    "partition": ["partition_simple", "build_partition", "find_halo_nodes"],
}


def test_public_signatures_accept_every_reference_call():
    """Every public function of the mirror takes torch-sla's parameters in
    torch-sla's order and kind with torch-sla's defaults (read from the
    installed package; a parameter torch-sla requires may have a default
    here); parameters the mirror adds come last and have defaults, so any
    call written against torch-sla binds the same way."""
    import json
    import subprocess
    import sys
    from conftest import torch_sla_path
    ref = torch_sla_path()
    if ref is None:
        pytest.skip("torch-sla not found (set TORCH_SLA_REF or install it into baseline/_ref)")
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sigs = {}
    for pkg, path in (("torch_sla", ref), ("torch_sla_b200", repo)):
        names = {f"{pkg}.{m}": fns for m, fns in PUBLIC.items()}
        out = subprocess.run([sys.executable, "-c", SIG_SCRIPT, path, json.dumps(names)],
                             capture_output=True, text=True, cwd="/tmp", timeout=300,
                             env={**os.environ, "PYTHONDONTWRITEBYTECODE": "1"})
        assert out.returncode == 0, out.stderr[-2000:]
        sigs[pkg] = {k.split(".", 1)[1]: v
                     for k, v in json.loads(out.stdout.strip().splitlines()[-1]).items()}
    for name, theirs in sigs["torch_sla"].items():
        mine = sigs["torch_sla_b200"][name]
        assert len(mine) >= len(theirs), (name, theirs, mine)
        for (tn, td, tk), (mn, md, mk) in zip(theirs, mine):
            assert (tn, tk) == (mn, mk), (name, theirs, mine)
            assert td is None or td == md, (name, tn, td, md)
        assert all(default is not None for _, default, _ in mine[len(theirs):]), (name, mine)
