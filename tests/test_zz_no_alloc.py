"""The allocation-free PCG entry point, sla_pcg_noalloc, called through the C ABI.

Some callers cannot allocate device memory when they solve: their device
memory belongs to another framework's pool, or a cudaMalloc (which may
synchronise the device or fail under memory pressure) is not allowed on
their solve path. For them sla_pcg_noalloc keeps its scratch vectors in a
fixed 16 MiB device array inside the library instead of a caller workspace.
These tests check it against sla_pcg (same kernels, caller workspace) on two
calls in a row, because the array is shared and keeps the previous call's
contents, and check that oversized systems are refused.
"""
import ctypes

import pytest
import torch

from torch_sla_b200 import _lib as L
from torch_sla_b200 import problems as P
from torch_sla_b200.backends import pytorch_backend as PB

pytestmark = pytest.mark.gpu


def _workspace_pcg(A, dinv, b, atol, rtol, flags):
    lib = L.lib()
    need = ctypes.c_size_t(0)
    L.check("sla_pcg_workspace", lib.sla_pcg_workspace(A.csr.code, A.n, ctypes.byref(need)))
    ws = L.workspace(need.value, A.device)
    x = torch.empty_like(b)
    info = L.SolveInfo()
    st = lib.sla_pcg(A.csr.code, A.sell().ref(), L.ptr(dinv), L.ptr(b), L.ptr(x), 0, atol, rtol,
                     10000, flags, L.ptr(ws), ws.numel(), ctypes.byref(info),
                     L.stream_handle(A.device))
    L.check("sla_pcg", st)
    return x, info


def _noalloc_pcg(A, dinv, b, atol, rtol, flags):
    x = torch.empty_like(b)
    info = L.SolveInfo()
    st = L.lib().sla_pcg_noalloc(A.csr.code, A.sell().ref(), L.ptr(dinv), L.ptr(b), L.ptr(x), 0,
                                 atol, rtol, 10000, flags, ctypes.byref(info),
                                 L.stream_handle(A.device))
    L.check("sla_pcg_noalloc", st)
    return x, info


@pytest.mark.parametrize("flags", [L.SLA_PCG_AUTO, L.SLA_PCG_STREAMED, L.SLA_PCG_PERSISTENT])
@pytest.mark.parametrize("case", ["poisson3d_jacobi", "poisson2d_none", "poisson3d_f32"])
def test_noalloc_matches_workspace_entry_point(case, flags):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    dev = torch.device("cuda", 0)
    dtype = torch.float32 if case.endswith("f32") else torch.float64
    if case.startswith("poisson3d"):
        v, r, c, sh = P.poisson_3d_7pt(40, dtype=dtype, device=dev)
        b = P.rhs_normal(sh[0], 1, dtype).to(dev)
        pc, atol, rtol = "jacobi", 0.0, (1e-5 if dtype == torch.float32 else 1e-8)
    else:
        v, r, c, sh = P.poisson_2d_5pt(200, dtype=dtype, device=dev)
        b = P.rhs_uniform_pm1(sh[0], 0, dtype).to(dev)
        pc, atol, rtol = "none", 0.0, 1e-10
    A = PB.CachedSparseMatrix(v, r, c, sh)
    dinv = PB.get_preconditioner(A, pc).dinv
    x_ref, info_ref = _workspace_pcg(A, dinv, b, atol, rtol, flags)
    tol = 1e-5 if dtype == torch.float32 else 1e-12
    for _ in range(2):  # the shared array keeps the last call's contents
        x, info = _noalloc_pcg(A, dinv, b, atol, rtol, flags)
        assert info.status == info_ref.status == 0
        assert info.iterations == info_ref.iterations
        err = float((x - x_ref).abs().max() / x_ref.abs().max())
        assert err <= tol, err


def test_noalloc_refuses_systems_beyond_its_array():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    dev = torch.device("cuda", 0)
    v, r, c, sh = P.poisson_2d_5pt(800, device=dev)  # 640,000 rows > 500,000
    A = PB.CachedSparseMatrix(v, r, c, sh)
    b = torch.ones(sh[0], dtype=torch.float64, device=dev)
    x = torch.zeros_like(b)
    info = L.SolveInfo()
    st = L.lib().sla_pcg_noalloc(A.csr.code, A.sell().ref(), None, L.ptr(b), L.ptr(x), 0, 0.0,
                                 1e-8, 100, 0, ctypes.byref(info), L.stream_handle(dev))
    assert st == L.SLA_ERR_UNSUPPORTED
    assert float(x.abs().max()) == 0.0


def _f32_row_limit():
    """Largest float32 row count whose PCG scratch (sla_pcg_workspace) fits
    the library's fixed array."""
    lib = L.lib()
    need = ctypes.c_size_t(0)

    def fits(n):
        L.check("sla_pcg_workspace", lib.sla_pcg_workspace(L.SLA_F32, n, ctypes.byref(need)))
        return need.value <= L.SLA_PCG_NOALLOC_SCRATCH_BYTES

    lo, hi = 1, 1 << 24
    while hi - lo > 1:
        mid = (lo + hi) // 2
        lo, hi = (mid, hi) if fits(mid) else (lo, mid)
    return lo


def test_noalloc_float32_size_limit():
    """float32 systems just under the array's limit solve and match sla_pcg;
    one row more is refused without touching x."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    dev = torch.device("cuda", 0)
    n_max = _f32_row_limit()
    for n in (n_max, n_max + 1):
        # diagonally dominant 1-D three-point system: converges in a few tens
        # of iterations at any n
        v, r, c = P.grid_coo((n,), 4.0, P.axis_edges(1, -1.0), torch.float32, dev)
        A = PB.CachedSparseMatrix(v, r, c, (n, n))
        dinv = PB.get_preconditioner(A, "jacobi").dinv
        b = P.rhs_normal(n, 3, torch.float32).to(dev)
        if n == n_max:
            x_ref, info_ref = _workspace_pcg(A, dinv, b, 0.0, 1e-6, L.SLA_PCG_AUTO)
            x, info = _noalloc_pcg(A, dinv, b, 0.0, 1e-6, L.SLA_PCG_AUTO)
            assert info.status == info_ref.status == 0
            assert info.iterations == info_ref.iterations
            assert float((x - x_ref).abs().max() / x_ref.abs().max()) <= 1e-5
        else:
            x = torch.zeros_like(b)
            info = L.SolveInfo()
            st = L.lib().sla_pcg_noalloc(L.SLA_F32, A.sell().ref(), L.ptr(dinv), L.ptr(b),
                                         L.ptr(x), 0, 0.0, 1e-6, 100, L.SLA_PCG_AUTO,
                                         ctypes.byref(info), L.stream_handle(dev))
            assert st == L.SLA_ERR_UNSUPPORTED
            assert float(x.abs().max()) == 0.0
