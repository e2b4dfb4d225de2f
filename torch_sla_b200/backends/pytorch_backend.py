"""B200 (sm_100a) implementation of torch-sla's `pytorch` iterative backend.

Same function names, signatures, return conventions and warnings as
torch_sla/backends/pytorch_backend.py, restricted to the hot path: CG and
BiCGStab with the 'jacobi' / 'none' preconditioners, the CSR cache and the
batched same-pattern CG. Every solve runs in libsla_b200 kernels on the GPU;
CPU tensors raise (there is no CPU fallback).
"""
from __future__ import annotations

import ctypes
import warnings
from typing import Callable, NamedTuple, Optional, Tuple

import torch
from torch import Tensor

from .. import _lib as L
from .._csr import DeviceCSR, Sell, coo_value_grad

__all__ = [
    "SolveResult", "CachedSparseMatrix", "JacobiPreconditioner", "IdentityPreconditioner",
    "jacobi_preconditioner", "get_preconditioner", "pcg_solve_optimized", "pcg_solve_fused",
    "pbicgstab_solve", "pytorch_solve", "batched_cg_same_pattern", "last_solve_info",
    "MixedPrecisionMatrix", "pcg_solve_mixed_precision", "sparse_matvec", "extract_diagonal",
    "pcg_solve", "cg_solve", "bicgstab_solve", "batched_pcg_solve", "batched_cg_solve",
]


class SolveResult(NamedTuple):
    """Result of an iterative solve (pytorch_backend.py:35-40)."""
    x: Tensor
    num_iters: int
    residual: float
    converged: bool


_LAST_INFO: dict = {}


def last_solve_info() -> dict:
    """Iterations / residual / status of the most recent solve on this process."""
    return dict(_LAST_INFO)


def _record(kind: str, info: L.SolveInfo) -> None:
    _LAST_INFO.clear()
    _LAST_INFO.update(kind=kind, iterations=int(info.iterations), residual=float(info.residual),
                      status=int(info.status), reason=int(info.reason))


class CachedSparseMatrix:
    """GPU CSR cache of a COO matrix (pytorch_backend.py:107-215).

    The COO -> CSR conversion, the SELL-32 view the solver kernels read and
    the diagonal are built by libsla_b200 on the device.
    """

    def __init__(self, val: Tensor, row: Tensor, col: Tensor, shape: Tuple[int, int],
                 use_rcm: bool = False):
        if use_rcm:
            raise NotImplementedError("torch_sla_b200: RCM reordering is not part of the B200 path")
        L.dtype_code(val.dtype)
        self.val, self.row, self.col = val, row, col
        self.shape = (int(shape[0]), int(shape[1]))
        self.device = val.device
        self.dtype = val.dtype
        self.n = self.shape[0]
        self.use_rcm = False
        self.csr = DeviceCSR(val, row, col, self.shape)
        self._diag = None

    def matvec(self, x: Tensor) -> Tensor:
        """Sparse matrix-vector product y = A @ x."""
        L.require_cuda(x)
        return self.csr.matvec(x.to(self.dtype))

    matvec_reordered = matvec

    @property
    def diagonal(self) -> Tensor:
        if self._diag is None:
            self._diag = self.csr.diagonal()
        return self._diag

    def sell(self):
        return self.csr.sell()


class JacobiPreconditioner:
    """M^{-1} = diag(A)^{-1} with |d| < 100 eps -> 1 (pytorch_backend.py:221-235).

    Callable like the reference's closure; the fused solver kernels read
    `dinv` directly instead of calling it.
    """

    def __init__(self, A: CachedSparseMatrix):
        self.dinv = A.csr.jacobi_inverse(L.SLA_JACOBI_EPS)

    def __call__(self, r: Tensor) -> Tensor:
        return self.dinv * r


class IdentityPreconditioner:
    """preconditioner='none' (pytorch_backend.py:916-917)."""
    dinv = None

    def __call__(self, r: Tensor) -> Tensor:
        return r


def jacobi_preconditioner(A: CachedSparseMatrix) -> JacobiPreconditioner:
    return JacobiPreconditioner(A)


def get_preconditioner(A: CachedSparseMatrix, name: str = "jacobi",
                       mixed_precision: bool = False, method: str = "cg"):
    """'jacobi' and 'none' (pytorch_backend.py:855-929). 'auto' resolves to
    'jacobi', the only preconditioner of the B200 path."""
    if mixed_precision and A.dtype == torch.float64:
        raise NotImplementedError("torch_sla_b200: float32 application of a float64 "
                                  "preconditioner is not part of the B200 path")
    if name is None or name == "none":
        return IdentityPreconditioner()
    if name in ("jacobi", "auto"):
        return jacobi_preconditioner(A)
    raise NotImplementedError(
        f"torch_sla_b200: preconditioner {name!r} is not implemented on the B200 path "
        "(available: jacobi, none)")


def _as_dinv(preconditioner, A: CachedSparseMatrix):
    if preconditioner is None:
        return jacobi_preconditioner(A).dinv
    if isinstance(preconditioner, (JacobiPreconditioner, IdentityPreconditioner)):
        return preconditioner.dinv
    raise NotImplementedError("torch_sla_b200: the fused kernels accept the preconditioners "
                              "built by get_preconditioner ('jacobi', 'none') only")


def _pcg_core(A: CachedSparseMatrix, b: Tensor, x0, dinv, atol, rtol, maxiter, flags=0,
              sell=None):
    """sla_pcg on A's SELL view (or on `sell`, another view of the same rows)."""
    L.require_cuda(b, x0)
    if b.dim() != 1 or b.shape[0] != A.n:
        raise ValueError(f"torch_sla_b200: b must have shape [{A.n}]")
    b = b.to(A.dtype).contiguous()
    sell = A.sell() if sell is None else sell
    lib = L.lib()
    need = ctypes.c_size_t(0)
    L.check("sla_pcg_workspace", lib.sla_pcg_workspace(A.csr.code, A.n, ctypes.byref(need)))
    ws = L.workspace(need.value, A.device)
    x = x0.to(A.dtype).clone().contiguous() if x0 is not None else torch.empty_like(b)
    info = L.SolveInfo()
    st = lib.sla_pcg(A.csr.code, sell.ref(), L.ptr(dinv), L.ptr(b), L.ptr(x),
                     int(x0 is not None), float(atol), float(rtol), int(maxiter), int(flags),
                     L.ptr(ws), ws.numel(), ctypes.byref(info), L.stream_handle(A.device))
    L.check("sla_pcg", st)
    _record("pcg", info)
    return x, info


def pcg_solve_optimized(A: CachedSparseMatrix, b: Tensor, x0: Optional[Tensor] = None,
                        atol: float = 1e-10, rtol: float = 1e-6, maxiter: int = 10000,
                        preconditioner: Callable[[Tensor], Tensor] = None,
                        check_interval: int = 50) -> SolveResult:
    """Jacobi-PCG with the start-of-iteration stopping test
    (pytorch_backend.py:1262-1362): per iteration a search-direction pass, an
    SpMV and an update kernel (one cooperative kernel for small systems)."""
    dinv = _as_dinv(preconditioner, A)
    x, info = _pcg_core(A, b, x0, dinv, atol, rtol, maxiter)
    converged = info.status == L.SLA_OK
    if not converged:
        warnings.warn(f"PCG did not converge in {maxiter} iterations "
                      f"(residual={info.residual:.2e})")
    return SolveResult(x, int(info.iterations), float(info.residual), converged)


def pcg_solve_fused(val: Tensor, row: Tensor, col: Tensor, shape: Tuple[int, int], b: Tensor,
                    x0: Optional[Tensor] = None, atol: float = 1e-10, rtol: float = 1e-6,
                    maxiter: int = 10000, preconditioner: str = "auto") -> SolveResult:
    """CSR build + preconditioner + PCG (pytorch_backend.py:1466-1501)."""
    A = CachedSparseMatrix(val, row, col, shape)
    M = get_preconditioner(A, preconditioner, method="cg")
    return pcg_solve_optimized(A, b, x0=x0, atol=atol, rtol=rtol, maxiter=maxiter, preconditioner=M)


# ------------------------------------------------------ mixed-precision PCG
class MixedPrecisionMatrix:
    """float32 matrix with float64 input and output (pytorch_backend.py:1143-1173):
    x is rounded to float32, multiplied in float32 and the result widened."""

    def __init__(self, val: Tensor, row: Tensor, col: Tensor, shape: Tuple[int, int],
                 cached: Optional[CachedSparseMatrix] = None):
        self.shape = (int(shape[0]), int(shape[1]))
        self.device = val.device
        self.n = self.shape[0]
        self.val, self.row, self.col = val, row, col
        # a float32 CachedSparseMatrix of the same COO is reused as is
        self.A32 = (cached if cached is not None and cached.dtype == torch.float32
                    else CachedSparseMatrix(val.to(torch.float32), row, col, self.shape))
        self._dinv64 = None

    def matvec(self, x_f64: Tensor) -> Tensor:
        return self.A32.matvec(x_f64.to(torch.float32)).to(torch.float64)

    def jacobi_inverse64(self) -> Tensor:
        """1/d with |d| < 100 eps(float64) -> 1, d the float64 sum of the
        diagonal entries (pytorch_backend.py:1156-1158, 1211-1216)."""
        if self._dinv64 is None:
            A64 = CachedSparseMatrix(self.val.to(torch.float64), self.row, self.col, self.shape)
            self._dinv64 = A64.csr.jacobi_inverse(L.SLA_JACOBI_EPS)
        return self._dinv64


class Float32Preconditioner:
    """pytorch_solve's M_f64 (pytorch_backend.py:2281-2283): applies a
    float32 preconditioner to r rounded to float32 and widens the result."""

    def __init__(self, inner):
        self.inner = inner

    def __call__(self, r: Tensor) -> Tensor:
        return self.inner(r.to(torch.float32)).to(torch.float64)


def _mixed_mode(preconditioner, Am: MixedPrecisionMatrix):
    """(SLA_MIXED_M_* mode, inverse diagonal) of a preconditioner argument."""
    if preconditioner is None:
        return L.SLA_MIXED_M_F64_JACOBI, Am.jacobi_inverse64()
    if isinstance(preconditioner, Float32Preconditioner):
        inner = preconditioner.inner
        if isinstance(inner, IdentityPreconditioner):
            return L.SLA_MIXED_M_F32_NONE, None
        if isinstance(inner, JacobiPreconditioner) and inner.dinv.dtype == torch.float32:
            return L.SLA_MIXED_M_F32_JACOBI, inner.dinv
    elif isinstance(preconditioner, IdentityPreconditioner):
        return L.SLA_MIXED_M_F64_NONE, None
    elif isinstance(preconditioner, JacobiPreconditioner):
        # dinv * r with float64 r promotes to float64: the widened inverse
        return L.SLA_MIXED_M_F64_JACOBI, preconditioner.dinv.to(torch.float64)
    raise NotImplementedError("torch_sla_b200: mixed-precision PCG accepts the preconditioners "
                              "built by get_preconditioner ('jacobi', 'none') only")


def pcg_solve_mixed_precision(A: CachedSparseMatrix, b: Tensor, x0: Optional[Tensor] = None,
                              atol: float = 1e-10, rtol: float = 1e-6, maxiter: int = 10000,
                              preconditioner: Callable[[Tensor], Tensor] = None) -> SolveResult:
    """Mixed-precision PCG (pytorch_backend.py:1176-1255): float32 SpMV,
    float64 vectors, dots and updates; stops when ||r|| < max(atol, rtol||b||)
    after an update; p'Ap <= 0 stops with a warning. x is float64."""
    L.require_cuda(b, x0)
    if b.dim() != 1 or b.shape[0] != A.n:
        raise ValueError(f"torch_sla_b200: b must have shape [{A.n}]")
    Am = MixedPrecisionMatrix(A.val, A.row, A.col, A.shape, cached=A)
    mode, dinv = _mixed_mode(preconditioner, Am)
    if b.dtype not in (torch.float32, torch.float64):
        b = b.to(torch.float64)
    b = b.contiguous()
    lib = L.lib()
    need = ctypes.c_size_t(0)
    L.check("sla_pcg_mixed_workspace", lib.sla_pcg_mixed_workspace(A.n, ctypes.byref(need)))
    ws = L.workspace(need.value, A.device)
    x = (x0.to(torch.float64).clone().contiguous() if x0 is not None
         else torch.empty(A.n, dtype=torch.float64, device=A.device))
    info = L.SolveInfo()
    pap = ctypes.c_double(0.0)
    st = lib.sla_pcg_mixed(Am.A32.sell().ref(), int(mode), L.ptr(dinv), L.dtype_code(b.dtype),
                           L.ptr(b), L.ptr(x), int(x0 is not None), float(atol), float(rtol),
                           int(maxiter), L.ptr(ws), ws.numel(), ctypes.byref(info),
                           ctypes.byref(pap), L.stream_handle(A.device))
    L.check("sla_pcg_mixed", st)
    _record("pcg_mixed", info)
    if info.status == L.SLA_BREAKDOWN:
        warnings.warn(f"PCG: Matrix not positive definite (p'Ap = {pap.value:.2e})")
        return SolveResult(x, int(info.iterations), float(info.residual), False)
    converged = info.status == L.SLA_OK
    if not converged:
        warnings.warn(f"Mixed PCG did not converge in {maxiter} iterations "
                      f"(residual={info.residual:.2e})")
    return SolveResult(x, int(info.iterations), float(info.residual), converged)


def _bicgstab_core(A: CachedSparseMatrix, b: Tensor, x0, dinv, atol, rtol, maxiter):
    L.require_cuda(b, x0)
    b = b.to(A.dtype).contiguous()
    lib = L.lib()
    need = ctypes.c_size_t(0)
    L.check("sla_bicgstab_workspace", lib.sla_bicgstab_workspace(A.csr.code, A.n, ctypes.byref(need)))
    ws = L.workspace(need.value, A.device)
    x = x0.to(A.dtype).clone().contiguous() if x0 is not None else torch.empty_like(b)
    info = L.SolveInfo()
    st = lib.sla_bicgstab(A.csr.code, A.sell().ref(), L.ptr(dinv), L.ptr(b), L.ptr(x),
                          int(x0 is not None), float(atol), float(rtol), int(maxiter), L.ptr(ws),
                          ws.numel(), ctypes.byref(info), L.stream_handle(A.device))
    L.check("sla_bicgstab", st)
    _record("bicgstab", info)
    return x, info


def pbicgstab_solve(val: Tensor, row: Tensor, col: Tensor, shape: Tuple[int, int], b: Tensor,
                    x0: Optional[Tensor] = None, atol: float = 1e-10, rtol: float = 1e-6,
                    maxiter: int = 10000, preconditioner: str = "auto") -> Tuple[Tensor, int, float]:
    """Jacobi-PBiCGStab (pytorch_backend.py:1508-1596); returns (x, iters, residual)."""
    A = CachedSparseMatrix(val, row, col, shape)
    M = get_preconditioner(A, preconditioner, method="bicgstab")
    x, info = _bicgstab_core(A, b, x0, M.dinv, atol, rtol, maxiter)
    if info.reason == 3:
        warnings.warn("PBiCGStab: rho became too small")
    if info.status != L.SLA_OK:
        warnings.warn(f"PBiCGStab did not converge in {maxiter} iterations "
                      f"(residual={info.residual:.2e})")
    return x, int(info.iterations), float(info.residual)


def pytorch_solve(val: Tensor, row: Tensor, col: Tensor, shape: Tuple[int, int], b: Tensor,
                  method: str = "cg", atol: float = 1e-10, rtol: float = 1e-6,
                  maxiter: int = 10000, x0: Optional[Tensor] = None,
                  preconditioner: str = "jacobi", mixed_precision: bool = False) -> Tensor:
    """Method switch of the pytorch backend (pytorch_backend.py:2224-2337)."""
    L.require_cuda(val, b)
    if method == "cg":
        if b.dim() == 2:
            A_mat = CachedSparseMatrix(val, row, col, shape)
            M = get_preconditioner(A_mat, preconditioner)
            return batched_pcg_solve(A_mat, b, X0=x0, atol=atol, rtol=rtol, maxiter=maxiter,
                                     preconditioner=M).X
        if mixed_precision and val.dtype == torch.float32:
            A = CachedSparseMatrix(val, row, col, shape)
            M = Float32Preconditioner(get_preconditioner(A, preconditioner))
            return pcg_solve_mixed_precision(A, b, x0=x0, atol=atol, rtol=rtol, maxiter=maxiter,
                                             preconditioner=M).x
        return pcg_solve_fused(val, row, col, shape, b, x0=x0, atol=atol, rtol=rtol,
                               maxiter=maxiter, preconditioner=preconditioner).x
    if method == "bicgstab":
        if b.dim() == 2:
            cols = [pbicgstab_solve(val, row, col, shape, b[:, k], x0=None, atol=atol, rtol=rtol,
                                    maxiter=maxiter, preconditioner=preconditioner)[0]
                    for k in range(b.shape[1])]
            return torch.stack(cols, dim=1)
        return pbicgstab_solve(val, row, col, shape, b, x0=x0, atol=atol, rtol=rtol,
                               maxiter=maxiter, preconditioner=preconditioner)[0]
    if method in ("gmres", "minres", "lsqr", "lsmr"):
        raise NotImplementedError(f"torch_sla_b200: method {method!r} is outside the B200 "
                                  "hot path (cg, bicgstab)")
    raise ValueError(f"Unknown method: {method}. Available: cg, bicgstab, gmres, minres, lsqr, lsmr")


# ------------------------------------------------- legacy / helper entries
def sparse_matvec(val: Tensor, row: Tensor, col: Tensor, shape: Tuple[int, int],
                  x: Tensor) -> Tensor:
    """y = A @ x from COO, values taken in x's dtype (pytorch_backend.py:2153-2158)."""
    L.require_cuda(val, x)
    return DeviceCSR(val.to(x.dtype), row, col, tuple(shape)).matvec(x)


def extract_diagonal(val: Tensor, row: Tensor, col: Tensor, shape: Tuple[int, int]) -> Tensor:
    """Sum of the diagonal COO entries, length min(shape) (pytorch_backend.py:2161-2167)."""
    L.require_cuda(val)
    n = min(int(shape[0]), int(shape[1]))
    return DeviceCSR(val, row, col, tuple(shape)).diagonal()[:n]


def pcg_solve(val: Tensor, row: Tensor, col: Tensor, shape: Tuple[int, int], b: Tensor,
              x0: Optional[Tensor] = None, atol: float = 1e-10, rtol: float = 1e-6,
              maxiter: int = 10000, M_inv: Optional[Tensor] = None,
              callback: Optional[Callable] = None) -> Tuple[Tensor, int, float]:
    """Legacy interface (pytorch_backend.py:2170-2186): Jacobi PCG; M_inv and
    callback are accepted and unused, as in torch-sla."""
    res = pcg_solve_fused(val, row, col, shape, b, x0=x0, atol=atol, rtol=rtol, maxiter=maxiter,
                          preconditioner="jacobi")
    return res.x, res.num_iters, res.residual


def cg_solve(val: Tensor, row: Tensor, col: Tensor, shape: Tuple[int, int], b: Tensor,
             x0: Optional[Tensor] = None, atol: float = 1e-10, rtol: float = 1e-6,
             maxiter: int = 10000, callback: Optional[Callable] = None) -> Tuple[Tensor, int, float]:
    """pytorch_backend.py:2189-2204 ('auto' preconditioner, which is Jacobi here)."""
    res = pcg_solve_fused(val, row, col, shape, b, x0=x0, atol=atol, rtol=rtol, maxiter=maxiter,
                          preconditioner="auto")
    return res.x, res.num_iters, res.residual


def bicgstab_solve(val: Tensor, row: Tensor, col: Tensor, shape: Tuple[int, int], b: Tensor,
                   x0: Optional[Tensor] = None, atol: float = 1e-10, rtol: float = 1e-6,
                   maxiter: int = 10000,
                   callback: Optional[Callable] = None) -> Tuple[Tensor, int, float]:
    """pytorch_backend.py:2207-2221 ('auto' preconditioner, which is Jacobi here)."""
    return pbicgstab_solve(val, row, col, shape, b, x0=x0, atol=atol, rtol=rtol, maxiter=maxiter,
                           preconditioner="auto")


# ----------------------------------------------------------- multi-RHS CG
class BatchSolveResult(NamedTuple):
    """Result of the multi-RHS solve (pytorch_backend.py:2344-2349)."""
    X: Tensor
    num_iters: Tensor
    residuals: Tensor
    converged: Tensor


def batched_pcg_solve(A: CachedSparseMatrix, B: Tensor, X0: Optional[Tensor] = None,
                      atol: float = 1e-10, rtol: float = 1e-6, maxiter: int = 10000,
                      preconditioner=None, check_interval: int = 50) -> BatchSolveResult:
    """CG on the K columns of B (n, K) together (pytorch_backend.py:2352-2504).

    Jacobi is applied column by column. (torch-sla's own pytorch_solve hands
    its 1-D Jacobi closure a 2-D residual, which fails to broadcast unless
    n == K; the column-wise form here is what its batched_cg_solve wrapper
    and preconditioner=None do.)
    """
    L.require_cuda(B, X0)
    if B.dim() == 1:
        B = B.unsqueeze(1)
    n, K = int(B.shape[0]), int(B.shape[1])
    if n != A.n:
        raise ValueError(f"torch_sla_b200: B must have {A.n} rows")
    if preconditioner is None:
        d = 1.0 / A.diagonal
        dinv = torch.where(torch.isinf(d), torch.ones_like(d), d).contiguous()
    else:
        dinv = _as_dinv(preconditioner, A)
    Bc = B.to(A.dtype).contiguous()
    lib = L.lib()
    X = torch.empty_like(Bc)
    guess = X0 is not None
    if guess:
        X.copy_(X0 if X0.dim() == 2 else X0.unsqueeze(1))
    iters = torch.zeros(K, dtype=torch.int64)
    conv = torch.zeros(K, dtype=torch.int32)
    info = L.SolveInfo()
    for k0 in range(0, K, _MAX_BATCH):
        k1 = min(K, k0 + _MAX_BATCH)
        kk = k1 - k0
        Bk = Bc if kk == K else Bc[:, k0:k1].contiguous()
        Xk = X if kk == K else X[:, k0:k1].contiguous()
        need = ctypes.c_size_t(0)
        L.check("sla_multi_rhs_cg_workspace",
                lib.sla_multi_rhs_cg_workspace(A.csr.code, n, kk, ctypes.byref(need)))
        ws = L.workspace(need.value, A.device)
        tail = (L.ptr(dinv), L.ptr(Bk), L.ptr(Xk), int(guess), float(atol), float(rtol),
                int(maxiter), int(check_interval), iters[k0:k1].data_ptr(),
                conv[k0:k1].data_ptr(), L.ptr(ws), ws.numel(), ctypes.byref(info),
                L.stream_handle(A.device))
        sell = A.sell()
        if sell.diagonal_offsets and sell.row_ids is None and sell.row_base == 0:
            fn = "sla_multi_rhs_cg_diag"  # stencil matrix: columns computed, not loaded
            st = lib.sla_multi_rhs_cg_diag(A.csr.code, sell.ref(), kk, *tail)
        else:
            fn = "sla_multi_rhs_cg"
            st = lib.sla_multi_rhs_cg(A.csr.code, L.ptr(A.csr.rowptr), L.ptr(A.csr.colind),
                                      L.ptr(A.csr.vals), n, kk, *tail)
        L.check(fn, st)
        if kk != K:
            X[:, k0:k1].copy_(Xk)
    _record("multi_rhs_cg", info)
    R = Bc - torch.stack([A.matvec(X[:, j].contiguous()) for j in range(K)], dim=1)
    residuals = torch.linalg.vector_norm(R, dim=0)
    converged = conv.to(torch.bool).to(A.device)
    if not bool(converged.all()):
        n_failed = int((~converged).sum().item())
        warnings.warn(f"Batched PCG: {n_failed}/{K} RHS did not converge in {maxiter} iterations")
    return BatchSolveResult(X, iters.to(torch.int32).to(A.device), residuals, converged)


def batched_cg_solve(val: Tensor, row: Tensor, col: Tensor, shape: Tuple[int, int], B: Tensor,
                     X0: Optional[Tensor] = None, atol: float = 1e-10, rtol: float = 1e-6,
                     maxiter: int = 10000, preconditioner: str = "jacobi",
                     check_interval: int = 50) -> BatchSolveResult:
    """Multi-RHS CG from COO (pytorch_backend.py:2507-2572). 'jacobi' is
    1/diag with infinite entries set to 1, applied column by column."""
    A = CachedSparseMatrix(val, row, col, shape)
    M = None if preconditioner == "jacobi" else get_preconditioner(A, preconditioner)
    return batched_pcg_solve(A, B, X0=X0, atol=atol, rtol=rtol, maxiter=maxiter,
                             preconditioner=M, check_interval=check_interval)


# ----------------------------------------------------------------- batched
_MAX_BATCH = 1024


def batched_cg_same_pattern_info(val_batch: Tensor, row: Tensor, col: Tensor,
                                 shape: Tuple[int, int], b_batch: Tensor, atol: float = 1e-10,
                                 rtol: float = 1e-6, maxiter: int = 10000):
    """batched_cg_same_pattern plus the solver info of the (last) chunk."""
    m, n = shape
    assert m == n, "CG requires square systems"
    L.require_cuda(val_batch, b_batch)
    code = L.dtype_code(val_batch.dtype)
    Bn = int(val_batch.shape[0])
    dev = val_batch.device
    csr = DeviceCSR(None, row.to(dev), col.to(dev), (n, n), keep_map=True, dtype=val_batch.dtype)
    lib = L.lib()
    stream = L.stream_handle(dev)
    X = torch.empty(Bn, n, dtype=val_batch.dtype, device=dev)
    info = L.SolveInfo()
    # stencil patterns: values in the order of a diagonal-offset view, whose
    # SpMV computes columns instead of loading them
    diag = csr.diag_pattern()
    if diag is not None:
        offs, pos = diag
        w = len(offs)
        n_out = (n + 31) // 32 * 32 * w
        view = Sell(torch.zeros(1, dtype=torch.int32, device=dev), None, None, n, None,
                    max_width=w, uniform_width=w, n_cols=n, offsets=offs)
    # Members are coupled only through the "all converged" test; batches
    # beyond the kernel's 1024 lanes run as independent chunks.
    for s0 in range(0, Bn, _MAX_BATCH):
        vb = val_batch[s0:s0 + _MAX_BATCH].contiguous()
        bb = b_batch[s0:s0 + _MAX_BATCH].to(val_batch.dtype).contiguous()
        B = int(vb.shape[0])
        need = ctypes.c_size_t(0)
        L.check("sla_batched_cg_workspace", lib.sla_batched_cg_workspace(code, n, B, ctypes.byref(need)))
        ws = L.workspace(need.value, dev)
        xo = X[s0:s0 + B]
        tail = (L.ptr(bb), L.ptr(xo), float(atol), float(rtol), int(maxiter), L.ptr(ws),
                ws.numel(), ctypes.byref(info), stream)
        if diag is not None:
            vals = torch.empty(max(n_out * B, 1), dtype=val_batch.dtype, device=dev)
            L.check("sla_batched_values_at", lib.sla_batched_values_at(
                code, L.ptr(vb), B, int(vb.shape[1]), L.ptr(csr.src_index), L.ptr(csr.seg_ptr),
                csr.nnz, L.ptr(pos), n_out, L.ptr(vals), stream))
            L.check("sla_batched_cg_diag", lib.sla_batched_cg_diag(
                code, view.ref(), L.ptr(vals), B, *tail))
        else:
            vals = torch.empty(max(csr.nnz * B, 1), dtype=val_batch.dtype, device=dev)
            L.check("sla_batched_values", lib.sla_batched_values(
                code, L.ptr(vb), B, int(vb.shape[1]), L.ptr(csr.src_index), L.ptr(csr.seg_ptr),
                csr.nnz, L.ptr(vals), stream))
            L.check("sla_batched_cg", lib.sla_batched_cg(
                code, L.ptr(csr.rowptr), L.ptr(csr.colind), L.ptr(vals), n, B, *tail))
    _record("batched_cg", info)
    return X, info


def batched_cg_same_pattern(val_batch: Tensor, row: Tensor, col: Tensor, shape: Tuple[int, int],
                            b_batch: Tensor, atol: float = 1e-10, rtol: float = 1e-6,
                            maxiter: int = 10000) -> Tensor:
    """B Jacobi-PCG solves over one shared pattern (pytorch_backend.py:2575-2638)."""
    return batched_cg_same_pattern_info(val_batch, row, col, shape, b_batch, atol, rtol, maxiter)[0]


def value_gradient(row: Tensor, col: Tensor, gradb: Tensor, u: Tensor, n_rows: int,
                   n_cols: int) -> Tensor:
    """gradval = -gradb[row] * u[col] (summed over RHS columns when 2-D),
    linear_solve.py:321-323."""
    K = 1 if gradb.dim() == 1 else int(gradb.shape[1])
    return coo_value_grad(row.to(torch.int64).contiguous(), col.to(torch.int64).contiguous(),
                          gradb, u, n_rows, n_cols, K=K, batch=1)
