"""`spsolve` and the autograd Function of the pytorch backend
(torch_sla/linear_solve.py:283-324, 374-623), on the B200 kernels.

Only the `pytorch` backend exists here; backend='auto' resolves to it. The
adjoint solve of backward runs through the same kernels on the transposed
pattern, and the value gradient -gradb[row] * u[col] is one fused gather.
"""
from __future__ import annotations

import warnings
from typing import Tuple

import torch
from torch.autograd.function import Function

from .backends.pytorch_backend import pytorch_solve, value_gradient

BACKEND_METHODS = {"pytorch": ["cg", "bicgstab", "gmres", "minres", "lsqr", "lsmr"]}


def select_method(backend: str, is_symmetric: bool = False, is_spd: bool = False,
                  prefer_direct: bool = True) -> str:
    """pytorch backend rule of torch_sla/backends/__init__.py:337-379."""
    return "cg" if is_spd else "bicgstab"


class SparseLinearSolvePyTorch(Function):
    """Iterative solve with adjoint gradient support (linear_solve.py:283-324)."""

    @staticmethod
    def forward(ctx, val, row, col, shape, b, method, atol, rtol, maxiter, preconditioner,
                mixed_precision):
        u = pytorch_solve(val, row, col, shape, b, method=method, atol=atol, rtol=rtol,
                          maxiter=maxiter, preconditioner=preconditioner,
                          mixed_precision=mixed_precision)
        if mixed_precision and u.dtype != val.dtype:
            u = u.to(val.dtype)
        ctx.save_for_backward(val, row, col, u)
        ctx.shape = shape
        ctx.method = method
        ctx.atol = atol
        ctx.rtol = rtol
        ctx.maxiter = maxiter
        ctx.preconditioner = preconditioner
        ctx.mixed_precision = mixed_precision
        return u

    @staticmethod
    def backward(ctx, gradu):
        val, row, col, u = ctx.saved_tensors
        shape = ctx.shape
        # adjoint system A^T gradb = gradu on the swapped (col, row) pattern
        gradb = pytorch_solve(val, col, row, (shape[1], shape[0]), gradu.contiguous(),
                              method=ctx.method, atol=ctx.atol, rtol=ctx.rtol,
                              maxiter=ctx.maxiter, preconditioner=ctx.preconditioner,
                              mixed_precision=ctx.mixed_precision)
        if gradb.dtype != val.dtype:
            gradb = gradb.to(val.dtype)
        gradval = value_gradient(row, col, gradb, u, shape[0], shape[1])
        return gradval, None, None, None, gradb, None, None, None, None, None, None


def spsolve(val: torch.Tensor, row: torch.Tensor, col: torch.Tensor, shape: Tuple[int, int],
            b: torch.Tensor, backend: str = "auto", method: str = "auto", atol: float = 1e-10,
            maxiter: int = 10000, tol: float = 1e-12, matrix_type: str = "general",
            is_symmetric: bool = False, is_spd: bool = False, preconditioner: str = "jacobi",
            mixed_precision: bool = False, verbose: bool = False) -> torch.Tensor:
    """Solve A x = b with gradient support (linear_solve.py:374-623), pytorch
    backend only. The backend forces rtol = 1e-10 as torch-sla does
    (linear_solve.py:562)."""
    assert val.dim() == 1, f"val must be 1D tensor, got {val.dim()}"
    assert row.dim() == 1, f"row must be 1D tensor, got {row.dim()}"
    assert col.dim() == 1, f"col must be 1D tensor, got {col.dim()}"
    assert b.dim() in (1, 2), f"b must be 1D or 2D tensor, got {b.dim()}"
    assert shape[0] > 0, f"shape[0] must be positive, got {shape[0]}"
    assert shape[1] > 0, f"shape[1] must be positive, got {shape[1]}"
    assert val.size(0) == row.size(0), "val and row must have same size"
    assert val.size(0) == col.size(0), "val and col must have same size"
    assert b.size(0) == shape[0], "b and shape[0] must have same size"
    assert val.dtype == b.dtype, "val and b must have same dtype"

    if backend == "auto" and method != "auto":
        if method.startswith("pytorch_"):
            backend, method = "pytorch", method[len("pytorch_"):]
        elif method == "pytorch":
            backend, method = "pytorch", "auto"
    if backend == "auto":
        backend = "pytorch"
    if backend != "pytorch":
        raise ValueError(f"Unknown backend: {backend}. torch_sla_b200 provides the "
                         "'pytorch' backend only")
    if method == "auto":
        method = select_method(backend, is_symmetric=is_symmetric, is_spd=is_spd)
    valid = BACKEND_METHODS[backend]
    if method not in valid:
        raise ValueError(f"Method '{method}' not supported by backend '{backend}'. "
                         f"Available methods: {valid}")
    if verbose:
        dtype_str = str(val.dtype).replace("torch.", "")
        print(f"[torch-sla] solve: n={shape[0]}, nnz={val.numel()}, dtype={dtype_str}, "
              f"device={val.device.type}, symmetric={bool(is_symmetric)}, spd={bool(is_spd)}, "
              f"backend={backend}, method={method}")
    if val.dtype != torch.float64:
        warnings.warn("Using float64 is recommended for good precision with iterative solvers")
    rtol = 1e-10
    return SparseLinearSolvePyTorch.apply(val, row, col, shape, b, method, atol, rtol, maxiter,
                                          preconditioner, mixed_precision)
