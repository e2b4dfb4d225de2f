"""Same-pattern batched solve with autograd (torch_sla/batch_solve.py:46-256).

method='cg' runs the batched kernel (values interleaved [nnz][B], one
column index serving the whole batch); the backward pass is the batched CG
on the swapped pattern plus one fused value-gradient gather.
"""
from __future__ import annotations

from typing import Tuple

import torch
from torch.autograd.function import Function

from .backends.pytorch_backend import batched_cg_same_pattern, pytorch_solve
from ._csr import coo_value_grad

_PYTORCH_METHODS = ["cg", "bicgstab"]


class BatchSparseLinearSolveSameLayout(Function):
    """A_i x_i = b_i for matrices sharing (row, col) (batch_solve.py:46-177)."""

    @staticmethod
    def forward(ctx, val_batch, row, col, shape, b_batch, method, atol, maxiter, rtol=1e-6):
        m, n = shape
        if method == "cg":
            u_batch = batched_cg_same_pattern(val_batch, row, col, (m, n), b_batch, atol=atol,
                                              rtol=rtol, maxiter=maxiter)
        elif method in _PYTORCH_METHODS:
            u_batch = torch.stack([
                pytorch_solve(val_batch[i], row, col, (m, n), b_batch[i], method=method,
                              atol=atol, maxiter=maxiter)
                for i in range(val_batch.size(0))], dim=0)
        else:
            raise ValueError(f"Unknown method: {method}")
        ctx.save_for_backward(val_batch, row, col, u_batch)
        ctx.A_shape = shape
        ctx.method = method
        ctx.atol = atol
        ctx.maxiter = maxiter
        ctx.rtol = rtol
        return u_batch

    @staticmethod
    def backward(ctx, gradu_batch):
        val_batch, row, col, u_batch = ctx.saved_tensors
        m, n = ctx.A_shape
        gradu_batch = gradu_batch.contiguous()
        if ctx.method == "cg":
            gradb_batch = batched_cg_same_pattern(val_batch, col, row, (n, m), gradu_batch,
                                                  atol=ctx.atol, rtol=ctx.rtol,
                                                  maxiter=ctx.maxiter)
        else:
            gradb_batch = torch.stack([
                pytorch_solve(val_batch[i], col, row, (n, m), gradu_batch[i], method=ctx.method,
                              atol=ctx.atol, maxiter=ctx.maxiter)
                for i in range(val_batch.size(0))], dim=0)
        B = int(val_batch.size(0))
        gradval_batch = coo_value_grad(row.to(torch.int64).contiguous(),
                                       col.to(torch.int64).contiguous(), gradb_batch, u_batch,
                                       m, n, K=1, batch=B).reshape(B, -1)
        return gradval_batch, None, None, None, gradb_batch, None, None, None, None


def spsolve_batch_same_layout(val_batch: torch.Tensor, row: torch.Tensor, col: torch.Tensor,
                              shape: Tuple[int, int], b_batch: torch.Tensor,
                              method: str = "bicgstab", atol: float = 1e-10,
                              maxiter: int = 10000, rtol: float = 1e-6) -> torch.Tensor:
    """Batch solve of matrices with one sparsity pattern (batch_solve.py:180-256).

    `rtol` is an addition: torch-sla always uses batched_cg_same_pattern's
    default 1e-6 here; passing it explicitly reaches tighter tolerances.
    """
    assert val_batch.dim() == 2, f"val_batch must be 2D [batch, nnz], got {val_batch.dim()}D"
    assert b_batch.dim() == 2, f"b_batch must be 2D [batch, m], got {b_batch.dim()}D"
    assert val_batch.size(0) == b_batch.size(0), "Batch sizes must match"
    assert val_batch.size(1) == row.size(0), "val_batch[1] must equal nnz"
    assert val_batch.size(1) == col.size(0), "val_batch[1] must equal nnz"
    assert b_batch.size(1) == shape[0], "b_batch[1] must equal m"
    return BatchSparseLinearSolveSameLayout.apply(val_batch, row, col, shape, b_batch, method,
                                                  atol, maxiter, rtol)
