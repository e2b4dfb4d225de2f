"""`SparseTensor`: the COO container of torch-sla (sparse_tensor/core.py),
reduced to what the solve hot path touches: construction, `solve`, `@`,
the structural checks `solve` runs first, and `extract_partition`.

`A @ x` and `A.solve(b)` run on libsla_b200 kernels; a CPU SparseTensor can
be built and inspected, but computing with it raises (no CPU fallback).
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import _lib as L
from ._csr import DeviceCSR, coo_value_grad


class _SpMV(torch.autograd.Function):
    """y = A x with gradients for x (A^T y) and the COO values (y[row] x[col])."""

    @staticmethod
    def forward(ctx, values, x, st):
        ctx.st = st
        ctx.save_for_backward(values, x)
        return st._csr().matvec(x.to(values.dtype))

    @staticmethod
    def backward(ctx, gy):
        values, x = ctx.saved_tensors
        st = ctx.st
        gy = gy.contiguous()
        gx = gval = None
        if ctx.needs_input_grad[1]:
            gx = st._csr_t().matvec(gy)
        if ctx.needs_input_grad[0]:
            M, N = st.sparse_shape
            gval = coo_value_grad(st._row64(), st._col64(), -gy, x.to(values.dtype), M, N)
        return gval, gx, None


class SparseTensor:
    """COO sparse matrix [..., M, N] (torch_sla/sparse_tensor/core.py:16-250)."""

    def __init__(self, values: torch.Tensor, row_indices: torch.Tensor,
                 col_indices: torch.Tensor, shape: Tuple[int, ...], sparse_dim=None):
        if len(shape) < 2:
            raise ValueError("shape must have at least 2 dims (M, N)")
        self.values = values
        self.row_indices = row_indices
        self.col_indices = col_indices
        self._shape = tuple(int(s) for s in shape)
        if row_indices.dim() != 1 or col_indices.dim() != 1 or row_indices.numel() != col_indices.numel():
            raise ValueError("row_indices and col_indices must be 1-D of equal length")
        if values.shape[-1] != row_indices.numel():
            raise ValueError("values' last dim must equal nnz")
        if tuple(values.shape[:-1]) != self.batch_shape:
            raise ValueError(f"values shape {tuple(values.shape)} does not match batch shape "
                             f"{self.batch_shape}")
        self._is_symmetric_cache = None
        self._is_positive_definite_cache = None
        self._cache = {}

    # --------------------------------------------------------------- shapes
    @property
    def shape(self) -> Tuple[int, ...]:
        return self._shape

    @property
    def sparse_shape(self) -> Tuple[int, int]:
        return self._shape[-2], self._shape[-1]

    @property
    def batch_shape(self) -> Tuple[int, ...]:
        return self._shape[:-2]

    @property
    def is_batched(self) -> bool:
        return len(self.batch_shape) > 0

    @property
    def batch_size(self) -> int:
        n = 1
        for d in self.batch_shape:
            n *= d
        return n

    @property
    def is_block(self) -> bool:
        return False

    @property
    def is_square(self) -> bool:
        return self._shape[-2] == self._shape[-1]

    @property
    def nnz(self) -> int:
        return int(self.row_indices.numel())

    @property
    def dtype(self) -> torch.dtype:
        return self.values.dtype

    @property
    def device(self) -> torch.device:
        return self.values.device

    def __repr__(self) -> str:
        return (f"SparseTensor(shape={self.shape}, sparse={self.sparse_shape}, nnz={self.nnz}, "
                f"dtype={self.dtype}, device={self.device})")

    def to(self, device=None, dtype=None) -> "SparseTensor":
        v = self.values.to(device=device, dtype=dtype) if dtype else self.values.to(device)
        return SparseTensor(v, self.row_indices.to(device), self.col_indices.to(device), self._shape)

    def cuda(self, device=None) -> "SparseTensor":
        return self.to(torch.device("cuda", device) if isinstance(device, int) else (device or "cuda"))

    def cpu(self) -> "SparseTensor":
        return self.to("cpu")

    # --------------------------------------------------------------- caches
    def _row64(self):
        return self.row_indices.to(torch.int64).contiguous()

    def _col64(self):
        return self.col_indices.to(torch.int64).contiguous()

    def _csr(self) -> DeviceCSR:
        key = ("A", self.values.data_ptr(), self.values._version)
        c = self._cache.get("A")
        if c is None or c[0] != key:
            c = (key, DeviceCSR(self.values.detach(), self.row_indices, self.col_indices,
                                self.sparse_shape))
            self._cache["A"] = c
        return c[1]

    def _csr_t(self) -> DeviceCSR:
        key = ("AT", self.values.data_ptr(), self.values._version)
        c = self._cache.get("AT")
        if c is None or c[0] != key:
            M, N = self.sparse_shape
            c = (key, DeviceCSR(self.values.detach(), self.col_indices, self.row_indices, (N, M)))
            self._cache["AT"] = c
        return c[1]

    # ----------------------------------------------------------------- SpMV
    def __matmul__(self, x: torch.Tensor) -> torch.Tensor:
        """A @ x (sparse_tensor/matmul.py:10-85) on the SELL-32 SpMV kernel."""
        L.require_cuda(self.values, x)
        if self.is_batched:
            B = self.batch_size
            M, N = self.sparse_shape
            vals = self.values.reshape(B, self.nnz)
            if x.dim() == 1:
                xs = [x] * B
            else:
                xs = list(x.reshape(B, N, *x.shape[len(self.batch_shape) + 1:]))
            outs = [SparseTensor(vals[i], self.row_indices, self.col_indices, (M, N)) @ xs[i]
                    for i in range(B)]
            return torch.stack(outs).reshape(*self.batch_shape, *outs[0].shape)
        if x.dim() == 2:
            return torch.stack([self @ x[:, k] for k in range(x.shape[1])], dim=1)
        return _SpMV.apply(self.values, x, self)

    def matvec(self, x: torch.Tensor) -> torch.Tensor:
        return self @ x

    # ------------------------------------------------------- structure checks
    def is_symmetric(self, atol: float = 1e-8, rtol: float = 1e-5,
                     force_recompute: bool = False) -> torch.Tensor:
        """A == A^T within atol + rtol|a| (sparse_tensor/structural.py:63-95),
        compared on the coalesced CSR of A and of A^T."""
        if self._is_symmetric_cache is not None and not force_recompute:
            return self._is_symmetric_cache
        if not self.is_square:
            res = torch.tensor(False, device=self.device)
        elif self.is_batched:
            M, N = self.sparse_shape
            vals = self.values.reshape(self.batch_size, self.nnz)
            res = torch.stack([
                SparseTensor(vals[i], self.row_indices, self.col_indices, (M, N)).is_symmetric(atol, rtol)
                for i in range(self.batch_size)]).reshape(self.batch_shape)
        else:
            L.require_cuda(self.values)
            a, at = self._csr(), self._csr_t()
            same = (a.nnz == at.nnz and torch.equal(a.rowptr, at.rowptr)
                    and torch.equal(a.colind, at.colind))
            if same:
                diff = (a.vals - at.vals).abs()
                same = bool((diff <= atol + rtol * a.vals.abs()).all().item())
            res = torch.tensor(bool(same), device=self.device)
        self._is_symmetric_cache = res
        return res

    def is_positive_definite(self, method: str = "gershgorin",
                             force_recompute: bool = False) -> torch.Tensor:
        """Gershgorin sufficient test (sparse_tensor/structural.py:191-241)."""
        if self._is_positive_definite_cache is not None and not force_recompute:
            return self._is_positive_definite_cache
        if method != "gershgorin":
            raise NotImplementedError("torch_sla_b200: only the Gershgorin PD check is provided")
        M, _ = self.sparse_shape
        row = self.row_indices.to(torch.int64)
        is_diag = row == self.col_indices.to(torch.int64)
        vals = self.values.reshape(self.batch_size, self.nnz)
        diag = torch.zeros(self.batch_size, M, dtype=vals.dtype, device=self.device)
        diag.scatter_(1, row[is_diag].unsqueeze(0).expand(self.batch_size, -1), vals[:, is_diag])
        off = torch.zeros_like(diag)
        off.scatter_add_(1, row[~is_diag].unsqueeze(0).expand(self.batch_size, -1),
                         vals[:, ~is_diag].abs())
        ok = ((diag > off) & (diag > 0)).all(dim=-1)
        res = ok.reshape(self.batch_shape) if self.is_batched else torch.tensor(
            bool(ok[0].item()), device=self.device)
        self._is_positive_definite_cache = res
        return res

    # ---------------------------------------------------------------- solve
    def solve(self, b: torch.Tensor, backend: str = "auto", method: str = "auto",
              atol: float = 1e-10, maxiter: int = 10000, tol: float = 1e-12,
              verbose: bool = False) -> torch.Tensor:
        """Solve A x = b (sparse_tensor/linalg.py:17-175): structural checks,
        then spsolve per matrix (a batched tensor loops over its members)."""
        if not self.is_square:
            raise ValueError("Matrix must be square for solve()")
        from .linear_solve import spsolve
        is_sym = bool(self.is_symmetric().all().item())
        is_pd = bool(self.is_positive_definite().all().item())
        is_spd = is_sym and is_pd
        M, N = self.sparse_shape
        if self.is_batched:
            vals_flat = self.values.reshape(-1, self.nnz)
            b_flat = b.reshape(-1, M)
            out = [spsolve(vals_flat[i], self.row_indices, self.col_indices, (M, N), b_flat[i],
                           backend=backend, method=method, atol=atol, maxiter=maxiter, tol=tol,
                           is_symmetric=is_sym, is_spd=is_spd, verbose=verbose and i == 0)
                   for i in range(vals_flat.size(0))]
            return torch.stack(out).reshape(*self.batch_shape, N)
        return spsolve(self.values, self.row_indices, self.col_indices, (M, N), b,
                       backend=backend, method=method, atol=atol, maxiter=maxiter, tol=tol,
                       is_symmetric=is_sym, is_spd=is_spd, verbose=verbose)

    # ------------------------------------------------------------ partition
    def extract_partition(self, partition) -> "SparseTensor":
        """Local (num_local x num_local) COO of one rank's owned rows
        (sparse_tensor/convert.py:72-130)."""
        if self.is_batched:
            raise ValueError("extract_partition() does not support batched SparseTensor.")
        dev = self.values.device
        g2l = partition.global_to_local.to(device=dev, dtype=torch.int64)
        num_owned = int(partition.owned_nodes.numel())
        num_local = num_owned + int(partition.halo_nodes.numel())
        rl = g2l[self.row_indices.to(device=dev, dtype=torch.int64)]
        cl = g2l[self.col_indices.to(device=dev, dtype=torch.int64)]
        keep = (rl >= 0) & (rl < num_owned) & (cl >= 0)
        return SparseTensor(self.values[keep], rl[keep], cl[keep], (num_local, num_local))
