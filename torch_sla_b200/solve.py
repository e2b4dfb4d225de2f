"""Unified `solve()` and the `SolverConfig` scope (torch_sla/solve.py:134-543),
restricted to the pytorch backend and DSparseTensor dispatch."""
from __future__ import annotations

import threading
from dataclasses import dataclass, fields
from typing import Any, NamedTuple, Optional, Tuple

import torch

_UNSET = object()
_tls = threading.local()


def _stack():
    if not hasattr(_tls, "stack"):
        _tls.stack = []
    return _tls.stack


def _active_defaults() -> dict:
    """Merged kwargs of the active SolverConfig scopes, innermost wins."""
    out: dict = {}
    for cfg in _stack():
        out.update(cfg._explicit())
    return out


@dataclass
class SolverConfig:
    """Thread-local default solver kwargs used as a context manager."""
    method: Any = _UNSET
    backend: Any = _UNSET
    preconditioner: Any = _UNSET
    atol: Any = _UNSET
    rtol: Any = _UNSET
    maxiter: Any = _UNSET
    verbose: Any = _UNSET
    mixed_precision: Any = _UNSET

    def _explicit(self) -> dict:
        return {f.name: getattr(self, f.name) for f in fields(self)
                if getattr(self, f.name) is not _UNSET}

    def __enter__(self):
        _stack().append(self)
        return self

    def __exit__(self, *exc):
        _stack().pop()
        return False


class SolveInfo(NamedTuple):
    iter_count: int
    residual: float
    converged: bool
    method: str
    backend: str


def _coerce_to_coo(A, shape=None, device=None, dtype=None):
    from .sparse_tensor import SparseTensor
    if isinstance(A, SparseTensor):
        M, N = A.sparse_shape
        return A.values, A.row_indices, A.col_indices, (M, N)
    if isinstance(A, tuple) and len(A) == 4:
        return A
    if isinstance(A, torch.Tensor) and A.is_sparse:
        A = A.coalesce()
        idx = A.indices()
        return A.values(), idx[0], idx[1], tuple(A.shape)
    raise TypeError("torch_sla_b200.solve accepts SparseTensor, (val, row, col, shape) or a "
                    "torch sparse COO tensor")


def solve(A, b: torch.Tensor, *, shape: Optional[Tuple[int, int]] = None, method: Any = _UNSET,
          backend: Any = _UNSET, preconditioner: Any = _UNSET, atol: Any = _UNSET,
          rtol: Any = _UNSET, maxiter: Any = _UNSET, x0: Any = _UNSET,
          matrix_type: Any = _UNSET, mixed_precision: Any = _UNSET, return_info: Any = _UNSET,
          verbose: Any = _UNSET, restart: Any = _UNSET):
    """Solve A x = b (torch_sla/solve.py:361-543): SolverConfig resolution,
    DSparseTensor -> shard solvers, everything else -> spsolve."""
    d = _active_defaults()
    given = dict(method=method, backend=backend, preconditioner=preconditioner, atol=atol,
                 rtol=rtol, maxiter=maxiter, x0=x0, matrix_type=matrix_type,
                 mixed_precision=mixed_precision, return_info=return_info, verbose=verbose,
                 restart=restart)
    hard = dict(method="auto", backend="auto", preconditioner=None, atol=1e-10, rtol=1e-6,
                maxiter=10_000, x0=None, matrix_type="general", mixed_precision=False,
                return_info=False, verbose=False, restart=30)
    kw = {k: (v if v is not _UNSET else d.get(k, hard[k])) for k, v in given.items()}

    try:
        from .distributed.core import DSparseTensor
    except ImportError:
        DSparseTensor = ()
    if DSparseTensor and isinstance(A, DSparseTensor) and A.spec is not None:
        m = "cg" if kw["method"] == "auto" else kw["method"]
        x = A.solve_distributed_shard(b, method=m, preconditioner=kw["preconditioner"],
                                      atol=kw["atol"], rtol=kw["rtol"], maxiter=kw["maxiter"],
                                      verbose=kw["verbose"])
        if not kw["return_info"]:
            return x
        return x, SolveInfo(0, float("nan"), True, m, "dsparse-shard")

    val, row, col, sh = _coerce_to_coo(A, shape=shape)
    pc = kw["preconditioner"]
    pc_str = "none" if pc is None else (pc if isinstance(pc, str) else getattr(pc, "kind", pc))
    from .linear_solve import spsolve
    x = spsolve(val, row, col, sh, b, backend=kw["backend"], method=kw["method"],
                atol=kw["atol"], maxiter=kw["maxiter"], matrix_type=kw["matrix_type"],
                preconditioner=pc_str, mixed_precision=kw["mixed_precision"],
                verbose=kw["verbose"])
    if not kw["return_info"]:
        return x
    from .backends.pytorch_backend import last_solve_info
    li = last_solve_info()
    return x, SolveInfo(int(li.get("iterations", 0)), float(li.get("residual", float("nan"))),
                        li.get("status", 1) == 0, kw["method"], "pytorch")
