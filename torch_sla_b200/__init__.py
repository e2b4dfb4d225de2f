"""torch_sla_b200: torch-sla's iterative-solve hot path on NVIDIA B200.

Drop-in for torch-sla's `pytorch` backend (CG / BiCGStab / batched CG, CSR
SpMV, the autograd adjoint solve) and for the row-sharded DSparseTensor
solvers. Host code mirrors torch-sla's Python interface; the compute runs in
libsla_b200.so (hand-written sm_100a kernels, C ABI in include/sla_b200.h).
"""
from . import _lib
from .backends.pytorch_backend import (CachedSparseMatrix, SolveResult, batched_cg_same_pattern,
                                       get_preconditioner, last_solve_info, pbicgstab_solve,
                                       pcg_solve_fused, pcg_solve_optimized, pytorch_solve)
from .batch_solve import BatchSparseLinearSolveSameLayout, spsolve_batch_same_layout
from .linear_solve import SparseLinearSolvePyTorch, spsolve
from .solve import SolverConfig, solve
from .sparse_tensor import SparseTensor

__version__ = "0.1.0"

__all__ = [
    "SparseTensor", "spsolve", "solve", "SolverConfig", "spsolve_batch_same_layout",
    "SparseLinearSolvePyTorch", "BatchSparseLinearSolveSameLayout", "pytorch_solve",
    "pcg_solve_fused", "pcg_solve_optimized", "pbicgstab_solve", "batched_cg_same_pattern",
    "CachedSparseMatrix", "SolveResult", "get_preconditioner", "last_solve_info",
]


def __getattr__(name):
    # importlib rather than `from . import distributed`: the latter checks
    # hasattr(package, "distributed") first, which re-enters this function.
    if name in ("DSparseTensor", "Partition", "distributed"):
        import importlib
        mod = importlib.import_module(__name__ + ".distributed")
        return mod if name == "distributed" else getattr(mod, name)
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
