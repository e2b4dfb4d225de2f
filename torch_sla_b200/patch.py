"""Plug the B200 kernels into an installed torch-sla.

`install()` rebinds the hot-path functions of a loaded `torch_sla` package
so CUDA tensors run on libsla_b200 while CPU tensors keep torch-sla's own CPU
implementation (that CPU path is torch-sla's, not a fallback of this
package). The names rebound are torch-sla's patch points: `pytorch_solve` is
bound by name in `linear_solve.py:60`, the batched CG and the shard
functions are imported lazily at call time (`batch_solve.py:72,135`,
`distributed/core.py:1693, 2013-2023`), so rebinding the module attributes
is enough.
"""
from __future__ import annotations

import functools


def _cuda_first(ours, theirs):
    @functools.wraps(theirs)
    def call(*args, **kwargs):
        tensors = [a for a in list(args) + list(kwargs.values()) if hasattr(a, "is_cuda")]
        if tensors and tensors[0].is_cuda:
            return ours(*args, **kwargs)
        return theirs(*args, **kwargs)
    call.__wrapped_b200__ = ours
    return call


def install(torch_sla=None):
    """Rebind torch-sla's pytorch-backend and shard hot path. Returns the list
    of rebound attributes."""
    if torch_sla is None:
        import torch_sla  # noqa: F401
    import importlib
    from .backends import pytorch_backend as ours
    from .distributed import solve as our_shard
    from .distributed import matvec as our_matvec
    from .distributed.core import _ShardPlan, check_halo_symmetry

    ref_pb = importlib.import_module("torch_sla.backends.pytorch_backend")
    ref_ls = importlib.import_module("torch_sla.linear_solve")
    done = []
    for name in ("pytorch_solve", "batched_cg_same_pattern", "pcg_solve_fused",
                 "pbicgstab_solve"):
        wrapped = _cuda_first(getattr(ours, name), getattr(ref_pb, name))
        setattr(ref_pb, name, wrapped)
        done.append(f"torch_sla.backends.pytorch_backend.{name}")
    ref_ls.pytorch_solve = ref_pb.pytorch_solve
    done.append("torch_sla.linear_solve.pytorch_solve")

    try:
        ref_core = importlib.import_module("torch_sla.distributed.core")
        ref_dsolve = importlib.import_module("torch_sla.distributed.solve")
        ref_dmv = importlib.import_module("torch_sla.distributed.matvec")
    except ImportError:
        return done
    DS = ref_core.DSparseTensor

    def _shard_plan(self):
        plan = getattr(self, "_plan_b200", None)
        if plan is None:
            plan = _ShardPlan(self)
            check_halo_symmetry(plan, getattr(self, "_group", None))
            plan.enable_p2p()
            self._plan_b200 = plan
        return plan

    if not hasattr(DS, "_group"):
        DS._group = None
    DS._shard_plan = _shard_plan

    def _shard_pc(theirs):
        @functools.wraps(theirs)
        def make(D, kind, **kw):
            if D._local_tensor.values.is_cuda:
                return our_shard.make_preconditioner(D, kind, **kw)
            return theirs(D, kind, **kw)
        return make

    ref_dsolve.make_preconditioner = _shard_pc(ref_dsolve.make_preconditioner)
    for name in ("cg_shard", "bicgstab_shard"):
        setattr(ref_dsolve, name, _cuda_first(getattr(our_shard, name), getattr(ref_dsolve, name)))
        done.append(f"torch_sla.distributed.solve.{name}")
    # shard_matvec / shard_rmatvec are imported lazily by DSparseTensor
    # (core.py:2013-2023); the halo exchanges are module globals of matvec.py
    for name in ("shard_matvec", "shard_rmatvec", "halo_exchange", "reverse_halo_exchange"):
        setattr(ref_dmv, name, _cuda_first(getattr(our_matvec, name), getattr(ref_dmv, name)))
        done.append(f"torch_sla.distributed.matvec.{name}")
    return done
