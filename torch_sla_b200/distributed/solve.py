"""Shard(0) CG / BiCGStab and their preconditioners
(torch_sla/distributed/solve.py:32-436) on the fused shard kernels.

Each solve runs entirely inside libsla_b200: per iteration the search
direction is computed inside the SpMV gather, its halo values travel by
grouped NCCL send/recv while the interior rows compute, and the dot products
of each reduction point are combined by one small ncclAllReduce (CG: 2 per
iteration; BiCGStab: 3). On a single node both solvers instead store halo
values and dot products straight into the other GPUs' memory from inside
their kernels (sla_shard_cg_p2p: three launches per iteration -- the search
direction and the halo send, the SpMV, the update; sla_shard_bicgstab_p2p:
three). The stopping test runs every 10 iterations on
the allreduced norms, as in the reference.
"""
from __future__ import annotations

import ctypes
from typing import Any, Callable

import torch

from .. import _lib as L
from .comm import communicators

CHECK_EVERY = 10  # distributed/solve.py:318, 389


class ShardJacobi:
    """1 / clamp_min(diag, 1e-30) on the owned rows (distributed/solve.py:95-115)."""

    def __init__(self, D):
        self.dinv = D._shard_plan().dinv("jacobi")

    def __call__(self, r):
        return self.dinv * r


class ShardIdentity:
    dinv = None

    def __call__(self, r):
        return r


def make_preconditioner(D, kind: Any, *, omega: float = 1.0, degree: int = 2) -> Callable:
    """'jacobi' / None / 'none' (distributed/solve.py:32-263)."""
    if kind is None or (isinstance(kind, str) and kind.lower() == "none"):
        return ShardIdentity()
    if isinstance(kind, (ShardJacobi, ShardIdentity)):
        return kind
    if isinstance(kind, str) and kind.lower() == "jacobi":
        return ShardJacobi(D)
    raise NotImplementedError(f"torch_sla_b200: shard preconditioner {kind!r} is not provided "
                              "(available: jacobi, none)")


def _run(fn_name, D, b_owned, M_apply, atol, rtol, maxiter, verbose):
    plan = D._shard_plan()
    L.require_cuda(b_owned)
    no = plan.n_owned
    if b_owned.shape[0] != no:
        raise ValueError(f"b_owned size {b_owned.shape[0]} != num_owned {no}; Shard(0) solves "
                         "require b to be the local owned slice.")
    if not isinstance(M_apply, (ShardJacobi, ShardIdentity)):
        raise NotImplementedError("torch_sla_b200: the fused shard solvers take the "
                                  "preconditioners of make_preconditioner ('jacobi', 'none')")
    b = b_owned.to(plan.dtype).contiguous()
    x = torch.empty(max(no, 1), dtype=plan.dtype, device=plan.device)[:no]
    lib = L.lib()
    need = ctypes.c_size_t(0)
    L.check("sla_shard_krylov_workspace", lib.sla_shard_krylov_workspace(
        plan.code, no, plan.n_halo, plan.n_send, ctypes.byref(need)))
    ws = L.workspace(need.value, plan.device)
    info = L.SolveInfo()
    args = (ctypes.byref(plan.plan), plan.code, plan.sell_int.ref(), plan.sell_bnd.ref(),
            L.ptr(M_apply.dinv), L.ptr(b), L.ptr(x), float(atol), float(rtol), int(maxiter),
            CHECK_EVERY, L.ptr(ws), ws.numel(), ctypes.byref(info), L.stream_handle(plan.device))
    if getattr(plan, "p2p", None) is not None:
        fn_name += "_p2p"  # same algorithm on the peer-memory exchange buffers
        st = getattr(lib, fn_name)(plan.p2p, *args)
    else:
        comms = communicators(D._group)
        st = getattr(lib, fn_name)(comms.halo, comms.reduce, *args)
    L.check(fn_name, st)
    D._last_info = dict(iterations=int(info.iterations), residual=float(info.residual),
                        status=int(info.status))
    if verbose:
        print(f"[shard-{'PCG' if fn_name == 'sla_shard_cg' else 'PBiCGStab'}] "
              f"{info.iterations} iterations, ||r||={info.residual:.3e}")
    return x


class _ShardCGSolve(torch.autograd.Function):
    """x = A^{-1} b on the owned rows. CG needs A symmetric positive
    definite, so the adjoint system is A itself: the backward pass is one
    more distributed solve with the incoming gradient (the single-process
    adjoint of linear_solve.py:283-324, in Shard(0) space); every rank takes
    part in it."""

    @staticmethod
    def forward(ctx, b_owned, D, M_apply, atol, rtol, maxiter, verbose):
        ctx.D = D
        ctx.args = (M_apply, atol, rtol, maxiter, verbose)
        return _run("sla_shard_cg", D, b_owned.detach(), M_apply, atol, rtol, maxiter, verbose)

    @staticmethod
    def backward(ctx, g):
        M_apply, atol, rtol, maxiter, verbose = ctx.args
        gb = _run("sla_shard_cg", ctx.D, g.contiguous(), M_apply, atol, rtol, maxiter, verbose)
        return gb, None, None, None, None, None, None


def cg_shard(D, b_owned: torch.Tensor, *, M_apply: Callable, atol: float, rtol: float,
             maxiter: int, verbose: bool) -> torch.Tensor:
    """Preconditioned CG in Shard(0) space (distributed/solve.py:279-350);
    differentiable in b (adjoint solve on the same shards)."""
    if torch.is_grad_enabled() and b_owned.requires_grad:
        return _ShardCGSolve.apply(b_owned, D, M_apply, atol, rtol, maxiter, verbose)
    return _run("sla_shard_cg", D, b_owned, M_apply, atol, rtol, maxiter, verbose)


def bicgstab_shard(D, b_owned: torch.Tensor, *, M_apply: Callable, atol: float, rtol: float,
                   maxiter: int, verbose: bool) -> torch.Tensor:
    """Preconditioned BiCGStab in Shard(0) space (distributed/solve.py:356-436),
    including the reference's reuse of the SpMV output buffer: the p update
    of iteration k reads t of iteration k-1 where textbook BiCGStab reads v."""
    return _run("sla_shard_bicgstab", D, b_owned, M_apply, atol, rtol, maxiter, verbose)
