"""Halo exchange and row-sharded SpMV (torch_sla/distributed/matvec.py:26-303)
on the libsla_b200 shard kernels: pack -> grouped NCCL send/recv on a side
stream overlapped with the interior rows -> unpack -> boundary rows."""
from __future__ import annotations

import torch

from .. import _lib as L
from .comm import communicators


def halo_exchange(D, x: torch.Tensor, partition=None) -> torch.Tensor:
    """Fill the halo slots x[num_owned:] from the neighbours, in place
    (matvec.py:26-93)."""
    plan = D._shard_plan()
    L.require_cuda(x)
    if x.numel() != plan.n_owned + plan.n_halo or not x.is_contiguous():
        raise ValueError("halo_exchange expects a contiguous [num_owned + num_halo] vector")
    comms = communicators(D._group)
    L.check("sla_halo_exchange", L.lib().sla_halo_exchange(
        comms.halo, plan.plan, L.dtype_code(x.dtype), L.ptr(x), L.ptr(plan.sendbuf),
        L.ptr(plan.recvbuf), L.stream_handle(x.device)))
    return x


def shard_matvec(D, x_owned: torch.Tensor) -> torch.Tensor:
    """Owned-row slice of A x (matvec.py:235-303); x is the owned slice or the
    padded local vector."""
    plan = D._shard_plan()
    L.require_cuda(x_owned)
    no, nl = plan.n_owned, plan.n_owned + plan.n_halo
    xp = torch.empty(max(nl, 1), dtype=plan.dtype, device=plan.device)[:nl]
    if x_owned.shape[0] == no:
        xp[:no].copy_(x_owned)
    elif x_owned.shape[0] == nl:
        xp.copy_(x_owned)
    else:
        raise ValueError(f"x shape[0]={x_owned.shape[0]}, expected num_owned={no} or "
                         f"num_local={nl}")
    y = torch.empty(max(no, 1), dtype=plan.dtype, device=plan.device)[:no]
    comms = communicators(D._group)
    L.check("sla_shard_spmv", L.lib().sla_shard_spmv(
        comms.halo, plan.plan, plan.code, plan.sell_int.ref(), plan.sell_bnd.ref(), L.ptr(xp),
        L.ptr(y), L.ptr(plan.sendbuf), L.ptr(plan.recvbuf), L.stream_handle(plan.device)))
    return y


def matmul_row_shard(D, x):
    """D @ x for the row-storage layout (matvec.py:173-203)."""
    from .core import _is_wrapped
    x_local = x.to_local() if _is_wrapped(x) else x
    y = shard_matvec(D, x_local)
    return D._wrap(y) if _is_wrapped(x) else y
