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


class _RowShardMatvec(torch.autograd.Function):
    """y = A x on the owned rows; the backward pass is the distributed
    adjoint A^T g (local transpose SpMV + reverse halo exchange), so every
    rank takes part in it."""

    @staticmethod
    def forward(ctx, x_owned, D):
        ctx.D = D
        return shard_matvec(D, x_owned)

    @staticmethod
    def backward(ctx, g):
        return shard_rmatvec(ctx.D, g.contiguous()), None


def matmul_row_shard(D, x):
    """D @ x for the row-storage layout (matvec.py:173-203); differentiable
    in an owned-size x."""
    from .core import _is_wrapped
    x_local = x.to_local() if _is_wrapped(x) else x
    if (torch.is_grad_enabled() and x_local.requires_grad
            and x_local.shape[0] == D._shard_plan().n_owned):
        y = _RowShardMatvec.apply(x_local, D)
    else:
        y = shard_matvec(D, x_local)
    return D._wrap(y) if _is_wrapped(x) else y


def _transpose_view(D):
    plan = D._shard_plan()
    if getattr(plan, "sell_t", None) is None:
        from .._csr import DeviceCSR
        st = D._local_tensor
        nl = plan.n_owned + plan.n_halo
        plan.csr_t = DeviceCSR(st.values, st.col_indices, st.row_indices, (nl, plan.n_owned))
        # sla_shard_rmatvec writes slot i to row i: no SELL-C-sigma reordering
        plan.sell_t = plan.csr_t.sell(sigma=1)
        plan.rev_send = torch.empty(max(plan.n_halo, 1), dtype=plan.dtype, device=plan.device)
        plan.rev_recv = torch.empty(max(plan.n_send, 1), dtype=plan.dtype, device=plan.device)
    return plan


def reverse_halo_exchange(D, w: torch.Tensor, partition=None) -> torch.Tensor:
    """Send the halo slots of w to their owners and add the incoming
    contributions onto the owned slots, in place (matvec.py:96-170)."""
    plan = _transpose_view(D)
    L.require_cuda(w)
    if w.numel() != plan.n_owned + plan.n_halo or not w.is_contiguous():
        raise ValueError("reverse_halo_exchange expects a contiguous [num_owned + num_halo] vector")
    comms = communicators(D._group)
    L.check("sla_reverse_halo_exchange", L.lib().sla_reverse_halo_exchange(
        comms.halo, plan.plan, L.dtype_code(w.dtype), L.ptr(w), L.ptr(plan.rev_send),
        L.ptr(plan.rev_recv), L.stream_handle(w.device)))
    return w


def shard_rmatvec(D, y_owned: torch.Tensor) -> torch.Tensor:
    """Owned slice of A^T y (matvec.py:306-348): local transpose SpMV, then the
    reverse halo exchange."""
    plan = _transpose_view(D)
    L.require_cuda(y_owned)
    if y_owned.shape[0] != plan.n_owned:
        raise ValueError(f"y shape[0]={y_owned.shape[0]}, expected num_owned={plan.n_owned}")
    y = y_owned.to(plan.dtype).contiguous()
    nl = plan.n_owned + plan.n_halo
    w = torch.empty(max(nl, 1), dtype=plan.dtype, device=plan.device)[:nl]
    comms = communicators(D._group)
    L.check("sla_shard_rmatvec", L.lib().sla_shard_rmatvec(
        comms.halo, plan.plan, plan.code, plan.sell_t.ref(), L.ptr(y), L.ptr(w),
        L.ptr(plan.rev_send), L.ptr(plan.rev_recv), L.stream_handle(plan.device)))
    return w[: plan.n_owned].contiguous()
