"""`DSparseTensor`, the row-partitioned (VertexShard) distributed sparse
matrix of torch-sla (torch_sla/distributed/core.py:176-2036), reduced to the
solve hot path: partition / from_sparse_local / scatter / `D @ x` /
solve_distributed_shard, with the shard kernels of libsla_b200 underneath.

Vectors crossing the API are `OwnedShard`s (the owned-row slice of a global
vector, whose full_tensor() scatters by owned global ids, as torch-sla's
_OwnedShardDTensor does) or plain owned-slice tensors; any object with
`to_local()` (a torch DTensor) is accepted as input.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from typing import Any, Optional, Tuple

import torch
import torch.distributed as dist

from .. import _lib as L
from .._csr import DeviceCSR
from ..partition import (Partition, build_partition, build_partition_from_rows,
                         resolve_partition_ids, simple_range)
from ..sparse_tensor import SparseTensor
from .collectives import gather_owned_to_global


@dataclass(frozen=True)
class VertexShard:
    """Row-storage vertex partition (distributed/core.py:176-205)."""
    partition: Optional[Partition] = None

    def __eq__(self, other):
        if not isinstance(other, VertexShard):
            return False
        a = self.partition.partition_id if self.partition else None
        b = other.partition.partition_id if other.partition else None
        return a == b

    def __hash__(self):
        return hash(("VertexShard", self.partition.partition_id if self.partition else -1))


@dataclass(frozen=True)
class DSparseSpec:
    placement: VertexShard
    mesh: Any
    global_shape: Tuple[int, int]


def _group_of(mesh):
    if mesh is None:
        return None
    get = getattr(mesh, "get_group", None)
    if get is not None:
        try:
            return get()
        except Exception:
            return None
    return None


class OwnedShard:
    """Owned-row slice of a row-sharded global vector."""

    def __init__(self, local: torch.Tensor, owned_nodes: torch.Tensor, n_global: int, group=None):
        self._local = local
        self._owned = owned_nodes
        self._n_global = int(n_global)
        self._group = group

    def to_local(self) -> torch.Tensor:
        return self._local

    def full_tensor(self) -> torch.Tensor:
        return gather_owned_to_global(self._owned, self._local.contiguous(), self._n_global,
                                      self._group)

    @property
    def shape(self):
        return torch.Size([self._n_global])

    @property
    def dtype(self):
        return self._local.dtype

    @property
    def device(self):
        return self._local.device

    def _like(self, local):
        return OwnedShard(local, self._owned, self._n_global, self._group)

    @staticmethod
    def _val(o):
        return o._local if isinstance(o, OwnedShard) else o

    def __add__(self, o): return self._like(self._local + self._val(o))
    def __radd__(self, o): return self._like(self._val(o) + self._local)
    def __sub__(self, o): return self._like(self._local - self._val(o))
    def __rsub__(self, o): return self._like(self._val(o) - self._local)
    def __mul__(self, o): return self._like(self._local * self._val(o))
    def __rmul__(self, o): return self._like(self._val(o) * self._local)
    def __truediv__(self, o): return self._like(self._local / self._val(o))
    def __neg__(self): return self._like(-self._local)

    def norm(self) -> torch.Tensor:
        d = torch.dot(self._local, self._local)
        if dist.is_initialized():
            dist.all_reduce(d, group=self._group)
        return d.sqrt()

    def __repr__(self):
        return f"OwnedShard(local={tuple(self._local.shape)}, global={self._n_global})"


def _is_wrapped(x) -> bool:
    return hasattr(x, "to_local") and callable(x.to_local)


class _ShardPlan:
    """Device side of one rank: int32 CSR of the local block, SELL-32 views
    of the interior rows (no halo column) and of the boundary rows, the halo
    exchange plan and the Jacobi inverse of the owned rows."""

    def __init__(self, D: "DSparseTensor"):
        part = D._spec.placement.partition
        st = D._local_tensor
        L.require_cuda(st.values)
        self.device = st.values.device
        self.dtype = st.values.dtype
        self.code = L.dtype_code(self.dtype)
        no = int(part.owned_nodes.numel())
        nl = int(part.local_to_global.numel())
        self.n_owned, self.n_halo = no, nl - no
        self.csr = DeviceCSR(st.values, st.row_indices, st.col_indices, (nl, nl))
        counts = (self.csr.rowptr[1:] - self.csr.rowptr[:-1]).to(torch.int64)
        rows = torch.repeat_interleave(torch.arange(nl, device=self.device), counts)
        bmask = torch.zeros(max(no, 1), dtype=torch.bool, device=self.device)[:no]
        hit = rows[self.csr.colind.to(torch.int64) >= no]
        bmask[hit[hit < no]] = True
        self.boundary = bmask.nonzero().squeeze(-1).to(torch.int32)
        self.interior = (~bmask).nonzero().squeeze(-1).to(torch.int32)
        # interior rows read owned columns only (diagonal-offset layout when
        # the local stencil allows it); boundary rows keep explicit columns,
        # their halo columns do not sit on fixed diagonals
        self.sell_int = self.csr.sell(row_ids=self.interior, n_cols=no)
        self.sell_bnd = self.csr.sell(row_ids=self.boundary, diagonal=False)
        nbrs = sorted(int(q) for q in part.neighbor_partitions)
        self.neighbors = nbrs
        send = [part.send_indices[q].to(torch.int64) for q in nbrs]
        recv = [part.recv_indices[q].to(torch.int64) for q in nbrs]
        self.send_counts = [int(t.numel()) for t in send]
        self.recv_counts = [int(t.numel()) for t in recv]
        soff = [0]
        for n in self.send_counts:
            soff.append(soff[-1] + n)
        roff = [0]
        for n in self.recv_counts:
            roff.append(roff[-1] + n)
        self.n_send = soff[-1]
        self.send_index = (torch.cat(send).to(device=self.device, dtype=torch.int32)
                           if send else torch.zeros(1, dtype=torch.int32, device=self.device))
        recv_slots = (torch.cat(recv) - no) if recv else torch.zeros(0, dtype=torch.int64)
        if roff[-1] != self.n_halo:
            raise ValueError("torch_sla_b200: recv_indices do not cover the halo exactly")
        self.halo_src = None
        if recv_slots.numel() and not torch.equal(recv_slots.cpu(), torch.arange(self.n_halo)):
            src = torch.empty(self.n_halo, dtype=torch.int64)
            src[recv_slots.cpu()] = torch.arange(self.n_halo)
            self.halo_src = src.to(device=self.device, dtype=torch.int32)
        self._nb = (ctypes.c_int32 * max(len(nbrs), 1))(*nbrs)
        self._so = (ctypes.c_int64 * len(soff))(*soff)
        self._ro = (ctypes.c_int64 * len(roff))(*roff)
        self.plan = L.HaloPlan(len(nbrs), ctypes.cast(self._nb, ctypes.c_void_p).value,
                               ctypes.cast(self._so, ctypes.c_void_p).value,
                               ctypes.cast(self._ro, ctypes.c_void_p).value,
                               L.ptr(self.send_index), L.ptr(self.halo_src), no, self.n_halo)
        self.sendbuf = torch.empty(max(self.n_send, 1), dtype=self.dtype, device=self.device)
        self.recvbuf = torch.empty(max(self.n_halo, 1), dtype=self.dtype, device=self.device)
        self._dinv = {}
        self.p2p = None
        self._group = D._group

    def enable_p2p(self) -> None:
        """Map the peer-memory exchange buffers of the shard CG (collective;
        stays None when any rank cannot, or TORCH_SLA_B200_P2P=0). A one-rank
        group gets a plan too: it maps no peer and runs the same kernels as
        several ranks do."""
        if self.p2p is not None or os.environ.get("TORCH_SLA_B200_P2P", "1") == "0":
            return
        if not dist.is_initialized():
            return
        from .comm import communicators, register_p2p
        h = ctypes.c_void_p()
        L.check("sla_p2p_create", L.lib().sla_p2p_create(
            communicators(self._group).halo, ctypes.byref(self.plan), self.code,
            ctypes.byref(h)))
        if h.value:
            self.p2p = h
            register_p2p(h)

    def p2p_timers(self, reset: bool = True) -> dict | None:
        """Device-timer readings of the peer-memory CG kernels since the last
        reset (recorded only while profiling is on; None without a plan)."""
        if self.p2p is None:
            return None
        out = (ctypes.c_ulonglong * 8)()
        L.check("sla_p2p_profile_read", L.lib().sla_p2p_profile_read(self.p2p, int(reset), out, 8))
        keys = ("send_ns", "wait_ns", "sum_pap_ns", "sum_rr_ns", "ka_blocks", "iterations",
                "kp_blocks")
        return {k: int(out[i]) for i, k in enumerate(keys)}

    def dinv(self, kind: str):
        if kind not in self._dinv:
            self._dinv[kind] = self.csr.jacobi_inverse(L.SLA_JACOBI_CLAMP, n_rows=self.n_owned)
        return self._dinv[kind]


def check_halo_symmetry(plan: _ShardPlan, group=None) -> None:
    """Every rank's send count to q must equal q's recv count from it, or the
    grouped send/recv would wait forever: check on the host first."""
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return
    me = dist.get_rank(group)
    mine = {q: (s, r) for q, s, r in zip(plan.neighbors, plan.send_counts, plan.recv_counts)}
    allmaps = [None] * dist.get_world_size(group)
    dist.all_gather_object(allmaps, mine, group=group)
    for q, (s, _) in mine.items():
        other = allmaps[q].get(me)
        if other is None or other[1] != s:
            raise ValueError(f"torch_sla_b200: halo plan of ranks {me} and {q} disagree "
                             "(structurally non-symmetric pattern?)")


class DSparseTensor:
    """Row-partitioned sparse matrix with halo exchange (distributed/core.py)."""

    # ------------------------------------------------------------ construct
    @classmethod
    def from_sparse_local(cls, local_tensor: SparseTensor, mesh: Any, partition: Partition, *,
                          axis: int = 0, global_shape: Optional[Tuple[int, int]] = None):
        """Wrap a local (num_local x num_local) block and its Partition
        (distributed/core.py:393-465)."""
        if axis != 0:
            raise NotImplementedError("torch_sla_b200: only the row-storage VertexShard layout")
        if global_shape is None:
            n = int(partition.local_to_global.numel())
            global_shape = (n, n)
        self = cls.__new__(cls)
        self._shape = tuple(int(s) for s in global_shape)
        self._num_partitions = mesh.size() if mesh is not None else (
            dist.get_world_size() if dist.is_initialized() else 1)
        self._local_tensor = local_tensor
        self._device = local_tensor.values.device
        self._spec = DSparseSpec(placement=VertexShard(partition=partition), mesh=mesh,
                                 global_shape=self._shape)
        self._group = _group_of(mesh)
        self._plan = None
        return self

    @classmethod
    def partition(cls, A: SparseTensor, mesh: Any, *, partition_method: str = "simple",
                  coords=None, verbose: bool = False) -> "DSparseTensor":
        """Partition a global SparseTensor held by every rank
        (distributed/core.py:533-672). The 'simple' ids are a deterministic
        function of (N, world), so every rank computes the same ones."""
        group = _group_of(mesh)
        rank = dist.get_rank(group) if dist.is_initialized() else 0
        world = mesh.size() if mesh is not None else 1
        n = int(A.shape[0])
        ids = resolve_partition_ids(A.row_indices, A.col_indices, n, world,
                                    method=partition_method, coords=coords)
        part = build_partition(A.row_indices, A.col_indices, n, ids, rank)
        local = A.extract_partition(part)
        if verbose:
            print(f"[DSparseTensor] rank {rank}: owned={part.owned_nodes.numel()} "
                  f"halo={part.halo_nodes.numel()} neighbours={part.neighbor_partitions}")
        return cls.from_sparse_local(local, mesh, part, global_shape=tuple(A.shape))

    @classmethod
    def from_owned_rows(cls, val: torch.Tensor, row_g: torch.Tensor, col_g: torch.Tensor,
                        global_shape: Tuple[int, int], mesh: Any = None, group=None,
                        rank: Optional[int] = None, world: Optional[int] = None):
        """Build this rank's shard from the COO entries of its own rows only
        (global indices), under the 'simple' partition: the large-system path
        where no rank can hold the global matrix. The pattern must be
        structurally symmetric (every stencil here is)."""
        group = group if group is not None else _group_of(mesh)
        if rank is None:
            rank = dist.get_rank(group) if dist.is_initialized() else 0
        if world is None:
            world = dist.get_world_size(group) if dist.is_initialized() else 1
        n = int(global_shape[0])
        lo, hi = simple_range(n, world, rank)
        part = build_partition_from_rows(row_g, col_g, lo, hi, n, world, rank)
        g2l = part.global_to_local.to(val.device)
        rl = g2l[row_g.to(torch.int64)]
        cl = g2l[col_g.to(torch.int64)]
        nl = int(part.local_to_global.numel())
        local = SparseTensor(val, rl, cl, (nl, nl))
        D = cls.from_sparse_local(local, mesh, part, global_shape=tuple(global_shape))
        D._group = group
        return D

    # ------------------------------------------------------------ properties
    @property
    def spec(self) -> DSparseSpec:
        return self._spec

    @property
    def shape(self):
        return self._shape

    @property
    def nnz(self) -> int:
        return self._local_tensor.nnz

    @property
    def dtype(self):
        return self._local_tensor.dtype

    @property
    def device(self):
        return self._device

    @property
    def partition_info(self) -> Partition:
        return self._spec.placement.partition

    def __repr__(self) -> str:
        return (f"DSparseTensor(shape={tuple(self._shape)}, num_partitions={self._num_partitions}, "
                f"local_nnz={self.nnz}, device={self._device})")

    def _num_owned(self) -> int:
        return int(self._spec.placement.partition.owned_nodes.numel())

    def _shard_plan(self) -> _ShardPlan:
        if self._plan is None:
            self._plan = _ShardPlan(self)
            check_halo_symmetry(self._plan, self._group)
            self._plan.enable_p2p()
        return self._plan

    # --------------------------------------------------------------- vectors
    def scatter(self, global_vec: torch.Tensor) -> OwnedShard:
        """Owned slice of a global vector every rank holds (core.py:681-705)."""
        part = self._spec.placement.partition
        owned = part.owned_nodes.to(device=global_vec.device, dtype=torch.int64)
        return OwnedShard(global_vec[owned].contiguous(), part.owned_nodes, self._shape[0],
                          self._group)

    def _wrap(self, local):
        return OwnedShard(local, self._spec.placement.partition.owned_nodes, self._shape[0],
                          self._group)

    # ----------------------------------------------------------------- SpMV
    def __matmul__(self, x):
        """D @ x: halo exchange + local SpMV, owned-row result (core.py:1561-1601)."""
        from .matvec import matmul_row_shard
        return matmul_row_shard(self, x)

    def _shard_matvec(self, x_owned: torch.Tensor) -> torch.Tensor:
        from .matvec import shard_matvec
        return shard_matvec(self, x_owned)

    def _shard_rmatvec(self, y_owned: torch.Tensor) -> torch.Tensor:
        """Owned slice of A^T y (core.py:2017-2023)."""
        from .matvec import shard_rmatvec
        return shard_rmatvec(self, y_owned)

    def _shard_dot(self, u: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        d = torch.dot(u, v)
        if dist.is_initialized():
            dist.all_reduce(d, op=dist.ReduceOp.SUM, group=self._group)
        return d

    def _shard_norm(self, u: torch.Tensor) -> torch.Tensor:
        return self._shard_dot(u, u).sqrt()

    # ---------------------------------------------------------------- solve
    def solve_distributed_shard(self, b: Any, *, method: Any = None, preconditioner: Any = None,
                                atol: Any = None, rtol: Any = None, maxiter: Any = None,
                                restart: Any = None, verbose: Any = None) -> Any:
        """Shard(0) Krylov dispatcher (core.py:1613-1735): kwargs fall back to
        the active SolverConfig scope, then to atol 1e-10, rtol 0.0,
        maxiter 1000."""
        from ..solve import _active_defaults
        from . import solve as _ds
        if not dist.is_initialized():
            raise RuntimeError("solve_distributed_shard() requires torch.distributed to be "
                               "initialised.")
        d = _active_defaults()

        def pick(v, name, hard):
            return v if v is not None else d.get(name, hard)
        method = pick(method, "method", "cg")
        atol = pick(atol, "atol", 1e-10)
        rtol = pick(rtol, "rtol", 0.0)
        maxiter = pick(maxiter, "maxiter", 1000)
        verbose = pick(verbose, "verbose", False)
        if preconditioner is None and "preconditioner" in d:
            preconditioner = d["preconditioner"]
        M_apply = _ds.make_preconditioner(self, preconditioner)
        wrapped = _is_wrapped(b)
        b_owned = b.to_local() if wrapped else b
        ml = str(method).lower()
        common = dict(M_apply=M_apply, atol=atol, rtol=rtol, maxiter=maxiter, verbose=verbose)
        if ml in ("cg", "pcg"):
            x = _ds.cg_shard(self, b_owned, **common)
        elif ml == "bicgstab":
            x = _ds.bicgstab_shard(self, b_owned, **common)
        elif ml in ("gmres", "fgmres", "minres", "lsqr", "lsmr"):
            raise NotImplementedError(f"torch_sla_b200: distributed {method!r} is outside the "
                                      "B200 path (cg, bicgstab)")
        else:
            raise ValueError(f"Unknown distributed solve method {method!r}; expected one of cg, "
                             "bicgstab, gmres, fgmres, minres, lsqr, lsmr.")
        return self._wrap(x) if wrapped else x

    def solve(self, b: Any, **kwargs) -> Any:
        """Sugar for solve_distributed_shard (core.py:1838-1875)."""
        return self.solve_distributed_shard(b, **kwargs)
