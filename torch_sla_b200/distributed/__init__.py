"""Row-partitioned (Shard(0)) distributed solve path: DSparseTensor, halo
exchange and the shard CG/BiCGStab, one process per GPU over NCCL."""
from ..partition import (Partition, build_partition, build_partition_from_rows, find_halo_nodes,
                         partition_simple, resolve_partition_ids)
from .collectives import gather_owned_to_global
from .comm import communicators, destroy_all
from .core import DSparseSpec, DSparseTensor, OwnedShard, VertexShard
from .matvec import (halo_exchange, matmul_row_shard, reverse_halo_exchange, shard_matvec,
                     shard_rmatvec)
from .solve import bicgstab_shard, cg_shard, make_preconditioner

__all__ = ["DSparseTensor", "DSparseSpec", "VertexShard", "OwnedShard", "Partition",
           "partition_simple", "build_partition", "build_partition_from_rows", "find_halo_nodes",
           "resolve_partition_ids", "gather_owned_to_global", "halo_exchange", "shard_matvec",
           "matmul_row_shard", "reverse_halo_exchange", "shard_rmatvec", "cg_shard", "bicgstab_shard", "make_preconditioner",
           "communicators", "destroy_all"]
