"""Row partition maps of the distributed path (torch_sla/partition.py:27-423):
the `Partition` struct, the contiguous 'simple' partitioner and the
owned/halo/send/recv maps, bit-exact with torch-sla's.

`build_partition_from_rows` is an addition for systems too large to hold
globally on each rank: for a contiguous owned row range of a structurally
symmetric pattern it derives the same maps from the owned rows' entries
alone (checked equal to `build_partition` in the tests).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Tuple

import torch


@dataclass
class Partition:
    """One rank's view of the global graph (partition.py:27-81)."""
    partition_id: int
    local_nodes: torch.Tensor
    owned_nodes: torch.Tensor
    halo_nodes: torch.Tensor
    neighbor_partitions: List[int]
    send_indices: Dict[int, torch.Tensor]
    recv_indices: Dict[int, torch.Tensor]
    global_to_local: torch.Tensor
    local_to_global: torch.Tensor

    def to(self, device) -> "Partition":
        return Partition(
            partition_id=self.partition_id,
            local_nodes=self.local_nodes.to(device),
            owned_nodes=self.owned_nodes.to(device),
            halo_nodes=self.halo_nodes.to(device),
            neighbor_partitions=list(self.neighbor_partitions),
            send_indices={k: v.to(device) for k, v in self.send_indices.items()},
            recv_indices={k: v.to(device) for k, v in self.recv_indices.items()},
            global_to_local=self.global_to_local.to(device),
            local_to_global=self.local_to_global.to(device),
        )


def partition_simple(num_nodes: int, num_parts: int) -> torch.Tensor:
    """Rank k owns the k-th ceil(N/P)-sized contiguous slice (partition.py:115-120)."""
    per = (num_nodes + num_parts - 1) // num_parts
    return torch.clamp(torch.arange(num_nodes, dtype=torch.int64) // per, max=num_parts - 1)


def simple_range(num_nodes: int, num_parts: int, rank: int) -> Tuple[int, int]:
    """[lo, hi) owned by `rank` under partition_simple."""
    per = (num_nodes + num_parts - 1) // num_parts
    lo = min(rank * per, num_nodes)
    hi = num_nodes if rank == num_parts - 1 else min((rank + 1) * per, num_nodes)
    return lo, hi


def resolve_partition_ids(row, col, num_nodes: int, num_parts: int, method: str,
                          coords=None) -> torch.Tensor:
    """'simple' (and 'auto' without coordinates) -- the partitioner of the
    B200 path (partition.py:285-314); graph/geometric partitioners are out of
    its scope."""
    if method == "auto" and coords is None:
        method = "simple"
    if method == "simple":
        return partition_simple(num_nodes, num_parts)
    raise NotImplementedError(f"torch_sla_b200: partition method {method!r} is not provided "
                              "(available: simple)")


def find_halo_nodes(row: torch.Tensor, col: torch.Tensor, partition_ids: torch.Tensor,
                    partition_id: int):
    """Halo = sorted unique off-rank endpoints of entries with exactly one
    owned endpoint; send_map[q] = sorted unique owned endpoints of the
    entries whose other endpoint q owns (partition.py:373-423)."""
    row = row.to(torch.int64).cpu()
    col = col.to(torch.int64).cpu()
    ids = partition_ids.cpu()
    owned = ids == partition_id
    ro, co = owned[row], owned[col]
    m1, m2 = ro & ~co, co & ~ro
    halo_pts = torch.cat([col[m1], row[m2]])
    mine = torch.cat([row[m1], col[m2]])
    nb = ids[halo_pts]
    halo_nodes = torch.unique(halo_pts, sorted=True)
    send_map: Dict[int, torch.Tensor] = {}
    for q in torch.unique(nb).tolist():
        send_map[int(q)] = torch.unique(mine[nb == q], sorted=True)
    return halo_nodes, send_map


def _assemble(pid: int, owned: torch.Tensor, halo: torch.Tensor, send_map: Dict[int, torch.Tensor],
              num_nodes: int, owner_of) -> Partition:
    dev = owned.device
    local = torch.cat([owned, halo])
    g2l = torch.full((num_nodes,), -1, dtype=torch.int64, device=dev)
    g2l[local] = torch.arange(local.numel(), dtype=torch.int64, device=dev)
    halo_owner = owner_of(halo)
    recv: Dict[int, torch.Tensor] = {}
    for q in send_map:
        # halo slots of the nodes q owns, ascending global id
        sel = (halo_owner == q).nonzero().squeeze(-1)
        recv[q] = sel + owned.numel()
    send = {q: g2l[nodes] for q, nodes in send_map.items()}
    return Partition(partition_id=pid, local_nodes=local, owned_nodes=owned, halo_nodes=halo,
                     neighbor_partitions=list(send_map.keys()), send_indices=send,
                     recv_indices=recv, global_to_local=g2l, local_to_global=local.clone())


def build_partition(row: torch.Tensor, col: torch.Tensor, num_nodes: int,
                    partition_ids: torch.Tensor, my_partition: int) -> Partition:
    """Owned/halo sets, global<->local maps and send/recv plans of one rank
    (partition.py:317-370). Local order: owned ascending, then halo ascending."""
    ids = partition_ids.cpu().to(torch.int64)
    owned = (ids == my_partition).nonzero().squeeze(-1)
    halo, send_map = find_halo_nodes(row, col, ids, my_partition)
    return _assemble(int(my_partition), owned, halo, send_map, num_nodes, lambda g: ids[g])


def build_partition_from_rows(row_g: torch.Tensor, col_g: torch.Tensor, lo: int, hi: int,
                              num_nodes: int, num_parts: int, my_partition: int) -> Partition:
    """build_partition for a 'simple' partition from the owned rows [lo, hi)
    only (their COO entries in global ids). Requires a structurally symmetric
    pattern, for which the entries with an owned column and an off-rank row
    mirror the owned-row entries. Runs on the device of the entries (the
    O(nnz) masks and sorts of a large shard stay on the GPU); the maps come
    back on that device."""
    per = (num_nodes + num_parts - 1) // num_parts
    owner = lambda g: torch.clamp(g // per, max=num_parts - 1)  # noqa: E731
    row_g = row_g.to(torch.int64)
    col_g = col_g.to(device=row_g.device, dtype=torch.int64)
    owned = torch.arange(lo, hi, dtype=torch.int64, device=row_g.device)
    off = (col_g < lo) | (col_g >= hi)
    halo_pts = col_g[off]
    mine = row_g[off]
    nb = owner(halo_pts)
    halo = torch.unique(halo_pts, sorted=True)
    send_map: Dict[int, torch.Tensor] = {}
    for q in torch.unique(nb).tolist():
        send_map[int(q)] = torch.unique(mine[nb == q], sorted=True)
    return _assemble(int(my_partition), owned, halo, send_map, num_nodes, owner)
