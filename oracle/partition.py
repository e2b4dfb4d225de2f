"""numpy restatement of torch-sla's row partition maps (test infrastructure
only). Integer maps; compared bit-exactly against the product and the
reference fixtures."""
from __future__ import annotations

import numpy as np


def partition_simple(num_nodes: int, num_parts: int) -> np.ndarray:
    """partition.py:115-120: rank k owns the k-th ceil(N/P)-sized slice."""
    per = (num_nodes + num_parts - 1) // num_parts
    return np.minimum(np.arange(num_nodes, dtype=np.int64) // per, num_parts - 1)


def find_halo_nodes(row, col, ids, pid):
    """partition.py:373-423. Halo = sorted unique off-rank endpoints of every
    COO entry with exactly one owned endpoint; send_map[nb] = sorted unique
    owned endpoints of those entries whose other endpoint nb owns."""
    row = np.asarray(row, dtype=np.int64)
    col = np.asarray(col, dtype=np.int64)
    owned = ids == pid
    ro, co = owned[row], owned[col]
    m1 = ro & ~co
    m2 = co & ~ro
    halo_pts = np.concatenate([col[m1], row[m2]])
    mine = np.concatenate([row[m1], col[m2]])
    nbr = ids[halo_pts]
    halo = np.unique(halo_pts)
    send = {int(q): np.unique(mine[nbr == q]) for q in np.unique(nbr)}
    return halo, send


def build_partition(row, col, num_nodes, ids, pid):
    """partition.py:317-370: local order [owned ascending, halo ascending];
    recv_indices[nb] = local slots of halo nodes owned by nb (ascending
    global id); send_indices[nb] = local slots of send_map[nb]."""
    ids = np.asarray(ids, dtype=np.int64)
    owned = np.nonzero(ids == pid)[0].astype(np.int64)
    halo, send = find_halo_nodes(row, col, ids, pid)
    local = np.concatenate([owned, halo])
    g2l = np.full(num_nodes, -1, dtype=np.int64)
    g2l[local] = np.arange(local.size, dtype=np.int64)
    h2l = np.full(num_nodes, -1, dtype=np.int64)
    h2l[halo] = np.arange(halo.size, dtype=np.int64) + owned.size
    recv = {}
    for q in send:
        loc = h2l[np.nonzero(ids == q)[0]]
        recv[q] = loc[loc >= 0]
    return {
        "partition_id": int(pid),
        "owned_nodes": owned,
        "halo_nodes": halo,
        "local_nodes": local,
        "neighbor_partitions": sorted(send.keys()),
        "send_indices": {q: g2l[v] for q, v in send.items()},
        "recv_indices": recv,
        "global_to_local": g2l,
    }


def extract_partition(val, row, col, part):
    """sparse_tensor/convert.py:72-130: keep owned-row entries whose column is
    local, in local coordinates."""
    g2l = part["global_to_local"]
    no = part["owned_nodes"].size
    rl = g2l[np.asarray(row, dtype=np.int64)]
    cl = g2l[np.asarray(col, dtype=np.int64)]
    keep = (rl >= 0) & (rl < no) & (cl >= 0)
    return np.asarray(val)[keep], rl[keep], cl[keep]
