"""Partition maps built on the GPU from a rank's own rows are the same
integers as the CPU build (and as build_partition on the global pattern)."""
import pytest
import torch

from torch_sla_b200 import problems as P
from torch_sla_b200.partition import (build_partition, build_partition_from_rows,
                                      partition_simple, simple_range)

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world,rank", [(2, 0), (3, 1), (4, 3)])
def test_partition_from_rows_on_gpu_matches_cpu(dev, world, rank):
    m = 6
    dims = (m * world, 5, 4)
    n = dims[0] * dims[1] * dims[2]
    lo, hi = simple_range(n, world, rank)
    v, r, c = P.stencil27_rows(dims, rank * m, m, seed=4)
    cpu = build_partition_from_rows(r, c, lo, hi, n, world, rank)
    gpu = build_partition_from_rows(r.to(dev), c.to(dev), lo, hi, n, world, rank)
    assert gpu.owned_nodes.is_cuda
    vg, rg, cg = P.stencil27_rows(dims, 0, dims[0], seed=4)
    ref = build_partition(rg, cg, n, partition_simple(n, world), rank)
    for part in (cpu, gpu):
        assert part.neighbor_partitions == ref.neighbor_partitions
        for name in ("owned_nodes", "halo_nodes", "local_to_global", "global_to_local"):
            assert torch.equal(getattr(part, name).cpu(), getattr(ref, name)), name
        for q in ref.neighbor_partitions:
            assert torch.equal(part.send_indices[q].cpu(), ref.send_indices[q])
            assert torch.equal(part.recv_indices[q].cpu(), ref.recv_indices[q])
