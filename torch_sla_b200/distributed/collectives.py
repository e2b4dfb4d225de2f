"""Owned-slice -> global vector gather used by full_tensor() for verification
(torch_sla/distributed/collectives.py:28-101)."""
from __future__ import annotations

import torch
import torch.distributed as dist


def gather_owned_to_global(owned: torch.Tensor, val: torch.Tensor, n_global: int,
                           group=None) -> torch.Tensor:
    """Every rank receives the length-n_global vector holding each rank's
    values at its owned global ids (zeros elsewhere)."""
    device, dtype = val.device, val.dtype
    if not dist.is_initialized():
        out = torch.zeros(n_global, dtype=dtype, device=device)
        out[owned.to(device)] = val
        return out
    world = dist.get_world_size(group)
    n_local = torch.tensor([owned.numel()], dtype=torch.int64, device=device)
    sizes = [torch.zeros_like(n_local) for _ in range(world)]
    dist.all_gather(sizes, n_local, group=group)
    sizes = torch.cat(sizes)
    width = int(sizes.max().item())
    out = torch.zeros(n_global, dtype=dtype, device=device)
    if width == 0:
        return out
    idx = torch.zeros(width, dtype=torch.int64, device=device)
    vals = torch.zeros(width, dtype=dtype, device=device)
    idx[: owned.numel()] = owned.to(device=device, dtype=torch.int64)
    vals[: val.numel()] = val
    all_idx = [torch.empty_like(idx) for _ in range(world)]
    all_val = [torch.empty_like(vals) for _ in range(world)]
    dist.all_gather(all_idx, idx, group=group)
    dist.all_gather(all_val, vals, group=group)
    for k in range(world):
        n = int(sizes[k])
        out[all_idx[k][:n]] = all_val[k][:n]
    return out
