"""Synthetic sparse systems with the shapes, sizes and value distributions of
the solver workloads (structured-grid stencils in COO, nodes flattened
row-major with axis 0 slowest, as torch_sla/datasets/problems.py:50-103
lays them out). Generators take a `device`, so the same call builds the
matrix on the GPU for the solver and on the CPU for the oracle; random
inputs come from seeded CPU generators (or an integer hash) so both agree
bit for bit.
"""
from __future__ import annotations

import math
from typing import Sequence

import torch


def _strides(dims):
    s = [1] * len(dims)
    for a in range(len(dims) - 2, -1, -1):
        s[a] = s[a + 1] * dims[a + 1]
    return s


def grid_coo_rows(dims: Sequence[int], z0: int, nz_local: int, diag, edges,
                  dtype=torch.float64, device="cpu"):
    """Rows of the stencil COO whose axis-0 coordinate lies in
    [z0, z0 + nz_local), with GLOBAL indices: diagonal entries first, then one
    block per (axis, step, weight) coupling, only where the neighbour is
    in-bounds; couplings to the same neighbour stay separate entries (summed
    on coalesce). Returns (val, row, col)."""
    dims = tuple(int(d) for d in dims)
    st = _strides(dims)
    p = torch.arange(nz_local * st[0], device=device, dtype=torch.int64) + z0 * st[0]
    rows, cols = [p], [p]
    vals = [torch.full((p.numel(),), float(diag), dtype=dtype, device=device)]
    for axis, step, w in edges:
        coord = (p // st[axis]) % dims[axis]
        nb = coord + step
        keep = (nb >= 0) & (nb < dims[axis])
        src = p[keep]
        rows.append(src)
        cols.append(src + step * st[axis])
        vals.append(torch.full((src.numel(),), float(w), dtype=dtype, device=device))
    return torch.cat(vals), torch.cat(rows), torch.cat(cols)


def grid_coo(dims: Sequence[int], diag, edges, dtype=torch.float64, device="cpu"):
    """The whole stencil COO (all rows) in grid_coo_rows' entry order."""
    dims = tuple(int(d) for d in dims)
    return grid_coo_rows(dims, 0, dims[0], diag, edges, dtype, device)


def axis_edges(ndim: int, w):
    return [(a, s, w) for a in range(ndim) for s in (1, -1)]


def poisson_2d_5pt(m: int, dtype=torch.float64, device="cpu"):
    """5-point Dirichlet Laplacian on m x m (diag 4, off -1)."""
    v, r, c = grid_coo((m, m), 4.0, axis_edges(2, -1.0), dtype, device)
    return v, r, c, (m * m, m * m)


def poisson_3d_7pt(dims, dtype=torch.float64, device="cpu"):
    """7-point Laplacian on dims = (nz, ny, nx) (diag 6, off -1)."""
    if isinstance(dims, int):
        dims = (dims, dims, dims)
    v, r, c = grid_coo(dims, 6.0, axis_edges(3, -1.0), dtype, device)
    n = math.prod(dims)
    return v, r, c, (n, n)


def rhs_uniform_pm1(n: int, seed: int, dtype=torch.float64):
    """b ~ U(-1, 1) from a CPU generator."""
    g = torch.Generator().manual_seed(seed)
    return (torch.rand(n, generator=g, dtype=torch.float64) * 2 - 1).to(dtype)


def rhs_normal(n: int, seed: int, dtype=torch.float64):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(n, generator=g, dtype=torch.float64).to(dtype)


def rhs_uniform01(n: int, seed: int, dtype=torch.float64):
    g = torch.Generator().manual_seed(seed)
    return torch.rand(n, generator=g, dtype=torch.float64).to(dtype)


def convdiff_3d_upwind(m: int, velocity=(10.0, 5.0, 2.5), diffusion: float = 1.0,
                       dtype=torch.float64, device="cpu"):
    """Non-symmetric 7-point upwind convection-diffusion on m^3, h = 1/(m+1):
    diagonal 6D/h^2 + sum_a v_a/h, off-diagonals -D/h^2 to the six
    neighbours plus -v_a/h toward the i-1 neighbour of each axis (kept as
    separate entries, summed on coalesce)."""
    h = 1.0 / (m + 1)
    inv = diffusion / (h * h)
    edges = axis_edges(3, -inv) + [(a, -1, -velocity[a] / h) for a in range(3)]
    v, r, c = grid_coo((m, m, m), 6.0 * inv + sum(velocity) / h, edges, dtype, device)
    n = m ** 3
    return v, r, c, (n, n)


def diffusion_2d_batched(batch: int, m: int, seed: int = 2, dtype=torch.float64, device="cpu"):
    """Batch of 5-point variable-coefficient diffusion matrices sharing one
    pattern. Cell conductivity k = exp(N(0,1)) (CPU generator `seed`), face
    value 2 k_i k_j / (k_i + k_j), boundary faces k_i, off-diagonal -face,
    diagonal sum(faces) + 1e-3. b ~ N(0,1) from the same generator after k.
    Returns (val_batch [B, nnz], row, col, shape, b_batch [B, n])."""
    g = torch.Generator().manual_seed(seed)
    k = torch.exp(torch.randn(batch, m, m, generator=g, dtype=torch.float64))
    b = torch.randn(batch, m * m, generator=g, dtype=torch.float64)
    n = m * m
    kf = k.reshape(batch, n)
    p = torch.arange(n)
    iy, ix = p // m, p % m
    diag = torch.full((batch, n), 1e-3, dtype=torch.float64)
    rows, cols, vals = [p], [p], []
    offs = []
    for axis, step in ((0, 1), (0, -1), (1, 1), (1, -1)):
        coord = iy if axis == 0 else ix
        nb = coord + step
        inside = (nb >= 0) & (nb < m)
        q = p + step * (m if axis == 0 else 1)
        kj = kf[:, q.clamp(0, n - 1)]
        face = torch.where(inside, 2 * kf * kj / (kf + kj), kf)
        diag = diag + face
        src = p[inside]
        rows.append(src)
        cols.append(q[inside])
        offs.append(-face[:, inside])
    vals = torch.cat([diag] + offs, dim=1)
    row = torch.cat(rows)
    col = torch.cat(cols)
    return (vals.to(dtype=dtype, device=device), row.to(device), col.to(device), (n, n),
            b.to(dtype=dtype, device=device))


def poisson_3d_7pt_rows(dims, z0: int, nz_local: int, dtype=torch.float64, device="cpu"):
    """Rows [z0, z0 + nz_local) of poisson_3d_7pt on dims = (nz, ny, nx)."""
    return grid_coo_rows(dims, z0, nz_local, 6.0, axis_edges(3, -1.0), dtype, device)


def convdiff_3d_upwind_rows(m: int, z0: int, nz_local: int, velocity=(10.0, 5.0, 2.5),
                            diffusion: float = 1.0, dtype=torch.float64, device="cpu", nz=None):
    """Rows [z0, z0 + nz_local) of the upwind convection-diffusion operator on
    a (nz or m) x m x m grid with h = 1/(m+1) (convdiff_3d_upwind's stencil)."""
    h = 1.0 / (m + 1)
    inv = diffusion / (h * h)
    edges = axis_edges(3, -inv) + [(a, -1, -velocity[a] / h) for a in range(3)]
    return grid_coo_rows((nz or m, m, m), z0, nz_local, 6.0 * inv + sum(velocity) / h, edges,
                         dtype, device)


# --------------------------------------------------------------- 27-point
_OFFS13 = [(dz, dy, dx) for dz in (-1, 0, 1) for dy in (-1, 0, 1) for dx in (-1, 0, 1)
           if (dz, dy, dx) > (0, 0, 0)]
_M32 = 0xFFFFFFFF


def _mix32(x: torch.Tensor) -> torch.Tensor:
    # 32-bit avalanche in int64 arithmetic; every product stays below 2^63
    x = x & _M32
    x = x ^ (x >> 16)
    x = (x * 0x7FEB352D) & _M32
    x = x ^ (x >> 15)
    x = (x * 0x5BD1E995) & _M32
    x = x ^ (x >> 16)
    return x


def edge_uniform(edge_id: torch.Tensor, seed: int) -> torch.Tensor:
    """Deterministic U[0,1) per (seed, edge id): identical on CPU and GPU."""
    lo = edge_id & _M32
    hi = edge_id >> 32
    h = _mix32(lo ^ _mix32(torch.full_like(lo, seed * 0x9E37 + 1)))
    h = _mix32(h ^ _mix32(hi + 0x632B))
    return h.to(torch.float64) / 4294967296.0


def stencil27_rows(dims, z0: int, nz_local: int, seed: int = 4, dtype=torch.float64,
                   device="cpu"):
    """Rows of the global 27-point matrix on grid dims = (nz, ny, nx) whose z
    lies in [z0, z0 + nz_local). Off-diagonal (u, v) = -(0.5 + U) with U drawn
    once per undirected edge from edge_uniform(min(u,v)*13 + direction),
    diagonal = sum |off| + 0.01. Returns (val, row, col) with GLOBAL indices,
    diagonal entries first then the 26 neighbour blocks."""
    nz, ny, nx = dims
    sz, sy = ny * nx, nx
    base = z0 * sz
    p = torch.arange(nz_local * sz, device=device, dtype=torch.int64) + base
    z, y, x = p // sz, (p // sy) % ny, p % nx
    rows, cols, vals = [], [], []
    diag = torch.full((p.numel(),), 0.01, dtype=torch.float64, device=device)
    for dz in (-1, 0, 1):
        for dy in (-1, 0, 1):
            for dx in (-1, 0, 1):
                if (dz, dy, dx) == (0, 0, 0):
                    continue
                zz, yy, xx = z + dz, y + dy, x + dx
                keep = (zz >= 0) & (zz < nz) & (yy >= 0) & (yy < ny) & (xx >= 0) & (xx < nx)
                src = p[keep]
                dst = src + dz * sz + dy * sy + dx
                if (dz, dy, dx) > (0, 0, 0):
                    low, d = src, _OFFS13.index((dz, dy, dx))
                else:
                    low, d = dst, _OFFS13.index((-dz, -dy, -dx))
                w = 0.5 + edge_uniform(low * 13 + d, seed)
                diag.index_add_(0, src - base, w)
                rows.append(src)
                cols.append(dst)
                vals.append(-w)
    row = torch.cat([p] + rows)
    col = torch.cat([p] + cols)
    val = torch.cat([diag] + vals).to(dtype)
    return val, row, col


# ------------------------------------------------------------ irregular rows
def powerlaw_coo(n: int, avg: float = 16.0, shape_a: float = 1.5, seed: int = 5,
                 band: int = 1024, spd: bool = False, dtype=torch.float64, device="cpu"):
    """Sparse n x n matrix with power-law (Pareto, shape `shape_a`) row
    lengths of mean about `avg`, capped at min(n, 64 avg): the skewed row
    lengths of FEM meshes with refined regions or of graph matrices. Half of
    a row's columns lie within +-`band` of the diagonal, half anywhere;
    off-diagonal values are -U(0.1, 1). Every row also holds a diagonal
    entry equal to the sum of its off-diagonal magnitudes plus 1. With
    spd=True the off-diagonal part is symmetrised first (B + B^T), making
    the matrix symmetric positive definite. Duplicate (row, col) pairs are
    left in the COO (summed when it is converted). Seeded CPU generator:
    identical on every device. Returns (val, row, col, shape)."""
    g = torch.Generator().manual_seed(seed)
    cap = int(min(n, 64 * avg))
    xm = avg * (shape_a - 1.0) / shape_a
    u = torch.rand(n, generator=g, dtype=torch.float64).clamp_min(1e-12)
    lens = (xm * u.pow(-1.0 / shape_a)).floor().clamp(1, cap).to(torch.int64)
    rows = torch.repeat_interleave(torch.arange(n), lens)
    m = rows.numel()
    near = torch.rand(m, generator=g) < 0.5
    off = torch.randint(-band, band + 1, (m,), generator=g)
    far = torch.randint(0, n, (m,), generator=g)
    cols = torch.where(near, (rows + off).clamp(0, n - 1), far)
    keep = cols != rows
    rows, cols = rows[keep], cols[keep]
    vals = -(0.1 + 0.9 * torch.rand(rows.numel(), generator=g, dtype=torch.float64))
    if spd:
        rows, cols = torch.cat([rows, cols]), torch.cat([cols, rows])
        vals = torch.cat([vals, vals])
    diag = torch.ones(n, dtype=torch.float64)
    diag.index_add_(0, rows, vals.abs())
    idx = torch.arange(n)
    val = torch.cat([diag, vals]).to(dtype)
    row = torch.cat([idx, rows])
    col = torch.cat([idx, cols])
    return val.to(device), row.to(device), col.to(device), (n, n)
