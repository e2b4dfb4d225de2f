#!/usr/bin/env python
"""Benchmark: fp64 Jacobi-PCG iterations/s on the 3-D 7-point Poisson system,
256^3 unknowns per GPU (weak scaling across GPUs, z-slab row partition).

One step = one full solve to rtol 1e-8 from x0 = 0 (b ~ N(0,1), seed 1).
value = CG iterations/s summed over GPUs (each GPU advances its 256^3 slab
by one iteration per global iteration), with matrix and b resident in HBM;
e2e = the same metric through the public call pytorch_solve() with the COO
matrix and b in pinned host memory, copies included.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

M = 256          # grid edge per GPU
RTOL = 1e-8
SEED = 1
METRIC = "fp64 Jacobi-PCG iterations/s (3-D 7-point Poisson, 256^3 unknowns per GPU)"


def peaks():
    try:
        with open(os.path.join(HERE, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class Clocks:
    """nvidia-smi sampler running during the timed region."""

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.rows = []
        self.proc = None

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([s.strip() for s in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
                for k, nm in enumerate(names):
                    if r[5 + k].lower().startswith("active"):
                        reasons.add(nm)
            except Exception:
                continue
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(sm)}


def matrix_bytes(nnz: int, n: int, V: int = 8) -> int:
    return nnz * (V + 4) + 4 * (n + 1)


def e2e_run(args, v, r, c, b_host, sh, dev):
    """pytorch_solve() with the COO matrix and b in pinned host memory; the
    timed region holds the H2D copies, the CSR build, the solve and the D2H
    copy of x."""
    import torch_sla_b200 as T
    from torch_sla_b200.backends import pytorch_backend as PB
    vh, rh, ch = v.cpu().pin_memory(), r.cpu().pin_memory(), c.cpu().pin_memory()
    bh = b_host.pin_memory()
    h2d = vh.numel() * 8 + rh.numel() * 8 + ch.numel() * 8 + bh.numel() * 8
    e_iters = 0
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e_steps = max(1, min(args.steps, 3))
    e0.record()
    for _ in range(e_steps):
        vd, rd, cd, bd = (t.to(dev, non_blocking=True) for t in (vh, rh, ch, bh))
        x = T.pytorch_solve(vd, rd, cd, sh, bd, method="cg", atol=0.0, rtol=RTOL,
                            preconditioner="jacobi")
        x.cpu()
        e_iters += PB.last_solve_info()["iterations"]
    e1.record()
    torch.cuda.synchronize()
    return e_iters, e0.elapsed_time(e1), e_steps, h2d


def run_b200(args):
    import torch.distributed as dist

    import torch_sla_b200 as T
    from torch_sla_b200 import _lib as L
    from torch_sla_b200 import problems as P
    from torch_sla_b200.backends import pytorch_backend as PB

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        return run_b200_sharded(args, world, rank, local)

    m = args.grid
    n = m ** 3
    v, r, c, sh = P.poisson_3d_7pt(m, device=dev)
    b_host = P.rhs_normal(n, SEED)
    b = b_host.to(dev)
    A = PB.CachedSparseMatrix(v, r, c, sh)
    Mj = PB.get_preconditioner(A, "jacobi")
    nnz = A.csr.nnz

    def solve_once():
        x, info = PB._pcg_core(A, b, None, Mj.dinv, 0.0, RTOL, 10000)
        return info

    for _ in range(args.warmup):
        solve_once()
    torch.cuda.synchronize()
    L.profile_enable(True, 8)
    launches0 = L.launch_count()
    iters = 0
    with Clocks(local) as clk:
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        t0.record()
        for _ in range(args.steps):
            info = solve_once()
            iters += int(info.iterations)
        t1.record()
        torch.cuda.synchronize()
    ms = t0.elapsed_time(t1)
    launches = L.launch_count() - launches0
    ka_ms, ka_n = L.profile_read(0)
    kb_ms, kb_n = L.profile_read(1)
    L.profile_enable(False)
    value = iters / (ms / 1e3)

    # roofline of the dominant kernel (SpMV with the fused p update)
    ka_bytes = matrix_bytes(nnz, n) + 5 * 8 * n
    ka_avg = ka_ms / max(ka_n, 1)
    peak, peak_kind = peaks()
    achieved = ka_bytes / (ka_avg / 1e3) / 1e9 if ka_n else None
    iter_bytes = matrix_bytes(nnz, n) + 13 * 8 * n
    traffic = read_traffic("cg_spmv_kernel")

    # end to end through pytorch_solve with pinned host COO + b
    e_iters, e_ms, e_steps, h2d = 0, float("nan"), 0, 0
    if not args.no_e2e:
        e_iters, e_ms, e_steps, h2d = e2e_run(args, v, r, c, b_host, sh, dev)

    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "iterations/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic",
        "config": {"workload": "jacobi_pcg_poisson3d_7pt", "grid": [m, m, m], "n": n, "nnz": nnz,
                   "rtol": RTOL, "b": "N(0,1) seed 1", "iterations_per_solve": iters // args.steps,
                   "format": "SELL-32 int32 (sigma=1)", "l2": "inputs larger than L2 (1.4 GB matrix)",
                   "parallelism": "single GPU"},
        "iteration_roofline": {"bytes_per_iter": iter_bytes,
                               "achieved_gbs": round(iter_bytes * value / 1e9, 1),
                               "frac": round(iter_bytes * value / 1e9 / peak, 4),
                               "peak_kind": peak_kind},
        "roofline": {"kernel": "cg_spmv_kernel", "bound": "hbm",
                     "achieved": None if achieved is None else round(achieved, 1),
                     "peak": peak, "unit": "GB/s",
                     "frac": None if achieved is None else round(achieved / peak, 4),
                     "traffic": traffic, "algorithmic_bytes": ka_bytes,
                     "avg_launch_ms": round(ka_avg, 5), "sampled_launches": ka_n,
                     "update_kernel_avg_ms": round(kb_ms / max(kb_n, 1), 5),
                     "peak_kind": peak_kind},
        "e2e": {"value": round(e_iters / (e_ms / 1e3), 2) if e_steps else None,
                "unit": "iterations/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": n * 8,
                "ms_per_step": round(e_ms / e_steps, 3) if e_steps else None, "steps": e_steps},
        "gpu_launches": launches,
        "clocks": clk.summary(),
    }
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(A_gpu=A, b_host=b_host, budget_s=args.cpu_seconds)
    print(json.dumps(line), flush=True)


def read_traffic(kernel: str):
    """Per-launch DRAM bytes of `kernel` at the full workload, from the
    committed ncu summary (profiles/traffic.txt: '<kernel> <bytes>')."""
    path = os.path.join(HERE, "profiles", "traffic.txt")
    try:
        with open(path) as f:
            for line in f:
                parts = line.split()
                if len(parts) >= 2 and parts[0] == kernel:
                    return int(float(parts[1]))
    except OSError:
        pass
    return None


def cpu_csr_from_device(A):
    """torch CPU CSR (int64 indices, as torch-sla's to_sparse_csr builds)
    of the device CSR: skips the ~40 s CPU COO sort at 256^3."""
    csr = A.csr
    return torch.sparse_csr_tensor(csr.rowptr.cpu().long(), csr.colind.cpu().long(),
                                   csr.vals.cpu(), csr.shape)


def cpu_baseline(A_gpu=None, b_host=None, budget_s=15.0):
    """Reference CPU path (the oracle: torch-sla's own ATen ops) on the host
    cores, on a bounded number of PCG iterations of the same system."""
    from oracle import krylov as K
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    Acpu = cpu_csr_from_device(A_gpu)
    n = Acpu.shape[0]
    dinv = K.jacobi_inverse(K.csr_diagonal(Acpu), "eps")
    t0 = time.perf_counter()
    it = K.pcg_iterations(Acpu, b_host, dinv, budget_s=budget_s)
    dt = time.perf_counter() - t0
    return {"value": round(it / dt, 3), "unit": "iterations/s", "cores": cores, "kind": "port",
            "sample": f"{it} Jacobi-PCG iterations of the same 7-point system (n={n}) with "
                      "torch CPU CSR mv/vdot/addcmul, as torch-sla's pytorch backend runs them"}


def run_reference(args):
    """--impl reference: torch-sla's CPU pytorch-backend arithmetic (the
    oracle port) on the host cores, same metric, bounded sample per step."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import krylov as K
    from torch_sla_b200 import problems as P
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    n = M ** 3
    v, r, c, sh = P.poisson_3d_7pt(M)
    # the reference sorts its COO on every solve (~40 s here); that setup is
    # excluded, only iterations are timed
    Acpu = K.csr(v, r, c, sh)
    del v, r, c
    b = P.rhs_normal(n, SEED)
    dinv = K.jacobi_inverse(K.csr_diagonal(Acpu), "eps")
    per_step = 3
    for _ in range(args.warmup):
        K.pcg_iterations(Acpu, b, dinv, iterations=1)
    t0 = time.perf_counter()
    its = 0
    for _ in range(args.steps):
        its += K.pcg_iterations(Acpu, b, dinv, iterations=per_step)
    dt = time.perf_counter() - t0
    value = its / dt
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 3),
            "unit": "iterations/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(dt / args.steps * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": {"workload": "jacobi_pcg_poisson3d_7pt", "grid": [M, M, M], "n": n,
                       "rtol": RTOL, "parallelism": "host CPU"},
            "cpu_baseline": {"value": round(value, 3), "unit": "iterations/s", "cores": cores,
                             "kind": "port",
                             "sample": f"{per_step} PCG iterations per step on the 256^3 system"},
            "e2e": {"value": round(value, 3), "unit": "iterations/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_b200_sharded(args, world, rank, local):
    """N GPUs: global grid (256 N) x 256 x 256, rank k owns z-slab k (the
    'simple' row partition), built from its own rows only."""
    import datetime

    import torch.distributed as dist

    from torch_sla_b200 import _lib as L
    from torch_sla_b200 import problems as P
    from torch_sla_b200.distributed import DSparseTensor, destroy_all

    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                            device_id=dev)
    m = args.grid
    dims = (m * world, m, m)
    n_glob = dims[0] * dims[1] * dims[2]
    n_loc = m ** 3
    v, r, c = P.poisson_3d_7pt_rows(dims, rank * m, m, device=dev)
    D = DSparseTensor.from_owned_rows(v, r, c, (n_glob, n_glob), rank=rank, world=world)
    del v, r, c
    b_full = P.rhs_normal(n_glob, SEED)
    b_host = b_full[rank * n_loc:(rank + 1) * n_loc].clone().pin_memory()
    del b_full
    b = b_host.to(dev)
    plan = D._shard_plan()
    nnz = plan.csr.nnz

    def solve_once(bb):
        x = D.solve_distributed_shard(bb, method="cg", preconditioner="jacobi", atol=0.0,
                                      rtol=RTOL, maxiter=100000)
        return x, D._last_info["iterations"]

    for _ in range(args.warmup):
        solve_once(b)
    torch.cuda.synchronize()
    dist.barrier()
    L.profile_enable(True, 8)
    launches0 = L.launch_count()
    iters = 0
    with Clocks(local) as clk:
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        dist.barrier()
        t0.record()
        for _ in range(args.steps):
            _, it = solve_once(b)
            iters += it
        t1.record()
        torch.cuda.synchronize()
        dist.barrier()
    ms_local = t0.elapsed_time(t1)
    launches = L.launch_count() - launches0
    ka_ms, ka_n = L.profile_read(0)
    kb_ms, kb_n = L.profile_read(1)
    L.profile_enable(False)
    t = torch.tensor([ms_local], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    value = iters * world / (ms / 1e3)

    # end to end through D.solve with b in pinned host memory, x read back
    e_steps = max(1, min(args.steps, 3))
    dist.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    e_iters = 0
    for _ in range(e_steps):
        x, it = solve_once(b_host.to(dev, non_blocking=True))
        x.cpu()
        e_iters += it
    e1.record()
    torch.cuda.synchronize()
    te = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
    dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e_ms = float(te.item())

    ka_interior = plan.sell_int.n_slots
    ka_bytes = matrix_bytes(nnz, n_loc) + 5 * 8 * n_loc
    ka_bytes_int = int(ka_bytes * ka_interior / max(n_loc, 1))
    ka_avg = ka_ms / max(ka_n, 1)
    peak, peak_kind = peaks()
    achieved = ka_bytes_int / (ka_avg / 1e3) / 1e9 if ka_n else None
    iter_bytes = matrix_bytes(nnz, n_loc) + 13 * 8 * n_loc
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "iterations/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic",
            "config": {"workload": "jacobi_pcg_poisson3d_7pt", "grid": list(dims), "n": n_glob,
                       "n_per_gpu": n_loc, "nnz_per_gpu": nnz, "rtol": RTOL,
                       "b": "N(0,1) seed 1 (global vector)",
                       "iterations_per_solve": iters // args.steps,
                       "partition": "z-slabs (partition_simple), halo one z-layer per neighbour",
                       "halo_bytes_per_neighbour": m * m * 8, "check_every": 10,
                       "format": "SELL-32 int32 (sigma=1)", "l2": "inputs larger than L2",
                       "parallelism": f"row-sharded x{world} (NCCL)"},
            "iteration_roofline": {"bytes_per_iter_per_gpu": iter_bytes,
                                   "achieved_gbs_per_gpu": round(iter_bytes * value / world / 1e9, 1),
                                   "frac": round(iter_bytes * value / world / 1e9 / peak, 4),
                                   "peak_kind": peak_kind},
            "roofline": {"kernel": "shard_cg_spmv (interior rows)", "bound": "hbm",
                         "achieved": None if achieved is None else round(achieved, 1),
                         "peak": peak, "unit": "GB/s",
                         "frac": None if achieved is None else round(achieved / peak, 4),
                         "traffic": read_traffic("shard_cg_spmv"),
                         "algorithmic_bytes": ka_bytes_int, "avg_launch_ms": round(ka_avg, 5),
                         "sampled_launches": ka_n, "peak_kind": peak_kind},
            "e2e": {"value": round(e_iters * world / (e_ms / 1e3), 2), "unit": "iterations/s",
                    "h2d_bytes_per_step": n_loc * 8 * world, "d2h_bytes_per_step": n_loc * 8 * world,
                    "ms_per_step": round(e_ms / e_steps, 3), "steps": e_steps,
                    "note": "matrix setup (partition maps, CSR) done once before timing"},
            "gpu_launches": launches,
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    del D, plan
    destroy_all()
    dist.barrier()
    dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--grid", type=int, default=M, help="grid edge per GPU (default 256)")
    ap.add_argument("--no-e2e", action="store_true")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
