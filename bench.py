#!/usr/bin/env python
"""Benchmark of the torch-sla iterative-solve hot path on B200.

Default workload (the one the headline metric is quoted on): fp64 Jacobi
PCG on the 3-D 7-point Poisson system with 256^3 unknowns per GPU, b ~ N(0,1)
seed 1, rtol 1e-8. One step = one full solve. At N GPUs the global grid is
(256 N) x 256 x 256, row-partitioned into z-slabs (weak scaling); value =
CG iterations/s x N (each GPU advances its 256^3 slab once per iteration),
with the matrix and b resident in HBM; e2e = the same metric through the
public API with host buffers and the copies inside the timed region.

Other workloads (--workload): cg2d (2-D 256^2 plain CG, rtol 1e-10,
persistent kernel), spmv (256^3 SpMV fp64 and fp32), batched (64 x 512^2
same-pattern CG, rtol 1e-8, with backward), bicgstab (192^3 convection-
diffusion, Jacobi BiCGStab), pcg27 (27-point variable-coefficient 256^3 per
GPU), mrhs (128^3 7-point with 16 right-hand sides, multi-RHS CG), mixed
(256^3 7-point mixed-precision PCG: float32 matrix, float64 vectors).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                  [--workload pcg7|cg2d|spmv|batched|bicgstab|pcg27|mrhs|mixed] [--grid M]
                  [--layout auto|explicit]
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import socket
import statistics
import subprocess
import sys
import threading
import time

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

M = 256
RTOL = 1e-8
SEED = 1
METRIC = "fp64 Jacobi-PCG iterations/s (3-D 7-point Poisson, 256^3 unknowns per GPU)"


# ------------------------------------------------------------------ helpers
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
    """Algorithmic matrix bytes on int32 CSR."""
    return nnz * (V + 4) + 4 * (n + 1)


def read_traffic(key: str):
    """Per-launch DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum)
    of a kernel on one workload, from the ncu summary profiles/traffic.txt
    ('<kernel>@<workload>:<size> <bytes>' lines); None when not captured."""
    try:
        with open(os.path.join(HERE, "profiles", "traffic.txt")) as f:
            for line in f:
                parts = line.split()
                if len(parts) >= 2 and parts[0] == key:
                    return int(float(parts[1]))
    except OSError:
        pass
    return None


def timed(fn, steps, dev, clocks_gpu):
    """Run fn() `steps` times between synchronisations, CUDA events on the
    current stream; returns (ms, results, clocks summary)."""
    out = []
    with Clocks(clocks_gpu) as clk:
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(dev)
        t0.record()
        for _ in range(steps):
            out.append(fn())
        t1.record()
        torch.cuda.synchronize(dev)
    return t0.elapsed_time(t1), out, clk.summary()


def base_line(args, metric, value, unit, ms, n_gpus, dtype="f64", hib=True):
    return {"metric": metric, "value": round(value, 3), "unit": unit, "n_gpus": n_gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3),
            "higher_is_better": hib, "scaling": "weak", "vs_baseline": None, "dtype": dtype,
            "data": "synthetic"}


def sell_format(sell, V=8):
    """Layout of a SELL view and the matrix bytes that layout itself moves
    per sweep (padding included): a diagonal-offset view reads values only,
    the explicit layout values and int32 columns."""
    if sell.diagonal_offsets:
        return {"format": f"SELL-32 diagonal-offset ({sell.uniform_width} diagonals, "
                          "no column array)", "matrix_bytes": sell.padded_nnz * V}
    rows = 4 * sell.n_slots if sell.row_ids is not None else 0  # row ids of a sorted view
    return {"format": f"SELL-32 int32 (sigma={getattr(sell, 'sigma', 1)})",
            "matrix_bytes": sell.padded_nnz * (V + 4) + rows}


def roofline(kernel, alg_bytes, ms_total, launches, traffic_key, format_bytes=None):
    """Roofline of one kernel from its in-situ CUDA-event mean launch time.

    achieved / frac: the bytes this kernel must move per launch in the
    layout it runs on (the matrix as stored, padding included, plus its
    vectors) over the mean launch time -- for the diagonal-offset view these
    are values only, no column array, and they match the ncu-measured DRAM
    traffic within a few per cent. alg_achieved / alg_frac: the same time
    against the int32-CSR algorithmic bytes (nnz (V+4) + 4 (N+1) + vectors),
    which read above 1 where the layout stores less than int32 CSR does.
    traffic_frac: the ncu DRAM bytes of one launch (profiles/traffic.txt)
    over the same time."""
    peak, kind = peaks()
    avg = ms_total / max(launches, 1)
    sec = avg / 1e3
    basis = format_bytes if format_bytes is not None else alg_bytes
    traffic = read_traffic(traffic_key)

    def gbs(nbytes):
        return nbytes / sec / 1e9 if launches and nbytes is not None else None

    def rnd(v, d):
        return None if v is None else round(v, d)

    ach, alg, tr = gbs(basis), gbs(alg_bytes), gbs(traffic)
    return {"kernel": kernel, "bound": "hbm", "achieved": rnd(ach, 1), "peak": peak,
            "unit": "GB/s", "frac": rnd(ach / peak if ach else None, 4),
            "traffic": traffic, "traffic_key": traffic_key,
            "traffic_frac": rnd(tr / peak if tr else None, 4),
            "bytes": int(basis),
            "bytes_basis": ("layout (matrix as stored + vectors)" if format_bytes is not None
                            else "int32 CSR (nnz (V+4) + 4 (N+1) + vectors)"),
            "alg_bytes": int(alg_bytes), "alg_achieved": rnd(alg, 1),
            "alg_frac": rnd(alg / peak if alg else None, 4),
            "avg_launch_ms": round(avg, 5), "sampled_launches": launches,
            "peak_kind": ("measured (MEASURED_PEAKS.json hbm_gbs)" if kind == "measured"
                          else kind)}


# ----------------------------------------------------- single-GPU workloads
def wl_pcg7(args, dev, local):
    """3-D 7-point Poisson 256^3, fp64 Jacobi PCG, rtol 1e-8 (the headline workload)."""
    from torch_sla_b200 import _lib as L
    from torch_sla_b200 import problems as P
    from torch_sla_b200.backends import pytorch_backend as PB
    m = args.grid
    n = m ** 3
    v, r, c, sh = P.poisson_3d_7pt(m, device=dev)
    b_host = P.rhs_normal(n, SEED)
    b = b_host.to(dev)
    A = PB.CachedSparseMatrix(v, r, c, sh)
    Mj = PB.get_preconditioner(A, "jacobi")
    nnz = A.csr.nnz
    # --layout explicit: the whole solve on the int32-column view
    view = A.csr.sell(diagonal=False) if args.layout == "explicit" else A.sell()

    def solve_once():
        return PB._pcg_core(A, b, None, Mj.dinv, 0.0, RTOL, 10000, sell=view)[1].iterations

    for _ in range(args.warmup):
        solve_once()
    L.profile_enable(True, 7)
    l0 = L.launch_count()
    ms, its, clk = timed(solve_once, args.steps, dev, local)
    launches = L.launch_count() - l0
    ka_ms, ka_n = L.profile_read(0)
    kb_ms, kb_n = L.profile_read(1)
    kp_ms, kp_n = L.profile_read(2)
    L.profile_enable(False)
    iters = sum(its)
    value = iters / (ms / 1e3)
    peak, kind = peaks()
    iter_bytes = matrix_bytes(nnz, n) + 13 * 8 * n
    fm = sell_format(view)
    line = base_line(args, METRIC, value, "iterations/s", ms, 1)
    line["config"] = {"workload": "jacobi_pcg_poisson3d_7pt", "grid": [m, m, m], "n": n,
                      "nnz": nnz, "rtol": RTOL, "b": "N(0,1) seed 1",
                      "iterations_per_solve": iters // args.steps,
                      "format": fm["format"],
                      "l2": "inputs larger than L2 (0.9-1.4 GB matrix); no flush",
                      "parallelism": "single GPU"}
    # K_A: the SpMV over the search direction p (formed by cg_pform_kernel):
    # matrix + p read once + Ap written
    tkey = "pcg7-explicit" if args.layout == "explicit" else "pcg7"
    line["roofline"] = roofline("cg_spmv_split_kernel", matrix_bytes(nnz, n) + 2 * 8 * n, ka_ms,
                                ka_n, f"cg_spmv_split_kernel@{tkey}:{m}",
                                fm["matrix_bytes"] + 2 * 8 * n)
    line["roofline"]["update_kernel"] = {
        "kernel": "cg_update_kernel", "avg_launch_ms": round(kb_ms / max(kb_n, 1), 5),
        # 4 vector passes at even, 8 at odd iterations (x updated two steps at a time)
        "achieved": round(6 * 8 * n / (kb_ms / max(kb_n, 1) / 1e3) / 1e9, 1) if kb_n else None}
    line["roofline"]["pform_kernel"] = {
        "kernel": "cg_pform_kernel", "avg_launch_ms": round(kp_ms / max(kp_n, 1), 5),
        # r, dinv, p_old read, p written
        "achieved": round(4 * 8 * n / (kp_ms / max(kp_n, 1) / 1e3) / 1e9, 1) if kp_n else None}
    line["iteration_roofline"] = {"bytes_per_iter": iter_bytes,
                                  "achieved_gbs": round(iter_bytes * value / 1e9, 1),
                                  "alg_frac": round(iter_bytes * value / 1e9 / peak, 4),
                                  "alg_frac_of_8tbs": round(iter_bytes * value / 8e12, 4),
                                  "bytes_formula": "12 nnz + 4 (N+1) + 13 * 8 N",
                                  "layout_bytes_per_iter": fm["matrix_bytes"] + 12 * 8 * n,
                                  "frac": round((fm["matrix_bytes"] + 12 * 8 * n) * value
                                                / 1e9 / peak, 4)}
    if args.layout != "explicit":
        line["roofline"]["explicit"] = explicit_pcg7(A, b, Mj, n, nnz, m)
        line["float32"] = float32_pcg7(v, r, c, sh, b_host, dev, m, local)
    if not args.no_e2e:
        line["e2e"] = e2e_pcg7(args, v, r, c, b_host, sh, dev)
    line["gpu_launches"] = launches
    line["clocks"] = clk
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_pcg(A, b_host, args.cpu_seconds)
    return line


def explicit_pcg7(A, b, Mj, n, nnz, m):
    """The same solve on the explicit int32-column SELL view, the layout
    every non-stencil matrix takes: its SpMV K_A timed in situ (CUDA events
    on the launching stream) over two solves. Its bytes are the int32-CSR
    algorithmic bytes up to the slice padding."""
    from torch_sla_b200 import _lib as L
    from torch_sla_b200.backends import pytorch_backend as PB
    sell = A.csr.sell(diagonal=False)
    fm = sell_format(sell)
    PB._pcg_core(A, b, None, Mj.dinv, 0.0, RTOL, 10000, sell=sell)
    L.profile_enable(True, 7)
    its = [PB._pcg_core(A, b, None, Mj.dinv, 0.0, RTOL, 10000, sell=sell)[1].iterations
           for _ in range(2)]
    ka_ms, ka_n = L.profile_read(0)
    L.profile_enable(False)
    out = roofline("cg_spmv_split_kernel (explicit int32-column SELL)",
                   matrix_bytes(nnz, n) + 2 * 8 * n, ka_ms, ka_n,
                   f"cg_spmv_split_kernel@pcg7-explicit:{m}", fm["matrix_bytes"] + 2 * 8 * n)
    out.update(format=fm["format"], padded_nnz=sell.padded_nnz, iterations_per_solve=its[0])
    del sell
    return out


def float32_pcg7(v, r, c, sh, b_host, dev, m, local):
    """The same system in float32 (torch-sla's float32 PCG; this solver
    accumulates its dots in float64): iterations/s over two solves timed with
    CUDA events, and its SpMV K_A in situ. K_A bytes: float32 values + p
    read + Ap written (4-byte words)."""
    from torch_sla_b200 import _lib as L
    from torch_sla_b200.backends import pytorch_backend as PB
    n = sh[0]
    A = PB.CachedSparseMatrix(v.float(), r, c, sh)
    b = b_host.float().to(dev)
    Mj = PB.get_preconditioner(A, "jacobi")
    sell = A.sell()
    fm = sell_format(sell, V=4)
    PB._pcg_core(A, b, None, Mj.dinv, 0.0, RTOL, 10000, sell=sell)
    L.profile_enable(True, 7)
    ms, its, _ = timed(lambda: PB._pcg_core(A, b, None, Mj.dinv, 0.0, RTOL, 10000,
                                            sell=sell)[1].iterations, 2, dev, local)
    ka_ms, ka_n = L.profile_read(0)
    kb_ms, kb_n = L.profile_read(1)
    kp_ms, kp_n = L.profile_read(2)
    L.profile_enable(False)
    out = {"iterations_per_solve": its[0], "iterations_per_s": round(sum(its) / (ms / 1e3), 1),
           "format": fm["format"],
           "update_kernel_ms": round(kb_ms / max(kb_n, 1), 5),
           "pform_kernel_ms": round(kp_ms / max(kp_n, 1), 5)}
    out["roofline"] = roofline("cg_spmv_split_kernel (float32)",
                               matrix_bytes(A.csr.nnz, n, V=4) + 2 * 4 * n, ka_ms, ka_n,
                               f"cg_spmv_split_kernel@pcg7-f32:{m}", fm["matrix_bytes"] + 2 * 4 * n)
    del A, b, Mj, sell
    return out


def e2e_pcg7(args, v, r, c, b_host, sh, dev):
    """pytorch_solve() with the COO matrix and b in pinned host memory; the
    timed region holds the H2D copies, the CSR build, the solve and the D2H
    copy of x."""
    import torch_sla_b200 as T
    from torch_sla_b200.backends import pytorch_backend as PB
    vh, rh, ch = v.cpu().pin_memory(), r.cpu().pin_memory(), c.cpu().pin_memory()
    bh = b_host.pin_memory()
    xh = torch.empty_like(bh).pin_memory()
    h2d = (vh.numel() + rh.numel() + ch.numel() + bh.numel()) * 8
    steps = max(1, min(args.steps, 3))

    def once():
        vd, rd, cd, bd = (t.to(dev, non_blocking=True) for t in (vh, rh, ch, bh))
        x = T.pytorch_solve(vd, rd, cd, sh, bd, method="cg", atol=0.0, rtol=RTOL,
                            preconditioner="jacobi")
        xh.copy_(x)  # device -> pinned host read of the solution
        return PB.last_solve_info()["iterations"]

    ms, its, _ = timed(once, steps, dev, dev.index)
    return {"value": round(sum(its) / (ms / 1e3), 3), "unit": "iterations/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": bh.numel() * 8,
            "ms_per_step": round(ms / steps, 3), "steps": steps,
            "api": "torch_sla_b200.pytorch_solve (COO from pinned host memory)"}


def cpu_csr_from_device(csr):
    """torch CPU CSR (int64 indices, as torch-sla builds it) of a device CSR:
    skips the ~40 s CPU COO sort of the 256^3 matrix."""
    return torch.sparse_csr_tensor(csr.rowptr.cpu().long(), csr.colind.cpu().long(),
                                   csr.vals.cpu(), csr.shape)


def cpu_baseline_pcg(A, b_host, budget_s):
    """The oracle (torch-sla's CPU ops) on the host cores, a bounded number of
    PCG iterations of the same system."""
    from oracle import krylov as K
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    Acpu = cpu_csr_from_device(A.csr)
    dinv = K.jacobi_inverse(K.csr_diagonal(Acpu), "eps")
    t0 = time.perf_counter()
    it = K.pcg_iterations(Acpu, b_host, dinv, budget_s=budget_s)
    dt = time.perf_counter() - t0
    return {"value": round(it / dt, 3), "unit": "iterations/s", "cores": cores, "kind": "port",
            "sample": f"{it} Jacobi-PCG iterations of the same system (n={Acpu.shape[0]}) with "
                      "torch CPU CSR mv / vdot / addcmul, torch-sla's pytorch-backend ops"}


def wl_cg2d(args, dev, local):
    """2-D 5-point 256^2, b ~ U(-1,1) seed 0, plain CG rtol 1e-10."""
    from oracle import krylov as K
    from torch_sla_b200 import _lib as L
    from torch_sla_b200 import problems as P
    from torch_sla_b200.backends import pytorch_backend as PB
    v, r, c, sh = P.poisson_2d_5pt(256, device=dev)
    b_host = P.rhs_uniform_pm1(sh[0], 0)
    b = b_host.to(dev)
    A = PB.CachedSparseMatrix(v, r, c, sh)

    def once():
        return PB._pcg_core(A, b, None, None, 0.0, 1e-10, 10000)[1].iterations

    for _ in range(args.warmup):
        once()
    l0 = L.launch_count()
    ms, its, clk = timed(once, args.steps, dev, local)
    line = base_line(args, "fp64 CG solve time (2-D 5-point Poisson 256^2, rtol 1e-10)",
                     ms / args.steps, "ms/solve", ms, 1, hib=False)
    line["config"] = {"workload": "cg_poisson2d_5pt_256", "n": sh[0], "nnz": A.csr.nnz,
                      "iterations_per_solve": its[0], "preconditioner": "none",
                      "kernel": "cg_cluster_kernel (one thread-block cluster per solve: "
                                "values, search direction and partial sums in distributed "
                                "shared memory, cluster barriers)",
                      "iterations_per_s": round(sum(its) / (ms / 1e3), 1)}
    line["gpu_launches"] = L.launch_count() - l0
    # unpreconditioned CG: matrix + 11 vector passes per iteration; the
    # 9.9 MB working set stays in L2, so this is reported against HBM only
    # for comparison (the kernel is bound by its two grid barriers per
    # iteration, not by bandwidth)
    per_iter = matrix_bytes(A.csr.nnz, sh[0]) + 11 * 8 * sh[0]
    line["roofline"] = roofline("cg_cluster_kernel", per_iter * its[0], ms, args.steps,
                                "cg_cluster_kernel@cg2d:256")
    line["roofline"]["note"] = ("one launch per solve; the matrix and search direction live in "
                                "shared memory, so HBM is not the bound: latency of the three "
                                "cluster barriers per iteration is")
    # the cooperative-grid kernel on the same solve, for comparison
    l1 = L.launch_count()
    ms_p, its_p, _ = timed(lambda: PB._pcg_core(A, b, None, None, 0.0, 1e-10, 10000,
                                                L.SLA_PCG_PERSISTENT)[1].iterations,
                           args.steps, dev, local)
    line["config"]["persistent_grid_kernel"] = {"ms_per_solve": round(ms_p / args.steps, 3),
                                                "iterations_per_solve": its_p[0]}
    line["clocks"] = clk
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    vc, rc_, cc, shc = P.poisson_2d_5pt(256)
    t0 = time.perf_counter()
    _, it, _, _ = K.pcg(vc, rc_, cc, shc, b_host, atol=0.0, rtol=1e-10, precond="none")
    dt = time.perf_counter() - t0
    line["cpu_baseline"] = {"value": round(dt * 1e3, 2), "unit": "ms/solve", "cores": cores,
                            "kind": "port", "sample": f"one full solve ({it} iterations)"}
    return line


def wl_spmv(args, dev, local):
    """SpMV sweep: y = A x on the 256^3 7-point matrix, fp64 and fp32, on the
    diagonal-offset view the solvers pick for this stencil and on the explicit
    int32-column view every other pattern takes."""
    from torch_sla_b200 import problems as P
    from torch_sla_b200._csr import DeviceCSR, spmv
    res = {}
    m = args.grid
    n = m ** 3
    peak, _ = peaks()
    for dt, V in ((torch.float64, 8), (torch.float32, 4)):
        v, r, c, sh = P.poisson_3d_7pt(m, dtype=dt, device=dev)
        csr = DeviceCSR(v, r, c, sh)
        del v, r, c
        x = P.rhs_normal(n, SEED, dt).to(dev)
        y = torch.empty_like(x)
        for diagonal in (True, False):
            sell = csr.sell(diagonal=diagonal)
            reps = 50
            for _ in range(5):
                spmv(sell, x, n, y)
            ms, _, clk = timed(lambda: spmv(sell, x, n, y), reps, dev, local)
            alg = matrix_bytes(csr.nnz, n, V) + 2 * V * n
            fm = sell_format(sell, V)
            fb = fm["matrix_bytes"] + 2 * V * n
            sec = ms / reps / 1e3
            key = ("f64" if V == 8 else "f32") + ("" if diagonal else "_explicit")
            res[key] = {"us_per_spmv": round(sec * 1e6, 2),
                        "achieved_gbs": round(fb / sec / 1e9, 1),
                        "frac": round(fb / sec / 1e9 / peak, 4), "bytes": fb,
                        "format": fm["format"],
                        "alg_bytes": alg, "alg_achieved_gbs": round(alg / sec / 1e9, 1),
                        "alg_frac": round(alg / sec / 1e9 / peak, 4),
                        "alg_frac_of_8tbs": round(alg / sec / 8e12, 4),
                        "clocks": clk, "_ms": ms, "_reps": reps}
            del sell
        del csr, x, y
    res["irregular"] = spmv_irregular(dev, local, peak)
    f64 = res["f64"]
    line = base_line(args, "SpMV HBM GB/s (256^3 7-point, fp64)", f64["achieved_gbs"],
                     "GB/s", f64["us_per_spmv"] / 1e3 * args.steps, 1)
    line["roofline"] = roofline("spmv_kernel", f64["alg_bytes"], f64.pop("_ms"),
                                f64.pop("_reps"), f"spmv_kernel@spmv:{m}", f64["bytes"])
    for k, d in res.items():
        d.pop("_ms", None), d.pop("_reps", None)
    line["config"] = {"workload": "spmv_poisson3d_7pt", "grid": [m, m, m], "sweep": res,
                      "l2": "inputs larger than L2"}
    line["clocks"] = f64["clocks"]
    return line


def spmv_irregular(dev, local, peak, n=4_000_000, avg=16.0):
    """fp64 SpMV on a matrix with power-law row lengths (problems.powerlaw_coo:
    4M rows, about 16 entries per row, the longest 1025): the SELL-32 view in
    row order (sigma = 1) against the view sorted by length inside windows
    of sigma rows (SELL-32-sigma), with padding ratios and the bytes each
    layout moves."""
    from torch_sla_b200 import problems as P
    from torch_sla_b200._csr import DeviceCSR, spmv
    v, r, c, sh = P.powerlaw_coo(n, avg)
    csr = DeviceCSR(v.to(dev), r.to(dev), c.to(dev), sh)
    del v, r, c
    x = P.rhs_normal(n, SEED).to(dev)
    y = torch.empty_like(x)
    out = {"matrix": f"power-law row lengths, n={n}, nnz={csr.nnz}, "
                     f"longest row {int((csr.rowptr[1:] - csr.rowptr[:-1]).max())}"}
    for sigma in (1, 1024, 4096):
        sell = csr.sell(sigma=sigma)
        for _ in range(5):
            spmv(sell, x, n, y)
        ms, _, _ = timed(lambda: spmv(sell, x, n, y), 50, dev, local)
        sec = ms / 50 / 1e3
        fm = sell_format(sell)
        fb = fm["matrix_bytes"] + 2 * 8 * n
        alg = matrix_bytes(csr.nnz, n) + 2 * 8 * n
        out[f"sigma{sigma}"] = {"us_per_spmv": round(sec * 1e6, 2),
                                "padding": round(sell.padded_nnz / csr.nnz, 3),
                                "bytes": fb, "achieved_gbs": round(fb / sec / 1e9, 1),
                                "frac": round(fb / sec / 1e9 / peak, 4),
                                "alg_bytes": alg, "alg_frac": round(alg / sec / 1e9 / peak, 4)}
        del sell
    out["auto_sigma"] = csr.sell().sigma
    # the matvec view: long rows by the warp-per-row CSR pass, the rest sorted
    hv = csr.spmv_view()
    for _ in range(5):
        spmv(hv, x, n, y)
    ms, _, _ = timed(lambda: spmv(hv, x, n, y), 50, dev, local)
    sec = ms / 50 / 1e3
    n_long = int(hv.long_rows.numel()) if hv.long_rows is not None else 0
    long_nnz = (int((csr.rowptr[hv.long_rows.long() + 1] - csr.rowptr[hv.long_rows.long()]).sum())
                if n_long else 0)
    fb = sell_format(hv)["matrix_bytes"] + long_nnz * 12 + n_long * 12 + 2 * 8 * n
    out["hybrid"] = {"us_per_spmv": round(sec * 1e6, 2), "long_rows": n_long,
                     "long_row_entries": long_nnz,
                     "padding": round((hv.padded_nnz + long_nnz) / csr.nnz, 3), "bytes": fb,
                     "achieved_gbs": round(fb / sec / 1e9, 1),
                     "frac": round(fb / sec / 1e9 / peak, 4),
                     "alg_frac": round((matrix_bytes(csr.nnz, n) + 16 * n) / sec / 1e9 / peak, 4)}
    del csr, x, y, hv
    return out


def wl_batched(args, dev, local):
    """64 x 512^2 variable-coefficient diffusion, batched CG
    rtol 1e-8, forward + backward through spsolve_batch_same_layout."""
    import torch_sla_b200 as T
    from torch_sla_b200 import _lib as L
    from torch_sla_b200 import problems as P
    from torch_sla_b200.backends import pytorch_backend as PB
    B, m = 64, 512
    vb, r, c, sh, bb = P.diffusion_2d_batched(B, m, seed=2)
    vb, r, c, bb = vb.to(dev), r.to(dev), c.to(dev), bb.to(dev)

    def fwd():
        PB.batched_cg_same_pattern(vb, r, c, sh, bb, atol=0.0, rtol=RTOL)
        return PB.last_solve_info()["iterations"]

    def fwd_bwd():
        vg = vb.clone().requires_grad_(True)
        bg = bb.clone().requires_grad_(True)
        U = T.spsolve_batch_same_layout(vg, r, c, sh, bg, method="cg", atol=0.0, rtol=RTOL)
        (U * U).sum().backward()
        return 0

    for _ in range(args.warmup):
        fwd()
    L.profile_enable(True, 7)
    ms, its, clk = timed(fwd, args.steps, dev, local)
    ka_ms, ka_n = L.profile_read(0)
    L.profile_enable(False)
    ms_fb, _, _ = timed(fwd_bwd, max(1, args.steps // 2), dev, local)
    nnz = int(r.numel())
    n = sh[0]
    iters = sum(its)
    value = iters / (ms / 1e3)
    iter_bytes = B * nnz * 8 + 4 * nnz + 4 * (n + 1) + 13 * B * 8 * n
    peak, _ = peaks()
    line = base_line(args, "fp64 batched Jacobi-PCG iterations/s (64 x 512^2 diffusion)", value,
                     "iterations/s", ms, 1)
    line["config"] = {"workload": "batched_cg_diffusion2d", "batch": B, "grid": [m, m],
                      "iterations_per_solve": iters // args.steps, "rtol": RTOL,
                      "forward_backward_ms": round(ms_fb / max(1, args.steps // 2), 2),
                      "layout": "vectors [n][B]; values [entry][B] in the order of a "
                                "diagonal-offset view of the pattern (columns computed)"}
    line["iteration_roofline"] = {"bytes_per_iter": iter_bytes,
                                  "achieved_gbs": round(iter_bytes * value / 1e9, 1),
                                  "alg_frac": round(iter_bytes * value / 1e9 / peak, 4)}
    line["roofline"] = roofline("batch_spmv_kernel",
                                B * nnz * 8 + 4 * nnz + 4 * (n + 1) + 5 * B * 8 * n, ka_ms, ka_n,
                                f"batch_spmv_kernel@batched:{B}x{m}")
    line["clocks"] = clk
    return line


def wl_bicgstab(args, dev, local):
    """192^3 upwind convection-diffusion, Jacobi BiCGStab rtol 1e-8."""
    from torch_sla_b200 import _lib as L
    from torch_sla_b200 import problems as P
    from torch_sla_b200.backends import pytorch_backend as PB
    m = 192
    v, r, c, sh = P.convdiff_3d_upwind(m, device=dev)
    b = P.rhs_uniform01(sh[0], 3).to(dev)
    A = PB.CachedSparseMatrix(v, r, c, sh)
    Mj = PB.get_preconditioner(A, "jacobi")
    nnz, n = A.csr.nnz, sh[0]

    def once():
        return PB._bicgstab_core(A, b, None, Mj.dinv, 0.0, RTOL, 10000)[1].iterations

    for _ in range(args.warmup):
        once()
    L.profile_enable(True, 7)
    ms, its, clk = timed(once, args.steps, dev, local)
    k1_ms, k1_n = L.profile_read(0)
    L.profile_enable(False)
    iters = sum(its)
    value = iters / (ms / 1e3)
    iter_bytes = 2 * matrix_bytes(nnz, n) + 25 * 8 * n
    peak, _ = peaks()
    line = base_line(args, "fp64 Jacobi-BiCGStab iterations/s (192^3 convection-diffusion)",
                     value, "iterations/s", ms, 1)
    line["config"] = {"workload": "bicgstab_convdiff3d_192", "n": n, "nnz": nnz, "rtol": RTOL,
                      "iterations_per_solve": iters // args.steps}
    line["iteration_roofline"] = {"bytes_per_iter": iter_bytes,
                                  "achieved_gbs": round(iter_bytes * value / 1e9, 1),
                                  "alg_frac": round(iter_bytes * value / 1e9 / peak, 4),
                                  "bytes_formula": "2 (12 nnz + 4 (N+1)) + 25 * 8 N"}
    fm = sell_format(A.sell())
    line["config"]["format"] = fm["format"]
    line["roofline"] = roofline("bicg_k1", matrix_bytes(nnz, n) + 6 * 8 * n, k1_ms, k1_n,
                                f"bicg_k1@bicgstab:{m}", fm["matrix_bytes"] + 6 * 8 * n)
    line["clocks"] = clk
    return line


def wl_mrhs(args, dev, local):
    """Multi-RHS CG (pytorch_solve with a 2-D b, batched_pcg_solve): 3-D
    7-point 128^3 with 16 right-hand sides, Jacobi, rtol 1e-8."""
    from torch_sla_b200 import _lib as L
    from torch_sla_b200 import problems as P
    from torch_sla_b200.backends import pytorch_backend as PB
    m, K = 128, 16
    v, r, c, sh = P.poisson_3d_7pt(m, device=dev)
    n = sh[0]
    A = PB.CachedSparseMatrix(v, r, c, sh)
    M = PB.get_preconditioner(A, "jacobi")
    g = torch.Generator().manual_seed(5)
    B = torch.randn(n, K, generator=g, dtype=torch.float64).to(dev)
    nnz = A.csr.nnz

    def once():
        PB.batched_pcg_solve(A, B, atol=0.0, rtol=RTOL, maxiter=10000, preconditioner=M)
        return PB.last_solve_info()["iterations"]

    for _ in range(args.warmup):
        once()
    L.profile_enable(True, 7)
    ms, its, clk = timed(once, args.steps, dev, local)
    ka_ms, ka_n = L.profile_read(0)
    L.profile_enable(False)
    iters = sum(its)
    value = iters * K / (ms / 1e3)
    iter_bytes = nnz * 12 + 4 * (n + 1) + 13 * K * 8 * n
    peak, _ = peaks()
    line = base_line(args, "fp64 multi-RHS Jacobi-PCG column-iterations/s (128^3 7-point, 16 RHS)",
                     value, "column-iterations/s", ms, 1)
    line["config"] = {"workload": "multi_rhs_cg_poisson3d_7pt", "grid": [m, m, m], "n": n,
                      "rhs": K, "rtol": RTOL, "iterations_per_solve": iters // args.steps,
                      "layout": "X, B and work vectors [n][16]; matrix "
                                + ("diagonal-offset SELL (columns computed)"
                                   if A.sell().diagonal_offsets else "int32 CSR")
                                + ", shared by the columns",
                      "l2": "inputs larger than L2"}
    line["iteration_roofline"] = {"bytes_per_iter": iter_bytes,
                                  "achieved_gbs": round(iter_bytes * value / K / 1e9, 1),
                                  "alg_frac": round(iter_bytes * value / K / 1e9 / peak, 4),
                                  "bytes_formula": "12 nnz + 4 (N+1) + 13 * 16 * 8 N"}
    # K_A reads the matrix and the search directions P (formed by
    # mrhs_pform_kernel), writes AP
    sell = A.sell()
    fm = sell_format(sell)
    # 7-point diagonal view: P tiles staged in shared memory by bulk copies
    kname = ("mrhs_spmv_tile_kernel" if sell.diagonal_offsets and sell.uniform_width in (5, 7)
             else "mrhs_spmv_kernel")
    line["roofline"] = roofline(kname, nnz * 12 + 4 * (n + 1) + 2 * K * 8 * n,
                                ka_ms, ka_n, f"{kname}@mrhs:128x16",
                                fm["matrix_bytes"] + 2 * K * 8 * n)
    line["clocks"] = clk
    return line


def wl_mixed(args, dev, local):
    """Mixed-precision PCG (pytorch_solve(float32, mixed_precision=True)):
    3-D 7-point 256^3, float32 matrix and Jacobi inverse, float64 vectors,
    rtol 1e-8."""
    from torch_sla_b200 import _lib as L
    from torch_sla_b200 import problems as P
    from torch_sla_b200.backends import pytorch_backend as PB
    m = args.grid
    n = m ** 3
    v, r, c, sh = P.poisson_3d_7pt(m, dtype=torch.float32, device=dev)
    b = P.rhs_normal(n, SEED, torch.float32).to(dev)
    A = PB.CachedSparseMatrix(v, r, c, sh)
    M = PB.Float32Preconditioner(PB.get_preconditioner(A, "jacobi"))
    nnz = A.csr.nnz

    def once():
        return PB.pcg_solve_mixed_precision(A, b, atol=0.0, rtol=RTOL, maxiter=10000,
                                            preconditioner=M).num_iters

    for _ in range(args.warmup):
        once()
    L.profile_enable(True, 7)
    l0 = L.launch_count()
    ms, its, clk = timed(once, args.steps, dev, local)
    launches = L.launch_count() - l0
    ka_ms, ka_n = L.profile_read(0)
    kb_ms, kb_n = L.profile_read(1)
    kp_ms, kp_n = L.profile_read(2)
    L.profile_enable(False)
    iters = sum(its)
    value = iters / (ms / 1e3)
    peak, _ = peaks()
    # float32 matrix (8 B per entry with the int32 column), float64 vectors:
    # 11 vector passes of 8 B plus two float32 inverse-diagonal passes
    mat = matrix_bytes(nnz, n, V=4)
    iter_bytes = mat + (11 * 8 + 2 * 4) * n
    fm = sell_format(A.sell(), V=4)
    line = base_line(args, "mixed-precision Jacobi-PCG iterations/s (256^3 7-point)", value,
                     "iterations/s", ms, 1, dtype="f32 matrix / f64 vectors")
    line["config"] = {"workload": "mixed_pcg_poisson3d_7pt", "grid": [m, m, m], "n": n,
                      "nnz": nnz, "rtol": RTOL, "b": "N(0,1) seed 1, float32",
                      "iterations_per_solve": iters // args.steps, "format": fm["format"],
                      "l2": "inputs larger than L2; no flush", "parallelism": "single GPU"}
    # K_A: matrix + the float32 copy of p gathered (4 B) + p read at its own
    # row for the dot (8 B) + Ap written (8 B)
    line["roofline"] = roofline("mx_spmv_split_kernel", mat + 20 * n, ka_ms, ka_n,
                                f"mx_spmv_split_kernel@mixed:{m}", fm["matrix_bytes"] + 20 * n)
    line["roofline"]["update_kernel"] = {
        "kernel": "mx_update_kernel", "avg_launch_ms": round(kb_ms / max(kb_n, 1), 5),
        # r read/write, Ap, dinv; x two steps at odd iterations (mean 44 B per row)
        "achieved": round(44 * n / (kb_ms / max(kb_n, 1) / 1e3) / 1e9, 1) if kb_n else None}
    line["roofline"]["pform_kernel"] = {
        "kernel": "mx_pform_kernel", "avg_launch_ms": round(kp_ms / max(kp_n, 1), 5),
        # r, p_old (8 B), dinv (4 B) read; p (8 B) and its float32 copy (4 B) written
        "achieved": round(32 * n / (kp_ms / max(kp_n, 1) / 1e3) / 1e9, 1) if kp_n else None}
    line["iteration_roofline"] = {"bytes_per_iter": iter_bytes,
                                  "achieved_gbs": round(iter_bytes * value / 1e9, 1),
                                  "alg_frac": round(iter_bytes * value / 1e9 / peak, 4),
                                  "bytes_formula": "8 nnz + 4 (N+1) + (11 * 8 + 2 * 4) N"}
    line["gpu_launches"] = launches
    line["clocks"] = clk
    return line


WORKLOADS = {"pcg7": wl_pcg7, "cg2d": wl_cg2d, "spmv": wl_spmv, "batched": wl_batched,
             "bicgstab": wl_bicgstab, "mrhs": wl_mrhs, "mixed": wl_mixed}


# ------------------------------------------------------------ N GPUs
def sharded_rows(workload, m, world, rank, dev):
    from torch_sla_b200 import problems as P
    dims = (m * world, m, m)
    if workload == "pcg27":
        v, r, c = P.stencil27_rows(dims, rank * m, m, seed=4, device=dev)
    elif workload == "bicgstab":
        v, r, c = P.convdiff_3d_upwind_rows(m, rank * m, m, device=dev, nz=m * world)
    else:
        v, r, c = P.poisson_3d_7pt_rows(dims, rank * m, m, device=dev)
    return v, r, c, dims


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def run_sharded(args, world, rank, local):
    """N GPUs, one process each: rank k owns z-slab k (partition_simple), its
    shard built from its own rows only; NCCL halo + allreduces."""
    import torch.distributed as dist
    from torch_sla_b200 import _lib as L
    from torch_sla_b200 import problems as P
    from torch_sla_b200.distributed import DSparseTensor, destroy_all

    dev = torch.device("cuda", local)
    if "MASTER_ADDR" not in os.environ:  # single process outside torchrun
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(_free_port()), RANK="0",
                          WORLD_SIZE="1")
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    wl = args.workload if args.workload in ("pcg7", "pcg27", "bicgstab") else "pcg7"
    m = 192 if wl == "bicgstab" and args.grid == M else args.grid
    n_loc = m ** 3
    v, r, c, dims = sharded_rows(wl, m, world, rank, dev)
    n_glob = dims[0] * dims[1] * dims[2]
    D = DSparseTensor.from_owned_rows(v, r, c, (n_glob, n_glob), rank=rank, world=world)
    del v, r, c
    gen = P.rhs_uniform01 if wl == "bicgstab" else P.rhs_normal
    seed = 3 if wl == "bicgstab" else (4 if wl == "pcg27" else SEED)
    b_full = gen(n_glob, seed)
    b_host = b_full[rank * n_loc:(rank + 1) * n_loc].clone().pin_memory()
    del b_full
    b = b_host.to(dev)
    plan = D._shard_plan()
    nnz = plan.csr.nnz
    method = "bicgstab" if wl == "bicgstab" else "cg"

    maxiter = args.maxiter or 100000

    def once(bb=None):
        x = D.solve_distributed_shard(b if bb is None else bb, method=method,
                                      preconditioner="jacobi", atol=0.0, rtol=RTOL,
                                      maxiter=maxiter)
        return x, D._last_info["iterations"]

    for _ in range(args.warmup):
        once()
    torch.cuda.synchronize()
    dist.barrier()
    L.profile_enable(True, 7)
    if plan.p2p is not None:
        plan.p2p_timers(reset=True)
    l0 = L.launch_count()
    ms_local, outs, clk = timed(lambda: once()[1], args.steps, dev, local)
    dist.barrier()
    launches = L.launch_count() - l0
    ka_ms, ka_n = L.profile_read(0)
    kb_ms, kb_n = L.profile_read(1)
    kp_ms, kp_n = L.profile_read(2)
    L.profile_enable(False)
    timers = plan.p2p_timers(reset=True) if plan.p2p is not None else None
    t = torch.tensor([ms_local], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    iters = sum(outs)
    value = iters * world / (ms / 1e3)

    e_steps = max(1, min(args.steps, 3))
    dist.barrier()

    x_host = torch.empty_like(b_host).pin_memory()

    def e2e_once():
        x, it = once(b_host.to(dev, non_blocking=True))
        x_host.copy_(x.to_local() if hasattr(x, "to_local") else x)  # pinned read-back
        return it
    e_ms_local, e_its, _ = timed(e2e_once, e_steps, dev, local)
    te = torch.tensor([e_ms_local], dtype=torch.float64, device=dev)
    dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e_ms = float(te.item())

    halo = halo_report(D, plan, world, dev, m, timers, (kp_ms, kp_n), (ka_ms, ka_n),
                       (kb_ms, kb_n), method)
    V = 8
    interior_frac = plan.sell_int.n_slots / max(n_loc, 1)
    fm_int = sell_format(plan.sell_int, V)
    exchange = (("halo values and dot products stored into peer GPUs' memory by the solver "
                 f"kernels (CUDA IPC over NVLink), 3 launches per "
                 "iteration") if plan.p2p is not None else
                "NCCL grouped send/recv halo + allreduce per reduction point")
    mat = matrix_bytes(nnz, n_loc)
    if method == "cg":
        metric = (METRIC if wl == "pcg7" else
                  "fp64 Jacobi-PCG iterations/s (3-D 27-point, 256^3 unknowns per GPU)")
        iter_bytes = mat + 13 * V * n_loc
        if plan.p2p is not None:
            # K_A covers every owned row (interior, halo wait, boundary,
            # cross-rank sum) over the search direction K_P formed: matrix +
            # p gathered + Ap written
            ka_bytes = mat + 2 * V * n_loc
            ka_fmt = (fm_int["matrix_bytes"] + sell_format(plan.sell_bnd, V)["matrix_bytes"]
                      + 2 * V * n_loc)
            kname, rows = "shard_cg_p2p_spmv_split", "all rows, halo wait and cross-rank sum"
        else:
            # interior-row SpMV over the search direction the K_P pass formed
            ka_bytes = (mat + 2 * V * n_loc) * interior_frac
            ka_fmt = fm_int["matrix_bytes"] + 2 * V * plan.sell_int.n_slots
            kname, rows = "shard_cg_spmv_split", "interior rows"
    else:
        metric = "fp64 Jacobi-BiCGStab iterations/s (convection-diffusion, 192^3 per GPU)"
        iter_bytes = 2 * mat + 25 * V * n_loc
        if plan.p2p is not None:
            ka_bytes = mat + 6 * V * n_loc
            ka_fmt = (fm_int["matrix_bytes"] + sell_format(plan.sell_bnd, V)["matrix_bytes"]
                      + 6 * V * n_loc)
            kname, rows = "shard_bi_p2p_k1", "all rows, halo wait and cross-rank sum"
        else:
            ka_bytes = (mat + 6 * V * n_loc) * interior_frac
            ka_fmt = fm_int["matrix_bytes"] + 6 * V * plan.sell_int.n_slots
            kname, rows = "shard_bi_k1", "interior rows"
    peak, _ = peaks()
    if rank == 0:
        line = base_line(args, metric, value, "iterations/s", ms, world)
        line["config"] = {"workload": {"pcg7": "jacobi_pcg_poisson3d_7pt",
                                       "pcg27": "jacobi_pcg_stencil27",
                                       "bicgstab": "bicgstab_convdiff3d"}[wl],
                          "grid": list(dims), "n": n_glob, "n_per_gpu": n_loc,
                          "nnz_per_gpu": nnz, "rtol": RTOL,
                          "iterations_per_solve": iters // args.steps,
                          "partition": "z-slabs (partition_simple), one-layer halos",
                          "halo_bytes_per_neighbour": m * m * V, "check_every": 10,
                          "maxiter": maxiter,
                          "stopped_at_maxiter": iters // args.steps >= maxiter,
                          "format": fm_int["format"] + " interior rows; explicit boundary rows",
                          "l2": "inputs larger than L2",
                          "parallelism": f"row-sharded x{world} ({exchange})"}
        line["iteration_roofline"] = {"bytes_per_iter_per_gpu": iter_bytes,
                                      "achieved_gbs_per_gpu":
                                          round(iter_bytes * value / world / 1e9, 1),
                                      "alg_frac": round(iter_bytes * value / world / 1e9 / peak, 4)}
        line["roofline"] = roofline(f"{kname} ({rows})", ka_bytes, ka_ms, ka_n,
                                    f"{kname}@{wl}-shard:{m}", ka_fmt)
        line["e2e"] = {"value": round(sum(e_its) * world / (e_ms / 1e3), 3),
                       "unit": "iterations/s", "h2d_bytes_per_step": n_loc * V * world,
                       "d2h_bytes_per_step": n_loc * V * world,
                       "ms_per_step": round(e_ms / e_steps, 3), "steps": e_steps,
                       "api": "DSparseTensor.solve_distributed_shard, b from pinned host "
                              "memory, x read back; shard setup done once before timing"}
        line["halo"] = halo
        line["gpu_launches"] = launches
        line["clocks"] = clk
        print(json.dumps(line), flush=True)
    del D, plan
    destroy_all()
    dist.barrier()
    dist.destroy_process_group()


# Peer copy over NVLink measured on this pool's B200s (GB/s per direction);
# nominal NVLink 5 is 900 GB/s per direction per GPU.
NVLINK_PEER_GBS = 770.0


def halo_report(D, plan, world, dev, m, timers, kp, ka, kb, method):
    """Where the time of a sharded iteration goes, max over ranks: the
    in-situ CUDA-event means of the solver's kernels (K_P forms p and sends
    the halo, K_A the SpMV with the halo wait and the cross-rank (p,Ap) sum,
    K_B the update and the (r,r),(r,z) sum), the GPU-timer breakdown the
    peer-memory kernels record while profiling (mean per block: halo stores
    + fence in K_P, halo-arrival wait in K_A; the two cross-rank sums in the
    last block), and a standalone halo_exchange (NCCL grouped send/recv of
    one m^2 layer per neighbour, the reference's exchange step) timed over
    50 calls with CUDA events."""
    import torch.distributed as dist
    from torch_sla_b200.distributed import halo_exchange

    def mean(t):
        return t[0] / t[1] * 1e3 if t[1] else 0.0
    vals = [mean(kp), mean(ka), mean(kb)]
    if timers and timers["iterations"]:
        it = timers["iterations"]
        vals += [timers["send_ns"] / max(timers["kp_blocks"], 1) / 1e3,
                 timers["wait_ns"] / max(timers["ka_blocks"], 1) / 1e3,
                 timers["sum_pap_ns"] / it / 1e3, timers["sum_rr_ns"] / it / 1e3]
    else:
        vals += [-1.0, -1.0, -1.0, -1.0]
    ex_us = -1.0
    bytes_nb = m * m * 8
    if world > 1:
        xl = torch.zeros(plan.n_owned + plan.n_halo, dtype=torch.float64, device=dev)
        for _ in range(5):
            halo_exchange(D, xl)
        torch.cuda.synchronize()
        dist.barrier()
        reps = 50
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            halo_exchange(D, xl)
        e1.record()
        torch.cuda.synchronize()
        ex_us = e0.elapsed_time(e1) * 1e3 / reps
    vals.append(ex_us)
    t = torch.tensor(vals, dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    v = [round(float(a), 2) for a in t.tolist()]
    out = {"reduction": "max over ranks", "kernel_us": {"K_P": v[0], "K_A": v[1], "K_B": v[2]}
           if method == "cg" else {"K1": v[1]},
           "bytes_per_neighbour": bytes_nb,
           "neighbours_per_rank": "1 (end slabs) / 2 (middle slabs)" if world > 2 else
           ("1" if world == 2 else "0")}
    if v[3] >= 0:
        out["peer_memory_us_per_iteration"] = {
            "halo_send_per_block": v[3], "halo_wait_per_block": v[4],
            "cross_rank_sum_pap": v[5], "cross_rank_sum_rr": v[6],
            "timer": "GPU global timer in the solver kernels (profiling on)"}
    if world > 1 and v[7] > 0:
        gbs = bytes_nb / (v[7] / 1e6) / 1e9
        out["halo_exchange"] = {
            "api": "torch_sla_b200.distributed.halo_exchange (NCCL grouped send/recv)",
            "us_per_exchange": v[7], "gbs_per_direction_per_neighbour": round(gbs, 1),
            "nvlink_frac": round(gbs / NVLINK_PEER_GBS, 4),
            "nvlink_peak": f"{NVLINK_PEER_GBS} GB/s peer copy per direction (measured on this "
                           "pool); 900 nominal"}
    return out


# --------------------------------------------------------- reference arm
def run_reference(args):
    """--impl reference: torch-sla's CPU pytorch-backend arithmetic (the
    oracle port; torch-sla is pure Python, nothing to compile) on the host
    cores, same metric and config, a bounded number of PCG iterations per
    step. Under torchrun only rank 0 works."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if int(os.environ.get("RANK", "0")) != 0:
        return
    from oracle import krylov as K
    from torch_sla_b200 import problems as P
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    m = args.grid
    n = m ** 3
    v, r, c, sh = P.poisson_3d_7pt(m)
    Acpu = K.csr(v, r, c, sh)  # one-time COO sort, outside the timed region
    del v, r, c
    b = P.rhs_normal(n, SEED)
    dinv = K.jacobi_inverse(K.csr_diagonal(Acpu), "eps")
    per_step = 3
    for _ in range(args.warmup):
        K.pcg_iterations(Acpu, b, dinv, iterations=1)
    t0 = time.perf_counter()
    its = sum(K.pcg_iterations(Acpu, b, dinv, iterations=per_step) for _ in range(args.steps))
    dt = time.perf_counter() - t0
    # The host does every slab of the N-slab system in turn: one global
    # iteration costs N slab-iterations, so iterations/s x N (the metric of
    # the B200 arm) equals the one-slab rate measured here.
    value = its / dt
    line = base_line(args, METRIC, value, "iterations/s", dt * 1e3, world)
    line["impl"] = "reference"
    # the same config keys as the B200 arm's line for this workload
    line["config"] = {"workload": "jacobi_pcg_poisson3d_7pt", "grid": [m * world, m, m],
                      "n": n * world, "rtol": RTOL, "b": "N(0,1) seed 1",
                      "parallelism": "host CPU"}
    if world > 1:
        line["config"]["n_per_gpu"] = n
    else:
        line["config"]["nnz"] = int(Acpu.values().numel())
    sample = (f"{per_step} PCG iterations per step on one 256^3 slab; x{world} slabs" if world > 1
              else f"{per_step} PCG iterations per step on the 256^3 system")
    line["cpu_baseline"] = {"value": round(value, 3), "unit": "iterations/s", "cores": cores,
                            "kind": "port", "sample": sample}
    line["e2e"] = {"value": round(value, 3), "unit": "iterations/s", "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0}
    print(json.dumps(line), flush=True)


def main():
    # the JSON line must be the only output on stdout: NCCL prints its
    # version banner there at NCCL_DEBUG=VERSION and WARN, so those are
    # unset (no NCCL log at all); an explicit INFO or TRACE stays
    if os.environ.get("NCCL_DEBUG", "").upper() in ("VERSION", "WARN"):
        del os.environ["NCCL_DEBUG"]
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="pcg7",
                    choices=["pcg7", "cg2d", "spmv", "batched", "bicgstab", "pcg27", "mrhs",
                             "mixed"])
    ap.add_argument("--grid", type=int, default=M, help="grid edge per GPU (default 256)")
    ap.add_argument("--layout", default="auto", choices=["auto", "explicit"],
                    help="pcg7: the SELL view the solver picks, or the int32-column view")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--maxiter", type=int, default=0,
                    help="sharded solves: iteration cap per step (the metric stays iterations/s; "
                         "torch-sla's shard BiCGStab converges slowly at N > 1)")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1 or args.workload == "pcg27":
        return run_sharded(args, world, rank, local)
    dev = torch.device("cuda", local)
    print(json.dumps(WORKLOADS[args.workload](args, dev, local)), flush=True)


if __name__ == "__main__":
    main()
