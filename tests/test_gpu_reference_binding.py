"""torch-sla itself, unchanged, running on the B200 kernels after
torch_sla_b200.patch.install().

A maintainer binds this backend into torch-sla by rebinding its patch points
(pytorch_solve, batched_cg_same_pattern and the shard functions). This test
imports an installed torch-sla, installs the binding, and calls torch-sla's
own public API with CUDA tensors: spsolve with method='cg' and 'bicgstab'
and a backward pass (SparseLinearSolvePyTorch, linear_solve.py:283-324),
spsolve_batch_same_layout with a backward pass
(BatchSparseLinearSolveSameLayout, batch_solve.py:46-177) and
SparseTensor.solve. It checks that libsla_b200 kernels ran and that the
results match the fixtures torch-sla produced on the CPU.

torch-sla is looked for in $TORCH_SLA_REF, then in baseline/_ref (the
offline install of the reference package beside this repository); the test
skips when neither holds it. It runs in a fresh interpreter so the rebinding
does not leak into other tests.
"""
import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

from conftest import torch_sla_path

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


SCRIPT = r"""
import json, sys, warnings
sys.path.insert(0, {ref!r}); sys.path.insert(0, {repo!r}); sys.path.insert(0, {tests!r})
import torch
import torch_sla
import torch_sla_b200.patch as patch
from torch_sla_b200 import _lib as L
from conftest import load_golden, case_inputs

warnings.simplefilter("ignore")
done = patch.install(torch_sla)
dev = torch.device("cuda", 0)
g = load_golden()

def rel(a, b):
    a = a.detach().double().cpu(); b = b.detach().double().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-300))

out = {{"rebound": len(done)}}
n0 = L.launch_count()
for key, method in (("adj_cg_3d8", "cg"), ("adj_bicg_cd6", "bicgstab")):
    case = g[key]
    v, r, c, sh = case_inputs(case)
    vg = v.to(dev).requires_grad_(True)
    bg = case["b"].to(dev).requires_grad_(True)
    x = torch_sla.spsolve(vg, r.to(dev), c.to(dev), sh, bg, backend="pytorch", method=method)
    (x * x).sum().backward()
    out[key] = [x.is_cuda, rel(x, case["x"]), rel(vg.grad, case["grad_val"]),
                rel(bg.grad, case["grad_b"])]
case = g["batched_d2d12"]
vb, r, c, sh, bb = case_inputs(case)
vbg = vb.to(dev).requires_grad_(True)
bbg = bb.to(dev).requires_grad_(True)
U = torch_sla.spsolve_batch_same_layout(vbg, r.to(dev), c.to(dev), sh, bbg, method="cg",
                                        atol=1e-10, maxiter=10000)
(U * U).sum().backward()
out["batched"] = [U.is_cuda, rel(U, case["U_autograd"]), rel(vbg.grad, case["grad_val"]),
                  rel(bbg.grad, case["grad_b"])]
case = g["st_solve_2d10"]
v, r, c, sh = case_inputs(case)
A = torch_sla.SparseTensor(v.to(dev), r.to(dev), c.to(dev), sh)
xs = A.solve(case["b"].to(dev))
out["st_solve"] = [xs.is_cuda, rel(xs, case["x"])]
torch.cuda.synchronize()
out["launches"] = L.launch_count() - n0
print("RESULT " + json.dumps(out))
"""


def test_installed_torch_sla_runs_on_b200_kernels():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    ref = torch_sla_path()
    if ref is None:
        pytest.skip("torch-sla not found (set TORCH_SLA_REF or install it into baseline/_ref)")
    code = SCRIPT.format(ref=ref, repo=REPO, tests=os.path.join(REPO, "tests"))
    proc = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                          env={**os.environ, "PYTHONDONTWRITEBYTECODE": "1"}, timeout=600)
    assert proc.returncode == 0, proc.stderr[-3000:]
    line = [ln for ln in proc.stdout.splitlines() if ln.startswith("RESULT ")][-1]
    out = json.loads(line[len("RESULT "):])
    assert out["rebound"] >= 8
    # every call went through libsla_b200 (CSR build, SELL views, solvers,
    # adjoint value gradients): dozens of kernels at least
    assert out["launches"] >= 50, out
    for key in ("adj_cg_3d8", "adj_bicg_cd6", "batched"):
        is_cuda, ex, egv, egb = out[key]
        assert is_cuda, key
        # the reference's own fixtures: x and both gradients within 1e-8
        assert ex < 1e-8 and egv < 1e-8 and egb < 1e-8, (key, out[key])
    is_cuda, es = out["st_solve"]
    # SparseTensor.solve: torch-sla's auto choice on the CPU was a direct
    # solve; on CUDA without cuDSS it is the pytorch backend at rtol 1e-10
    assert is_cuda and es < 1e-8, out["st_solve"]
