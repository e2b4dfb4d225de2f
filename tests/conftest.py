import os
import sys

import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

GOLDEN = os.path.join(REPO, "tests", "golden")


def torch_sla_path():
    """Directory holding an installed torch-sla package: $TORCH_SLA_REF, then
    baseline/_ref (the offline install beside this repository); None when
    neither has it."""
    for cand in (os.environ.get("TORCH_SLA_REF"), os.path.join(REPO, "baseline", "_ref")):
        if cand and os.path.isdir(os.path.join(cand, "torch_sla")):
            return cand
    return None


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and libsla_b200.so")


def load_golden(name="golden.pt"):
    return torch.load(os.path.join(GOLDEN, name), weights_only=False)


def case_inputs(case):
    """(val, row, col, shape) of a fixture: stored COO or a problems.* spec."""
    from torch_sla_b200 import problems as P
    if "gen" in case:
        name, args, kw = case["gen"]
        out = getattr(P, name)(*args, **kw)
        if name == "stencil27_rows":
            v, r, c = out
            n = args[0][0] * args[0][1] * args[0][2]
            return v, r, c, (n, n)
        if name == "diffusion_2d_batched":
            return out
        return out
    return case["val"], case["row"], case["col"], tuple(case["shape"])


@pytest.fixture(scope="session")
def golden():
    return load_golden()


@pytest.fixture(scope="session")
def golden_shard():
    return load_golden("golden_shard.pt")


def cuda_ok():
    return torch.cuda.is_available()


@pytest.fixture(scope="session")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda", 0)
