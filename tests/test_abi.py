"""The C-ABI library loads without a GPU and exports every entry point that
include/sla_b200.h declares (no compute calls here)."""
import ctypes
import os
import re

import pytest

from torch_sla_b200 import _lib as L

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                      "sla_b200.h")


def header_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^[a-z][\w\s\*]*?\b(sla_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_the_entry_points():
    syms = header_symbols()
    assert "sla_pcg" in syms and "sla_shard_cg" in syms and "sla_csr_build" in syms
    assert len(syms) >= 28


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(L.LIB_PATH)
    missing = [s for s in header_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_binding_table_matches_header():
    assert set(L.declared_symbols()) == set(header_symbols())


def test_status_strings_and_version():
    lib = L.lib()
    assert lib.sla_abi_version() == L.ABI_VERSION == 5
    assert lib.sla_status_string(L.SLA_ERR_UNSUPPORTED) == b"unsupported problem shape"
    assert lib.sla_status_string(L.SLA_NOT_CONVERGED).startswith(b"did not converge")


def test_invalid_arguments_are_rejected_before_any_device_work():
    lib = L.lib()
    info = L.SolveInfo()
    assert lib.sla_pcg(1, None, None, None, None, 0, 0.0, 1e-8, 10, 0, None, 0,
                       ctypes.byref(info), None) == L.SLA_ERR_INVALID
    assert lib.sla_spmv(7, None, None, None, None) == L.SLA_ERR_INVALID
    assert lib.sla_pcg_mixed(None, L.SLA_MIXED_M_F32_JACOBI, None, L.SLA_F32, None, None, 0,
                             0.0, 1e-8, 10, None, 0, ctypes.byref(info), None,
                             None) == L.SLA_ERR_INVALID
    assert lib.sla_csr_build(1, None, None, None, 10, 0, 5, None, None, None, None, None,
                             None, None, 0, None) == L.SLA_ERR_INVALID
    assert lib.sla_shard_cg(None, None, None, 1, None, None, None, None, None, 0.0, 0.0, 1, 10,
                            None, 0, ctypes.byref(info), None) == L.SLA_ERR_INVALID


@pytest.mark.parametrize("n,nnz", [(10, 30), (1000, 7000)])
def test_workspace_queries(n, nnz):
    lib = L.lib()
    need = ctypes.c_size_t(0)
    assert lib.sla_csr_build_workspace(n, nnz, ctypes.byref(need)) == 0 and need.value > 0
    assert lib.sla_sell_layout_workspace(n, ctypes.byref(need)) == 0 and need.value > 0
    assert lib.sla_bicgstab_workspace(2, n, ctypes.byref(need)) == L.SLA_ERR_INVALID


def _view(**kw):
    v = L.SellView()
    v.n_slots, v.n_slices = kw.get("n_slots", 64), kw.get("n_slices", 2)
    v.slice_ptr, v.val = 1 << 20, 1 << 20  # never dereferenced: rejected on the host
    v.col = kw.get("col", None)
    v.row_ids = kw.get("row_ids", None)
    v.max_width = v.uniform_width = kw.get("width", 7)
    v.n_cols, v.row_base = kw.get("n_cols", 64), kw.get("row_base", 0)
    offs = kw.get("offsets", [-8, -4, -1, 0, 1, 4, 8])
    v.n_diags = kw.get("n_diags", len(offs))
    for i, o in enumerate(offs):
        v.diag_offsets[i] = o
    return v


@pytest.mark.parametrize("bad", [
    dict(offsets=[-8, -4, -1, 0, 1, 4, 8, 9, 10], width=9),   # 9 diagonals: no kernel for it
    dict(offsets=[-4, -8, -1, 0, 1, 4, 8]),                    # offsets not ascending
    dict(width=5),                                              # width != n_diags
    dict(n_cols=0),                                             # no column bound
    dict(row_ids=1 << 20, row_base=3),                          # row ids and a row base
    dict(n_slices=3),                                           # n_slices != ceil(n_slots / 32)
    dict(n_diags=0, col=None),                                  # explicit view without columns
])
def test_malformed_sell_views_are_rejected_on_the_host(bad):
    """sla_spmv validates the view before any CUDA call: no GPU needed."""
    v = _view(**bad)
    assert L.lib().sla_spmv(L.SLA_F64, ctypes.byref(v), 1 << 20, 1 << 20, None) == L.SLA_ERR_INVALID


@pytest.mark.parametrize("width,offsets", [(7, [-65536, -256, -1, 0, 1, 256, 65536]),
                                           (27, list(range(-13, 14)))])
def test_views_whose_int32_offsets_would_wrap_are_refused(width, offsets):
    """A uniform view addresses entry j of slice s as 32*width*s + 32*j + lane
    in int32; a view with more than 2^31 padded entries is refused with
    SLA_ERR_UNSUPPORTED before any device work (a stencil matrix with nnz just
    below the CSR builder's 2^31 limit would otherwise wrap once padded)."""
    n_slots = (2 ** 31) // (32 * width) * 32 + 32  # one slice past the limit
    v = _view(n_slots=n_slots, n_slices=(n_slots + 31) // 32, width=width, offsets=offsets,
              n_cols=n_slots)
    lib = L.lib()
    assert lib.sla_spmv(L.SLA_F64, ctypes.byref(v), 1 << 20, 1 << 20, None) == L.SLA_ERR_UNSUPPORTED
    info = L.SolveInfo()
    assert lib.sla_pcg(L.SLA_F64, ctypes.byref(v), None, 1 << 20, 1 << 20, 0, 0.0, 1e-8, 10, 0,
                       1 << 20, 1 << 40, ctypes.byref(info), None) == L.SLA_ERR_UNSUPPORTED
    # one slice fewer fits: the same view is then only refused for other reasons
    # (here the missing workspace), never for its size
    ok = _view(n_slots=n_slots - 32, n_slices=(n_slots - 32 + 31) // 32, width=width,
               offsets=offsets, n_cols=n_slots - 32)
    assert lib.sla_pcg(L.SLA_F64, ctypes.byref(ok), None, 1 << 20, 1 << 20, 0, 0.0, 1e-8, 10, 0,
                       None, 0, ctypes.byref(info), None) == L.SLA_ERR_WORKSPACE
    arr = (L.c_i32 * L.MAX_DIAGS)(*offsets)
    assert lib.sla_sell_diag_fill(L.SLA_F64, 1 << 20, 1 << 20, 1 << 20, None, n_slots, arr,
                                  width, 1 << 20, None, 0, None) == L.SLA_ERR_UNSUPPORTED


def test_misaligned_workspace_is_refused_on_the_host():
    """Solver workspaces are carved into 256-byte aligned arrays from their
    base, which the vector loads need 16-byte aligned: a base off that
    alignment is refused with SLA_ERR_WORKSPACE before any device work."""
    v = _view()
    info = L.SolveInfo()
    lib = L.lib()
    need = ctypes.c_size_t(0)
    assert lib.sla_bicgstab_workspace(L.SLA_F64, 64, ctypes.byref(need)) == 0
    assert lib.sla_bicgstab(L.SLA_F64, ctypes.byref(v), None, 1 << 20, 1 << 20, 0, 0.0, 1e-8,
                            10, (1 << 20) + 8, need.value, ctypes.byref(info),
                            None) == L.SLA_ERR_WORKSPACE
