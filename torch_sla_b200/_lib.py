"""ctypes binding of libsla_b200.so (C ABI declared in include/sla_b200.h).

Everything below the Python mirror of torch-sla's interface goes through
these entry points; there is no CPU fallback. Loading the library needs no
GPU (it links the CUDA runtime statically), but every compute call requires
CUDA tensors and raises otherwise.
"""
from __future__ import annotations

import ctypes
import os
import warnings

import torch

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libsla_b200.so")

SLA_F32, SLA_F64 = 0, 1
SLA_OK, SLA_NOT_CONVERGED, SLA_BREAKDOWN = 0, 1, 2
SLA_ERR_INVALID, SLA_ERR_CUDA, SLA_ERR_NCCL = -1, -2, -3
SLA_ERR_TIMEOUT, SLA_ERR_UNSUPPORTED, SLA_ERR_WORKSPACE, SLA_ERR_INDEX = -4, -5, -6, -7
SLA_JACOBI_EPS, SLA_JACOBI_CLAMP, SLA_JACOBI_NONZERO = 0, 1, 2
SLA_PCG_AUTO, SLA_PCG_STREAMED, SLA_PCG_PERSISTENT, SLA_PCG_CLUSTER = 0, 1, 2, 3
SLA_PCG_NOALLOC_SCRATCH_BYTES = 16 << 20  # size of sla_pcg_noalloc's fixed device array
SLA_MIXED_M_F32_NONE, SLA_MIXED_M_F32_JACOBI, SLA_MIXED_M_F64_JACOBI, SLA_MIXED_M_F64_NONE = (
    0, 1, 2, 3)

c_i32, c_i64, c_dbl, c_ptr, c_sz = (ctypes.c_int32, ctypes.c_int64, ctypes.c_double,
                                    ctypes.c_void_p, ctypes.c_size_t)


MAX_DIAGS = 32  # SLA_MAX_DIAGS
ABI_VERSION = 5  # SLA_ABI_VERSION


class SellView(ctypes.Structure):
    _fields_ = [("n_slots", c_i64), ("n_slices", c_i64), ("slice_ptr", c_ptr),
                ("col", c_ptr), ("val", c_ptr), ("row_ids", c_ptr), ("max_width", c_i32),
                ("uniform_width", c_i32), ("n_cols", c_i64), ("row_base", c_i64),
                ("n_diags", c_i32),
                ("diag_offsets", c_i32 * MAX_DIAGS)]


class SolveInfo(ctypes.Structure):
    _fields_ = [("iterations", c_i64), ("residual", c_dbl), ("status", c_i32),
                ("reason", c_i32)]


class HaloPlan(ctypes.Structure):
    _fields_ = [("n_neighbors", c_i32), ("neighbor_rank", c_ptr), ("send_offset", c_ptr),
                ("recv_offset", c_ptr), ("send_index", c_ptr), ("halo_src", c_ptr),
                ("n_owned", c_i64), ("n_halo", c_i64)]


_P = ctypes.POINTER
_SIGNATURES = {
    "sla_abi_version": (ctypes.c_int, []),
    "sla_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "sla_kernel_launch_count": (c_i64, []),
    "sla_profile_enable": (ctypes.c_int, [ctypes.c_int, ctypes.c_int]),
    "sla_profile_read": (ctypes.c_int, [ctypes.c_int, _P(c_dbl), _P(c_i64)]),
    "sla_csr_build_workspace": (ctypes.c_int, [c_i64, c_i64, _P(c_sz)]),
    "sla_csr_build": (ctypes.c_int, [ctypes.c_int, c_ptr, c_ptr, c_ptr, c_i64, c_i64, c_i64,
                                     c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, _P(c_i64), c_ptr, c_sz,
                                     c_ptr]),
    "sla_sell_layout_workspace": (ctypes.c_int, [c_i64, _P(c_sz)]),
    "sla_sell_layout": (ctypes.c_int, [c_ptr, c_ptr, c_i64, c_i32, c_ptr, _P(c_i64), _P(c_i32),
                                       c_ptr, c_sz, c_ptr]),
    "sla_sell_fill": (ctypes.c_int, [ctypes.c_int, c_ptr, c_ptr, c_ptr, c_ptr, c_i64, c_ptr,
                                     c_ptr, c_ptr, c_ptr]),
    "sla_sell_sigma_order": (ctypes.c_int, [c_ptr, c_ptr, c_i64, c_i32, c_ptr, c_ptr]),
    "sla_sell_diag_probe_workspace": (ctypes.c_int, [_P(c_sz)]),
    "sla_sell_diag_probe": (ctypes.c_int, [c_ptr, c_ptr, c_ptr, c_i64, _P(c_i32), _P(c_i32),
                                           c_ptr, c_sz, c_ptr]),
    "sla_sell_diag_positions": (ctypes.c_int, [c_ptr, c_ptr, c_i64, _P(c_i32), c_i32, c_ptr,
                                               c_ptr, c_sz, c_ptr]),
    "sla_sell_diag_fill": (ctypes.c_int, [ctypes.c_int, c_ptr, c_ptr, c_ptr, c_ptr, c_i64,
                                          _P(c_i32), c_i32, c_ptr, c_ptr, c_sz, c_ptr]),
    "sla_jacobi_inverse": (ctypes.c_int, [ctypes.c_int, c_ptr, c_ptr, c_ptr, c_i64,
                                          ctypes.c_int, c_ptr, c_ptr]),
    "sla_spmv": (ctypes.c_int, [ctypes.c_int, _P(SellView), c_ptr, c_ptr, c_ptr]),
    "sla_spmv_rows_csr": (ctypes.c_int, [ctypes.c_int, c_ptr, c_ptr, c_ptr, c_ptr, c_i64, c_ptr,
                                         c_ptr, c_ptr]),
    "sla_coo_value_grad": (ctypes.c_int, [ctypes.c_int, c_ptr, c_ptr, c_i64, c_ptr, c_ptr,
                                          c_i64, c_i64, c_i64, c_i64, c_ptr, c_ptr]),
    "sla_pcg_workspace": (ctypes.c_int, [ctypes.c_int, c_i64, _P(c_sz)]),
    "sla_pcg": (ctypes.c_int, [ctypes.c_int, _P(SellView), c_ptr, c_ptr, c_ptr, ctypes.c_int,
                               c_dbl, c_dbl, c_i64, ctypes.c_int, c_ptr, c_sz, _P(SolveInfo),
                               c_ptr]),
    "sla_pcg_noalloc": (ctypes.c_int, [ctypes.c_int, _P(SellView), c_ptr, c_ptr, c_ptr,
                                       ctypes.c_int, c_dbl, c_dbl, c_i64, ctypes.c_int,
                                       _P(SolveInfo), c_ptr]),
    "sla_pcg_mixed_workspace": (ctypes.c_int, [c_i64, _P(c_sz)]),
    "sla_pcg_mixed": (ctypes.c_int, [_P(SellView), ctypes.c_int, c_ptr, ctypes.c_int, c_ptr,
                                     c_ptr, ctypes.c_int, c_dbl, c_dbl, c_i64, c_ptr, c_sz,
                                     _P(SolveInfo), _P(c_dbl), c_ptr]),
    "sla_bicgstab_workspace": (ctypes.c_int, [ctypes.c_int, c_i64, _P(c_sz)]),
    "sla_bicgstab": (ctypes.c_int, [ctypes.c_int, _P(SellView), c_ptr, c_ptr, c_ptr,
                                    ctypes.c_int, c_dbl, c_dbl, c_i64, c_ptr, c_sz,
                                    _P(SolveInfo), c_ptr]),
    "sla_batched_values": (ctypes.c_int, [ctypes.c_int, c_ptr, c_i64, c_i64, c_ptr, c_ptr,
                                          c_i64, c_ptr, c_ptr]),
    "sla_batched_values_at": (ctypes.c_int, [ctypes.c_int, c_ptr, c_i64, c_i64, c_ptr, c_ptr,
                                             c_i64, c_ptr, c_i64, c_ptr, c_ptr]),
    "sla_batched_cg_diag": (ctypes.c_int, [ctypes.c_int, _P(SellView), c_ptr, c_i64, c_ptr,
                                           c_ptr, c_dbl, c_dbl, c_i64, c_ptr, c_sz,
                                           _P(SolveInfo), c_ptr]),
    "sla_batched_cg_workspace": (ctypes.c_int, [ctypes.c_int, c_i64, c_i64, _P(c_sz)]),
    "sla_batched_cg": (ctypes.c_int, [ctypes.c_int, c_ptr, c_ptr, c_ptr, c_i64, c_i64, c_ptr,
                                      c_ptr, c_dbl, c_dbl, c_i64, c_ptr, c_sz, _P(SolveInfo),
                                      c_ptr]),
    "sla_multi_rhs_cg_workspace": (ctypes.c_int, [ctypes.c_int, c_i64, c_i64, _P(c_sz)]),
    "sla_multi_rhs_cg": (ctypes.c_int, [ctypes.c_int, c_ptr, c_ptr, c_ptr, c_i64, c_i64, c_ptr,
                                        c_ptr, c_ptr, ctypes.c_int, c_dbl, c_dbl, c_i64, c_i64,
                                        c_ptr, c_ptr, c_ptr, c_sz, _P(SolveInfo), c_ptr]),
    "sla_multi_rhs_cg_diag": (ctypes.c_int, [ctypes.c_int, _P(SellView), c_i64, c_ptr, c_ptr,
                                             c_ptr, ctypes.c_int, c_dbl, c_dbl, c_i64, c_i64,
                                             c_ptr, c_ptr, c_ptr, c_sz, _P(SolveInfo), c_ptr]),
    "sla_comm_unique_id": (ctypes.c_int, [c_ptr]),
    "sla_comm_init": (ctypes.c_int, [_P(c_ptr), ctypes.c_int, c_ptr, ctypes.c_int]),
    "sla_comm_destroy": (ctypes.c_int, [c_ptr]),
    "sla_halo_exchange": (ctypes.c_int, [c_ptr, _P(HaloPlan), ctypes.c_int, c_ptr, c_ptr,
                                         c_ptr, c_ptr]),
    "sla_shard_spmv": (ctypes.c_int, [c_ptr, _P(HaloPlan), ctypes.c_int, _P(SellView),
                                      _P(SellView), c_ptr, c_ptr, c_ptr, c_ptr, c_ptr]),
    "sla_reverse_halo_exchange": (ctypes.c_int, [c_ptr, _P(HaloPlan), ctypes.c_int, c_ptr, c_ptr,
                                                 c_ptr, c_ptr]),
    "sla_shard_rmatvec": (ctypes.c_int, [c_ptr, _P(HaloPlan), ctypes.c_int, _P(SellView), c_ptr,
                                         c_ptr, c_ptr, c_ptr, c_ptr]),
    "sla_shard_krylov_workspace": (ctypes.c_int, [ctypes.c_int, c_i64, c_i64, c_i64, _P(c_sz)]),
    "sla_shard_cg": (ctypes.c_int, [c_ptr, c_ptr, _P(HaloPlan), ctypes.c_int, _P(SellView),
                                    _P(SellView), c_ptr, c_ptr, c_ptr, c_dbl, c_dbl, c_i64, c_i64,
                                    c_ptr, c_sz, _P(SolveInfo), c_ptr]),
    "sla_shard_bicgstab": (ctypes.c_int, [c_ptr, c_ptr, _P(HaloPlan), ctypes.c_int,
                                          _P(SellView), _P(SellView), c_ptr, c_ptr, c_ptr, c_dbl,
                                          c_dbl, c_i64, c_i64, c_ptr, c_sz, _P(SolveInfo),
                                          c_ptr]),
    "sla_p2p_create": (ctypes.c_int, [c_ptr, _P(HaloPlan), ctypes.c_int, _P(c_ptr)]),
    "sla_p2p_destroy": (ctypes.c_int, [c_ptr]),
    "sla_p2p_profile_read": (ctypes.c_int, [c_ptr, ctypes.c_int, _P(ctypes.c_ulonglong),
                                            ctypes.c_int]),
    "sla_shard_cg_p2p": (ctypes.c_int, [c_ptr, _P(HaloPlan), ctypes.c_int, _P(SellView),
                                        _P(SellView), c_ptr, c_ptr, c_ptr, c_dbl, c_dbl, c_i64,
                                        c_i64, c_ptr, c_sz, _P(SolveInfo), c_ptr]),
    "sla_shard_bicgstab_p2p": (ctypes.c_int, [c_ptr, _P(HaloPlan), ctypes.c_int, _P(SellView),
                                              _P(SellView), c_ptr, c_ptr, c_ptr, c_dbl, c_dbl,
                                              c_i64, c_i64, c_ptr, c_sz, _P(SolveInfo), c_ptr]),
}

_lib = None


def declared_symbols() -> list[str]:
    return sorted(_SIGNATURES)


def lib():
    """Load libsla_b200.so once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"torch_sla_b200: {LIB_PATH} is missing; build it with "
            "`python -m torch_sla_b200.build` (nvcc, sm_100a)")
    handle = ctypes.CDLL(LIB_PATH)
    handle.sla_abi_version.restype = ctypes.c_int
    if handle.sla_abi_version() != ABI_VERSION:
        raise RuntimeError(f"torch_sla_b200: {LIB_PATH} has interface version "
                           f"{handle.sla_abi_version()}, this package needs {ABI_VERSION}; "
                           "rebuild it with `python -m torch_sla_b200.build`")
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(handle, name, None)
        if fn is None:
            continue
        fn.restype = res
        fn.argtypes = args
    _lib = handle
    return handle


class SlaError(RuntimeError):
    """A negative status from libsla_b200."""

    def __init__(self, fn: str, status: int):
        msg = lib().sla_status_string(status).decode()
        super().__init__(f"torch_sla_b200: {fn} failed with status {status} ({msg})")
        self.status = status


def check(fn: str, status: int) -> int:
    if status == SLA_ERR_INDEX:
        raise ValueError(f"torch_sla_b200: {fn}: COO index outside the matrix shape")
    if status < 0:
        raise SlaError(fn, status)
    return status


def dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.float64:
        return SLA_F64
    if dtype == torch.float32:
        return SLA_F32
    if dtype.is_complex:
        raise TypeError("torch_sla_b200 implements the real (float32/float64) "
                        "path only; complex matrices are not supported")
    raise TypeError(f"torch_sla_b200: unsupported dtype {dtype}")


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    """The product path runs only on CUDA tensors: no CPU fallback."""
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise RuntimeError(
                "torch_sla_b200 runs the solve on the GPU only; move the matrix "
                "and right-hand side to a CUDA device (no CPU fallback)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"torch_sla_b200: tensors on different devices ({dev}, {t.device})")
    return dev


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def stream_handle(device=None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def workspace(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


def launch_count() -> int:
    return int(lib().sla_kernel_launch_count())


def profile_enable(enable: bool, sample_every: int = 8) -> None:
    lib().sla_profile_enable(int(enable), int(sample_every))


def profile_read(kernel_class: int) -> tuple[float, int]:
    ms, n = c_dbl(0.0), c_i64(0)
    check("sla_profile_read", lib().sla_profile_read(kernel_class, ctypes.byref(ms),
                                                     ctypes.byref(n)))
    return ms.value, n.value


def warn_once(msg: str) -> None:
    warnings.warn(msg)
