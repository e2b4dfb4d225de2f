"""Device-resident int32 CSR and SELL-32 views built by libsla_b200.

`DeviceCSR` replaces the COO -> CSR conversion that torch-sla's
`CachedSparseMatrix` performs on every solve
(backends/pytorch_backend.py:114-152); the conversion, the SELL-32 layout
used by the solver kernels and the Jacobi diagonal are all built on the GPU.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib as L


class Sell:
    """SELL-32 view (slice pointers, padded columns/values) of some CSR rows.

    uniform_width > 0 marks a layout whose slices all have that width, which
    the kernels address arithmetically. A diagonal-offset view (`offsets`
    given, `col` None) stores no columns: entry j of a row belongs to column
    row + offsets[j]."""

    def __init__(self, slice_ptr, col, val, n_slots, row_ids=None, max_width=0,
                 uniform_width=0, n_cols=0, offsets=None):
        self.slice_ptr, self.col, self.val = slice_ptr, col, val
        self.row_base = 0
        # a contiguous run of rows is addressed as row_base + slot (no row
        # id loads in the kernels)
        if row_ids is not None and row_ids.numel() > 0:
            r0 = int(row_ids[0])
            if int(row_ids[-1]) - r0 + 1 == row_ids.numel() and bool(
                    (row_ids[1:] - row_ids[:-1] == 1).all()):
                row_ids, self.row_base = None, r0
        self.row_ids = row_ids
        self.n_slots = int(n_slots)
        self.n_slices = (self.n_slots + 31) // 32
        self.max_width = int(max_width)
        self.uniform_width = int(uniform_width)
        self.n_cols = int(n_cols)
        self.offsets = list(offsets) if offsets else []
        self.sigma = 1  # rows sorted by length inside windows of sigma rows (explicit views)
        self.long_rows = None  # hybrid SpMV views: rows summed by the warp-per-row CSR pass
        arr = (L.c_i32 * L.MAX_DIAGS)(*self.offsets)
        self.view = L.SellView(self.n_slots, self.n_slices, L.ptr(slice_ptr), L.ptr(col),
                               L.ptr(val), L.ptr(self.row_ids), self.max_width,
                               self.uniform_width, self.n_cols, self.row_base,
                               len(self.offsets), arr)

    def ref(self):
        return ctypes.byref(self.view)

    @property
    def diagonal_offsets(self) -> bool:
        return bool(self.offsets)

    @property
    def padded_nnz(self) -> int:
        return int(self.val.numel())


class DeviceCSR:
    """int32 CSR of a COO matrix, with duplicates summed in input order.

    keep_map=True also keeps `src_index` (input position of each sorted
    entry) and `seg_ptr` (sorted-entry range of each CSR entry), which the
    batched solver uses to gather per-matrix values.
    """

    def __init__(self, val, row, col, shape, *, keep_map: bool = False, dtype=None):
        n_rows, n_cols = int(shape[0]), int(shape[1])
        dev = L.require_cuda(row, col, val)
        if val is not None:
            dtype = val.dtype
            val = val.contiguous()
        self.dtype = dtype
        self.code = L.dtype_code(dtype)
        self.device = dev
        self.shape = (n_rows, n_cols)
        row = row.to(device=dev, dtype=torch.int64).contiguous()
        col = col.to(device=dev, dtype=torch.int64).contiguous()
        nnz = int(row.numel())
        if col.numel() != nnz or (val is not None and val.numel() != nnz):
            raise ValueError("torch_sla_b200: row, col and values must have the same length")
        lib = L.lib()
        need = ctypes.c_size_t(0)
        L.check("sla_csr_build_workspace", lib.sla_csr_build_workspace(n_rows, nnz, ctypes.byref(need)))
        ws = L.workspace(need.value, dev)
        rowptr = torch.empty(n_rows + 1, dtype=torch.int32, device=dev)
        colind = torch.empty(max(nnz, 1), dtype=torch.int32, device=dev)
        vals = torch.empty(max(nnz, 1), dtype=dtype, device=dev)
        src = torch.empty(max(nnz, 1), dtype=torch.int64, device=dev) if keep_map else None
        seg = torch.empty(nnz + 1, dtype=torch.int32, device=dev) if keep_map else None
        out = ctypes.c_int64(0)
        L.check("sla_csr_build", lib.sla_csr_build(
            self.code, L.ptr(row), L.ptr(col), L.ptr(val), nnz, n_rows, n_cols, L.ptr(rowptr),
            L.ptr(colind), L.ptr(vals) if val is not None else None, L.ptr(src), L.ptr(seg),
            ctypes.byref(out), L.ptr(ws), ws.numel(), L.stream_handle(dev)))
        self.nnz = int(out.value)
        self.rowptr = rowptr
        self.colind = colind[: self.nnz]
        self.vals = vals[: self.nnz] if val is not None else None
        self.src_index = src[:nnz] if keep_map else None
        self.seg_ptr = seg[: self.nnz + 1] if keep_map else None
        self._sell = None

    # ------------------------------------------------------------------ SELL
    # widths the kernels have diagonal-offset instantiations for
    DIAG_WIDTHS = (5, 7, 27)
    # largest padding (zero entries / stored entries) a diagonal-offset view
    # may add over the rows' own entries
    DIAG_MAX_PAD = 0.10

    # SELL-32-sigma: an explicit view of all rows sorts the rows by length
    # inside windows of SIGMA rows when the sigma = 1 layout pads more than
    # SIGMA_PAD over the stored entries, and keeps the sorted layout when it
    # moves at least SIGMA_GAIN fewer bytes per SpMV (row ids read and the
    # scattered row writes charged to it)
    SIGMA = 4096
    SIGMA_PAD = 0.10
    SIGMA_GAIN = 0.05

    def sell(self, row_ids: torch.Tensor | None = None, values: torch.Tensor | None = None,
             n_cols: int | None = None, diagonal: bool = True,
             sigma: int | None = None) -> Sell:
        """SELL-32 view of all rows (row_ids=None) or of the listed rows.

        When the rows' columns lie on 5, 7 or 27 diagonals (stencil
        matrices) the view stores no column indices (diagonal-offset
        layout); `n_cols` bounds the columns the kernels may touch (default:
        the matrix's column count) and must exceed every stored column of
        the rows. diagonal=False forces the explicit layout. sigma (explicit
        views of all rows): 1 keeps row order, a power of two in [32, 4096]
        sorts rows by length inside windows of that many rows (SELL-C-sigma),
        None picks between them by the bytes each layout moves."""
        cacheable = (row_ids is None and values is None and n_cols is None and diagonal
                     and sigma is None)
        if cacheable and self._sell is not None:
            return self._sell
        vals = self.vals if values is None else values
        if vals is None:
            raise ValueError("torch_sla_b200: SELL view needs matrix values")
        lib = L.lib()
        dev = self.device
        n_slots = self.shape[0] if row_ids is None else int(row_ids.numel())
        if row_ids is not None:
            row_ids = row_ids.to(device=dev, dtype=torch.int32).contiguous()
        n_cols = self.shape[1] if n_cols is None else int(n_cols)
        n_slices = (n_slots + 31) // 32
        stream = L.stream_handle(dev)
        s = self._diagonal_view(row_ids, n_slots, n_cols, vals, stream) if diagonal else None
        if s is None:
            s = self._explicit_view(row_ids, n_slots, n_cols, vals, stream, sigma)
        if cacheable:
            self._sell = s
        return s

    def _diag_offsets(self, row_ids, n_slots, stream):
        """Ascending diagonal offsets of the listed rows when they fit a
        diagonal-offset view (5, 7 or 27 diagonals, padding <= DIAG_MAX_PAD),
        else None, plus the probe workspace."""
        if n_slots == 0 or self.nnz == 0:
            return None, None
        lib = L.lib()
        need = ctypes.c_size_t(0)
        L.check("sla_sell_diag_probe_workspace", lib.sla_sell_diag_probe_workspace(ctypes.byref(need)))
        ws = L.workspace(need.value, self.device)
        offs = (L.c_i32 * L.MAX_DIAGS)()
        count = L.c_i32(0)
        L.check("sla_sell_diag_probe", lib.sla_sell_diag_probe(
            L.ptr(self.rowptr), L.ptr(self.colind), L.ptr(row_ids), n_slots, offs,
            ctypes.byref(count), L.ptr(ws), ws.numel(), stream))
        w = int(count.value)
        if w not in self.DIAG_WIDTHS:
            return None, ws
        if row_ids is None:
            nnz_view = self.nnz
        else:
            rl = row_ids.to(torch.int64)
            nnz_view = int((self.rowptr[rl + 1] - self.rowptr[rl]).sum())
        padded = (n_slots + 31) // 32 * 32 * w
        if padded > (1.0 + self.DIAG_MAX_PAD) * max(nnz_view, 1):
            return None, ws
        if padded > 2 ** 31 - 1:  # entry offsets are int32 in the kernels
            return None, ws
        return list(offs)[:w], ws

    def diag_pattern(self):
        """(offsets, positions) of the whole matrix as a diagonal-offset view
        -- positions[k] is CSR entry k's place in that view -- or None."""
        stream = L.stream_handle(self.device)
        offs, ws = self._diag_offsets(None, self.shape[0], stream)
        if offs is None or self.shape[0] != self.shape[1]:
            return None
        pos = torch.empty(max(self.nnz, 1), dtype=torch.int64, device=self.device)
        arr = (L.c_i32 * L.MAX_DIAGS)(*offs)
        L.check("sla_sell_diag_positions", L.lib().sla_sell_diag_positions(
            L.ptr(self.rowptr), L.ptr(self.colind), self.shape[0], arr, len(offs), L.ptr(pos),
            L.ptr(ws), ws.numel(), stream))
        return offs, pos[: self.nnz]

    def _diagonal_view(self, row_ids, n_slots, n_cols, vals, stream):
        offs, ws = self._diag_offsets(row_ids, n_slots, stream)
        if offs is None:
            return None
        lib = L.lib()
        dev = self.device
        w = len(offs)
        n_slices = (n_slots + 31) // 32
        padded = n_slices * 32 * w
        arr = (L.c_i32 * L.MAX_DIAGS)(*offs)
        sval = torch.empty(padded, dtype=self.dtype, device=dev)
        L.check("sla_sell_diag_fill", lib.sla_sell_diag_fill(
            self.code, L.ptr(self.rowptr), L.ptr(self.colind), L.ptr(vals), L.ptr(row_ids),
            n_slots, arr, w, L.ptr(sval), L.ptr(ws), ws.numel(), stream))
        slice_ptr = (torch.arange(n_slices + 1, device=dev, dtype=torch.int64) * (32 * w)).to(
            torch.int32)
        return Sell(slice_ptr, None, sval, n_slots, row_ids, max_width=w, uniform_width=w,
                    n_cols=n_cols, offsets=offs)

    def sigma_order(self, sigma: int, row_ids: torch.Tensor | None = None) -> torch.Tensor:
        """Rows of the view (row_ids, or all rows) sorted by decreasing length
        inside windows of `sigma` rows (sla_sell_sigma_order)."""
        n_slots = self.shape[0] if row_ids is None else int(row_ids.numel())
        order = torch.empty(max(n_slots, 1), dtype=torch.int32, device=self.device)[:n_slots]
        L.check("sla_sell_sigma_order", L.lib().sla_sell_sigma_order(
            L.ptr(self.rowptr), L.ptr(row_ids), n_slots, int(sigma), L.ptr(order),
            L.stream_handle(self.device)))
        return order

    def _explicit_view(self, row_ids, n_slots, n_cols, vals, stream, sigma=None):
        lib = L.lib()
        dev = self.device
        n_slices = (n_slots + 31) // 32
        slice_ptr = torch.empty(n_slices + 1, dtype=torch.int32, device=dev)
        need = ctypes.c_size_t(0)
        L.check("sla_sell_layout_workspace", lib.sla_sell_layout_workspace(n_slots, ctypes.byref(need)))
        ws = L.workspace(need.value, dev)
        padded = ctypes.c_int64(0)
        widest = ctypes.c_int32(0)

        def layout(min_width):
            L.check("sla_sell_layout", lib.sla_sell_layout(
                L.ptr(self.rowptr), L.ptr(row_ids), n_slots, int(min_width), L.ptr(slice_ptr),
                ctypes.byref(padded), ctypes.byref(widest), L.ptr(ws), ws.numel(), stream))

        layout(0)
        used_sigma = 1
        if row_ids is None and n_slots > 0 and sigma != 1:
            want = sigma if sigma is not None else self.SIGMA
            if sigma is not None or padded.value > (1.0 + self.SIGMA_PAD) * max(self.nnz, 1):
                V = torch.empty((), dtype=self.dtype).element_size()
                plain_bytes = padded.value * (V + 4)
                plain = padded.value
                order = self.sigma_order(want)
                row_ids = order
                layout(0)
                # row id loads (4 B) and the scattered row writes (up to a
                # 32 B sector for an 8 B value) are charged to the sorted view
                sorted_bytes = padded.value * (V + 4) + 28 * n_slots
                if sigma is None and sorted_bytes > (1.0 - self.SIGMA_GAIN) * plain_bytes:
                    row_ids = None
                    layout(0)
                    assert padded.value == plain
                else:
                    used_sigma = want
        uniform = 0
        w = int(widest.value)
        # pad every slice to the widest one when that costs <= 3 % more
        # entries: the kernels then address slices arithmetically
        if 0 < w <= 32 and n_slices * 32 * w <= 1.03 * padded.value:
            layout(w)
            uniform = w
        scol = torch.empty(max(padded.value, 1), dtype=torch.int32, device=dev)
        sval = torch.empty(max(padded.value, 1), dtype=self.dtype, device=dev)
        L.check("sla_sell_fill", lib.sla_sell_fill(
            self.code, L.ptr(self.rowptr), L.ptr(self.colind), L.ptr(vals), L.ptr(row_ids), n_slots,
            L.ptr(slice_ptr), L.ptr(scol), L.ptr(sval), stream))
        view = Sell(slice_ptr, scol, sval, n_slots, row_ids, max_width=widest.value,
                    uniform_width=uniform, n_cols=n_cols)
        view.sigma = used_sigma
        return view

    # --------------------------------------------------------------- helpers
    def jacobi_inverse(self, rule: int, n_rows: int | None = None) -> torch.Tensor:
        n = self.shape[0] if n_rows is None else int(n_rows)
        dinv = torch.empty(max(n, 1), dtype=self.dtype, device=self.device)[:n]
        L.check("sla_jacobi_inverse", L.lib().sla_jacobi_inverse(
            self.code, L.ptr(self.rowptr), L.ptr(self.colind), L.ptr(self.vals), n, rule,
            L.ptr(dinv), L.stream_handle(self.device)))
        return dinv

    def diagonal(self) -> torch.Tensor:
        rows = torch.repeat_interleave(
            torch.arange(self.shape[0], device=self.device),
            (self.rowptr[1:] - self.rowptr[:-1]).to(torch.int64))
        mask = rows == self.colind.to(torch.int64)
        d = torch.zeros(self.shape[0], dtype=self.dtype, device=self.device)
        d.index_add_(0, rows[mask], self.vals[mask])
        return d

    # hybrid SpMV (matvec only): rows longer than LONG_ROW_MIN entries, and
    # longer than LONG_ROW_AVG times the average row, go to a warp-per-row
    # CSR pass (sla_spmv_rows_csr) over the CSR arrays themselves; the other
    # rows form a SELL-32-sigma view
    LONG_ROW_MIN = 64
    LONG_ROW_AVG = 8

    def spmv_view(self) -> Sell:
        """The view `matvec` runs on: the solvers' view (`sell()`), or, when
        that is a length-sorted explicit view whose longest rows exceed the
        long-row threshold, a hybrid: a SELL-32-sigma view of the shorter rows
        plus the list of long rows (`view.long_rows`) for the warp-per-row
        pass. Long rows are summed lane-strided (agrees with the sequential
        sum to rounding); every other row is bitwise the same as in `sell()`."""
        if getattr(self, "_spmv_view", None) is not None:
            return self._spmv_view
        base = self.sell()
        view = base
        if base.sigma > 1 and self.vals is not None:
            lens = (self.rowptr[1:] - self.rowptr[:-1]).to(torch.int64)
            avg = max(1.0, self.nnz / max(self.shape[0], 1))
            limit = max(self.LONG_ROW_MIN, int(self.LONG_ROW_AVG * avg + 0.999))
            long_mask = lens > limit
            n_long = int(long_mask.sum())
            if n_long > 0:
                rows = torch.arange(self.shape[0], device=self.device, dtype=torch.int32)
                short = rows[~long_mask]
                order = self.sigma_order(self.SIGMA, row_ids=short) if short.numel() else short
                view = self._explicit_view(order, int(short.numel()), self.shape[1], self.vals,
                                           L.stream_handle(self.device), sigma=1)
                view.sigma = self.SIGMA
                view.long_rows = rows[long_mask].contiguous()
                view.csr_arrays = (self.rowptr, self.colind, self.vals)
        self._spmv_view = view
        return view

    def matvec(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        return spmv(self.spmv_view(), x, self.shape[0], out)


def spmv(sell: Sell, x: torch.Tensor, n_out: int, out: torch.Tensor | None = None) -> torch.Tensor:
    x = x.contiguous()
    if out is None:
        out = torch.empty(n_out, dtype=x.dtype, device=x.device)
    code, stream = L.dtype_code(x.dtype), L.stream_handle(x.device)
    L.check("sla_spmv", L.lib().sla_spmv(code, sell.ref(), L.ptr(x), L.ptr(out), stream))
    long_rows = getattr(sell, "long_rows", None)
    if long_rows is not None:
        rowptr, colind, vals = sell.csr_arrays
        L.check("sla_spmv_rows_csr", L.lib().sla_spmv_rows_csr(
            code, L.ptr(rowptr), L.ptr(colind), L.ptr(vals), L.ptr(long_rows),
            int(long_rows.numel()), L.ptr(x), L.ptr(out), stream))
    return out


def coo_value_grad(row, col, a, b, n_a, n_b, K=1, batch=1) -> torch.Tensor:
    """g[k] = -sum_c a[row[k], c] * b[col[k], c] (per batch member)."""
    nnz = int(row.numel())
    a = a.contiguous()
    b = b.contiguous()
    g = torch.empty((batch, nnz) if batch > 1 else (nnz,), dtype=a.dtype, device=a.device)
    L.check("sla_coo_value_grad", L.lib().sla_coo_value_grad(
        L.dtype_code(a.dtype), L.ptr(row), L.ptr(col), nnz, L.ptr(a), L.ptr(b), n_a, n_b, K,
        batch, L.ptr(g), L.stream_handle(a.device)))
    return g
