// COO -> CSR on the device, SELL-32 layout/fill and the Jacobi inverse
// diagonal.
//
// COO -> CSR (replaces torch.sparse_coo_tensor(...).to_sparse_csr() in
// CachedSparseMatrix, backends/pytorch_backend.py:138-142). Input whose
// (row, col) keys strictly increase is copied through (see the sorted fast
// path below); otherwise: bucket entries by
// row with an atomic histogram + exclusive scan, sort each row by
// (col, input position) so duplicates are merged in input order, then emit
// int32 CSR. Rows of <= 32 entries sort in registers of one thread, rows of
// <= 2048 entries in shared memory of one block, longer rows with an
// in-place bitonic network in global memory.
#include <algorithm>

#include "common.cuh"

namespace sla {

// ------------------------------------------------------------------ scan
constexpr int kScanItems = 8;
constexpr int kScanTile = kBlock * kScanItems;

template <typename In>
__global__ void scan_tile_kernel(const In *__restrict__ in, int64_t *__restrict__ out,
                                 int64_t n, int64_t *__restrict__ tile_sums) {
  __shared__ int64_t warp_tot[kWarps];
  const int64_t base = (int64_t)blockIdx.x * kScanTile + (int64_t)threadIdx.x * kScanItems;
  int64_t v[kScanItems];
  int64_t s = 0;
#pragma unroll
  for (int i = 0; i < kScanItems; ++i) {
    int64_t idx = base + i;
    v[i] = idx < n ? (int64_t)in[idx] : 0;
    s += v[i];
  }
  // inclusive warp scan of per-thread sums
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int64_t inc = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int64_t t = __shfl_up_sync(kFull, inc, o);
    if (lane >= o) inc += t;
  }
  if (lane == 31) warp_tot[warp] = inc;
  __syncthreads();
  int64_t warp_off = 0;
  for (int w = 0; w < warp; ++w) warp_off += warp_tot[w];
  int64_t run = warp_off + inc - s;  // exclusive prefix of this thread
#pragma unroll
  for (int i = 0; i < kScanItems; ++i) {
    int64_t idx = base + i;
    if (idx < n) out[idx] = run;
    run += v[i];
  }
  if (threadIdx.x == kBlock - 1) tile_sums[blockIdx.x] = warp_off + inc;
}

__global__ void scan_add_kernel(int64_t *__restrict__ out, int64_t n,
                                const int64_t *__restrict__ tile_off) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; i < n; i += stride) out[i] += tile_off[i / kScanTile];
}

static size_t scan_workspace(int64_t n) {
  size_t bytes = 0;
  while (n > kScanTile) {
    int64_t tiles = (n + kScanTile - 1) / kScanTile;
    bytes += 2 * align_up(tiles * sizeof(int64_t));
    n = tiles;
  }
  return bytes + 2 * align_up(sizeof(int64_t));
}

// Exclusive scan of n values into int64 out. ws must hold scan_workspace(n).
template <typename In>
static int exclusive_scan(const In *in, int64_t *out, int64_t n, char *ws,
                          cudaStream_t s) {
  if (n <= 0) return SLA_OK;
  int64_t tiles = (n + kScanTile - 1) / kScanTile;
  int64_t *sums = (int64_t *)ws;
  ws += align_up(tiles * sizeof(int64_t));
  int64_t *offs = (int64_t *)ws;
  ws += align_up(tiles * sizeof(int64_t));
  SLA_LAUNCH(scan_tile_kernel<In>, (unsigned)tiles, kBlock, 0, s, in, out, n, sums);
  if (tiles > 1) {
    SLA_TRY(exclusive_scan<int64_t>(sums, offs, tiles, ws, s));
    SLA_LAUNCH(scan_add_kernel, grid_for(n), kBlock, 0, s, out, n, offs);
  }
  return SLA_OK;
}

// -------------------------------------------------------------- COO -> CSR
__global__ void coo_count_kernel(const int64_t *__restrict__ row, const int64_t *__restrict__ col,
                                 int64_t nnz, int64_t n_rows, int64_t n_cols,
                                 int32_t *__restrict__ counts, int32_t *__restrict__ err) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; i < nnz; i += stride) {
    int64_t r = row[i], c = col[i];
    if (r < 0 || r >= n_rows || c < 0 || c >= n_cols) { atomicOr(err, 1); continue; }
    atomicAdd(counts + r, 1);
  }
}

__global__ void coo_scatter_kernel(const int64_t *__restrict__ row, const int64_t *__restrict__ col,
                                   int64_t nnz, const int64_t *__restrict__ rowstart,
                                   int32_t *__restrict__ cursor, int32_t *__restrict__ tcol,
                                   int32_t *__restrict__ tidx) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; i < nnz; i += stride) {
    int64_t r = row[i];
    int64_t pos = rowstart[r] + atomicAdd(cursor + r, 1);
    tcol[pos] = (int32_t)col[i];
    tidx[pos] = (int32_t)i;
  }
}

__device__ __forceinline__ bool key_less(int32_t c0, int32_t i0, int32_t c1, int32_t i1) {
  return c0 < c1 || (c0 == c1 && i0 < i1);
}

constexpr int kSmallRow = 32;
constexpr int kSmemRow = 2048;

// One thread per row: insertion sort of rows up to kSmallRow entries;
// longer rows are queued for the block sorter.
__global__ void row_sort_small_kernel(const int64_t *__restrict__ rowstart, int64_t n_rows,
                                      int32_t *__restrict__ tcol, int32_t *__restrict__ tidx,
                                      int32_t *__restrict__ long_rows, int32_t *__restrict__ n_long) {
  int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; r < n_rows; r += stride) {
    int64_t b = rowstart[r], e = rowstart[r + 1];
    int len = (int)(e - b);
    if (len <= 1) continue;
    if (len > kSmallRow) {
      int slot = atomicAdd(n_long, 1);
      long_rows[slot] = (int32_t)r;
      continue;
    }
    int32_t kc[kSmallRow], ki[kSmallRow];
    for (int j = 0; j < len; ++j) { kc[j] = tcol[b + j]; ki[j] = tidx[b + j]; }
    for (int j = 1; j < len; ++j) {
      int32_t c = kc[j], x = ki[j];
      int k = j - 1;
      while (k >= 0 && key_less(c, x, kc[k], ki[k])) { kc[k + 1] = kc[k]; ki[k + 1] = ki[k]; --k; }
      kc[k + 1] = c; ki[k + 1] = x;
    }
    for (int j = 0; j < len; ++j) { tcol[b + j] = kc[j]; tidx[b + j] = ki[j]; }
  }
}

// Direction-free bitonic network over len elements (virtual +inf padding to
// the next power of two): every compare-exchange puts the smaller key at the
// lower index, so padding never has to move.
template <bool SHARED>
__device__ void bitonic_sort(int32_t *kc, int32_t *ki, int len) {
  int P = 1;
  while (P < len) P <<= 1;
  for (int k = 2; k <= P; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < P; i += blockDim.x) {
        int partner = (j == (k >> 1)) ? (i ^ (k - 1)) : (i ^ j);
        if (partner > i && partner < len) {
          int32_t c0 = kc[i], i0 = ki[i], c1 = kc[partner], i1 = ki[partner];
          if (key_less(c1, i1, c0, i0)) {
            kc[i] = c1; ki[i] = i1; kc[partner] = c0; ki[partner] = i0;
          }
        }
      }
      if (SHARED) __syncthreads(); else { __threadfence_block(); __syncthreads(); }
    }
  }
}

__global__ void row_sort_long_kernel(const int64_t *__restrict__ rowstart,
                                     int32_t *__restrict__ tcol, int32_t *__restrict__ tidx,
                                     const int32_t *__restrict__ long_rows,
                                     const int32_t *__restrict__ n_long) {
  __shared__ int32_t sc[kSmemRow];
  __shared__ int32_t si[kSmemRow];
  const int count = *n_long;
  for (int q = blockIdx.x; q < count; q += gridDim.x) {
    int64_t r = long_rows[q];
    int64_t b = rowstart[r];
    int len = (int)(rowstart[r + 1] - b);
    if (len <= kSmemRow) {
      for (int j = threadIdx.x; j < len; j += blockDim.x) { sc[j] = tcol[b + j]; si[j] = tidx[b + j]; }
      __syncthreads();
      bitonic_sort<true>(sc, si, len);
      for (int j = threadIdx.x; j < len; j += blockDim.x) { tcol[b + j] = sc[j]; tidx[b + j] = si[j]; }
      __syncthreads();
    } else {
      bitonic_sort<false>(tcol + b, tidx + b, len);
      __syncthreads();
    }
  }
}

__global__ void row_unique_kernel(const int64_t *__restrict__ rowstart, int64_t n_rows,
                                  const int32_t *__restrict__ tcol, int32_t *__restrict__ ucount) {
  int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; r < n_rows; r += stride) {
    int64_t b = rowstart[r], e = rowstart[r + 1];
    int32_t u = 0;
    for (int64_t t = b; t < e; ++t) u += (t == b || tcol[t] != tcol[t - 1]) ? 1 : 0;
    ucount[r] = u;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) ucount[n_rows] = 0;
}

__global__ void rowptr_narrow_kernel(const int64_t *__restrict__ p64, int64_t n, int32_t *__restrict__ p32) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; i < n; i += stride) p32[i] = (int32_t)p64[i];
}

template <typename T>
__global__ void row_emit_kernel(const int64_t *__restrict__ rowstart, const int64_t *__restrict__ rp64,
                                int64_t n_rows, int64_t nnz, const int32_t *__restrict__ tcol,
                                const int32_t *__restrict__ tidx, const T *__restrict__ val,
                                int32_t *__restrict__ colind, T *__restrict__ vals,
                                int64_t *__restrict__ src_index, int32_t *__restrict__ seg_ptr) {
  int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; r < n_rows; r += stride) {
    int64_t b = rowstart[r], e = rowstart[r + 1];
    int64_t out = rp64[r] - 1;
    T acc = T(0);
    for (int64_t t = b; t < e; ++t) {
      int32_t idx = tidx[t];
      if (src_index) src_index[t] = idx;
      bool fresh = (t == b || tcol[t] != tcol[t - 1]);
      if (fresh) {
        if (out >= rp64[r] && vals) vals[out] = acc;
        ++out;
        colind[out] = tcol[t];
        if (seg_ptr) seg_ptr[out] = (int32_t)t;
        acc = val ? val[idx] : T(0);
      } else if (val) {
        acc = add_rn(acc, val[idx]);
      }
    }
    if (e > b && vals) vals[out] = acc;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0 && seg_ptr) seg_ptr[rp64[n_rows]] = (int32_t)nnz;
}

// ------------------------------------------- already-sorted COO fast path
// A COO whose (row, col) keys strictly increase is already in CSR order with
// no duplicates: the CSR is the narrowed input, row pointers come from the
// row boundaries, and the sort/merge passes (which would reproduce exactly
// these arrays) are skipped. flags[0]: an index outside the shape;
// flags[2]: some key does not exceed its predecessor.
__global__ void coo_sorted_check_kernel(const int64_t *__restrict__ row,
                                        const int64_t *__restrict__ col, int64_t nnz,
                                        int64_t n_rows, int64_t n_cols,
                                        int32_t *__restrict__ flags) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  bool bad = false, unsorted = false;
  for (; i < nnz; i += stride) {
    const int64_t r = row[i], c = col[i];
    if (r < 0 || r >= n_rows || c < 0 || c >= n_cols) { bad = true; continue; }
    if (i > 0) {
      const int64_t rp = row[i - 1], cp = col[i - 1];
      if (rp > r || (rp == r && cp >= c)) unsorted = true;
    }
  }
  if (bad) atomicOr(flags, 1);
  if (unsorted) atomicOr(flags + 2, 1);
}

// rowptr[r] = number of entries of rows < r, written at each row boundary
// (positions 0 .. nnz; the rows of a gap between two boundaries are empty).
__global__ void sorted_rowptr_kernel(const int64_t *__restrict__ row, int64_t nnz, int64_t n_rows,
                                     int32_t *__restrict__ rowptr) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; i <= nnz; i += stride) {
    const int64_t prev = i == 0 ? -1 : row[i - 1];
    const int64_t cur = i == nnz ? n_rows : row[i];
    for (int64_t r = prev + 1; r <= cur; ++r) rowptr[r] = (int32_t)i;
  }
}

template <typename T>
__global__ void sorted_emit_kernel(const int64_t *__restrict__ col, const T *__restrict__ val,
                                   int64_t nnz, int32_t *__restrict__ colind, T *__restrict__ vals,
                                   int64_t *__restrict__ src_index, int32_t *__restrict__ seg_ptr) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; i < nnz; i += stride) {
    colind[i] = (int32_t)col[i];
    if (vals) vals[i] = val ? val[i] : T(0);
    if (src_index) src_index[i] = i;
    if (seg_ptr) seg_ptr[i] = (int32_t)i;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0 && seg_ptr) seg_ptr[nnz] = (int32_t)nnz;
}

struct CsrWs {
  int32_t *counts, *cursor, *tcol, *tidx, *ucount, *long_rows, *flags;
  int64_t *rowstart, *rp64;
  char *scan;
};

static size_t csr_ws_bytes(int64_t n_rows, int64_t nnz) {
  Sizer z;
  z.take<int32_t>(n_rows + 1);  // counts
  z.take<int32_t>(n_rows + 1);  // cursor
  z.take<int32_t>(nnz + 1);     // tcol
  z.take<int32_t>(nnz + 1);     // tidx
  z.take<int32_t>(n_rows + 1);  // ucount
  z.take<int32_t>(n_rows + 1);  // long_rows
  z.take<int32_t>(8);           // flags: [0]=err [1]=n_long
  z.take<int64_t>(n_rows + 1);  // rowstart
  z.take<int64_t>(n_rows + 1);  // rp64
  return z.off + scan_workspace(n_rows + 1);
}

template <typename T>
static int csr_build_impl(const int64_t *row, const int64_t *col, const T *val, int64_t nnz,
                          int64_t n_rows, int64_t n_cols, int32_t *rowptr, int32_t *colind,
                          T *vals, int64_t *src_index, int32_t *seg_ptr, int64_t *nnz_out,
                          void *workspace, size_t ws_bytes, cudaStream_t s) {
  if (n_rows <= 0 || n_cols <= 0 || nnz < 0 || !rowptr || !nnz_out) return SLA_ERR_INVALID;
  if (n_rows >= INT32_MAX || n_cols >= INT32_MAX || nnz >= INT32_MAX) return SLA_ERR_UNSUPPORTED;
  if (nnz > 0 && (!row || !col || !colind)) return SLA_ERR_INVALID;
  if (ws_bytes < csr_ws_bytes(n_rows, nnz)) return SLA_ERR_WORKSPACE;
  Carver c(workspace, ws_bytes);
  CsrWs w;
  w.counts = c.take<int32_t>(n_rows + 1);
  w.cursor = c.take<int32_t>(n_rows + 1);
  w.tcol = c.take<int32_t>(nnz + 1);
  w.tidx = c.take<int32_t>(nnz + 1);
  w.ucount = c.take<int32_t>(n_rows + 1);
  w.long_rows = c.take<int32_t>(n_rows + 1);
  w.flags = c.take<int32_t>(8);
  w.rowstart = c.take<int64_t>(n_rows + 1);
  w.rp64 = c.take<int64_t>(n_rows + 1);
  w.scan = (char *)c.base + c.off;
  if (!c.ok) return SLA_ERR_WORKSPACE;
  SLA_CUDA_TRY(cudaMemsetAsync(w.flags, 0, sizeof(int32_t) * 8, s));
  if (nnz > 0) {
    SLA_LAUNCH(coo_sorted_check_kernel, grid_for(nnz), kBlock, 0, s, row, col, nnz, n_rows,
               n_cols, w.flags);
    int32_t f[3] = {0, 0, 0};
    SLA_CUDA_TRY(cudaMemcpyAsync(f, w.flags, sizeof(f), cudaMemcpyDeviceToHost, s));
    SLA_CUDA_TRY(cudaStreamSynchronize(s));
    if (f[0]) return SLA_ERR_INDEX;
    if (!f[2]) {
      SLA_LAUNCH(sorted_rowptr_kernel, grid_for(nnz + 1), kBlock, 0, s, row, nnz, n_rows, rowptr);
      SLA_LAUNCH(sorted_emit_kernel<T>, grid_for(nnz), kBlock, 0, s, col, val, nnz, colind, vals,
                 src_index, seg_ptr);
      *nnz_out = nnz;
      return SLA_OK;
    }
    SLA_CUDA_TRY(cudaMemsetAsync(w.flags, 0, sizeof(int32_t) * 8, s));
  }
  SLA_CUDA_TRY(cudaMemsetAsync(w.counts, 0, sizeof(int32_t) * (n_rows + 1), s));
  SLA_CUDA_TRY(cudaMemsetAsync(w.cursor, 0, sizeof(int32_t) * (n_rows + 1), s));
  if (nnz > 0)
    SLA_LAUNCH(coo_count_kernel, grid_for(nnz), kBlock, 0, s, row, col, nnz, n_rows, n_cols,
               w.counts, w.flags);
  SLA_TRY(exclusive_scan<int32_t>(w.counts, w.rowstart, n_rows + 1, w.scan, s));
  int32_t host_flags[2] = {0, 0};
  SLA_CUDA_TRY(cudaMemcpyAsync(host_flags, w.flags, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
  SLA_CUDA_TRY(cudaStreamSynchronize(s));
  if (host_flags[0]) return SLA_ERR_INDEX;
  if (nnz > 0) {
    SLA_LAUNCH(coo_scatter_kernel, grid_for(nnz), kBlock, 0, s, row, col, nnz, w.rowstart,
               w.cursor, w.tcol, w.tidx);
    SLA_LAUNCH(row_sort_small_kernel, grid_for(n_rows), kBlock, 0, s, w.rowstart, n_rows,
               w.tcol, w.tidx, w.long_rows, w.flags + 1);
    SLA_LAUNCH(row_sort_long_kernel, device_info().sm_count * 2, kBlock, 0, s, w.rowstart,
               w.tcol, w.tidx, w.long_rows, w.flags + 1);
  }
  SLA_LAUNCH(row_unique_kernel, grid_for(n_rows), kBlock, 0, s, w.rowstart, n_rows, w.tcol,
             w.ucount);
  SLA_TRY(exclusive_scan<int32_t>(w.ucount, w.rp64, n_rows + 1, w.scan, s));
  SLA_LAUNCH(rowptr_narrow_kernel, grid_for(n_rows + 1), kBlock, 0, s, w.rp64, n_rows + 1, rowptr);
  SLA_LAUNCH(row_emit_kernel<T>, grid_for(n_rows), kBlock, 0, s, w.rowstart, w.rp64, n_rows, nnz,
             w.tcol, w.tidx, val, colind, vals, src_index, seg_ptr);
  int64_t total = 0;
  SLA_CUDA_TRY(cudaMemcpyAsync(&total, w.rp64 + n_rows, sizeof(int64_t), cudaMemcpyDeviceToHost, s));
  SLA_CUDA_TRY(cudaStreamSynchronize(s));
  *nnz_out = total;
  return SLA_OK;
}

// --------------------------------------------------------------- SELL-32
__global__ void sell_width_kernel(const int32_t *__restrict__ rowptr, const int32_t *__restrict__ row_ids,
                                  int64_t n_slots, int64_t n_slices, int32_t min_width,
                                  int64_t *__restrict__ slice_len, int32_t *__restrict__ max_width) {
  const int lane = threadIdx.x & 31;
  int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t sl = warp; sl < n_slices; sl += nwarps) {
    int64_t slot = sl * 32 + lane;
    int len = 0;
    if (slot < n_slots) {
      int64_t r = row_ids ? row_ids[slot] : slot;
      len = rowptr[r + 1] - rowptr[r];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) len = max(len, __shfl_xor_sync(kFull, len, o));
    if (lane == 0) {
      atomicMax(max_width, len);
      slice_len[sl] = (int64_t)max(len, (int)min_width) * 32;
    }
  }
}

template <typename T>
__global__ void sell_fill_kernel(const int32_t *__restrict__ rowptr, const int32_t *__restrict__ colind,
                                 const T *__restrict__ vals, const int32_t *__restrict__ row_ids,
                                 int64_t n_slots, int64_t n_slices, const int32_t *__restrict__ slice_ptr,
                                 int32_t *__restrict__ scol, T *__restrict__ sval) {
  int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; t < n_slices * 32; t += stride) {
    int64_t sl = t >> 5;
    int lane = (int)(t & 31);
    int32_t base = slice_ptr[sl];
    int width = (slice_ptr[sl + 1] - base) >> 5;
    int32_t rb = 0, len = 0;
    if (t < n_slots) {
      int64_t r = row_ids ? row_ids[t] : t;
      rb = rowptr[r];
      len = rowptr[r + 1] - rb;
    }
    for (int j = 0; j < width; ++j) {
      int64_t o = (int64_t)base + 32 * j + lane;
      if (j < len) {
        scol[o] = colind[rb + j];
        sval[o] = vals ? vals[rb + j] : T(0);
      } else {
        scol[o] = -1;
        sval[o] = T(0);
      }
    }
  }
}

// ------------------------------------------------------------- SELL-C-sigma
// Row order of a SELL-32-sigma view: inside each window of sigma consecutive
// rows (of the listed rows, or of all rows) the rows are sorted by decreasing
// length, equal lengths in ascending row order, so each 32-row slice holds
// rows of similar length and pads less. One block per window sorts the keys
// (INT32_MAX - length) << 32 | position in shared memory (bitonic network,
// sigma a power of two in [32, 4096]). The sorted window is then rotated by
// (window mod sigma/32) slices: the widest slice of window w sits at slice
// w mod (sigma/32) of the window, not always at its start, so the kernels'
// grid-stride slice walks (whose warp count is a multiple of 32) do not hand
// every window's widest slice to the same few warps. The last window, when
// partial, is not rotated.
constexpr int kSigmaMax = 4096;

__global__ void __launch_bounds__(1024)
sigma_order_kernel(const int32_t *__restrict__ rowptr, const int32_t *__restrict__ row_ids,
                   int64_t n_slots, int sigma, int32_t *__restrict__ order) {
  extern __shared__ unsigned long long key[];
  const int64_t w0 = (int64_t)blockIdx.x * sigma;
  for (int i = threadIdx.x; i < sigma; i += blockDim.x) {
    const int64_t t = w0 + i;
    unsigned long long k = ~0ull;  // empty positions sort last
    if (t < n_slots) {
      const int64_t r = row_ids ? row_ids[t] : t;
      const unsigned len = (unsigned)(rowptr[r + 1] - rowptr[r]);
      k = ((unsigned long long)(0x7fffffffu - len) << 32) | (unsigned)i;
    }
    key[i] = k;
  }
  __syncthreads();
  for (int size = 2; size <= sigma; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < sigma; i += blockDim.x) {
        const int j = i ^ stride;
        if (j > i) {
          const unsigned long long a = key[i], b = key[j];
          if ((a > b) == ((i & size) == 0)) {
            key[i] = b;
            key[j] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  const bool full = w0 + sigma <= n_slots;
  const int rot = full ? (int)(blockIdx.x % (unsigned)(sigma / 32)) * 32 : 0;
  for (int i = threadIdx.x; i < sigma; i += blockDim.x) {
    const int64_t t = w0 + i;
    if (t < n_slots) {
      const int k = (i - rot + sigma) & (sigma - 1);
      const int64_t src = w0 + (int64_t)(key[k] & 0xffffffffull);
      order[t] = row_ids ? row_ids[src] : (int32_t)src;
    }
  }
}

template <typename T>
__global__ void jacobi_kernel(const int32_t *__restrict__ rowptr, const int32_t *__restrict__ colind,
                              const T *__restrict__ vals, int64_t n, int rule, T *__restrict__ dinv) {
  int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const T eps100 = (sizeof(T) == 8) ? T(2.220446049250313e-14) : T(1.1920928955078125e-05);
  for (; r < n; r += stride) {
    T d = T(0);
    for (int32_t k = rowptr[r]; k < rowptr[r + 1]; ++k)
      if (colind[k] == (int32_t)r) d = add_rn(d, vals[k]);
    T out;
    if (rule == SLA_JACOBI_EPS) {
      T dd = (fabs(d) < eps100) ? T(1) : d;
      out = T(1) / dd;
    } else if (rule == SLA_JACOBI_CLAMP) {
      T dd = (d > T(1e-30)) ? d : T(1e-30);
      if (d != d) dd = d;  // clamp_min propagates NaN
      out = T(1) / dd;
    } else {
      out = (fabs(d) > T(0)) ? T(1) / d : T(1);
    }
    dinv[r] = out;
  }
}


// ------------------------------------------------ diagonal-offset SELL views
// Distinct col - row values of the listed rows: each block collects them in
// a 64-slot shared table (insert only after a miss), then merges its table
// into the global one. More than 32 distinct values sets the overflow flag.
constexpr int kDiagTable = 64;
constexpr int32_t kDiagEmpty = INT32_MIN;

__device__ __forceinline__ bool diag_insert(int32_t *tab, int32_t d) {
  unsigned h = ((unsigned)d * 2654435761u) >> 26;  // 6 bits
  for (int probe = 0; probe < kDiagTable; ++probe, h = (h + 1) & (kDiagTable - 1)) {
    int32_t cur = ((volatile int32_t *)tab)[h];
    if (cur == d) return true;
    if (cur == kDiagEmpty) {
      cur = atomicCAS(tab + h, kDiagEmpty, d);
      if (cur == kDiagEmpty || cur == d) return true;
    }
  }
  return false;  // table full
}

__global__ void __launch_bounds__(kBlock)
diag_probe_kernel(const int32_t *__restrict__ rowptr, const int32_t *__restrict__ colind,
                  const int32_t *__restrict__ row_ids, int64_t n_slots, int32_t *gtab,
                  int *overflow) {
  __shared__ int32_t tab[kDiagTable];
  __shared__ int full;
  for (int i = threadIdx.x; i < kDiagTable; i += blockDim.x) tab[i] = kDiagEmpty;
  if (threadIdx.x == 0) full = 0;
  __syncthreads();
  int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; t < n_slots; t += stride) {
    if (*(volatile int *)&full) break;
    const int64_t r = row_ids ? row_ids[t] : t;
    for (int32_t k = rowptr[r]; k < rowptr[r + 1]; ++k) {
      const int32_t d = (int32_t)((int64_t)colind[k] - r);
      if (!diag_insert(tab, d)) { full = 1; break; }
    }
  }
  __syncthreads();
  if (full) {
    if (threadIdx.x == 0) atomicExch(overflow, 1);
    return;
  }
  for (int i = threadIdx.x; i < kDiagTable; i += blockDim.x)
    if (tab[i] != kDiagEmpty && !diag_insert(gtab, tab[i])) atomicExch(overflow, 1);
}

__global__ void diag_table_init_kernel(int32_t *gtab, int *overflow) {
  if (threadIdx.x < kDiagTable) gtab[threadIdx.x] = kDiagEmpty;
  if (threadIdx.x == 0) *overflow = 0;
}

struct DiagOffsets {
  int32_t n;
  int32_t off[SLA_MAX_DIAGS];
};

// Scatter the CSR entries of each slot onto its diagonal position; the value
// array is zeroed beforehand. An entry on no listed diagonal sets *bad.
template <typename T>
__global__ void __launch_bounds__(kBlock)
diag_fill_kernel(const int32_t *__restrict__ rowptr, const int32_t *__restrict__ colind,
                 const T *__restrict__ vals, const int32_t *__restrict__ row_ids, int64_t n_slots,
                 DiagOffsets D, T *__restrict__ sval, int *bad) {
  int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; t < n_slots; t += stride) {
    const int64_t r = row_ids ? row_ids[t] : t;
    const int64_t base = (t >> 5) * 32 * D.n + (t & 31);
    for (int32_t k = rowptr[r]; k < rowptr[r + 1]; ++k) {
      const int64_t d = (int64_t)colind[k] - r;
      int lo = 0, hi = D.n - 1, j = -1;
      while (lo <= hi) {
        const int mid = (lo + hi) >> 1;
        if (D.off[mid] == d) { j = mid; break; }
        if (D.off[mid] < d) lo = mid + 1; else hi = mid - 1;
      }
      if (j < 0) { atomicExch(bad, 1); continue; }
      sval[base + 32 * j] = vals[k];
    }
  }
}

// Position of every CSR entry in a diagonal-offset view of all rows:
// (row / 32) * 32 * W + 32 * j + row % 32, j the entry's diagonal.
__global__ void __launch_bounds__(kBlock)
diag_pos_kernel(const int32_t *__restrict__ rowptr, const int32_t *__restrict__ colind,
                int64_t n_rows, DiagOffsets D, int64_t *__restrict__ pos, int *bad) {
  int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; r < n_rows; r += stride) {
    const int64_t base = (r >> 5) * 32 * D.n + (r & 31);
    for (int32_t k = rowptr[r]; k < rowptr[r + 1]; ++k) {
      const int64_t d = (int64_t)colind[k] - r;
      int lo = 0, hi = D.n - 1, j = -1;
      while (lo <= hi) {
        const int mid = (lo + hi) >> 1;
        if (D.off[mid] == d) { j = mid; break; }
        if (D.off[mid] < d) lo = mid + 1; else hi = mid - 1;
      }
      if (j < 0) { atomicExch(bad, 1); pos[k] = -1; continue; }
      pos[k] = base + 32 * j;
    }
  }
}

}  // namespace sla

using namespace sla;

extern "C" {

int sla_csr_build_workspace(int64_t n_rows, int64_t nnz, size_t *bytes) {
  if (!bytes || n_rows < 0 || nnz < 0) return SLA_ERR_INVALID;
  *bytes = csr_ws_bytes(n_rows, nnz);
  return SLA_OK;
}

int sla_csr_build(int dtype, const int64_t *row, const int64_t *col, const void *val, int64_t nnz,
                  int64_t n_rows, int64_t n_cols, int32_t *rowptr, int32_t *colind, void *vals,
                  int64_t *src_index, int32_t *seg_ptr, int64_t *nnz_out, void *workspace,
                  size_t workspace_bytes, sla_stream_t stream) {
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == SLA_F64)
    return csr_build_impl<double>(row, col, (const double *)val, nnz, n_rows, n_cols, rowptr,
                                  colind, (double *)vals, src_index, seg_ptr, nnz_out, workspace,
                                  workspace_bytes, s);
  if (dtype == SLA_F32)
    return csr_build_impl<float>(row, col, (const float *)val, nnz, n_rows, n_cols, rowptr, colind,
                                 (float *)vals, src_index, seg_ptr, nnz_out, workspace,
                                 workspace_bytes, s);
  return SLA_ERR_INVALID;
}

int sla_sell_layout_workspace(int64_t n_slots, size_t *bytes) {
  if (!bytes || n_slots < 0) return SLA_ERR_INVALID;
  int64_t n_slices = (n_slots + 31) / 32;
  *bytes = 2 * align_up((n_slices + 1) * sizeof(int64_t)) + align_up(sizeof(int32_t)) +
           scan_workspace(n_slices + 1);
  return SLA_OK;
}

int sla_sell_layout(const int32_t *rowptr, const int32_t *row_ids, int64_t n_slots,
                    int32_t min_width, int32_t *slice_ptr, int64_t *padded_out,
                    int32_t *max_width_out, void *workspace, size_t workspace_bytes,
                    sla_stream_t stream) {
  cudaStream_t s = (cudaStream_t)stream;
  if (!rowptr || !slice_ptr || !padded_out || n_slots < 0 || min_width < 0) return SLA_ERR_INVALID;
  size_t need = 0;
  sla_sell_layout_workspace(n_slots, &need);
  if (workspace_bytes < need) return SLA_ERR_WORKSPACE;
  int64_t n_slices = (n_slots + 31) / 32;
  Carver c(workspace, workspace_bytes);
  int64_t *len = c.take<int64_t>(n_slices + 1);
  int64_t *ptr64 = c.take<int64_t>(n_slices + 1);
  int32_t *wmax = c.take<int32_t>(1);
  if (!c.ok) return SLA_ERR_WORKSPACE;
  char *scan = c.base + c.off;
  SLA_CUDA_TRY(cudaMemsetAsync(len, 0, sizeof(int64_t) * (n_slices + 1), s));
  SLA_CUDA_TRY(cudaMemsetAsync(wmax, 0, sizeof(int32_t), s));
  if (n_slices > 0)
    SLA_LAUNCH(sell_width_kernel, grid_for(n_slices * 32), kBlock, 0, s, rowptr, row_ids, n_slots,
               n_slices, min_width, len, wmax);
  SLA_TRY(exclusive_scan<int64_t>(len, ptr64, n_slices + 1, scan, s));
  int64_t total = 0;
  int32_t widest = 0;
  SLA_CUDA_TRY(cudaMemcpyAsync(&total, ptr64 + n_slices, sizeof(int64_t), cudaMemcpyDeviceToHost, s));
  SLA_CUDA_TRY(cudaMemcpyAsync(&widest, wmax, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
  SLA_CUDA_TRY(cudaStreamSynchronize(s));
  if (total >= INT32_MAX) return SLA_ERR_UNSUPPORTED;
  SLA_LAUNCH(rowptr_narrow_kernel, grid_for(n_slices + 1), kBlock, 0, s, ptr64, n_slices + 1,
             slice_ptr);
  *padded_out = total;
  if (max_width_out) *max_width_out = widest;
  return SLA_OK;
}

int sla_sell_fill(int dtype, const int32_t *rowptr, const int32_t *colind, const void *vals,
                  const int32_t *row_ids, int64_t n_slots, const int32_t *slice_ptr,
                  int32_t *sell_col, void *sell_val, sla_stream_t stream) {
  cudaStream_t s = (cudaStream_t)stream;
  if (!rowptr || !slice_ptr || n_slots < 0) return SLA_ERR_INVALID;
  int64_t n_slices = (n_slots + 31) / 32;
  if (n_slices == 0) return SLA_OK;
  if (dtype == SLA_F64)
    SLA_LAUNCH(sell_fill_kernel<double>, grid_for(n_slices * 32), kBlock, 0, s, rowptr, colind,
               (const double *)vals, row_ids, n_slots, n_slices, slice_ptr, sell_col,
               (double *)sell_val);
  else if (dtype == SLA_F32)
    SLA_LAUNCH(sell_fill_kernel<float>, grid_for(n_slices * 32), kBlock, 0, s, rowptr, colind,
               (const float *)vals, row_ids, n_slots, n_slices, slice_ptr, sell_col,
               (float *)sell_val);
  else
    return SLA_ERR_INVALID;
  return SLA_OK;
}

int sla_sell_sigma_order(const int32_t *rowptr, const int32_t *row_ids, int64_t n_slots,
                         int32_t sigma, int32_t *order, sla_stream_t stream) {
  if (!rowptr || !order || n_slots < 0 || n_slots >= INT32_MAX) return SLA_ERR_INVALID;
  if (sigma < 32 || sigma > kSigmaMax || (sigma & (sigma - 1))) return SLA_ERR_INVALID;
  if (n_slots == 0) return SLA_OK;
  const int64_t windows = (n_slots + sigma - 1) / sigma;
  const int threads = sigma < 1024 ? sigma : 1024;
  SLA_LAUNCH(sigma_order_kernel, (unsigned)windows, threads,
             (size_t)sigma * sizeof(unsigned long long), (cudaStream_t)stream, rowptr, row_ids,
             n_slots, (int)sigma, order);
  return SLA_OK;
}

int sla_jacobi_inverse(int dtype, const int32_t *rowptr, const int32_t *colind, const void *vals,
                       int64_t n_rows, int rule, void *dinv, sla_stream_t stream) {
  cudaStream_t s = (cudaStream_t)stream;
  if (!rowptr || !dinv || n_rows < 0 || rule < 0 || rule > 2) return SLA_ERR_INVALID;
  if (n_rows == 0) return SLA_OK;
  if (dtype == SLA_F64)
    SLA_LAUNCH(jacobi_kernel<double>, grid_for(n_rows), kBlock, 0, s, rowptr, colind,
               (const double *)vals, n_rows, rule, (double *)dinv);
  else if (dtype == SLA_F32)
    SLA_LAUNCH(jacobi_kernel<float>, grid_for(n_rows), kBlock, 0, s, rowptr, colind,
               (const float *)vals, n_rows, rule, (float *)dinv);
  else
    return SLA_ERR_INVALID;
  return SLA_OK;
}

int sla_sell_diag_probe_workspace(size_t *bytes) {
  if (!bytes) return SLA_ERR_INVALID;
  *bytes = align_up(kDiagTable * sizeof(int32_t)) + align_up(sizeof(int));
  return SLA_OK;
}

int sla_sell_diag_probe(const int32_t *rowptr, const int32_t *colind, const int32_t *row_ids,
                        int64_t n_slots, int32_t *offsets_out, int32_t *count_out,
                        void *workspace, size_t workspace_bytes, sla_stream_t stream) {
  if (!rowptr || !offsets_out || !count_out || n_slots < 0) return SLA_ERR_INVALID;
  size_t need = 0;
  sla_sell_diag_probe_workspace(&need);
  if (!workspace || workspace_bytes < need) return SLA_ERR_WORKSPACE;
  cudaStream_t s = (cudaStream_t)stream;
  Carver c(workspace, workspace_bytes);
  int32_t *gtab = c.take<int32_t>(kDiagTable);
  int *overflow = c.take<int>(1);
  if (!c.ok) return SLA_ERR_WORKSPACE;
  SLA_LAUNCH(diag_table_init_kernel, 1, kDiagTable, 0, s, gtab, overflow);
  if (n_slots > 0) {
    if (!colind) return SLA_ERR_INVALID;
    SLA_LAUNCH(diag_probe_kernel, grid_for(n_slots), kBlock, 0, s, rowptr, colind, row_ids,
               n_slots, gtab, overflow);
  }
  int32_t tab[kDiagTable];
  int of = 0;
  SLA_CUDA_TRY(cudaMemcpyAsync(tab, gtab, sizeof(tab), cudaMemcpyDeviceToHost, s));
  SLA_CUDA_TRY(cudaMemcpyAsync(&of, overflow, sizeof(int), cudaMemcpyDeviceToHost, s));
  SLA_CUDA_TRY(cudaStreamSynchronize(s));
  std::vector<int32_t> got;
  for (int i = 0; i < kDiagTable; ++i)
    if (tab[i] != kDiagEmpty) got.push_back(tab[i]);
  if (of || (int)got.size() > SLA_MAX_DIAGS) {
    *count_out = -1;
    return SLA_OK;
  }
  std::sort(got.begin(), got.end());
  for (size_t i = 0; i < got.size(); ++i) offsets_out[i] = got[i];
  *count_out = (int32_t)got.size();
  return SLA_OK;
}

int sla_sell_diag_fill(int dtype, const int32_t *rowptr, const int32_t *colind, const void *vals,
                       const int32_t *row_ids, int64_t n_slots, const int32_t *offsets,
                       int32_t n_diags, void *sell_val, void *workspace, size_t workspace_bytes,
                       sla_stream_t stream) {
  if (!rowptr || !offsets || n_slots < 0 || n_diags < 1 || n_diags > SLA_MAX_DIAGS)
    return SLA_ERR_INVALID;
  // the view's entries are addressed with int32 offsets
  if ((n_slots + 31) / 32 * 32 * (int64_t)n_diags > (int64_t)INT32_MAX) return SLA_ERR_UNSUPPORTED;
  size_t need = 0;
  sla_sell_diag_probe_workspace(&need);
  if (!workspace || workspace_bytes < need) return SLA_ERR_WORKSPACE;
  if (dtype != SLA_F32 && dtype != SLA_F64) return SLA_ERR_INVALID;
  DiagOffsets D;
  D.n = n_diags;
  for (int i = 0; i < SLA_MAX_DIAGS; ++i) D.off[i] = i < n_diags ? offsets[i] : INT32_MAX;
  for (int i = 1; i < n_diags; ++i)
    if (D.off[i] <= D.off[i - 1]) return SLA_ERR_INVALID;
  if (n_slots == 0) return SLA_OK;
  if (!colind || !vals || !sell_val) return SLA_ERR_INVALID;
  cudaStream_t s = (cudaStream_t)stream;
  const size_t elem = dtype == SLA_F64 ? 8 : 4;
  const int64_t padded = (n_slots + 31) / 32 * 32 * n_diags;
  SLA_CUDA_TRY(cudaMemsetAsync(sell_val, 0, elem * padded, s));
  int *bad = (int *)workspace;
  SLA_CUDA_TRY(cudaMemsetAsync(bad, 0, sizeof(int), s));
  if (dtype == SLA_F64)
    SLA_LAUNCH(diag_fill_kernel<double>, grid_for(n_slots), kBlock, 0, s, rowptr, colind,
               (const double *)vals, row_ids, n_slots, D, (double *)sell_val, bad);
  else
    SLA_LAUNCH(diag_fill_kernel<float>, grid_for(n_slots), kBlock, 0, s, rowptr, colind,
               (const float *)vals, row_ids, n_slots, D, (float *)sell_val, bad);
  int hb = 0;
  SLA_CUDA_TRY(cudaMemcpyAsync(&hb, bad, sizeof(int), cudaMemcpyDeviceToHost, s));
  SLA_CUDA_TRY(cudaStreamSynchronize(s));
  return hb ? SLA_ERR_INVALID : SLA_OK;
}

int sla_sell_diag_positions(const int32_t *rowptr, const int32_t *colind, int64_t n_rows,
                            const int32_t *offsets, int32_t n_diags, int64_t *pos,
                            void *workspace, size_t workspace_bytes, sla_stream_t stream) {
  if (!rowptr || !offsets || n_rows < 0 || n_diags < 1 || n_diags > SLA_MAX_DIAGS)
    return SLA_ERR_INVALID;
  size_t need = 0;
  sla_sell_diag_probe_workspace(&need);
  if (!workspace || workspace_bytes < need) return SLA_ERR_WORKSPACE;
  DiagOffsets D;
  D.n = n_diags;
  for (int i = 0; i < SLA_MAX_DIAGS; ++i) D.off[i] = i < n_diags ? offsets[i] : INT32_MAX;
  for (int i = 1; i < n_diags; ++i)
    if (D.off[i] <= D.off[i - 1]) return SLA_ERR_INVALID;
  if (n_rows == 0) return SLA_OK;
  if (!colind || !pos) return SLA_ERR_INVALID;
  cudaStream_t s = (cudaStream_t)stream;
  int *bad = (int *)workspace;
  SLA_CUDA_TRY(cudaMemsetAsync(bad, 0, sizeof(int), s));
  SLA_LAUNCH(diag_pos_kernel, grid_for(n_rows), kBlock, 0, s, rowptr, colind, n_rows, D, pos, bad);
  int hb = 0;
  SLA_CUDA_TRY(cudaMemcpyAsync(&hb, bad, sizeof(int), cudaMemcpyDeviceToHost, s));
  SLA_CUDA_TRY(cudaStreamSynchronize(s));
  return hb ? SLA_ERR_INVALID : SLA_OK;
}

}  // extern "C"
