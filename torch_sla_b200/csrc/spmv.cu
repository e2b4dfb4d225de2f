// Standalone SELL-32 SpMV, the adjoint's COO value gradient and the
// batched-value gather of the same-pattern solver.
#include <type_traits>

#include "sell.cuh"

namespace sla {

template <typename T, int WS>
__global__ void __launch_bounds__(kBlock, kSpmvMinBlocks) spmv_kernel(Sell<T> A, const T *__restrict__ x,
                                                      T *__restrict__ y) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  PlainGather<T> g{x};
  for_each_slice<WS, true>(A, warp, nwarps, lane, [&](int64_t s, int32_t sbase, int swidth) {
    T sum = sell_row_at<WS>(A, s, sbase, swidth, lane, g);
    int64_t slot = s * 32 + lane;
    if (slot < A.n_slots) {
      int64_t row = slot_row(A, slot);
      y[row] = sum;
    }
  });
}

// float32 SpMV on uniform views of at most eight entries per row, two rows
// per lane (sell_rows_x2): 8-byte value (and column) loads, paired aligned
// gathers. Same per-row sums as spmv_kernel. x and y 8-byte aligned.
template <int WS>
__global__ void __launch_bounds__(kBlock, kSpmvMinBlocks)
spmv_x2_kernel(Sell<float> A, const float *__restrict__ x, float *__restrict__ y) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for_each_slice_x2(A.n_slices, warp, nwarps, lane, [&](int64_t s, int hl) {
    int64_t r0, r1;
    float s0, s1;
    sell_rows_x2<WS>(A, s, hl, x, r0, r1, s0, s1);
    if (r0 >= 0 && r1 == r0 + 1 && (r0 & 1) == 0) {
      *reinterpret_cast<float2 *>(y + r0) = make_float2(s0, s1);
    } else {
      if (r0 >= 0) y[r0] = s0;
      if (r1 >= 0) y[r1] = s1;
    }
  });
}

// y[r] for the CSR rows listed in `rows`, one warp per row: lane l takes the
// row's entries l, l + 32, l + 64, ... in ascending order (four in flight per
// lane), then a fixed butterfly adds the 32 lane sums. The long rows of a
// hybrid SpMV: a row walked by one lane of a SELL slice would keep that warp
// busy long after the others finished.
template <typename T>
__global__ void __launch_bounds__(kBlock)
spmv_rows_csr_kernel(const int32_t *__restrict__ rowptr, const int32_t *__restrict__ colind,
                     const T *__restrict__ vals, const int32_t *__restrict__ rows, int64_t n_rows,
                     const T *__restrict__ x, T *__restrict__ y) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t i = warp; i < n_rows; i += nwarps) {
    const int32_t r = __ldg(rows + i);
    const int32_t k1 = __ldg(rowptr + r + 1);
    int32_t k = __ldg(rowptr + r) + lane;
    T acc = T(0);
    for (; k + 96 < k1; k += 128) {
      int32_t c[4];
      T v[4], xv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        c[u] = ld_stream(colind + k + 32 * u);
        v[u] = ld_stream(vals + k + 32 * u);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) xv[u] = __ldg(x + c[u]);
#pragma unroll
      for (int u = 0; u < 4; ++u) acc = fma(v[u], xv[u], acc);
    }
    for (; k < k1; k += 32) acc = fma(ld_stream(vals + k), __ldg(x + ld_stream(colind + k)), acc);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(kFull, acc, o);
    if (lane == 0) y[r] = acc;
  }
}

template <typename T>
int spmv_launch(const sla_sell_t *A, const void *x, void *y, cudaStream_t s) {
  Sell<T> a = make_sell<T>(A);
  if (a.n_slices == 0) return SLA_OK;
  // one wave of resident blocks, never more blocks than warps have slices
  // (slice pairs for the two-rows-per-lane kernel)
  if constexpr (std::is_same_v<T, float>) {
    // float32 views of at most eight entries per row: two rows per lane
    if (aligned8(x, y)) {
      bool done = false;
      SLA_WS_DISPATCH(width_spec(A), {
        if constexpr (kRowsX2<WS>) {
          const int g = occupancy_grid((const void *)spmv_x2_kernel<WS>);
          const int64_t want = ((a.n_slices + 1) / 2 + kWarps - 1) / kWarps;
          SLA_LAUNCH(spmv_x2_kernel<WS>, want < g ? (int)want : g, kBlock, 0, s, a,
                     (const float *)x, (float *)y);
          done = true;
        }
      });
      if (done) return SLA_OK;
    }
  }
  SLA_WS_DISPATCH(width_spec(A), {
    const int g = occupancy_grid((const void *)spmv_kernel<T, WS>);
    const int64_t want = (a.n_slices + kWarps - 1) / kWarps;
    SLA_LAUNCH((spmv_kernel<T, WS>), want < g ? (int)want : g, kBlock, 0, s, a, (const T *)x,
               (T *)y);
  });
  return SLA_OK;
}
template int spmv_launch<float>(const sla_sell_t *, const void *, void *, cudaStream_t);
template int spmv_launch<double>(const sla_sell_t *, const void *, void *, cudaStream_t);

template <typename T>
__global__ void coo_value_grad_kernel(const int64_t *__restrict__ row, const int64_t *__restrict__ col,
                                      int64_t nnz, const T *__restrict__ a, const T *__restrict__ b,
                                      int64_t n_a, int64_t n_b, int64_t K, int64_t batch,
                                      T *__restrict__ g) {
  int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; t < nnz * batch; t += stride) {
    int64_t bi = t / nnz, k = t - bi * nnz;
    const T *ab = a + bi * n_a * K + row[k] * K;
    const T *bb = b + bi * n_b * K + col[k] * K;
    T acc = mul_rn(-ab[0], bb[0]);
    for (int64_t c = 1; c < K; ++c) acc = add_rn(acc, mul_rn(-ab[c], bb[c]));
    g[t] = acc;
  }
}

// Per-member values gathered from the COO batch: out[(pos ? pos[e] : e) * batch + b]
// = sum of the COO duplicates of CSR entry e (in input order) of member b.
template <typename T>
__global__ void batched_values_kernel(const T *__restrict__ vb, int64_t batch, int64_t nnz_coo,
                                      const int64_t *__restrict__ src, const int32_t *__restrict__ seg,
                                      int64_t nnz_csr, const int64_t *__restrict__ pos,
                                      T *__restrict__ out) {
  int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; t < nnz_csr * batch; t += stride) {
    int64_t e = t / batch, bi = t - e * batch;
    const T *v = vb + bi * nnz_coo;
    int32_t s0 = seg[e], s1 = seg[e + 1];
    T acc = v[src[s0]];
    for (int32_t q = s0 + 1; q < s1; ++q) acc = add_rn(acc, v[src[q]]);
    out[(pos ? pos[e] : e) * batch + bi] = acc;
  }
}

}  // namespace sla

using namespace sla;

extern "C" {

int sla_spmv_rows_csr(int dtype, const int32_t *rowptr, const int32_t *colind, const void *vals,
                      const int32_t *rows, int64_t n_rows, const void *x, void *y,
                      sla_stream_t stream) {
  if (n_rows < 0 || (n_rows > 0 && (!rowptr || !colind || !vals || !rows || !x || !y)))
    return SLA_ERR_INVALID;
  if (dtype != SLA_F32 && dtype != SLA_F64) return SLA_ERR_INVALID;
  if (n_rows == 0) return SLA_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t want = (n_rows + kWarps - 1) / kWarps;
  if (dtype == SLA_F64) {
    const int g = occupancy_grid((const void *)spmv_rows_csr_kernel<double>);
    SLA_LAUNCH(spmv_rows_csr_kernel<double>, want < g ? (int)want : g, kBlock, 0, s, rowptr,
               colind, (const double *)vals, rows, n_rows, (const double *)x, (double *)y);
  } else {
    const int g = occupancy_grid((const void *)spmv_rows_csr_kernel<float>);
    SLA_LAUNCH(spmv_rows_csr_kernel<float>, want < g ? (int)want : g, kBlock, 0, s, rowptr,
               colind, (const float *)vals, rows, n_rows, (const float *)x, (float *)y);
  }
  return SLA_OK;
}

int sla_spmv(int dtype, const sla_sell_t *A, const void *x, void *y, sla_stream_t stream) {
  SLA_TRY(sell_check(A));
  if (A->n_slots > 0 && (!x || !y)) return SLA_ERR_INVALID;
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == SLA_F64) return spmv_launch<double>(A, x, y, s);
  if (dtype == SLA_F32) return spmv_launch<float>(A, x, y, s);
  return SLA_ERR_INVALID;
}

int sla_coo_value_grad(int dtype, const int64_t *row, const int64_t *col, int64_t nnz,
                       const void *a, const void *b, int64_t n_a, int64_t n_b, int64_t K,
                       int64_t batch, void *g, sla_stream_t stream) {
  if (nnz < 0 || K < 1 || batch < 1 || n_a < 1 || n_b < 1) return SLA_ERR_INVALID;
  if (nnz == 0) return SLA_OK;
  if (!row || !col || !a || !b || !g) return SLA_ERR_INVALID;
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == SLA_F64)
    SLA_LAUNCH(coo_value_grad_kernel<double>, grid_for(nnz * batch), kBlock, 0, s, row, col, nnz,
               (const double *)a, (const double *)b, n_a, n_b, K, batch, (double *)g);
  else if (dtype == SLA_F32)
    SLA_LAUNCH(coo_value_grad_kernel<float>, grid_for(nnz * batch), kBlock, 0, s, row, col, nnz,
               (const float *)a, (const float *)b, n_a, n_b, K, batch, (float *)g);
  else
    return SLA_ERR_INVALID;
  return SLA_OK;
}

int sla_batched_values(int dtype, const void *val_batch, int64_t batch, int64_t nnz_coo,
                       const int64_t *src_index, const int32_t *seg_ptr, int64_t nnz_csr,
                       void *out, sla_stream_t stream) {
  if (batch < 1 || nnz_coo < 0 || nnz_csr < 0) return SLA_ERR_INVALID;
  if (nnz_csr == 0) return SLA_OK;
  if (!val_batch || !src_index || !seg_ptr || !out) return SLA_ERR_INVALID;
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == SLA_F64)
    SLA_LAUNCH(batched_values_kernel<double>, grid_for(nnz_csr * batch), kBlock, 0, s,
               (const double *)val_batch, batch, nnz_coo, src_index, seg_ptr, nnz_csr,
               (const int64_t *)nullptr, (double *)out);
  else if (dtype == SLA_F32)
    SLA_LAUNCH(batched_values_kernel<float>, grid_for(nnz_csr * batch), kBlock, 0, s,
               (const float *)val_batch, batch, nnz_coo, src_index, seg_ptr, nnz_csr,
               (const int64_t *)nullptr, (float *)out);
  else
    return SLA_ERR_INVALID;
  return SLA_OK;
}

int sla_batched_values_at(int dtype, const void *val_batch, int64_t batch, int64_t nnz_coo,
                          const int64_t *src_index, const int32_t *seg_ptr, int64_t nnz_csr,
                          const int64_t *pos, int64_t n_out, void *out, sla_stream_t stream) {
  if (batch < 1 || nnz_coo < 0 || nnz_csr < 0 || n_out < 0 || !pos || !out)
    return SLA_ERR_INVALID;
  if (dtype != SLA_F32 && dtype != SLA_F64) return SLA_ERR_INVALID;
  cudaStream_t s = (cudaStream_t)stream;
  const size_t elem = dtype == SLA_F64 ? 8 : 4;
  SLA_CUDA_TRY(cudaMemsetAsync(out, 0, elem * (size_t)n_out * (size_t)batch, s));
  if (nnz_csr == 0) return SLA_OK;
  if (!val_batch || !src_index || !seg_ptr) return SLA_ERR_INVALID;
  if (dtype == SLA_F64)
    SLA_LAUNCH(batched_values_kernel<double>, grid_for(nnz_csr * batch), kBlock, 0, s,
               (const double *)val_batch, batch, nnz_coo, src_index, seg_ptr, nnz_csr, pos,
               (double *)out);
  else
    SLA_LAUNCH(batched_values_kernel<float>, grid_for(nnz_csr * batch), kBlock, 0, s,
               (const float *)val_batch, batch, nnz_coo, src_index, seg_ptr, nnz_csr, pos,
               (float *)out);
  return SLA_OK;
}

}  // extern "C"
