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

// float32 diagonal-offset SpMV, two rows per lane: half-warp h of a warp
// takes slice 2 pr + h, and lane l of the half rows 2l and 2l + 1 of it. The
// two rows' values of entry j are adjacent, so one 8-byte load fetches both
// (256 B per warp load, the width of an fp64 view's loads, where the
// one-row-per-lane kernel issues 128 B loads); where row + off[j] is even
// the two gathered x values are adjacent and 8-byte aligned as well (one
// load), otherwise they are gathered separately. Each row still sums its W
// entries in ascending j with the same FMAs, so y equals spmv_kernel's.
// Views without row ids; x and y 8-byte aligned.
template <int W>
__global__ void __launch_bounds__(kBlock, kSpmvMinBlocks)
spmv_diag_f32x2_kernel(Sell<float> A, const float *__restrict__ x, float *__restrict__ y) {
  const int lane = threadIdx.x & 31;
  const int h = lane >> 4, hl = lane & 15;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t npairs = (A.n_slices + 1) >> 1;
  for (int64_t pr = warp; pr < npairs; pr += nwarps) {
    const int64_t s = 2 * pr + h;
    if (s >= A.n_slices) continue;
    const int64_t slot0 = s * 32 + 2 * hl;
    const bool ok0 = slot0 < A.n_slots, ok1 = slot0 + 1 < A.n_slots;
    const int64_t r0 = A.row_base + slot0;
    const float *__restrict__ vp = A.val + s * 32 * W + 2 * hl;
    float2 v[W];
#pragma unroll
    for (int j = 0; j < W; ++j) v[j] = __ldcs(reinterpret_cast<const float2 *>(vp + 32 * j));
    float x0[W], x1[W];
#pragma unroll
    for (int j = 0; j < W; ++j) {
      const int64_t c0 = r0 + A.off[j], c1 = c0 + 1;
      const bool in0 = ok0 && c0 >= 0 && c0 < A.n_cols;
      const bool in1 = ok1 && c1 >= 0 && c1 < A.n_cols;
      if (in0 && in1 && (c0 & 1) == 0) {
        const float2 xv = __ldg(reinterpret_cast<const float2 *>(x + c0));
        x0[j] = xv.x;
        x1[j] = xv.y;
      } else {
        x0[j] = in0 ? __ldg(x + c0) : 0.f;
        x1[j] = in1 ? __ldg(x + c1) : 0.f;
      }
    }
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int j = 0; j < W; ++j) {
      s0 = fmaf(v[j].x, x0[j], s0);
      s1 = fmaf(v[j].y, x1[j], s1);
    }
    if (ok0 && ok1 && (r0 & 1) == 0) {
      *reinterpret_cast<float2 *>(y + r0) = make_float2(s0, s1);
    } else {
      if (ok0) y[r0] = s0;
      if (ok1) y[r0 + 1] = s1;
    }
  }
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
  // one wave of resident blocks (fp32 views fit five 256-thread blocks per
  // SM), never more blocks than warps have slices
  if constexpr (std::is_same_v<T, float>) {
    // float32 diagonal views of 5 or 7 diagonals: two rows per lane
    if (a.n_diags == 5 || a.n_diags == 7) {
      if (!a.row_ids && aligned8(x, y)) {
        const int64_t want = ((a.n_slices + 1) / 2 + kWarps - 1) / kWarps;
        if (a.n_diags == 7) {
          const int g = occupancy_grid((const void *)spmv_diag_f32x2_kernel<7>);
          SLA_LAUNCH(spmv_diag_f32x2_kernel<7>, want < g ? (int)want : g, kBlock, 0, s, a,
                     (const float *)x, (float *)y);
        } else {
          const int g = occupancy_grid((const void *)spmv_diag_f32x2_kernel<5>);
          SLA_LAUNCH(spmv_diag_f32x2_kernel<5>, want < g ? (int)want : g, kBlock, 0, s, a,
                     (const float *)x, (float *)y);
        }
        return SLA_OK;
      }
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
