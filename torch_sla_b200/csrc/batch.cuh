// Batch-interleaved reductions shared by the batched same-pattern CG and the
// multi-RHS CG: thread t of a block owns batch member t % B of row t / B.
#pragma once

#include "solver.cuh"

namespace sla {

// sum_k val(k) * g(colind[k]) over the CSR entries [k0, k1), in load batches
// of kRowBatch (all column/value loads of a batch, then all its gathers), in
// ascending k order.
template <typename T, typename V, typename G>
__device__ __forceinline__ T csr_row_batched(const int32_t *__restrict__ colind, int32_t k0,
                                             int32_t k1, const V &val, const G &g) {
  T sum = T(0);
  for (int32_t kb = k0; kb < k1; kb += kRowBatch) {
    int32_t c[kRowBatch];
    T v[kRowBatch], x[kRowBatch];
#pragma unroll
    for (int u = 0; u < kRowBatch; ++u) {
      if (kb + u < k1) {
        c[u] = __ldg(colind + kb + u);
        v[u] = val(kb + u);
      } else {
        c[u] = -1;
        v[u] = T(0);
      }
    }
#pragma unroll
    for (int u = 0; u < kRowBatch; ++u) x[u] = c[u] >= 0 ? g(c[u]) : T(0);
#pragma unroll
    for (int u = 0; u < kRowBatch; ++u) sum = fma(v[u], x[u], sum);
  }
  return sum;
}

inline int batch_block(int64_t B) {
  if (B <= 256) return (int)(B * (256 / B));
  return (int)B;
}

// Per-member totals over all rows: thread tid<B ends with member tid's sum.
// acc is this thread's partial for member (threadIdx.x % B).
template <int NV>
__device__ bool batch_last_block(double (&acc)[NV], int B, double *smem, double *partials,
                                 unsigned *counter) {
  __shared__ unsigned s_last;
  const int TB = blockDim.x;
  const int rpb = TB / B;
  const unsigned G = gridDim.x;
#pragma unroll
  for (int k = 0; k < NV; ++k) smem[k * TB + threadIdx.x] = acc[k];
  __syncthreads();
  if (threadIdx.x < B) {
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      double t = 0.0;
      for (int q = 0; q < rpb; ++q) t += smem[k * TB + q * B + threadIdx.x];
      partials[((size_t)k * B + threadIdx.x) * G + blockIdx.x] = t;
    }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned t = atomicAdd(counter, 1u);
    s_last = (t == G - 1) ? 1u : 0u;
  }
  __syncthreads();
  if (!s_last) return false;
  __threadfence();
  if (threadIdx.x < B) {
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      double t = 0.0;
      const double *pp = partials + ((size_t)k * B + threadIdx.x) * G;
      for (unsigned g = 0; g < G; ++g) t += ld_l2(pp + g);
      acc[k] = t;
    }
  }
  if (threadIdx.x == 0) *counter = 0u;
  return true;
}

inline int batch_grid(int64_t n, int B) {
  int tb = batch_block(B);
  int rpb = tb / B;
  int64_t want = (n + rpb - 1) / rpb;
  int64_t cap = (int64_t)device_info().sm_count * (2048 / tb > 0 ? 2048 / tb : 1);
  return (int)(want < cap ? (want < 1 ? 1 : want) : cap);
}

}  // namespace sla
