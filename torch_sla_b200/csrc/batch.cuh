// Batch-interleaved reductions shared by the batched same-pattern CG and the
// multi-RHS CG: thread t of a block owns batch member t % B of row t / B.
#pragma once

#include "solver.cuh"

namespace sla {

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
