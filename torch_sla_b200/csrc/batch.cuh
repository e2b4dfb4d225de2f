// Batch-interleaved kernels shared by the batched same-pattern CG and the
// multi-RHS CG.
//
// Vectors are [n][B] (member fastest). The B members of a row are covered by
// TR = B / VEC threads, each owning VEC consecutive members and moving them
// with one vector load/store (16 bytes for fp64 pairs and fp32 quads). A
// block of TR * RPB threads covers RPB rows per step of its grid-stride loop.
// Per-member dot products are reduced in a fixed order (rows of the block,
// then blocks), so repeated solves are bitwise identical.
#pragma once

#include "solver.cuh"

namespace sla {

// Threads per block of the vectorised batch kernels (VEC > 1); the scalar
// kernels use up to 1024 so that one block can hold a whole row of B <= 1024.
constexpr int kBatchThreads = 512;

// Load batch (entries per dependent round trip) of the vectorised row walk
// and the resident blocks per SM the vectorised kernels are compiled for.
// Measured on 64 x 512^2 5-point fp64 (iteration bytes vs. HBM copy peak):
// 3 entries 90.8 %, 2: 88.9 %, 4: 87.8 %, 5: 87.8 % at two 512-thread
// blocks per SM (64 registers); 4 entries at one block per SM: 68.4 %, and
// 8 entries (106 registers, one block per SM): 69.0 %. Occupancy -- gathers
// of 32 warps per SM in flight instead of 16 -- is what counts.
#ifndef SLA_BATCH_RB
#define SLA_BATCH_RB 3
#endif
#ifndef SLA_BATCH_MINB
#define SLA_BATCH_MINB 2
#endif
constexpr int kBatchRB = SLA_BATCH_RB;
constexpr int kBatchMinBlocks = SLA_BATCH_MINB;

template <typename T, int VEC> struct VecType;
template <> struct VecType<double, 1> { using type = double; };
template <> struct VecType<double, 2> { using type = double2; };
template <> struct VecType<float, 1> { using type = float; };
template <> struct VecType<float, 2> { using type = float2; };
template <> struct VecType<float, 4> { using type = float4; };

template <typename T, int VEC>
struct Pack {
  T v[VEC];
};

enum LoadMode { kLoadPlain = 0, kLoadRO = 1, kLoadStream = 2 };

template <typename T, int VEC, int MODE = kLoadPlain>
__device__ __forceinline__ Pack<T, VEC> vload(const T *p) {
  using V = typename VecType<T, VEC>::type;
  const V *q = reinterpret_cast<const V *>(p);
  V raw;
  if (MODE == kLoadRO) raw = __ldg(q);
  else if (MODE == kLoadStream) raw = __ldcs(q);
  else raw = *q;
  Pack<T, VEC> out;
  const T *e = reinterpret_cast<const T *>(&raw);
#pragma unroll
  for (int u = 0; u < VEC; ++u) out.v[u] = e[u];
  return out;
}

template <typename T, int VEC>
__device__ __forceinline__ void vstore(T *p, const Pack<T, VEC> &x) {
  using V = typename VecType<T, VEC>::type;
  V raw;
  T *e = reinterpret_cast<T *>(&raw);
#pragma unroll
  for (int u = 0; u < VEC; ++u) e[u] = x.v[u];
  *reinterpret_cast<V *>(p) = raw;
}

template <typename T, int VEC>
__device__ __forceinline__ Pack<T, VEC> splat(T x) {
  Pack<T, VEC> out;
#pragma unroll
  for (int u = 0; u < VEC; ++u) out.v[u] = x;
  return out;
}

// Position of this thread in the batch layout.
struct BatchLane {
  int tr;    // threads per row
  int rpb;   // rows per block step
  int m0;    // first member owned
  int rl;    // row lane inside the block step
  __device__ __forceinline__ BatchLane(int B, int vec) {
    tr = B / vec;
    rpb = blockDim.x / tr;
    m0 = (threadIdx.x % tr) * vec;
    rl = threadIdx.x / tr;
  }
};

// sum[u] = sum_k val(k)[u] * g(colind[k])[u] over the CSR entries [k0, k1),
// in load batches of RB (all column/value loads of a batch, then all its
// gathers), in ascending k order for every member.
template <typename T, int VEC, int RB, typename V, typename G>
__device__ __forceinline__ void csr_row_vec(const int32_t *__restrict__ colind, int32_t k0,
                                            int32_t k1, const V &val, const G &g,
                                            T (&sum)[VEC]) {
#pragma unroll
  for (int u = 0; u < VEC; ++u) sum[u] = T(0);
  for (int32_t kb = k0; kb < k1; kb += RB) {
    int32_t c[RB];
    Pack<T, VEC> v[RB], x[RB];
#pragma unroll
    for (int q = 0; q < RB; ++q) {
      if (kb + q < k1) {
        c[q] = __ldg(colind + kb + q);
        v[q] = val(kb + q);
      } else {
        c[q] = -1;
        v[q] = splat<T, VEC>(T(0));
      }
    }
#pragma unroll
    for (int q = 0; q < RB; ++q) x[q] = c[q] >= 0 ? g(c[q]) : splat<T, VEC>(T(0));
#pragma unroll
    for (int q = 0; q < RB; ++q) {
#pragma unroll
      for (int u = 0; u < VEC; ++u) sum[u] = fma(v[q].v[u], x[q].v[u], sum[u]);
    }
  }
}

// Block size of the batch kernels for B members in VEC-wide groups.
inline int batch_block(int64_t B, int vec) {
  const int tr = (int)(B / vec);
  const int cap = vec == 1 ? 1024 : kBatchThreads;
  int rpb = (vec == 1 ? kBatchThreads : cap) / tr;
  if (rpb < 1) rpb = 1;
  if (tr * rpb > cap) rpb = cap / tr;
  return tr * rpb;
}

// Dynamic shared memory of batch_reduce<NV, VEC> at block size tb.
inline size_t batch_smem(int nv, int tb, int vec) { return (size_t)nv * tb * vec * sizeof(double); }

// Upper bound of any batch kernel's grid (sizes the partial buffers).
inline int batch_max_grid() { return solver_grid(); }

// Per-member grid totals of NV quantities.
//
// acc[k][u] is this thread's partial of quantity k for member m0 + u. Every
// block writes its per-member totals to partials ([grid][NV][B], coalesced);
// the last block to finish sums them with all its threads (thread groups
// stride over the blocks, then the groups are added in order) and returns
// true with the totals in smem[k * B + m], all threads synchronised.
// smem: NV * blockDim.x * VEC doubles (dynamic shared memory).
template <int NV, int VEC>
__device__ bool batch_reduce(double (&acc)[NV][VEC], int B, double *smem, double *partials,
                             unsigned *counter) {
  __shared__ unsigned s_last;
  const BatchLane ln(B, VEC);
  const int TB = blockDim.x;
  const unsigned G = gridDim.x;
  const int P = NV * B;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
#pragma unroll
    for (int u = 0; u < VEC; ++u) smem[(k * ln.rpb + ln.rl) * B + ln.m0 + u] = acc[k][u];
  }
  __syncthreads();
  for (int q = threadIdx.x; q < P; q += TB) {
    const int k = q / B, m = q - k * B;
    double t = 0.0;
    for (int j = 0; j < ln.rpb; ++j) t += smem[(k * ln.rpb + j) * B + m];
    partials[(size_t)blockIdx.x * P + q] = t;
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned t = atomicAdd(counter, 1u);
    s_last = (t == G - 1) ? 1u : 0u;
  }
  __syncthreads();
  if (!s_last) return false;
  __threadfence();
  const int groups = TB >= P ? TB / P : 1;
  for (int idx = threadIdx.x; idx < groups * P; idx += TB) {
    const int q = idx % P, j = idx / P;
    double t = 0.0;
#pragma unroll 4
    for (unsigned g = j; g < G; g += groups) t += ld_l2(partials + (size_t)g * P + q);
    smem[j * P + q] = t;
  }
  __syncthreads();
  for (int q = threadIdx.x; q < P; q += TB) {
    double t = smem[q];
    for (int j = 1; j < groups; ++j) t += smem[j * P + q];
    smem[q] = t;
  }
  __syncthreads();
  if (threadIdx.x == 0) *counter = 0u;
  return true;
}

}  // namespace sla
