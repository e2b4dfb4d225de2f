// SELL-32 row kernels shared by the SpMV-bearing solver kernels.
//
// One warp owns one 32-slot slice; lane l owns slot l. Entry j of a slot sits
// at slice_ptr[s] + 32*j + l, so the column/value loads of a warp are single
// 128 B / 256 B transactions and the padded tail costs one predicated lane.
// The gathered vector is produced by a functor so a solver can fuse the
// vector update that precedes the SpMV (p = z + beta p, p_hat = M^{-1} p,
// s_hat = M^{-1}(r - alpha v)) into the gather instead of a separate pass.
#pragma once

#include "common.cuh"

namespace sla {

template <typename T>
struct Sell {
  int64_t n_slots;
  int64_t n_slices;
  const int32_t *__restrict__ slice_ptr;
  const int32_t *__restrict__ col;
  const T *__restrict__ val;
  const int32_t *__restrict__ row_ids;
};

template <typename T>
inline Sell<T> make_sell(const sla_sell_t *A) {
  Sell<T> s;
  s.n_slots = A ? A->n_slots : 0;
  s.n_slices = A ? A->n_slices : 0;
  s.slice_ptr = A ? A->slice_ptr : nullptr;
  s.col = A ? A->col : nullptr;
  s.val = A ? (const T *)A->val : nullptr;
  s.row_ids = A ? A->row_ids : nullptr;
  return s;
}

inline bool sell_ok(const sla_sell_t *A) {
  if (!A) return false;
  if (A->n_slots < 0 || A->n_slices != (A->n_slots + 31) / 32) return false;
  if (A->n_slices > 0 && (!A->slice_ptr || !A->col || !A->val)) return false;
  return true;
}

// Entries per load batch: a batch issues all its column/value loads, then all
// its gathers, so a row of up to kRowBatch entries costs one dependent
// load -> gather round trip (7-point rows fit one batch, 27-point rows four).
constexpr int kRowBatch = 8;

// sum_j val[j] * g(col[j]) over the entries of this lane's slot of the slice
// starting at entry `base` with `width` entries per slot.
template <typename T, typename G>
__device__ __forceinline__ T sell_row_at(const Sell<T> &A, int32_t base, int width, int lane,
                                         const G &g) {
  const int32_t *__restrict__ cp = A.col + base + lane;
  const T *__restrict__ vp = A.val + base + lane;
  T sum = T(0);
  for (int j = 0; j < width; j += kRowBatch) {
    int32_t c[kRowBatch];
    T v[kRowBatch], x[kRowBatch];
#pragma unroll
    for (int u = 0; u < kRowBatch; ++u) {
      if (j + u < width) {
        c[u] = ld_stream(cp + 32 * (j + u));
        v[u] = ld_stream(vp + 32 * (j + u));
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

template <typename T, typename G>
__device__ __forceinline__ T sell_row(const Sell<T> &A, int64_t slice, int lane, const G &g) {
  const int32_t base = A.slice_ptr[slice];
  return sell_row_at(A, base, (A.slice_ptr[slice + 1] - base) >> 5, lane, g);
}

// Grid-stride walk over the slices owned by this warp (slices warp,
// warp + nwarps, ...). The slice pointers of the next 32 slices are fetched
// by the 32 lanes at once and broadcast by shuffles, so a slice's column and
// value loads never wait on a dependent slice_ptr load.
// body(slice, base, width) is called with warp-uniform arguments.
template <typename T, typename Body>
__device__ __forceinline__ void for_each_slice(const Sell<T> &A, int64_t warp, int64_t nwarps,
                                               int lane, Body body) {
  for (int64_t s0 = warp; s0 < A.n_slices; s0 += 32 * nwarps) {
    const int64_t mine = s0 + (int64_t)lane * nwarps;
    int32_t b0 = 0, b1 = 0;
    if (mine < A.n_slices) {
      b0 = __ldg(A.slice_ptr + mine);
      b1 = __ldg(A.slice_ptr + mine + 1);
    }
    const int64_t left = (A.n_slices - s0 + nwarps - 1) / nwarps;
    const int count = left < 32 ? (int)left : 32;
    for (int q = 0; q < count; ++q) {
      const int32_t base = __shfl_sync(kFull, b0, q);
      const int32_t end = __shfl_sync(kFull, b1, q);
      body(s0 + (int64_t)q * nwarps, base, (end - base) >> 5);
    }
  }
}

// Blocks per SM the SpMV-bearing kernels are compiled for (register cap):
// enough warps to keep ~8 batched loads each in flight.
constexpr int kSpmvMinBlocks = 4;

template <typename T>
struct PlainGather {
  const T *__restrict__ x;
  __device__ __forceinline__ T operator()(int32_t c) const { return __ldg(x + c); }
};

}  // namespace sla
