// SELL-32 row kernels shared by the SpMV-bearing solver kernels.
//
// One warp owns one 32-slot slice; lane l owns slot l. Entry j of a slot sits
// at slice_ptr[s] + 32*j + l, so the column/value loads of a warp are single
// 128 B / 256 B transactions and the padded tail costs one predicated lane.
// The gathered vector is produced by a functor so a solver can fuse the
// vector update that precedes the SpMV (p = z + beta p, p_hat = M^{-1} p,
// s_hat = M^{-1}(r - alpha v)) into the gather instead of a separate pass.
//
// Width specialisation (template parameter WS): the row loop is cheapest
// when its trip count is known at compile time, so kernels are instantiated
//   WS > 1000  diagonal-offset view of width WS - 1000 (5, 7, 27): columns
//              are row + off[j], no column array is read at all;
//   WS > 0     uniform layout, every slice WS entries wide (slice base is
//              32*WS*s, no slice_ptr load): the 7- and 27-point stencils;
//   WS < 0     at most -WS batches of kRowBatch entries (static batch loop);
//   WS == 0    any width (runtime loop).
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
  int32_t max_width;
  int32_t uniform_width;
  int64_t n_cols;
  int64_t row_base;
  int32_t n_diags;
  int32_t off[SLA_MAX_DIAGS];
};

// Matrix row of a slot: the row id list, or row_base + slot.
template <typename T>
__device__ __forceinline__ int64_t slot_row(const Sell<T> &A, int64_t slot) {
  return A.row_ids ? (int64_t)__ldg(A.row_ids + slot) : A.row_base + slot;
}

constexpr int kDiagSpec = 1000;  // WS = kDiagSpec + width: diagonal-offset view
constexpr int ws_width(int ws) { return ws > kDiagSpec ? ws - kDiagSpec : ws; }

template <typename T>
inline Sell<T> make_sell(const sla_sell_t *A) {
  Sell<T> s;
  s.n_slots = A ? A->n_slots : 0;
  s.n_slices = A ? A->n_slices : 0;
  s.slice_ptr = A ? A->slice_ptr : nullptr;
  s.col = A ? A->col : nullptr;
  s.val = A ? (const T *)A->val : nullptr;
  s.row_ids = A ? A->row_ids : nullptr;
  s.max_width = A ? A->max_width : 0;
  s.uniform_width = A ? A->uniform_width : 0;
  s.n_cols = A ? A->n_cols : 0;
  s.row_base = A ? A->row_base : 0;
  s.n_diags = A ? A->n_diags : 0;
  for (int i = 0; i < SLA_MAX_DIAGS; ++i) s.off[i] = A ? A->diag_offsets[i] : 0;
  return s;
}

inline bool diag_width_supported(int w) { return w == 5 || w == 7 || w == 27; }

// Entry offsets of a uniform-width view (diagonal-offset or uniform explicit)
// are computed in int32 as 32 * width * slice + 32 * entry + lane: the
// padded entry count must stay below 2^31. Non-uniform explicit views carry
// their offsets in int32 slice pointers, bounded when they were built.
inline bool sell_offsets_fit(const sla_sell_t *A) {
  const int64_t w = A->uniform_width > 0 ? A->uniform_width : A->n_diags;
  return w <= 0 || A->n_slices * 32 * w <= (int64_t)INT32_MAX;
}

inline bool sell_ok(const sla_sell_t *A) {
  if (!A) return false;
  if (A->n_slots < 0 || A->n_slices != (A->n_slots + 31) / 32) return false;
  if (A->max_width < 0 || A->uniform_width < 0) return false;
  if (A->uniform_width > 0 && A->uniform_width != A->max_width) return false;
  if (A->row_base < 0 || (A->row_ids && A->row_base != 0)) return false;
  if (A->row_base + A->n_slots > INT32_MAX) return false;
  if (A->n_diags > 0) {
    if (!diag_width_supported(A->n_diags) || A->uniform_width != A->n_diags) return false;
    if (A->n_slices > 0 && !A->val) return false;
    if (A->n_cols <= 0 || A->n_cols > INT32_MAX) return false;
    for (int i = 1; i < A->n_diags; ++i)
      if (A->diag_offsets[i] <= A->diag_offsets[i - 1]) return false;
    return true;
  }
  if (A->n_diags < 0) return false;
  if (A->n_slices > 0 && (!A->slice_ptr || !A->col || !A->val)) return false;
  return true;
}

// SLA_OK for a valid view, SLA_ERR_UNSUPPORTED when its int32 entry
// offsets would wrap, SLA_ERR_INVALID otherwise.
inline int sell_check(const sla_sell_t *A) {
  if (!A) return SLA_ERR_INVALID;
  if (A->n_slices >= 0 && !sell_offsets_fit(A)) return SLA_ERR_UNSUPPORTED;
  return sell_ok(A) ? SLA_OK : SLA_ERR_INVALID;
}

// Entries per load batch: a batch issues all its column/value loads, then all
// its gathers, so a row of up to kRowBatch entries costs one dependent
// load -> gather round trip (7-point rows fit one batch, 27-point rows four).
constexpr int kRowBatch = 8;

// Blocks per SM the SpMV-bearing kernels are compiled for (register cap):
// enough warps to keep ~8 batched loads each in flight.
#ifndef SLA_SPMV_MIN_BLOCKS
#define SLA_SPMV_MIN_BLOCKS 4
#endif
constexpr int kSpmvMinBlocks = SLA_SPMV_MIN_BLOCKS;

// CG search direction: formed by a streaming pass before a plain SpMV
// (SLA_CG_SPLIT 1), or inside the SpMV's gather, once per entry (0).
// Measured on 256^3 7-point fp64: fused K_A 284.5 us; split 265.7 us for
// both kernels (one more vector pass, but the SpMV streams at ~7 TB/s once
// its gathers are a single vector): 2400 -> 2535 it/s.
#ifndef SLA_CG_SPLIT
#define SLA_CG_SPLIT 1
#endif
constexpr bool kCgSplit = SLA_CG_SPLIT != 0;

// Grid of the SpMV kernels whose blocks also reduce a dot product: the
// resident blocks their launch bounds guarantee (kSpmvMinBlocks per SM),
// whatever registers an instantiation ends up with, so the summation order
// of the dot -- and with it every iterate -- is the same for every layout
// of a matrix.
inline int spmv_grid() { return kSpmvMinBlocks * device_info().sm_count; }


// Width spec of a view: the template value its kernels are launched with.
inline int width_spec(const sla_sell_t *A) {
  if (!A) return 0;
  if (A->n_diags > 0) return kDiagSpec + A->n_diags;
  if (A->uniform_width == 7 || A->uniform_width == 27) return A->uniform_width;
  const int w = A->max_width;
  if (w <= kRowBatch) return -1;
  if (w <= 2 * kRowBatch) return -2;
  if (w <= 4 * kRowBatch) return -4;
  return 0;
}

// Host dispatch: runs the statement(s) with WS bound to the view's spec.
#define SLA_WS_DISPATCH(ws, ...)                          \
  switch (ws) {                                           \
    case kDiagSpec + 5: { constexpr int WS = kDiagSpec + 5; __VA_ARGS__; } break; \
    case kDiagSpec + 7: { constexpr int WS = kDiagSpec + 7; __VA_ARGS__; } break; \
    case kDiagSpec + 27: { constexpr int WS = kDiagSpec + 27; __VA_ARGS__; } break; \
    case 7: { constexpr int WS = 7; __VA_ARGS__; } break;   \
    case 27: { constexpr int WS = 27; __VA_ARGS__; } break; \
    case -1: { constexpr int WS = -1; __VA_ARGS__; } break; \
    case -2: { constexpr int WS = -2; __VA_ARGS__; } break; \
    case -4: { constexpr int WS = -4; __VA_ARGS__; } break; \
    default: { constexpr int WS = 0; __VA_ARGS__; } break;  \
  }

template <typename T, typename G>
__device__ __forceinline__ void row_batch(const int32_t *__restrict__ cp, const T *__restrict__ vp,
                                          int j, int lim, const G &g, T &sum) {
  int32_t c[kRowBatch];
  T v[kRowBatch], x[kRowBatch];
#pragma unroll
  for (int u = 0; u < kRowBatch; ++u) {
    if (j + u < lim) {
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

// Diagonal-offset twin of row_batch: entry j of the slot is column
// row + off[j]; columns outside [0, n_cols) are skipped like padding, and
// entries the row does not use hold 0.
template <int W, typename T, typename G>
__device__ __forceinline__ void row_batch_diag(const Sell<T> &A, const T *__restrict__ vp,
                                               int64_t row, int j, const G &g, T &sum) {
  int32_t c[kRowBatch];
  T v[kRowBatch], x[kRowBatch];
#pragma unroll
  for (int u = 0; u < kRowBatch; ++u) {
    if (j + u < W) {
      const int64_t cc = row + A.off[j + u];
      c[u] = (cc >= 0 && cc < A.n_cols) ? (int32_t)cc : -1;
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

// sum_j val[j] * g(col[j]) over the entries of this lane's slot of slice s
// starting at entry `base` with `width` entries per slot (ascending j).
template <int WS, typename T, typename G>
__device__ __forceinline__ T sell_row_at(const Sell<T> &A, int64_t s, int32_t base, int width,
                                         int lane, const G &g) {
  const T *__restrict__ vp = A.val + base + lane;
  T sum = T(0);
  if constexpr (WS > kDiagSpec) {
    constexpr int W = WS - kDiagSpec;
    const int64_t slot = s * 32 + lane;
    const int64_t row = slot < A.n_slots ? slot_row(A, slot) : -((int64_t)1 << 40);
#pragma unroll
    for (int j = 0; j < W; j += kRowBatch) row_batch_diag<W>(A, vp, row, j, g, sum);
  } else if constexpr (WS > 0) {
    const int32_t *__restrict__ cp = A.col + base + lane;
#pragma unroll
    for (int j = 0; j < WS; j += kRowBatch) row_batch(cp, vp, j, WS, g, sum);
  } else if constexpr (WS < 0) {
    const int32_t *__restrict__ cp = A.col + base + lane;
#pragma unroll
    for (int jb = 0; jb < -WS; ++jb) row_batch(cp, vp, jb * kRowBatch, width, g, sum);
  } else {
    const int32_t *__restrict__ cp = A.col + base + lane;
    for (int j = 0; j < width; j += kRowBatch) row_batch(cp, vp, j, width, g, sum);
  }
  return sum;
}

// Grid-stride walk over the slices owned by this warp (slices warp,
// warp + nwarps, ...). Uniform layouts compute each slice's base; otherwise
// the slice pointers of the next 32 slices are fetched by the 32 lanes at once
// and broadcast by shuffles, so a slice's column and value loads never wait on
// a dependent slice_ptr load. body(slice, base, width) gets warp-uniform
// arguments.
//
// PF (uniform layouts): while a slice runs, prefetch into L2 the values of
// the warp's next slice (no registers held). Measured on the 256^3 7-point
// fp64 SpMV: 183 -> 171 us, where the streamed values are half the loads.
// Kernels that gather one stored vector (the plain SpMV, the CG SpMV over a
// formed search direction) turn it on; it gains nothing where each entry
// gathers three vectors (the fused CG K_A stayed at 285 us, BiCGStab K1
// went 147 -> 151 us).
template <int WS, bool PF = false, typename T, typename Body>
__device__ __forceinline__ void for_each_slice(const Sell<T> &A, int64_t warp, int64_t nwarps,
                                               int lane, Body body) {
  if constexpr (WS > 0) {
    constexpr int W = ws_width(WS);
    constexpr int kLines = 32 * W * (int)sizeof(T) / 128;  // 128-byte lines of a slice
    for (int64_t s = warp; s < A.n_slices; s += nwarps) {
      if (PF && s + nwarps < A.n_slices && lane < kLines)
        prefetch_l2(reinterpret_cast<const char *>(A.val + (s + nwarps) * 32 * W) + lane * 128);
      body(s, (int32_t)(s * 32 * W), W);
    }
  } else {
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
}

template <typename T>
struct PlainGather {
  const T *__restrict__ x;
  __device__ __forceinline__ T operator()(int32_t c) const { return __ldg(x + c); }
};

// ---------------------------------------------- float32, two rows per lane
// 4-byte values leave a one-row-per-lane warp with 128 B loads; here
// half-warp h of a warp takes slice 2 pr + h and lane l of the half its slots
// 2l and 2l + 1, whose entries j sit side by side in the SELL layout: one
// 8-byte load fetches both values (and both columns of an explicit view),
// 256 B per warp load as for fp64. Where the two gathered columns are
// adjacent and the first is even, one 8-byte load fetches both x values.
// Each row sums its entries in ascending j with the same FMAs as
// sell_row_at, so per-row results are unchanged; the row-to-thread mapping
// is the same for the diagonal-offset and the explicit 7-wide view of a
// matrix, so dot products reduced over it agree between the two views.
// x must be 8-byte aligned. Used for uniform views of at most eight
// entries per row (one load batch); the solver kernels take it for the
// 7-wide views only, whose diagonal-offset and explicit forms both qualify.
template <int WS>
constexpr bool kRowsX2 = WS > 0 && ws_width(WS) <= kRowBatch;
template <int WS>
constexpr bool kSolverRowsX2 = WS == kDiagSpec + 7 || WS == 7;

template <int WS>
__device__ __forceinline__ void sell_rows_x2(const Sell<float> &A, int64_t s, int hl,
                                             const float *__restrict__ x, int64_t &r0,
                                             int64_t &r1, float &s0, float &s1) {
  constexpr int W = ws_width(WS);
  const int64_t slot0 = s * 32 + 2 * hl;
  const bool ok0 = slot0 < A.n_slots, ok1 = slot0 + 1 < A.n_slots;
  const bool ids = A.row_ids != nullptr;
  const int64_t a0 = ids ? (ok0 ? (int64_t)__ldg(A.row_ids + slot0) : 0) : A.row_base + slot0;
  const int64_t a1 = ids ? (ok1 ? (int64_t)__ldg(A.row_ids + slot0 + 1) : 0) : a0 + 1;
  r0 = ok0 ? a0 : -1;
  r1 = ok1 ? a1 : -1;
  const int64_t e0 = s * 32 * W + 2 * hl;
  float2 v[W];
#pragma unroll
  for (int j = 0; j < W; ++j) v[j] = __ldcs(reinterpret_cast<const float2 *>(A.val + e0 + 32 * j));
  float x0[W], x1[W];
  if constexpr (WS > kDiagSpec) {
    if (!ids) {
      // consecutive rows: the two columns of entry j are adjacent. (The
      // parity test is per lane on purpose: the same test written on the
      // warp-uniform row_base + off[j] measured 123 us against 97 us for
      // the float32 SpMV at 256^3.)
#pragma unroll
      for (int j = 0; j < W; ++j) {
        const int64_t c0 = a0 + A.off[j], c1 = c0 + 1;
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
    } else {
#pragma unroll
      for (int j = 0; j < W; ++j) {
        const int64_t c0 = a0 + A.off[j], c1 = a1 + A.off[j];
        const bool in0 = ok0 && c0 >= 0 && c0 < A.n_cols;
        const bool in1 = ok1 && c1 >= 0 && c1 < A.n_cols;
        x0[j] = in0 ? __ldg(x + c0) : 0.f;
        x1[j] = in1 ? __ldg(x + c1) : 0.f;
      }
    }
  } else {
    int2 c[W];
#pragma unroll
    for (int j = 0; j < W; ++j) c[j] = __ldcs(reinterpret_cast<const int2 *>(A.col + e0 + 32 * j));
#pragma unroll
    for (int j = 0; j < W; ++j) {
      const int32_t c0 = ok0 ? c[j].x : -1, c1 = ok1 ? c[j].y : -1;
      if (c0 >= 0 && c1 == c0 + 1 && (c0 & 1) == 0) {
        const float2 xv = __ldg(reinterpret_cast<const float2 *>(x + c0));
        x0[j] = xv.x;
        x1[j] = xv.y;
      } else {
        x0[j] = c0 >= 0 ? __ldg(x + c0) : 0.f;
        x1[j] = c1 >= 0 ? __ldg(x + c1) : 0.f;
      }
    }
  }
  s0 = 0.f;
  s1 = 0.f;
#pragma unroll
  for (int j = 0; j < W; ++j) {
    s0 = fmaf(v[j].x, x0[j], s0);
    s1 = fmaf(v[j].y, x1[j], s1);
  }
}

// Walk of the slice pairs of a warp: body(s, hl) for the slice of this
// lane's half-warp, skipping a last odd slice's missing partner.
template <typename Body>
__device__ __forceinline__ void for_each_slice_x2(int64_t n_slices, int64_t warp, int64_t nwarps,
                                                  int lane, Body body) {
  const int h = lane >> 4, hl = lane & 15;
  const int64_t npairs = (n_slices + 1) >> 1;
  for (int64_t pr = warp; pr < npairs; pr += nwarps) {
    const int64_t s = 2 * pr + h;
    if (s < n_slices) body(s, hl);
  }
}

}  // namespace sla
