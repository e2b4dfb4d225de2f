// Multi-RHS CG: A X = B for K right-hand sides of one matrix
// (batched_pcg_solve, backends/pytorch_backend.py:2352-2504, reached through
// pytorch_solve with a 2-D b).
//
// X, B and every work vector are [n][K] row-major -- the layout of a 2-D b --
// so thread t of a block owns column t % K of row t / K, one column index
// and one matrix value serve the K lanes of a row, and the lanes read
// contiguous memory. Control flow of the reference: per-column alpha with
// (p,Ap) <= 0 replaced by 1, beta = rz_new / (rz_old + 1e-30), convergence
// tested every `check_every` iterations after the X/R update, columns keep
// iterating until all have converged.
#include "batch.cuh"

namespace sla {

struct MrhsState {
  long long iter, maxiter, iters_out;
  long long check_every;
  int done;  // 0 running, 1 all converged, 2 maxiter
  int pad;
  unsigned counter[4];
};

struct MrhsCols {
  double *rz, *alpha, *beta, *tol_sq, *rr, *alpha_prev;
  long long *iters;   // per column, 0 until converged
  int *conv;          // per column convergence flag
};

// Row access of the multi-RHS kernels: int32 CSR, or a diagonal-offset SELL
// view of a stencil matrix (column = row + offset: no column or row-pointer
// loads, so every load of a row is independent of the others).
template <typename T>
struct CsrRows {
  static constexpr int kWidth = 0;
  const int32_t *rowptr, *colind;
  const T *vals;
  template <int VEC, int RB, typename G>
  __device__ __forceinline__ void sum(int64_t row, const G &g, T (&s)[VEC]) const {
    csr_row_vec<T, VEC, RB>(
        colind, __ldg(rowptr + row), __ldg(rowptr + row + 1),
        [&](int32_t k) { return splat<T, VEC>(__ldg(vals + k)); }, g, s);
  }
  template <typename G>
  __device__ __forceinline__ T sum1(int64_t row, const G &g) const {
    T ax = T(0);
    for (int32_t k = rowptr[row]; k < rowptr[row + 1]; ++k) ax = fma(vals[k], g(colind[k]), ax);
    return ax;
  }
};

template <typename T, int W>
struct DiagRows {
  static constexpr int kWidth = W;
  Sell<T> A;
  template <int VEC, int RB, typename G>
  __device__ __forceinline__ void sum(int64_t row, const G &g, T (&s)[VEC]) const {
#pragma unroll
    for (int u = 0; u < VEC; ++u) s[u] = T(0);
    const T *__restrict__ vp = A.val + (row >> 5) * 32 * W + (row & 31);
#pragma unroll
    for (int j0 = 0; j0 < W; j0 += RB) {
      T v[RB];
      Pack<T, VEC> x[RB];
#pragma unroll
      for (int q = 0; q < RB; ++q) {
        v[q] = T(0);
        x[q] = splat<T, VEC>(T(0));
        if (j0 + q < W) {
          const int64_t c = row + A.off[j0 + q];
          v[q] = __ldg(vp + 32 * (j0 + q));
          if (c >= 0 && c < A.n_cols) x[q] = g((int32_t)c);
        }
      }
#pragma unroll
      for (int q = 0; q < RB; ++q) {
#pragma unroll
        for (int u = 0; u < VEC; ++u) s[u] = fma(v[q], x[q].v[u], s[u]);
      }
    }
  }
  template <typename G>
  __device__ __forceinline__ T sum1(int64_t row, const G &g) const {
    T ax = T(0);
    const T *__restrict__ vp = A.val + (row >> 5) * 32 * W + (row & 31);
#pragma unroll
    for (int j = 0; j < W; ++j) {
      const int64_t c = row + A.off[j];
      if (c >= 0 && c < A.n_cols) ax = fma(__ldg(vp + 32 * j), g((int32_t)c), ax);
    }
    return ax;
  }
};

template <typename T, bool PREC, typename M>
__global__ void __launch_bounds__(1024)
mrhs_init_kernel(M mat, int64_t n, int K, const T *__restrict__ b,
                 T *__restrict__ x, int guess, const T *__restrict__ dinv, T *__restrict__ r,
                 T *__restrict__ p_old, MrhsState *st, MrhsCols cs, double *partials,
                 double atol, double rtol) {
  extern __shared__ double smem[];
  const BatchLane ln(K, 1);
  const int bi = ln.m0;
  double acc[2][1] = {{0.0}, {0.0}};
  for (int64_t row = (int64_t)blockIdx.x * ln.rpb + ln.rl; row < n;
       row += (int64_t)gridDim.x * ln.rpb) {
    const int64_t o = row * K + bi;
    T bv = b[o];
    T rv = bv;
    if (guess) {  // R = B - A X0
      const T ax = mat.sum1(row, [&](int32_t c) { return x[(int64_t)c * K + bi]; });
      rv = sub_rn(bv, ax);
    }
    r[o] = rv;
    p_old[o] = T(0);
    T z = PREC ? mul_rn(dinv[row], rv) : rv;
    acc[0][0] += (double)rv * (double)z;
    acc[1][0] += (double)bv * (double)bv;
  }
  if (!batch_reduce<2, 1>(acc, K, smem, partials, &st->counter[0])) return;
  for (int c = threadIdx.x; c < K; c += blockDim.x) {
    cs.rz[c] = smem[c];
    double bn = sqrt(smem[K + c]);
    if (bn == 0.0) bn = 1.0;
    double tol = fmax(atol, rtol * bn);
    cs.tol_sq[c] = tol * tol;
    cs.beta[c] = 0.0;
    cs.iters[c] = 0;
    cs.conv[c] = 0;
  }
  if (threadIdx.x == 0) {
    st->iter = 0;
    st->done = st->maxiter <= 0 ? 2 : 0;
  }
}

// The zeroing of x when no guess is given runs as a separate pass (the init
// kernel reads x for the guess).
template <typename T>
__global__ void zero_kernel(T *__restrict__ x, int64_t n) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; i < n; i += stride) x[i] = T(0);
}

// P = Z + beta P (pytorch_backend.py:2487) is formed once per row by
// mrhs_pform_kernel and K_A gathers it (SLA_MRHS_SPLIT 1), or K_A forms it
// inside the gather, every row recomputing it for each of its entries
// (SLA_MRHS_SPLIT 0). Measured on 128^3 7-point x 16 columns fp64: the
// split costs one more [n][K] pass but halves the loads per gathered entry,
// K_A 366 -> 184 us, 26.5 k -> 29.0 k column-iterations/s; 7-entry load
// batches on the split gather: 28.6 k.
#ifndef SLA_MRHS_SPLIT
#define SLA_MRHS_SPLIT 1
#endif
constexpr bool kMrhsSplit = SLA_MRHS_SPLIT != 0;

template <typename T, bool PREC, int VEC>
__device__ __forceinline__ Pack<T, VEC> mrhs_p(const T *__restrict__ r, const T *__restrict__ dinv,
                                               const T *__restrict__ p_old, int64_t c, int32_t ci,
                                               const T (&beta)[VEC]) {
  const Pack<T, VEC> rv = vload<T, VEC, kLoadRO>(r + c);
  const Pack<T, VEC> po = vload<T, VEC, kLoadRO>(p_old + c);
  const T d = PREC ? __ldg(dinv + ci) : T(1);
  Pack<T, VEC> out;
#pragma unroll
  for (int u = 0; u < VEC; ++u) {
    const T z = PREC ? mul_rn(d, rv.v[u]) : rv.v[u];
    out.v[u] = add_rn(z, mul_rn(beta[u], po.v[u]));
  }
  return out;
}

template <typename T, bool PREC, int VEC>
__global__ void __launch_bounds__(VEC == 1 ? 1024 : kBatchThreads, VEC == 1 ? 1 : kBatchMinBlocks)
mrhs_pform_kernel(int64_t n, int K, const T *__restrict__ r, const T *__restrict__ dinv,
                  const T *__restrict__ p_old, T *__restrict__ p_new, const MrhsState *st,
                  MrhsCols cs) {
  if (*(volatile const int *)&st->done) return;
  const BatchLane ln(K, VEC);
  T beta[VEC];
#pragma unroll
  for (int u = 0; u < VEC; ++u) beta[u] = (T)cs.beta[ln.m0 + u];
  for (int64_t row = (int64_t)blockIdx.x * ln.rpb + ln.rl; row < n;
       row += (int64_t)gridDim.x * ln.rpb) {
    const int64_t o = row * K + ln.m0;
    vstore(p_new + o, mrhs_p<T, PREC, VEC>(r, dinv, p_old, o, (int32_t)row, beta));
  }
}

// AP = A P, per-column (P, AP); the last block forms alpha with
// (P, AP) <= 0 -> 1.
template <typename T, bool PREC, int VEC, int RB, typename M>
__global__ void __launch_bounds__(VEC == 1 ? 1024 : kBatchThreads, VEC == 1 ? 1 : kBatchMinBlocks)
mrhs_spmv_kernel(M mat, int64_t n, int K, const T *__restrict__ r,
                 const T *__restrict__ dinv, const T *__restrict__ p_old, T *__restrict__ p_new,
                 T *__restrict__ Ap, MrhsState *st, MrhsCols cs, double *partials) {
  extern __shared__ double smem[];
  if (*(volatile int *)&st->done) return;
  const BatchLane ln(K, VEC);
  T beta[VEC];
#pragma unroll
  for (int u = 0; u < VEC; ++u) beta[u] = (T)cs.beta[ln.m0 + u];
  double acc[1][VEC];
#pragma unroll
  for (int u = 0; u < VEC; ++u) acc[0][u] = 0.0;
  for (int64_t row = (int64_t)blockIdx.x * ln.rpb + ln.rl; row < n;
       row += (int64_t)gridDim.x * ln.rpb) {
    T sum[VEC];
    mat.template sum<VEC, RB>(
        row,
        [&](int32_t ci) {
          const int64_t c = (int64_t)ci * K + ln.m0;
          if constexpr (kMrhsSplit) return vload<T, VEC, kLoadRO>(p_new + c);
          else return mrhs_p<T, PREC, VEC>(r, dinv, p_old, c, ci, beta);
        },
        sum);
    const int64_t o = row * K + ln.m0;
    Pack<T, VEC> pn, ap;
    if constexpr (kMrhsSplit) pn = vload<T, VEC, kLoadRO>(p_new + o);
    else pn = mrhs_p<T, PREC, VEC>(r, dinv, p_old, o, (int32_t)row, beta);
#pragma unroll
    for (int u = 0; u < VEC; ++u) {
      ap.v[u] = sum[u];
      acc[0][u] += (double)pn.v[u] * (double)sum[u];
    }
    if constexpr (!kMrhsSplit) vstore(p_new + o, pn);
    vstore(Ap + o, ap);
  }
  if (!batch_reduce<1, VEC>(acc, K, smem, partials, &st->counter[1])) return;
  for (int c = threadIdx.x; c < K; c += blockDim.x) {
    const double pap = smem[c];
    cs.alpha[c] = cs.rz[c] / (pap > 0.0 ? pap : 1.0);
  }
}

// ------------------------------------------------ SpMM over staged P tiles
// For a diagonal-offset view whose offsets are [-b, -1, 0, 1, b] (W = 5) or
// [-a, -b, -1, 0, 1, b, a] (W = 7) -- 2-D and 3-D structured grids -- the rows
// a tile of rpb consecutive rows r0 .. r0+rpb-1 gathers from lie in at most
// five contiguous ranges of P ([n][K] rows): r0-1 .. r0+rpb (the rows and
// their +-1 neighbours) and r0 -+ b, r0 -+ a (rpb rows each); the tile's
// matrix values are the contiguous SELL slices that hold its rows. One
// thread of the block copies all of it into shared memory with bulk copies
// (cp.async.bulk, completion counted on an mbarrier), double-buffered so
// that the next tile streams in while this one computes; the block then
// reads nothing else from global memory, and one barrier per tile both
// releases the buffer and agrees on a timeout. Each row sums its entries in
// ascending diagonal order from the same values as mrhs_spmv_kernel. Waits
// are bounded (kWaitLimitNs); a timeout stops the solve with state 4.
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}
__device__ __forceinline__ void bulk_copy_g2s(void *dst, const void *src, uint32_t bytes,
                                              uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for phase `parity` of an mbarrier.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  while (!mbar_try_wait(bar, parity))
    if (global_ns() - t0 > kWaitLimitNs) return false;
  return true;
}

constexpr int kMrhsTimeout = 4;  // MrhsState::done when a tile never arrived

// Elements of one staged tile: P rows (range 0 holds rpb + 2 rows, r0-1 ..
// r0+rpb, the others rpb rows each), then the values of the SELL slices the
// tile's rows span (at most (rpb + 31) / 32 + 1 slices of 32 W entries).
inline size_t tile_p_rows(int W, int rpb) { return (size_t)(W == 7 ? 5 : 3) * rpb + 2; }
inline size_t tile_elems(int W, int rpb, int K) {
  return tile_p_rows(W, rpb) * K + (size_t)((rpb + 31) / 32 + 1) * 32 * W;
}

template <typename T, bool PREC, int VEC, int W>
__global__ void __launch_bounds__(kBatchThreads, kBatchMinBlocks)
mrhs_spmv_tile_kernel(Sell<T> A, int64_t n, int K, const T *__restrict__ p, T *__restrict__ Ap,
                      MrhsState *st, MrhsCols cs, double *partials) {
  extern __shared__ __align__(128) unsigned char mt_smem[];
  __shared__ uint64_t bar[2];
  __shared__ int s_stop;
  if (threadIdx.x == 0) {
    // one read for the whole block: a block of this launch that timed out
    // may set st->done while others start
    s_stop = *(volatile int *)&st->done;
    if (!s_stop) {
      mbar_init(&bar[0], 1);
      mbar_init(&bar[1], 1);
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
  }
  __syncthreads();
  if (s_stop) return;
  const BatchLane ln(K, VEC);
  const int rpb = ln.rpb;
  constexpr int NR = W == 7 ? 5 : 3;  // P ranges
  const int TR = NR * rpb + 2;
  T *const buf0 = reinterpret_cast<T *>(mt_smem);
  const size_t buf_elems = (size_t)TR * K + (size_t)((rpb + 31) / 32 + 1) * 32 * W;
  double *red = reinterpret_cast<double *>(buf0 + 2 * buf_elems);
  const int64_t b_off = -(int64_t)A.off[W == 7 ? 1 : 0];
  const int64_t a_off = W == 7 ? -(int64_t)A.off[0] : 0;
  // first buffer row of each range: A (r0-1..), B (-b), C (+b), D (-a), E (+a)
  const int base_b = rpb + 2, base_c = 2 * rpb + 2, base_d = 3 * rpb + 2, base_e = 4 * rpb + 2;
  const int64_t ntiles = (n + rpb - 1) / rpb;
  const size_t row_bytes = (size_t)K * sizeof(T);
  // thread 0: copy the P ranges and the values of tile t into buffer q
  auto issue = [&](int64_t t, int q) {
    const int64_t r0 = t * rpb;
    const int64_t lo[5] = {r0 - 1, r0 - b_off, r0 + b_off, r0 - a_off, r0 + a_off};
    const int cnt[5] = {rpb + 2, rpb, rpb, rpb, rpb};
    const int dst[5] = {0, base_b, base_c, base_d, base_e};
    int64_t g0[5], g1[5];
    const int64_t last = (r0 + rpb < n ? r0 + rpb : n) - 1;
    const int64_t s_lo = r0 >> 5, s_hi = last >> 5;
    const uint32_t vbytes = (uint32_t)((s_hi - s_lo + 1) * 32 * W * sizeof(T));
    uint32_t bytes = vbytes;
#pragma unroll
    for (int k = 0; k < NR; ++k) {
      g0[k] = lo[k] < 0 ? 0 : lo[k];
      g1[k] = lo[k] + cnt[k] > n ? n : lo[k] + cnt[k];
      if (g1[k] > g0[k]) bytes += (uint32_t)((g1[k] - g0[k]) * row_bytes);
    }
    T *b = buf0 + q * buf_elems;
    mbar_expect_tx(&bar[q], bytes);
    bulk_copy_g2s(b + (size_t)TR * K, A.val + s_lo * 32 * W, vbytes, &bar[q]);
#pragma unroll
    for (int k = 0; k < NR; ++k)
      if (g1[k] > g0[k])
        bulk_copy_g2s(b + (size_t)(dst[k] + (g0[k] - lo[k])) * K, p + g0[k] * K,
                      (uint32_t)((g1[k] - g0[k]) * row_bytes), &bar[q]);
  };
  double acc[1][VEC];
#pragma unroll
  for (int u = 0; u < VEC; ++u) acc[0][u] = 0.0;
  uint32_t phase = 0u;  // bit q: parity of buffer q's next phase
  int64_t t = blockIdx.x;
  if (t < ntiles && threadIdx.x == 0) issue(t, 0);
  int q = 0;
  bool failed = false, pending_other = false;
  for (; t < ntiles; t += gridDim.x, q ^= 1) {
    const int64_t tn = t + gridDim.x;
    pending_other = tn < ntiles;
    if (pending_other && threadIdx.x == 0) {
      // buffer q^1 was last read before the previous iteration's barrier
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(tn, q ^ 1);
    }
    const bool ok = mbar_wait_bounded(&bar[q], (phase >> q) & 1u);
    phase ^= 1u << q;
    const int64_t row = t * rpb + ln.rl;
    if (ok && row < n) {
      const T *tile = buf0 + q * buf_elems;
      const T *vp = tile + (size_t)TR * K + ((row >> 5) - ((t * rpb) >> 5)) * 32 * W + (row & 31);
      int idx[W];
      if constexpr (W == 7) {
        idx[0] = base_d; idx[1] = base_b; idx[2] = 0; idx[3] = 1; idx[4] = 2;
        idx[5] = base_c; idx[6] = base_e;
      } else {
        idx[0] = base_b; idx[1] = 0; idx[2] = 1; idx[3] = 2; idx[4] = base_c;
      }
      T sum[VEC];
#pragma unroll
      for (int u = 0; u < VEC; ++u) sum[u] = T(0);
#pragma unroll
      for (int j = 0; j < W; ++j) {
        const T v = vp[32 * j];
        const int64_t c = row + A.off[j];
        Pack<T, VEC> xv = splat<T, VEC>(T(0));
        if (c >= 0 && c < A.n_cols)
          xv = vload<T, VEC>(tile + (size_t)(idx[j] + ln.rl) * K + ln.m0);
#pragma unroll
        for (int u = 0; u < VEC; ++u) sum[u] = fma(v, xv.v[u], sum[u]);
      }
      const Pack<T, VEC> pn = vload<T, VEC>(tile + (size_t)(1 + ln.rl) * K + ln.m0);
      Pack<T, VEC> ap;
#pragma unroll
      for (int u = 0; u < VEC; ++u) {
        ap.v[u] = sum[u];
        acc[0][u] += (double)pn.v[u] * (double)sum[u];
      }
      vstore(Ap + row * K + ln.m0, ap);
    }
    // releases buffer q for the copy issued at the top of the next step,
    // and agrees on a timeout
    if (__syncthreads_or(!ok)) {
      failed = true;
      break;
    }
  }
  if (failed) {
    // wait (bounded) for the copy still in flight into the other buffer
    if (pending_other) mbar_wait_bounded(&bar[q ^ 1], (phase >> (q ^ 1)) & 1u);
    if (threadIdx.x == 0) st->done = kMrhsTimeout;
  }
  if (!batch_reduce<1, VEC>(acc, K, red, partials, &st->counter[1])) return;
  for (int c = threadIdx.x; c < K; c += blockDim.x) {
    const double pap = red[c];
    cs.alpha[c] = cs.rz[c] / (pap > 0.0 ? pap : 1.0);
  }
}

// Offsets of a view the staged-tile SpMM serves: [-b, -1, 0, 1, b] or
// [-a, -b, -1, 0, 1, b, a] with 1 < b < a.
template <typename T>
inline bool tile_offsets_ok(const CsrRows<T> &) { return false; }
template <typename T, int W>
inline bool tile_offsets_ok(const DiagRows<T, W> &m) {
  const int32_t *o = m.A.off;
  if (W == 5) return o[1] == -1 && o[2] == 0 && o[3] == 1 && o[4] == -o[0] && o[4] > 1;
  if (W == 7)
    return o[2] == -1 && o[3] == 0 && o[4] == 1 && o[5] == -o[1] && o[6] == -o[0] && o[5] > 1 &&
           o[6] > o[5];
  return false;
}

// X is updated at odd iterations only, X = (X + alpha_prev P_prev) + alpha P
// (the same two roundings as two single steps), while both directions sit
// in the ping-pong buffers; mrhs_xflush_kernel applies a step left pending.
template <typename T, bool PREC, int VEC>
__global__ void __launch_bounds__(VEC == 1 ? 1024 : kBatchThreads, VEC == 1 ? 1 : kBatchMinBlocks)
mrhs_update_kernel(int64_t n, int K, T *__restrict__ x, T *__restrict__ r, const T *__restrict__ p,
                   const T *__restrict__ p_prev, const T *__restrict__ Ap,
                   const T *__restrict__ dinv, MrhsState *st, MrhsCols cs, double *partials,
                   int xu) {
  extern __shared__ double smem[];
  __shared__ int s_all;
  if (*(volatile int *)&st->done) return;
  const BatchLane ln(K, VEC);
  T alpha[VEC], alpha_prev[VEC];
#pragma unroll
  for (int u = 0; u < VEC; ++u) {
    alpha[u] = (T)cs.alpha[ln.m0 + u];
    alpha_prev[u] = (T)cs.alpha_prev[ln.m0 + u];
  }
  double acc[2][VEC];
#pragma unroll
  for (int u = 0; u < VEC; ++u) acc[0][u] = acc[1][u] = 0.0;
  for (int64_t row = (int64_t)blockIdx.x * ln.rpb + ln.rl; row < n;
       row += (int64_t)gridDim.x * ln.rpb) {
    const int64_t o = row * K + ln.m0;
    Pack<T, VEC> rv = vload<T, VEC>(r + o);
    const Pack<T, VEC> av = vload<T, VEC, kLoadStream>(Ap + o);
    const T d = PREC ? __ldg(dinv + row) : T(1);
    if (xu) {
      Pack<T, VEC> xv = vload<T, VEC>(x + o);
      const Pack<T, VEC> pv = vload<T, VEC, kLoadStream>(p + o);
      const Pack<T, VEC> qv = vload<T, VEC, kLoadStream>(p_prev + o);
#pragma unroll
      for (int u = 0; u < VEC; ++u)
        xv.v[u] = add_rn(add_rn(xv.v[u], mul_rn(alpha_prev[u], qv.v[u])),
                         mul_rn(alpha[u], pv.v[u]));
      vstore(x + o, xv);
    }
#pragma unroll
    for (int u = 0; u < VEC; ++u) {
      rv.v[u] = sub_rn(rv.v[u], mul_rn(alpha[u], av.v[u]));
      const T zi = PREC ? mul_rn(d, rv.v[u]) : rv.v[u];
      acc[0][u] += (double)rv.v[u] * (double)rv.v[u];
      acc[1][u] += (double)rv.v[u] * (double)zi;
    }
    vstore(r + o, rv);
  }
  if (!batch_reduce<2, VEC>(acc, K, smem, partials, &st->counter[2])) return;
  const long long it = st->iter + 1;
  const bool check = (it % st->check_every) == 0;
  if (threadIdx.x == 0) s_all = 1;
  __syncthreads();
  for (int c = threadIdx.x; c < K; c += blockDim.x) {
    const double rr = smem[c], rz = smem[K + c];
    cs.rr[c] = rr;
    if (check && !cs.conv[c] && rr < cs.tol_sq[c]) {
      cs.conv[c] = 1;
      cs.iters[c] = it;
    }
    if (!cs.conv[c]) atomicAnd(&s_all, 0);
    const double rz_old = cs.rz[c];
    cs.beta[c] = rz / (rz_old + 1e-30);
    cs.rz[c] = rz;
    cs.alpha_prev[c] = cs.alpha[c];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    st->iter = it;
    if (check && s_all) { st->done = 1; st->iters_out = it; }
    else if (it >= st->maxiter) { st->done = 2; st->iters_out = st->maxiter; }
  }
}

// Pending X step after a last even iteration (st->iter odd).
template <typename T>
__global__ void mrhs_xflush_kernel(int64_t n, int K, T *__restrict__ x,
                                   const T *__restrict__ p_last, const MrhsState *st,
                                   MrhsCols cs) {
  if ((st->iter & 1) == 0) return;
  int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; t < n * K; t += stride)
    x[t] = add_rn(x[t], mul_rn((T)cs.alpha_prev[t % K], p_last[t]));
}

static size_t mrhs_ws_bytes(size_t elem, int64_t n, int64_t K) {
  return 4 * align_up(elem * (size_t)(n * K)) +
         3 * align_up(2 * (size_t)K * batch_max_grid() * sizeof(double)) +
         6 * align_up((size_t)K * sizeof(double)) + align_up((size_t)K * sizeof(long long)) +
         align_up((size_t)K * sizeof(int)) + align_up(sizeof(MrhsState));
}


template <typename T, bool PREC, int VEC, typename M>
static int mrhs_loop(M mat, int64_t n, int K, const T *dinv, T *x, T *r, T *pA, T *pB, T *Ap,
                     MrhsState *st, MrhsCols cs, double *const part[3], int64_t maxiter,
                     cudaStream_t s) {
  auto spmv = mrhs_spmv_kernel<T, PREC, VEC, kBatchRB, M>;
  auto upd = mrhs_update_kernel<T, PREC, VEC>;
  const int TB = batch_block(K, VEC);
  const size_t sm1 = batch_smem(1, TB, VEC), sm2 = batch_smem(2, TB, VEC);
  const int G1 = occupancy_grid((const void *)spmv, TB, sm1);
  const int G2 = occupancy_grid((const void *)upd, TB, sm2);
  auto pform = mrhs_pform_kernel<T, PREC, VEC>;
  const int G0 = kMrhsSplit ? occupancy_grid((const void *)pform, TB, 0) : 0;
  // staged-tile SpMM (TMA bulk copies of the gathered P ranges) where the
  // view's offsets allow it
  const void *tk = nullptr;
  size_t smt = 0;
  int Gt = 0;
  if constexpr (kMrhsSplit && VEC > 1) {
    if (tile_offsets_ok(mat) && aligned16(pA, pB, Ap) && (K * sizeof(T)) % 16 == 0) {
      constexpr int Wv = M::kWidth;
      if constexpr (Wv == 5 || Wv == 7) {
        tk = (const void *)mrhs_spmv_tile_kernel<T, PREC, VEC, Wv>;
        const int rpb = TB / (K / VEC);
        smt = 2 * tile_elems(Wv, rpb, K) * sizeof(T) + sm1;
        SLA_CUDA_TRY(cudaFuncSetAttribute(tk, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)smt));
        Gt = occupancy_grid(tk, TB, smt);
      }
    }
  }
  return run_chunked(maxiter, 8, &st->done, s, [&](int64_t it) -> int {
    T *p_old = (it & 1) ? pB : pA, *p_new = (it & 1) ? pA : pB;
    cudaEvent_t ev;
    if (kMrhsSplit) SLA_LAUNCH(pform, G0, TB, 0, s, n, K, r, dinv, p_old, p_new, st, cs);
    profiler().begin(0, it, s, &ev);
    if (tk) {
      if constexpr (kMrhsSplit && VEC > 1) {
        if constexpr (M::kWidth == 5 || M::kWidth == 7) {
          SLA_LAUNCH((mrhs_spmv_tile_kernel<T, PREC, VEC, M::kWidth>), Gt, TB, smt, s, mat.A, n,
                     K, (const T *)p_new, Ap, st, cs, part[1]);
        }
      }
    } else {
      SLA_LAUNCH(spmv, G1, TB, sm1, s, mat, n, K, r, dinv, p_old, p_new, Ap, st, cs, part[1]);
    }
    profiler().end(0, s, ev);
    SLA_LAUNCH(upd, G2, TB, sm2, s, n, K, x, r, p_new, p_old, Ap, dinv, st, cs, part[2],
               (int)(it & 1));
    return SLA_OK;
  });
}

template <typename T, bool PREC, typename M>
static int mrhs_impl(M mat, int64_t n, int K, const T *dinv, const T *b, T *x, bool guess,
                     double atol, double rtol,
                     int64_t maxiter, int64_t every, int64_t *iters_out, int32_t *conv_out,
                     void *ws, size_t ws_bytes, sla_solve_info_t *info, cudaStream_t s) {
  Carver c(ws, ws_bytes);
  const size_t nk = (size_t)(n * K);
  T *r = c.take<T>(nk), *pA = c.take<T>(nk), *pB = c.take<T>(nk), *Ap = c.take<T>(nk);
  double *part[3];
  for (int q = 0; q < 3; ++q) part[q] = c.take<double>(2 * (size_t)K * batch_max_grid());
  MrhsCols cs;
  cs.rz = c.take<double>(K); cs.alpha = c.take<double>(K); cs.beta = c.take<double>(K);
  cs.tol_sq = c.take<double>(K); cs.rr = c.take<double>(K); cs.alpha_prev = c.take<double>(K);
  cs.iters = c.take<long long>(K);
  cs.conv = c.take<int>(K);
  MrhsState *st = c.take<MrhsState>(1);
  if (!c.ok) return SLA_ERR_WORKSPACE;
  MrhsState init{};
  init.maxiter = maxiter;
  init.check_every = every;
  SLA_CUDA_TRY(cudaMemcpyAsync(st, &init, sizeof(init), cudaMemcpyHostToDevice, s));
  {
    auto init_fn = mrhs_init_kernel<T, PREC, M>;
    const int TB0 = batch_block(K, 1);
    const size_t sm0 = batch_smem(2, TB0, 1);
    const int G0 = occupancy_grid((const void *)init_fn, TB0, sm0);
    SLA_LAUNCH(init_fn, G0, TB0, sm0, s, mat, n, K, b, x, guess ? 1 : 0, dinv, r, pA, st, cs,
               part[0], atol, rtol);
  }
  if (!guess) SLA_LAUNCH(zero_kernel<T>, grid_for((int64_t)nk), kBlock, 0, s, x, (int64_t)nk);
  // 16-byte vector groups of columns where K and the caller's x allow it
  constexpr int kVec = 16 / sizeof(T);
  int rc;
  if (K % kVec == 0 && aligned16(x))
    rc = mrhs_loop<T, PREC, kVec>(mat, n, K, dinv, x, r, pA, pB, Ap, st, cs, part, maxiter, s);
  else
    rc = mrhs_loop<T, PREC, 1>(mat, n, K, dinv, x, r, pA, pB, Ap, st, cs, part, maxiter, s);
  SLA_TRY(rc);
  // a last even iteration's direction sits in pB
  SLA_LAUNCH(mrhs_xflush_kernel<T>, grid_for((int64_t)nk), kBlock, 0, s, n, K, x, pB, st, cs);
  MrhsState out;
  std::vector<double> rr(K), tol_sq(K);
  std::vector<long long> its(K);
  std::vector<int> conv(K);
  SLA_CUDA_TRY(cudaMemcpyAsync(&out, st, sizeof(out), cudaMemcpyDeviceToHost, s));
  SLA_CUDA_TRY(cudaMemcpyAsync(rr.data(), cs.rr, sizeof(double) * K, cudaMemcpyDeviceToHost, s));
  SLA_CUDA_TRY(cudaMemcpyAsync(tol_sq.data(), cs.tol_sq, sizeof(double) * K, cudaMemcpyDeviceToHost, s));
  SLA_CUDA_TRY(cudaMemcpyAsync(its.data(), cs.iters, sizeof(long long) * K, cudaMemcpyDeviceToHost, s));
  SLA_CUDA_TRY(cudaMemcpyAsync(conv.data(), cs.conv, sizeof(int) * K, cudaMemcpyDeviceToHost, s));
  SLA_CUDA_TRY(cudaStreamSynchronize(s));
  profiler().resolve();
  // final bookkeeping of batched_pcg_solve: unconverged columns report
  // maxiter; a final residual below its tolerance still counts as converged
  bool all = true;
  double worst = 0.0;
  for (int k = 0; k < K; ++k) {
    if (!conv[k]) its[k] = maxiter;
    bool ok = conv[k] || sqrt(rr[k]) < sqrt(tol_sq[k]);
    all = all && ok;
    worst = fmax(worst, sqrt(rr[k]));
    if (iters_out) iters_out[k] = its[k];
    if (conv_out) conv_out[k] = ok ? 1 : 0;
  }
  info->iterations = out.done == 0 ? maxiter : out.iters_out;
  info->residual = worst;
  info->reason = out.done;
  info->status = out.done == kMrhsTimeout ? SLA_ERR_TIMEOUT : all ? SLA_OK : SLA_NOT_CONVERGED;
  return info->status;
}

static int mrhs_args_ok(int dtype, int64_t n, int64_t k, const void *b, void *x,
                        sla_solve_info_t *info, int64_t check_every, void *workspace,
                        size_t workspace_bytes) {
  if (!b || !x || !info || n <= 0 || n >= INT32_MAX) return SLA_ERR_INVALID;
  if (k < 1 || check_every < 1) return SLA_ERR_INVALID;
  if (k > 1024) return SLA_ERR_UNSUPPORTED;
  info->iterations = 0; info->residual = 0; info->status = 0; info->reason = 0;
  size_t need = 0;
  SLA_TRY(sla_multi_rhs_cg_workspace(dtype, n, k, &need));
  if (workspace_bytes < need || !workspace) return SLA_ERR_WORKSPACE;
  return SLA_OK;
}

// Dispatch on dtype and preconditioning for one row-access type.
template <template <typename> class Mk>
static int mrhs_run(int dtype, Mk<double> md, Mk<float> mf, int64_t n, int K, const void *dinv,
                    const void *b, void *x, bool g, double atol, double rtol, int64_t maxiter,
                    int64_t every, int64_t *iters_out, int32_t *conv_out, void *ws,
                    size_t ws_bytes, sla_solve_info_t *info, cudaStream_t s) {
  if (dtype == SLA_F64) {
    if (dinv)
      return mrhs_impl<double, true>(md, n, K, (const double *)dinv, (const double *)b,
                                     (double *)x, g, atol, rtol, maxiter, every, iters_out,
                                     conv_out, ws, ws_bytes, info, s);
    return mrhs_impl<double, false>(md, n, K, nullptr, (const double *)b, (double *)x, g, atol,
                                    rtol, maxiter, every, iters_out, conv_out, ws, ws_bytes,
                                    info, s);
  }
  if (dtype == SLA_F32) {
    if (dinv)
      return mrhs_impl<float, true>(mf, n, K, (const float *)dinv, (const float *)b, (float *)x,
                                    g, atol, rtol, maxiter, every, iters_out, conv_out, ws,
                                    ws_bytes, info, s);
    return mrhs_impl<float, false>(mf, n, K, nullptr, (const float *)b, (float *)x, g, atol,
                                   rtol, maxiter, every, iters_out, conv_out, ws, ws_bytes, info,
                                   s);
  }
  return SLA_ERR_INVALID;
}

template <int W> struct DiagW {
  template <typename T> using type = DiagRows<T, W>;
};

}  // namespace sla

using namespace sla;

extern "C" {

int sla_multi_rhs_cg_workspace(int dtype, int64_t n, int64_t k, size_t *bytes) {
  if (!bytes || n < 0 || k < 1 || k > 1024) return SLA_ERR_INVALID;
  if (dtype != SLA_F32 && dtype != SLA_F64) return SLA_ERR_INVALID;
  *bytes = mrhs_ws_bytes(dtype == SLA_F64 ? 8 : 4, n, k);
  return SLA_OK;
}

int sla_multi_rhs_cg(int dtype, const int32_t *rowptr, const int32_t *colind, const void *vals,
                     int64_t n, int64_t k, const void *dinv, const void *b, void *x,
                     int x_is_guess, double atol, double rtol, int64_t maxiter,
                     int64_t check_every, int64_t *iters_out, int32_t *converged_out,
                     void *workspace, size_t workspace_bytes, sla_solve_info_t *info,
                     sla_stream_t stream) {
  if (!rowptr || !colind || !vals) return SLA_ERR_INVALID;
  SLA_TRY(mrhs_args_ok(dtype, n, k, b, x, info, check_every, workspace, workspace_bytes));
  CsrRows<double> md{rowptr, colind, (const double *)vals};
  CsrRows<float> mf{rowptr, colind, (const float *)vals};
  return mrhs_run<CsrRows>(dtype, md, mf, n, (int)k, dinv, b, x, x_is_guess != 0, atol, rtol,
                           maxiter, check_every, iters_out, converged_out, workspace,
                           workspace_bytes, info, (cudaStream_t)stream);
}

int sla_multi_rhs_cg_diag(int dtype, const sla_sell_t *A, int64_t k, const void *dinv,
                          const void *b, void *x, int x_is_guess, double atol, double rtol,
                          int64_t maxiter, int64_t check_every, int64_t *iters_out,
                          int32_t *converged_out, void *workspace, size_t workspace_bytes,
                          sla_solve_info_t *info, sla_stream_t stream) {
  SLA_TRY(sell_check(A));
  if (A->n_diags <= 0 || A->row_ids || A->row_base) return SLA_ERR_INVALID;
  const int64_t n = A->n_slots;
  if (A->n_cols != n) return SLA_ERR_INVALID;  // square system
  SLA_TRY(mrhs_args_ok(dtype, n, k, b, x, info, check_every, workspace, workspace_bytes));
  cudaStream_t s = (cudaStream_t)stream;
  const bool g = x_is_guess != 0;
  switch (A->n_diags) {
    case 5:
      return mrhs_run<DiagW<5>::type>(dtype, {make_sell<double>(A)}, {make_sell<float>(A)}, n,
                                      (int)k, dinv, b, x, g, atol, rtol, maxiter, check_every,
                                      iters_out, converged_out, workspace, workspace_bytes, info,
                                      s);
    case 7:
      return mrhs_run<DiagW<7>::type>(dtype, {make_sell<double>(A)}, {make_sell<float>(A)}, n,
                                      (int)k, dinv, b, x, g, atol, rtol, maxiter, check_every,
                                      iters_out, converged_out, workspace, workspace_bytes, info,
                                      s);
    case 27:
      return mrhs_run<DiagW<27>::type>(dtype, {make_sell<double>(A)}, {make_sell<float>(A)}, n,
                                       (int)k, dinv, b, x, g, atol, rtol, maxiter, check_every,
                                       iters_out, converged_out, workspace, workspace_bytes,
                                       info, s);
    default:
      return SLA_ERR_UNSUPPORTED;
  }
}

}  // extern "C"
