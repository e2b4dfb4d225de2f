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
  return run_chunked(maxiter, 8, &st->done, s, [&](int64_t it) -> int {
    T *p_old = (it & 1) ? pB : pA, *p_new = (it & 1) ? pA : pB;
    cudaEvent_t ev;
    if (kMrhsSplit) SLA_LAUNCH(pform, G0, TB, 0, s, n, K, r, dinv, p_old, p_new, st, cs);
    profiler().begin(0, it, s, &ev);
    SLA_LAUNCH(spmv, G1, TB, sm1, s, mat, n, K, r, dinv, p_old, p_new, Ap, st, cs, part[1]);
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
  info->status = all ? SLA_OK : SLA_NOT_CONVERGED;
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
