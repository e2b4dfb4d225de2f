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
  double *rz, *alpha, *beta, *tol_sq, *rr;
  long long *iters;   // per column, 0 until converged
  int *conv;          // per column convergence flag
};

template <typename T, bool PREC>
__global__ void __launch_bounds__(1024)
mrhs_init_kernel(const int32_t *__restrict__ rowptr, const int32_t *__restrict__ colind,
                 const T *__restrict__ vals, int64_t n, int K, const T *__restrict__ b,
                 T *__restrict__ x, int guess, const T *__restrict__ dinv, T *__restrict__ r,
                 T *__restrict__ p_old, MrhsState *st, MrhsCols cs, double *partials,
                 double atol, double rtol) {
  __shared__ double smem[2 * 1024];
  const int rpb = blockDim.x / K;
  const int bi = threadIdx.x % K, rl = threadIdx.x / K;
  double acc[2] = {0.0, 0.0};
  if (rl < rpb) {
    for (int64_t row = (int64_t)blockIdx.x * rpb + rl; row < n; row += (int64_t)gridDim.x * rpb) {
      const int64_t o = row * K + bi;
      T bv = b[o];
      T rv = bv;
      if (guess) {  // R = B - A X0
        T ax = T(0);
        for (int32_t k = rowptr[row]; k < rowptr[row + 1]; ++k)
          ax = fma(vals[k], x[(int64_t)colind[k] * K + bi], ax);
        rv = sub_rn(bv, ax);
      }
      r[o] = rv;
      p_old[o] = T(0);
      T z = PREC ? mul_rn(dinv[row], rv) : rv;
      acc[0] += (double)rv * (double)z;
      acc[1] += (double)bv * (double)bv;
    }
  }
  if (batch_last_block<2>(acc, K, smem, partials, &st->counter[0]) && threadIdx.x < K) {
    const int c = threadIdx.x;
    cs.rz[c] = acc[0];
    double bn = sqrt(acc[1]);
    if (bn == 0.0) bn = 1.0;
    double tol = fmax(atol, rtol * bn);
    cs.tol_sq[c] = tol * tol;
    cs.beta[c] = 0.0;
    cs.iters[c] = 0;
    cs.conv[c] = 0;
    if (c == 0) {
      st->iter = 0;
      st->done = st->maxiter <= 0 ? 2 : 0;
    }
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

template <typename T, bool PREC>
__global__ void __launch_bounds__(1024)
mrhs_spmv_kernel(const int32_t *__restrict__ rowptr, const int32_t *__restrict__ colind,
                 const T *__restrict__ vals, int64_t n, int K, const T *__restrict__ r,
                 const T *__restrict__ dinv, const T *__restrict__ p_old, T *__restrict__ p_new,
                 T *__restrict__ Ap, MrhsState *st, MrhsCols cs, double *partials) {
  __shared__ double smem[1024];
  if (*(volatile int *)&st->done) return;
  const int rpb = blockDim.x / K;
  const int bi = threadIdx.x % K, rl = threadIdx.x / K;
  double acc[1] = {0.0};
  if (rl < rpb) {
    const T beta = (T)cs.beta[bi];
    for (int64_t row = (int64_t)blockIdx.x * rpb + rl; row < n; row += (int64_t)gridDim.x * rpb) {
      // P = Z + beta P (pytorch_backend.py:2487), formed inside the gather
      const T sum = csr_row_batched<T>(
          colind, rowptr[row], rowptr[row + 1], [&](int32_t k) { return __ldg(vals + k); },
          [&](int32_t cidx) {
            const int64_t c = (int64_t)cidx * K + bi;
            T z = PREC ? mul_rn(__ldg(dinv + cidx), __ldg(r + c)) : __ldg(r + c);
            return add_rn(z, mul_rn(beta, __ldg(p_old + c)));
          });
      const int64_t o = row * K + bi;
      T z = PREC ? mul_rn(dinv[row], r[o]) : r[o];
      T pn = add_rn(z, mul_rn(beta, p_old[o]));
      p_new[o] = pn;
      Ap[o] = sum;
      acc[0] += (double)pn * (double)sum;
    }
  }
  if (batch_last_block<1>(acc, K, smem, partials, &st->counter[1]) && threadIdx.x < K) {
    double pap = acc[0];
    cs.alpha[threadIdx.x] = cs.rz[threadIdx.x] / (pap > 0.0 ? pap : 1.0);
  }
}

template <typename T, bool PREC>
__global__ void __launch_bounds__(1024)
mrhs_update_kernel(int64_t n, int K, T *__restrict__ x, T *__restrict__ r, const T *__restrict__ p,
                   const T *__restrict__ Ap, const T *__restrict__ dinv, MrhsState *st,
                   MrhsCols cs, double *partials) {
  __shared__ double smem[2 * 1024];
  __shared__ int s_all;
  if (*(volatile int *)&st->done) return;
  const int rpb = blockDim.x / K;
  const int bi = threadIdx.x % K, rl = threadIdx.x / K;
  double acc[2] = {0.0, 0.0};
  if (rl < rpb) {
    const T alpha = (T)cs.alpha[bi];
    for (int64_t row = (int64_t)blockIdx.x * rpb + rl; row < n; row += (int64_t)gridDim.x * rpb) {
      const int64_t o = row * K + bi;
      T xi = add_rn(x[o], mul_rn(alpha, p[o]));
      T ri = sub_rn(r[o], mul_rn(alpha, Ap[o]));
      x[o] = xi;
      r[o] = ri;
      T zi = PREC ? mul_rn(dinv[row], ri) : ri;
      acc[0] += (double)ri * (double)ri;
      acc[1] += (double)ri * (double)zi;
    }
  }
  if (!batch_last_block<2>(acc, K, smem, partials, &st->counter[2])) return;
  const long long it = st->iter + 1;
  const bool check = (it % st->check_every) == 0;
  if (threadIdx.x == 0) s_all = 1;
  __syncthreads();
  if (threadIdx.x < K) {
    const int c = threadIdx.x;
    cs.rr[c] = acc[0];
    if (check && !cs.conv[c] && acc[0] < cs.tol_sq[c]) {
      cs.conv[c] = 1;
      cs.iters[c] = it;
    }
    if (!cs.conv[c]) atomicAnd(&s_all, 0);
    double rz_old = cs.rz[c];
    cs.beta[c] = acc[1] / (rz_old + 1e-30);
    cs.rz[c] = acc[1];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    st->iter = it;
    if (check && s_all) { st->done = 1; st->iters_out = it; }
    else if (it >= st->maxiter) { st->done = 2; st->iters_out = st->maxiter; }
  }
}

static size_t mrhs_ws_bytes(size_t elem, int64_t n, int64_t K, int G) {
  return 5 * align_up(elem * (size_t)(n * K)) + 3 * align_up(2 * (size_t)K * G * sizeof(double)) +
         5 * align_up((size_t)K * sizeof(double)) + align_up((size_t)K * sizeof(long long)) +
         align_up((size_t)K * sizeof(int)) + align_up(sizeof(MrhsState));
}

template <typename T, bool PREC>
static int mrhs_impl(const int32_t *rowptr, const int32_t *colind, const T *vals, int64_t n, int K,
                     const T *dinv, const T *b, T *x, bool guess, double atol, double rtol,
                     int64_t maxiter, int64_t every, int64_t *iters_out, int32_t *conv_out,
                     void *ws, size_t ws_bytes, sla_solve_info_t *info, cudaStream_t s) {
  const int G = batch_grid(n, K);
  const int TB = batch_block(K);
  Carver c(ws, ws_bytes);
  const size_t nk = (size_t)(n * K);
  T *r = c.take<T>(nk), *pA = c.take<T>(nk), *pB = c.take<T>(nk), *Ap = c.take<T>(nk);
  c.take<T>(nk);
  double *part[3];
  for (int q = 0; q < 3; ++q) part[q] = c.take<double>(2 * (size_t)K * G);
  MrhsCols cs;
  cs.rz = c.take<double>(K); cs.alpha = c.take<double>(K); cs.beta = c.take<double>(K);
  cs.tol_sq = c.take<double>(K); cs.rr = c.take<double>(K);
  cs.iters = c.take<long long>(K);
  cs.conv = c.take<int>(K);
  MrhsState *st = c.take<MrhsState>(1);
  if (!c.ok) return SLA_ERR_WORKSPACE;
  MrhsState init{};
  init.maxiter = maxiter;
  init.check_every = every;
  SLA_CUDA_TRY(cudaMemcpyAsync(st, &init, sizeof(init), cudaMemcpyHostToDevice, s));
  SLA_LAUNCH((mrhs_init_kernel<T, PREC>), G, TB, 0, s, rowptr, colind, vals, n, K, b, x,
             guess ? 1 : 0, dinv, r, pA, st, cs, part[0], atol, rtol);
  if (!guess) SLA_LAUNCH(zero_kernel<T>, grid_for((int64_t)nk), kBlock, 0, s, x, (int64_t)nk);
  SLA_TRY(run_chunked(maxiter, 8, &st->done, s, [&](int64_t it) -> int {
    T *p_old = (it & 1) ? pB : pA, *p_new = (it & 1) ? pA : pB;
    cudaEvent_t ev;
    profiler().begin(0, it, s, &ev);
    SLA_LAUNCH((mrhs_spmv_kernel<T, PREC>), G, TB, 0, s, rowptr, colind, vals, n, K, r, dinv,
               p_old, p_new, Ap, st, cs, part[1]);
    profiler().end(0, s, ev);
    SLA_LAUNCH((mrhs_update_kernel<T, PREC>), G, TB, 0, s, n, K, x, r, p_new, Ap, dinv, st, cs,
               part[2]);
    return SLA_OK;
  }));
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

}  // namespace sla

using namespace sla;

extern "C" {

int sla_multi_rhs_cg_workspace(int dtype, int64_t n, int64_t k, size_t *bytes) {
  if (!bytes || n < 0 || k < 1 || k > 1024) return SLA_ERR_INVALID;
  if (dtype != SLA_F32 && dtype != SLA_F64) return SLA_ERR_INVALID;
  *bytes = mrhs_ws_bytes(dtype == SLA_F64 ? 8 : 4, n, k, batch_grid(n, (int)k));
  return SLA_OK;
}

int sla_multi_rhs_cg(int dtype, const int32_t *rowptr, const int32_t *colind, const void *vals,
                     int64_t n, int64_t k, const void *dinv, const void *b, void *x,
                     int x_is_guess, double atol, double rtol, int64_t maxiter,
                     int64_t check_every, int64_t *iters_out, int32_t *converged_out,
                     void *workspace, size_t workspace_bytes, sla_solve_info_t *info,
                     sla_stream_t stream) {
  if (!rowptr || !colind || !vals || !b || !x || !info || n <= 0 || n >= INT32_MAX)
    return SLA_ERR_INVALID;
  if (k < 1 || check_every < 1) return SLA_ERR_INVALID;
  if (k > 1024) return SLA_ERR_UNSUPPORTED;
  info->iterations = 0; info->residual = 0; info->status = 0; info->reason = 0;
  size_t need = 0;
  SLA_TRY(sla_multi_rhs_cg_workspace(dtype, n, k, &need));
  if (workspace_bytes < need || !workspace) return SLA_ERR_WORKSPACE;
  cudaStream_t s = (cudaStream_t)stream;
  const bool g = x_is_guess != 0;
  const int K = (int)k;
  if (dtype == SLA_F64) {
    if (dinv)
      return mrhs_impl<double, true>(rowptr, colind, (const double *)vals, n, K,
                                     (const double *)dinv, (const double *)b, (double *)x, g,
                                     atol, rtol, maxiter, check_every, iters_out, converged_out,
                                     workspace, workspace_bytes, info, s);
    return mrhs_impl<double, false>(rowptr, colind, (const double *)vals, n, K, nullptr,
                                    (const double *)b, (double *)x, g, atol, rtol, maxiter,
                                    check_every, iters_out, converged_out, workspace,
                                    workspace_bytes, info, s);
  }
  if (dtype == SLA_F32) {
    if (dinv)
      return mrhs_impl<float, true>(rowptr, colind, (const float *)vals, n, K, (const float *)dinv,
                                    (const float *)b, (float *)x, g, atol, rtol, maxiter,
                                    check_every, iters_out, converged_out, workspace,
                                    workspace_bytes, info, s);
    return mrhs_impl<float, false>(rowptr, colind, (const float *)vals, n, K, nullptr,
                                   (const float *)b, (float *)x, g, atol, rtol, maxiter,
                                   check_every, iters_out, converged_out, workspace,
                                   workspace_bytes, info, s);
  }
  return SLA_ERR_INVALID;
}

}  // extern "C"
