// B Jacobi-PCG solves that share one sparsity pattern
// (batched_cg_same_pattern, backends/pytorch_backend.py:2575-2638).
//
// Layout: every vector and the values are batch-interleaved ([n][B] and
// [nnz][B]), so one column index serves B values and the B lanes of a row
// read contiguous memory. Thread t of a block owns batch member t % B of row
// (t / B) of the block's row group; the per-member dots are reduced in a
// fixed order (rows of the block, then blocks), so results are
// deterministic. Stops when every ||R_b|| <= max(atol, rtol*||b_b||), with
// all members iterating until then, as the reference does.
#include "batch.cuh"

namespace sla {

constexpr int kMaxBatch = 1024;

struct BatchState {
  long long iter, maxiter, iters_out;
  int done;  // 0 running, 1 all converged, 2 maxiter
  int pad;
  unsigned counter[4];
};

// Device arrays of per-member scalars live next to the state.
struct BatchScalars {
  double *rz, *alpha, *beta, *tol, *rr;
};

template <typename T>
__global__ void __launch_bounds__(1024)
batch_init_kernel(const int32_t *__restrict__ rowptr, const int32_t *__restrict__ colind,
                  const T *__restrict__ vals, int64_t n, int B, const T *__restrict__ b_in,
                  T *__restrict__ x, T *__restrict__ r, T *__restrict__ p_old, T *__restrict__ dinv,
                  BatchState *st, BatchScalars sc, double *partials, double atol, double rtol) {
  __shared__ double smem[2 * 1024];
  const int rpb = blockDim.x / B;
  const int bi = threadIdx.x % B, rl = threadIdx.x / B;
  double acc[2] = {0.0, 0.0};
  if (rl < rpb) {
    for (int64_t row = (int64_t)blockIdx.x * rpb + rl; row < n; row += (int64_t)gridDim.x * rpb) {
      T d = T(0);
      for (int32_t k = rowptr[row]; k < rowptr[row + 1]; ++k)
        if (colind[k] == (int32_t)row) d = vals[(int64_t)k * B + bi];
      T di = (fabs(d) > T(0)) ? T(1) / d : T(1);
      T bv = b_in[(int64_t)bi * n + row];
      int64_t o = row * B + bi;
      dinv[o] = di;
      r[o] = bv;
      x[o] = T(0);
      p_old[o] = T(0);
      T z = mul_rn(di, bv);
      acc[0] += (double)bv * (double)z;
      acc[1] += (double)bv * (double)bv;
    }
  }
  if (batch_last_block<2>(acc, B, smem, partials, &st->counter[0]) && threadIdx.x < B) {
    sc.rz[threadIdx.x] = acc[0];
    double bn = fmax(sqrt(acc[1]), 1e-30);
    sc.tol[threadIdx.x] = fmax(rtol * bn, atol);
    sc.beta[threadIdx.x] = 0.0;
    if (threadIdx.x == 0) {
      st->iter = 0;
      st->done = st->maxiter <= 0 ? 2 : 0;
      st->iters_out = 0;
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(1024)
batch_spmv_kernel(const int32_t *__restrict__ rowptr, const int32_t *__restrict__ colind,
                  const T *__restrict__ vals, int64_t n, int B, const T *__restrict__ r,
                  const T *__restrict__ dinv, const T *__restrict__ p_old, T *__restrict__ p_new,
                  T *__restrict__ Ap, BatchState *st, BatchScalars sc, double *partials) {
  __shared__ double smem[1024];
  if (*(volatile int *)&st->done) return;
  const int rpb = blockDim.x / B;
  const int bi = threadIdx.x % B, rl = threadIdx.x / B;
  double acc[1] = {0.0};
  if (rl < rpb) {
    const T beta = (T)sc.beta[bi];
    for (int64_t row = (int64_t)blockIdx.x * rpb + rl; row < n; row += (int64_t)gridDim.x * rpb) {
      const T sum = csr_row_batched<T>(
          colind, rowptr[row], rowptr[row + 1],
          [&](int32_t k) { return ld_stream(vals + (int64_t)k * B + bi); },
          [&](int32_t ci) {
            const int64_t c = (int64_t)ci * B + bi;
            return add_rn(mul_rn(__ldg(p_old + c), beta), mul_rn(__ldg(dinv + c), __ldg(r + c)));
          });
      const int64_t o = row * B + bi;
      T pn = add_rn(mul_rn(p_old[o], beta), mul_rn(dinv[o], r[o]));
      p_new[o] = pn;
      Ap[o] = sum;
      acc[0] += (double)pn * (double)sum;
    }
  }
  if (batch_last_block<1>(acc, B, smem, partials, &st->counter[1]) && threadIdx.x < B) {
    double pap = acc[0];
    sc.alpha[threadIdx.x] = sc.rz[threadIdx.x] / (fabs(pap) > 0.0 ? pap : 1e-30);
  }
}

template <typename T>
__global__ void __launch_bounds__(1024)
batch_update_kernel(int64_t n, int B, T *__restrict__ x, T *__restrict__ r, const T *__restrict__ p,
                    const T *__restrict__ Ap, const T *__restrict__ dinv, BatchState *st,
                    BatchScalars sc, double *partials) {
  __shared__ double smem[2 * 1024];
  __shared__ int s_all;
  if (*(volatile int *)&st->done) return;
  const int rpb = blockDim.x / B;
  const int bi = threadIdx.x % B, rl = threadIdx.x / B;
  double acc[2] = {0.0, 0.0};
  if (rl < rpb) {
    const T alpha = (T)sc.alpha[bi];
    for (int64_t row = (int64_t)blockIdx.x * rpb + rl; row < n; row += (int64_t)gridDim.x * rpb) {
      const int64_t o = row * B + bi;
      T xi = add_rn(x[o], mul_rn(alpha, p[o]));
      T ri = sub_rn(r[o], mul_rn(alpha, Ap[o]));
      x[o] = xi;
      r[o] = ri;
      T zi = mul_rn(dinv[o], ri);
      acc[0] += (double)ri * (double)ri;
      acc[1] += (double)ri * (double)zi;
    }
  }
  bool last = batch_last_block<2>(acc, B, smem, partials, &st->counter[2]);
  if (!last) return;
  if (threadIdx.x == 0) s_all = 1;
  __syncthreads();
  if (threadIdx.x < B) {
    const int b = threadIdx.x;
    sc.rr[b] = acc[0];
    if (!(sqrt(acc[0]) <= sc.tol[b])) atomicAnd(&s_all, 0);
    double rz_old = sc.rz[b];
    sc.beta[b] = acc[1] / (fabs(rz_old) > 0.0 ? rz_old : 1e-30);
    sc.rz[b] = acc[1];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const long long it = st->iter + 1;
    st->iter = it;
    if (s_all) { st->done = 1; st->iters_out = it; }
    else if (it >= st->maxiter) { st->done = 2; st->iters_out = st->maxiter; }
  }
}

template <typename T>
__global__ void batch_unpack_kernel(int64_t n, int B, const T *__restrict__ xi, T *__restrict__ xo) {
  int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; t < n * B; t += stride) {
    int64_t b = t / n, row = t - b * n;
    xo[t] = xi[row * B + b];
  }
}

static size_t batch_ws_bytes(size_t elem, int64_t n, int64_t B, int G) {
  return 6 * align_up(elem * (size_t)(n * B)) + 3 * align_up(2 * (size_t)B * G * sizeof(double)) +
         5 * align_up((size_t)B * sizeof(double)) + align_up(sizeof(BatchState));
}

template <typename T>
static int batched_impl(const int32_t *rowptr, const int32_t *colind, const T *vals, int64_t n,
                        int B, const T *b, T *x, double atol, double rtol, int64_t maxiter,
                        void *ws, size_t ws_bytes, sla_solve_info_t *info, cudaStream_t s) {
  const int G = batch_grid(n, B);
  const int TB = batch_block(B);
  Carver c(ws, ws_bytes);
  const size_t nb = (size_t)(n * B);
  T *r = c.take<T>(nb), *xi = c.take<T>(nb), *pA = c.take<T>(nb), *pB = c.take<T>(nb);
  T *Ap = c.take<T>(nb), *dinv = c.take<T>(nb);
  double *part[3];
  for (int k = 0; k < 3; ++k) part[k] = c.take<double>(2 * (size_t)B * G);
  BatchScalars sc;
  sc.rz = c.take<double>(B); sc.alpha = c.take<double>(B); sc.beta = c.take<double>(B);
  sc.tol = c.take<double>(B); sc.rr = c.take<double>(B);
  BatchState *st = c.take<BatchState>(1);
  if (!c.ok) return SLA_ERR_WORKSPACE;
  BatchState init{};
  init.maxiter = maxiter;
  SLA_CUDA_TRY(cudaMemcpyAsync(st, &init, sizeof(BatchState), cudaMemcpyHostToDevice, s));
  SLA_LAUNCH(batch_init_kernel<T>, G, TB, 0, s, rowptr, colind, vals, n, B, b, xi, r, pA, dinv, st,
             sc, part[0], atol, rtol);
  SLA_TRY(run_chunked(maxiter, 8, &st->done, s, [&](int64_t it) -> int {
    T *p_old = (it & 1) ? pB : pA, *p_new = (it & 1) ? pA : pB;
    cudaEvent_t ev;
    profiler().begin(0, it, s, &ev);
    SLA_LAUNCH(batch_spmv_kernel<T>, G, TB, 0, s, rowptr, colind, vals, n, B, r, dinv, p_old, p_new,
               Ap, st, sc, part[1]);
    profiler().end(0, s, ev);
    profiler().begin(1, it, s, &ev);
    SLA_LAUNCH(batch_update_kernel<T>, G, TB, 0, s, n, B, xi, r, p_new, Ap, dinv, st, sc, part[2]);
    profiler().end(1, s, ev);
    return SLA_OK;
  }));
  SLA_LAUNCH(batch_unpack_kernel<T>, grid_for(n * B), kBlock, 0, s, n, B, xi, x);
  BatchState out;
  SLA_CUDA_TRY(cudaMemcpyAsync(&out, st, sizeof(BatchState), cudaMemcpyDeviceToHost, s));
  std::vector<double> rr(B);
  SLA_CUDA_TRY(cudaMemcpyAsync(rr.data(), sc.rr, sizeof(double) * B, cudaMemcpyDeviceToHost, s));
  SLA_CUDA_TRY(cudaStreamSynchronize(s));
  profiler().resolve();
  double worst = 0.0;
  for (int k = 0; k < B; ++k) worst = fmax(worst, sqrt(rr[k]));
  info->iterations = out.done == 0 ? maxiter : out.iters_out;
  info->residual = worst;
  info->reason = out.done;
  info->status = out.done == 1 ? SLA_OK : SLA_NOT_CONVERGED;
  return info->status;
}

}  // namespace sla

using namespace sla;

extern "C" {

int sla_batched_cg_workspace(int dtype, int64_t n, int64_t batch, size_t *bytes) {
  if (!bytes || n < 0 || batch < 1 || batch > kMaxBatch) return SLA_ERR_INVALID;
  if (dtype != SLA_F32 && dtype != SLA_F64) return SLA_ERR_INVALID;
  *bytes = batch_ws_bytes(dtype == SLA_F64 ? 8 : 4, n, batch, batch_grid(n, (int)batch));
  return SLA_OK;
}

int sla_batched_cg(int dtype, const int32_t *rowptr, const int32_t *colind,
                   const void *vals_interleaved, int64_t n, int64_t batch, const void *b, void *x,
                   double atol, double rtol, int64_t maxiter, void *workspace,
                   size_t workspace_bytes, sla_solve_info_t *info, sla_stream_t stream) {
  if (!rowptr || !b || !x || !info || n <= 0 || n >= INT32_MAX) return SLA_ERR_INVALID;
  if (batch < 1) return SLA_ERR_INVALID;
  if (batch > kMaxBatch) return SLA_ERR_UNSUPPORTED;
  info->iterations = 0; info->residual = 0; info->status = 0; info->reason = 0;
  size_t need = 0;
  SLA_TRY(sla_batched_cg_workspace(dtype, n, batch, &need));
  if (workspace_bytes < need || !workspace) return SLA_ERR_WORKSPACE;
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == SLA_F64)
    return batched_impl<double>(rowptr, colind, (const double *)vals_interleaved, n, (int)batch,
                                (const double *)b, (double *)x, atol, rtol, maxiter, workspace,
                                workspace_bytes, info, s);
  if (dtype == SLA_F32)
    return batched_impl<float>(rowptr, colind, (const float *)vals_interleaved, n, (int)batch,
                               (const float *)b, (float *)x, atol, rtol, maxiter, workspace,
                               workspace_bytes, info, s);
  return SLA_ERR_INVALID;
}

}  // extern "C"
