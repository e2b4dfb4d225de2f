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
#include <type_traits>

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
  double *rz, *alpha, *beta, *tol, *rr, *alpha_prev;
};

// Row access of the batched kernels: CSR with [nnz][B] values, or a
// diagonal-offset view of a stencil pattern with values [slot entry][B] in
// the view's order (column = row + offset: no column or row-pointer loads).
template <typename T>
struct CsrBatch {
  const int32_t *rowptr, *colind;
  const T *vals;
  template <int VEC, int RB, typename G>
  __device__ __forceinline__ void sum(int64_t row, int B, int m0, const G &g, T (&s)[VEC]) const {
    csr_row_vec<T, VEC, RB>(
        colind, __ldg(rowptr + row), __ldg(rowptr + row + 1),
        [&](int32_t k) { return vload<T, VEC, kLoadStream>(vals + (int64_t)k * B + m0); }, g, s);
  }
  // member bi's diagonal entry (0 when the row stores none)
  __device__ __forceinline__ T diag(int64_t row, int B, int bi) const {
    T d = T(0);
    for (int32_t k = rowptr[row]; k < rowptr[row + 1]; ++k)
      if (colind[k] == (int32_t)row) d = vals[(int64_t)k * B + bi];
    return d;
  }
};

template <typename T, int W>
struct DiagBatch {
  Sell<T> A;      // pattern: offsets and column bound (its own values unused)
  const T *vals;  // [n_slices * 32 * W][B]
  int j0;         // index of offset 0, -1 if none
  template <int VEC, int RB, typename G>
  __device__ __forceinline__ void sum(int64_t row, int B, int m0, const G &g, T (&s)[VEC]) const {
#pragma unroll
    for (int u = 0; u < VEC; ++u) s[u] = T(0);
    const int64_t e0 = (row >> 5) * 32 * W + (row & 31);
#pragma unroll
    for (int jb = 0; jb < W; jb += RB) {
      Pack<T, VEC> v[RB], x[RB];
#pragma unroll
      for (int q = 0; q < RB; ++q) {
        v[q] = splat<T, VEC>(T(0));
        x[q] = splat<T, VEC>(T(0));
        if (jb + q < W) {
          const int64_t c = row + A.off[jb + q];
          v[q] = vload<T, VEC, kLoadStream>(vals + (e0 + 32 * (jb + q)) * B + m0);
          if (c >= 0 && c < A.n_cols) x[q] = g((int32_t)c);
        }
      }
#pragma unroll
      for (int q = 0; q < RB; ++q) {
#pragma unroll
        for (int u = 0; u < VEC; ++u) s[u] = fma(v[q].v[u], x[q].v[u], s[u]);
      }
    }
  }
  __device__ __forceinline__ T diag(int64_t row, int B, int bi) const {
    if (j0 < 0) return T(0);
    return vals[((row >> 5) * 32 * W + (row & 31) + 32 * j0) * B + bi];
  }
};

template <typename T, typename M>
__global__ void __launch_bounds__(1024)
batch_init_kernel(M mat, int64_t n, int B, const T *__restrict__ b_in,
                  T *__restrict__ x, T *__restrict__ r, T *__restrict__ p_old, T *__restrict__ dinv,
                  BatchState *st, BatchScalars sc, double *partials, double atol, double rtol) {
  extern __shared__ double smem[];
  const BatchLane ln(B, 1);
  const int bi = ln.m0;
  double acc[2][1] = {{0.0}, {0.0}};
  for (int64_t row = (int64_t)blockIdx.x * ln.rpb + ln.rl; row < n;
       row += (int64_t)gridDim.x * ln.rpb) {
    const T d = mat.diag(row, B, bi);
    T di = (fabs(d) > T(0)) ? T(1) / d : T(1);
    T bv = b_in[(int64_t)bi * n + row];
    int64_t o = row * B + bi;
    dinv[o] = di;
    r[o] = bv;
    x[o] = T(0);
    p_old[o] = T(0);
    T z = mul_rn(di, bv);
    acc[0][0] += (double)bv * (double)z;
    acc[1][0] += (double)bv * (double)bv;
  }
  if (!batch_reduce<2, 1>(acc, B, smem, partials, &st->counter[0])) return;
  for (int m = threadIdx.x; m < B; m += blockDim.x) {
    sc.rz[m] = smem[m];
    double bn = fmax(sqrt(smem[B + m]), 1e-30);
    sc.tol[m] = fmax(rtol * bn, atol);
    sc.beta[m] = 0.0;
  }
  if (threadIdx.x == 0) {
    st->iter = 0;
    st->done = st->maxiter <= 0 ? 2 : 0;
    st->iters_out = 0;
  }
}

// K_A: p = p_old * beta + D^-1 r formed inside the gather, Ap = A p, writes
// p and Ap, per-member (p, Ap); the last block forms alpha.
template <typename T, int VEC, int RB, typename M>
__global__ void __launch_bounds__(VEC == 1 ? 1024 : kBatchThreads, VEC == 1 ? 1 : kBatchMinBlocks)
batch_spmv_kernel(M mat, int64_t n, int B, const T *__restrict__ r,
                  const T *__restrict__ dinv, const T *__restrict__ p_old, T *__restrict__ p_new,
                  T *__restrict__ Ap, BatchState *st, BatchScalars sc, double *partials) {
  extern __shared__ double smem[];
  if (*(volatile int *)&st->done) return;
  const BatchLane ln(B, VEC);
  T beta[VEC];
#pragma unroll
  for (int u = 0; u < VEC; ++u) beta[u] = (T)sc.beta[ln.m0 + u];
  double acc[1][VEC];
#pragma unroll
  for (int u = 0; u < VEC; ++u) acc[0][u] = 0.0;
  for (int64_t row = (int64_t)blockIdx.x * ln.rpb + ln.rl; row < n;
       row += (int64_t)gridDim.x * ln.rpb) {
    T sum[VEC];
    mat.template sum<VEC, RB>(
        row, B, ln.m0,
        [&](int32_t ci) {
          const int64_t c = (int64_t)ci * B + ln.m0;
          const Pack<T, VEC> po = vload<T, VEC, kLoadRO>(p_old + c);
          const Pack<T, VEC> d = vload<T, VEC, kLoadRO>(dinv + c);
          const Pack<T, VEC> rv = vload<T, VEC, kLoadRO>(r + c);
          Pack<T, VEC> out;
#pragma unroll
          for (int u = 0; u < VEC; ++u)
            out.v[u] = add_rn(mul_rn(po.v[u], beta[u]), mul_rn(d.v[u], rv.v[u]));
          return out;
        },
        sum);
    const int64_t o = row * B + ln.m0;
    const Pack<T, VEC> po = vload<T, VEC, kLoadRO>(p_old + o);
    const Pack<T, VEC> d = vload<T, VEC, kLoadRO>(dinv + o);
    const Pack<T, VEC> rv = vload<T, VEC, kLoadRO>(r + o);
    Pack<T, VEC> pn, ap;
#pragma unroll
    for (int u = 0; u < VEC; ++u) {
      pn.v[u] = add_rn(mul_rn(po.v[u], beta[u]), mul_rn(d.v[u], rv.v[u]));
      ap.v[u] = sum[u];
      acc[0][u] += (double)pn.v[u] * (double)sum[u];
    }
    vstore(p_new + o, pn);
    vstore(Ap + o, ap);
  }
  if (!batch_reduce<1, VEC>(acc, B, smem, partials, &st->counter[1])) return;
  for (int m = threadIdx.x; m < B; m += blockDim.x) {
    const double pap = smem[m];
    sc.alpha[m] = sc.rz[m] / (fabs(pap) > 0.0 ? pap : 1e-30);
  }
}

// K_B: r -= alpha Ap, per-member (r, r) and (r, D^-1 r); the last block
// forms beta and the all-members stop test. x is updated at odd iterations
// only, x = (x + alpha_prev p_prev) + alpha p (the same two roundings as two
// single steps) while both directions sit in the ping-pong buffers;
// batch_xflush_kernel applies a step left pending at the end.
template <typename T, int VEC>
__global__ void __launch_bounds__(VEC == 1 ? 1024 : kBatchThreads, VEC == 1 ? 1 : kBatchMinBlocks)
batch_update_kernel(int64_t n, int B, T *__restrict__ x, T *__restrict__ r, const T *__restrict__ p,
                    const T *__restrict__ p_prev, const T *__restrict__ Ap,
                    const T *__restrict__ dinv, BatchState *st, BatchScalars sc,
                    double *partials, int xu) {
  extern __shared__ double smem[];
  __shared__ int s_all;
  if (*(volatile int *)&st->done) return;
  const BatchLane ln(B, VEC);
  T alpha[VEC], alpha_prev[VEC];
#pragma unroll
  for (int u = 0; u < VEC; ++u) {
    alpha[u] = (T)sc.alpha[ln.m0 + u];
    alpha_prev[u] = (T)sc.alpha_prev[ln.m0 + u];
  }
  double acc[2][VEC];
#pragma unroll
  for (int u = 0; u < VEC; ++u) acc[0][u] = acc[1][u] = 0.0;
  for (int64_t row = (int64_t)blockIdx.x * ln.rpb + ln.rl; row < n;
       row += (int64_t)gridDim.x * ln.rpb) {
    const int64_t o = row * B + ln.m0;
    Pack<T, VEC> rv = vload<T, VEC>(r + o);
    const Pack<T, VEC> av = vload<T, VEC, kLoadStream>(Ap + o);
    const Pack<T, VEC> dv = vload<T, VEC, kLoadRO>(dinv + o);
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
      const T zi = mul_rn(dv.v[u], rv.v[u]);
      acc[0][u] += (double)rv.v[u] * (double)rv.v[u];
      acc[1][u] += (double)rv.v[u] * (double)zi;
    }
    vstore(r + o, rv);
  }
  if (!batch_reduce<2, VEC>(acc, B, smem, partials, &st->counter[2])) return;
  if (threadIdx.x == 0) s_all = 1;
  __syncthreads();
  for (int m = threadIdx.x; m < B; m += blockDim.x) {
    const double rr = smem[m], rz = smem[B + m];
    sc.rr[m] = rr;
    if (!(sqrt(rr) <= sc.tol[m])) atomicAnd(&s_all, 0);
    const double rz_old = sc.rz[m];
    sc.beta[m] = rz / (fabs(rz_old) > 0.0 ? rz_old : 1e-30);
    sc.rz[m] = rz;
    sc.alpha_prev[m] = sc.alpha[m];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const long long it = st->iter + 1;
    st->iter = it;
    if (s_all) { st->done = 1; st->iters_out = it; }
    else if (it >= st->maxiter) { st->done = 2; st->iters_out = st->maxiter; }
  }
}

// Pending x step after a last even iteration (st->iter odd).
template <typename T>
__global__ void batch_xflush_kernel(int64_t n, int B, T *__restrict__ x,
                                    const T *__restrict__ p_last, const BatchState *st,
                                    BatchScalars sc) {
  if ((st->iter & 1) == 0) return;
  int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; t < n * B; t += stride)
    x[t] = add_rn(x[t], mul_rn((T)sc.alpha_prev[t % B], p_last[t]));
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

static size_t batch_ws_bytes(size_t elem, int64_t n, int64_t B) {
  return 6 * align_up(elem * (size_t)(n * B)) +
         3 * align_up(2 * (size_t)B * batch_max_grid() * sizeof(double)) +
         6 * align_up((size_t)B * sizeof(double)) + align_up(sizeof(BatchState));
}

// Row load batch of the vectorised SpMV: one dependent round trip covers a
// row of up to RB entries (5- and 7-point stencils).

template <typename T, int VEC, typename M>
static int batched_loop(M mat, int64_t n, int B, T *xi, T *r, T *pA, T *pB, T *Ap, T *dinv,
                        BatchState *st, BatchScalars sc, double *const part[3], int64_t maxiter,
                        cudaStream_t s) {
  auto spmv = batch_spmv_kernel<T, VEC, kBatchRB, M>;
  auto upd = batch_update_kernel<T, VEC>;
  const int TB = batch_block(B, VEC);
  const size_t sm1 = batch_smem(1, TB, VEC), sm2 = batch_smem(2, TB, VEC);
  const int G1 = occupancy_grid((const void *)spmv, TB, sm1);
  const int G2 = occupancy_grid((const void *)upd, TB, sm2);
  return run_chunked(maxiter, 8, &st->done, s, [&](int64_t it) -> int {
    T *p_old = (it & 1) ? pB : pA, *p_new = (it & 1) ? pA : pB;
    cudaEvent_t ev;
    profiler().begin(0, it, s, &ev);
    SLA_LAUNCH(spmv, G1, TB, sm1, s, mat, n, B, r, dinv, p_old, p_new, Ap, st, sc, part[1]);
    profiler().end(0, s, ev);
    profiler().begin(1, it, s, &ev);
    SLA_LAUNCH(upd, G2, TB, sm2, s, n, B, xi, r, p_new, p_old, Ap, dinv, st, sc, part[2],
               (int)(it & 1));
    profiler().end(1, s, ev);
    return SLA_OK;
  });
}

template <typename T, typename M>
static int batched_impl(M mat, const T *vals, int64_t n, int B, const T *b, T *x, double atol,
                        double rtol, int64_t maxiter, void *ws, size_t ws_bytes,
                        sla_solve_info_t *info, cudaStream_t s) {
  Carver c(ws, ws_bytes);
  const size_t nb = (size_t)(n * B);
  T *r = c.take<T>(nb), *xi = c.take<T>(nb), *pA = c.take<T>(nb), *pB = c.take<T>(nb);
  T *Ap = c.take<T>(nb), *dinv = c.take<T>(nb);
  double *part[3];
  for (int k = 0; k < 3; ++k) part[k] = c.take<double>(2 * (size_t)B * batch_max_grid());
  BatchScalars sc;
  sc.rz = c.take<double>(B); sc.alpha = c.take<double>(B); sc.beta = c.take<double>(B);
  sc.tol = c.take<double>(B); sc.rr = c.take<double>(B); sc.alpha_prev = c.take<double>(B);
  BatchState *st = c.take<BatchState>(1);
  if (!c.ok) return SLA_ERR_WORKSPACE;
  BatchState init{};
  init.maxiter = maxiter;
  SLA_CUDA_TRY(cudaMemcpyAsync(st, &init, sizeof(BatchState), cudaMemcpyHostToDevice, s));
  {
    const int TB0 = batch_block(B, 1);
    const size_t sm0 = batch_smem(2, TB0, 1);
    auto init_fn = batch_init_kernel<T, M>;
    const int G0 = occupancy_grid((const void *)init_fn, TB0, sm0);
    SLA_LAUNCH(init_fn, G0, TB0, sm0, s, mat, n, B, b, xi, r, pA, dinv, st, sc, part[0], atol,
               rtol);
  }
  // 16-byte vector groups of members where B allows it (the interleaved
  // buffers are all 256-byte aligned)
  constexpr int kVec = 16 / sizeof(T);
  int rc;
  if (B % kVec == 0 && aligned16(vals))
    rc = batched_loop<T, kVec>(mat, n, B, xi, r, pA, pB, Ap, dinv, st, sc, part, maxiter, s);
  else
    rc = batched_loop<T, 1>(mat, n, B, xi, r, pA, pB, Ap, dinv, st, sc, part, maxiter, s);
  SLA_TRY(rc);
  // a last even iteration's direction sits in pB
  SLA_LAUNCH(batch_xflush_kernel<T>, grid_for(n * B), kBlock, 0, s, n, B, xi, pB, st, sc);
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

static int batched_args_ok(int dtype, int64_t n, int64_t batch, const void *b, void *x,
                           sla_solve_info_t *info, void *workspace, size_t workspace_bytes) {
  if (!b || !x || !info || n <= 0 || n >= INT32_MAX) return SLA_ERR_INVALID;
  if (dtype != SLA_F32 && dtype != SLA_F64) return SLA_ERR_INVALID;
  if (batch < 1) return SLA_ERR_INVALID;
  if (batch > kMaxBatch) return SLA_ERR_UNSUPPORTED;
  info->iterations = 0; info->residual = 0; info->status = 0; info->reason = 0;
  size_t need = 0;
  SLA_TRY(sla_batched_cg_workspace(dtype, n, batch, &need));
  if (workspace_bytes < need || !workspace) return SLA_ERR_WORKSPACE;
  return SLA_OK;
}

}  // namespace sla

using namespace sla;

extern "C" {

int sla_batched_cg_workspace(int dtype, int64_t n, int64_t batch, size_t *bytes) {
  if (!bytes || n < 0 || batch < 1 || batch > kMaxBatch) return SLA_ERR_INVALID;
  if (dtype != SLA_F32 && dtype != SLA_F64) return SLA_ERR_INVALID;
  *bytes = batch_ws_bytes(dtype == SLA_F64 ? 8 : 4, n, batch);
  return SLA_OK;
}

int sla_batched_cg(int dtype, const int32_t *rowptr, const int32_t *colind,
                   const void *vals_interleaved, int64_t n, int64_t batch, const void *b, void *x,
                   double atol, double rtol, int64_t maxiter, void *workspace,
                   size_t workspace_bytes, sla_solve_info_t *info, sla_stream_t stream) {
  if (!rowptr || !colind) return SLA_ERR_INVALID;
  SLA_TRY(batched_args_ok(dtype, n, batch, b, x, info, workspace, workspace_bytes));
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == SLA_F64) {
    const double *v = (const double *)vals_interleaved;
    return batched_impl<double>(CsrBatch<double>{rowptr, colind, v}, v, n, (int)batch,
                                (const double *)b, (double *)x, atol, rtol, maxiter, workspace,
                                workspace_bytes, info, s);
  }
  const float *v = (const float *)vals_interleaved;
  return batched_impl<float>(CsrBatch<float>{rowptr, colind, v}, v, n, (int)batch,
                             (const float *)b, (float *)x, atol, rtol, maxiter, workspace,
                             workspace_bytes, info, s);
}

int sla_batched_cg_diag(int dtype, const sla_sell_t *A, const void *vals_diag, int64_t batch,
                        const void *b, void *x, double atol, double rtol, int64_t maxiter,
                        void *workspace, size_t workspace_bytes, sla_solve_info_t *info,
                        sla_stream_t stream) {
  if (!A || A->n_diags <= 0 || A->row_ids || A->row_base) return SLA_ERR_INVALID;
  sla_sell_t pat = *A;
  if (!pat.val) pat.val = vals_diag;  // the pattern view needs no values of its own
  SLA_TRY(sell_check(&pat));
  if (!vals_diag) return SLA_ERR_INVALID;
  const int64_t n = pat.n_slots;
  if (pat.n_cols != n) return SLA_ERR_INVALID;  // square systems
  SLA_TRY(batched_args_ok(dtype, n, batch, b, x, info, workspace, workspace_bytes));
  int j0 = -1;
  for (int j = 0; j < pat.n_diags; ++j)
    if (pat.diag_offsets[j] == 0) j0 = j;
  cudaStream_t s = (cudaStream_t)stream;
  auto run = [&](auto tag, auto wtag) -> int {
    using T = decltype(tag);
    constexpr int W = decltype(wtag)::value;
    const T *v = (const T *)vals_diag;
    return batched_impl<T>(DiagBatch<T, W>{make_sell<T>(&pat), v, j0}, v, n, (int)batch,
                           (const T *)b, (T *)x, atol, rtol, maxiter, workspace, workspace_bytes,
                           info, s);
  };
  auto by_width = [&](auto tag) -> int {
    switch (pat.n_diags) {
      case 5: return run(tag, std::integral_constant<int, 5>{});
      case 7: return run(tag, std::integral_constant<int, 7>{});
      case 27: return run(tag, std::integral_constant<int, 27>{});
      default: return SLA_ERR_UNSUPPORTED;
    }
  };
  return dtype == SLA_F64 ? by_width(double(0)) : by_width(float(0));
}

}  // extern "C"
