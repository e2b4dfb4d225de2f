// Mixed-precision PCG: pytorch_solve's float32 + mixed_precision branch
// (backends/pytorch_backend.py:2278-2285) into pcg_solve_mixed_precision
// (:1176-1255) with MixedPrecisionMatrix (:1143-1173).
//
// The matrix (and a float32 Jacobi inverse) stay float32; x, r, p, Ap and
// every dot product and update are float64. A p is the float32 product of
// the float32 matrix and p rounded to float32, widened to float64. There is
// no start-of-iteration test: iteration i stops when ||r|| < tol after its
// r update (iterations = i + 1), and p'Ap <= 0 stops before the update
// (iterations = i, residual of the previous update).
//
// Two kernels per iteration, as in the float64 PCG:
//   K_A  p_new = p_old*beta + z(r) inside the gather (z = M r in the mode's
//        precision), Ap = (double)(A (float)p_new), write p_new and Ap,
//        partial (p_new, Ap); last block: p'Ap test, alpha
//   K_B  r -= alpha Ap, partials (r,r), (r,z(r)); x is updated at odd
//        iterations only with x = (x + alpha_prev p_prev) + alpha p (the same
//        two roundings as two single steps); last block: stop test, beta
// HBM per iteration: float32 matrix + 12 float64 vector passes (+ the
// float32 or float64 inverse diagonal twice) at the two-iteration average.
#include <type_traits>

#include "solver.cuh"

namespace sla {

struct MixState {
  double rz;
  double rr;
  double pAp;
  double alpha;
  double alpha_prev;
  double beta;
  double tol;
  long long iter;
  long long maxiter;
  long long iters_out;
  int done;  // 0 running, 1 converged, 2 maxiter, 3 non-finite, 5 p'Ap <= 0
  int pad;
  unsigned counter[4];
};

enum { kMxRunning = 0, kMxConverged = 1, kMxMaxiter = 2, kMxNonFinite = 3, kMxNotSPD = 5 };

// z = M r for the four preconditioner modes (SLA_MIXED_M_*):
//   0  (double)(float)r                   'none' applied in float32
//   1  (double)(dinv32 * (float)r)        'jacobi' applied in float32
//   2  dinv64 * r                         float64 Jacobi
//   3  r                                  float64 identity
template <int MODE>
__device__ __forceinline__ double mx_z(double r, const void *dinv, int64_t i) {
  if constexpr (MODE == 0) {
    return (double)__double2float_rn(r);
  } else if constexpr (MODE == 1) {
    return (double)__fmul_rn(__ldg((const float *)dinv + i), __double2float_rn(r));
  } else if constexpr (MODE == 2) {
    return __dmul_rn(__ldg((const double *)dinv + i), r);
  } else {
    return r;
  }
}

template <int MODE>
struct MxPGather {
  const double *r;
  const void *dinv;
  const double *p_old;
  double beta;
  // p.mul_(beta).add_(z): two roundings
  __device__ __forceinline__ double p(int32_t c) const {
    return __dadd_rn(__dmul_rn(__ldg(p_old + c), beta), mx_z<MODE>(__ldg(r + c), dinv, c));
  }
  __device__ __forceinline__ float operator()(int32_t c) const { return __double2float_rn(p(c)); }
};

struct MxRound {
  const double *x;
  __device__ __forceinline__ float operator()(int32_t c) const {
    return __double2float_rn(__ldg(x + c));
  }
};

// y = (double)(A (float)x): MixedPrecisionMatrix.matvec for the initial guess.
template <int WS>
__global__ void __launch_bounds__(kBlock, kSpmvMinBlocks)
mx_matvec_kernel(Sell<float> A, const double *__restrict__ x, double *__restrict__ y) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  MxRound g{x};
  for_each_slice<WS>(A, warp, nwarps, lane, [&](int64_t s, int32_t sbase, int swidth) {
    const float sum = sell_row_at<WS>(A, s, sbase, swidth, lane, g);
    const int64_t slot = s * 32 + lane;
    if (slot < A.n_slots) y[slot_row(A, slot)] = (double)sum;
  });
}

template <typename TB, int MODE>
__global__ void __launch_bounds__(kBlock)
mx_init_kernel(int64_t n, const TB *__restrict__ b, double *__restrict__ x,
               const double *__restrict__ Ax, const void *dinv, double *__restrict__ r,
               double *__restrict__ p_old, MixState *st, double *partials, double atol,
               double rtol) {
  __shared__ double smem[3 * kWarps];
  double acc[3] = {0.0, 0.0, 0.0};
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; i < n; i += stride) {
    const double bi = (double)b[i];
    const double ri = Ax ? __dsub_rn(bi, Ax[i]) : bi;
    if (!Ax) x[i] = 0.0;
    r[i] = ri;
    p_old[i] = 0.0;
    const double zi = mx_z<MODE>(ri, dinv, i);
    acc[0] += ri * ri;
    acc[1] += ri * zi;
    acc[2] += bi * bi;
  }
  if (last_block_sum<3, kBlock>(acc, partials, &st->counter[0], smem) && threadIdx.x == 0) {
    st->rr = acc[0];
    st->rz = acc[1];
    double bnorm = sqrt(acc[2]);
    if (bnorm == 0.0) bnorm = 1.0;
    st->tol = fmax(atol, rtol * bnorm);
    st->beta = 0.0;
    st->iter = 0;
    if (st->maxiter <= 0) { st->done = kMxMaxiter; st->iters_out = 0; }
    else st->done = kMxRunning;
  }
}

template <int MODE, int WS>
__global__ void __launch_bounds__(kBlock, kSpmvMinBlocks)
mx_spmv_kernel(Sell<float> A, const double *__restrict__ r, const void *dinv,
               const double *__restrict__ p_old, double *__restrict__ p_new,
               double *__restrict__ Ap, MixState *st, double *partials) {
  __shared__ double smem[kWarps];
  if (*(volatile int *)&st->done) return;
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  MxPGather<MODE> g{r, dinv, p_old, st->beta};
  double acc[1] = {0.0};
  for_each_slice<WS>(A, warp, nwarps, lane, [&](int64_t s, int32_t sbase, int swidth) {
    const float sum = sell_row_at<WS>(A, s, sbase, swidth, lane, g);
    const int64_t slot = s * 32 + lane;
    if (slot < A.n_slots) {
      const int64_t row = slot_row(A, slot);
      const double pn = g.p((int32_t)row);
      const double ap = (double)sum;
      p_new[row] = pn;
      Ap[row] = ap;
      acc[0] += pn * ap;
    }
  });
  if (last_block_sum<1, kBlock>(acc, partials, &st->counter[1], smem) && threadIdx.x == 0) {
    st->pAp = acc[0];
    if (acc[0] <= 0.0) {  // NaN continues, as `if pAp <= 0` does
      st->done = kMxNotSPD;
      st->iters_out = st->iter;
    } else {
      st->alpha = st->rz / acc[0];
    }
  }
}

// Split K_A (kCgSplit): a streaming pass forms p (float64) and its float32
// rounding once per row; the SpMV then gathers the float32 copy (4 bytes
// per entry instead of r, p_old and the inverse diagonal). Same values as
// the gather above: (float)p of the same float64 p.
// z = M r for two consecutive rows 2k, 2k + 1 (8- / 16-byte loads of the
// inverse diagonal); same roundings as mx_z.
template <int MODE>
__device__ __forceinline__ double2 mx_z2(double2 r, const void *dinv, int64_t k) {
  if constexpr (MODE == 0) {
    return make_double2((double)__double2float_rn(r.x), (double)__double2float_rn(r.y));
  } else if constexpr (MODE == 1) {
    const float2 d = __ldg((const float2 *)dinv + k);
    return make_double2((double)__fmul_rn(d.x, __double2float_rn(r.x)),
                        (double)__fmul_rn(d.y, __double2float_rn(r.y)));
  } else if constexpr (MODE == 2) {
    const double2 d = __ldg((const double2 *)dinv + k);
    return make_double2(__dmul_rn(d.x, r.x), __dmul_rn(d.y, r.y));
  } else {
    return r;
  }
}

// VEC: two rows per thread step with 16-byte loads of r and p_old and
// 16- / 8-byte stores of p and its float32 copy (pointers checked by the
// launch).
template <int MODE, bool VEC>
__global__ void __launch_bounds__(kBlock)
mx_pform_kernel(int64_t n, const double *__restrict__ r, const void *dinv,
                const double *__restrict__ p_old, double *__restrict__ p_new,
                float *__restrict__ p32, const MixState *st) {
  if (*(volatile const int *)&st->done) return;
  const MxPGather<MODE> g{r, dinv, p_old, st->beta};
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t tail = 0;
  if (VEC) {
    const double beta = st->beta;
    const int64_t n2 = n >> 1;
    for (int64_t k = tid; k < n2; k += stride) {
      const double2 rv = __ldcs((const double2 *)r + k), pv = __ldcs((const double2 *)p_old + k);
      const double2 z = mx_z2<MODE>(rv, dinv, k);
      const double2 out = make_double2(__dadd_rn(__dmul_rn(pv.x, beta), z.x),
                                       __dadd_rn(__dmul_rn(pv.y, beta), z.y));
      ((double2 *)p_new)[k] = out;
      ((float2 *)p32)[k] = make_float2(__double2float_rn(out.x), __double2float_rn(out.y));
    }
    tail = n2 * 2;
  }
  for (int64_t i = tail + tid; i < n; i += stride) {
    const double pv = g.p((int32_t)i);
    p_new[i] = pv;
    p32[i] = __double2float_rn(pv);
  }
}

template <int WS>
__global__ void __launch_bounds__(kBlock, kSpmvMinBlocks)
mx_spmv_split_kernel(Sell<float> A, const float *__restrict__ p32, const double *__restrict__ p,
                     double *__restrict__ Ap, MixState *st, double *partials) {
  __shared__ double smem[kWarps];
  if (*(volatile int *)&st->done) return;
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  PlainGather<float> g{p32};
  double acc[1] = {0.0};
  if constexpr (kSolverRowsX2<WS>) {
    // 7-wide views: two rows per lane (p32 8-byte aligned: workspace)
    for_each_slice_x2(A.n_slices, warp, nwarps, lane, [&](int64_t s, int hl) {
      int64_t r0, r1;
      float s0, s1;
      sell_rows_x2<WS>(A, s, hl, p32, r0, r1, s0, s1);
      if (r0 >= 0) {
        Ap[r0] = (double)s0;
        acc[0] += __ldg(p + r0) * (double)s0;
      }
      if (r1 >= 0) {
        Ap[r1] = (double)s1;
        acc[0] += __ldg(p + r1) * (double)s1;
      }
    });
  } else {
    for_each_slice<WS, true>(A, warp, nwarps, lane, [&](int64_t s, int32_t sbase, int swidth) {
      const float sum = sell_row_at<WS>(A, s, sbase, swidth, lane, g);
      const int64_t slot = s * 32 + lane;
      if (slot < A.n_slots) {
        const int64_t row = slot_row(A, slot);
        const double ap = (double)sum;
        Ap[row] = ap;
        acc[0] += __ldg(p + row) * ap;
      }
    });
  }
  if (last_block_sum<1, kBlock>(acc, partials, &st->counter[1], smem) && threadIdx.x == 0) {
    st->pAp = acc[0];
    if (acc[0] <= 0.0) {
      st->done = kMxNotSPD;
      st->iters_out = st->iter;
    } else {
      st->alpha = st->rz / acc[0];
    }
  }
}

template <int MODE>
__device__ __forceinline__ void mx_rupd(double &ri, double api, double alpha, const void *dinv,
                                        int64_t i, double (&acc)[2]) {
  ri = __dsub_rn(ri, __dmul_rn(alpha, api));
  const double zi = mx_z<MODE>(ri, dinv, i);
  acc[0] += ri * ri;
  acc[1] += ri * zi;
}

template <int MODE, bool VEC, bool XU>
__global__ void __launch_bounds__(kBlock)
mx_update_kernel(int64_t n, double *__restrict__ x, double *__restrict__ r,
                 const double *__restrict__ p, const double *__restrict__ p_prev,
                 const double *__restrict__ Ap, const void *dinv, MixState *st,
                 double *partials) {
  __shared__ double smem[2 * kWarps];
  if (*(volatile int *)&st->done) return;
  const double alpha = st->alpha;
  const double alpha_prev = st->alpha_prev;
  double acc[2] = {0.0, 0.0};
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  auto xstep = [&](double xi, double pp, double pc) {
    return __dadd_rn(__dadd_rn(xi, __dmul_rn(alpha_prev, pp)), __dmul_rn(alpha, pc));
  };
  int64_t tail = 0;
  if (VEC) {
    const int64_t n2 = n >> 1;
    for (int64_t i = tid; i < n2; i += stride) {
      double2 rv = ((double2 *)r)[i];
      const double2 av = __ldcs((const double2 *)Ap + i);
      if (XU) {
        double2 xv = ((double2 *)x)[i];
        const double2 pv = __ldcs((const double2 *)p + i), qv = __ldcs((const double2 *)p_prev + i);
        xv.x = xstep(xv.x, qv.x, pv.x);
        xv.y = xstep(xv.y, qv.y, pv.y);
        ((double2 *)x)[i] = xv;
      }
      mx_rupd<MODE>(rv.x, av.x, alpha, dinv, 2 * i, acc);
      mx_rupd<MODE>(rv.y, av.y, alpha, dinv, 2 * i + 1, acc);
      ((double2 *)r)[i] = rv;
    }
    tail = n2 * 2;
  }
  for (int64_t i = tail + tid; i < n; i += stride) {
    if (XU) x[i] = xstep(x[i], p_prev[i], p[i]);
    double ri = r[i];
    mx_rupd<MODE>(ri, Ap[i], alpha, dinv, i, acc);
    r[i] = ri;
  }
  if (last_block_sum<2, kBlock>(acc, partials, &st->counter[2], smem) && threadIdx.x == 0) {
    const long long it = st->iter + 1;
    st->iter = it;
    st->alpha_prev = st->alpha;
    st->rr = acc[0];
    st->beta = acc[1] / st->rz;
    st->rz = acc[1];
    if (sqrt(acc[0]) < st->tol) { st->done = kMxConverged; st->iters_out = it; }
    else if (!isfinite(acc[0])) { st->done = kMxNonFinite; st->iters_out = st->maxiter; }
    else if (it >= st->maxiter) { st->done = kMxMaxiter; st->iters_out = st->maxiter; }
  }
}

// The x step of a last even iteration, left pending by the deferred update
// (st->iter odd); p_last is that iteration's direction.
__global__ void __launch_bounds__(kBlock)
mx_xflush_kernel(int64_t n, double *__restrict__ x, const double *__restrict__ p_last,
                 const MixState *st) {
  if ((st->iter & 1) == 0) return;
  const double alpha = st->alpha_prev;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; i < n; i += stride) x[i] = __dadd_rn(x[i], __dmul_rn(alpha, p_last[i]));
}

static size_t mx_ws_bytes(int64_t n) {
  const size_t G = (size_t)solver_grid();
  return 4 * align_up(sizeof(double) * (size_t)n) + align_up(sizeof(float) * (size_t)n) +
         2 * align_up(4 * G * sizeof(double)) + align_up(sizeof(MixState));
}

template <int MODE>
static int mx_update_launch(bool vec, int64_t it, int64_t n, double *x, double *r,
                            const double *p_new, const double *p_old, const double *Ap,
                            const void *dinv, MixState *st, double *part, cudaStream_t s) {
  auto go = [&](auto fn) -> int {
    SLA_LAUNCH(fn, occupancy_grid((const void *)fn), kBlock, 0, s, n, x, r, p_new, p_old, Ap, dinv,
               st, part);
    return SLA_OK;
  };
  const bool odd = (it & 1) != 0;
  if (vec) return odd ? go(mx_update_kernel<MODE, true, true>) : go(mx_update_kernel<MODE, true, false>);
  return odd ? go(mx_update_kernel<MODE, false, true>) : go(mx_update_kernel<MODE, false, false>);
}

template <int MODE, int WS>
static int pcg_mixed_impl(const sla_sell_t *Ad, const void *dinv, int b_dtype, const void *b,
                          double *x, bool guess, double atol, double rtol, int64_t maxiter,
                          void *ws, size_t ws_bytes, sla_solve_info_t *info, double *pap_out,
                          cudaStream_t s) {
  Sell<float> A = make_sell<float>(Ad);
  const int64_t n = A.n_slots;
  Carver c(ws, ws_bytes);
  double *r = c.take<double>(n), *pA = c.take<double>(n), *pB = c.take<double>(n),
         *Ap = c.take<double>(n);
  float *p32 = c.take<float>(n);
  const int G = solver_grid();
  double *part0 = c.take<double>(4 * (size_t)G), *part1 = c.take<double>(4 * (size_t)G);
  MixState *st = c.take<MixState>(1);
  if (!c.ok) return SLA_ERR_WORKSPACE;
  MixState init{};
  init.maxiter = maxiter;
  SLA_CUDA_TRY(cudaMemcpyAsync(st, &init, sizeof(MixState), cudaMemcpyHostToDevice, s));
  if (guess)
    SLA_LAUNCH(mx_matvec_kernel<WS>, occupancy_grid((const void *)mx_matvec_kernel<WS>), kBlock, 0,
               s, A, x, Ap);
  if (b_dtype == SLA_F32)
    SLA_LAUNCH((mx_init_kernel<float, MODE>), grid_for(n), kBlock, 0, s, n, (const float *)b, x,
               guess ? Ap : nullptr, dinv, r, pA, st, part0, atol, rtol);
  else
    SLA_LAUNCH((mx_init_kernel<double, MODE>), grid_for(n), kBlock, 0, s, n, (const double *)b, x,
               guess ? Ap : nullptr, dinv, r, pA, st, part0, atol, rtol);
  const int grid_a = kCgSplit ? spmv_grid()
                              : occupancy_grid((const void *)mx_spmv_kernel<MODE, WS>);
  const int grid_p = occupancy_grid((const void *)mx_pform_kernel<MODE, true>);
  const bool vec = aligned16(x, r, pA, pB, Ap);
  const bool vec_p = aligned16(r, pA, pB) && aligned8(p32) &&
                     (MODE == 1 ? aligned8(dinv) : MODE == 2 ? aligned16(dinv) : true);
  SLA_TRY(run_chunked(maxiter, 8, &st->done, s, [&](int64_t it) -> int {
    double *p_old = (it & 1) ? pB : pA;
    double *p_new = (it & 1) ? pA : pB;
    cudaEvent_t ev;
    if (kCgSplit) {
      profiler().begin(2, it, s, &ev);
      if (vec_p)
        SLA_LAUNCH((mx_pform_kernel<MODE, true>), grid_p, kBlock, 0, s, n, r, dinv, p_old, p_new,
                   p32, st);
      else
        SLA_LAUNCH((mx_pform_kernel<MODE, false>), grid_p, kBlock, 0, s, n, r, dinv, p_old, p_new,
                   p32, st);
      profiler().end(2, s, ev);
      profiler().begin(0, it, s, &ev);
      SLA_LAUNCH((mx_spmv_split_kernel<WS>), grid_a, kBlock, 0, s, A, (const float *)p32,
                 (const double *)p_new, Ap, st, part0);
      profiler().end(0, s, ev);
    } else {
      profiler().begin(0, it, s, &ev);
      SLA_LAUNCH((mx_spmv_kernel<MODE, WS>), grid_a, kBlock, 0, s, A, r, dinv, p_old, p_new, Ap,
                 st, part0);
      profiler().end(0, s, ev);
    }
    profiler().begin(1, it, s, &ev);
    SLA_TRY((mx_update_launch<MODE>(vec, it, n, x, r, p_new, p_old, Ap, dinv, st, part1, s)));
    profiler().end(1, s, ev);
    return SLA_OK;
  }));
  SLA_LAUNCH(mx_xflush_kernel, grid_for(n), kBlock, 0, s, n, x, pB, st);
  MixState out;
  SLA_CUDA_TRY(cudaMemcpyAsync(&out, st, sizeof(MixState), cudaMemcpyDeviceToHost, s));
  SLA_CUDA_TRY(cudaStreamSynchronize(s));
  profiler().resolve();
  info->residual = sqrt(out.rr);
  info->reason = out.done;
  info->iterations = out.iters_out;
  if (pap_out) *pap_out = out.pAp;
  info->status = out.done == kMxConverged ? SLA_OK
                 : out.done == kMxNotSPD  ? SLA_BREAKDOWN
                                          : SLA_NOT_CONVERGED;
  return info->status;
}

}  // namespace sla

using namespace sla;

extern "C" {

int sla_pcg_mixed_workspace(int64_t n, size_t *bytes) {
  if (!bytes || n < 0) return SLA_ERR_INVALID;
  *bytes = mx_ws_bytes(n);
  return SLA_OK;
}

int sla_pcg_mixed(const sla_sell_t *A, int precond, const void *dinv, int b_dtype, const void *b,
                  double *x, int x_is_guess, double atol, double rtol, int64_t maxiter,
                  void *workspace, size_t workspace_bytes, sla_solve_info_t *info,
                  double *pap_out, sla_stream_t stream) {
  SLA_TRY(sell_check(A));
  if (!b || !x || !info || A->row_base) return SLA_ERR_INVALID;
  if (A->n_diags > 0 && A->n_cols > A->n_slots) return SLA_ERR_INVALID;  // square system
  if (A->n_slots <= 0 || A->n_slots >= INT32_MAX) return SLA_ERR_INVALID;
  if (b_dtype != SLA_F32 && b_dtype != SLA_F64) return SLA_ERR_INVALID;
  if (precond < SLA_MIXED_M_F32_NONE || precond > SLA_MIXED_M_F64_NONE) return SLA_ERR_INVALID;
  const bool wants_dinv = precond == SLA_MIXED_M_F32_JACOBI || precond == SLA_MIXED_M_F64_JACOBI;
  if (wants_dinv != (dinv != nullptr)) return SLA_ERR_INVALID;
  info->iterations = 0; info->residual = 0; info->status = 0; info->reason = 0;
  if (pap_out) *pap_out = 0.0;
  if (workspace_bytes < mx_ws_bytes(A->n_slots) || !workspace) return SLA_ERR_WORKSPACE;
  cudaStream_t s = (cudaStream_t)stream;
  const bool g = x_is_guess != 0;
  const int wspec = width_spec(A);
  auto run = [&](auto mode) -> int {
    constexpr int M = decltype(mode)::value;
    SLA_WS_DISPATCH(wspec, return pcg_mixed_impl<M, WS>(A, dinv, b_dtype, b, x, g, atol, rtol,
                                                        maxiter, workspace, workspace_bytes, info,
                                                        pap_out, s));
    return SLA_ERR_INVALID;
  };
  switch (precond) {
    case SLA_MIXED_M_F32_NONE: return run(std::integral_constant<int, 0>{});
    case SLA_MIXED_M_F32_JACOBI: return run(std::integral_constant<int, 1>{});
    case SLA_MIXED_M_F64_JACOBI: return run(std::integral_constant<int, 2>{});
    default: return run(std::integral_constant<int, 3>{});
  }
}

}  // extern "C"
