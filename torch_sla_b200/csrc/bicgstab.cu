// Jacobi-preconditioned BiCGStab with the control flow of pbicgstab_solve
// (backends/pytorch_backend.py:1508-1596): half-step exit on ||s|| < tol,
// full-step exit on ||r|| < tol, breakdown exits on |rho| < 1e-30,
// (t,t) < 1e-30 and |omega| < 1e-30 (those report maxiter iterations, as the
// reference does after `break`).
//
// Three kernels per iteration; s = r - alpha v is never stored:
//   K1  p = r + beta q (own rows and inside the gather),
//       v = A M^{-1} p, partial (r_hat, v)          -> alpha
//   K2  t = A M^{-1} (r - alpha v) (gather),
//       partials (s,s), (t,t), (t,s)                -> exit mode / omega
//   K3  x += alpha M^{-1} p [+ omega M^{-1} s], r = s - omega t,
//       q = p - omega v for the next K1,
//       partials (r,r), (r_hat, r)                  -> convergence, next rho
// q holds the reference's (p - omega * v), rounded exactly as it rounds it;
// K3 reads p and v anyway, and storing q lets K1 gather three vectors per
// entry (r, q, dinv) instead of four. HBM per iteration: 2 x matrix + 19
// vector passes.
#include "solver.cuh"

namespace sla {

struct BicgState {
  double rho_old, rho_new, alpha, omega;
  double tol, residual;
  double ss, tt, ts;
  long long iter, maxiter, iters_out;
  int done;  // 0 running, 1 converged, 2 maxiter, 3 rho guard, 4 (t,t) guard, 5 omega guard
  int mode;  // set by K2: 0 full step, 1 half-step convergence, 2 (t,t) breakdown
  unsigned counter[4];
};

enum { bRunning = 0, bConverged = 1, bMaxiter = 2, bRho = 3, bTT = 4, bOmega = 5 };

template <typename T, bool PREC>
struct PGather {  // p_hat = M^{-1}(r + beta q), q = p - omega v
  const T *r, *q, *dinv;
  T beta;
  __device__ __forceinline__ T pval(int32_t c) const {
    return add_rn(__ldg(r + c), mul_rn(beta, __ldg(q + c)));
  }
  __device__ __forceinline__ T operator()(int32_t c) const {
    T pc = pval(c);
    return PREC ? mul_rn(__ldg(dinv + c), pc) : pc;
  }
};

template <typename T, bool PREC>
struct SGather {  // s_hat = M^{-1}(r - alpha v)
  const T *r, *v, *dinv;
  T alpha;
  __device__ __forceinline__ T sval(int32_t c) const {
    return sub_rn(__ldg(r + c), mul_rn(alpha, __ldg(v + c)));
  }
  __device__ __forceinline__ T operator()(int32_t c) const {
    T sc = sval(c);
    return PREC ? mul_rn(__ldg(dinv + c), sc) : sc;
  }
};

template <typename T>
__global__ void __launch_bounds__(kBlock)
bicg_init_kernel(int64_t n, const T *__restrict__ b, T *__restrict__ x, const T *__restrict__ Ax,
                 T *__restrict__ r, T *__restrict__ rhat, T *__restrict__ q,
                 BicgState *st, double *partials, double atol, double rtol) {
  __shared__ double smem[2 * kWarps];
  double acc[2] = {0.0, 0.0};
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; i < n; i += stride) {
    T bi = b[i];
    T ri = Ax ? sub_rn(bi, Ax[i]) : bi;
    if (!Ax) x[i] = T(0);
    r[i] = ri;
    rhat[i] = ri;
    q[i] = T(0);  // p = v = 0
    acc[0] += (double)ri * (double)ri;
    acc[1] += (double)bi * (double)bi;
  }
  if (last_block_sum<2, kBlock>(acc, partials, &st->counter[0], smem) && threadIdx.x == 0) {
    double bnorm = sqrt(acc[1]);
    if (bnorm == 0.0) bnorm = 1.0;
    st->tol = fmax(atol, rtol * bnorm);
    st->residual = sqrt(acc[0]);
    st->rho_old = 1.0;
    st->alpha = 1.0;
    st->omega = 1.0;
    st->rho_new = acc[0];  // (r_hat, r) with r_hat = r
    st->iter = 0;
    if (st->maxiter <= 0) { st->done = bMaxiter; st->iters_out = st->maxiter; }
    else if (fabs(acc[0]) < 1e-30) { st->done = bRho; st->iters_out = st->maxiter; }
    else st->done = bRunning;
  }
}

template <typename T, bool PREC, int WS>
__global__ void __launch_bounds__(kBlock, kSpmvMinBlocks)
bicg_k1(Sell<T> A, const T *__restrict__ r, const T *__restrict__ rhat, const T *__restrict__ q,
        const T *__restrict__ dinv, T *__restrict__ p_new, T *__restrict__ v_new, BicgState *st,
        double *partials) {
  __shared__ double smem[kWarps];
  if (*(volatile int *)&st->done) return;
  const double beta = (st->rho_new / st->rho_old) * (st->alpha / st->omega);
  PGather<T, PREC> g{r, q, dinv, (T)beta};
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  double acc[1] = {0.0};
  for_each_slice<WS>(A, warp, nwarps, lane, [&](int64_t s, int32_t sbase, int swidth) {
    T sum = sell_row_at<WS>(A, s, sbase, swidth, lane, g);
    const int64_t slot = s * 32 + lane;
    if (slot < A.n_slots) {
      const int64_t row = slot_row(A, slot);
      p_new[row] = g.pval((int32_t)row);
      v_new[row] = sum;
      acc[0] += (double)rhat[row] * (double)sum;
    }
  });
  if (last_block_sum<1, kBlock>(acc, partials, &st->counter[1], smem) && threadIdx.x == 0)
    st->alpha = st->rho_new / acc[0];
}

template <typename T, bool PREC, int WS>
__global__ void __launch_bounds__(kBlock, kSpmvMinBlocks)
bicg_k2(Sell<T> A, const T *__restrict__ r, const T *__restrict__ v, const T *__restrict__ dinv,
        T *__restrict__ t, BicgState *st, double *partials) {
  __shared__ double smem[3 * kWarps];
  if (*(volatile int *)&st->done) return;
  SGather<T, PREC> g{r, v, dinv, (T)st->alpha};
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  double acc[3] = {0.0, 0.0, 0.0};
  for_each_slice<WS>(A, warp, nwarps, lane, [&](int64_t s, int32_t sbase, int swidth) {
    T sum = sell_row_at<WS>(A, s, sbase, swidth, lane, g);
    const int64_t slot = s * 32 + lane;
    if (slot < A.n_slots) {
      const int64_t row = slot_row(A, slot);
      T si = g.sval((int32_t)row);
      t[row] = sum;
      acc[0] += (double)si * (double)si;
      acc[1] += (double)sum * (double)sum;
      acc[2] += (double)sum * (double)si;
    }
  });
  if (last_block_sum<3, kBlock>(acc, partials, &st->counter[2], smem) && threadIdx.x == 0) {
    st->ss = acc[0];
    st->tt = acc[1];
    st->ts = acc[2];
    if (sqrt(acc[0]) < st->tol) {
      st->mode = 1;
      st->residual = sqrt(acc[0]);
    } else if (acc[1] < 1e-30) {
      st->mode = 2;
    } else {
      st->mode = 0;
      st->omega = acc[2] / acc[1];
    }
  }
}

template <typename T> struct Vec16;
template <> struct Vec16<double> { using type = double2; static constexpr int E = 2; };
template <> struct Vec16<float> { using type = float4; static constexpr int E = 4; };
template <typename T, typename V>
__device__ __forceinline__ T &lane_of(V &v, int u) { return reinterpret_cast<T *>(&v)[u]; }

template <typename T, bool PREC, bool VEC>
__global__ void __launch_bounds__(kBlock)
bicg_k3(int64_t n, T *__restrict__ x, T *__restrict__ r, const T *__restrict__ rhat,
        const T *__restrict__ p, const T *__restrict__ v, const T *__restrict__ t,
        const T *__restrict__ dinv, T *__restrict__ q, BicgState *st, double *partials) {
  __shared__ double smem[2 * kWarps];
  if (*(volatile int *)&st->done) return;
  const int mode = st->mode;
  const T alpha = (T)st->alpha, omega = (T)st->omega;
  double acc[2] = {0.0, 0.0};
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  // one element: x += alpha M^{-1} p [+ omega M^{-1} s], r = s - omega t,
  // q = p - omega v
  auto elem = [&](T pi, T di, T &xi, T ri, T vi, T ti, T rh, T &qi, T &r_out) {
    T ph = PREC ? mul_rn(di, pi) : pi;
    xi = add_rn(xi, mul_rn(alpha, ph));
    if (mode == 0) {
      qi = sub_rn(pi, mul_rn(omega, vi));
      T si = sub_rn(ri, mul_rn(alpha, vi));
      T sh = PREC ? mul_rn(di, si) : si;
      xi = add_rn(xi, mul_rn(omega, sh));
      r_out = sub_rn(si, mul_rn(omega, ti));
      acc[0] += (double)r_out * (double)r_out;
      acc[1] += (double)rh * (double)r_out;
    }
  };
  int64_t tail = 0;
  if (VEC) {
    // 16-byte vectors (all pointers checked aligned by the launch)
    using V = typename Vec16<T>::type;
    constexpr int E = Vec16<T>::E;
    const int64_t nv = n / E;
    for (int64_t i = tid; i < nv; i += stride) {
      V pv = __ldcs((const V *)p + i), xv = ((V *)x)[i];
      V dv = pv, rv = pv, vv = pv, tv = pv, hv = pv, qv = pv, ro = pv;
      if (PREC) dv = __ldg((const V *)dinv + i);
      if (mode == 0) {
        rv = ((V *)r)[i];
        vv = __ldcs((const V *)v + i);
        tv = __ldcs((const V *)t + i);
        hv = __ldg((const V *)rhat + i);
      }
#pragma unroll
      for (int u = 0; u < E; ++u)
        elem(lane_of<T>(pv, u), lane_of<T>(dv, u), lane_of<T>(xv, u), lane_of<T>(rv, u),
             lane_of<T>(vv, u), lane_of<T>(tv, u), lane_of<T>(hv, u), lane_of<T>(qv, u),
             lane_of<T>(ro, u));
      ((V *)x)[i] = xv;
      if (mode == 0) {
        ((V *)q)[i] = qv;
        ((V *)r)[i] = ro;
      }
    }
    tail = nv * E;
  }
  for (int64_t i = tail + tid; i < n; i += stride) {
    T xi = x[i], qi = T(0), ro = T(0);
    const bool full = mode == 0;
    elem(p[i], PREC ? dinv[i] : T(0), xi, full ? r[i] : T(0), full ? v[i] : T(0),
         full ? t[i] : T(0), full ? rhat[i] : T(0), qi, ro);
    x[i] = xi;
    if (full) {
      q[i] = qi;
      r[i] = ro;
    }
  }
  if (last_block_sum<2, kBlock>(acc, partials, &st->counter[3], smem) && threadIdx.x == 0) {
    const long long it = st->iter + 1;
    st->iter = it;
    if (mode == 1) { st->done = bConverged; st->iters_out = it; return; }
    if (mode == 2) { st->done = bTT; st->iters_out = st->maxiter; return; }
    double res = sqrt(acc[0]);
    st->residual = res;
    if (res < st->tol) { st->done = bConverged; st->iters_out = it; return; }
    if (fabs(st->omega) < 1e-30) { st->done = bOmega; st->iters_out = st->maxiter; return; }
    if (it >= st->maxiter) { st->done = bMaxiter; st->iters_out = st->maxiter; return; }
    st->rho_old = st->rho_new;
    st->rho_new = acc[1];
    if (fabs(acc[1]) < 1e-30) { st->done = bRho; st->iters_out = st->maxiter; }
  }
}

static size_t bicg_ws_bytes(size_t elem, int64_t n) {
  size_t G = (size_t)solver_grid();
  return 6 * align_up(elem * (size_t)n) + 4 * align_up(4 * G * sizeof(double)) +
         align_up(sizeof(BicgState));
}

template <typename T, bool PREC, int WS>
static int bicg_impl(const sla_sell_t *Ad, const T *dinv, const T *b, T *x, bool guess,
                     double atol, double rtol, int64_t maxiter, void *ws, size_t ws_bytes,
                     sla_solve_info_t *info, cudaStream_t s) {
  Sell<T> A = make_sell<T>(Ad);
  const int64_t n = A.n_slots;
  Carver c(ws, ws_bytes);
  T *r = c.take<T>(n), *rhat = c.take<T>(n), *p = c.take<T>(n), *q = c.take<T>(n);
  T *v = c.take<T>(n), *t = c.take<T>(n);
  const int G = solver_grid();
  double *part[4];
  for (int k = 0; k < 4; ++k) part[k] = c.take<double>(4 * (size_t)G);
  BicgState *st = c.take<BicgState>(1);
  if (!c.ok) return SLA_ERR_WORKSPACE;
  BicgState init{};
  init.maxiter = maxiter;
  SLA_CUDA_TRY(cudaMemcpyAsync(st, &init, sizeof(BicgState), cudaMemcpyHostToDevice, s));
  if (guess) SLA_TRY(spmv_launch<T>(Ad, x, t, s));
  SLA_LAUNCH(bicg_init_kernel<T>, grid_for(n), kBlock, 0, s, n, b, x, guess ? t : nullptr, r, rhat,
             q, st, part[0], atol, rtol);
  const int g1 = occupancy_grid((const void *)bicg_k1<T, PREC, WS>);
  const int g2 = occupancy_grid((const void *)bicg_k2<T, PREC, WS>);
  const bool vec = aligned16(x, r, rhat, p, q, v, t) && (!PREC || aligned16(dinv));
  const int g3 = vec ? occupancy_grid((const void *)bicg_k3<T, PREC, true>)
                     : occupancy_grid((const void *)bicg_k3<T, PREC, false>);
  SLA_TRY(run_chunked(maxiter, 8, &st->done, s, [&](int64_t it) -> int {
    cudaEvent_t ev;
    profiler().begin(0, it, s, &ev);
    SLA_LAUNCH((bicg_k1<T, PREC, WS>), g1, kBlock, 0, s, A, r, rhat, q, dinv, p, v, st, part[1]);
    profiler().end(0, s, ev);
    profiler().begin(1, it, s, &ev);
    SLA_LAUNCH((bicg_k2<T, PREC, WS>), g2, kBlock, 0, s, A, r, v, dinv, t, st, part[2]);
    profiler().end(1, s, ev);
    profiler().begin(2, it, s, &ev);
    if (vec)
      SLA_LAUNCH((bicg_k3<T, PREC, true>), g3, kBlock, 0, s, n, x, r, rhat, p, v, t, dinv, q, st,
                 part[3]);
    else
      SLA_LAUNCH((bicg_k3<T, PREC, false>), g3, kBlock, 0, s, n, x, r, rhat, p, v, t, dinv, q, st,
                 part[3]);
    profiler().end(2, s, ev);
    return SLA_OK;
  }));
  BicgState out;
  SLA_CUDA_TRY(cudaMemcpyAsync(&out, st, sizeof(BicgState), cudaMemcpyDeviceToHost, s));
  SLA_CUDA_TRY(cudaStreamSynchronize(s));
  profiler().resolve();
  info->iterations = out.iters_out;
  info->residual = out.residual;
  info->reason = out.done;
  info->status = out.done == bConverged ? SLA_OK
                 : (out.done == bMaxiter ? SLA_NOT_CONVERGED : SLA_BREAKDOWN);
  return info->status;
}

}  // namespace sla

using namespace sla;

extern "C" {

int sla_bicgstab_workspace(int dtype, int64_t n, size_t *bytes) {
  if (!bytes || n < 0 || (dtype != SLA_F32 && dtype != SLA_F64)) return SLA_ERR_INVALID;
  *bytes = bicg_ws_bytes(dtype == SLA_F64 ? 8 : 4, n);
  return SLA_OK;
}

int sla_bicgstab(int dtype, const sla_sell_t *A, const void *dinv, const void *b, void *x,
                 int x_is_guess, double atol, double rtol, int64_t maxiter, void *workspace,
                 size_t workspace_bytes, sla_solve_info_t *info, sla_stream_t stream) {
  SLA_TRY(sell_check(A));
  if (!b || !x || !info || A->row_base) return SLA_ERR_INVALID;
  if (A->n_diags > 0 && A->n_cols > A->n_slots) return SLA_ERR_INVALID;  // square system
  if (A->n_slots <= 0 || A->n_slots >= INT32_MAX) return SLA_ERR_INVALID;
  info->iterations = 0; info->residual = 0; info->status = 0; info->reason = 0;
  size_t need = 0;
  SLA_TRY(sla_bicgstab_workspace(dtype, A->n_slots, &need));
  if (workspace_bytes < need || !workspace) return SLA_ERR_WORKSPACE;
  cudaStream_t s = (cudaStream_t)stream;
  bool g = x_is_guess != 0;
  const int wspec = width_spec(A);
  if (dtype == SLA_F64) {
    if (dinv)
      SLA_WS_DISPATCH(wspec, return bicg_impl<double, true, WS>(A, (const double *)dinv, (const double *)b, (double *)x, g,
                                     atol, rtol, maxiter, workspace, workspace_bytes, info, s));
    SLA_WS_DISPATCH(wspec, return bicg_impl<double, false, WS>(A, nullptr, (const double *)b, (double *)x, g, atol, rtol,
                                    maxiter, workspace, workspace_bytes, info, s));
  }
  if (dtype == SLA_F32) {
    if (dinv)
      SLA_WS_DISPATCH(wspec, return bicg_impl<float, true, WS>(A, (const float *)dinv, (const float *)b, (float *)x, g, atol,
                                    rtol, maxiter, workspace, workspace_bytes, info, s));
    SLA_WS_DISPATCH(wspec, return bicg_impl<float, false, WS>(A, nullptr, (const float *)b, (float *)x, g, atol, rtol, maxiter,
                                   workspace, workspace_bytes, info, s));
  }
  return SLA_ERR_INVALID;
}

}  // extern "C"
