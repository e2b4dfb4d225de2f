// Row-sharded (Shard(0)) SpMV and Krylov solvers over NCCL, one process per
// GPU (distributed/matvec.py:26-93, 235-303; distributed/solve.py:279-436).
//
// Local vectors are laid out [owned | halo]. Per SpMV the owned rows that a
// neighbour needs are packed (for the solvers: the search direction computed
// on the fly, so the packed values are the ones the SpMV uses), exchanged with
// grouped ncclSend/ncclRecv on a side stream, and the interior rows (no halo
// column) run on the compute stream meanwhile; the boundary rows run after
// the halo arrives. Dot products are summed per rank by the kernels'
// last block and combined by one small ncclAllReduce per reduction point.
// Stopping decisions are computed by every kernel from the allreduced values
// (identical on all ranks), so every rank enqueues the same NCCL sequence.
#include <nccl.h>

#include <chrono>
#include <cstddef>
#include <vector>
#include <cstring>
#include <thread>

#include "solver.cuh"

namespace sla {

#define SLA_NCCL_TRY(expr)                                                          \
  do {                                                                              \
    ncclResult_t _r = (expr);                                                       \
    if (_r != ncclSuccess) {                                                        \
      fprintf(stderr, "[sla_b200] %s failed: %s\n", #expr, ncclGetErrorString(_r)); \
      return SLA_ERR_NCCL;                                                          \
    }                                                                               \
  } while (0)

struct Comm {
  ncclComm_t nccl = nullptr;
  int rank = 0, nranks = 1;
  cudaStream_t side = nullptr;
  cudaEvent_t ev_ready = nullptr, ev_halo = nullptr;
};

template <typename T> inline ncclDataType_t nccl_type();
template <> inline ncclDataType_t nccl_type<double>() { return ncclFloat64; }
template <> inline ncclDataType_t nccl_type<float>() { return ncclFloat32; }

// Host-side bounded wait: a peer that stops answering turns into
// SLA_ERR_TIMEOUT (after aborting the communicator) instead of a hang.
constexpr double kWaitSeconds = 600.0;

static int wait_bounded(cudaEvent_t ev, Comm *c) {
  auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    cudaError_t e = cudaEventQuery(ev);
    if (e == cudaSuccess) return SLA_OK;
    if (e != cudaErrorNotReady) {
      fprintf(stderr, "[sla_b200] event wait failed: %s\n", cudaGetErrorString(e));
      return SLA_ERR_CUDA;
    }
    ncclResult_t async = ncclSuccess;
    if (c && c->nccl && ncclCommGetAsyncError(c->nccl, &async) == ncclSuccess &&
        async != ncclSuccess && async != ncclInProgress) {
      fprintf(stderr, "[sla_b200] NCCL async error: %s\n", ncclGetErrorString(async));
      ncclCommAbort(c->nccl);
      c->nccl = nullptr;
      return SLA_ERR_NCCL;
    }
    double dt = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (dt > kWaitSeconds) {
      fprintf(stderr, "[sla_b200] shard solve: no progress for %.0f s, aborting communicator\n", dt);
      if (c && c->nccl) { ncclCommAbort(c->nccl); c->nccl = nullptr; }
      return SLA_ERR_TIMEOUT;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

static bool plan_ok(const sla_halo_plan_t *p) {
  if (!p || p->n_owned < 0 || p->n_halo < 0 || p->n_neighbors < 0) return false;
  if (p->n_neighbors > 0 && (!p->neighbor_rank || !p->send_offset || !p->recv_offset))
    return false;
  if (p->n_neighbors > 0 && p->recv_offset[p->n_neighbors] != p->n_halo) return false;
  if (p->n_neighbors > 0 && p->send_offset[p->n_neighbors] > 0 && !p->send_index) return false;
  return true;
}

// One spec for the interior and boundary views of a shard (a uniform width
// only when both views have it). A diagonal-offset interior view keeps its
// own spec; the boundary launches then use the runtime-width walk
// (boundary_spec), boundary views are always explicit.
static int width_spec2(const sla_sell_t *a, const sla_sell_t *b) {
  if (a->n_slots == 0) return width_spec(b);
  if (width_spec(a) > kDiagSpec) return width_spec(a);
  if (b->n_slots == 0) return width_spec(a);
  int wa = width_spec(a), wb = width_spec(b);
  if (wa == wb) return wa;
  auto batches = [](int w) { return w > 0 ? -((w + kRowBatch - 1) / kRowBatch) : w; };
  int ba = batches(wa), bb = batches(wb);
  if (ba == 0 || bb == 0) return 0;
  int m = ba < bb ? ba : bb;
  return m == -3 ? -4 : m;
}

constexpr int boundary_spec(int ws) { return ws > kDiagSpec ? 0 : ws; }

static int64_t n_send(const sla_halo_plan_t *p) {
  return p->n_neighbors > 0 ? p->send_offset[p->n_neighbors] : 0;
}

// Grouped send/recv of the packed halo on the side stream, ordered after
// everything already enqueued on `s`.
template <typename T>
static int halo_enqueue(Comm *c, const sla_halo_plan_t *p, const T *sendbuf, T *recvbuf,
                        cudaStream_t s) {
  SLA_CUDA_TRY(cudaEventRecord(c->ev_ready, s));
  SLA_CUDA_TRY(cudaStreamWaitEvent(c->side, c->ev_ready, 0));
  if (p->n_neighbors > 0) {
    SLA_NCCL_TRY(ncclGroupStart());
    for (int i = 0; i < p->n_neighbors; ++i) {
      const int64_t so = p->send_offset[i], sc = p->send_offset[i + 1] - so;
      const int64_t ro = p->recv_offset[i], rc = p->recv_offset[i + 1] - ro;
      if (sc > 0)
        SLA_NCCL_TRY(ncclSend(sendbuf + so, (size_t)sc, nccl_type<T>(), p->neighbor_rank[i],
                              c->nccl, c->side));
      if (rc > 0)
        SLA_NCCL_TRY(ncclRecv(recvbuf + ro, (size_t)rc, nccl_type<T>(), p->neighbor_rank[i],
                              c->nccl, c->side));
    }
    SLA_NCCL_TRY(ncclGroupEnd());
  }
  SLA_CUDA_TRY(cudaEventRecord(c->ev_halo, c->side));
  return SLA_OK;
}

template <typename T, typename V>
__global__ void halo_pack_kernel(const int32_t *__restrict__ idx, int64_t n, V val,
                                 T *__restrict__ out, const int *stopped) {
  if (stopped && *(volatile const int *)stopped) return;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; i < n; i += stride) out[i] = val(idx[i]);
}

template <typename T>
__global__ void halo_unpack_kernel(const T *__restrict__ recv, const int32_t *__restrict__ src,
                                   int64_t n_halo, T *__restrict__ dst, const int *stopped) {
  if (stopped && *(volatile const int *)stopped) return;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; i < n_halo; i += stride) dst[i] = recv[src ? src[i] : i];
}

template <typename T>
struct LoadVal {
  const T *x;
  __device__ __forceinline__ T operator()(int32_t c) const { return x[c]; }
};

// Gather that reads owned columns through `inner` and halo columns from the
// received buffer.
template <typename T, typename Inner>
struct HaloGather {
  Inner inner;
  const T *halo;
  int32_t n_own;
  __device__ __forceinline__ T operator()(int32_t c) const {
    return c < n_own ? inner(c) : __ldg(halo + (c - n_own));
  }
};

template <typename T, typename G, int WS>
__global__ void __launch_bounds__(kBlock, kSpmvMinBlocks)
shard_spmv_rows_kernel(Sell<T> A, G g, T *__restrict__ y) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for_each_slice<WS>(A, warp, nwarps, lane, [&](int64_t s, int32_t sbase, int swidth) {
    T sum = sell_row_at<WS>(A, s, sbase, swidth, lane, g);
    int64_t slot = s * 32 + lane;
    if (slot < A.n_slots) y[slot_row(A, slot)] = sum;
  });
}

// Reverse exchange helpers: halo slot h goes to recv-order position
// halo_src[h] (identity when NULL); received contributions are added onto
// the owned rows a neighbour was sent in the forward direction.
template <typename T>
__global__ void rev_pack_kernel(const T *__restrict__ w_halo, const int32_t *__restrict__ src,
                                int64_t n_halo, T *__restrict__ out) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; i < n_halo; i += stride) out[src ? src[i] : i] = w_halo[i];
}

template <typename T>
__global__ void rev_add_kernel(const T *__restrict__ recv, const int32_t *__restrict__ idx,
                               int64_t n, T *__restrict__ w) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; i < n; i += stride) w[idx[i]] = add_rn(w[idx[i]], recv[i]);
}

// Reverse direction of halo_enqueue: send recv-order halo contributions,
// receive owned-row contributions.
template <typename T>
static int rev_halo_enqueue(Comm *c, const sla_halo_plan_t *p, const T *sendbuf, T *recvbuf,
                            cudaStream_t s) {
  SLA_CUDA_TRY(cudaEventRecord(c->ev_ready, s));
  SLA_CUDA_TRY(cudaStreamWaitEvent(c->side, c->ev_ready, 0));
  if (p->n_neighbors > 0) {
    SLA_NCCL_TRY(ncclGroupStart());
    for (int i = 0; i < p->n_neighbors; ++i) {
      const int64_t ro = p->recv_offset[i], rc = p->recv_offset[i + 1] - ro;
      const int64_t so = p->send_offset[i], sc = p->send_offset[i + 1] - so;
      if (rc > 0)
        SLA_NCCL_TRY(ncclSend(sendbuf + ro, (size_t)rc, nccl_type<T>(), p->neighbor_rank[i],
                              c->nccl, c->side));
      if (sc > 0)
        SLA_NCCL_TRY(ncclRecv(recvbuf + so, (size_t)sc, nccl_type<T>(), p->neighbor_rank[i],
                              c->nccl, c->side));
    }
    SLA_NCCL_TRY(ncclGroupEnd());
  }
  SLA_CUDA_TRY(cudaEventRecord(c->ev_halo, c->side));
  SLA_CUDA_TRY(cudaStreamWaitEvent(s, c->ev_halo, 0));
  return SLA_OK;
}

template <typename T>
static int reverse_exchange(Comm *c, const sla_halo_plan_t *p, T *w, T *sendbuf, T *recvbuf,
                            cudaStream_t s) {
  const int64_t nh = p->n_halo, no = p->n_owned;
  if (nh > 0)
    SLA_LAUNCH(rev_pack_kernel<T>, grid_for(nh), kBlock, 0, s, w + no, p->halo_src, nh, sendbuf);
  SLA_TRY(rev_halo_enqueue<T>(c, p, sendbuf, recvbuf, s));
  for (int i = 0; i < p->n_neighbors; ++i) {  // ascending neighbours, one add pass each
    const int64_t so = p->send_offset[i], sc = p->send_offset[i + 1] - so;
    if (sc > 0)
      SLA_LAUNCH(rev_add_kernel<T>, grid_for(sc), kBlock, 0, s, recvbuf + so, p->send_index + so,
                 sc, w);
  }
  return SLA_OK;
}

// ================================================================ shard CG
struct ShardState {
  int stopped;
  int pad;
  long long iters;
  long long kb_done;     // CG updates executed (x is updated at odd ones, see shard_cg_update)
  double pap_int;        // interior-rows part of the local (p, Ap)
  double part3[3];       // interior-rows parts of the local (s,s),(t,t),(t,s)
  double alpha_prev, omega_prev;
  unsigned counter[8];
};

// Reduction buffers (allreduced in place), doubles.
struct CgRed {
  double init[2];   // (r,z), (b,b)
  double pap[1];    // (p, Ap)
  double pad0;
  double loc[2][2]; // per iteration parity: (r,r), (r,z)
};

__device__ __forceinline__ double cg_rz(const CgRed *R, long long k) {
  return k == 0 ? R->init[0] : R->loc[(k - 1) & 1][1];
}

// p_new = p_old * beta + M^{-1} r  (distributed/solve.py:324-348 order)
template <typename T, bool PREC>
struct ShardP {
  const T *r, *dinv, *p_old;
  T beta;
  __device__ __forceinline__ T operator()(int32_t c) const {
    T z = PREC ? mul_rn(__ldg(dinv + c), __ldg(r + c)) : __ldg(r + c);
    return add_rn(mul_rn(__ldg(p_old + c), beta), z);
  }
};

__device__ __forceinline__ double cg_beta(const CgRed *R, long long k) {
  return k == 0 ? 0.0 : cg_rz(R, k) / cg_rz(R, k - 1);
}

// Stop test of iteration k-1 evaluated at the start of iteration k
// (the reference breaks after iteration k-1's updates, before its p update).
__device__ __forceinline__ bool cg_stop(const CgRed *R, long long k, long long every, double tol) {
  if (k == 0 || ((k - 1) % every) != 0) return false;
  return sqrt(R->loc[(k - 1) & 1][0]) < tol;
}

__device__ __forceinline__ double cg_tol(const CgRed *R, double atol, double rtol) {
  return fmax(atol, rtol * sqrt(R->init[1]));
}

template <typename T, bool PREC>
__global__ void __launch_bounds__(kBlock)
shard_cg_init(int64_t n, const T *__restrict__ b, T *__restrict__ x, const T *__restrict__ dinv,
              T *__restrict__ r, T *__restrict__ p_old, ShardState *st, CgRed *R,
              double *partials) {
  __shared__ double smem[2 * kWarps];
  double acc[2] = {0.0, 0.0};
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; i < n; i += stride) {
    T bi = b[i];
    x[i] = T(0);
    r[i] = bi;
    p_old[i] = T(0);
    T zi = PREC ? mul_rn(dinv[i], bi) : bi;
    acc[0] += (double)bi * (double)zi;
    acc[1] += (double)bi * (double)bi;
  }
  if (last_block_sum<2, kBlock>(acc, partials, &st->counter[0], smem) && threadIdx.x == 0) {
    R->init[0] = acc[0];
    R->init[1] = acc[1];
  }
}

template <typename T, bool PREC>
__global__ void shard_cg_pack(const int32_t *__restrict__ idx, int64_t n, const T *r,
                              const T *dinv, const T *p_old, T *__restrict__ out, ShardState *st,
                              const CgRed *R, long long k, long long every, double atol,
                              double rtol) {
  if (*(volatile int *)&st->stopped) return;
  if (cg_stop(R, k, every, cg_tol(R, atol, rtol))) {
    if (blockIdx.x == 0 && threadIdx.x == 0) { st->stopped = 1; st->iters = k; }
    return;
  }
  ShardP<T, PREC> p{r, dinv, p_old, (T)cg_beta(R, k)};
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; i < n; i += stride) out[i] = p(idx[i]);
}

template <typename T, bool PREC, bool HALO, int WS>
__global__ void __launch_bounds__(kBlock, kSpmvMinBlocks)
shard_cg_spmv(Sell<T> A, int32_t n_own, const T *__restrict__ r, const T *__restrict__ dinv,
              const T *__restrict__ p_old, const T *__restrict__ phalo, T *__restrict__ p_new,
              T *__restrict__ Ap, ShardState *st, CgRed *R, double *partials, long long k) {
  __shared__ double smem[kWarps];
  if (*(volatile int *)&st->stopped) return;
  ShardP<T, PREC> inner{r, dinv, p_old, (T)cg_beta(R, k)};
  HaloGather<T, ShardP<T, PREC>> g{inner, phalo, n_own};
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  double acc[1] = {0.0};
  for_each_slice<WS>(A, warp, nwarps, lane, [&](int64_t s, int32_t sbase, int swidth) {
    T sum = HALO ? sell_row_at<WS>(A, s, sbase, swidth, lane, g) : sell_row_at<WS>(A, s, sbase, swidth, lane, inner);
    int64_t slot = s * 32 + lane;
    if (slot < A.n_slots) {
      int32_t row = (int32_t)slot_row(A, slot);
      T pn = inner(row);
      p_new[row] = pn;
      Ap[row] = sum;
      acc[0] += (double)pn * (double)sum;
    }
  });
  if (last_block_sum<1, kBlock>(acc, partials, &st->counter[HALO ? 2 : 1], smem) &&
      threadIdx.x == 0) {
    if (!HALO) st->pap_int = acc[0];
    else R->pap[0] = st->pap_int + acc[0];
  }
}

// x += alpha p is applied two iterations at a time (at odd k:
// x = (x + alpha_prev p_prev) + alpha p, the same two roundings as two
// steps) while both directions sit in the ping-pong buffers; a solve whose
// last update was an even one gets the pending step from shard_cg_xflush.
template <typename T>
__device__ __forceinline__ T cg_x2(T xi, T ap, T pp, T a, T pc) {
  return add_rn(add_rn(xi, mul_rn(ap, pp)), mul_rn(a, pc));
}

template <typename T, bool PREC>
__global__ void __launch_bounds__(kBlock)
shard_cg_update(int64_t n, T *__restrict__ x, T *__restrict__ r, const T *__restrict__ p,
                const T *__restrict__ p_prev, const T *__restrict__ Ap,
                const T *__restrict__ dinv, ShardState *st, CgRed *R, double *partials,
                long long k) {
  __shared__ double smem[2 * kWarps];
  if (*(volatile int *)&st->stopped) return;
  const double alpha_d = cg_rz(R, k) / R->pap[0];
  const T alpha = (T)alpha_d, alpha_prev = (T)st->alpha_prev;
  const bool xu = (k & 1) != 0;
  double acc[2] = {0.0, 0.0};
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; i < n; i += stride) {
    // torch.addcmul(x, alpha, p, value=1) / (r, alpha, Ap, value=-1)
    if (xu) x[i] = cg_x2(x[i], alpha_prev, p_prev[i], alpha, p[i]);
    T ri = sub_rn(r[i], mul_rn(alpha, Ap[i]));
    r[i] = ri;
    T zi = PREC ? mul_rn(dinv[i], ri) : ri;
    acc[0] += (double)ri * (double)ri;
    acc[1] += (double)ri * (double)zi;
  }
  if (last_block_sum<2, kBlock>(acc, partials, &st->counter[3], smem) && threadIdx.x == 0) {
    R->loc[k & 1][0] = acc[0];
    R->loc[k & 1][1] = acc[1];
    st->alpha_prev = alpha_d;
    st->kb_done = k + 1;
  }
}

// Pending x step after a last even update (kb_done odd); p_last is its
// direction.
template <typename T>
__global__ void __launch_bounds__(kBlock)
shard_cg_xflush(int64_t n, T *__restrict__ x, const T *__restrict__ p_last,
                const ShardState *st) {
  if ((st->kb_done & 1) == 0) return;
  const T a = (T)st->alpha_prev;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; i < n; i += stride) x[i] = add_rn(x[i], mul_rn(a, p_last[i]));
}

// ========================================================== shard BiCGStab
struct BiRed {
  double init[2];   // (r,r) = (r_hat, r), (b,b)
  double rv[1];     // (r_hat, v)
  double pad0;
  double stt[3];    // (s,s), (t,t), (t,s)
  double pad1;
  double rr[2][2];  // per iteration parity: (r,r), (r_hat, r)
};

__device__ __forceinline__ double bi_rho(const BiRed *R, long long k) {
  return k == 0 ? R->init[0] : R->rr[(k - 1) & 1][1];
}

__device__ __forceinline__ double bi_tol(const BiRed *R, double atol, double rtol) {
  return fmax(atol, rtol * sqrt(R->init[1]));
}

// Full-step stop test of iteration k-1, evaluated at the start of k.
__device__ __forceinline__ bool bi_stop(const BiRed *R, long long k, long long every, double tol) {
  if (k == 0 || ((k - 1) % every) != 0) return false;
  double rn = sqrt(R->rr[(k - 1) & 1][0]);
  return rn < tol || isnan(rn);
}

// p_hat = M^{-1}(r + beta (p - omega t_prev)). torch-sla's shard_matvec
// returns a view of one cached buffer, so its v is overwritten by t before
// the next p update reads it; t_prev is that value.
template <typename T, bool PREC>
struct BiP {
  const T *r, *p, *tp, *dinv;
  T beta, omega;
  __device__ __forceinline__ T pval(int32_t c) const {
    T u = sub_rn(__ldg(p + c), mul_rn(omega, __ldg(tp + c)));
    return add_rn(__ldg(r + c), mul_rn(beta, u));
  }
  __device__ __forceinline__ T operator()(int32_t c) const {
    T pc = pval(c);
    return PREC ? mul_rn(__ldg(dinv + c), pc) : pc;
  }
};

template <typename T, bool PREC>
struct BiS {  // s_hat = M^{-1}(r - alpha v)
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

__device__ __forceinline__ double bi_beta(const BiRed *R, const ShardState *st, long long k) {
  if (k == 0) return 0.0;
  double rho_prev = k == 1 ? R->init[0] : R->rr[(k - 2) & 1][1];
  return (bi_rho(R, k) / rho_prev) * (st->alpha_prev / st->omega_prev);
}

template <typename T>
__global__ void __launch_bounds__(kBlock)
shard_bi_init(int64_t n, const T *__restrict__ b, T *__restrict__ x, T *__restrict__ r,
              T *__restrict__ rhat, T *__restrict__ p, T *__restrict__ t, ShardState *st,
              BiRed *R, double *partials) {
  __shared__ double smem[2 * kWarps];
  double acc[2] = {0.0, 0.0};
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; i < n; i += stride) {
    T bi = b[i];
    x[i] = T(0);
    r[i] = bi;
    rhat[i] = bi;
    p[i] = T(0);
    t[i] = T(0);
    acc[0] += (double)bi * (double)bi;
    acc[1] += (double)bi * (double)bi;
  }
  if (last_block_sum<2, kBlock>(acc, partials, &st->counter[0], smem) && threadIdx.x == 0) {
    R->init[0] = acc[0];
    R->init[1] = acc[1];
    st->alpha_prev = 1.0;
    st->omega_prev = 1.0;
  }
}

template <typename T, bool PREC>
__global__ void shard_bi_pack1(const int32_t *__restrict__ idx, int64_t n, BiP<T, PREC> g0,
                               T *__restrict__ out, ShardState *st, const BiRed *R, long long k,
                               long long every, double atol, double rtol) {
  if (*(volatile int *)&st->stopped) return;
  if (bi_stop(R, k, every, bi_tol(R, atol, rtol))) {
    if (blockIdx.x == 0 && threadIdx.x == 0) { st->stopped = 1; st->iters = k; }
    return;
  }
  BiP<T, PREC> g = g0;
  g.beta = (T)bi_beta(R, st, k);
  g.omega = (T)st->omega_prev;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; i < n; i += stride) out[i] = g(idx[i]);
}

template <typename T, bool PREC, bool HALO, int WS>
__global__ void __launch_bounds__(kBlock, kSpmvMinBlocks)
shard_bi_k1(Sell<T> A, int32_t n_own, BiP<T, PREC> g0, const T *__restrict__ phalo,
            const T *__restrict__ rhat, T *__restrict__ p_new, T *__restrict__ v, ShardState *st,
            BiRed *R, double *partials, long long k) {
  __shared__ double smem[kWarps];
  if (*(volatile int *)&st->stopped) return;
  BiP<T, PREC> inner = g0;
  inner.beta = (T)bi_beta(R, st, k);
  inner.omega = (T)st->omega_prev;
  HaloGather<T, BiP<T, PREC>> g{inner, phalo, n_own};
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  double acc[1] = {0.0};
  for_each_slice<WS>(A, warp, nwarps, lane, [&](int64_t s, int32_t sbase, int swidth) {
    T sum = HALO ? sell_row_at<WS>(A, s, sbase, swidth, lane, g) : sell_row_at<WS>(A, s, sbase, swidth, lane, inner);
    int64_t slot = s * 32 + lane;
    if (slot < A.n_slots) {
      int32_t row = (int32_t)slot_row(A, slot);
      p_new[row] = inner.pval(row);
      v[row] = sum;
      acc[0] += (double)rhat[row] * (double)sum;
    }
  });
  if (last_block_sum<1, kBlock>(acc, partials, &st->counter[HALO ? 2 : 1], smem) &&
      threadIdx.x == 0) {
    if (!HALO) st->pap_int = acc[0];
    else R->rv[0] = st->pap_int + acc[0];
  }
}

template <typename T, bool PREC>
__global__ void shard_bi_pack2(const int32_t *__restrict__ idx, int64_t n, BiS<T, PREC> g0,
                               T *__restrict__ out, ShardState *st, const BiRed *R, long long k) {
  if (*(volatile int *)&st->stopped) return;
  BiS<T, PREC> g = g0;
  g.alpha = (T)(bi_rho(R, k) / R->rv[0]);
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; i < n; i += stride) out[i] = g(idx[i]);
}

template <typename T, bool PREC, bool HALO, int WS>
__global__ void __launch_bounds__(kBlock, kSpmvMinBlocks)
shard_bi_k2(Sell<T> A, int32_t n_own, BiS<T, PREC> g0, const T *__restrict__ shalo,
            T *__restrict__ t, ShardState *st, BiRed *R, double *partials, long long k) {
  __shared__ double smem[3 * kWarps];
  if (*(volatile int *)&st->stopped) return;
  BiS<T, PREC> inner = g0;
  inner.alpha = (T)(bi_rho(R, k) / R->rv[0]);
  HaloGather<T, BiS<T, PREC>> g{inner, shalo, n_own};
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  double acc[3] = {0.0, 0.0, 0.0};
  for_each_slice<WS>(A, warp, nwarps, lane, [&](int64_t s, int32_t sbase, int swidth) {
    T sum = HALO ? sell_row_at<WS>(A, s, sbase, swidth, lane, g) : sell_row_at<WS>(A, s, sbase, swidth, lane, inner);
    int64_t slot = s * 32 + lane;
    if (slot < A.n_slots) {
      int32_t row = (int32_t)slot_row(A, slot);
      T si = inner.sval(row);
      t[row] = sum;
      acc[0] += (double)si * (double)si;
      acc[1] += (double)sum * (double)sum;
      acc[2] += (double)sum * (double)si;
    }
  });
  if (last_block_sum<3, kBlock>(acc, partials, &st->counter[HALO ? 4 : 3], smem) &&
      threadIdx.x == 0) {
    if (!HALO) {
      st->part3[0] = acc[0]; st->part3[1] = acc[1]; st->part3[2] = acc[2];
    } else {
      R->stt[0] = st->part3[0] + acc[0];
      R->stt[1] = st->part3[1] + acc[1];
      R->stt[2] = st->part3[2] + acc[2];
    }
  }
}

template <typename T, bool PREC>
__global__ void __launch_bounds__(kBlock)
shard_bi_k3(int64_t n, T *__restrict__ x, T *__restrict__ r, const T *__restrict__ rhat,
            const T *__restrict__ p, const T *__restrict__ v, const T *__restrict__ t,
            const T *__restrict__ dinv, ShardState *st, BiRed *R, double *partials, long long k,
            long long every, double atol, double rtol) {
  __shared__ double smem[2 * kWarps];
  if (*(volatile int *)&st->stopped) return;
  const double alpha_d = bi_rho(R, k) / R->rv[0];
  const T alpha = (T)alpha_d;
  const bool half = (k % every) == 0 && sqrt(R->stt[0]) < bi_tol(R, atol, rtol);
  const double omega_d = R->stt[2] / R->stt[1];
  const T omega = (T)omega_d;
  double acc[2] = {0.0, 0.0};
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; i < n; i += stride) {
    T ph = PREC ? mul_rn(dinv[i], p[i]) : p[i];
    T xi = add_rn(x[i], mul_rn(alpha, ph));
    if (!half) {
      T si = sub_rn(r[i], mul_rn(alpha, v[i]));
      T sh = PREC ? mul_rn(dinv[i], si) : si;
      xi = add_rn(xi, mul_rn(omega, sh));
      T ri = sub_rn(si, mul_rn(omega, t[i]));
      r[i] = ri;
      acc[0] += (double)ri * (double)ri;
      acc[1] += (double)rhat[i] * (double)ri;
    }
    x[i] = xi;
  }
  if (last_block_sum<2, kBlock>(acc, partials, &st->counter[5], smem) && threadIdx.x == 0) {
    if (half) {
      st->stopped = 1;
      st->iters = k + 1;
    } else {
      R->rr[k & 1][0] = acc[0];
      R->rr[k & 1][1] = acc[1];
      st->alpha_prev = alpha_d;
      st->omega_prev = omega_d;
    }
  }
}

// ================================================================= drivers
static size_t shard_ws_bytes(size_t elem, int64_t n_own, int64_t n_halo, int64_t n_snd) {
  size_t G = (size_t)solver_grid();
  return 6 * align_up(elem * (size_t)(n_own + 1)) + align_up(elem * (size_t)(n_snd + 1)) +
         2 * align_up(elem * (size_t)(n_halo + 1)) + 6 * align_up(4 * G * sizeof(double)) +
         align_up(sizeof(ShardState)) + align_up(sizeof(BiRed)) + align_up(sizeof(CgRed));
}

// Poll the sticky stop flag once per chunk, one chunk in flight; all ranks
// see identical flags at identical points, so they stop enqueueing together.
template <typename Body>
static int shard_loop(Comm *c, int64_t maxiter, int64_t chunk, const int *d_stopped,
                      cudaStream_t s, Body body) {
  HostPoll &hp = host_poll();
  SLA_TRY(hp.init());
  int slot = 0;
  bool pending[2] = {false, false};
  for (int64_t k = 0; k < maxiter;) {
    int64_t n = maxiter - k < chunk ? maxiter - k : chunk;
    for (int64_t j = 0; j < n; ++j) SLA_TRY(body(k + j));
    k += n;
    SLA_CUDA_TRY(cudaMemcpyAsync(hp.flags + slot, d_stopped, sizeof(int), cudaMemcpyDeviceToHost, s));
    SLA_CUDA_TRY(cudaEventRecord(hp.ev[slot], s));
    pending[slot] = true;
    int other = slot ^ 1;
    if (pending[other]) {
      SLA_TRY(wait_bounded(hp.ev[other], c));
      pending[other] = false;
      if (hp.flags[other] != 0) break;
    }
    slot = other;
  }
  return SLA_OK;
}

template <typename T, bool PREC, int WS>
static int shard_cg_impl(Comm *ch, Comm *cr, const sla_halo_plan_t *plan, const sla_sell_t *Ai,
                         const sla_sell_t *Ab, const T *dinv, const T *b, T *x, double atol,
                         double rtol, int64_t maxiter, int64_t every, void *ws, size_t ws_bytes,
                         sla_solve_info_t *info, cudaStream_t s) {
  Sell<T> AI = make_sell<T>(Ai), AB = make_sell<T>(Ab);
  const int64_t no = plan->n_owned, nh = plan->n_halo, ns = n_send(plan);
  Carver c(ws, ws_bytes);
  T *r = c.take<T>(no + 1), *pA = c.take<T>(no + 1), *pB = c.take<T>(no + 1);
  T *Ap = c.take<T>(no + 1);
  T *sendbuf = c.take<T>(ns + 1), *recvbuf = c.take<T>(nh + 1), *halo = c.take<T>(nh + 1);
  const int G = solver_grid();
  double *part[4];
  for (int q = 0; q < 4; ++q) part[q] = c.take<double>(4 * (size_t)G);
  ShardState *st = c.take<ShardState>(1);
  CgRed *R = c.take<CgRed>(1);
  if (!c.ok) return SLA_ERR_WORKSPACE;
  ShardState init{};
  SLA_CUDA_TRY(cudaMemcpyAsync(st, &init, sizeof(init), cudaMemcpyHostToDevice, s));
  SLA_CUDA_TRY(cudaMemsetAsync(R, 0, sizeof(CgRed), s));
  SLA_LAUNCH((shard_cg_init<T, PREC>), grid_for(no), kBlock, 0, s, no, b, x, dinv, r, pA, st, R,
             part[0]);
  SLA_NCCL_TRY(ncclAllReduce(R->init, R->init, 2, ncclFloat64, ncclSum, cr->nccl, s));
  const T *hsrc = plan->halo_src ? halo : recvbuf;
  const int gi = occupancy_grid((const void *)shard_cg_spmv<T, PREC, false, WS>);
  const int gb = occupancy_grid((const void *)shard_cg_spmv<T, PREC, true, boundary_spec(WS)>);
  const int gu = occupancy_grid((const void *)shard_cg_update<T, PREC>);
  SLA_TRY(shard_loop(cr, maxiter, every, &st->stopped, s, [&](int64_t k) -> int {
    T *p_old = (k & 1) ? pB : pA, *p_new = (k & 1) ? pA : pB;
    if (ns > 0)
      SLA_LAUNCH((shard_cg_pack<T, PREC>), grid_for(ns), kBlock, 0, s, plan->send_index, ns, r,
                 dinv, p_old, sendbuf, st, R, (long long)k, (long long)every, atol, rtol);
    else
      SLA_LAUNCH((shard_cg_pack<T, PREC>), 1, 32, 0, s, plan->send_index, (int64_t)0, r, dinv,
                 p_old, sendbuf, st, R, (long long)k, (long long)every, atol, rtol);
    SLA_TRY(halo_enqueue<T>(ch, plan, sendbuf, recvbuf, s));
    cudaEvent_t ev;
    profiler().begin(0, k, s, &ev);
    SLA_LAUNCH((shard_cg_spmv<T, PREC, false, WS>), gi, kBlock, 0, s, AI, (int32_t)no, r, dinv, p_old,
               hsrc, p_new, Ap, st, R, part[1], (long long)k);
    profiler().end(0, s, ev);
    SLA_CUDA_TRY(cudaStreamWaitEvent(s, ch->ev_halo, 0));
    if (plan->halo_src && nh > 0)
      SLA_LAUNCH(halo_unpack_kernel<T>, grid_for(nh), kBlock, 0, s, recvbuf, plan->halo_src, nh,
                 halo, &st->stopped);
    SLA_LAUNCH((shard_cg_spmv<T, PREC, true, boundary_spec(WS)>), gb, kBlock, 0, s, AB, (int32_t)no, r, dinv, p_old,
               hsrc, p_new, Ap, st, R, part[2], (long long)k);
    SLA_NCCL_TRY(ncclAllReduce(R->pap, R->pap, 1, ncclFloat64, ncclSum, cr->nccl, s));
    profiler().begin(1, k, s, &ev);
    SLA_LAUNCH((shard_cg_update<T, PREC>), gu, kBlock, 0, s, no, x, r, p_new, p_old, Ap, dinv, st,
               R, part[3], (long long)k);
    profiler().end(1, s, ev);
    SLA_NCCL_TRY(ncclAllReduce(R->loc[k & 1], R->loc[k & 1], 2, ncclFloat64, ncclSum, cr->nccl, s));
    return SLA_OK;
  }));
  SLA_LAUNCH(shard_cg_xflush<T>, grid_for(no), kBlock, 0, s, no, x, pB, st);
  ShardState out;
  CgRed red;
  SLA_CUDA_TRY(cudaMemcpyAsync(&out, st, sizeof(out), cudaMemcpyDeviceToHost, s));
  SLA_CUDA_TRY(cudaMemcpyAsync(&red, R, sizeof(red), cudaMemcpyDeviceToHost, s));
  cudaEvent_t done;
  SLA_CUDA_TRY(cudaEventCreateWithFlags(&done, cudaEventDisableTiming));
  SLA_CUDA_TRY(cudaEventRecord(done, s));
  int w = wait_bounded(done, cr);
  cudaEventDestroy(done);
  SLA_TRY(w);
  profiler().resolve();
  info->iterations = out.stopped ? out.iters : maxiter;
  long long last = info->iterations - 1;
  info->residual = last >= 0 ? sqrt(red.loc[last & 1][0]) : sqrt(red.init[0]);
  info->status = out.stopped ? SLA_OK : SLA_NOT_CONVERGED;
  info->reason = out.stopped;
  return info->status;
}

template <typename T, bool PREC, int WS>
static int shard_bi_impl(Comm *ch, Comm *cr, const sla_halo_plan_t *plan, const sla_sell_t *Ai,
                         const sla_sell_t *Ab, const T *dinv, const T *b, T *x, double atol,
                         double rtol, int64_t maxiter, int64_t every, void *ws, size_t ws_bytes,
                         sla_solve_info_t *info, cudaStream_t s) {
  Sell<T> AI = make_sell<T>(Ai), AB = make_sell<T>(Ab);
  const int64_t no = plan->n_owned, nh = plan->n_halo, ns = n_send(plan);
  Carver c(ws, ws_bytes);
  T *r = c.take<T>(no + 1), *rhat = c.take<T>(no + 1), *pA = c.take<T>(no + 1);
  T *pB = c.take<T>(no + 1), *v = c.take<T>(no + 1), *t = c.take<T>(no + 1);
  T *sendbuf = c.take<T>(ns + 1), *recvbuf = c.take<T>(nh + 1), *halo = c.take<T>(nh + 1);
  const int G = solver_grid();
  double *part[6];
  for (int q = 0; q < 6; ++q) part[q] = c.take<double>(4 * (size_t)G);
  ShardState *st = c.take<ShardState>(1);
  BiRed *R = c.take<BiRed>(1);
  if (!c.ok) return SLA_ERR_WORKSPACE;
  ShardState init{};
  SLA_CUDA_TRY(cudaMemcpyAsync(st, &init, sizeof(init), cudaMemcpyHostToDevice, s));
  SLA_CUDA_TRY(cudaMemsetAsync(R, 0, sizeof(BiRed), s));
  SLA_LAUNCH(shard_bi_init<T>, grid_for(no), kBlock, 0, s, no, b, x, r, rhat, pA, t, st, R,
             part[0]);
  SLA_NCCL_TRY(ncclAllReduce(R->init, R->init, 2, ncclFloat64, ncclSum, cr->nccl, s));
  const T *hsrc = plan->halo_src ? halo : recvbuf;
  const unsigned pack_grid = ns > 0 ? (unsigned)grid_for(ns) : 1u;
  const int g1i = occupancy_grid((const void *)shard_bi_k1<T, PREC, false, WS>);
  const int g1b = occupancy_grid((const void *)shard_bi_k1<T, PREC, true, boundary_spec(WS)>);
  const int g2i = occupancy_grid((const void *)shard_bi_k2<T, PREC, false, WS>);
  const int g2b = occupancy_grid((const void *)shard_bi_k2<T, PREC, true, boundary_spec(WS)>);
  const int g3 = occupancy_grid((const void *)shard_bi_k3<T, PREC>);
  SLA_TRY(shard_loop(cr, maxiter, every, &st->stopped, s, [&](int64_t k) -> int {
    T *p_old = (k & 1) ? pB : pA, *p_new = (k & 1) ? pA : pB;
    BiP<T, PREC> gp{r, p_old, t, dinv, T(0), T(1)};
    BiS<T, PREC> gs{r, v, dinv, T(0)};
    // p_hat halo, then v = A p_hat
    SLA_LAUNCH((shard_bi_pack1<T, PREC>), pack_grid, kBlock, 0, s, plan->send_index, ns, gp,
               sendbuf, st, R, (long long)k, (long long)every, atol, rtol);
    SLA_TRY(halo_enqueue<T>(ch, plan, sendbuf, recvbuf, s));
    cudaEvent_t ev;
    profiler().begin(0, k, s, &ev);
    SLA_LAUNCH((shard_bi_k1<T, PREC, false, WS>), g1i, kBlock, 0, s, AI, (int32_t)no, gp, hsrc, rhat,
               p_new, v, st, R, part[1], (long long)k);
    profiler().end(0, s, ev);
    SLA_CUDA_TRY(cudaStreamWaitEvent(s, ch->ev_halo, 0));
    if (plan->halo_src && nh > 0)
      SLA_LAUNCH(halo_unpack_kernel<T>, grid_for(nh), kBlock, 0, s, recvbuf, plan->halo_src, nh,
                 halo, &st->stopped);
    SLA_LAUNCH((shard_bi_k1<T, PREC, true, boundary_spec(WS)>), g1b, kBlock, 0, s, AB, (int32_t)no, gp, hsrc, rhat,
               p_new, v, st, R, part[2], (long long)k);
    SLA_NCCL_TRY(ncclAllReduce(R->rv, R->rv, 1, ncclFloat64, ncclSum, cr->nccl, s));
    // s_hat halo, then t = A s_hat
    SLA_LAUNCH((shard_bi_pack2<T, PREC>), pack_grid, kBlock, 0, s, plan->send_index, ns, gs,
               sendbuf, st, R, (long long)k);
    SLA_TRY(halo_enqueue<T>(ch, plan, sendbuf, recvbuf, s));
    SLA_LAUNCH((shard_bi_k2<T, PREC, false, WS>), g2i, kBlock, 0, s, AI, (int32_t)no, gs, hsrc, t, st, R,
               part[3], (long long)k);
    SLA_CUDA_TRY(cudaStreamWaitEvent(s, ch->ev_halo, 0));
    if (plan->halo_src && nh > 0)
      SLA_LAUNCH(halo_unpack_kernel<T>, grid_for(nh), kBlock, 0, s, recvbuf, plan->halo_src, nh,
                 halo, &st->stopped);
    SLA_LAUNCH((shard_bi_k2<T, PREC, true, boundary_spec(WS)>), g2b, kBlock, 0, s, AB, (int32_t)no, gs, hsrc, t, st, R,
               part[4], (long long)k);
    SLA_NCCL_TRY(ncclAllReduce(R->stt, R->stt, 3, ncclFloat64, ncclSum, cr->nccl, s));
    SLA_LAUNCH((shard_bi_k3<T, PREC>), g3, kBlock, 0, s, no, x, r, rhat, p_new, v, t, dinv, st, R,
               part[5], (long long)k, (long long)every, atol, rtol);
    SLA_NCCL_TRY(ncclAllReduce(R->rr[k & 1], R->rr[k & 1], 2, ncclFloat64, ncclSum, cr->nccl, s));
    return SLA_OK;
  }));
  ShardState out;
  BiRed red;
  SLA_CUDA_TRY(cudaMemcpyAsync(&out, st, sizeof(out), cudaMemcpyDeviceToHost, s));
  SLA_CUDA_TRY(cudaMemcpyAsync(&red, R, sizeof(red), cudaMemcpyDeviceToHost, s));
  cudaEvent_t done;
  SLA_CUDA_TRY(cudaEventCreateWithFlags(&done, cudaEventDisableTiming));
  SLA_CUDA_TRY(cudaEventRecord(done, s));
  int w = wait_bounded(done, cr);
  cudaEventDestroy(done);
  SLA_TRY(w);
  profiler().resolve();
  info->iterations = out.stopped ? out.iters : maxiter;
  long long last = info->iterations - 1;
  info->residual = last >= 0 ? sqrt(red.rr[last & 1][0]) : sqrt(red.init[0]);
  info->status = out.stopped ? SLA_OK : SLA_NOT_CONVERGED;
  info->reason = out.stopped;
  return info->status;
}


// ============================================================ peer-memory path
// Single-node path of the shard CG: halo values and dot products travel as
// stores into the other GPUs' memory (CUDA IPC mappings over NVLink /
// NVSwitch) from inside the solver kernels. An iteration is two launches:
//   K_A  stop test; send this rank's share of the neighbours' halo (the
//        search direction computed on the fly) straight into their halo
//        buffers, the last block raising an arrival sequence number;
//        interior rows; wait for the neighbours' arrivals; boundary rows;
//        (p, Ap) summed over the grid and then over the ranks in rank order
//   K_B  x / r update, (r, r) and (r, z) summed the same way.
// K_A is a cooperative launch (all blocks co-resident), so no block can
// wait on a block that has not started; every wait is bounded (wait_ns of
// the descriptor, default kWaitLimitNs on the GPU's global timer)
// and a timeout stops the solve with SLA_ERR_TIMEOUT on the host. Sequence
// numbers are (solve epoch << 32) + iteration + 1, so flags left from an
// earlier solve never satisfy a wait.
constexpr int kP2PMaxRanks = 8;
constexpr int kRedPoints = 4;  // CG: 0 init, 1 (p,Ap), 2 (r,r)/(r,z); BiCGStab: 0..3
constexpr int kRedValues = 4;
constexpr int kStopTimeout = 3;

struct P2PHeader {
  long long recv_off[kP2PMaxRanks];  // where rank q's values start in my halo; -1 none
  unsigned long long arrive[kP2PMaxRanks];
  unsigned long long red_flag[2][kRedPoints][kP2PMaxRanks];
  double red_val[2][kRedPoints][kP2PMaxRanks][kRedValues];
  unsigned send_count;
  unsigned pad[63];
};

template <typename T>
struct P2PDev {
  int world, me, n_nb, pad;
  P2PHeader *local;
  P2PHeader *hdr[kP2PMaxRanks];  // every rank's header (hdr[me] == local)
  T *dst[kP2PMaxRanks];          // per neighbour: its halo buffer + my offset there
  int nb_rank[kP2PMaxRanks];
  long long send_off[kP2PMaxRanks + 1];
  const T *halo;                 // my halo buffer (written by the neighbours)
  unsigned long long seq;        // epoch << 32
  unsigned long long wait_ns;    // bound of every wait on another GPU
};

struct P2PPlan {
  Comm *comm = nullptr;
  int world = 1, me = 0, n_nb = 0;
  int64_t n_halo = 0, n_owned = 0;
  size_t elem = 8;
  char *local = nullptr;
  int *barrier = nullptr;  // device int inside `local` for the solve-start barrier
  char *peer[kP2PMaxRanks] = {};
  int nb_rank[kP2PMaxRanks] = {};
  long long dst_off[kP2PMaxRanks] = {};
  long long send_off[kP2PMaxRanks + 1] = {};
  unsigned long long epoch = 0;
  unsigned long long wait_ns = kWaitLimitNs;
};

inline size_t p2p_halo_offset() { return align_up(sizeof(P2PHeader)); }

__device__ __forceinline__ void st_release_sys(unsigned long long *p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// Bounded wait until *p >= want (sequence numbers only grow).
__device__ __forceinline__ bool wait_seq(const unsigned long long *p, unsigned long long want,
                                         unsigned long long limit_ns) {
  if (ld_acquire_sys(p) >= want) return true;
  const unsigned long long t0 = global_ns();
  while (ld_acquire_sys(p) < want) {
    if (global_ns() - t0 > limit_ns) return false;
    __nanosleep(32);
  }
  return true;
}

// This block's share of the halo values of all neighbours, then the arrival
// signal from the last block to finish (all threads of the block call it).
template <typename T, typename PV>
__device__ __forceinline__ void p2p_send_halo(const P2PDev<T> &P, const int32_t *__restrict__ idx,
                                              const PV &pval, unsigned long long seq) {
  const long long ns = P.send_off[P.n_nb];
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < ns;
       i += (long long)gridDim.x * blockDim.x) {
    int nb = 0;
    while (i >= P.send_off[nb + 1]) ++nb;
    P.dst[nb][i - P.send_off[nb]] = pval(idx[i]);
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned t = atomicAdd(&P.local->send_count, 1u);
    if (t == gridDim.x - 1) {
      P.local->send_count = 0u;
      __threadfence_system();
      for (int nb = 0; nb < P.n_nb; ++nb) st_release_sys(&P.hdr[P.nb_rank[nb]]->arrive[P.me], seq);
    }
  }
}

// Wait until every neighbour's halo values of this iteration have landed.
template <typename T>
__device__ __forceinline__ bool p2p_wait_halo(const P2PDev<T> &P, unsigned long long seq) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  if (threadIdx.x < P.n_nb &&
      !wait_seq(&P.local->arrive[P.nb_rank[threadIdx.x]], seq, P.wait_ns))
    s_ok = 0;
  __syncthreads();
  return s_ok != 0;
}

// Sum of NV rank totals over all ranks in rank order (identical on every
// rank). Called by all threads of one block; v holds this rank's totals.
template <int NV, typename T>
__device__ __forceinline__ bool p2p_allreduce(const P2PDev<T> &P, int point, int par,
                                              unsigned long long seq, double (&v)[NV]) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  if (threadIdx.x < P.world) {
    P2PHeader *h = P.hdr[threadIdx.x];
#pragma unroll
    for (int i = 0; i < NV; ++i) h->red_val[par][point][P.me][i] = v[i];
    __threadfence_system();
    st_release_sys(&h->red_flag[par][point][P.me], seq);
    if (!wait_seq(&P.local->red_flag[par][point][threadIdx.x], seq, P.wait_ns)) s_ok = 0;
  }
  __syncthreads();
  if (!s_ok) return false;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    double t = 0.0;
    for (int q = 0; q < P.world; ++q) t += ld_l2(&P.local->red_val[par][point][q][i]);
    v[i] = t;
  }
  return true;
}

template <typename T, typename Inner>
struct HaloGatherL2 {  // halo written by other GPUs during this launch: L2 loads
  Inner inner;
  const T *halo;
  int32_t n_own;
  __device__ __forceinline__ T operator()(int32_t c) const {
    return c < n_own ? inner(c) : ld_l2(halo + (c - n_own));
  }
};

template <typename T, bool PREC>
__global__ void __launch_bounds__(kBlock)
shard_cg_p2p_init(int64_t n, const T *__restrict__ b, T *__restrict__ x, const T *__restrict__ dinv,
                  T *__restrict__ r, T *__restrict__ p_old, ShardState *st, CgRed *R,
                  double *partials, P2PDev<T> P) {
  __shared__ double smem[2 * kWarps];
  double acc[2] = {0.0, 0.0};
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; i < n; i += stride) {
    T bi = b[i];
    x[i] = T(0);
    r[i] = bi;
    p_old[i] = T(0);
    T zi = PREC ? mul_rn(dinv[i], bi) : bi;
    acc[0] += (double)bi * (double)zi;
    acc[1] += (double)bi * (double)bi;
  }
  if (!last_block_sum<2, kBlock>(acc, partials, &st->counter[0], smem)) return;
  if (!p2p_allreduce<2>(P, 0, 0, P.seq, acc)) {
    if (threadIdx.x == 0) st->stopped = kStopTimeout;
    return;
  }
  if (threadIdx.x == 0) {
    R->init[0] = acc[0];
    R->init[1] = acc[1];
  }
}

template <typename T, bool PREC, int WS>
__global__ void __launch_bounds__(kBlock, kSpmvMinBlocks)
shard_cg_p2p_spmv(Sell<T> AI, Sell<T> AB, int32_t n_own, const int32_t *__restrict__ send_index,
                  const T *__restrict__ r, const T *__restrict__ dinv, const T *__restrict__ p_old,
                  T *__restrict__ p_new, T *__restrict__ Ap, ShardState *st, CgRed *R,
                  double *partials, long long k, long long every, double atol, double rtol,
                  P2PDev<T> P) {
  constexpr int WSB = boundary_spec(WS);
  __shared__ double smem[kWarps];
  if (*(volatile int *)&st->stopped) return;
  if (cg_stop(R, k, every, cg_tol(R, atol, rtol))) {
    if (blockIdx.x == 0 && threadIdx.x == 0) { st->stopped = 1; st->iters = k; }
    return;
  }
  const unsigned long long seq = P.seq + (unsigned long long)(k + 1);
  ShardP<T, PREC> inner{r, dinv, p_old, (T)cg_beta(R, k)};
  p2p_send_halo(P, send_index, inner, seq);
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  double acc[1] = {0.0};
  auto emit = [&](const Sell<T> &A, int64_t s, T sum) {
    const int64_t slot = s * 32 + lane;
    if (slot < A.n_slots) {
      const int32_t row = (int32_t)slot_row(A, slot);
      const T pn = inner(row);
      p_new[row] = pn;
      Ap[row] = sum;
      acc[0] += (double)pn * (double)sum;
    }
  };
  for_each_slice<WS>(AI, warp, nwarps, lane, [&](int64_t s, int32_t sbase, int swidth) {
    emit(AI, s, sell_row_at<WS>(AI, s, sbase, swidth, lane, inner));
  });
  if (!p2p_wait_halo(P, seq)) {
    if (threadIdx.x == 0) st->stopped = kStopTimeout;
    return;
  }
  HaloGatherL2<T, ShardP<T, PREC>> g{inner, P.halo, n_own};
  for_each_slice<WSB>(AB, warp, nwarps, lane, [&](int64_t s, int32_t sbase, int swidth) {
    emit(AB, s, sell_row_at<WSB>(AB, s, sbase, swidth, lane, g));
  });
  if (!last_block_sum<1, kBlock>(acc, partials, &st->counter[1], smem)) return;
  if (!p2p_allreduce<1>(P, 1, (int)(k & 1), seq, acc)) {
    if (threadIdx.x == 0) st->stopped = kStopTimeout;
    return;
  }
  if (threadIdx.x == 0) R->pap[0] = acc[0];
}

template <typename T, bool PREC>
__global__ void __launch_bounds__(kBlock)
shard_cg_p2p_update(int64_t n, T *__restrict__ x, T *__restrict__ r, const T *__restrict__ p,
                    const T *__restrict__ p_prev, const T *__restrict__ Ap,
                    const T *__restrict__ dinv, ShardState *st, CgRed *R, double *partials,
                    long long k, P2PDev<T> P) {
  __shared__ double smem[2 * kWarps];
  if (*(volatile int *)&st->stopped) return;
  const double alpha_d = cg_rz(R, k) / R->pap[0];
  const T alpha = (T)alpha_d, alpha_prev = (T)st->alpha_prev;
  const bool xu = (k & 1) != 0;  // deferred x update, as in shard_cg_update
  double acc[2] = {0.0, 0.0};
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; i < n; i += stride) {
    if (xu) x[i] = cg_x2(x[i], alpha_prev, p_prev[i], alpha, p[i]);
    T ri = sub_rn(r[i], mul_rn(alpha, Ap[i]));
    r[i] = ri;
    T zi = PREC ? mul_rn(dinv[i], ri) : ri;
    acc[0] += (double)ri * (double)ri;
    acc[1] += (double)ri * (double)zi;
  }
  if (!last_block_sum<2, kBlock>(acc, partials, &st->counter[3], smem)) return;
  if (!p2p_allreduce<2>(P, 2, (int)(k & 1), P.seq + (unsigned long long)(k + 1), acc)) {
    if (threadIdx.x == 0) st->stopped = kStopTimeout;
    return;
  }
  if (threadIdx.x == 0) {
    R->loc[k & 1][0] = acc[0];
    R->loc[k & 1][1] = acc[1];
    st->alpha_prev = alpha_d;
    st->kb_done = k + 1;
  }
}

// ------------------------------------------------ peer-memory shard BiCGStab
// Same scheme as the CG: K1 (v = A p_hat) and K2 (t = A s_hat) each send
// their halo share first (arrival sequence numbers 2k+1 and 2k+2), run the
// interior rows, wait, run the boundary rows and sum their dots over the
// ranks; K3 updates x and r and sums (r,r), (r_hat,r). The halo buffer is
// reused by both SpMVs: a neighbour can only start the next send after the
// cross-rank sum that needs this rank's completed SpMV.
template <typename T>
__global__ void __launch_bounds__(kBlock)
shard_bi_p2p_init(int64_t n, const T *__restrict__ b, T *__restrict__ x, T *__restrict__ r,
                  T *__restrict__ rhat, T *__restrict__ p, T *__restrict__ t, ShardState *st,
                  BiRed *R, double *partials, P2PDev<T> P) {
  __shared__ double smem[2 * kWarps];
  double acc[2] = {0.0, 0.0};
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; i < n; i += stride) {
    T bi = b[i];
    x[i] = T(0);
    r[i] = bi;
    rhat[i] = bi;
    p[i] = T(0);
    t[i] = T(0);
    acc[0] += (double)bi * (double)bi;
    acc[1] += (double)bi * (double)bi;
  }
  if (!last_block_sum<2, kBlock>(acc, partials, &st->counter[0], smem)) return;
  if (!p2p_allreduce<2>(P, 0, 0, P.seq, acc)) {
    if (threadIdx.x == 0) st->stopped = kStopTimeout;
    return;
  }
  if (threadIdx.x == 0) {
    R->init[0] = acc[0];
    R->init[1] = acc[1];
    st->alpha_prev = 1.0;
    st->omega_prev = 1.0;
  }
}

template <typename T, bool PREC, int WS>
__global__ void __launch_bounds__(kBlock, kSpmvMinBlocks)
shard_bi_p2p_k1(Sell<T> AI, Sell<T> AB, int32_t n_own, const int32_t *__restrict__ send_index,
                BiP<T, PREC> g0, const T *__restrict__ rhat, T *__restrict__ p_new,
                T *__restrict__ v, ShardState *st, BiRed *R, double *partials, long long k,
                long long every, double atol, double rtol, P2PDev<T> P) {
  constexpr int WSB = boundary_spec(WS);
  __shared__ double smem[kWarps];
  if (*(volatile int *)&st->stopped) return;
  if (bi_stop(R, k, every, bi_tol(R, atol, rtol))) {
    if (blockIdx.x == 0 && threadIdx.x == 0) { st->stopped = 1; st->iters = k; }
    return;
  }
  BiP<T, PREC> inner = g0;
  inner.beta = (T)bi_beta(R, st, k);
  inner.omega = (T)st->omega_prev;
  const unsigned long long seq = P.seq + (unsigned long long)(2 * k + 1);
  p2p_send_halo(P, send_index, inner, seq);
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  double acc[1] = {0.0};
  auto emit = [&](const Sell<T> &A, int64_t s, T sum) {
    const int64_t slot = s * 32 + lane;
    if (slot < A.n_slots) {
      const int32_t row = (int32_t)slot_row(A, slot);
      p_new[row] = inner.pval(row);
      v[row] = sum;
      acc[0] += (double)rhat[row] * (double)sum;
    }
  };
  for_each_slice<WS>(AI, warp, nwarps, lane, [&](int64_t s, int32_t sbase, int swidth) {
    emit(AI, s, sell_row_at<WS>(AI, s, sbase, swidth, lane, inner));
  });
  if (!p2p_wait_halo(P, seq)) {
    if (threadIdx.x == 0) st->stopped = kStopTimeout;
    return;
  }
  HaloGatherL2<T, BiP<T, PREC>> g{inner, P.halo, n_own};
  for_each_slice<WSB>(AB, warp, nwarps, lane, [&](int64_t s, int32_t sbase, int swidth) {
    emit(AB, s, sell_row_at<WSB>(AB, s, sbase, swidth, lane, g));
  });
  if (!last_block_sum<1, kBlock>(acc, partials, &st->counter[1], smem)) return;
  if (!p2p_allreduce<1>(P, 1, (int)(k & 1), P.seq + (unsigned long long)(k + 1), acc)) {
    if (threadIdx.x == 0) st->stopped = kStopTimeout;
    return;
  }
  if (threadIdx.x == 0) R->rv[0] = acc[0];
}

template <typename T, bool PREC, int WS>
__global__ void __launch_bounds__(kBlock, kSpmvMinBlocks)
shard_bi_p2p_k2(Sell<T> AI, Sell<T> AB, int32_t n_own, const int32_t *__restrict__ send_index,
                BiS<T, PREC> g0, T *__restrict__ t, ShardState *st, BiRed *R, double *partials,
                long long k, P2PDev<T> P) {
  constexpr int WSB = boundary_spec(WS);
  __shared__ double smem[3 * kWarps];
  if (*(volatile int *)&st->stopped) return;
  BiS<T, PREC> inner = g0;
  inner.alpha = (T)(bi_rho(R, k) / R->rv[0]);
  const unsigned long long seq = P.seq + (unsigned long long)(2 * k + 2);
  p2p_send_halo(P, send_index, inner, seq);
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  double acc[3] = {0.0, 0.0, 0.0};
  auto emit = [&](const Sell<T> &A, int64_t s, T sum) {
    const int64_t slot = s * 32 + lane;
    if (slot < A.n_slots) {
      const int32_t row = (int32_t)slot_row(A, slot);
      const T si = inner.sval(row);
      t[row] = sum;
      acc[0] += (double)si * (double)si;
      acc[1] += (double)sum * (double)sum;
      acc[2] += (double)sum * (double)si;
    }
  };
  for_each_slice<WS>(AI, warp, nwarps, lane, [&](int64_t s, int32_t sbase, int swidth) {
    emit(AI, s, sell_row_at<WS>(AI, s, sbase, swidth, lane, inner));
  });
  if (!p2p_wait_halo(P, seq)) {
    if (threadIdx.x == 0) st->stopped = kStopTimeout;
    return;
  }
  HaloGatherL2<T, BiS<T, PREC>> g{inner, P.halo, n_own};
  for_each_slice<WSB>(AB, warp, nwarps, lane, [&](int64_t s, int32_t sbase, int swidth) {
    emit(AB, s, sell_row_at<WSB>(AB, s, sbase, swidth, lane, g));
  });
  if (!last_block_sum<3, kBlock>(acc, partials, &st->counter[3], smem)) return;
  if (!p2p_allreduce<3>(P, 2, (int)(k & 1), P.seq + (unsigned long long)(k + 1), acc)) {
    if (threadIdx.x == 0) st->stopped = kStopTimeout;
    return;
  }
  if (threadIdx.x == 0) {
    R->stt[0] = acc[0];
    R->stt[1] = acc[1];
    R->stt[2] = acc[2];
  }
}

template <typename T, bool PREC>
__global__ void __launch_bounds__(kBlock)
shard_bi_p2p_k3(int64_t n, T *__restrict__ x, T *__restrict__ r, const T *__restrict__ rhat,
                const T *__restrict__ p, const T *__restrict__ v, const T *__restrict__ t,
                const T *__restrict__ dinv, ShardState *st, BiRed *R, double *partials,
                long long k, long long every, double atol, double rtol, P2PDev<T> P) {
  __shared__ double smem[2 * kWarps];
  if (*(volatile int *)&st->stopped) return;
  const double alpha_d = bi_rho(R, k) / R->rv[0];
  const T alpha = (T)alpha_d;
  // the same allreduced (s,s) on every rank: all ranks take the same branch
  const bool half = (k % every) == 0 && sqrt(R->stt[0]) < bi_tol(R, atol, rtol);
  const double omega_d = R->stt[2] / R->stt[1];
  const T omega = (T)omega_d;
  double acc[2] = {0.0, 0.0};
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; i < n; i += stride) {
    T ph = PREC ? mul_rn(dinv[i], p[i]) : p[i];
    T xi = add_rn(x[i], mul_rn(alpha, ph));
    if (!half) {
      T si = sub_rn(r[i], mul_rn(alpha, v[i]));
      T sh = PREC ? mul_rn(dinv[i], si) : si;
      xi = add_rn(xi, mul_rn(omega, sh));
      T ri = sub_rn(si, mul_rn(omega, t[i]));
      r[i] = ri;
      acc[0] += (double)ri * (double)ri;
      acc[1] += (double)rhat[i] * (double)ri;
    }
    x[i] = xi;
  }
  if (!last_block_sum<2, kBlock>(acc, partials, &st->counter[5], smem)) return;
  if (half) {
    if (threadIdx.x == 0) { st->stopped = 1; st->iters = k + 1; }
    return;
  }
  if (!p2p_allreduce<2>(P, 3, (int)(k & 1), P.seq + (unsigned long long)(k + 1), acc)) {
    if (threadIdx.x == 0) st->stopped = kStopTimeout;
    return;
  }
  if (threadIdx.x == 0) {
    R->rr[k & 1][0] = acc[0];
    R->rr[k & 1][1] = acc[1];
    st->alpha_prev = alpha_d;
    st->omega_prev = omega_d;
  }
}

template <typename T>
static P2PDev<T> p2p_dev(const P2PPlan *pp) {
  P2PDev<T> d{};
  d.world = pp->world;
  d.me = pp->me;
  d.n_nb = pp->n_nb;
  d.local = (P2PHeader *)pp->local;
  for (int q = 0; q < pp->world; ++q) d.hdr[q] = (P2PHeader *)pp->peer[q];
  for (int i = 0; i < pp->n_nb; ++i) {
    d.nb_rank[i] = pp->nb_rank[i];
    d.dst[i] = (T *)(pp->peer[pp->nb_rank[i]] + p2p_halo_offset()) + pp->dst_off[i];
  }
  for (int i = 0; i <= pp->n_nb; ++i) d.send_off[i] = pp->send_off[i];
  d.halo = (const T *)(pp->local + p2p_halo_offset());
  d.seq = pp->epoch << 32;
  d.wait_ns = pp->wait_ns;
  return d;
}

template <typename T, bool PREC, int WS>
static int shard_cg_p2p_impl(P2PPlan *pp, const sla_halo_plan_t *plan, const sla_sell_t *Ai,
                             const sla_sell_t *Ab, const T *dinv, const T *b, T *x, double atol,
                             double rtol, int64_t maxiter, int64_t every, void *ws,
                             size_t ws_bytes, sla_solve_info_t *info, cudaStream_t s) {
  Sell<T> AI = make_sell<T>(Ai), AB = make_sell<T>(Ab);
  const int64_t no = plan->n_owned;
  Carver c(ws, ws_bytes);
  T *r = c.take<T>(no + 1), *pA = c.take<T>(no + 1), *pB = c.take<T>(no + 1);
  T *Ap = c.take<T>(no + 1);
  const int G = solver_grid();
  double *part[4];
  for (int q = 0; q < 4; ++q) part[q] = c.take<double>(4 * (size_t)G);
  ShardState *st = c.take<ShardState>(1);
  CgRed *R = c.take<CgRed>(1);
  if (!c.ok) return SLA_ERR_WORKSPACE;
  ++pp->epoch;
  P2PDev<T> P = p2p_dev<T>(pp);
  // the ranks enter the solve together (one NCCL barrier per solve), so the
  // bounded waits inside the kernels only ever cover in-step skew
  SLA_NCCL_TRY(ncclAllReduce(pp->barrier, pp->barrier, 1, ncclInt32, ncclSum, pp->comm->nccl, s));
  ShardState init{};
  SLA_CUDA_TRY(cudaMemcpyAsync(st, &init, sizeof(init), cudaMemcpyHostToDevice, s));
  SLA_CUDA_TRY(cudaMemsetAsync(R, 0, sizeof(CgRed), s));
  SLA_LAUNCH((shard_cg_p2p_init<T, PREC>), grid_for(no), kBlock, 0, s, no, b, x, dinv, r, pA, st,
             R, part[0], P);
  // co-resident grid for the kernel whose blocks wait on other GPUs
  const void *ka = (const void *)shard_cg_p2p_spmv<T, PREC, WS>;
  int per_sm = 0;
  SLA_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, ka, kBlock, 0));
  if (per_sm < 1) return SLA_ERR_UNSUPPORTED;
  int ga = per_sm * device_info().sm_count;
  if (ga > G) ga = G;
  const int gu = occupancy_grid((const void *)shard_cg_p2p_update<T, PREC>);
  const int32_t n_own = (int32_t)no;
  SLA_TRY(shard_loop(pp->comm, maxiter, every, &st->stopped, s, [&](int64_t k) -> int {
    T *p_old = (k & 1) ? pB : pA, *p_new = (k & 1) ? pA : pB;
    long long kk = (long long)k, ev_ = (long long)every;
    void *args[] = {&AI, &AB, (void *)&n_own, (void *)&plan->send_index, (void *)&r,
                    (void *)&dinv, (void *)&p_old, (void *)&p_new, (void *)&Ap, (void *)&st,
                    (void *)&R, (void *)&part[1], &kk, &ev_, (void *)&atol, (void *)&rtol, &P};
    cudaEvent_t e;
    profiler().begin(0, k, s, &e);
    SLA_CUDA_TRY(cudaLaunchCooperativeKernel(ka, dim3(ga), dim3(kBlock), args, 0, s));
    g_launches.fetch_add(1, std::memory_order_relaxed);
    profiler().end(0, s, e);
    profiler().begin(1, k, s, &e);
    SLA_LAUNCH((shard_cg_p2p_update<T, PREC>), gu, kBlock, 0, s, no, x, r, p_new, p_old, Ap, dinv,
               st, R, part[3], kk, P);
    profiler().end(1, s, e);
    return SLA_OK;
  }));
  SLA_LAUNCH(shard_cg_xflush<T>, grid_for(no), kBlock, 0, s, no, x, pB, st);
  ShardState out;
  CgRed red;
  SLA_CUDA_TRY(cudaMemcpyAsync(&out, st, sizeof(out), cudaMemcpyDeviceToHost, s));
  SLA_CUDA_TRY(cudaMemcpyAsync(&red, R, sizeof(red), cudaMemcpyDeviceToHost, s));
  cudaEvent_t done;
  SLA_CUDA_TRY(cudaEventCreateWithFlags(&done, cudaEventDisableTiming));
  SLA_CUDA_TRY(cudaEventRecord(done, s));
  int wrc = wait_bounded(done, pp->comm);
  cudaEventDestroy(done);
  SLA_TRY(wrc);
  profiler().resolve();
  if (out.stopped == kStopTimeout) {
    fprintf(stderr, "[sla_b200] shard CG: a peer did not answer within the bounded wait\n");
    return SLA_ERR_TIMEOUT;
  }
  const long long iters = out.stopped == 1 ? out.iters : maxiter;
  info->iterations = iters;
  info->residual = iters > 0 ? sqrt(red.loc[(iters - 1) & 1][0]) : sqrt(red.init[0]);
  info->reason = out.stopped;
  info->status = out.stopped == 1 ? SLA_OK : SLA_NOT_CONVERGED;
  return info->status;
}


template <typename T, bool PREC, int WS>
static int shard_bi_p2p_impl(P2PPlan *pp, const sla_halo_plan_t *plan, const sla_sell_t *Ai,
                             const sla_sell_t *Ab, const T *dinv, const T *b, T *x, double atol,
                             double rtol, int64_t maxiter, int64_t every, void *ws,
                             size_t ws_bytes, sla_solve_info_t *info, cudaStream_t s) {
  Sell<T> AI = make_sell<T>(Ai), AB = make_sell<T>(Ab);
  const int64_t no = plan->n_owned;
  Carver c(ws, ws_bytes);
  T *r = c.take<T>(no + 1), *rhat = c.take<T>(no + 1), *pA = c.take<T>(no + 1);
  T *pB = c.take<T>(no + 1), *v = c.take<T>(no + 1), *t = c.take<T>(no + 1);
  const int G = solver_grid();
  double *part[6];
  for (int q = 0; q < 6; ++q) part[q] = c.take<double>(4 * (size_t)G);
  ShardState *st = c.take<ShardState>(1);
  BiRed *R = c.take<BiRed>(1);
  if (!c.ok) return SLA_ERR_WORKSPACE;
  ++pp->epoch;
  P2PDev<T> P = p2p_dev<T>(pp);
  SLA_NCCL_TRY(ncclAllReduce(pp->barrier, pp->barrier, 1, ncclInt32, ncclSum, pp->comm->nccl, s));
  ShardState init{};
  SLA_CUDA_TRY(cudaMemcpyAsync(st, &init, sizeof(init), cudaMemcpyHostToDevice, s));
  SLA_CUDA_TRY(cudaMemsetAsync(R, 0, sizeof(BiRed), s));
  SLA_LAUNCH(shard_bi_p2p_init<T>, grid_for(no), kBlock, 0, s, no, b, x, r, rhat, pA, t, st, R,
             part[0], P);
  const void *k1 = (const void *)shard_bi_p2p_k1<T, PREC, WS>;
  const void *k2 = (const void *)shard_bi_p2p_k2<T, PREC, WS>;
  int per1 = 0, per2 = 0;
  SLA_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per1, k1, kBlock, 0));
  SLA_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per2, k2, kBlock, 0));
  if (per1 < 1 || per2 < 1) return SLA_ERR_UNSUPPORTED;
  const int sms = device_info().sm_count;
  const int g1 = per1 * sms < G ? per1 * sms : G, g2 = per2 * sms < G ? per2 * sms : G;
  const int g3 = occupancy_grid((const void *)shard_bi_p2p_k3<T, PREC>);
  const int32_t n_own = (int32_t)no;
  SLA_TRY(shard_loop(pp->comm, maxiter, every, &st->stopped, s, [&](int64_t k) -> int {
    T *p_old = (k & 1) ? pB : pA, *p_new = (k & 1) ? pA : pB;
    BiP<T, PREC> gp{r, p_old, t, dinv, T(0), T(1)};
    BiS<T, PREC> gs{r, v, dinv, T(0)};
    long long kk = (long long)k, ev_ = (long long)every;
    void *a1[] = {&AI, &AB, (void *)&n_own, (void *)&plan->send_index, &gp, (void *)&rhat,
                  (void *)&p_new, (void *)&v, (void *)&st, (void *)&R, (void *)&part[1], &kk,
                  &ev_, (void *)&atol, (void *)&rtol, &P};
    cudaEvent_t e;
    profiler().begin(0, k, s, &e);
    SLA_CUDA_TRY(cudaLaunchCooperativeKernel(k1, dim3(g1), dim3(kBlock), a1, 0, s));
    g_launches.fetch_add(1, std::memory_order_relaxed);
    profiler().end(0, s, e);
    void *a2[] = {&AI, &AB, (void *)&n_own, (void *)&plan->send_index, &gs, (void *)&t,
                  (void *)&st, (void *)&R, (void *)&part[3], &kk, &P};
    SLA_CUDA_TRY(cudaLaunchCooperativeKernel(k2, dim3(g2), dim3(kBlock), a2, 0, s));
    g_launches.fetch_add(1, std::memory_order_relaxed);
    SLA_LAUNCH((shard_bi_p2p_k3<T, PREC>), g3, kBlock, 0, s, no, x, r, rhat, p_new, v, t, dinv,
               st, R, part[5], kk, ev_, atol, rtol, P);
    return SLA_OK;
  }));
  ShardState out;
  BiRed red;
  SLA_CUDA_TRY(cudaMemcpyAsync(&out, st, sizeof(out), cudaMemcpyDeviceToHost, s));
  SLA_CUDA_TRY(cudaMemcpyAsync(&red, R, sizeof(red), cudaMemcpyDeviceToHost, s));
  cudaEvent_t done;
  SLA_CUDA_TRY(cudaEventCreateWithFlags(&done, cudaEventDisableTiming));
  SLA_CUDA_TRY(cudaEventRecord(done, s));
  int wrc = wait_bounded(done, pp->comm);
  cudaEventDestroy(done);
  SLA_TRY(wrc);
  profiler().resolve();
  if (out.stopped == kStopTimeout) {
    fprintf(stderr, "[sla_b200] shard BiCGStab: a peer did not answer within the bounded wait\n");
    return SLA_ERR_TIMEOUT;
  }
  info->iterations = out.stopped == 1 ? out.iters : maxiter;
  const long long last = info->iterations - 1;
  info->residual = last >= 0 ? sqrt(red.rr[last & 1][0]) : sqrt(red.init[0]);
  info->status = out.stopped == 1 ? SLA_OK : SLA_NOT_CONVERGED;
  info->reason = out.stopped;
  return info->status;
}
}  // namespace sla

using namespace sla;

extern "C" {

int sla_comm_unique_id(unsigned char id[128]) {
  if (!id) return SLA_ERR_INVALID;
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId size");
  ncclUniqueId uid;
  SLA_NCCL_TRY(ncclGetUniqueId(&uid));
  memcpy(id, &uid, sizeof(uid));
  return SLA_OK;
}

int sla_comm_init(void **comm, int nranks, const unsigned char id[128], int rank) {
  if (!comm || !id || nranks < 1 || rank < 0 || rank >= nranks) return SLA_ERR_INVALID;
  Comm *c = new Comm();
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  ncclResult_t r = ncclCommInitRank(&c->nccl, nranks, uid, rank);
  if (r != ncclSuccess) {
    fprintf(stderr, "[sla_b200] ncclCommInitRank failed: %s\n", ncclGetErrorString(r));
    delete c;
    return SLA_ERR_NCCL;
  }
  c->rank = rank;
  c->nranks = nranks;
  if (cudaStreamCreateWithFlags(&c->side, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreateWithFlags(&c->ev_ready, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&c->ev_halo, cudaEventDisableTiming) != cudaSuccess) {
    ncclCommDestroy(c->nccl);
    delete c;
    return SLA_ERR_CUDA;
  }
  *comm = c;
  return SLA_OK;
}

int sla_comm_destroy(void *comm) {
  Comm *c = (Comm *)comm;
  if (!c) return SLA_OK;
  if (c->side) cudaStreamSynchronize(c->side);
  if (c->nccl) ncclCommDestroy(c->nccl);
  if (c->ev_ready) cudaEventDestroy(c->ev_ready);
  if (c->ev_halo) cudaEventDestroy(c->ev_halo);
  if (c->side) cudaStreamDestroy(c->side);
  delete c;
  return SLA_OK;
}

int sla_halo_exchange(void *comm, const sla_halo_plan_t *plan, int dtype, void *x_local,
                      void *sendbuf, void *recvbuf, sla_stream_t stream) {
  Comm *c = (Comm *)comm;
  if (!c || !c->nccl || !plan_ok(plan) || !x_local) return SLA_ERR_INVALID;
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t ns = n_send(plan), nh = plan->n_halo, no = plan->n_owned;
  if ((ns > 0 && !sendbuf) || (nh > 0 && !recvbuf)) return SLA_ERR_INVALID;
  auto run = [&](auto tag) -> int {
    using T = decltype(tag);
    T *x = (T *)x_local;
    if (ns > 0)
      SLA_LAUNCH((halo_pack_kernel<T, LoadVal<T>>), grid_for(ns), kBlock, 0, s, plan->send_index,
                 ns, LoadVal<T>{x}, (T *)sendbuf, (const int *)nullptr);
    SLA_TRY(halo_enqueue<T>(c, plan, (const T *)sendbuf, (T *)recvbuf, s));
    SLA_CUDA_TRY(cudaStreamWaitEvent(s, c->ev_halo, 0));
    if (nh > 0)
      SLA_LAUNCH(halo_unpack_kernel<T>, grid_for(nh), kBlock, 0, s, (const T *)recvbuf,
                 plan->halo_src, nh, x + no, (const int *)nullptr);
    return SLA_OK;
  };
  if (dtype == SLA_F64) return run(double(0));
  if (dtype == SLA_F32) return run(float(0));
  return SLA_ERR_INVALID;
}

int sla_shard_spmv(void *comm, const sla_halo_plan_t *plan, int dtype, const sla_sell_t *A_interior,
                   const sla_sell_t *A_boundary, void *x_local, void *y_owned, void *sendbuf,
                   void *recvbuf, sla_stream_t stream) {
  Comm *c = (Comm *)comm;
  if (!c || !c->nccl || !plan_ok(plan) || !x_local || !y_owned) return SLA_ERR_INVALID;
  if (!sell_ok(A_interior) || !sell_ok(A_boundary)) return SLA_ERR_INVALID;
  if (A_boundary->n_diags > 0) return SLA_ERR_UNSUPPORTED;
  if (A_interior->n_diags > 0 && A_interior->n_cols > plan->n_owned + plan->n_halo)
    return SLA_ERR_INVALID;
  if ((!A_interior->row_ids && A_interior->row_base + A_interior->n_slots > plan->n_owned) ||
      (!A_boundary->row_ids && A_boundary->row_base + A_boundary->n_slots > plan->n_owned))
    return SLA_ERR_INVALID;

  cudaStream_t s = (cudaStream_t)stream;
  const int64_t ns = n_send(plan), nh = plan->n_halo, no = plan->n_owned;
  if ((ns > 0 && !sendbuf) || (nh > 0 && !recvbuf)) return SLA_ERR_INVALID;
  auto run = [&](auto tag) -> int {
    using T = decltype(tag);
    T *x = (T *)x_local;
    Sell<T> AI = make_sell<T>(A_interior), AB = make_sell<T>(A_boundary);
    if (ns > 0)
      SLA_LAUNCH((halo_pack_kernel<T, LoadVal<T>>), grid_for(ns), kBlock, 0, s, plan->send_index,
                 ns, LoadVal<T>{x}, (T *)sendbuf, (const int *)nullptr);
    SLA_TRY(halo_enqueue<T>(c, plan, (const T *)sendbuf, (T *)recvbuf, s));
    const int wspec = width_spec2(A_interior, A_boundary);
    if (AI.n_slices > 0)
      SLA_WS_DISPATCH(wspec, SLA_LAUNCH((shard_spmv_rows_kernel<T, PlainGather<T>, WS>),
                                        grid_for(AI.n_slices * 32, kBlock, 4), kBlock, 0, s, AI,
                                        PlainGather<T>{x}, (T *)y_owned));
    SLA_CUDA_TRY(cudaStreamWaitEvent(s, c->ev_halo, 0));
    if (nh > 0)
      SLA_LAUNCH(halo_unpack_kernel<T>, grid_for(nh), kBlock, 0, s, (const T *)recvbuf,
                 plan->halo_src, nh, x + no, (const int *)nullptr);
    if (AB.n_slices > 0)
      SLA_WS_DISPATCH(boundary_spec(wspec),
                      SLA_LAUNCH((shard_spmv_rows_kernel<T, PlainGather<T>, WS>),
                                 grid_for(AB.n_slices * 32, kBlock, 4), kBlock, 0, s, AB,
                                 PlainGather<T>{x}, (T *)y_owned));
    return SLA_OK;
  };
  if (dtype == SLA_F64) return run(double(0));
  if (dtype == SLA_F32) return run(float(0));
  return SLA_ERR_INVALID;
}

int sla_reverse_halo_exchange(void *comm, const sla_halo_plan_t *plan, int dtype, void *w_local,
                              void *sendbuf, void *recvbuf, sla_stream_t stream) {
  Comm *c = (Comm *)comm;
  if (!c || !c->nccl || !plan_ok(plan) || !w_local) return SLA_ERR_INVALID;
  if ((plan->n_halo > 0 && !sendbuf) || (n_send(plan) > 0 && !recvbuf)) return SLA_ERR_INVALID;
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == SLA_F64)
    return reverse_exchange<double>(c, plan, (double *)w_local, (double *)sendbuf,
                                    (double *)recvbuf, s);
  if (dtype == SLA_F32)
    return reverse_exchange<float>(c, plan, (float *)w_local, (float *)sendbuf, (float *)recvbuf,
                                   s);
  return SLA_ERR_INVALID;
}

int sla_shard_rmatvec(void *comm, const sla_halo_plan_t *plan, int dtype, const sla_sell_t *AT,
                      const void *y_owned, void *w_local, void *sendbuf, void *recvbuf,
                      sla_stream_t stream) {
  Comm *c = (Comm *)comm;
  if (!c || !c->nccl || !plan_ok(plan) || !sell_ok(AT) || !w_local) return SLA_ERR_INVALID;
  if (AT->n_slots != plan->n_owned + plan->n_halo || AT->row_ids || AT->row_base)
    return SLA_ERR_INVALID;
  if (AT->n_diags > 0 && AT->n_cols > plan->n_owned) return SLA_ERR_INVALID;
  if ((plan->n_owned > 0 && !y_owned) || (plan->n_halo > 0 && !sendbuf) ||
      (n_send(plan) > 0 && !recvbuf))
    return SLA_ERR_INVALID;
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == SLA_F64) {
    SLA_TRY(spmv_launch<double>(AT, y_owned, w_local, s));
    return reverse_exchange<double>(c, plan, (double *)w_local, (double *)sendbuf,
                                    (double *)recvbuf, s);
  }
  if (dtype == SLA_F32) {
    SLA_TRY(spmv_launch<float>(AT, y_owned, w_local, s));
    return reverse_exchange<float>(c, plan, (float *)w_local, (float *)sendbuf, (float *)recvbuf,
                                   s);
  }
  return SLA_ERR_INVALID;
}

int sla_shard_krylov_workspace(int dtype, int64_t n_owned, int64_t n_halo, int64_t n_send_,
                               size_t *bytes) {
  if (!bytes || n_owned < 0 || n_halo < 0 || n_send_ < 0) return SLA_ERR_INVALID;
  if (dtype != SLA_F32 && dtype != SLA_F64) return SLA_ERR_INVALID;
  *bytes = shard_ws_bytes(dtype == SLA_F64 ? 8 : 4, n_owned, n_halo, n_send_);
  return SLA_OK;
}

static int shard_args_ok(void *ch, void *cr, const sla_halo_plan_t *plan, const sla_sell_t *Ai,
                         const sla_sell_t *Ab, const void *b, void *x, sla_solve_info_t *info,
                         int64_t every) {
  if (!ch || !cr || !((Comm *)ch)->nccl || !((Comm *)cr)->nccl) return SLA_ERR_INVALID;
  if (!plan_ok(plan) || !sell_ok(Ai) || !sell_ok(Ab) || !info || every < 1) return SLA_ERR_INVALID;
  if (Ab->n_diags > 0) return SLA_ERR_UNSUPPORTED;
  // interior gathers read owned vectors only
  if (Ai->n_diags > 0 && Ai->n_cols > plan->n_owned) return SLA_ERR_INVALID;
  if (plan->n_owned > 0 && (!b || !x)) return SLA_ERR_INVALID;
  if (Ai->n_slots + Ab->n_slots != plan->n_owned) return SLA_ERR_INVALID;
  if ((!Ai->row_ids && Ai->row_base + Ai->n_slots > plan->n_owned) ||
      (!Ab->row_ids && Ab->row_base + Ab->n_slots > plan->n_owned))
    return SLA_ERR_INVALID;
  if (plan->n_owned + plan->n_halo >= INT32_MAX) return SLA_ERR_UNSUPPORTED;
  return SLA_OK;
}

int sla_shard_cg(void *comm_halo, void *comm_reduce, const sla_halo_plan_t *plan, int dtype,
                 const sla_sell_t *A_interior, const sla_sell_t *A_boundary, const void *dinv,
                 const void *b, void *x, double atol, double rtol, int64_t maxiter,
                 int64_t check_every, void *workspace, size_t workspace_bytes,
                 sla_solve_info_t *info, sla_stream_t stream) {
  SLA_TRY(shard_args_ok(comm_halo, comm_reduce, plan, A_interior, A_boundary, b, x, info,
                        check_every));
  info->iterations = 0; info->residual = 0; info->status = 0; info->reason = 0;
  size_t need = 0;
  SLA_TRY(sla_shard_krylov_workspace(dtype, plan->n_owned, plan->n_halo, n_send(plan), &need));
  if (workspace_bytes < need || !workspace) return SLA_ERR_WORKSPACE;
  Comm *ch = (Comm *)comm_halo, *cr = (Comm *)comm_reduce;
  cudaStream_t s = (cudaStream_t)stream;
  const int wspec = width_spec2(A_interior, A_boundary);
  if (dtype == SLA_F64) {
    if (dinv)
      SLA_WS_DISPATCH(wspec, return shard_cg_impl<double, true, WS>(ch, cr, plan, A_interior, A_boundary, (const double *)dinv,
                                         (const double *)b, (double *)x, atol, rtol, maxiter,
                                         check_every, workspace, workspace_bytes, info, s));
    SLA_WS_DISPATCH(wspec, return shard_cg_impl<double, false, WS>(ch, cr, plan, A_interior, A_boundary, nullptr,
                                        (const double *)b, (double *)x, atol, rtol, maxiter,
                                        check_every, workspace, workspace_bytes, info, s));
  }
  if (dtype == SLA_F32) {
    if (dinv)
      SLA_WS_DISPATCH(wspec, return shard_cg_impl<float, true, WS>(ch, cr, plan, A_interior, A_boundary, (const float *)dinv,
                                        (const float *)b, (float *)x, atol, rtol, maxiter,
                                        check_every, workspace, workspace_bytes, info, s));
    SLA_WS_DISPATCH(wspec, return shard_cg_impl<float, false, WS>(ch, cr, plan, A_interior, A_boundary, nullptr,
                                       (const float *)b, (float *)x, atol, rtol, maxiter,
                                       check_every, workspace, workspace_bytes, info, s));
  }
  return SLA_ERR_INVALID;
}

int sla_shard_bicgstab(void *comm_halo, void *comm_reduce, const sla_halo_plan_t *plan, int dtype,
                       const sla_sell_t *A_interior, const sla_sell_t *A_boundary,
                       const void *dinv, const void *b, void *x, double atol, double rtol,
                       int64_t maxiter, int64_t check_every, void *workspace,
                       size_t workspace_bytes, sla_solve_info_t *info, sla_stream_t stream) {
  SLA_TRY(shard_args_ok(comm_halo, comm_reduce, plan, A_interior, A_boundary, b, x, info,
                        check_every));
  info->iterations = 0; info->residual = 0; info->status = 0; info->reason = 0;
  size_t need = 0;
  SLA_TRY(sla_shard_krylov_workspace(dtype, plan->n_owned, plan->n_halo, n_send(plan), &need));
  if (workspace_bytes < need || !workspace) return SLA_ERR_WORKSPACE;
  Comm *ch = (Comm *)comm_halo, *cr = (Comm *)comm_reduce;
  cudaStream_t s = (cudaStream_t)stream;
  const int wspec = width_spec2(A_interior, A_boundary);
  if (dtype == SLA_F64) {
    if (dinv)
      SLA_WS_DISPATCH(wspec, return shard_bi_impl<double, true, WS>(ch, cr, plan, A_interior, A_boundary, (const double *)dinv,
                                         (const double *)b, (double *)x, atol, rtol, maxiter,
                                         check_every, workspace, workspace_bytes, info, s));
    SLA_WS_DISPATCH(wspec, return shard_bi_impl<double, false, WS>(ch, cr, plan, A_interior, A_boundary, nullptr,
                                        (const double *)b, (double *)x, atol, rtol, maxiter,
                                        check_every, workspace, workspace_bytes, info, s));
  }
  if (dtype == SLA_F32) {
    if (dinv)
      SLA_WS_DISPATCH(wspec, return shard_bi_impl<float, true, WS>(ch, cr, plan, A_interior, A_boundary, (const float *)dinv,
                                        (const float *)b, (float *)x, atol, rtol, maxiter,
                                        check_every, workspace, workspace_bytes, info, s));
    SLA_WS_DISPATCH(wspec, return shard_bi_impl<float, false, WS>(ch, cr, plan, A_interior, A_boundary, nullptr,
                                       (const float *)b, (float *)x, atol, rtol, maxiter,
                                       check_every, workspace, workspace_bytes, info, s));
  }
  return SLA_ERR_INVALID;
}

// ----------------------------------------------------------- peer-memory path
static void p2p_release(P2PPlan *pp) {
  if (!pp) return;
  for (int q = 0; q < pp->world; ++q)
    if (q != pp->me && pp->peer[q]) cudaIpcCloseMemHandle(pp->peer[q]);
  if (pp->local) cudaFree(pp->local);
  delete pp;
}

// Trade the IPC handles over NCCL and agree on the outcome; fills pp->peer
// and pp->dst_off. Returns a negative status only when the collective
// itself failed; *all_ok says whether every rank mapped every buffer.
static int p2p_exchange(P2PPlan *pp, Comm *c, int ok, const cudaIpcMemHandle_t &mine,
                        int *all_ok) {
  const int world = pp->world, me = pp->me;
  const size_t hs = sizeof(cudaIpcMemHandle_t);
  cudaStream_t s = c->side;
  unsigned char *dbuf = nullptr;  // handles of all ranks + agreement flag
  cudaEvent_t ev = nullptr;
  int rc = SLA_OK;
  std::vector<cudaIpcMemHandle_t> all(world);
  auto done = [&](int r) {
    if (ev) cudaEventDestroy(ev);
    if (dbuf) cudaFree(dbuf);
    return r;
  };
  if (cudaMalloc((void **)&dbuf, hs * world + 16) != cudaSuccess ||
      cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess)
    return done(SLA_ERR_CUDA);
  int *flag = (int *)(dbuf + hs * world);
  if (cudaMemcpy(dbuf + hs * me, &mine, hs, cudaMemcpyHostToDevice) != cudaSuccess)
    return done(SLA_ERR_CUDA);
  if (ncclAllGather(dbuf + hs * me, dbuf, hs, ncclUint8, c->nccl, s) != ncclSuccess)
    return done(SLA_ERR_NCCL);
  if (cudaEventRecord(ev, s) != cudaSuccess) return done(SLA_ERR_CUDA);
  if ((rc = wait_bounded(ev, c)) != SLA_OK) return done(rc);
  if (cudaMemcpy(all.data(), dbuf, hs * world, cudaMemcpyDeviceToHost) != cudaSuccess)
    return done(SLA_ERR_CUDA);
  pp->peer[me] = pp->local;
  for (int q = 0; q < world && ok; ++q) {
    if (q == me) continue;
    void *ptr = nullptr;
    if (cudaIpcOpenMemHandle(&ptr, all[q], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) ok = 0;
    else pp->peer[q] = (char *)ptr;
  }
  // where this rank's values go in each neighbour's halo
  for (int i = 0; i < pp->n_nb && ok; ++i) {
    long long off = -1;
    const int q = pp->nb_rank[i];
    if (cudaMemcpy(&off, pp->peer[q] + offsetof(P2PHeader, recv_off) + sizeof(long long) * me,
                   sizeof(off), cudaMemcpyDeviceToHost) != cudaSuccess || off < 0)
      ok = 0;
    pp->dst_off[i] = off;
  }
  cudaGetLastError();  // a refused mapping is an answer, not a sticky error
  if (cudaMemcpy(flag, &ok, sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess)
    return done(SLA_ERR_CUDA);
  if (ncclAllReduce(flag, flag, 1, ncclInt32, ncclMin, c->nccl, s) != ncclSuccess)
    return done(SLA_ERR_NCCL);
  if (cudaEventRecord(ev, s) != cudaSuccess) return done(SLA_ERR_CUDA);
  if ((rc = wait_bounded(ev, c)) != SLA_OK) return done(rc);
  if (cudaMemcpy(all_ok, flag, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
    return done(SLA_ERR_CUDA);
  return done(SLA_OK);
}

int sla_p2p_create(void *comm, const sla_halo_plan_t *plan, int dtype, void **p2p_out) {
  if (!p2p_out) return SLA_ERR_INVALID;
  *p2p_out = nullptr;
  Comm *c = (Comm *)comm;
  if (!c || !c->nccl || !plan_ok(plan)) return SLA_ERR_INVALID;
  if (dtype != SLA_F32 && dtype != SLA_F64) return SLA_ERR_INVALID;
  const int world = c->nranks, me = c->rank;
  if (world < 2 || world > kP2PMaxRanks) return SLA_OK;  // same answer on every rank
  P2PPlan *pp = new P2PPlan();
  pp->comm = c;
  pp->world = world;
  pp->me = me;
  pp->n_nb = plan->n_neighbors;
  pp->n_halo = plan->n_halo;
  pp->n_owned = plan->n_owned;
  pp->elem = dtype == SLA_F64 ? 8 : 4;
  int ok = plan->halo_src == nullptr && plan->n_neighbors < kP2PMaxRanks ? 1 : 0;
  const size_t bytes = p2p_halo_offset() + align_up(pp->elem * (size_t)(plan->n_halo + 1));
  cudaIpcMemHandle_t mine{};
  if (ok && cudaMalloc((void **)&pp->local, bytes) != cudaSuccess) ok = 0;
  if (ok) {
    P2PHeader h{};
    for (int q = 0; q < kP2PMaxRanks; ++q) h.recv_off[q] = -1;
    for (int i = 0; i < plan->n_neighbors; ++i) {
      h.recv_off[plan->neighbor_rank[i]] = plan->recv_offset[i];
      pp->nb_rank[i] = plan->neighbor_rank[i];
      pp->send_off[i] = plan->send_offset[i];
    }
    pp->send_off[plan->n_neighbors] =
        plan->n_neighbors > 0 ? plan->send_offset[plan->n_neighbors] : 0;
    if (cudaMemset(pp->local, 0, bytes) != cudaSuccess ||
        cudaMemcpy(pp->local, &h, sizeof(h), cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaIpcGetMemHandle(&mine, pp->local) != cudaSuccess)
      ok = 0;
  }
  cudaGetLastError();
  int all_ok = 0;
  const int rc = p2p_exchange(pp, c, ok, mine, &all_ok);
  if (rc != SLA_OK || !all_ok) {
    p2p_release(pp);
    return rc;  // SLA_OK with *p2p_out NULL: the NCCL path serves
  }
  pp->barrier = (int *)(pp->local + offsetof(P2PHeader, pad));
  if (const char *w = getenv("TORCH_SLA_B200_P2P_WAIT_S")) {
    const double sec = atof(w);
    if (sec > 0.0) pp->wait_ns = (unsigned long long)(sec * 1e9);
  }
  *p2p_out = pp;
  return SLA_OK;
}

int sla_p2p_destroy(void *p2p) {
  P2PPlan *pp = (P2PPlan *)p2p;
  if (!pp) return SLA_OK;
  // every rank is past its last remote store before any mapping goes away
  int rc = SLA_OK;
  Comm *c = pp->comm;
  if (c && c->nccl) {
    cudaStream_t s = c->side;
    int *d = nullptr;
    if (cudaMalloc((void **)&d, sizeof(int)) == cudaSuccess) {
      if (ncclAllReduce(d, d, 1, ncclInt32, ncclSum, c->nccl, s) != ncclSuccess) rc = SLA_ERR_NCCL;
      cudaEvent_t ev;
      if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) == cudaSuccess) {
        cudaEventRecord(ev, s);
        int w = wait_bounded(ev, c);
        if (w != SLA_OK) rc = w;
        cudaEventDestroy(ev);
      }
      cudaFree(d);
    }
  }
  cudaDeviceSynchronize();
  p2p_release(pp);
  return rc;
}

static int p2p_args_ok(P2PPlan *pp, const sla_halo_plan_t *plan, int dtype, const sla_sell_t *Ai,
                       const sla_sell_t *Ab, const void *b, void *x, sla_solve_info_t *info,
                       int64_t every, size_t workspace_bytes, void *workspace) {
  if (!pp || !pp->comm) return SLA_ERR_INVALID;
  SLA_TRY(shard_args_ok(pp->comm, pp->comm, plan, Ai, Ab, b, x, info, every));
  if (plan->n_owned != pp->n_owned || plan->n_halo != pp->n_halo ||
      plan->n_neighbors != pp->n_nb || plan->halo_src)
    return SLA_ERR_INVALID;
  if (dtype != SLA_F32 && dtype != SLA_F64) return SLA_ERR_INVALID;
  if ((dtype == SLA_F64 ? 8u : 4u) != pp->elem) return SLA_ERR_INVALID;
  if (!device_info().coop) return SLA_ERR_UNSUPPORTED;
  size_t need = 0;
  SLA_TRY(sla_shard_krylov_workspace(dtype, plan->n_owned, plan->n_halo, n_send(plan), &need));
  if (workspace_bytes < need || !workspace) return SLA_ERR_WORKSPACE;
  return SLA_OK;
}

int sla_shard_cg_p2p(void *p2p, const sla_halo_plan_t *plan, int dtype,
                     const sla_sell_t *A_interior, const sla_sell_t *A_boundary, const void *dinv,
                     const void *b, void *x, double atol, double rtol, int64_t maxiter,
                     int64_t check_every, void *workspace, size_t workspace_bytes,
                     sla_solve_info_t *info, sla_stream_t stream) {
  P2PPlan *pp = (P2PPlan *)p2p;
  SLA_TRY(p2p_args_ok(pp, plan, dtype, A_interior, A_boundary, b, x, info, check_every,
                      workspace_bytes, workspace));
  info->iterations = 0; info->residual = 0; info->status = 0; info->reason = 0;
  cudaStream_t s = (cudaStream_t)stream;
  const int wspec = width_spec2(A_interior, A_boundary);
  if (dtype == SLA_F64) {
    if (dinv)
      SLA_WS_DISPATCH(wspec, return shard_cg_p2p_impl<double, true, WS>(pp, plan, A_interior, A_boundary, (const double *)dinv,
                                                                 (const double *)b, (double *)x, atol, rtol, maxiter, check_every,
                                                                 workspace, workspace_bytes, info, s));
    SLA_WS_DISPATCH(wspec, return shard_cg_p2p_impl<double, false, WS>(pp, plan, A_interior, A_boundary, nullptr,
                                                                (const double *)b, (double *)x, atol, rtol, maxiter, check_every,
                                                                workspace, workspace_bytes, info, s));
  }
  if (dinv)
    SLA_WS_DISPATCH(wspec, return shard_cg_p2p_impl<float, true, WS>(pp, plan, A_interior, A_boundary, (const float *)dinv,
                                                              (const float *)b, (float *)x, atol, rtol, maxiter, check_every,
                                                              workspace, workspace_bytes, info, s));
  SLA_WS_DISPATCH(wspec, return shard_cg_p2p_impl<float, false, WS>(pp, plan, A_interior, A_boundary, nullptr,
                                                             (const float *)b, (float *)x, atol, rtol, maxiter, check_every,
                                                             workspace, workspace_bytes, info, s));
  return SLA_ERR_INVALID;
}

int sla_shard_bicgstab_p2p(void *p2p, const sla_halo_plan_t *plan, int dtype,
                           const sla_sell_t *A_interior, const sla_sell_t *A_boundary,
                           const void *dinv, const void *b, void *x, double atol, double rtol,
                           int64_t maxiter, int64_t check_every, void *workspace,
                           size_t workspace_bytes, sla_solve_info_t *info, sla_stream_t stream) {
  P2PPlan *pp = (P2PPlan *)p2p;
  SLA_TRY(p2p_args_ok(pp, plan, dtype, A_interior, A_boundary, b, x, info, check_every,
                      workspace_bytes, workspace));
  info->iterations = 0; info->residual = 0; info->status = 0; info->reason = 0;
  cudaStream_t s = (cudaStream_t)stream;
  const int wspec = width_spec2(A_interior, A_boundary);
  if (dtype == SLA_F64) {
    if (dinv)
      SLA_WS_DISPATCH(wspec, return shard_bi_p2p_impl<double, true, WS>(pp, plan, A_interior, A_boundary, (const double *)dinv,
                                                                 (const double *)b, (double *)x, atol, rtol, maxiter, check_every,
                                                                 workspace, workspace_bytes, info, s));
    SLA_WS_DISPATCH(wspec, return shard_bi_p2p_impl<double, false, WS>(pp, plan, A_interior, A_boundary, nullptr,
                                                                (const double *)b, (double *)x, atol, rtol, maxiter, check_every,
                                                                workspace, workspace_bytes, info, s));
  }
  if (dinv)
    SLA_WS_DISPATCH(wspec, return shard_bi_p2p_impl<float, true, WS>(pp, plan, A_interior, A_boundary, (const float *)dinv,
                                                              (const float *)b, (float *)x, atol, rtol, maxiter, check_every,
                                                              workspace, workspace_bytes, info, s));
  SLA_WS_DISPATCH(wspec, return shard_bi_p2p_impl<float, false, WS>(pp, plan, A_interior, A_boundary, nullptr,
                                                             (const float *)b, (float *)x, atol, rtol, maxiter, check_every,
                                                             workspace, workspace_bytes, info, s));
  return SLA_ERR_INVALID;
}

}  // extern "C"
