// Definitions shared by the NCCL path (shard.cu) and the peer-memory path
// (shard_p2p.cu) of the row-sharded solvers: communicator handle, plan
// checks, per-solve state, the search-direction functors of the shard CG and
// BiCGStab (distributed/solve.py:279-436) and the host loop.
#pragma once

#include <nccl.h>

#include <chrono>
#include <cstddef>
#include <cstring>
#include <thread>
#include <vector>

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

inline int wait_bounded(cudaEvent_t ev, Comm *c) {
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

inline bool plan_ok(const sla_halo_plan_t *p) {
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
inline int width_spec2(const sla_sell_t *a, const sla_sell_t *b) {
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

inline int64_t n_send(const sla_halo_plan_t *p) {
  return p->n_neighbors > 0 ? p->send_offset[p->n_neighbors] : 0;
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

// x += alpha p is applied two iterations at a time (at odd k:
// x = (x + alpha_prev p_prev) + alpha p, the same two roundings as two
// steps) while both directions sit in the ping-pong buffers; a solve whose
// last update was an even one gets the pending step from shard_cg_xflush.
template <typename T>
__device__ __forceinline__ T cg_x2(T xi, T ap, T pp, T a, T pc) {
  return add_rn(add_rn(xi, mul_rn(ap, pp)), mul_rn(a, pc));
}

// Pending x step after a last even update (kb_done odd); p_last is its
// direction.
template <typename T>
static __global__ void __launch_bounds__(kBlock)
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

// ================================================================= drivers
inline size_t shard_ws_bytes(size_t elem, int64_t n_own, int64_t n_halo, int64_t n_snd) {
  size_t G = (size_t)solver_grid();
  return 6 * align_up(elem * (size_t)(n_own + 1)) + align_up(elem * (size_t)(n_snd + 1)) +
         2 * align_up(elem * (size_t)(n_halo + 1)) + 6 * align_up(4 * G * sizeof(double)) +
         align_up(sizeof(ShardState)) + align_up(sizeof(BiRed)) + align_up(sizeof(CgRed));
}

// Poll the sticky stop flag once per chunk, one chunk in flight; all ranks
// see identical flags at identical points, so they stop enqueueing together.
template <typename Body>
inline int shard_loop(Comm *c, int64_t maxiter, int64_t chunk, const int *d_stopped,
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


inline int shard_args_ok(void *ch, void *cr, const sla_halo_plan_t *plan, const sla_sell_t *Ai,
                         const sla_sell_t *Ab, const void *b, void *x, sla_solve_info_t *info,
                         int64_t every) {
  if (!ch || !cr || !((Comm *)ch)->nccl || !((Comm *)cr)->nccl) return SLA_ERR_INVALID;
  SLA_TRY(sell_check(Ai));
  SLA_TRY(sell_check(Ab));
  if (!plan_ok(plan) || !info || every < 1) return SLA_ERR_INVALID;
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

}  // namespace sla
