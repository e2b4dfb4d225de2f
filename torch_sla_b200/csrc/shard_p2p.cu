// Peer-memory path of the row-sharded CG and BiCGStab (one node, 2..8
// ranks): halo values and dot products are stored by the solver kernels
// straight into the other GPUs' memory through CUDA IPC mappings.
#include "shard.cuh"

namespace sla {

// ============================================================ peer-memory path
// Single-node path of the shard CG: halo values and dot products travel as
// stores into the other GPUs' memory (CUDA IPC mappings over NVLink /
// NVSwitch) from inside the solver kernels. An iteration is three launches:
//   K_P  stop test; form the search direction p; send this rank's share of
//        the neighbours' halo straight into their halo buffers, the last
//        block raising an arrival sequence number
//   K_A  stop test; interior rows; wait for the neighbours' arrivals;
//        boundary rows; (p, Ap) summed over the grid and then over the
//        ranks in rank order
//   K_B  x / r update, (r, r) and (r, z) summed the same way.
// (With SLA_CG_SPLIT 0, K_P's work runs at the start of K_A, p computed on
// the fly inside the gathers.)
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
  // instrumentation of this rank's solver kernels, written only while the
  // library's profiling is on (kTimer* slots, nanoseconds summed)
  unsigned long long timers[8];
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
  unsigned long long *timers;    // &local->timers while profiling, else null
};

// Timer slots (sums over launches; per-block slots also over the blocks):
//   kTimerSend   K_P, every block: storing its share of the neighbours' halo
//                and the system-scope fence that makes the stores visible
//   kTimerWait   K_A, every block: waiting for the neighbours' arrivals
//   kTimerRedA   K_A, the last block: the cross-rank (p, Ap) sum
//   kTimerRedB   K_B, the last block: the cross-rank (r,r), (r,z) sum
//   kTimerBlocks K_A: blocks per launch summed (divides kTimerWait)
//   kTimerIters  K_A launches that ran (iterations)
//   kTimerSendBlocks K_P: blocks per launch summed (divides kTimerSend)
enum { kTimerSend = 0, kTimerWait, kTimerRedA, kTimerRedB, kTimerBlocks, kTimerIters,
       kTimerSendBlocks, kTimerCount };

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

template <typename T>
__device__ __forceinline__ unsigned long long p2p_tic(const P2PDev<T> &P) {
  return P.timers ? global_ns() : 0ull;
}
// Adds the time since t0 to a timer slot (thread 0 of the calling block).
template <typename T>
__device__ __forceinline__ void p2p_toc(const P2PDev<T> &P, int slot, unsigned long long t0) {
  if (P.timers && threadIdx.x == 0) atomicAdd(P.timers + slot, global_ns() - t0);
}
template <typename T>
__device__ __forceinline__ void p2p_count(const P2PDev<T> &P, int slot, unsigned long long v) {
  if (P.timers && threadIdx.x == 0) atomicAdd(P.timers + slot, v);
}

// The first kHaloBlocks blocks store the halo values of all neighbours
// (the other blocks skip the system fence the stores need), then the last
// of them to finish raises the arrival flags (all threads of a block call
// it).
constexpr int kHaloBlocks = 64;

template <typename T, typename PV>
__device__ __forceinline__ void p2p_send_halo(const P2PDev<T> &P, const int32_t *__restrict__ idx,
                                              const PV &pval, unsigned long long seq) {
  const unsigned senders = gridDim.x < kHaloBlocks ? gridDim.x : kHaloBlocks;
  if (P.n_nb == 0 || blockIdx.x >= senders) return;  // no neighbour waits on this rank
  const long long ns = P.send_off[P.n_nb];
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < ns;
       i += (long long)senders * blockDim.x) {
    int nb = 0;
    while (i >= P.send_off[nb + 1]) ++nb;
    P.dst[nb][i - P.send_off[nb]] = pval(idx[i]);
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned t = atomicAdd(&P.local->send_count, 1u);
    if (t == senders - 1) {
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
    // the release store orders this thread's value stores before the flag
    // at system scope (no separate fence)
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
  const unsigned long long tw = p2p_tic(P);
  if (!p2p_wait_halo(P, seq)) {
    if (threadIdx.x == 0) st->stopped = kStopTimeout;
    return;
  }
  p2p_toc(P, kTimerWait, tw);
  if (blockIdx.x == 0) {
    p2p_count(P, kTimerBlocks, gridDim.x);
    p2p_count(P, kTimerIters, 1);
  }
  HaloGatherL2<T, ShardP<T, PREC>> g{inner, P.halo, n_own};
  for_each_slice<WSB>(AB, warp, nwarps, lane, [&](int64_t s, int32_t sbase, int swidth) {
    emit(AB, s, sell_row_at<WSB>(AB, s, sbase, swidth, lane, g));
  });
  if (!last_block_sum<1, kBlock>(acc, partials, &st->counter[1], smem)) return;
  const unsigned long long tr = p2p_tic(P);
  if (!p2p_allreduce<1>(P, 1, (int)(k & 1), seq, acc)) {
    if (threadIdx.x == 0) st->stopped = kStopTimeout;
    return;
  }
  p2p_toc(P, kTimerRedA, tr);
  if (threadIdx.x == 0) R->pap[0] = acc[0];
}

// Split form of K_A (SLA_CG_SPLIT, as in the single-GPU CG): a streaming
// pass forms p_new for every owned row and sends the neighbours' halo share,
// then the cooperative SpMV gathers p_new. Both kernels take the same stop
// decision from the summed residual; only the SpMV records it.
template <typename T, bool PREC>
__global__ void __launch_bounds__(kBlock)
shard_cg_p2p_pform(int64_t n, const int32_t *__restrict__ send_index, const T *__restrict__ r,
                   const T *__restrict__ dinv, const T *__restrict__ p_old, T *__restrict__ p_new,
                   const ShardState *st, const CgRed *R, long long k, long long every,
                   double atol, double rtol, P2PDev<T> P) {
  if (*(volatile const int *)&st->stopped) return;
  if (cg_stop(R, k, every, cg_tol(R, atol, rtol))) return;
  ShardP<T, PREC> inner{r, dinv, p_old, (T)cg_beta(R, k)};
  const unsigned long long t0 = p2p_tic(P);
  p2p_send_halo(P, send_index, inner, P.seq + (unsigned long long)(k + 1));
  p2p_toc(P, kTimerSend, t0);
  if (blockIdx.x == 0) p2p_count(P, kTimerSendBlocks, gridDim.x);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    p_new[i] = inner((int32_t)i);
}

template <typename T, int WS>
__global__ void __launch_bounds__(kBlock, kSpmvMinBlocks)
shard_cg_p2p_spmv_split(Sell<T> AI, Sell<T> AB, int32_t n_own, const T *__restrict__ p,
                        T *__restrict__ Ap, ShardState *st, CgRed *R, double *partials,
                        long long k, long long every, double atol, double rtol, P2PDev<T> P) {
  constexpr int WSB = boundary_spec(WS);
  __shared__ double smem[kWarps];
  if (*(volatile int *)&st->stopped) return;
  if (cg_stop(R, k, every, cg_tol(R, atol, rtol))) {
    if (blockIdx.x == 0 && threadIdx.x == 0) { st->stopped = 1; st->iters = k; }
    return;
  }
  const unsigned long long seq = P.seq + (unsigned long long)(k + 1);
  PlainGather<T> inner{p};
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  double acc[1] = {0.0};
  auto emit = [&](const Sell<T> &A, int64_t s, T sum) {
    const int64_t slot = s * 32 + lane;
    if (slot < A.n_slots) {
      const int32_t row = (int32_t)slot_row(A, slot);
      const T pn = __ldg(p + row);
      Ap[row] = sum;
      acc[0] += (double)pn * (double)sum;
    }
  };
  for_each_slice<WS, true>(AI, warp, nwarps, lane, [&](int64_t s, int32_t sbase, int swidth) {
    emit(AI, s, sell_row_at<WS>(AI, s, sbase, swidth, lane, inner));
  });
  const unsigned long long tw = p2p_tic(P);
  if (!p2p_wait_halo(P, seq)) {
    if (threadIdx.x == 0) st->stopped = kStopTimeout;
    return;
  }
  p2p_toc(P, kTimerWait, tw);
  if (blockIdx.x == 0) {
    p2p_count(P, kTimerBlocks, gridDim.x);
    p2p_count(P, kTimerIters, 1);
  }
  HaloGatherL2<T, PlainGather<T>> g{inner, P.halo, n_own};
  for_each_slice<WSB>(AB, warp, nwarps, lane, [&](int64_t s, int32_t sbase, int swidth) {
    emit(AB, s, sell_row_at<WSB>(AB, s, sbase, swidth, lane, g));
  });
  if (!last_block_sum<1, kBlock>(acc, partials, &st->counter[1], smem)) return;
  const unsigned long long tr = p2p_tic(P);
  if (!p2p_allreduce<1>(P, 1, (int)(k & 1), seq, acc)) {
    if (threadIdx.x == 0) st->stopped = kStopTimeout;
    return;
  }
  p2p_toc(P, kTimerRedA, tr);
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
  const unsigned long long tr = p2p_tic(P);
  if (!p2p_allreduce<2>(P, 2, (int)(k & 1), P.seq + (unsigned long long)(k + 1), acc)) {
    if (threadIdx.x == 0) st->stopped = kStopTimeout;
    return;
  }
  p2p_toc(P, kTimerRedB, tr);
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
  d.timers = profiler().enabled
                 ? (unsigned long long *)(pp->local + offsetof(P2PHeader, timers))
                 : nullptr;
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
  const void *ka = kCgSplit ? (const void *)shard_cg_p2p_spmv_split<T, WS>
                            : (const void *)shard_cg_p2p_spmv<T, PREC, WS>;
  int per_sm = 0;
  SLA_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, ka, kBlock, 0));
  if (per_sm < 1) return SLA_ERR_UNSUPPORTED;
  int ga = per_sm * device_info().sm_count;
  if (ga > G) ga = G;
  const int gu = occupancy_grid((const void *)shard_cg_p2p_update<T, PREC>);
  const int gp = occupancy_grid((const void *)shard_cg_p2p_pform<T, PREC>);
  const int32_t n_own = (int32_t)no;
  SLA_TRY(shard_loop(pp->comm, maxiter, every, &st->stopped, s, [&](int64_t k) -> int {
    T *p_old = (k & 1) ? pB : pA, *p_new = (k & 1) ? pA : pB;
    long long kk = (long long)k, ev_ = (long long)every;
    void *args[] = {&AI, &AB, (void *)&n_own, (void *)&plan->send_index, (void *)&r,
                    (void *)&dinv, (void *)&p_old, (void *)&p_new, (void *)&Ap, (void *)&st,
                    (void *)&R, (void *)&part[1], &kk, &ev_, (void *)&atol, (void *)&rtol, &P};
    void *args_split[] = {&AI, &AB, (void *)&n_own, (void *)&p_new, (void *)&Ap, (void *)&st,
                          (void *)&R, (void *)&part[1], &kk, &ev_, (void *)&atol, (void *)&rtol,
                          &P};
    cudaEvent_t e;
    if (kCgSplit) {
      profiler().begin(2, k, s, &e);
      SLA_LAUNCH((shard_cg_p2p_pform<T, PREC>), gp, kBlock, 0, s, no, plan->send_index, r, dinv,
                 p_old, p_new, st, R, kk, ev_, atol, rtol, P);
      profiler().end(2, s, e);
    }
    profiler().begin(0, k, s, &e);
    SLA_CUDA_TRY(cudaLaunchCooperativeKernel(ka, dim3(ga), dim3(kBlock),
                                             kCgSplit ? args_split : args, 0, s));
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
  // one rank has no peer to map but runs the same kernels (its cross-rank
  // sums cover itself), so one and several GPUs time the same code
  if (world < 1 || world > kP2PMaxRanks) return SLA_OK;  // same answer on every rank
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

int sla_p2p_profile_read(void *p2p, int reset, unsigned long long *out, int n_out) {
  P2PPlan *pp = (P2PPlan *)p2p;
  if (!pp || !out || n_out < 0) return SLA_ERR_INVALID;
  unsigned long long t[kTimerCount] = {};
  char *dev = pp->local + offsetof(P2PHeader, timers);
  SLA_CUDA_TRY(cudaDeviceSynchronize());
  SLA_CUDA_TRY(cudaMemcpy(t, dev, sizeof(t), cudaMemcpyDeviceToHost));
  if (reset) SLA_CUDA_TRY(cudaMemset(dev, 0, sizeof(t)));
  for (int i = 0; i < n_out; ++i) out[i] = i < kTimerCount ? t[i] : 0ull;
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
