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
// On one node the solvers run instead on peer-memory exchange buffers
// (shard_p2p.cu); the definitions both share are in shard.cuh.
#include "shard.cuh"

namespace sla {

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

// Split form of the NCCL-path K_A (SLA_CG_SPLIT, as on one GPU and on the
// peer-memory path): a streaming pass takes the stop decision and forms
// p_new = p_old*beta + M^{-1} r once per owned row; the send rows are then
// packed from p_new, and the interior and boundary SpMVs gather p_new (and
// the received halo) instead of recomputing p for every entry.
template <typename T, bool PREC>
__global__ void __launch_bounds__(kBlock)
shard_cg_pform(int64_t n, const T *__restrict__ r, const T *__restrict__ dinv,
               const T *__restrict__ p_old, T *__restrict__ p_new, ShardState *st,
               const CgRed *R, long long k, long long every, double atol, double rtol) {
  if (*(volatile int *)&st->stopped) return;
  if (cg_stop(R, k, every, cg_tol(R, atol, rtol))) {
    if (blockIdx.x == 0 && threadIdx.x == 0) { st->stopped = 1; st->iters = k; }
    return;
  }
  ShardP<T, PREC> inner{r, dinv, p_old, (T)cg_beta(R, k)};
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    p_new[i] = inner((int32_t)i);
}

template <typename T>
__global__ void shard_pack_rows(const int32_t *__restrict__ idx, int64_t n,
                                const T *__restrict__ src, T *__restrict__ out,
                                const ShardState *st) {
  if (*(volatile const int *)&st->stopped) return;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = src[idx[i]];
}

template <typename T, bool HALO, int WS>
__global__ void __launch_bounds__(kBlock, kSpmvMinBlocks)
shard_cg_spmv_split(Sell<T> A, int32_t n_own, const T *__restrict__ p,
                    const T *__restrict__ phalo, T *__restrict__ Ap, ShardState *st, CgRed *R,
                    double *partials) {
  __shared__ double smem[kWarps];
  if (*(volatile int *)&st->stopped) return;
  PlainGather<T> inner{p};
  HaloGather<T, PlainGather<T>> g{inner, phalo, n_own};
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  double acc[1] = {0.0};
  for_each_slice<WS, !HALO>(A, warp, nwarps, lane, [&](int64_t s, int32_t sbase, int swidth) {
    T sum = HALO ? sell_row_at<WS>(A, s, sbase, swidth, lane, g)
                 : sell_row_at<WS>(A, s, sbase, swidth, lane, inner);
    const int64_t slot = s * 32 + lane;
    if (slot < A.n_slots) {
      const int32_t row = (int32_t)slot_row(A, slot);
      Ap[row] = sum;
      acc[0] += (double)__ldg(p + row) * (double)sum;
    }
  });
  if (last_block_sum<1, kBlock>(acc, partials, &st->counter[HALO ? 2 : 1], smem) &&
      threadIdx.x == 0) {
    if (!HALO) st->pap_int = acc[0];
    else R->pap[0] = st->pap_int + acc[0];
  }
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
  const int gi = kCgSplit ? spmv_grid()
                          : occupancy_grid((const void *)shard_cg_spmv<T, PREC, false, WS>);
  const int gb = kCgSplit ? spmv_grid()
                          : occupancy_grid((const void *)shard_cg_spmv<T, PREC, true,
                                                                       boundary_spec(WS)>);
  const int gu = occupancy_grid((const void *)shard_cg_update<T, PREC>);
  const int gp = occupancy_grid((const void *)shard_cg_pform<T, PREC>);
  SLA_TRY(shard_loop(cr, maxiter, every, &st->stopped, s, [&](int64_t k) -> int {
    T *p_old = (k & 1) ? pB : pA, *p_new = (k & 1) ? pA : pB;
    if (kCgSplit) {
      cudaEvent_t ev;
      profiler().begin(2, k, s, &ev);
      SLA_LAUNCH((shard_cg_pform<T, PREC>), gp, kBlock, 0, s, no, r, dinv, p_old, p_new, st, R,
                 (long long)k, (long long)every, atol, rtol);
      profiler().end(2, s, ev);
      SLA_LAUNCH(shard_pack_rows<T>, ns > 0 ? grid_for(ns) : 1, kBlock, 0, s, plan->send_index,
                 ns, (const T *)p_new, sendbuf, st);
      SLA_TRY(halo_enqueue<T>(ch, plan, sendbuf, recvbuf, s));
      profiler().begin(0, k, s, &ev);
      SLA_LAUNCH((shard_cg_spmv_split<T, false, WS>), gi, kBlock, 0, s, AI, (int32_t)no,
                 (const T *)p_new, hsrc, Ap, st, R, part[1]);
      profiler().end(0, s, ev);
      SLA_CUDA_TRY(cudaStreamWaitEvent(s, ch->ev_halo, 0));
      if (plan->halo_src && nh > 0)
        SLA_LAUNCH(halo_unpack_kernel<T>, grid_for(nh), kBlock, 0, s, recvbuf, plan->halo_src, nh,
                   halo, &st->stopped);
      SLA_LAUNCH((shard_cg_spmv_split<T, true, boundary_spec(WS)>), gb, kBlock, 0, s, AB,
                 (int32_t)no, (const T *)p_new, hsrc, Ap, st, R, part[2]);
      SLA_NCCL_TRY(ncclAllReduce(R->pap, R->pap, 1, ncclFloat64, ncclSum, cr->nccl, s));
      profiler().begin(1, k, s, &ev);
      SLA_LAUNCH((shard_cg_update<T, PREC>), gu, kBlock, 0, s, no, x, r, p_new, p_old, Ap, dinv,
                 st, R, part[3], (long long)k);
      profiler().end(1, s, ev);
      SLA_NCCL_TRY(ncclAllReduce(R->loc[k & 1], R->loc[k & 1], 2, ncclFloat64, ncclSum,
                                 cr->nccl, s));
      return SLA_OK;
    }
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
  SLA_TRY(sell_check(A_interior));
  SLA_TRY(sell_check(A_boundary));
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
  SLA_TRY(sell_check(AT));
  if (!c || !c->nccl || !plan_ok(plan) || !w_local) return SLA_ERR_INVALID;
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

}  // extern "C"
