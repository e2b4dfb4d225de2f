// Shared device/host utilities of libsla_b200: status plumbing, launch
// accounting, deterministic fp64 reductions, a bounded grid barrier and
// rounding-explicit arithmetic.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstdio>
#include <vector>

#include "../../include/sla_b200.h"

namespace sla {

constexpr int kBlock = 256;           // threads per block of the streaming kernels
constexpr int kWarps = kBlock / 32;   // warps per block
constexpr unsigned kFull = 0xffffffffu;
// Bound of every device-side wait (grid barrier, flags written by other
// GPUs), measured on the GPU's nanosecond global timer: after it the kernel
// records a timeout status and returns.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

// ----------------------------------------------------------------- host side
extern std::atomic<int64_t> g_launches;

struct DeviceInfo {
  int sm_count = 0;
  int max_threads_per_sm = 0;
  bool coop = false;
};
const DeviceInfo &device_info();

// Profiling of the kernel class that carries the SpMV of a solver.
struct Profiler {
  bool enabled = false;
  int sample_every = 8;
  double total_ms[4] = {0, 0, 0, 0};
  int64_t launches[4] = {0, 0, 0, 0};
  struct Pending { cudaEvent_t a, b; int cls; };
  std::vector<Pending> pending;
  std::vector<cudaEvent_t> pool;
  cudaEvent_t get_event();
  void begin(int cls, int64_t iter, cudaStream_t s, cudaEvent_t *a);
  void end(int cls, cudaStream_t s, cudaEvent_t a);
  void resolve();  // after a stream sync
};
Profiler &profiler();

#define SLA_CUDA_TRY(expr)                                                   \
  do {                                                                       \
    cudaError_t _e = (expr);                                                 \
    if (_e != cudaSuccess) {                                                 \
      fprintf(stderr, "[sla_b200] %s failed: %s (%s:%d)\n", #expr,           \
              cudaGetErrorString(_e), __FILE__, __LINE__);                   \
      return SLA_ERR_CUDA;                                                   \
    }                                                                        \
  } while (0)

#define SLA_TRY(expr)                                                        \
  do {                                                                       \
    int _s = (expr);                                                         \
    if (_s < 0) return _s;                                                   \
  } while (0)

// Launch + accounting + immediate launch-error check.
#define SLA_LAUNCH(kernel, grid, block, smem, stream, ...)                   \
  do {                                                                       \
    kernel<<<(grid), (block), (smem), (stream)>>>(__VA_ARGS__);              \
    ::sla::g_launches.fetch_add(1, std::memory_order_relaxed);               \
    cudaError_t _e = cudaGetLastError();                                     \
    if (_e != cudaSuccess) {                                                 \
      fprintf(stderr, "[sla_b200] launch of %s failed: %s\n", #kernel,       \
              cudaGetErrorString(_e));                                       \
      return SLA_ERR_CUDA;                                                   \
    }                                                                        \
  } while (0)

inline int grid_for(int64_t work_items, int per_block = kBlock,
                    int blocks_per_sm = 8) {
  const DeviceInfo &d = device_info();
  int64_t want = (work_items + per_block - 1) / per_block;
  int64_t cap = (int64_t)d.sm_count * blocks_per_sm;
  if (want < 1) want = 1;
  return (int)(want < cap ? want : cap);
}

// Upper bound of the solver grids (sizes the per-block partial buffers).
inline int solver_grid() { return device_info().sm_count * 8; }

// One wave of resident blocks of `fn` on the current device (cached per
// kernel): grid-stride kernels get no tail wave, and the grid (hence the
// reduction order) is the same in every launch.
int occupancy_grid(const void *fn, int block = kBlock, size_t smem = 0);

// True when every pointer is 16-byte aligned (vectorised streaming paths).
inline bool aligned16() { return true; }
template <typename P, typename... R>
inline bool aligned16(const P *p, R... rest) {
  return (((uintptr_t)p) & 15u) == 0 && aligned16(rest...);
}

// True when every pointer is 8-byte aligned (float2 paths).
inline bool aligned8() { return true; }
template <typename P, typename... R>
inline bool aligned8(const P *p, R... rest) {
  return (((uintptr_t)p) & 7u) == 0 && aligned8(rest...);
}

inline size_t align_up(size_t x, size_t a = 256) { return (x + a - 1) / a * a; }

// Carve sub-buffers out of a caller-provided workspace.
struct Carver {
  char *base;
  size_t cap;
  size_t off = 0;
  bool ok = true;
  // the carved arrays are 256-byte aligned offsets from the base, so the
  // base must be 16-byte aligned for the vector loads (cudaMalloc and
  // torch allocations are 256-byte aligned)
  Carver(void *b, size_t c) : base((char *)b), cap(c), ok(((uintptr_t)b & 15u) == 0) {}
  template <typename U>
  U *take(size_t count) {
    size_t bytes = align_up(count * sizeof(U));
    if (off + bytes > cap) { ok = false; return nullptr; }
    U *p = (U *)(base + off);
    off += bytes;
    return p;
  }
};
// Size-only twin of Carver, for the *_workspace queries.
struct Sizer {
  size_t off = 0;
  template <typename U>
  void take(size_t count) { off += align_up(count * sizeof(U)); }
};

// ---------------------------------------------------------------- device side
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
template <typename T> __device__ __forceinline__ T mul_rn(T a, T b);
template <> __device__ __forceinline__ double mul_rn(double a, double b) { return __dmul_rn(a, b); }
template <> __device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
template <typename T> __device__ __forceinline__ T add_rn(T a, T b);
template <> __device__ __forceinline__ double add_rn(double a, double b) { return __dadd_rn(a, b); }
template <> __device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }
template <typename T> __device__ __forceinline__ T sub_rn(T a, T b);
template <> __device__ __forceinline__ double sub_rn(double a, double b) { return __dsub_rn(a, b); }
template <> __device__ __forceinline__ float sub_rn(float a, float b) { return __fsub_rn(a, b); }

// Streaming (evict-first) loads for matrix entries that are read once per
// sweep, so the L2 keeps the gathered vectors instead.
template <typename U> __device__ __forceinline__ U ld_stream(const U *p) { return __ldcs(p); }
// L1-bypassing loads for data written by other blocks of the same launch.
template <typename U> __device__ __forceinline__ U ld_l2(const U *p) { return __ldcg(p); }
__device__ __forceinline__ void prefetch_l2(const void *p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// Deterministic block sum of NV doubles (fixed shuffle + fixed smem order).
// Every thread returns with v[] holding the block total. smem: NV*BS/32.
template <int NV, int BS>
__device__ __forceinline__ void block_sum(double (&v)[NV], double *smem) {
  constexpr int NW = BS / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v[k] += __shfl_xor_sync(kFull, v[k], o);
  }
  if (lane == 0) {
#pragma unroll
    for (int k = 0; k < NV; ++k) smem[k * NW + warp] = v[k];
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    double t = 0.0;
    // every warp reduces the same NW values in the same order
    for (int w = 0; w < NW; ++w) t += smem[k * NW + w];
    v[k] = t;
  }
  __syncthreads();
}

// Block partial -> per-launch partial array; the last block to finish sums
// all partials in block order and returns true (all its threads), with the
// grid totals in v[]. partials layout: [NV][gridDim.x]. The counter is reset
// by that last block so the next launch can reuse it.
template <int NV, int BS>
__device__ __forceinline__ bool last_block_sum(double (&v)[NV], double *partials,
                                               unsigned *counter, double *smem) {
  __shared__ unsigned s_last;
  block_sum<NV, BS>(v, smem);
  const unsigned G = gridDim.x;
  if (threadIdx.x == 0) {
#pragma unroll
    for (int k = 0; k < NV; ++k) partials[k * G + blockIdx.x] = v[k];
    __threadfence();
    unsigned t = atomicAdd(counter, 1u);
    s_last = (t == G - 1) ? 1u : 0u;
  }
  __syncthreads();
  if (!s_last) return false;
  __threadfence();
  double acc[NV];
#pragma unroll
  for (int k = 0; k < NV; ++k) acc[k] = 0.0;
  // fixed order: thread t sums blocks t, t+BS, ... then the fixed block sum
  for (unsigned i = threadIdx.x; i < G; i += BS) {
#pragma unroll
    for (int k = 0; k < NV; ++k) acc[k] += ld_l2(partials + k * G + i);
  }
  block_sum<NV, BS>(acc, smem);
#pragma unroll
  for (int k = 0; k < NV; ++k) v[k] = acc[k];
  if (threadIdx.x == 0) *counter = 0u;
  return true;
}

// Grid barrier for cooperative (co-resident) launches with a bounded spin.
struct GridBarrier {
  unsigned count;
  unsigned gen;
  int err;
  int pad;
};

__device__ __forceinline__ bool grid_sync(GridBarrier *gb) {
  __syncthreads();
  if (threadIdx.x == 0) {
    volatile unsigned *vgen = &gb->gen;
    volatile int *verr = &gb->err;
    const unsigned g = *vgen;
    __threadfence();
    const unsigned arrived = atomicAdd(&gb->count, 1u);
    if (arrived == gridDim.x - 1) {
      atomicExch(&gb->count, 0u);
      __threadfence();
      atomicAdd(&gb->gen, 1u);
    } else {
      const unsigned long long t0 = global_ns();
      while (*vgen == g) {
        if (*verr) break;
        if (global_ns() - t0 > kWaitLimitNs) { atomicExch(&gb->err, 1); break; }
        __nanosleep(40);
      }
    }
    __threadfence();
  }
  __syncthreads();
  return *(volatile int *)&gb->err == 0;
}

}  // namespace sla
