// Process-wide state of libsla_b200: launch counter, device properties,
// kernel-time sampling and status strings.
#include <map>
#include <mutex>
#include <tuple>
#include <unordered_map>

#include "solver.cuh"

namespace sla {

std::atomic<int64_t> g_launches{0};

const DeviceInfo &device_info() {
  static std::mutex mu;
  static std::unordered_map<int, DeviceInfo> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(dev);
  if (it != cache.end()) return it->second;
  DeviceInfo info;
  cudaDeviceGetAttribute(&info.sm_count, cudaDevAttrMultiProcessorCount, dev);
  cudaDeviceGetAttribute(&info.max_threads_per_sm,
                         cudaDevAttrMaxThreadsPerMultiProcessor, dev);
  int coop = 0;
  cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev);
  info.coop = coop != 0;
  if (info.sm_count <= 0) info.sm_count = 1;
  return cache.emplace(dev, info).first->second;
}

int occupancy_grid(const void *fn, int block, size_t smem) {
  static std::mutex mu;
  static std::map<std::tuple<int, const void *, int, size_t>, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  auto key = std::make_tuple(dev, fn, block, smem);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, block, smem) != cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  const int sms = device_info().sm_count;
  int cap = sms * 8;
  int grid = per_sm * sms;
  if (grid > cap) grid = cap;
  cache.emplace(key, grid);
  return grid;
}

static thread_local HostPoll t_poll;
HostPoll &host_poll() { return t_poll; }

Profiler &profiler() {
  static Profiler p;
  return p;
}

cudaEvent_t Profiler::get_event() {
  if (!pool.empty()) {
    cudaEvent_t e = pool.back();
    pool.pop_back();
    return e;
  }
  cudaEvent_t e;
  cudaEventCreate(&e);
  return e;
}

void Profiler::begin(int cls, int64_t iter, cudaStream_t s, cudaEvent_t *a) {
  *a = nullptr;
  if (!enabled || cls < 0 || cls > 3) return;
  if (sample_every > 1 && (iter % sample_every) != 0) return;
  *a = get_event();
  cudaEventRecord(*a, s);
}

void Profiler::end(int cls, cudaStream_t s, cudaEvent_t a) {
  if (!a) return;
  cudaEvent_t b = get_event();
  cudaEventRecord(b, s);
  pending.push_back({a, b, cls});
}

void Profiler::resolve() {
  for (auto &p : pending) {
    float ms = 0.f;
    if (cudaEventSynchronize(p.b) == cudaSuccess &&
        cudaEventElapsedTime(&ms, p.a, p.b) == cudaSuccess) {
      total_ms[p.cls] += ms;
      launches[p.cls] += 1;
    }
    pool.push_back(p.a);
    pool.push_back(p.b);
  }
  pending.clear();
}

}  // namespace sla

extern "C" {

int sla_abi_version(void) { return SLA_ABI_VERSION; }

const char *sla_status_string(int status) {
  switch (status) {
    case SLA_OK: return "ok";
    case SLA_NOT_CONVERGED: return "did not converge within maxiter";
    case SLA_BREAKDOWN: return "Krylov breakdown guard fired";
    case SLA_ERR_INVALID: return "invalid argument";
    case SLA_ERR_CUDA: return "CUDA runtime error";
    case SLA_ERR_NCCL: return "NCCL error";
    case SLA_ERR_TIMEOUT: return "bounded device wait timed out";
    case SLA_ERR_UNSUPPORTED: return "unsupported problem shape";
    case SLA_ERR_WORKSPACE: return "workspace too small";
    case SLA_ERR_INDEX: return "COO index outside the matrix shape";
    default: return "unknown status";
  }
}

int64_t sla_kernel_launch_count(void) {
  return sla::g_launches.load(std::memory_order_relaxed);
}

int sla_profile_enable(int enable, int sample_every) {
  auto &p = sla::profiler();
  p.resolve();
  p.enabled = enable != 0;
  p.sample_every = sample_every > 0 ? sample_every : 1;
  for (int i = 0; i < 4; ++i) { p.total_ms[i] = 0; p.launches[i] = 0; }
  return SLA_OK;
}

int sla_profile_read(int kernel_class, double *total_ms, int64_t *launches) {
  if (kernel_class < 0 || kernel_class > 3 || !total_ms || !launches)
    return SLA_ERR_INVALID;
  auto &p = sla::profiler();
  p.resolve();
  *total_ms = p.total_ms[kernel_class];
  *launches = p.launches[kernel_class];
  return SLA_OK;
}

}  // extern "C"
