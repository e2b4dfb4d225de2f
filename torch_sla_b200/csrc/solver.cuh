// Host-side polling of the device-resident Krylov loops (chunked launches
// with one chunk in flight) shared by the drivers.
#pragma once

#include "sell.cuh"

namespace sla {

struct HostPoll {
  int *flags = nullptr;  // pinned
  cudaEvent_t ev[2] = {nullptr, nullptr};
  bool ready = false;
  int init() {
    if (ready) return SLA_OK;
    SLA_CUDA_TRY(cudaHostAlloc((void **)&flags, 4 * sizeof(int), cudaHostAllocDefault));
    SLA_CUDA_TRY(cudaEventCreateWithFlags(&ev[0], cudaEventDisableTiming));
    SLA_CUDA_TRY(cudaEventCreateWithFlags(&ev[1], cudaEventDisableTiming));
    ready = true;
    return SLA_OK;
  }
};
HostPoll &host_poll();  // one per host thread (runtime.cu)

// Enqueue `body(iter)` for up to maxiter iterations in chunks, polling the
// device `done` flag with one chunk in flight.
template <typename Body>
int run_chunked(int64_t maxiter, int64_t chunk, const int *d_done, cudaStream_t s, Body body) {
  HostPoll &hp = host_poll();
  SLA_TRY(hp.init());
  int slot = 0;
  bool pending[2] = {false, false};
  for (int64_t it = 0; it < maxiter;) {
    int64_t c = maxiter - it < chunk ? maxiter - it : chunk;
    for (int64_t j = 0; j < c; ++j) SLA_TRY(body(it + j));
    it += c;
    SLA_CUDA_TRY(cudaMemcpyAsync(hp.flags + slot, d_done, sizeof(int), cudaMemcpyDeviceToHost, s));
    SLA_CUDA_TRY(cudaEventRecord(hp.ev[slot], s));
    pending[slot] = true;
    int other = slot ^ 1;
    if (pending[other]) {
      SLA_CUDA_TRY(cudaEventSynchronize(hp.ev[other]));
      pending[other] = false;
      if (hp.flags[other] != 0) break;
    }
    slot = other;
  }
  return SLA_OK;
}

template <typename T>
int spmv_launch(const sla_sell_t *A, const void *x, void *y, cudaStream_t s);

}  // namespace sla
