// Block copy engine of the weight streamer: one host -> device copy per block into a ring slot, ordered on the device.
//
// Reference behaviour (h3turbo/h3/stream.py:1-21, :333-362, :376-437): a copy into slot s first waits (on the copy
// stream) for the slot's `done` event, recorded by release() on the compute stream after the last kernel that reads the
// slot; acquire() makes the compute stream wait for the slot's `ready` event, recorded after the copy.  Nothing blocks
// the host except the staging path, which must not overwrite a page-locked staging buffer a copy is still reading.
//
// Sources: mode 0 "direct" -- page-locked memory (registered file mapping or a pinned copy): one cudaMemcpyAsync;
// mode 1 "staged" -- pageable memory (the file mapping): a multi-threaded memcpy into one of the engine's page-locked
// staging buffers, then an async copy from it; mode 2 "pageable" -- cudaMemcpyAsync straight from pageable memory (the
// driver stages it; the call returns when the source has been read).
#pragma once

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

#include "h3b_common.cuh"

namespace h3b {

struct StreamEngine {
  int device = 0;
  cudaStream_t copy = nullptr;
  std::vector<cudaEvent_t> ready, done;
  std::vector<char> done_set;
  std::vector<void*> staging;
  std::vector<cudaEvent_t> stage_ev;
  std::vector<char> stage_used;
  size_t stage_bytes = 0;
  int stage_next = 0;
  int memcpy_threads = 8;
  std::mutex mu;
  std::atomic<unsigned long long> copies{0}, bytes{0}, busy_ns{0};
};

static double now_s() {
  return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

// Poll an event until it completes or `timeout_s` passes (never an unbounded wait).
static int event_wait(cudaEvent_t ev, double timeout_s, const char* what) {
  const double t0 = now_s();
  for (int spin = 0;; ++spin) {
    const cudaError_t e = cudaEventQuery(ev);
    if (e == cudaSuccess) return H3B_OK;
    if (e != cudaErrorNotReady) return cuda_fail(e, what);
    if (now_s() - t0 > timeout_s) return fail(H3B_ERR_DEVICE, std::string(what) + ": timed out");
    if (spin > 64) std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

static void parallel_memcpy(void* dst, const void* src, size_t n, int threads) {
  const size_t min_chunk = 8u << 20;
  int t = static_cast<int>(std::min<size_t>(static_cast<size_t>(std::max(threads, 1)), std::max<size_t>(1, n / min_chunk)));
  if (t <= 1) {
    std::memcpy(dst, src, n);
    return;
  }
  const size_t chunk = (n / t + 4095) / 4096 * 4096;
  std::vector<std::thread> pool;
  pool.reserve(t);
  for (int i = 0; i < t; ++i) {
    const size_t a = std::min(n, static_cast<size_t>(i) * chunk), b = std::min(n, a + chunk);
    if (a >= b) break;
    pool.emplace_back([=] { std::memcpy(static_cast<char*>(dst) + a, static_cast<const char*>(src) + a, b - a); });
  }
  for (auto& th : pool) th.join();
}

static void engine_free(StreamEngine* e) {
  if (!e) return;
  cudaSetDevice(e->device);
  if (e->copy) cudaStreamSynchronize(e->copy);
  for (auto ev : e->ready) if (ev) cudaEventDestroy(ev);
  for (auto ev : e->done) if (ev) cudaEventDestroy(ev);
  for (auto ev : e->stage_ev) if (ev) cudaEventDestroy(ev);
  for (auto p : e->staging) if (p) cudaFreeHost(p);
  if (e->copy) cudaStreamDestroy(e->copy);
  delete e;
}

}  // namespace h3b
