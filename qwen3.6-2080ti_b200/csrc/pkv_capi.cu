// Library-level plumbing of the C ABI: per-thread last-error message, call counters, version.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <string>

#include "pkv_common.cuh"

namespace pkv {

namespace {
thread_local std::string g_last_error;
std::atomic<int64_t> g_stats[kNumStats];
}  // namespace

void set_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
}

void clear_error() { g_last_error.clear(); }

void bump_stat(int index) {
  if (index >= 0 && index < kNumStats) g_stats[index].fetch_add(1, std::memory_order_relaxed);
}

int cuda_status(cudaError_t err, const char* what) {
  if (err == cudaSuccess) return PKV_OK;
  set_error("%s: CUDA error %d (%s)", what, static_cast<int>(err), cudaGetErrorString(err));
  return PKV_ERR_CUDA;
}

}  // namespace pkv

extern "C" {

const char* pkv_last_error(void) { return pkv::g_last_error.c_str(); }

int pkv_abi_version(void) { return 1; }

int pkv_stats(int64_t* out, int n) {
  if (out != nullptr) {
    for (int i = 0; i < n && i < pkv::kNumStats; ++i) out[i] = pkv::g_stats[i].load(std::memory_order_relaxed);
  }
  return pkv::kNumStats;
}

void pkv_reset_stats(void) {
  for (int i = 0; i < pkv::kNumStats; ++i) pkv::g_stats[i].store(0, std::memory_order_relaxed);
}

}  // extern "C"
