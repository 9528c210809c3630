// Library-level C ABI: error reporting, launch accounting, device status.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "common.cuh"

namespace {
thread_local char g_last_error[512] = "";
std::atomic<uint64_t> g_launches{0};
std::mutex g_status_mu;
constexpr int kMaxDevices = 64;
int* g_status[kMaxDevices] = {nullptr};
}  // namespace

namespace ps_host {

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: launch failed: %s", what, cudaGetErrorString(e));
    return PS_ERR_CUDA;
  }
  return PS_OK;
}

void count_launch(int n) { g_launches.fetch_add(static_cast<uint64_t>(n), std::memory_order_relaxed); }

// One block of PS_TU_COUNT status words per device, allocated on first use
// (before any graph capture: the model wrappers touch it at construction).
int* status_word(int tu) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_status_mu);
  if (!g_status[dev]) {
    int* p = nullptr;
    if (cudaMalloc(&p, sizeof(int) * PS_TU_COUNT) != cudaSuccess) return nullptr;
    if (cudaMemset(p, 0, sizeof(int) * PS_TU_COUNT) != cudaSuccess) return nullptr;
    g_status[dev] = p;
  }
  return g_status[dev] + tu;
}

bool pdl_enabled() {
  static const bool v = [] {
    const char* e = std::getenv("PS_PDL");
    return !(e && e[0] == '0');
  }();
  return v;
}

}  // namespace ps_host

extern "C" {

int ps_abi_version(void) { return 1; }

const char* ps_last_error(void) { return g_last_error; }

uint64_t ps_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int ps_device_status(int* code, int clear, ps_stream_t stream) {
  if (!code) {
    ps_host::set_error("ps_device_status: code is NULL");
    return PS_ERR_INVALID;
  }
  *code = 0;
  int* base = ps_host::status_word(0);
  if (!base) {
    ps_host::set_error("ps_device_status: no device status word");
    return PS_ERR_CUDA;
  }
  int host[PS_TU_COUNT];
  cudaError_t e = cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(stream));
  if (e == cudaSuccess) e = cudaMemcpy(host, base, sizeof(host), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && clear) e = cudaMemset(base, 0, sizeof(host));
  if (e != cudaSuccess) {
    ps_host::set_error("ps_device_status: %s", cudaGetErrorString(e));
    return PS_ERR_CUDA;
  }
  for (int i = 0; i < PS_TU_COUNT; ++i)
    if (host[i]) {
      *code = host[i];
      break;
    }
  return PS_OK;
}

}  // extern "C"
