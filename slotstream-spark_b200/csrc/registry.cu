// Library-wide entry points: version, device check, shared-memory registry.
#include <cuda_runtime.h>
#include <string.h>

#include <atomic>
#include <mutex>
#include <string>
#include <unordered_map>

#include "../../include/slotstream_b200.h"
#include "registry.h"

namespace {
std::mutex g_mu;
std::atomic<int64_t> g_barrier_ns{250LL * 1000 * 1000};   // grid-barrier wait bound of the cooperative kernels
std::unordered_map<std::string, int>& table() {
  static std::unordered_map<std::string, int> t;
  return t;
}
}  // namespace

void ssb_note_smem_bytes(const char* name, int bytes) {
  std::lock_guard<std::mutex> g(g_mu);
  table()[name] = bytes;
}

extern "C" int ssb_kernel_smem(const char* name) {
  if (!name) return -1;
  std::lock_guard<std::mutex> g(g_mu);
  auto it = table().find(name);
  return it == table().end() ? -1 : it->second;
}

extern "C" const char* ssb_version(void) { return "slotstream_b200 0.1.0 (sm_100a)"; }

extern "C" int ssb_device_check(void) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    (void)cudaGetLastError();
    return SSB_ENODEVICE;
  }
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  return (major == 10 && minor == 0) ? SSB_OK : SSB_ENODEVICE;
}

uint64_t ssb_barrier_wait_ns() { return (uint64_t)g_barrier_ns.load(std::memory_order_relaxed); }

extern "C" int ssb_set_wait_limit_ns(int64_t ns) {
  if (ns < 0) return SSB_EINVAL;
  g_barrier_ns.store(ns, std::memory_order_relaxed);
  return SSB_OK;
}
