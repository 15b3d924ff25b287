// Library-wide C-ABI entry points: version, last error, PDL switch.
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <utility>

#include "afb_launch.h"

namespace afb {

namespace {
thread_local std::string g_last_error;
int g_pdl = -1;  // -1: read AFB_PDL from the environment on first use
}  // namespace

void set_error(const std::string& msg) { g_last_error = msg; }
const std::string& last_error() { return g_last_error; }

const DeviceInfo& device_info() {
  static std::mutex mu;
  static std::map<int, DeviceInfo> cache;
  int dev = 0;
  DeviceInfo bad;
  bad.error = cudaGetDevice(&dev);
  if (bad.error != cudaSuccess) {
    static thread_local DeviceInfo err;
    err = bad;
    return err;
  }
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(dev);
  if (it != cache.end()) return it->second;
  DeviceInfo info;
  int smem = 0;
  info.error = cudaDeviceGetAttribute(&info.sms, cudaDevAttrMultiProcessorCount, dev);
  if (info.error == cudaSuccess)
    info.error = cudaDeviceGetAttribute(&smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  info.max_smem_optin = static_cast<size_t>(smem);
  return cache.emplace(dev, info).first->second;
}

cudaError_t ensure_smem_raw(const void* kernel, size_t bytes, bool max_shared) {
  static std::mutex mu;
  struct State {
    size_t bytes = 0;
    bool carveout = false;
  };
  static std::map<std::pair<int, const void*>, State> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  State& have = done[{dev, kernel}];
  if (have.bytes < bytes) {
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
    if (e != cudaSuccess) return e;
    have.bytes = bytes;
  }
  if (max_shared && !have.carveout) {
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return e;
    have.carveout = true;
  }
  return cudaSuccess;
}

bool pdl_enabled() {
  if (g_pdl < 0) {
    const char* env = std::getenv("AFB_PDL");
    g_pdl = (env != nullptr && std::strcmp(env, "0") == 0) ? 0 : 1;
  }
  return g_pdl != 0;
}

}  // namespace afb

extern "C" int afb_abi_version(void) { return 1; }

// Device status word of the current device (0: no bounded wait ever gave
// up): the OR of every file's word, each cleared after reading if `clear`.
static int device_status(int* status, bool clear, const char* name) {
  using Reader = cudaError_t (*)(int*, bool);
  static const Reader readers[] = {afb::read_status_adaln_fwd, afb::read_status_headnorm_fwd,
                                   afb::read_status_headnorm_bwd, afb::read_status_adaln_bwd,
                                   afb::read_status_rms, afb::read_status_probe};
  int all = 0;
  for (Reader r : readers) {
    int v = 0;
    const cudaError_t e = r(&v, clear);
    if (e != cudaSuccess) {
      afb::set_error(std::string(name) + ": " + cudaGetErrorString(e));
      return static_cast<int>(e);
    }
    all |= v;
  }
  *status = all;
  return 0;
}

extern "C" int afb_device_status(int* status) { return device_status(status, false, "afb_device_status"); }

extern "C" int afb_take_device_status(int* status) {
  return device_status(status, true, "afb_take_device_status");
}

extern "C" const char* afb_last_error(void) { return afb::g_last_error.c_str(); }

extern "C" void afb_clear_error(void) { afb::g_last_error.clear(); }

extern "C" void afb_set_pdl(int enabled) { afb::g_pdl = enabled ? 1 : 0; }

extern "C" int afb_get_pdl(void) { return afb::pdl_enabled() ? 1 : 0; }
