// C-ABI utilities: error strings, the device status word, cached device
// attributes and the library version.  Every entry point returns AK_OK (0) or
// a negative AK_ERR_* code and leaves a message for ak_last_error(); nothing in
// the library aborts or traps.
#include "ak_common.cuh"

#include <cstdarg>
#include <cstdio>
#include <mutex>

namespace ak {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int launch_status(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: launch failed: %s", what, cudaGetErrorString(e));
    return AK_ERR_LAUNCH;
  }
  return AK_OK;
}

__device__ int g_status = 0;

static DeviceInfo g_info[kMaxDevices];
static std::once_flag g_once[kMaxDevices];

int current_device() {
  int dev = 0;
  cudaGetDevice(&dev);
  return (dev < 0 || dev >= kMaxDevices) ? 0 : dev;
}

const DeviceInfo& device_info() {
  const int dev = current_device();
  std::call_once(g_once[dev], [dev]() {
    DeviceInfo& d = g_info[dev];
    cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaDeviceGetAttribute(&d.l2_bytes, cudaDevAttrL2CacheSize, dev);
    cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (d.sm_count <= 0) d.sm_count = 148;
  });
  return g_info[dev];
}

}  // namespace ak

extern "C" const char* ak_last_error(void) { return ak::g_err; }

extern "C" int ak_version(void) { return AK_VERSION; }

extern "C" int ak_device_status(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, ak::g_status, sizeof(int)) != cudaSuccess) {
    ak::set_error("ak_device_status: %s", cudaGetErrorString(cudaGetLastError()));
    return AK_ERR_LAUNCH;
  }
  if (clear && v) {
    int z = 0;
    cudaMemcpyToSymbol(ak::g_status, &z, sizeof(int));
  }
  return v;
}

extern "C" int ak_sm_count(void) { return ak::device_info().sm_count; }
