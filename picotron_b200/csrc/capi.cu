// Host-side plumbing of the C ABI: thread-local error strings, pointer validation,
// the per-device SM-count cache and the capability probe.
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "common.cuh"

namespace pt {

namespace {
thread_local char g_last_error[512] = "";

constexpr int kMaxDevices = 64;
// Write-once cache: 0 = not yet queried. Guarded by g_sm_mutex for the first write.
int g_sm_count[kMaxDevices] = {0};
std::mutex g_sm_mutex;
}  // namespace

int set_error(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

int ok() {
  g_last_error[0] = '\0';
  return PT_OK;
}

int current_device_info(int* device, int* sm_count) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(PT_ERR_DEVICE, "no CUDA device: %s", cudaGetErrorString(e));
  }
  if (dev < 0 || dev >= kMaxDevices)
    return set_error(PT_ERR_DEVICE, "device index %d out of range", dev);
  int sms = 0;
  {
    std::lock_guard<std::mutex> lock(g_sm_mutex);
    sms = g_sm_count[dev];
    if (sms == 0) {
      e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      if (e != cudaSuccess || sms <= 0) {
        cudaGetLastError();
        return set_error(PT_ERR_DEVICE, "cannot query SM count of device %d", dev);
      }
      g_sm_count[dev] = sms;
    }
  }
  if (device) *device = dev;
  if (sm_count) *sm_count = sms;
  return PT_OK;
}

int check_device_ptr(const void* p, const char* name) {
  if (p == nullptr) return set_error(PT_ERR_INVALID_ARGUMENT, "%s is NULL", name);
  cudaPointerAttributes attr;
  cudaError_t e = cudaPointerGetAttributes(&attr, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(PT_ERR_DEVICE, "%s is not a CUDA pointer: %s", name, cudaGetErrorString(e));
  }
  if (attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged)
    return set_error(PT_ERR_DEVICE, "%s is not device memory", name);
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return set_error(PT_ERR_DEVICE, "no current CUDA device");
  }
  if (attr.type == cudaMemoryTypeDevice && attr.device != dev)
    return set_error(PT_ERR_DEVICE, "%s lives on device %d but device %d is current", name,
                     attr.device, dev);
  return PT_OK;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return set_error(PT_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return ok();
}

}  // namespace pt

extern "C" {

int pt_abi_version(void) { return PT_ABI_VERSION; }

const char* pt_last_error(void) { return pt::g_last_error; }

int pt_probe(int device, int* cc_major, int* cc_minor, int* sm_count) {
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return pt::set_error(PT_ERR_DEVICE, "no CUDA device: %s", cudaGetErrorString(e));
  }
  if (device < 0 || device >= count)
    return pt::set_error(PT_ERR_DEVICE, "device %d does not exist (%d visible)", device, count);
  int major = 0, minor = 0, sms = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess ||
      cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) {
    cudaGetLastError();
    return pt::set_error(PT_ERR_DEVICE, "cannot query device %d", device);
  }
  if (cc_major) *cc_major = major;
  if (cc_minor) *cc_minor = minor;
  if (sm_count) *sm_count = sms;
  if (major != 10 || minor != 0)
    return pt::set_error(PT_ERR_DEVICE,
                         "device %d has compute capability %d.%d; this library is built for "
                         "sm_100a (compute capability 10.0) only",
                         device, major, minor);
  return pt::ok();
}

}  // extern "C"
