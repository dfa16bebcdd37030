// The error channel and version of the C ABI.
#include <cstdarg>
#include <cstdio>

#include "ekv_common.cuh"

namespace ekv {

namespace {
thread_local char g_error[512] = "";
}

int fail(int code, const char* fmt, ...) {
  va_list args;
  va_start(args, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, args);
  va_end(args);
  return code;
}

void clear_error() { g_error[0] = '\0'; }

int check_launch(const char* what) {
  const cudaError_t err = cudaGetLastError();
  if (err == cudaSuccess) return EKV_OK;
  return fail(EKV_ECUDA, "%s: %s", what, cudaGetErrorString(err));
}

int current_device(int* device) {
  *device = 0;
  const cudaError_t err = cudaGetDevice(device);
  if (err != cudaSuccess) return fail(EKV_ECUDA, "cudaGetDevice: %s", cudaGetErrorString(err));
  if (*device < 0 || *device >= kMaxDevices)
    return fail(EKV_ENOTSUP, "device %d: this library serves devices 0 to %d", *device, kMaxDevices - 1);
  return EKV_OK;
}

}  // namespace ekv

extern "C" const char* ekv_last_error_string(void) { return ekv::g_error; }

extern "C" int ekv_abi_version(void) { return 7; }
