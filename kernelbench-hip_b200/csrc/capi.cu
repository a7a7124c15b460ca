// capi.cu — library-level C ABI: version, status strings, thread-local error
// text and cached per-device properties.
#include <stdarg.h>
#include <stdio.h>

#include "kb_common.cuh"

#define KB_VERSION_MAJOR 0
#define KB_VERSION_MINOR 1
#define KB_VERSION_PATCH 0

namespace kb {

static thread_local char g_err[512] = "";

int set_error(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return status;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(KB_ERR_CUDA, "%s launch: %s", what, cudaGetErrorString(e));
  return KB_OK;
}

namespace {
constexpr int kMaxDev = 64;
int g_sms[kMaxDev] = {0};
int g_smem[kMaxDev] = {0};

int current_device() {
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess) return 0;
  return (d >= 0 && d < kMaxDev) ? d : 0;
}
}  // namespace

int sm_count() {
  int d = current_device();
  if (g_sms[d] == 0) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, d);
    g_sms[d] = v > 0 ? v : 148;
  }
  return g_sms[d];
}

int max_smem_optin() {
  int d = current_device();
  if (g_smem[d] == 0) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, d);
    g_smem[d] = v > 0 ? v : 48 * 1024;
  }
  return g_smem[d];
}

}  // namespace kb

extern "C" {

int kb_version(void) {
  return KB_VERSION_MAJOR * 10000 + KB_VERSION_MINOR * 100 + KB_VERSION_PATCH;
}

const char* kb_status_string(int status) {
  switch (status) {
    case KB_OK: return "ok";
    case KB_ERR_INVALID_ARG: return "invalid argument";
    case KB_ERR_UNSUPPORTED: return "unsupported shape";
    case KB_ERR_WORKSPACE: return "workspace too small";
    case KB_ERR_CUDA: return "CUDA runtime error";
    case KB_ERR_DEVICE: return "unsupported device";
    default: return "unknown status";
  }
}

const char* kb_last_error(void) { return kb::g_err; }

int kb_device_sm_count(int device) {
  int v = -1;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return -1;
  return v;
}

}  // extern "C"
