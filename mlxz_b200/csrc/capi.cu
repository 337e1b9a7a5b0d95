// Error plumbing and cached device properties behind the C ABI.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace mz {

namespace {
thread_local char t_msg[512] = "";
thread_local int t_code = MZ_OK;

std::once_flag g_sm_once[kMaxDevices];
int g_sm_count[kMaxDevices];
}  // namespace

int fail(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_msg, sizeof(t_msg), fmt, ap);
  va_end(ap);
  t_code = code;
  return code;
}

int cuda_fail(cudaError_t e, const char *what) {
  return fail(MZ_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

int dtype_bytes(int dtype) {
  switch (dtype) {
    case MZ_DTYPE_F16:
    case MZ_DTYPE_BF16:
      return 2;
    case MZ_DTYPE_F32:
      return 4;
    default:
      return 0;
  }
}

int current_device() {
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess) return -1;
  return d;
}

int sm_count(int device) {
  if (device < 0 || device >= kMaxDevices) return 0;
  std::call_once(g_sm_once[device], [device]() {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) n = 0;
    g_sm_count[device] = n;
  });
  return g_sm_count[device];
}

}  // namespace mz

extern "C" int mz_abi_version(void) { return 6; }

extern "C" int mz_last_error(char *buf, size_t len) {
  if (buf && len) {
    strncpy(buf, mz::t_msg, len - 1);
    buf[len - 1] = '\0';
  }
  return mz::t_code;
}
