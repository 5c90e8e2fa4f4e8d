// Error reporting and device queries shared by every C-ABI entry point.
#include <mutex>

#include "qx_b200.h"
#include "qx_common.cuh"

namespace qx {

static thread_local char g_last_error[1024] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(QX_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return QX_OK;
}

int device_sm_count() {
  static std::mutex mu;
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lk(mu);
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

}  // namespace qx

extern "C" const char* qx_last_error(void) { return qx::g_last_error; }

extern "C" const char* qx_version(void) { return "qextract_infer_b200 0.1.0 (sm_100a)"; }

extern "C" int qx_copy_async(void* dst, const void* src, size_t bytes, qx_stream_t stream) {
  if (bytes == 0) return QX_OK;
  QX_REQUIRE(dst && src, "copy_async: null pointer");
  QX_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, reinterpret_cast<cudaStream_t>(stream)),
              "copy_async");
  return QX_OK;
}
