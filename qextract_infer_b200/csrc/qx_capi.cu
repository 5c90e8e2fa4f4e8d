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

namespace {
struct TraceTarget {
  unsigned long long* buf = nullptr;
  int next = 0, launches = 0;
};
std::mutex g_trace_mu;
TraceTarget g_trace[2];  // QX_TRACE_GEMV, QX_TRACE_DECODE_ATTENTION
}  // namespace

unsigned long long* trace_next(int kernel, int* launch) {
#ifdef QX_TRACE
  std::lock_guard<std::mutex> lk(g_trace_mu);
  TraceTarget& t = g_trace[kernel];
  if (t.buf == nullptr || t.next >= t.launches) return nullptr;
  *launch = t.next++;
  return t.buf;
#else
  (void)kernel;
  *launch = 0;
  return nullptr;
#endif
}

}  // namespace qx

extern "C" int qx_trace_launches(int kernel, void* buf, int launches) {
  QX_REQUIRE(kernel == QX_TRACE_GEMV || kernel == QX_TRACE_DECODE_ATTENTION, "trace: unknown kernel %d",
             kernel);
  QX_REQUIRE(buf == nullptr || launches > 0, "trace: launches=%d", launches);
#ifdef QX_TRACE
  std::lock_guard<std::mutex> lk(qx::g_trace_mu);
  qx::g_trace[kernel].buf = static_cast<unsigned long long*>(buf);
  qx::g_trace[kernel].next = 0;
  qx::g_trace[kernel].launches = buf ? launches : 0;
  return QX_OK;
#else
  return qx::fail(QX_ERR_UNSUPPORTED,
                  "trace: this library was built without tracing (profiling build: "
                  "python -m qextract_infer_b200.build --trace)");
#endif
}

extern "C" const char* qx_last_error(void) { return qx::g_last_error; }

extern "C" const char* qx_version(void) { return "qextract_infer_b200 0.1.0 (sm_100a)"; }

extern "C" int qx_copy_async(void* dst, const void* src, size_t bytes, qx_stream_t stream) {
  if (bytes == 0) return QX_OK;
  QX_REQUIRE(dst && src, "copy_async: null pointer");
  QX_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, reinterpret_cast<cudaStream_t>(stream)),
              "copy_async");
  return QX_OK;
}
