// Shared device/host helpers for the sm_100a kernels of qextract_infer_b200.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>

#include "qx_b200.h"

namespace qx {

// ---------------------------------------------------------------- errors --
// Every C-ABI entry point returns QX_OK (0) or a negative QX_ERR_* status
// (qx_b200.h); the message of the last failure on the calling thread is kept
// by set_error / fail and returned by qx_last_error().

void set_error(const char* fmt, ...);
int fail(int code, const char* fmt, ...);
int check_launch(const char* what);

#define QX_REQUIRE(cond, ...)                                 \
  do {                                                        \
    if (!(cond)) return ::qx::fail(QX_ERR_INVALID, __VA_ARGS__); \
  } while (0)

#define QX_CUDA_TRY(call, what)                                                    \
  do {                                                                             \
    cudaError_t e_ = (call);                                                       \
    if (e_ != cudaSuccess)                                                         \
      return ::qx::fail(QX_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e_)); \
  } while (0)

int device_sm_count();  // SM count of the current device (cached per device)

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// ---------------------------------------------------------------- device --
// Limit of every bounded wait inside a kernel (mbarrier phases), measured with
// %globaltimer: 2 s, far above any healthy wait, so that a GPU time-sliced
// with other processes does not trip it; a wait that runs out sets an error
// bit read by qx_get_device_error and the kernel returns.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint4 ldg_stream_v4(const void* p) {
  // weights are read exactly once per call: do not keep them in L1
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ uint4 ldg_v4(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}

__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
  // (a & b) | c
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ uint32_t hfma2_u32(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// D(16x8, f32) += A(16x16, f16, row) * B(16x8, f16, col)
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// D(16x8, f32) = A(16x16, f16, row) * B(16x8, f16, col)
__device__ __forceinline__ void mma_16816_zc(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                             uint32_t a3, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.f));
}

__device__ __forceinline__ float2 h2_to_f2(uint32_t v) {
  __half2 h = *reinterpret_cast<__half2*>(&v);
  return __half22float2(h);
}

// Lets the next kernel in the stream launch now if it was launched with
// programmatic dependent launch (the GEMVs): it streams its weights while this
// kernel runs and waits for this kernel's completion before reading its
// inputs.  No effect on kernels launched without that attribute.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;"); }
// Waits for the previous kernel in the stream to complete (its writes
// visible); a no-op when this kernel was launched without programmatic
// dependent launch.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

extern std::atomic<int> g_pdl_enabled;  // w4a16_gemv.cu (qx_set_pdl)

// Launch with programmatic dependent launch when it is on: the kernel may
// start while the previous one finishes and must call pdl_wait() before it
// reads anything that kernel wrote.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = g_pdl_enabled.load(std::memory_order_relaxed) ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

// ---------------------------------------------------------------- trace --
// Per-CTA phase timestamps for profiling builds (-DQX_TRACE,
// libqx_b200_trace.so): a traced launch writes QX_TRACE_SLOTS uint64 per CTA
// (slot QX_TRACE_SLOTS - 1: the SM id).  In the product build trace_base()
// is a constant null and every trace_stamp() compiles to nothing.
// Host side: the next trace buffer and launch index of a kernel family
// (nullptr when tracing is off or the build has no tracing).
unsigned long long* trace_next(int kernel, int* launch);

__device__ __forceinline__ unsigned long long* trace_base(unsigned long long* buf, int launch) {
#ifdef QX_TRACE
  if (buf == nullptr) return nullptr;
  const size_t grid = size_t(gridDim.x) * gridDim.y * gridDim.z;
  const size_t cta = (size_t(blockIdx.z) * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
  unsigned long long* b = buf + (size_t(launch) * grid + cta) * QX_TRACE_SLOTS;
  if (threadIdx.x == 0) {
    unsigned sm;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(sm));
    b[QX_TRACE_SLOTS - 1] = sm;
  }
  return b;
#else
  (void)buf;
  (void)launch;
  return nullptr;
#endif
}
__device__ __forceinline__ void trace_stamp(unsigned long long* b, int slot, bool who) {
#ifdef QX_TRACE
  if (b != nullptr && who) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    b[slot] = t;
  }
#else
  (void)b;
  (void)slot;
  (void)who;
#endif
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// One warp, one attention head of 32 * EPL elements (lane holds elements
// lane*EPL .. lane*EPL + EPL - 1): Qwen3's per-head RMSNorm (fp16 result, as
// the HF module stores it) followed by rotate-half RoPE with the products and
// the sum rounded as torch does them in fp32; writes the fp16 head to dst.
// The rotate-half partner of element i (i +- D/2) sits 16 lanes away.
template <int EPL>
__device__ __forceinline__ void head_norm_rope(const __half* __restrict__ src, const __half* __restrict__ nw,
                                               float eps, const float* __restrict__ cosr,
                                               const float* __restrict__ sinr, __half* dst, int lane) {
  constexpr int D = EPL * 32;
  float v[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) v[e] = __half2float(src[lane * EPL + e]);
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < EPL; ++e) ss = fmaf(v[e], v[e], ss);
  ss = warp_sum(ss);
  const float r = 1.0f / sqrtf(ss * (1.0f / D) + eps);
#pragma unroll
  for (int e = 0; e < EPL; ++e)  // the head norm's fp16 output
    v[e] = __half2float(__float2half_rn((v[e] * r) * __half2float(nw[lane * EPL + e])));
  const bool lo = lane < 16;  // first half of the head
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    const float partner = __shfl_xor_sync(0xffffffffu, v[e], 16);
    const float rot = lo ? -partner : partner;
    const int i = lane * EPL + e;
    dst[i] = __float2half_rn(__fadd_rn(__fmul_rn(v[e], cosr[i]), __fmul_rn(rot, sinr[i])));
  }
}

}  // namespace qx
