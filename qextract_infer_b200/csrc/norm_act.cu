// Fused RMSNorm and SwiGLU bandwidth kernels for sm_100a.
//
// RMSNorm replaces fused_rmsnorm_vec_kernel / fused_rmsnorm_kernel
// (csrc/kernels/rmsnorm.cu:22-159): the reference reads each row twice (sum of
// squares, then normalise); here each thread keeps its slice of the row in
// registers, so x is read once (1 read + 1 write per element).
//   y = fp16((x * rsqrt(mean(x^2) + eps)) * w), all math in fp32
//   (rmsnorm.cu:134,153).
// SwiGLU replaces fused_swiglu_vec_kernel / fused_swiglu_kernel
// (csrc/kernels/swiglu.cu:23-71):
//   y = fp16(g / (1 + exp(-g)) * u) in fp32, one rounding; like the reference
//   (built with --use_fast_math, setup.py:15) it uses the fast exp/divide.
#include <algorithm>

#include "qx_b200.h"
#include "qx_common.cuh"

namespace qx {
namespace norm {

// One CTA per row; each thread owns VPT 16-byte chunks of the row.
template <int VPT>
__global__ void __launch_bounds__(1024) rmsnorm_vec_kernel(const uint4* __restrict__ x,
                                                           const uint4* __restrict__ w,
                                                           uint4* __restrict__ y, int h8,
                                                           float inv_h, float eps) {
  pdl_trigger();
  __shared__ float s_part[32];
  __shared__ float s_r;
  const size_t row = blockIdx.x;
  const uint4* xr = x + row * h8;
  uint4 v[VPT];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int idx = threadIdx.x + i * blockDim.x;
    v[i] = idx < h8 ? xr[idx] : make_uint4(0u, 0u, 0u, 0u);
    const uint32_t wd[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = h2_to_f2(wd[j]);
      ss = fmaf(f.x, f.x, ss);
      ss = fmaf(f.y, f.y, ss);
    }
  }
  ss = warp_sum(ss);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) s_part[wid] = ss;
  __syncthreads();
  if (wid == 0) {
    const int nw = (blockDim.x + 31) >> 5;
    float t = lane < nw ? s_part[lane] : 0.f;
    t = warp_sum(t);
    if (lane == 0) s_r = 1.0f / sqrtf(t * inv_h + eps);
  }
  __syncthreads();
  const float r = s_r;
  uint4* yr = y + row * h8;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int idx = threadIdx.x + i * blockDim.x;
    if (idx < h8) {
      const uint4 wv = __ldg(w + idx);
      const uint32_t xd[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
      const uint32_t wd[4] = {wv.x, wv.y, wv.z, wv.w};
      uint32_t od[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 fx = h2_to_f2(xd[j]), fw = h2_to_f2(wd[j]);
        __half2 o = __floats2half2_rn((fx.x * r) * fw.x, (fx.y * r) * fw.y);
        od[j] = *reinterpret_cast<uint32_t*>(&o);
      }
      yr[idx] = make_uint4(od[0], od[1], od[2], od[3]);
    }
  }
}

// General fallback (any H, any alignment): two passes over the row.
__global__ void __launch_bounds__(256) rmsnorm_scalar_kernel(const __half* __restrict__ x,
                                                             const __half* __restrict__ w,
                                                             __half* __restrict__ y, int h,
                                                             float inv_h, float eps) {
  __shared__ float s_part[32];
  __shared__ float s_r;
  const size_t row = blockIdx.x;
  const __half* xr = x + row * h;
  float ss = 0.f;
  for (int i = threadIdx.x; i < h; i += blockDim.x) {
    const float f = __half2float(xr[i]);
    ss = fmaf(f, f, ss);
  }
  ss = warp_sum(ss);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) s_part[wid] = ss;
  __syncthreads();
  if (wid == 0) {
    float t = lane < int(blockDim.x >> 5) ? s_part[lane] : 0.f;
    t = warp_sum(t);
    if (lane == 0) s_r = 1.0f / sqrtf(t * inv_h + eps);
  }
  __syncthreads();
  const float r = s_r;
  for (int i = threadIdx.x; i < h; i += blockDim.x)
    y[row * h + i] = __float2half_rn((__half2float(xr[i]) * r) * __half2float(w[i]));
}

__device__ __forceinline__ float silu_mul(float g, float u) {
  return __fdividef(g, 1.0f + __expf(-g)) * u;
}

__global__ void __launch_bounds__(256) swiglu_vec_kernel(const uint4* __restrict__ gate,
                                                         const uint4* __restrict__ up,
                                                         uint4* __restrict__ out, int64_t n8) {
  pdl_trigger();
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n8; i += stride) {
    const uint4 gv = __ldcs(gate + i);
    const uint4 uv = __ldcs(up + i);
    const uint32_t gd[4] = {gv.x, gv.y, gv.z, gv.w};
    const uint32_t ud[4] = {uv.x, uv.y, uv.z, uv.w};
    uint32_t od[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 fg = h2_to_f2(gd[j]), fu = h2_to_f2(ud[j]);
      __half2 o = __floats2half2_rn(silu_mul(fg.x, fu.x), silu_mul(fg.y, fu.y));
      od[j] = *reinterpret_cast<uint32_t*>(&o);
    }
    __stcs(out + i, make_uint4(od[0], od[1], od[2], od[3]));
  }
}

__global__ void __launch_bounds__(256) swiglu_scalar_kernel(const __half* __restrict__ gate,
                                                            const __half* __restrict__ up,
                                                            __half* __restrict__ out, int64_t n) {
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
    out[i] = __float2half_rn(silu_mul(__half2float(gate[i]), __half2float(up[i])));
}

}  // namespace norm
}  // namespace qx

using namespace qx;

extern "C" int qx_fused_rmsnorm(const void* x, const void* weight, void* y, int64_t rows,
                                int hidden, float eps, qx_stream_t stream) {
  QX_REQUIRE(rows >= 0 && hidden > 0, "fused_rmsnorm: bad sizes rows=%lld hidden=%d",
             (long long)rows, hidden);
  if (rows == 0) return QX_OK;
  QX_REQUIRE(rows <= 0x7fffffffLL, "fused_rmsnorm: too many rows (%lld)", (long long)rows);
  QX_REQUIRE(x && weight && y, "fused_rmsnorm: null pointer");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const float inv_h = 1.0f / float(hidden);
  const bool vec = (hidden % 8 == 0) && aligned(x, 16) && aligned(weight, 16) && aligned(y, 16);
  const int h8 = hidden / 8;
  if (vec && h8 <= 8 * 1024) {
    int vpt = std::max(1, (h8 + 255) / 256);
    vpt = vpt <= 1 ? 1 : vpt <= 2 ? 2 : vpt <= 4 ? 4 : 8;
    int threads = (h8 + vpt - 1) / vpt;
    threads = std::min(1024, (threads + 31) / 32 * 32);
    const unsigned grid = unsigned(rows);
    auto X = static_cast<const uint4*>(x);
    auto W = static_cast<const uint4*>(weight);
    auto Y = static_cast<uint4*>(y);
    switch (vpt) {
      case 1: norm::rmsnorm_vec_kernel<1><<<grid, threads, 0, st>>>(X, W, Y, h8, inv_h, eps); break;
      case 2: norm::rmsnorm_vec_kernel<2><<<grid, threads, 0, st>>>(X, W, Y, h8, inv_h, eps); break;
      case 4: norm::rmsnorm_vec_kernel<4><<<grid, threads, 0, st>>>(X, W, Y, h8, inv_h, eps); break;
      default: norm::rmsnorm_vec_kernel<8><<<grid, threads, 0, st>>>(X, W, Y, h8, inv_h, eps); break;
    }
  } else {
    const int threads = std::min(256, (hidden + 31) / 32 * 32);
    norm::rmsnorm_scalar_kernel<<<unsigned(rows), threads, 0, st>>>(
        static_cast<const __half*>(x), static_cast<const __half*>(weight), static_cast<__half*>(y),
        hidden, inv_h, eps);
  }
  return check_launch("fused_rmsnorm");
}

extern "C" int qx_fused_swiglu(const void* gate, const void* up, void* y, int64_t n,
                               qx_stream_t stream) {
  QX_REQUIRE(n >= 0, "fused_swiglu: bad size %lld", (long long)n);
  if (n == 0) return QX_OK;
  QX_REQUIRE(gate && up && y, "fused_swiglu: null pointer");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int64_t max_blocks = int64_t(device_sm_count()) * 8;
  if (n % 8 == 0 && aligned(gate, 16) && aligned(up, 16) && aligned(y, 16)) {
    const int64_t n8 = n / 8;
    const int64_t blocks = std::min<int64_t>((n8 + 255) / 256, max_blocks);
    norm::swiglu_vec_kernel<<<unsigned(blocks), 256, 0, st>>>(
        static_cast<const uint4*>(gate), static_cast<const uint4*>(up), static_cast<uint4*>(y), n8);
  } else {
    const int64_t blocks = std::min<int64_t>((n + 255) / 256, max_blocks);
    norm::swiglu_scalar_kernel<<<unsigned(blocks), 256, 0, st>>>(
        static_cast<const __half*>(gate), static_cast<const __half*>(up), static_cast<__half*>(y), n);
  }
  return check_launch("fused_swiglu");
}
