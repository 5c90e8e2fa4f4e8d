// Fused elementwise kernels of the tensor-parallel decode step (new
// components: the reference's patched Qwen3 layer, qextract/patch.py,
// runs these as separate torch ops around its GEMV calls).  Each keeps the
// rounding points of the unfused sequence, so results equal it:
//
//   add_rmsnorm          x <- fp16(x + d) (the residual add, in place), then
//                        y = fp16((x * rsqrt(mean(x^2) + eps)) * w) in fp32
//                        (the same formula as qx_fused_rmsnorm).
//   qk_norm_rope_append  per row and head of the fused q|k|v projection output:
//                        q and k heads RMSNorm'd over head_dim (fp16 result),
//                        then rotated (rotate-half RoPE, fp32 cos/sin of the
//                        position, products and sum rounded separately, one
//                        fp16 rounding); q heads to q_out, k heads to the ring
//                        slot of the position, v heads copied to that slot.
//   swiglu_packed        y[r, i] = fp16(silu(g) u), g = gu[r, i], u = gu[r, I + i]
//                        (the fused gate|up projection output), the formula of
//                        qx_fused_swiglu.
#include <algorithm>

#include "qx_b200.h"
#include "qx_common.cuh"

namespace qx {
namespace dfused {

// One CTA per row, 256 threads, each owning up to VPT 16-byte chunks.
template <int VPT>
__global__ void __launch_bounds__(256) add_rmsnorm_kernel(uint4* __restrict__ x,
                                                          const uint4* __restrict__ d,
                                                          const uint4* __restrict__ w,
                                                          uint4* __restrict__ y, int h8, float inv_h,
                                                          float eps) {
  pdl_trigger();
  pdl_wait();  // inputs come from the previous kernel
  __shared__ float s_part[8];
  __shared__ float s_r;
  const size_t row = blockIdx.x;
  uint4 v[VPT];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int idx = threadIdx.x + i * 256;
    v[i] = make_uint4(0u, 0u, 0u, 0u);
    if (idx < h8) {
      const uint4 a = x[row * h8 + idx], b = d[row * h8 + idx];
      const uint32_t ad[4] = {a.x, a.y, a.z, a.w}, bd[4] = {b.x, b.y, b.z, b.w};
      uint32_t od[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 fa = h2_to_f2(ad[j]), fb = h2_to_f2(bd[j]);
        const __half2 s2 = __floats2half2_rn(fa.x + fb.x, fa.y + fb.y);  // the fp16 residual add
        od[j] = *reinterpret_cast<const uint32_t*>(&s2);
        const float2 f = __half22float2(s2);
        ss = fmaf(f.x, f.x, ss);
        ss = fmaf(f.y, f.y, ss);
      }
      v[i] = make_uint4(od[0], od[1], od[2], od[3]);
      x[row * h8 + idx] = v[i];
    }
  }
  ss = warp_sum(ss);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) s_part[wid] = ss;
  __syncthreads();
  if (wid == 0) {
    float t = lane < 8 ? s_part[lane] : 0.f;
    t = warp_sum(t);
    if (lane == 0) s_r = 1.0f / sqrtf(t * inv_h + eps);
  }
  __syncthreads();
  const float r = s_r;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int idx = threadIdx.x + i * 256;
    if (idx < h8) {
      const uint4 wv = w[idx];
      const uint32_t vd[4] = {v[i].x, v[i].y, v[i].z, v[i].w}, wd[4] = {wv.x, wv.y, wv.z, wv.w};
      uint32_t od[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = h2_to_f2(vd[j]), g = h2_to_f2(wd[j]);
        const __half2 o = __floats2half2_rn((f.x * r) * g.x, (f.y * r) * g.y);
        od[j] = *reinterpret_cast<const uint32_t*>(&o);
      }
      y[row * h8 + idx] = make_uint4(od[0], od[1], od[2], od[3]);
    }
  }
}

// One warp per (row, head); EPL = head_dim / 32 consecutive elements per lane,
// so element i + head_dim/2 (the rotate-half partner) sits 16 lanes away.
template <int EPL>
__global__ void __launch_bounds__(128) qk_norm_rope_append_kernel(
    const __half* __restrict__ qkv, int batch, int hq, int hkv, const __half* __restrict__ qw,
    const __half* __restrict__ kw, float eps, const float* __restrict__ cosr,
    const float* __restrict__ sinr, __half* __restrict__ q_out, __half* __restrict__ k_cache,
    __half* __restrict__ v_cache, int cap, int64_t slot) {
  pdl_trigger();
  pdl_wait();  // inputs come from the previous kernel
  constexpr int D = EPL * 32;
  const int lane = threadIdx.x & 31;
  const int item = blockIdx.x * 4 + (threadIdx.x >> 5);
  const int heads = hq + 2 * hkv;
  if (item >= batch * heads) return;
  const int b = item / heads, h = item - b * heads;
  const __half* src = qkv + (size_t(b) * heads + h) * D + lane * EPL;
  if (h >= hq + hkv) {  // v head: copy to the ring slot
    __half* dst = v_cache + ((size_t(b) * cap + slot) * hkv + (h - hq - hkv)) * D + lane * EPL;
#pragma unroll
    for (int e = 0; e < EPL; ++e) dst[e] = src[e];
    return;
  }
  const bool is_q = h < hq;
  __half* dst = is_q ? q_out + (size_t(b) * hq + h) * D
                     : k_cache + ((size_t(b) * cap + slot) * hkv + (h - hq)) * D;
  head_norm_rope<EPL>(qkv + (size_t(b) * heads + h) * D, is_q ? qw : kw, eps, cosr, sinr, dst, lane);
}

__device__ __forceinline__ float silu_mul(float g, float u) {
  return __fdividef(g, 1.0f + __expf(-g)) * u;
}

__global__ void __launch_bounds__(256) swiglu_packed_kernel(const uint4* __restrict__ gu,
                                                            uint4* __restrict__ y, int64_t rows,
                                                            int i8) {
  pdl_trigger();
  pdl_wait();  // inputs come from the previous kernel
  const int64_t n = rows * i8;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; t < n; t += stride) {
    const int64_t r = t / i8, c = t - r * i8;
    const uint4 gv = gu[r * 2 * i8 + c], uv = gu[r * 2 * i8 + i8 + c];
    const uint32_t gd[4] = {gv.x, gv.y, gv.z, gv.w}, ud[4] = {uv.x, uv.y, uv.z, uv.w};
    uint32_t od[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 fg = h2_to_f2(gd[j]), fu = h2_to_f2(ud[j]);
      const __half2 o = __floats2half2_rn(silu_mul(fg.x, fu.x), silu_mul(fg.y, fu.y));
      od[j] = *reinterpret_cast<const uint32_t*>(&o);
    }
    y[t] = make_uint4(od[0], od[1], od[2], od[3]);
  }
}

}  // namespace dfused
}  // namespace qx

using namespace qx;

extern "C" int qx_add_rmsnorm(void* x, const void* delta, const void* weight, void* y, int64_t rows,
                              int hidden, float eps, qx_stream_t stream) {
  QX_REQUIRE(rows >= 0 && hidden > 0, "add_rmsnorm: bad sizes rows=%lld hidden=%d", (long long)rows,
             hidden);
  if (rows == 0) return QX_OK;
  QX_REQUIRE(x && delta && weight && y, "add_rmsnorm: null pointer");
  QX_REQUIRE(hidden % 8 == 0 && hidden <= 8192, "add_rmsnorm: hidden=%d must be a multiple of 8, <= 8192",
             hidden);
  QX_REQUIRE(aligned(x, 16) && aligned(delta, 16) && aligned(weight, 16) && aligned(y, 16),
             "add_rmsnorm: x, delta, weight and y must be 16-byte aligned");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int h8 = hidden / 8;
  const float inv_h = 1.0f / float(hidden);
  auto X = static_cast<uint4*>(x);
  auto D = static_cast<const uint4*>(delta);
  auto W = static_cast<const uint4*>(weight);
  auto Y = static_cast<uint4*>(y);
  const dim3 grid{static_cast<unsigned>(rows)};
  if (h8 <= 256)
    QX_CUDA_TRY(launch_pdl(dfused::add_rmsnorm_kernel<1>, grid, dim3(256), 0, st, X, D, W, Y, h8, inv_h, eps),
                "add_rmsnorm: launch");
  else if (h8 <= 512)
    QX_CUDA_TRY(launch_pdl(dfused::add_rmsnorm_kernel<2>, grid, dim3(256), 0, st, X, D, W, Y, h8, inv_h, eps),
                "add_rmsnorm: launch");
  else
    QX_CUDA_TRY(launch_pdl(dfused::add_rmsnorm_kernel<4>, grid, dim3(256), 0, st, X, D, W, Y, h8, inv_h, eps),
                "add_rmsnorm: launch");
  return check_launch("add_rmsnorm");
}

extern "C" int qx_qk_norm_rope_append(const void* qkv, int batch, int q_heads, int kv_heads,
                                      int head_dim, const void* q_norm_w, const void* k_norm_w,
                                      float eps, const float* cos_row, const float* sin_row,
                                      void* q_out, void* k_cache, void* v_cache, int sink, int window,
                                      int64_t pos, qx_stream_t stream) {
  QX_REQUIRE(batch >= 0 && q_heads > 0 && kv_heads > 0, "qk_norm_rope_append: bad sizes");
  if (batch == 0) return QX_OK;
  QX_REQUIRE(head_dim == 64 || head_dim == 128 || head_dim == 256,
             "qk_norm_rope_append: head_dim=%d must be 64, 128 or 256", head_dim);
  QX_REQUIRE(qkv && q_norm_w && k_norm_w && cos_row && sin_row && q_out && k_cache && v_cache,
             "qk_norm_rope_append: null pointer");
  QX_REQUIRE(sink >= 0 && window > 0 && pos >= 0, "qk_norm_rope_append: bad sink/window/pos");
  const int64_t slot = pos < sink ? pos : sink + (pos - sink) % window;  // ring write position
  const int cap = sink + window;
  const int items = batch * (q_heads + 2 * kv_heads);
  const dim3 grid(unsigned((items + 3) / 4));
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  auto Q = static_cast<const __half*>(qkv);
  auto QW = static_cast<const __half*>(q_norm_w);
  auto KW = static_cast<const __half*>(k_norm_w);
  auto QO = static_cast<__half*>(q_out);
  auto KC = static_cast<__half*>(k_cache);
  auto VC = static_cast<__half*>(v_cache);
  switch (head_dim) {
    case 64:
      QX_CUDA_TRY(launch_pdl(dfused::qk_norm_rope_append_kernel<2>, grid, dim3(128), 0, st, Q, batch,
                             q_heads, kv_heads, QW, KW, eps, cos_row, sin_row, QO, KC, VC, cap, slot),
                  "qk_norm_rope_append: launch");
      break;
    case 128:
      QX_CUDA_TRY(launch_pdl(dfused::qk_norm_rope_append_kernel<4>, grid, dim3(128), 0, st, Q, batch,
                             q_heads, kv_heads, QW, KW, eps, cos_row, sin_row, QO, KC, VC, cap, slot),
                  "qk_norm_rope_append: launch");
      break;
    default:
      QX_CUDA_TRY(launch_pdl(dfused::qk_norm_rope_append_kernel<8>, grid, dim3(128), 0, st, Q, batch,
                             q_heads, kv_heads, QW, KW, eps, cos_row, sin_row, QO, KC, VC, cap, slot),
                  "qk_norm_rope_append: launch");
      break;
  }
  return check_launch("qk_norm_rope_append");
}

extern "C" int qx_swiglu_packed(const void* gate_up, void* y, int64_t rows, int inter,
                                qx_stream_t stream) {
  QX_REQUIRE(rows >= 0 && inter > 0, "swiglu_packed: bad sizes");
  if (rows == 0) return QX_OK;
  QX_REQUIRE(gate_up && y, "swiglu_packed: null pointer");
  QX_REQUIRE(inter % 8 == 0 && aligned(gate_up, 16) && aligned(y, 16),
             "swiglu_packed: inter=%d must be a multiple of 8, tensors 16-byte aligned", inter);
  const int i8 = inter / 8;
  const int64_t n = rows * i8;
  const int sms = device_sm_count();
  const unsigned blocks = unsigned(std::min<int64_t>((n + 255) / 256, int64_t(sms) * 8));
  QX_CUDA_TRY(launch_pdl(dfused::swiglu_packed_kernel, dim3(blocks), dim3(256), 0,
                         reinterpret_cast<cudaStream_t>(stream), static_cast<const uint4*>(gate_up),
                         static_cast<uint4*>(y), rows, i8),
              "swiglu_packed: launch");
  return check_launch("swiglu_packed");
}
