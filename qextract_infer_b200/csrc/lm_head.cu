// Greedy sampling head: logits = h W (fp16 weights [H, V], V contiguous:
// this rank's vocabulary slice) and, per row, the largest logit and its index,
// in two launches instead of a library GEMV, a reduction and an index add.
//
// Kernel 1: a CTA owns 256 vocabulary columns (4 warps x 64) for every row
// (batch <= 32, one or two 16-row m-tiles).  64-row K tiles of W and of h are
// staged by cp.async (double buffered); W fragments come from ldmatrix.trans,
// h fragments from ldmatrix; mma.sync m16n8k16 with fp32 accumulation.  The
// logits are rounded to fp16 (the values a fp16 GEMV stores), and the CTA's
// per-row maximum with its smallest index is written to the workspace.
// Kernel 2: one warp per row reduces the CTAs' candidates in index order
// (ties go to the smallest index) and adds the slice's vocabulary offset.
#include <algorithm>
#include <cfloat>
#include <mutex>

#include "qx_b200.h"
#include "qx_common.cuh"

namespace qx {
namespace lmh {

constexpr int WARPS = 4;
constexpr int THREADS = WARPS * 32;
constexpr int COLS = 256;                  // vocabulary columns per CTA
constexpr int KT = 64;                     // K rows per tile
constexpr int MAXB = 32;                   // rows (two m-tiles)
constexpr int WROW = COLS * 2;             // bytes of one W tile row (512)
constexpr int W_TILE = KT * WROW;          // 32 KB
constexpr int HROW = KT * 2 + 16;          // bytes of one staged h row (+16: conflict-free ldmatrix)
constexpr int H_TILE = MAXB * HROW;        // 4.5 KB
constexpr int STAGE = W_TILE + H_TILE;
constexpr int SMEM = 2 * STAGE;            // 2 stages

struct Cand {
  float v;
  int i;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N));
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
// W tile row r (K), 16-byte chunk ch (8 columns): XOR swizzle over 8 rows
__device__ __forceinline__ uint32_t wswz(int r, int ch) {
  return uint32_t(r * WROW + ((ch ^ (r & 7)) << 4));
}
// larger value wins; equal values: the smaller index
__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

template <int MT>
__global__ void __launch_bounds__(THREADS) logits_argmax_kernel(const __half* __restrict__ h,
                                                               const __half* __restrict__ W, int B, int H,
                                                               int V, Cand* __restrict__ part) {
  pdl_trigger();
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ Cand s_best[WARPS][MAXB];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int n0 = blockIdx.x * COLS;
  const uint32_t sbase = smem_u32(smem);
  const int ktiles = H / KT;

  auto issue = [&](int kt, int stage) {
    const uint32_t ws = sbase + stage * STAGE, hs = ws + W_TILE;
    // W: 64 rows x 32 chunks of 16 B = 2048 chunks, 16 per thread
#pragma unroll
    for (int i = 0; i < (KT * (COLS / 8)) / THREADS; ++i) {
      const int idx = i * THREADS + tid, r = idx >> 5, ch = idx & 31;
      const int col = n0 + ch * 8;
      const bool ok = col < V;  // V % 8 == 0: a chunk is all in or all out
      const __half* src = W + (size_t(kt) * KT + r) * V + (ok ? col : 0);
      cp_async16(ws + wswz(r, ch), src, ok ? 16 : 0);
    }
    // h: B rows x 8 chunks (rows past B read as zero)
    for (int idx = tid; idx < MT * 16 * 8; idx += THREADS) {
      const int r = idx >> 3, ch = idx & 7;
      const bool ok = r < B;
      const __half* src = h + size_t(ok ? r : 0) * H + size_t(kt) * KT + ch * 8;
      cp_async16(hs + r * HROW + ch * 16, src, ok ? 16 : 0);
    }
    cp_async_commit();
  };

  float acc[MT][8][4];
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[m][j][0] = acc[m][j][1] = acc[m][j][2] = acc[m][j][3] = 0.f;

  pdl_wait();  // h comes from the previous kernel
  issue(0, 0);
  if (ktiles > 1) issue(1, 1);
  else cp_async_commit();
  const int mi = lane >> 3, ri = lane & 7;
  for (int kt = 0; kt < ktiles; ++kt) {
    cp_async_wait<1>();
    __syncthreads();
    const uint32_t ws = sbase + (kt & 1) * STAGE, hs = ws + W_TILE;
#pragma unroll
    for (int ks = 0; ks < KT / 16; ++ks) {
      // A fragments (h rows m*16.., k ks*16..): matrices (rows 0-7 | 8-15) x (k 0-7 | 8-15)
      uint32_t a[MT][4];
#pragma unroll
      for (int m = 0; m < MT; ++m)
        ldsm_x4(a[m], hs + (m * 16 + (mi & 1) * 8 + ri) * HROW + (ks * 16 + (mi >> 1) * 8) * 2);
      // B fragments: k16 x n8 of W for this warp's 8 n-tiles (two per ldmatrix.x4.trans)
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        uint32_t bw[4];
        const int ch = (warp * 64 + jj * 16) / 8 + (mi >> 1);
        ldsm_x4_t(bw, ws + wswz(ks * 16 + (mi & 1) * 8 + ri, ch));
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          mma_16816(acc[m][2 * jj], a[m][0], a[m][1], a[m][2], a[m][3], bw[0], bw[1]);
          mma_16816(acc[m][2 * jj + 1], a[m][0], a[m][1], a[m][2], a[m][3], bw[2], bw[3]);
        }
      }
    }
    __syncthreads();
    if (kt + 2 < ktiles) issue(kt + 2, kt & 1);
    else cp_async_commit();
  }
  cp_async_wait<0>();

  // per row: the fp16-rounded logits' maximum and its smallest index
#pragma unroll
  for (int m = 0; m < MT; ++m) {
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {  // rows g and g + 8 of the m-tile
      const int row = m * 16 + g + hr * 8;
      float bv = -FLT_MAX;
      int bi = 0x7fffffff;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int col = n0 + warp * 64 + j * 8 + 2 * c + e;
          const float v = __half2float(__float2half_rn(acc[m][j][hr * 2 + e]));
          if (col < V && better(v, col, bv, bi)) {
            bv = v;
            bi = col;
          }
        }
      }
#pragma unroll
      for (int o = 1; o < 4; o <<= 1) {  // the quad holding the row
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (better(ov, oi, bv, bi)) {
          bv = ov;
          bi = oi;
        }
      }
      if (c == 0 && row < MAXB) s_best[warp][row] = Cand{bv, bi};
    }
  }
  __syncthreads();
  for (int row = tid; row < B; row += THREADS) {
    Cand best = s_best[0][row];
    for (int w = 1; w < WARPS; ++w) {
      const Cand o = s_best[w][row];
      if (better(o.v, o.i, best.v, best.i)) best = o;
    }
    part[size_t(blockIdx.x) * MAXB + row] = best;
  }
}

__global__ void __launch_bounds__(128) argmax_finish_kernel(const Cand* __restrict__ part, int nblk, int B,
                                                             int64_t offset, float* __restrict__ out_val,
                                                             int64_t* __restrict__ out_idx) {
  pdl_trigger();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 4 + warp;
  if (row >= B) return;
  float bv = -FLT_MAX;
  int bi = 0x7fffffff;
  for (int k = lane; k < nblk; k += 32) {
    const Cand o = part[size_t(k) * MAXB + row];
    if (better(o.v, o.i, bv, bi)) {
      bv = o.v;
      bi = o.i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if (lane == 0) {
    out_val[row] = bv;
    out_idx[row] = int64_t(bi) + offset;
  }
}

}  // namespace lmh
}  // namespace qx

using namespace qx;

extern "C" size_t qx_lm_head_argmax_workspace_size(int vocab) {
  return vocab > 0 ? size_t((vocab + lmh::COLS - 1) / lmh::COLS) * lmh::MAXB * sizeof(lmh::Cand) : 0;
}

extern "C" int qx_lm_head_argmax(const void* h, const void* weight, int batch, int hidden, int vocab,
                                 int64_t vocab_offset, float* out_val, int64_t* out_idx, void* workspace,
                                 size_t workspace_bytes, qx_stream_t stream) {
  QX_REQUIRE(batch >= 1 && batch <= lmh::MAXB, "lm_head_argmax: batch=%d (1..%d)", batch, lmh::MAXB);
  QX_REQUIRE(hidden > 0 && hidden % lmh::KT == 0, "lm_head_argmax: hidden=%d must be a multiple of %d",
             hidden, lmh::KT);
  QX_REQUIRE(vocab > 0 && vocab % 8 == 0, "lm_head_argmax: vocab=%d must be a multiple of 8", vocab);
  QX_REQUIRE(h && weight && out_val && out_idx, "lm_head_argmax: null pointer");
  QX_REQUIRE(aligned(h, 16) && aligned(weight, 16), "lm_head_argmax: h and weight must be 16-byte aligned");
  const size_t need = qx_lm_head_argmax_workspace_size(vocab);
  if (!workspace || workspace_bytes < need || !aligned(workspace, 16))
    return fail(QX_ERR_WORKSPACE, "lm_head_argmax: workspace needs %zu bytes, 16-byte aligned", need);
  {
    static std::mutex mu;
    static bool done[64] = {};
    int dev = 0;
    QX_CUDA_TRY(cudaGetDevice(&dev), "lm_head_argmax: cudaGetDevice");
    QX_REQUIRE(dev >= 0 && dev < 64, "lm_head_argmax: device index %d unsupported", dev);
    std::lock_guard<std::mutex> lk(mu);
    if (!done[dev]) {
      QX_CUDA_TRY(cudaFuncSetAttribute(lmh::logits_argmax_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       lmh::SMEM),
                  "lm_head_argmax: set smem limit");
      QX_CUDA_TRY(cudaFuncSetAttribute(lmh::logits_argmax_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       lmh::SMEM),
                  "lm_head_argmax: set smem limit");
      done[dev] = true;
    }
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int nblk = (vocab + lmh::COLS - 1) / lmh::COLS;
  auto H = static_cast<const __half*>(h);
  auto Wt = static_cast<const __half*>(weight);
  auto part = static_cast<lmh::Cand*>(workspace);
  if (batch <= 16)
    QX_CUDA_TRY(launch_pdl(lmh::logits_argmax_kernel<1>, dim3(nblk), dim3(lmh::THREADS), lmh::SMEM, st, H, Wt,
                           batch, hidden, vocab, part),
                "lm_head_argmax: launch");
  else
    QX_CUDA_TRY(launch_pdl(lmh::logits_argmax_kernel<2>, dim3(nblk), dim3(lmh::THREADS), lmh::SMEM, st, H, Wt,
                           batch, hidden, vocab, part),
                "lm_head_argmax: launch");
  QX_CUDA_TRY(launch_pdl(lmh::argmax_finish_kernel, dim3((batch + 3) / 4), dim3(128), 0, st,
                         static_cast<const lmh::Cand*>(part), nblk, batch, vocab_offset, out_val, out_idx),
              "lm_head_argmax: finish launch");
  return check_launch("lm_head_argmax");
}
