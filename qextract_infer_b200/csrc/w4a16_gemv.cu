// W4A16 (GPTQ int4, group-wise scale/zero) + LoRA decode GEMV for sm_100a.
//
// Replaces the reference's two-launch path (lora_down_gemv_kernel +
// w4a16_lora_fused_gemv_kernel, csrc/kernels/w4a16_lora_gemv.cu:112-226):
// one launch streams every weight byte once from HBM, and the LoRA terms ride
// along.
//
// Work decomposition
//   CTA  = 8 warps x 32 output columns = 256 columns ("tile"), over one
//          contiguous range of K ("split").  grid = (tiles, splits), sized so
//          the whole grid is resident in one wave.
//   k-step = 32 rows of K = 4 packed int32 rows.  Lane (g = lane/4,
//          c = lane%4) loads one 128-bit word: packed row 4*ks + c, columns
//          4g..4g+3 of its warp -- each warp load is 4 rows x 128 contiguous
//          bytes, and every weight byte is loaded exactly once.
//   dot product: the nibbles are turned into exact fp16 integers with the
//          magic-number trick (q | 0x6400 is the fp16 value 1024 + q; see
//          Kim et al., "Who Says Elephants Can't Run", 2022) and fed to
//          mma.sync m16n8k16 with fp32 accumulation: MMA rows are output
//          columns, MMA columns are batch rows (up to 8 per n-tile), and the
//          MMA k order is a fixed permutation of the 32 rows of a k-step that
//          the staged activations follow.  The zero point is folded out:
//          sum_k (q-z) x = sum_k q x - z sum_k x, applied once per group with
//          the fp32 scale, so fractional fp16 zeros stay exact too.
//   LoRA: each CTA computes h_s = x[:, Ks] A[Ks, :] for its K range (the
//          LoRA product is linear in K); the last CTA of a tile sums the
//          splits' base partials and h_s in a fixed order (deterministic),
//          adds lora_scale * h.B and rounds to fp16 once.
// The reference math being reproduced: y = fp16(x.W + (alpha/r)(x.A).B) with
// W = s (q - z) and fp32 accumulation (w4a16_lora_gemv.cu:183-224).
#include <algorithm>
#include <mutex>

#include "qx_b200.h"
#include "qx_common.cuh"

namespace qx {
namespace gemv {

constexpr int WARPS = 8;
constexpr int THREADS = WARPS * 32;
constexpr int COLS = WARPS * 32;  // output columns per CTA
constexpr int KSTEP = 32;         // K rows per step (4 packed rows)
constexpr int U = 8;              // k-steps of weights held in registers at once
constexpr int MROWS = 32;         // batch rows per launch (4 n-tiles of 8)
constexpr int HMC = 2;            // batch rows per pass of the LoRA-down loop
constexpr int TS_CAP = 48;        // max k-steps per split (bounds shared memory)
// The workspace starts with a fixed-size counter region, so that counters of
// one call never overlap the partials of a call with a different shape.
constexpr int COUNTER_SLOTS = 8192;
// residency the split heuristic plans for (and the kernel's launch bound)
__host__ __device__ constexpr int ctas_per_sm(int nt) { return nt == 1 ? 3 : 2; }

struct Params {
  const __half* x;
  const uint32_t* qw;
  const __half* scales;
  const void* zeros;
  const __half* A;
  const __half* B;
  __half* y;
  int M, K, N, rank, group, zeros_packed, zero_offset;
  float lora_scale;
  int T, S, Ts_max, ng_max;
  float* partial;    // [S][M][N]
  float* hpart;      // [tiles][S][M][rank]
  unsigned* counters;  // [tiles]
};

struct Plan {
  int tiles, S, T, Ts_max, ng_max, NT;
  size_t smem, off_partial, off_hpart, total;
};

static inline size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

static Plan make_plan(int M, int K, int N, int rank, int group, int sms) {
  Plan pl{};
  pl.tiles = (N + COLS - 1) / COLS;
  pl.T = K / KSTEP;
  const int mc = std::min(M, MROWS);
  pl.NT = mc <= 8 ? 1 : (mc <= 16 ? 2 : 4);
  const int target = sms * ctas_per_sm(pl.NT);
  int S = std::max(1, target / pl.tiles);
  S = std::min(S, std::max(1, pl.T / 4));           // >= 4 k-steps per split
  S = std::max(S, (pl.T + TS_CAP - 1) / TS_CAP);    // bounded shared memory
  S = std::min(S, pl.T);
  pl.S = S;
  pl.Ts_max = (pl.T + S - 1) / S;
  pl.ng_max = (pl.Ts_max * KSTEP) / group + 2;
  pl.smem = size_t(pl.Ts_max) * pl.NT * 32 * 16      // xs
            + size_t(pl.Ts_max) * pl.NT * 8 * 4       // xks
            + size_t(2) * pl.ng_max * COLS * 4         // sc, zs
            + size_t(pl.NT) * 8 * rank * 4             // hs
            + size_t(WARPS) * HMC * rank * 4;          // red
  pl.off_partial = align256(size_t(COUNTER_SLOTS) * 4);
  pl.off_hpart = pl.off_partial + align256(size_t(S) * mc * N * 4);
  pl.total = pl.off_hpart + align256(size_t(pl.tiles) * S * mc * std::max(rank, 1) * 4);
  return pl;
}

__device__ __forceinline__ int inv_perm8(int k) {
  // position of row k (0..7) inside a staged 8-half group (0,4,1,5,2,6,3,7)
  return ((k & 3) << 1) | (k >> 2);
}

template <int NT>
__global__ void __launch_bounds__(THREADS, ctas_per_sm(NT)) w4a16_gemv_kernel(const Params p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ unsigned s_is_last;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int tile = blockIdx.x, s = blockIdx.y;
  const int ks0 = int((long long)s * p.T / p.S);
  const int ks1 = int((long long)(s + 1) * p.T / p.S);
  const int Ts = ks1 - ks0;
  const int M = p.M;
  const int n_tile0 = tile * COLS;
  const int ncol = n_tile0 + warp * 32 + 4 * g;  // first of this lane's 4 columns
  const bool col_ok = ncol < p.N;                // N % 8 == 0: all 4 or none
  const int k0 = ks0 * KSTEP;
  const int g_first = k0 / p.group;
  const int ng = (ks1 * KSTEP - 1) / p.group - g_first + 1;

  uint4* xs = reinterpret_cast<uint4*>(smem_raw);                  // [Ts_max][NT][32]
  float* xks = reinterpret_cast<float*>(xs + p.Ts_max * NT * 32);  // [Ts_max][NT*8]
  float* sc = xks + p.Ts_max * NT * 8;                              // [ng_max][COLS]
  float* zs = sc + p.ng_max * COLS;                                 // [ng_max][COLS]
  float* hs = zs + p.ng_max * COLS;                                 // [NT*8][rank]
  float* red = hs + NT * 8 * p.rank;                                // [WARPS][HMC][rank]

  // 1. issue the first register batch of weight loads before anything else
  const uint32_t* qcol = p.qw + ncol;
  uint4 w[U];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int ks = ks0 + u;
    w[u] = (col_ok && ks < ks1) ? ldg_stream_v4(qcol + size_t(ks * 4 + c) * p.N)
                                : make_uint4(0u, 0u, 0u, 0u);
  }

  // 2. stage activations in MMA-B order, plus per-k-step row sums
  for (int it = tid; it < Ts * NT * 32; it += THREADS) {
    const int t = it / (NT * 32);
    const int rem = it - t * (NT * 32);
    const int nt = rem >> 5, l = rem & 31, gg = l >> 2, cc = l & 3;
    const int m = nt * 8 + gg;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (m < M) v = ldg_v4(p.x + size_t(m) * p.K + size_t(ks0 + t) * KSTEP + cc * 8);
    uint4 o;
    o.x = prmt(v.x, v.z, 0x5410u);  // (x0, x4)
    o.y = prmt(v.x, v.z, 0x7632u);  // (x1, x5)
    o.z = prmt(v.y, v.w, 0x5410u);  // (x2, x6)
    o.w = prmt(v.y, v.w, 0x7632u);  // (x3, x7)
    xs[it] = o;
    const float2 a0 = h2_to_f2(v.x), a1 = h2_to_f2(v.y), a2 = h2_to_f2(v.z), a3 = h2_to_f2(v.w);
    float s8 = ((a0.x + a0.y) + (a1.x + a1.y)) + ((a2.x + a2.y) + (a3.x + a3.y));
    s8 += __shfl_xor_sync(0xffffffffu, s8, 1);
    s8 += __shfl_xor_sync(0xffffffffu, s8, 2);
    if (cc == 0) xks[t * (NT * 8) + nt * 8 + gg] = s8;
  }
  // scales / zero points of the split's groups for this tile's columns
  for (int it = tid; it < ng * COLS; it += THREADS) {
    const int gi = it / COLS, col = it - gi * COLS, n = n_tile0 + col, gr = g_first + gi;
    float sv = 0.f, zv = 0.f;
    if (n < p.N) {
      sv = __half2float(p.scales[size_t(gr) * p.N + n]);
      if (p.zeros_packed) {
        const uint32_t wz =
            reinterpret_cast<const uint32_t*>(p.zeros)[size_t(gr) * (p.N >> 3) + (n >> 3)];
        zv = float(((wz >> ((n & 7) * 4)) & 0xFu) + unsigned(p.zero_offset));
      } else {
        zv = __half2float(reinterpret_cast<const __half*>(p.zeros)[size_t(gr) * p.N + n]);
      }
    }
    sc[it] = sv;
    zs[it] = zv;
  }
  __syncthreads();

  // 3. LoRA down-projection restricted to this split: h_s = x[:, Ks] . A[Ks, :]
  if (p.rank > 0) {
    const int RC = p.rank >> 3;  // 16-byte chunks per row of A (power of two <= 16)
    const int rpp = THREADS / RC;
    const int j = tid & (RC - 1), kr0 = tid / RC;
    const int Ks = Ts * KSTEP;
    const __half* Ab = p.A + size_t(k0) * p.rank + j * 8;
    float* hdst = p.hpart + size_t(tile * p.S + s) * M * p.rank;
    for (int mb = 0; mb < M; mb += HMC) {
      float acc[HMC][8];
#pragma unroll
      for (int mm = 0; mm < HMC; ++mm)
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[mm][i] = 0.f;
      for (int kr = kr0; kr < Ks; kr += rpp) {
        const uint4 av = ldg_v4(Ab + size_t(kr) * p.rank);
        const float2 f0 = h2_to_f2(av.x), f1 = h2_to_f2(av.y), f2 = h2_to_f2(av.z),
                     f3 = h2_to_f2(av.w);
        const float af[8] = {f0.x, f0.y, f1.x, f1.y, f2.x, f2.y, f3.x, f3.y};
        const int t = kr >> 5, cc = (kr >> 3) & 3, pos = inv_perm8(kr & 7);
#pragma unroll
        for (int mm = 0; mm < HMC; ++mm) {
          const int m = mb + mm;
          if (m < M) {
            const __half* xh =
                reinterpret_cast<const __half*>(xs + (t * NT + (m >> 3)) * 32 + (m & 7) * 4 + cc);
            const float xv = __half2float(xh[pos]);
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[mm][i] = fmaf(xv, af[i], acc[mm][i]);
          }
        }
      }
      for (int o = RC; o < 32; o <<= 1)
#pragma unroll
        for (int mm = 0; mm < HMC; ++mm)
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[mm][i] += __shfl_xor_sync(0xffffffffu, acc[mm][i], o);
      if (lane < RC)
#pragma unroll
        for (int mm = 0; mm < HMC; ++mm)
#pragma unroll
          for (int i = 0; i < 8; ++i) red[(warp * HMC + mm) * p.rank + lane * 8 + i] = acc[mm][i];
      __syncthreads();
      for (int it = tid; it < HMC * p.rank; it += THREADS) {
        const int mm = it / p.rank, r = it - mm * p.rank, m = mb + mm;
        if (m < M) {
          float v = 0.f;
#pragma unroll
          for (int wv = 0; wv < WARPS; ++wv) v += red[(wv * HMC + mm) * p.rank + r];
          hdst[m * p.rank + r] = v;
        }
      }
      __syncthreads();
    }
  }

  // 4. main loop: dequantise + tensor-core dot products
  float acc[2][NT][4], cg[2][NT][4], xsa[NT][2];
#pragma unroll
  for (int pp = 0; pp < 2; ++pp)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[pp][nt][i] = cg[pp][nt][i] = 0.f;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) xsa[nt][0] = xsa[nt][1] = 0.f;

  int cur = g_first;
  auto flush = [&](int gr) {
    const int off = (gr - g_first) * COLS + warp * 32 + 4 * g;
    const float4 s4 = *reinterpret_cast<const float4*>(sc + off);
    const float4 z4 = *reinterpret_cast<const float4*>(zs + off);
    const float sv[4] = {s4.x, s4.y, s4.z, s4.w};
    const float zv[4] = {z4.x, z4.y, z4.z, z4.w};
#pragma unroll
    for (int pp = 0; pp < 2; ++pp)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        acc[pp][nt][0] = fmaf(sv[2 * pp], cg[pp][nt][0] - zv[2 * pp] * xsa[nt][0], acc[pp][nt][0]);
        acc[pp][nt][1] = fmaf(sv[2 * pp], cg[pp][nt][1] - zv[2 * pp] * xsa[nt][1], acc[pp][nt][1]);
        acc[pp][nt][2] =
            fmaf(sv[2 * pp + 1], cg[pp][nt][2] - zv[2 * pp + 1] * xsa[nt][0], acc[pp][nt][2]);
        acc[pp][nt][3] =
            fmaf(sv[2 * pp + 1], cg[pp][nt][3] - zv[2 * pp + 1] * xsa[nt][1], acc[pp][nt][3]);
        cg[pp][nt][0] = cg[pp][nt][1] = cg[pp][nt][2] = cg[pp][nt][3] = 0.f;
      }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) xsa[nt][0] = xsa[nt][1] = 0.f;
  };

  for (int base = ks0; base < ks1; base += U) {
    if (base != ks0) {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int ks = base + u;
        w[u] = (col_ok && ks < ks1) ? ldg_stream_v4(qcol + size_t(ks * 4 + c) * p.N)
                                    : make_uint4(0u, 0u, 0u, 0u);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int ks = base + u;
      if (ks < ks1) {
        const int gr = (ks * KSTEP) / p.group;
        if (gr != cur) {
          flush(cur);
          cur = gr;
        }
        const uint32_t wv[4] = {w[u].x, w[u].y, w[u].z, w[u].w};
        uint32_t q[4][4];
#pragma unroll
        for (int jw = 0; jw < 4; ++jw) {
          const uint32_t lo = wv[jw], hi = wv[jw] >> 8;
          q[jw][0] = hsub2_u32(lop3_and_or(lo, 0x000F000Fu, 0x64006400u), 0x64006400u);  // (q0,q4)
          q[jw][1] = hfma2_u32(lop3_and_or(lo, 0x00F000F0u, 0x64006400u), 0x2C002C00u,
                               0xD400D400u);                                               // (q1,q5)
          q[jw][2] = hsub2_u32(lop3_and_or(hi, 0x000F000Fu, 0x64006400u), 0x64006400u);  // (q2,q6)
          q[jw][3] = hfma2_u32(lop3_and_or(hi, 0x00F000F0u, 0x64006400u), 0x2C002C00u,
                               0xD400D400u);                                               // (q3,q7)
        }
        const int t = ks - ks0;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const uint4 bx = xs[(t * NT + nt) * 32 + lane];
          const float2 xk = *reinterpret_cast<const float2*>(xks + t * (NT * 8) + nt * 8 + 2 * c);
          xsa[nt][0] += xk.x;
          xsa[nt][1] += xk.y;
#pragma unroll
          for (int pp = 0; pp < 2; ++pp) {
            mma_16816(cg[pp][nt], q[2 * pp][0], q[2 * pp + 1][0], q[2 * pp][1], q[2 * pp + 1][1],
                      bx.x, bx.y);
            mma_16816(cg[pp][nt], q[2 * pp][2], q[2 * pp + 1][2], q[2 * pp][3], q[2 * pp + 1][3],
                      bx.z, bx.w);
          }
        }
      }
    }
  }
  flush(cur);

  // 5. this split's base partials: rows (nt*8 + 2c, +1), columns (ncol + 2pp, +1)
  if (col_ok) {
    float* part = p.partial + size_t(s) * M * p.N;
#pragma unroll
    for (int pp = 0; pp < 2; ++pp)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int m0 = nt * 8 + 2 * c, n0 = ncol + 2 * pp;
        if (m0 < M)
          *reinterpret_cast<float2*>(part + size_t(m0) * p.N + n0) =
              make_float2(acc[pp][nt][0], acc[pp][nt][2]);
        if (m0 + 1 < M)
          *reinterpret_cast<float2*>(part + size_t(m0 + 1) * p.N + n0) =
              make_float2(acc[pp][nt][1], acc[pp][nt][3]);
      }
  }

  // 6. the last CTA of this tile reduces the splits in a fixed order
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned prev = atomicAdd(p.counters + tile, 1u);
    s_is_last = (prev == unsigned(p.S - 1)) ? 1u : 0u;
  }
  __syncthreads();
  if (!s_is_last) return;
  __threadfence();

  if (p.rank > 0) {
    for (int it = tid; it < M * p.rank; it += THREADS) {
      float v = 0.f;
      for (int s2 = 0; s2 < p.S; ++s2)
        v += __ldcg(p.hpart + size_t(tile * p.S + s2) * M * p.rank + it);
      hs[it] = v;
    }
    __syncthreads();
  }
  const int n = n_tile0 + tid;
  if (n < p.N) {
    for (int m = 0; m < M; ++m) {
      float base = 0.f;
      for (int s2 = 0; s2 < p.S; ++s2) base += __ldcg(p.partial + (size_t(s2) * M + m) * p.N + n);
      float lora = 0.f;
      for (int r = 0; r < p.rank; ++r)
        lora = fmaf(hs[m * p.rank + r], __half2float(p.B[size_t(r) * p.N + n]), lora);
      p.y[size_t(m) * p.N + n] = __float2half_rn(fmaf(p.lora_scale, lora, base));
    }
  }
  if (tid == 0) p.counters[tile] = 0u;  // leave the workspace zeroed for the next call
}

template <int NT>
static int launch(const Params& prm, const Plan& pl, cudaStream_t st) {
  auto kern = w4a16_gemv_kernel<NT>;
  if (pl.smem > 48 * 1024) {
    static std::mutex mu;
    static int done[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(mu);
    if (dev < 0 || dev >= 64 || done[dev] < int(pl.smem)) {
      QX_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(228 * 1024 - 1024)),
                  "w4a16_gemv: set smem limit");
      if (dev >= 0 && dev < 64) done[dev] = 228 * 1024;
    }
  }
  kern<<<dim3(pl.tiles, pl.S), THREADS, pl.smem, st>>>(prm);
  return check_launch("w4a16_gemv");
}

}  // namespace gemv
}  // namespace qx

using namespace qx;

extern "C" size_t qx_w4a16_gemv_workspace_size(int M, int K, int N, int rank, int group_size) {
  if (M <= 0 || K <= 0 || N <= 0 || group_size <= 0 || K % gemv::KSTEP) return 0;
  return gemv::make_plan(M, K, N, rank, group_size, device_sm_count()).total;
}

extern "C" int qx_w4a16_lora_gemv(const void* x, const int32_t* qweight, const void* scales,
                                  const void* zeros, int zeros_packed, int zero_offset,
                                  const void* lora_A, const void* lora_B, void* y, int M, int K,
                                  int N, int rank, int group_size, float lora_scale,
                                  void* workspace, size_t workspace_bytes, qx_stream_t stream) {
  QX_REQUIRE(M >= 0 && K > 0 && N > 0, "w4a16_gemv: bad sizes M=%d K=%d N=%d", M, K, N);
  if (M == 0) return QX_OK;
  QX_REQUIRE(K % gemv::KSTEP == 0, "w4a16_gemv: K=%d must be a multiple of 32", K);
  QX_REQUIRE(group_size > 0 && group_size % gemv::KSTEP == 0 && K % group_size == 0,
             "w4a16_gemv: group_size=%d must be a multiple of 32 dividing K=%d", group_size, K);
  QX_REQUIRE(N % 8 == 0, "w4a16_gemv: N=%d must be a multiple of 8", N);
  QX_REQUIRE(N <= gemv::COLS * gemv::COUNTER_SLOTS, "w4a16_gemv: N=%d too large", N);
  QX_REQUIRE(rank == 0 || rank == 8 || rank == 16 || rank == 32 || rank == 64 || rank == 128,
             "w4a16_gemv: LoRA rank %d unsupported (0, 8, 16, 32, 64 or 128)", rank);
  QX_REQUIRE(x && qweight && scales && zeros && y, "w4a16_gemv: null tensor pointer");
  QX_REQUIRE(rank == 0 || (lora_A && lora_B), "w4a16_gemv: rank=%d but lora_A/lora_B missing",
             rank);
  QX_REQUIRE(aligned(x, 16) && aligned(qweight, 16) && (rank == 0 || aligned(lora_A, 16)),
             "w4a16_gemv: x, qweight and lora_A must be 16-byte aligned");
  QX_REQUIRE(aligned(scales, 2) && aligned(zeros, 4) && aligned(y, 2) &&
                 (rank == 0 || aligned(lora_B, 2)),
             "w4a16_gemv: misaligned scales/zeros/y/lora_B");
  QX_REQUIRE(zeros_packed == 0 || zeros_packed == 1, "w4a16_gemv: zeros_packed must be 0 or 1");
  const int sms = device_sm_count();
  const gemv::Plan pl = gemv::make_plan(M, K, N, rank, group_size, sms);
  if (!workspace || workspace_bytes < pl.total || !aligned(workspace, 256))
    return fail(QX_ERR_WORKSPACE, "w4a16_gemv: workspace needs %zu bytes, 256-byte aligned (got %zu)",
                pl.total, workspace_bytes);
  if (pl.smem > size_t(227 * 1024))
    return fail(QX_ERR_UNSUPPORTED, "w4a16_gemv: shape needs %zu bytes of shared memory", pl.smem);

  unsigned char* ws = static_cast<unsigned char*>(workspace);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  for (int m0 = 0; m0 < M; m0 += gemv::MROWS) {
    const int mc = std::min(gemv::MROWS, M - m0);
    const gemv::Plan pc = gemv::make_plan(mc, K, N, rank, group_size, sms);
    gemv::Params prm{};
    prm.x = static_cast<const __half*>(x) + size_t(m0) * K;
    prm.qw = reinterpret_cast<const uint32_t*>(qweight);
    prm.scales = static_cast<const __half*>(scales);
    prm.zeros = zeros;
    prm.A = static_cast<const __half*>(lora_A);
    prm.B = static_cast<const __half*>(lora_B);
    prm.y = static_cast<__half*>(y) + size_t(m0) * N;
    prm.M = mc;
    prm.K = K;
    prm.N = N;
    prm.rank = rank;
    prm.group = group_size;
    prm.zeros_packed = zeros_packed;
    prm.zero_offset = zero_offset;
    prm.lora_scale = rank > 0 ? lora_scale : 0.f;
    prm.T = pc.T;
    prm.S = pc.S;
    prm.Ts_max = pc.Ts_max;
    prm.ng_max = pc.ng_max;
    prm.counters = reinterpret_cast<unsigned*>(ws);
    prm.partial = reinterpret_cast<float*>(ws + pc.off_partial);
    prm.hpart = reinterpret_cast<float*>(ws + pc.off_hpart);
    int rc;
    if (pc.NT == 1) rc = gemv::launch<1>(prm, pc, st);
    else if (pc.NT == 2) rc = gemv::launch<2>(prm, pc, st);
    else rc = gemv::launch<4>(prm, pc, st);
    if (rc != QX_OK) return rc;
  }
  return QX_OK;
}
