// W4A16 (GPTQ int4, group-wise scale/zero) + LoRA decode GEMV for sm_100a.
//
// Replaces the reference's two-launch path (lora_down_gemv_kernel +
// w4a16_lora_fused_gemv_kernel, csrc/kernels/w4a16_lora_gemv.cu:112-226):
// one launch streams every weight byte once from HBM and the LoRA terms ride
// along.  Math reproduced: y = fp16(x.W + (alpha/r)(x.A).B) with
// W = s (q - z) and fp32 accumulation (w4a16_lora_gemv.cu:183-224).
//
// Work decomposition
//   tile    = 256 output columns (8 warps x 32 columns).
//   cluster = the S CTAs that split one tile's K range (grid (tiles, S),
//             cluster dims (1, S, 1), S in {1,2,4,8,16}); sized so the whole
//             grid is resident in one wave.
//   k-step  = 32 rows of K = 4 packed int32 rows.  Lane (g = lane/4,
//             c = lane%4) loads one 128-bit word per k-step: packed row
//             4*ks + c, columns 4g..4g+3 of its warp, so each warp load is
//             4 rows x 128 contiguous bytes and every weight byte is loaded
//             once.  A rolling window of U k-steps stays in flight per thread.
//   dot     = nibbles become exact fp16 integers with the magic-number trick
//             (q | 0x6400 is the fp16 value 1024 + q; Kim et al., "Who Says
//             Elephants Can't Run", 2022) and feed mma.sync m16n8k16 with
//             fp32 accumulation: MMA rows = output columns, MMA columns =
//             batch rows (8 per n-tile), MMA k order = a fixed permutation of
//             the 32 rows of a k-step that the staged activations follow.
//             The zero point is folded out, sum_k (q-z)x = sum_k qx - z sum_k x,
//             once per group together with the fp32 scale, so fractional fp16
//             zeros stay exact.
//   static operands (scales, zeros, the CTA's slice of LoRA A, its share of
//             LoRA B) are staged into shared memory with cp.async right after
//             the weight loads are issued; activations are staged after
//             griddepcontrol.wait, so with programmatic dependent launch the
//             weight stream of this GEMV overlaps the previous kernel's tail.
//   reduce  = each CTA leaves its fp32 base partial and its LoRA partial
//             h_s = x[:, Ks] A[Ks, :] in shared memory; after a cluster
//             barrier, CTA j of the cluster sums columns [j*256/S, (j+1)*256/S)
//             over the S CTAs through distributed shared memory, in rank
//             order (deterministic), adds lora_scale * h.B and rounds once.
//             No global scratch, no atomics.
#include <cooperative_groups.h>

#include <algorithm>
#include <atomic>
#include <mutex>

#include "qx_b200.h"
#include "qx_common.cuh"

namespace cg = cooperative_groups;

namespace qx {

std::atomic<int> g_pdl_enabled{0};

namespace gemv {

constexpr int WARPS = 8;
constexpr int THREADS = WARPS * 32;
constexpr int COLS = WARPS * 32;  // output columns per tile
constexpr int KSTEP = 32;         // K rows per step (4 packed rows)
constexpr int U = 8;              // k-steps of weights in flight per thread
constexpr int MROWS = 32;         // batch rows per launch (4 n-tiles of 8)
constexpr int MAX_S = 16;         // largest cluster (non-portable size)
constexpr size_t SMEM_LIMIT = 227 * 1024;

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
};

// Shared-memory carve-up (byte offsets), identical on host and device.
struct Layout {
  unsigned xraw, xs, xks, sc, zs, As, Bs, part, hs, red, hsum, total;
};

__host__ __device__ inline unsigned take(unsigned& o, size_t bytes) {
  const unsigned r = o;
  o += unsigned((bytes + 127) & ~size_t(127));
  return r;
}

__host__ __device__ inline Layout layout(int NT, int Ts_max, int ng_max, int rank, int S) {
  Layout L;
  unsigned o = 0;
  const size_t Ksmax = size_t(Ts_max) * KSTEP, Mp = size_t(NT) * 8;
  L.xraw = take(o, Mp * Ksmax * 2);                 // activations [Mp][Ks] as loaded
  L.xs = take(o, size_t(Ts_max) * NT * 32 * 16);    // activations in MMA-B order
  L.xks = take(o, size_t(Ts_max) * NT * 8 * 4);     // per k-step row sums
  L.sc = take(o, size_t(ng_max) * COLS * 2);        // scales fp16 [ng][256]
  L.zs = take(o, size_t(ng_max) * COLS * 2);        // zeros fp16 [ng][256] or packed [ng][32]
  L.As = take(o, Ksmax * rank * 2);                 // LoRA A slice [Ks][r]
  L.Bs = take(o, size_t(rank) * (COLS / S) * 2);    // LoRA B share [r][256/S]
  L.part = take(o, Mp * COLS * 4);                  // base partial [Mp][256]
  L.hs = take(o, Mp * rank * 4);                    // h_s [Mp][r]
  L.red = take(o, size_t(THREADS) * Mp * 4);        // LoRA-down reduction scratch
  L.hsum = take(o, Mp * rank * 4);                  // h summed over the cluster
  L.total = o;
  return L;
}

struct Plan {
  int tiles, S, T, Ts_max, ng_max, NT;
  size_t smem;
};

static Plan make_plan(int M, int K, int N, int rank, int group, int sms) {
  Plan pl{};
  pl.tiles = (N + COLS - 1) / COLS;
  pl.T = K / KSTEP;
  const int mc = std::min(M, MROWS);
  pl.NT = mc <= 8 ? 1 : (mc <= 16 ? 2 : 4);
  const int target = sms * ctas_per_sm(pl.NT);
  int S = 1;
  while (S * 2 <= MAX_S && pl.tiles * S * 2 <= target && S * 2 <= pl.T) S *= 2;
  for (;;) {
    pl.S = S;
    pl.Ts_max = (pl.T + S - 1) / S;
    pl.ng_max = (pl.Ts_max * KSTEP + group - 1) / group + 1;
    pl.smem = layout(pl.NT, pl.Ts_max, pl.ng_max, rank, S).total;
    if (pl.smem <= SMEM_LIMIT || S * 2 > MAX_S || S * 2 > pl.T) break;
    S *= 2;
  }
  return pl;
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src, int src_bytes) {
  const unsigned d = static_cast<unsigned>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(src_bytes));
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  const unsigned d = static_cast<unsigned>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(d), "l"(src));
}
__device__ __forceinline__ void cp_async_commit_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;"); }

template <int NT>
__global__ void __launch_bounds__(THREADS, ctas_per_sm(NT)) w4a16_gemv_kernel(const Params p) {
  extern __shared__ __align__(128) unsigned char smem[];
  cg::cluster_group cluster = cg::this_cluster();

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int tile = blockIdx.x;
  const int s = blockIdx.y;  // == rank in the (1, S, 1) cluster
  const int S = p.S;
  const int ks0 = int((long long)s * p.T / S);
  const int ks1 = int((long long)(s + 1) * p.T / S);
  const int Ts = ks1 - ks0;
  const int Ks = Ts * KSTEP;
  const int Ksmax = p.Ts_max * KSTEP;
  const int M = p.M, N = p.N, R = p.rank;
  constexpr int Mp = NT * 8;
  const int n_tile0 = tile * COLS;
  const int lcol = warp * 32 + 4 * g;  // first of this lane's 4 columns (tile-local)
  const int ncol = n_tile0 + lcol;
  const bool col_ok = ncol < N;        // N % 8 == 0: all 4 columns valid or none
  const int k0 = ks0 * KSTEP;
  const int g_first = k0 / p.group;
  const int ng = (ks1 * KSTEP - 1) / p.group - g_first + 1;
  const int CPR = COLS / S;            // columns this CTA finalises

  const Layout L = layout(NT, p.Ts_max, p.ng_max, R, S);
  __half* xraw = reinterpret_cast<__half*>(smem + L.xraw);
  uint4* xs = reinterpret_cast<uint4*>(smem + L.xs);
  float* xks = reinterpret_cast<float*>(smem + L.xks);
  __half* sc = reinterpret_cast<__half*>(smem + L.sc);
  unsigned char* zsb = smem + L.zs;
  __half* As = reinterpret_cast<__half*>(smem + L.As);
  __half* Bs = reinterpret_cast<__half*>(smem + L.Bs);
  float* part = reinterpret_cast<float*>(smem + L.part);
  float* hs = reinterpret_cast<float*>(smem + L.hs);
  float* red = reinterpret_cast<float*>(smem + L.red);
  float* hsum = reinterpret_cast<float*>(smem + L.hsum);

  // 1. first window of weight loads (weights are static: no dependency wait)
  const uint32_t* qcol = p.qw + ncol;
  uint4 w[U];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int ks = ks0 + u;
    w[u] = (col_ok && ks < ks1) ? ldg_stream_v4(qcol + size_t(ks * 4 + c) * N)
                                : make_uint4(0u, 0u, 0u, 0u);
  }

  // 2. stage the static operands with cp.async
  for (int it = tid; it < ng * (COLS / 8); it += THREADS) {  // scales: 16 B = 8 columns
    const int gi = it / (COLS / 8), ch = it - gi * (COLS / 8), n = n_tile0 + ch * 8;
    const bool ok = n < N;
    cp_async16(sc + gi * COLS + ch * 8, ok ? p.scales + size_t(g_first + gi) * N + n : p.scales,
               ok ? 16 : 0);
  }
  if (p.zeros_packed) {
    const int words = N >> 3;
    for (int it = tid; it < ng * (COLS / 8); it += THREADS) {  // 1 word = 8 columns
      const int gi = it / (COLS / 8), wd = it - gi * (COLS / 8), wn = (n_tile0 >> 3) + wd;
      uint32_t* dst = reinterpret_cast<uint32_t*>(zsb) + gi * (COLS / 8) + wd;
      if (wn < words)
        cp_async4(dst, reinterpret_cast<const uint32_t*>(p.zeros) + size_t(g_first + gi) * words + wn);
      else
        *dst = 0u;
    }
  } else {
    const __half* zh = reinterpret_cast<const __half*>(p.zeros);
    for (int it = tid; it < ng * (COLS / 8); it += THREADS) {
      const int gi = it / (COLS / 8), ch = it - gi * (COLS / 8), n = n_tile0 + ch * 8;
      const bool ok = n < N;
      cp_async16(reinterpret_cast<__half*>(zsb) + gi * COLS + ch * 8,
                 ok ? zh + size_t(g_first + gi) * N + n : zh, ok ? 16 : 0);
    }
  }
  if (R > 0) {
    const int a_chunks = Ks * R / 8;  // contiguous slice A[k0 : k0 + Ks, :]
    const __half* Ab = p.A + size_t(k0) * R;
    for (int it = tid; it < a_chunks; it += THREADS) cp_async16(As + it * 8, Ab + it * 8, 16);
    const int bcpr = CPR / 8;  // 16-byte chunks per B row share
    const int cbase = n_tile0 + s * CPR;
    for (int it = tid; it < R * bcpr; it += THREADS) {
      const int rr = it / bcpr, ch = it - rr * bcpr, n = cbase + ch * 8;
      const bool ok = n < N;
      cp_async16(Bs + rr * CPR + ch * 8, ok ? p.B + size_t(rr) * N + n : p.B, ok ? 16 : 0);
    }
  }

  // 3. activations may be produced by the previous kernel in the stream
  grid_dep_wait();
  {
    const int xchunks = Ks / 8;
    for (int it = tid; it < M * xchunks; it += THREADS) {
      const int m = it / xchunks, ch = it - m * xchunks;
      cp_async16(xraw + m * Ksmax + ch * 8, p.x + size_t(m) * p.K + k0 + ch * 8, 16);
    }
  }
  cp_async_commit_wait_all();
  __syncthreads();
  grid_dep_launch();

  // 4. activations in MMA-B order (rows >= M are zero) and per-k-step row sums
  for (int it = tid; it < Ts * NT * 32; it += THREADS) {
    const int t = it / (NT * 32);
    const int rem = it - t * (NT * 32);
    const int nt = rem >> 5, l = rem & 31, gg = l >> 2, cc = l & 3;
    const int m = nt * 8 + gg;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (m < M) v = *reinterpret_cast<const uint4*>(xraw + m * Ksmax + t * KSTEP + cc * 8);
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
  __syncthreads();

  // 5. main loop: dequantise + tensor-core dot products, rolling load window
  float acc[2][NT][4], cgr[2][NT][4], xsa[NT][2];
#pragma unroll
  for (int pp = 0; pp < 2; ++pp)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[pp][nt][i] = cgr[pp][nt][i] = 0.f;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) xsa[nt][0] = xsa[nt][1] = 0.f;

  int cur = g_first;
  auto flush = [&](int gr) {
    const int gi = gr - g_first;
    const uint2 sv2 = *reinterpret_cast<const uint2*>(sc + gi * COLS + lcol);
    const float2 s01 = h2_to_f2(sv2.x), s23 = h2_to_f2(sv2.y);
    const float sv[4] = {s01.x, s01.y, s23.x, s23.y};
    float zv[4];
    if (p.zeros_packed) {
      const uint32_t wz = reinterpret_cast<const uint32_t*>(zsb)[gi * (COLS / 8) + (lcol >> 3)];
      const int sh = (lcol & 7) * 4;
#pragma unroll
      for (int j = 0; j < 4; ++j) zv[j] = float(((wz >> (sh + 4 * j)) & 0xFu) + unsigned(p.zero_offset));
    } else {
      const uint2 zv2 = *reinterpret_cast<const uint2*>(reinterpret_cast<const __half*>(zsb) + gi * COLS + lcol);
      const float2 z01 = h2_to_f2(zv2.x), z23 = h2_to_f2(zv2.y);
      zv[0] = z01.x;
      zv[1] = z01.y;
      zv[2] = z23.x;
      zv[3] = z23.y;
    }
#pragma unroll
    for (int pp = 0; pp < 2; ++pp)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        acc[pp][nt][0] = fmaf(sv[2 * pp], cgr[pp][nt][0] - zv[2 * pp] * xsa[nt][0], acc[pp][nt][0]);
        acc[pp][nt][1] = fmaf(sv[2 * pp], cgr[pp][nt][1] - zv[2 * pp] * xsa[nt][1], acc[pp][nt][1]);
        acc[pp][nt][2] =
            fmaf(sv[2 * pp + 1], cgr[pp][nt][2] - zv[2 * pp + 1] * xsa[nt][0], acc[pp][nt][2]);
        acc[pp][nt][3] =
            fmaf(sv[2 * pp + 1], cgr[pp][nt][3] - zv[2 * pp + 1] * xsa[nt][1], acc[pp][nt][3]);
        cgr[pp][nt][0] = cgr[pp][nt][1] = cgr[pp][nt][2] = cgr[pp][nt][3] = 0.f;
      }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) xsa[nt][0] = xsa[nt][1] = 0.f;
  };

  for (int base = ks0; base < ks1; base += U) {
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
        {  // refill this slot with the k-step U ahead
          const int kn = ks + U;
          w[u] = (col_ok && kn < ks1) ? ldg_stream_v4(qcol + size_t(kn * 4 + c) * N)
                                      : make_uint4(0u, 0u, 0u, 0u);
        }
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
            mma_16816(cgr[pp][nt], q[2 * pp][0], q[2 * pp + 1][0], q[2 * pp][1], q[2 * pp + 1][1],
                      bx.x, bx.y);
            mma_16816(cgr[pp][nt], q[2 * pp][2], q[2 * pp + 1][2], q[2 * pp][3], q[2 * pp + 1][3],
                      bx.z, bx.w);
          }
        }
      }
    }
  }
  flush(cur);

  // 6. base partial into shared memory: rows nt*8 + 2c (+1), columns lcol + 2pp (+1)
#pragma unroll
  for (int pp = 0; pp < 2; ++pp)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int m0 = nt * 8 + 2 * c, cl = lcol + 2 * pp;
      *reinterpret_cast<float2*>(part + m0 * COLS + cl) = make_float2(acc[pp][nt][0], acc[pp][nt][2]);
      *reinterpret_cast<float2*>(part + (m0 + 1) * COLS + cl) =
          make_float2(acc[pp][nt][1], acc[pp][nt][3]);
    }

  // 7. LoRA down-projection over this CTA's K range: h_s = x[:, Ks] . A[Ks, :]
  if (R > 0) {
    const int j = tid % R, kq = tid / R, nq = THREADS / R;  // R divides 256
    for (int mb = 0; mb < M; mb += 8) {
      float a8[8];
#pragma unroll
      for (int mm = 0; mm < 8; ++mm) a8[mm] = 0.f;
      for (int k = kq; k < Ks; k += nq) {
        const float av = __half2float(As[k * R + j]);
#pragma unroll
        for (int mm = 0; mm < 8; ++mm)
          if (mb + mm < M) a8[mm] = fmaf(__half2float(xraw[(mb + mm) * Ksmax + k]), av, a8[mm]);
      }
#pragma unroll
      for (int mm = 0; mm < 8; ++mm)
        if (mb + mm < M) red[(kq * Mp + mb + mm) * R + j] = a8[mm];
    }
    __syncthreads();
    for (int it = tid; it < M * R; it += THREADS) {
      const int m = it / R, jj = it - m * R;
      float v = 0.f;
      for (int q2 = 0; q2 < nq; ++q2) v += red[(q2 * Mp + m) * R + jj];
      hs[m * R + jj] = v;
    }
  }

  // 8. cluster reduction through distributed shared memory
  cluster.sync();
  if (R > 0) {
    for (int it = tid; it < M * R; it += THREADS) {
      float v = 0.f;
      for (int r2 = 0; r2 < S; ++r2) v += cluster.map_shared_rank(hs, r2)[it];
      hsum[it] = v;
    }
    __syncthreads();
  }
  for (int it = tid; it < M * CPR; it += THREADS) {
    const int m = it / CPR, cc = it - m * CPR;
    const int cl = s * CPR + cc, n = n_tile0 + cl;
    if (n < N) {
      float vals[MAX_S];
#pragma unroll
      for (int r2 = 0; r2 < MAX_S; ++r2)
        vals[r2] = r2 < S ? cluster.map_shared_rank(part, r2)[m * COLS + cl] : 0.f;
      float base = 0.f;
#pragma unroll
      for (int r2 = 0; r2 < MAX_S; ++r2) base += vals[r2];
      float lora = 0.f;
      for (int jj = 0; jj < R; ++jj) lora = fmaf(hsum[m * R + jj], __half2float(Bs[jj * CPR + cc]), lora);
      p.y[size_t(m) * N + n] = __float2half_rn(fmaf(p.lora_scale, lora, base));
    }
  }
  cluster.sync();  // peers may still be reading this CTA's shared memory
}

template <int NT>
static int launch(const Params& prm, const Plan& pl, cudaStream_t st) {
  auto kern = w4a16_gemv_kernel<NT>;
  static std::mutex mu;
  static bool attr_done[64][3] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lk(mu);
    const int ti = NT == 1 ? 0 : NT == 2 ? 1 : 2;
    if (dev < 0 || dev >= 64 || !attr_done[dev][ti]) {
      QX_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(SMEM_LIMIT)),
                  "w4a16_gemv: set smem limit");
      QX_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1),
                  "w4a16_gemv: allow 16-CTA clusters");
      if (dev >= 0 && dev < 64) attr_done[dev][ti] = true;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.tiles, pl.S, 1);
  cfg.blockDim = dim3(THREADS, 1, 1);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = st;
  cudaLaunchAttribute attrs[2];
  int na = 0;
  attrs[na].id = cudaLaunchAttributeClusterDimension;
  attrs[na].val.clusterDim.x = 1;
  attrs[na].val.clusterDim.y = pl.S;
  attrs[na].val.clusterDim.z = 1;
  ++na;
  if (g_pdl_enabled.load(std::memory_order_relaxed)) {
    attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = na;
  QX_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, prm), "w4a16_gemv: launch");
  return check_launch("w4a16_gemv");
}

}  // namespace gemv
}  // namespace qx

using namespace qx;

extern "C" int qx_set_pdl(int enable) {
  g_pdl_enabled.store(enable ? 1 : 0);
  return QX_OK;
}

extern "C" int qx_w4a16_lora_gemv(const void* x, const int32_t* qweight, const void* scales,
                                  const void* zeros, int zeros_packed, int zero_offset,
                                  const void* lora_A, const void* lora_B, void* y, int M, int K,
                                  int N, int rank, int group_size, float lora_scale,
                                  qx_stream_t stream) {
  QX_REQUIRE(M >= 0 && K > 0 && N > 0, "w4a16_gemv: bad sizes M=%d K=%d N=%d", M, K, N);
  if (M == 0) return QX_OK;
  QX_REQUIRE(K % gemv::KSTEP == 0, "w4a16_gemv: K=%d must be a multiple of 32", K);
  QX_REQUIRE(group_size > 0 && group_size % gemv::KSTEP == 0 && K % group_size == 0,
             "w4a16_gemv: group_size=%d must be a multiple of 32 dividing K=%d", group_size, K);
  QX_REQUIRE(N % 8 == 0, "w4a16_gemv: N=%d must be a multiple of 8", N);
  QX_REQUIRE(rank == 0 || rank == 8 || rank == 16 || rank == 32 || rank == 64 || rank == 128,
             "w4a16_gemv: LoRA rank %d unsupported (0, 8, 16, 32, 64 or 128)", rank);
  QX_REQUIRE(x && qweight && scales && zeros && y, "w4a16_gemv: null tensor pointer");
  QX_REQUIRE(rank == 0 || (lora_A && lora_B), "w4a16_gemv: rank=%d but lora_A/lora_B missing",
             rank);
  QX_REQUIRE(aligned(x, 16) && aligned(qweight, 16) && aligned(scales, 16) &&
                 (rank == 0 || (aligned(lora_A, 16) && aligned(lora_B, 16))),
             "w4a16_gemv: x, qweight, scales, lora_A and lora_B must be 16-byte aligned");
  QX_REQUIRE(aligned(zeros, zeros_packed ? 4 : 16) && aligned(y, 2),
             "w4a16_gemv: misaligned zeros/y");
  QX_REQUIRE(zeros_packed == 0 || zeros_packed == 1, "w4a16_gemv: zeros_packed must be 0 or 1");
  const int sms = device_sm_count();
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  for (int m0 = 0; m0 < M; m0 += gemv::MROWS) {
    const int mc = std::min(gemv::MROWS, M - m0);
    const gemv::Plan pc = gemv::make_plan(mc, K, N, rank, group_size, sms);
    if (pc.smem > gemv::SMEM_LIMIT)
      return fail(QX_ERR_UNSUPPORTED, "w4a16_gemv: shape needs %zu bytes of shared memory",
                  pc.smem);
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
    int rc;
    if (pc.NT == 1) rc = gemv::launch<1>(prm, pc, st);
    else if (pc.NT == 2) rc = gemv::launch<2>(prm, pc, st);
    else rc = gemv::launch<4>(prm, pc, st);
    if (rc != QX_OK) return rc;
  }
  return QX_OK;
}
