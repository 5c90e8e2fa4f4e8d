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
//   dot     = one LOP3 per nibble pair builds exact fp16 operands with the
//             magic-number trick (Kim et al., "Who Says Elephants Can't Run",
//             2022): (v & 0x000F000F) | 0x64006400 is the half2 (1024 + q_i,
//             1024 + q_{i+4}) and (v & 0x00F000F0) | 0x64006400 is
//             (1024 + 16 q_{i+1}, ...).  These feed mma.sync m16n8k16 with
//             fp32 accumulation as they are: the activations staged for the
//             "x16" slots are pre-scaled by 1/16 (exact), so every product is
//             (1024 + q) x or (64 + q) x, and the offsets are removed with the
//             zero point once per group:
//               sum (q - z) x = C - (1024 + z) Xa - (64 + z) Xb,
//             Xa / Xb = sums of x over the two nibble classes.  MMA rows are
//             output columns, MMA columns batch rows (8 per n-tile), the MMA
//             k order a fixed permutation of a k-step that the staged
//             activations follow.  5 integer ops per 8 weights.
//   LoRA    = h_s = x[:, Ks] A[Ks, :] on the tensor cores (ldmatrix.trans of
//             the staged A slice), the LoRA product being linear in K.
//   static operands (scales, zeros, A slice, B share) are staged into shared
//             memory with cp.async right after the weight loads are issued;
//             activations are staged after griddepcontrol.wait, so with
//             programmatic dependent launch the weight stream overlaps the
//             previous kernel's tail.
//   reduce  = each CTA leaves its fp32 base partial and h_s in shared memory;
//             after a cluster barrier CTA j sums columns [j*256/S, (j+1)*256/S)
//             over the S CTAs through distributed shared memory in rank order
//             (deterministic), adds lora_scale * h.B and rounds once.  No
//             global scratch, no atomics.
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

// row stride of the staged activations (halves): +8 keeps ldmatrix rows on
// distinct banks
__host__ __device__ inline int xstride(int Ts_max) { return Ts_max * KSTEP + 8; }

__host__ __device__ inline Layout layout(int NT, int Ts_max, int ng_max, int rank, int S) {
  Layout L;
  unsigned o = 0;
  const size_t Ksmax = size_t(Ts_max) * KSTEP, Mp = size_t(NT) * 8;
  L.xraw = take(o, Mp * xstride(Ts_max) * 2);       // activations [Mp][Ks(+8)] as loaded
  L.xs = take(o, size_t(Ts_max) * NT * 32 * 16);    // activations in MMA-B order
  L.xks = take(o, size_t(Ts_max) * NT * 8 * 2 * 4); // per k-step (Xa, Xb) per row
  L.sc = take(o, size_t(ng_max) * COLS * 2);        // scales fp16 [ng][256]
  L.zs = take(o, size_t(ng_max) * COLS * 2);        // zeros fp16 [ng][256] or packed [ng][32]
  L.As = take(o, Ksmax * rank * 2);                 // LoRA A slice [Ks][r]
  L.Bs = take(o, size_t(rank) * (COLS / S) * 2);    // LoRA B share [r][256/S]
  L.part = take(o, Mp * COLS * 4);                  // base partial [Mp][256]
  L.hs = take(o, Mp * rank * 4);                    // h_s [Mp][r]
  L.red = take(o, size_t(WARPS) * 16 * 8 * 4);      // LoRA-down split-k partials
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
  const int kpg = group / KSTEP;
  const int Gt = K / group;  // splits hold whole quantisation groups
  int S = 1;
  while (S * 2 <= MAX_S && pl.tiles * S * 2 <= target && S * 2 <= Gt) S *= 2;
  for (;;) {
    pl.S = S;
    pl.ng_max = (Gt + S - 1) / S;
    pl.Ts_max = pl.ng_max * kpg;
    pl.smem = layout(pl.NT, pl.Ts_max, pl.ng_max, rank, S).total;
    if (pl.smem <= SMEM_LIMIT || S * 2 > MAX_S || S * 2 > Gt) break;
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
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  const unsigned a = static_cast<unsigned>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}
__device__ __forceinline__ void ldsm_x2(uint32_t (&r)[2], const void* p) {
  const unsigned a = static_cast<unsigned>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
               : "=r"(r[0]), "=r"(r[1])
               : "r"(a));
}
// Weights are read once per call: load them with an L2 evict-first policy so
// the stream does not push activations, scales or code out of L2.
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ uint4 ldg_weights(const void* ptr, uint64_t pol) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(ptr), "l"(pol));
  return r;
}
__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// KPG = k-steps per quantisation group (group_size / 32): splits cover whole
// groups, so the per-group correction sits at compile-time positions of the
// unrolled main loop.
template <int NT, int KPG>
__global__ void __launch_bounds__(THREADS, ctas_per_sm(NT)) w4a16_gemv_kernel(const Params p) {
  extern __shared__ __align__(128) unsigned char smem[];
  cg::cluster_group cluster = cg::this_cluster();

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int tile = blockIdx.x;
  const int s = blockIdx.y;  // == rank in the (1, S, 1) cluster
  const int S = p.S;
  const int Gt = p.T / KPG;  // quantisation groups along K
  const int ks0 = (s * Gt / S) * KPG;
  const int ks1 = ((s + 1) * Gt / S) * KPG;
  const int Ts = ks1 - ks0;
  const int Ks = Ts * KSTEP;
  const int XS = xstride(p.Ts_max);
  const int M = p.M, N = p.N, R = p.rank;
  constexpr int Mp = NT * 8;
  const int n_tile0 = tile * COLS;
  const int lcol = warp * 32 + 4 * g;  // first of this lane's 4 columns (tile-local)
  const int ncol = n_tile0 + lcol;
  const bool col_ok = ncol < N;        // N % 8 == 0: all 4 columns valid or none
  const int k0 = ks0 * KSTEP;
  const int g_first = ks0 / KPG;
  const int ng = (ks1 - ks0) / KPG;
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
  const size_t row_step = size_t(4) * N;  // one k-step down the packed rows
  const uint32_t* ld_ptr = p.qw + size_t(ks0 * 4 + c) * N + ncol;
  const uint64_t pol = evict_first_policy();
  uint4 w[U];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    w[u] = (col_ok && ks0 + u < ks1) ? ldg_weights(ld_ptr, pol) : make_uint4(0u, 0u, 0u, 0u);
    ld_ptr += row_step;
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
    const int a_chunks = (Ks * R) >> 3;  // contiguous slice A[k0 : k0 + Ks, :]
    const __half* Ab = p.A + size_t(k0) * R;
    for (int it = tid; it < a_chunks; it += THREADS) cp_async16(As + it * 8, Ab + it * 8, 16);
    const int bcpr = CPR >> 3;  // 16-byte chunks per B row share
    const int cbase = n_tile0 + s * CPR;
    for (int it = tid; it < R * bcpr; it += THREADS) {
      const int rr = it / bcpr, ch = it - rr * bcpr, n = cbase + ch * 8;
      const bool ok = n < N;
      cp_async16(Bs + rr * CPR + ch * 8, ok ? p.B + size_t(rr) * N + n : p.B, ok ? 16 : 0);
    }
  }

  // 3. activations may be produced by the previous kernel in the stream;
  //    rows >= M are zero-filled
  grid_dep_wait();
  {
    const int xchunks = Ks >> 3;
    for (int it = tid; it < Mp * xchunks; it += THREADS) {
      const int m = it / xchunks, ch = it - m * xchunks;
      const bool ok = m < M;
      cp_async16(xraw + m * XS + ch * 8, ok ? p.x + size_t(m) * p.K + k0 + ch * 8 : p.x,
                 ok ? 16 : 0);
    }
  }
  cp_async_commit_wait_all();
  __syncthreads();
  grid_dep_launch();

  // 4. activations in MMA-B order: (x0, x4, x1/16, x5/16, x2, x6, x3/16, x7/16)
  //    per packed row, plus per-k-step sums over the two nibble classes
  for (int it = tid; it < Ts * NT * 32; it += THREADS) {
    const int t = it / (NT * 32);
    const int rem = it - t * (NT * 32);
    const int nt = rem >> 5, l = rem & 31, gg = l >> 2, cc = l & 3;
    const int m = nt * 8 + gg;
    const uint4 v = *reinterpret_cast<const uint4*>(xraw + m * XS + t * KSTEP + cc * 8);
    uint4 o;
    o.x = prmt(v.x, v.z, 0x5410u);                         // (x0, x4)
    o.y = hmul2_u32(prmt(v.x, v.z, 0x7632u), 0x2C002C00u);  // (x1, x5) / 16
    o.z = prmt(v.y, v.w, 0x5410u);                         // (x2, x6)
    o.w = hmul2_u32(prmt(v.y, v.w, 0x7632u), 0x2C002C00u);  // (x3, x7) / 16
    xs[it] = o;
    const float2 a0 = h2_to_f2(v.x), a1 = h2_to_f2(v.y), a2 = h2_to_f2(v.z), a3 = h2_to_f2(v.w);
    float xa = (a0.x + a1.x) + (a2.x + a3.x);  // x0 + x2 + x4 + x6
    float xb = (a0.y + a1.y) + (a2.y + a3.y);  // x1 + x3 + x5 + x7
    xa += __shfl_xor_sync(0xffffffffu, xa, 1);
    xa += __shfl_xor_sync(0xffffffffu, xa, 2);
    xb += __shfl_xor_sync(0xffffffffu, xb, 1);
    xb += __shfl_xor_sync(0xffffffffu, xb, 2);
    if (cc == 0)
      *reinterpret_cast<float2*>(xks + ((t * NT + nt) * 8 + gg) * 2) = make_float2(xa, xb);
  }
  __syncthreads();

  // 5. main loop: tensor-core dot products on raw magic-number operands
  float acc[2][NT][4], cgr[2][NT][4], xsa[NT][4];  // xsa: (Xa, Xb) for rows 2c, 2c+1
#pragma unroll
  for (int pp = 0; pp < 2; ++pp)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[pp][nt][i] = cgr[pp][nt][i] = 0.f;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) xsa[nt][0] = xsa[nt][1] = xsa[nt][2] = xsa[nt][3] = 0.f;

  auto flush = [&](int gi) {
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
      const uint2 zv2 =
          *reinterpret_cast<const uint2*>(reinterpret_cast<const __half*>(zsb) + gi * COLS + lcol);
      const float2 z01 = h2_to_f2(zv2.x), z23 = h2_to_f2(zv2.y);
      zv[0] = z01.x;
      zv[1] = z01.y;
      zv[2] = z23.x;
      zv[3] = z23.y;
    }
#pragma unroll
    for (int pp = 0; pp < 2; ++pp) {
      const float za0 = 1024.f + zv[2 * pp], zb0 = 64.f + zv[2 * pp];
      const float za1 = 1024.f + zv[2 * pp + 1], zb1 = 64.f + zv[2 * pp + 1];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const float* xv = xsa[nt];
        acc[pp][nt][0] = fmaf(sv[2 * pp], cgr[pp][nt][0] - za0 * xv[0] - zb0 * xv[1], acc[pp][nt][0]);
        acc[pp][nt][1] = fmaf(sv[2 * pp], cgr[pp][nt][1] - za0 * xv[2] - zb0 * xv[3], acc[pp][nt][1]);
        acc[pp][nt][2] =
            fmaf(sv[2 * pp + 1], cgr[pp][nt][2] - za1 * xv[0] - zb1 * xv[1], acc[pp][nt][2]);
        acc[pp][nt][3] =
            fmaf(sv[2 * pp + 1], cgr[pp][nt][3] - za1 * xv[2] - zb1 * xv[3], acc[pp][nt][3]);
        cgr[pp][nt][0] = cgr[pp][nt][1] = cgr[pp][nt][2] = cgr[pp][nt][3] = 0.f;
      }
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) xsa[nt][0] = xsa[nt][1] = xsa[nt][2] = xsa[nt][3] = 0.f;
  };

  static_assert(U % KPG == 0, "a register window holds whole groups");
  int gi_cur = 0;  // group index relative to g_first
  for (int base = ks0; base < ks1; base += U) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int ks = base + u;
      if (ks < ks1) {
        const uint32_t wv[4] = {w[u].x, w[u].y, w[u].z, w[u].w};
        w[u] = (col_ok && ks + U < ks1) ? ldg_weights(ld_ptr, pol) : make_uint4(0u, 0u, 0u, 0u);
        ld_ptr += row_step;
        uint32_t q[4][4];
#pragma unroll
        for (int jw = 0; jw < 4; ++jw) {
          const uint32_t hi = wv[jw] >> 8;
          q[jw][0] = lop3_and_or(wv[jw], 0x000F000Fu, 0x64006400u);  // (1024+q0, 1024+q4)
          q[jw][1] = lop3_and_or(wv[jw], 0x00F000F0u, 0x64006400u);  // (1024+16q1, 1024+16q5)
          q[jw][2] = lop3_and_or(hi, 0x000F000Fu, 0x64006400u);      // (1024+q2, 1024+q6)
          q[jw][3] = lop3_and_or(hi, 0x00F000F0u, 0x64006400u);      // (1024+16q3, 1024+16q7)
        }
        const int t = ks - ks0;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const uint4 bx = xs[(t * NT + nt) * 32 + lane];
          const float4 xk = *reinterpret_cast<const float4*>(xks + ((t * NT + nt) * 8 + 2 * c) * 2);
          xsa[nt][0] += xk.x;
          xsa[nt][1] += xk.y;
          xsa[nt][2] += xk.z;
          xsa[nt][3] += xk.w;
#pragma unroll
          for (int pp = 0; pp < 2; ++pp) {
            mma_16816(cgr[pp][nt], q[2 * pp][0], q[2 * pp + 1][0], q[2 * pp][1], q[2 * pp + 1][1],
                      bx.x, bx.y);
            mma_16816(cgr[pp][nt], q[2 * pp][2], q[2 * pp + 1][2], q[2 * pp][3], q[2 * pp + 1][3],
                      bx.z, bx.w);
          }
        }
        if ((u + 1) % KPG == 0) {  // last k-step of a group (splits hold whole groups)
          flush(gi_cur);
          ++gi_cur;
        }
      }
    }
  }

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

  // 7. LoRA down-projection on the tensor cores: h_s^T[r][m] = A^T[r][Ks] . x^T[Ks][m]
  //    16 x 8 output tiles (rank rows x batch rows); tiles over warps, and
  //    when there are fewer tiles than warps the K range is split as well.
  if (R > 0) {
    const int RT = R >= 16 ? R / 16 : 1;
    const int ntiles = RT * NT;
    const int nsplit = ntiles >= WARPS ? 1 : WARPS / ntiles;
    const int KB = Ks / 16;
    for (int tl = warp % ntiles; tl < ntiles; tl += (ntiles >= WARPS ? WARPS : ntiles)) {
      const int rt = tl / NT, nt = tl - rt * NT;
      const int part_k = ntiles >= WARPS ? 0 : warp / ntiles;
      float h4[4] = {0.f, 0.f, 0.f, 0.f};
      const int mi = lane >> 3, ri = lane & 7;
      for (int kb = part_k; kb < KB; kb += nsplit) {
        uint32_t a[4];
        {
          const int k = kb * 16 + ri + 8 * (mi >> 1);
          const int j = rt * 16 + 8 * (mi & 1);
          if (R >= 16) {
            ldsm_x4_t(a, As + k * R + j);
          } else {  // rank 8: rows 8..15 of the tile are zero
            ldsm_x4_t(a, As + k * R + (j & 7));
            a[1] = 0u;
            a[3] = 0u;
          }
        }
        uint32_t b[2];
        {
          const int l16 = lane & 15;
          ldsm_x2(b, xraw + (nt * 8 + (l16 & 7)) * XS + kb * 16 + 8 * (l16 >> 3));
        }
        mma_16816(h4, a[0], a[1], a[2], a[3], b[0], b[1]);
      }
      // h4: (rank row g, batch 2c/2c+1) and (rank row g+8, ...)
      if (nsplit == 1) {
        const int j0 = rt * 16 + g, m0 = nt * 8 + 2 * c;
        hs[m0 * R + j0] = h4[0];
        hs[(m0 + 1) * R + j0] = h4[1];
        if (j0 + 8 < R) {
          hs[m0 * R + j0 + 8] = h4[2];
          hs[(m0 + 1) * R + j0 + 8] = h4[3];
        }
      } else {
        float* rw = red + warp * 128;  // [16][8]
        rw[g * 8 + 2 * c] = h4[0];
        rw[g * 8 + 2 * c + 1] = h4[1];
        rw[(g + 8) * 8 + 2 * c] = h4[2];
        rw[(g + 8) * 8 + 2 * c + 1] = h4[3];
      }
    }
    if (nsplit > 1) {
      __syncthreads();
      for (int it = tid; it < ntiles * 128; it += THREADS) {
        const int tl = it >> 7, e = it & 127, jr = e >> 3, mc = e & 7;
        const int rt = tl / NT, nt = tl - rt * NT;
        float v = 0.f;
        for (int q2 = 0; q2 < nsplit; ++q2) v += red[(q2 * ntiles + tl) * 128 + e];
        const int j = rt * 16 + jr;
        if (j < R) hs[(nt * 8 + mc) * R + j] = v;
      }
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

template <int NT, int KPG>
static int launch(const Params& prm, const Plan& pl, cudaStream_t st) {
  auto kern = w4a16_gemv_kernel<NT, KPG>;
  static std::mutex mu;
  static bool attr_done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lk(mu);
    const int ti = 0;
    if (dev < 0 || dev >= 64 || !attr_done[dev + ti]) {
      QX_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(SMEM_LIMIT)),
                  "w4a16_gemv: set smem limit");
      QX_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1),
                  "w4a16_gemv: allow 16-CTA clusters");
      if (dev >= 0 && dev < 64) attr_done[dev + ti] = true;
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

template <int NT>
static int dispatch_kpg(const Params& prm, const Plan& pl, int kpg, cudaStream_t st) {
  switch (kpg) {
    case 1: return launch<NT, 1>(prm, pl, st);
    case 2: return launch<NT, 2>(prm, pl, st);
    case 4: return launch<NT, 4>(prm, pl, st);
    default: return launch<NT, 8>(prm, pl, st);
  }
}

static int dispatch(const Params& prm, const Plan& pl, int kpg, cudaStream_t st) {
  if (pl.NT == 1) return dispatch_kpg<1>(prm, pl, kpg, st);
  if (pl.NT == 2) return dispatch_kpg<2>(prm, pl, kpg, st);
  return dispatch_kpg<4>(prm, pl, kpg, st);
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
  QX_REQUIRE((group_size == 32 || group_size == 64 || group_size == 128 || group_size == 256) &&
                 K % group_size == 0,
             "w4a16_gemv: group_size=%d must be 32, 64, 128 or 256 and divide K=%d", group_size, K);
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
    const int rc = gemv::dispatch(prm, pc, group_size / gemv::KSTEP, st);
    if (rc != QX_OK) return rc;
  }
  return QX_OK;
}
