// Decode W4A16-LoRA GEMV with the call's whole weight slice resident in
// shared memory before the dependency wait (a few rows, weights that fit).
//
// Same math as the clustered split-K GEMV in w4a16_gemv.cu and the reference
// path it replaces (w4a16_lora_gemv.cu:112-226): y = fp16(x.W + s_l (x.A).B)
// with W = s (q - z), one rounding at the end.
//
// Why a second decode kernel.  At one row the GEMV streams ~13 MB and its
// arithmetic after the activations arrive takes about a microsecond, so the
// call time is set by how early the weights start to move.  Programmatic
// dependent launch lets a call start streaming while the previous call
// computes, but only if its CTAs can be resident beside the previous call's.
// This kernel is sized for that: one CTA per SM, under half of the SM's
// shared memory (~112 KB at the Qwen3-4B gate_proj shape) and registers
// (__launch_bounds__(288, 2)), so consecutive calls overlap; the whole weight
// slice is requested by TMA before the wait.
//
// Work decomposition
//   CTA i owns the 8-column units [i U / P, (i+1) U / P) (U = N / 8, P CTAs,
//   one per SM) over the full K: no split-K, no reduction of y between CTAs.
//   One TMA box per 256 packed rows covers nb units (nb = the largest unit
//   count, rounded up to odd: the row pitch of nb*32 bytes then puts the four
//   packed rows of an MMA fragment in distinct banks); a CTA with fewer units
//   reads its neighbour's first unit as padding (an L2 hit).
//   LoRA down-projection: the P CTAs form clusters of C (2 by preference: a
//   pair of CTAs always fits one CTA per SM inside a GPC); CTA rank q computes
//   h_q = x[:, Kq] A[Kq, :] over its K / C rows (A loaded into registers
//   before the wait) and st.async-broadcasts h_q to every CTA of its cluster,
//   which sums the C parts in rank order: h is exchanged, not recomputed.
//   Warps: 8 compute warps + 1 producer (barriers, TMA, packed zero points).
//   The compute warps split the CTA's (16-column tile, quantisation group)
//   items in tile-major order into 8 contiguous ranges; partial sums meet in
//   shared memory and are added in warp order (deterministic).
//
// Integer tensor-core main loop.  The int4 dequantisation on the integer ALU
// bounds a half-precision MMA formulation (5 ALU operations per 8 weights at
// half the issue rate of an MMA).  Here the weights stay integers:
//   A operand (u8): for the word w of packed row p, lo = w & 0x0F0F0F0F holds
//   the even nibbles (rows 8p, 8p+2, 8p+4, 8p+6) and hi = (w >> 4) &
//   0x0F0F0F0F the odd ones: 3 operations per 8 weights, and one
//   mma.sync m16n8k32 (u8 x s8 / u8 x u8, int32 accumulate) covers 32 rows.
//   B operand: the activations of each (row, quantisation group) as exact
//   fixed point X = rint(x * 2^(14-E)) with 2^E >= max|x| of the group
//   (|X| < 2^14), split into X = 256 H + L with H signed and L unsigned bytes;
//   one MMA per digit.  Per group C = 256 C_H + C_L = sum_k q_k X_k exactly
//   (int32), and the group adds s 2^(E-14) (C - z sum_k X_k) to the fp32
//   accumulator.  The fixed point costs at most 2^-14 of the group's largest
//   activation per element (fp16 keeps 11 bits); a one-hot activation is
//   exact, so a dequantised weight reads back bit-exact.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <map>
#include <mutex>
#include <tuple>

#include "qx_b200.h"
#include "qx_common.cuh"

namespace qx {

extern std::atomic<int> g_pdl_enabled;  // w4a16_gemv.cu

namespace gres {

constexpr int WARPS = 8;                   // compute warps
constexpr int THREADS = (WARPS + 1) * 32;  // + the producer warp
constexpr int KSTEP = 32;                  // K rows per k-step (4 packed rows)
constexpr int MAX_M = 4;                   // batch rows (MMA n8; staged activations bound it)
constexpr int MAX_NB = 31;                 // units per TMA box (248 columns: a box is <= 256 wide)
constexpr int MAX_CHUNKS = 8;              // weight boxes per CTA (<= 256 packed rows each)
constexpr int NI_MAX = 10;                 // LoRA A uint4 loads per compute thread
constexpr size_t SMEM_BUDGET = 112 * 1024; // two CTAs per SM: 228 KB less 1 KB per CTA

static __device__ unsigned g_res_error = 0;

struct Layout {
  unsigned bars, w, sc, zq, bl, xd, xh, xsum, hr, hw, hs, red, total;
};

struct alignas(64) Params {
  CUtensorMap tw;  // qweight int32 [K/8][N], box {nb*8, rows_box}
  CUtensorMap ts;  // scales fp16 [G][N], box {nb*8, G}
  CUtensorMap tz;  // fp16 zeros [G][N], box {nb*8, G} (zeros_packed == 0)
  CUtensorMap tb;  // LoRA B fp16 [r][N], box {nb*8, r}
  const __half* x;
  const uint32_t* qz;  // packed GPTQ qzeros [G][N/8] (zeros_packed == 1)
  const __half* A;
  __half* y;
  int M, K, N, rank, zeros_packed, zero_offset;
  float lora_scale;
  int U, P, C, nb, rows_box, nchunk, ni, pdl;
  Layout lay;
};

__host__ __device__ inline unsigned take(unsigned& o, size_t bytes) {
  const unsigned r = o;
  o += unsigned((bytes + 127) & ~size_t(127));
  return r;
}

__host__ __device__ inline Layout layout(int M, int K, int group, int rank, int C, int nb,
                                         int zeros_packed) {
  const int PR = K / 8, G = K / group;
  Layout L;
  unsigned o = 0;
  L.bars = take(o, size_t(MAX_CHUNKS + 2) * 8);
  L.w = take(o, size_t(PR) * nb * 32);                      // [PR][nb*8] int32
  L.sc = take(o, size_t(G) * nb * 16);                      // [G][nb*8] fp16
  L.zq = take(o, zeros_packed ? size_t(G) * nb * 4 : size_t(G) * nb * 16);  // [G][nb] u32 | [G][nb*8] fp16
  L.bl = take(o, size_t(rank) * nb * 16);                   // [r][nb*8] fp16
  L.xd = take(o, size_t(K / KSTEP) * M * 64);               // [t][M][4] uint4 activation digits
  L.xh = take(o, size_t(M) * K * 2);                        // [M][K] fp16 activations (LoRA)
  L.xsum = take(o, size_t(G) * M * 8);                      // [G][M] (sum X, 2^(E-14))
  L.hr = take(o, size_t(C) * M * rank * 4);                 // h parts from the cluster [C][M][r]
  L.hw = take(o, size_t(WARPS) * M * rank * 4);             // per-warp h partials [WARPS][M][r]
  L.hs = take(o, size_t(M) * rank * 4);                     // scaled h [M][r]
  L.red = take(o, size_t(WARPS) * nb * 8 * M * 4);          // per-warp column partials [WARPS][nb*8][M]
  L.total = o;
  return L;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred P; mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 P, [%1], %2, %3; "
      "selp.u32 %0, 1, 0, P; }"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(1000000u)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Waits at most kWaitLimitNs (2 s); on timeout sets QX_DEVERR_MBAR_TIMEOUT and returns false.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (!mbar_try(bar, parity)) {
    if (global_ns() - t0 > kWaitLimitNs) {
      atomicOr(&g_res_error, QX_DEVERR_MBAR_TIMEOUT);
      return false;
    }
  }
  return true;
}
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
// 2-D tensor copy global -> this CTA's shared memory (x * element size is a
// multiple of 16 B at every call site: x = 8 * unit)
__device__ __forceinline__ void tma_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                       uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void tma_2d_hint(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            uint32_t bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar), "l"(pol)
      : "memory");
}
__device__ __forceinline__ uint32_t map_rank(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
// one float into a cluster peer's shared memory; completion counted in bytes
// on the peer's mbarrier
__device__ __forceinline__ void st_async_f32(uint32_t raddr, float v, uint32_t rbar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(raddr),
      "r"(__float_as_uint(v)), "r"(rbar)
      : "memory");
}
__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
// D(16x8, s32) (+)= A(16x32, u8, row) * B(32x8, s8 / u8, col)
__device__ __forceinline__ void imma_us(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                        uint32_t a3, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void imma_uu(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                        uint32_t a3, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// The 2*KPG integer MMAs of one quantisation group of one 16-column tile:
// rows g / g+8 of the A operand are the tile's two units (HB == false: unit b
// absent, its rows are discarded), B = the activation digits of batch row g
// (zero for g >= M).  Chains: digit (H, L) x k-step parity.
template <int KPG, bool HB>
__device__ __forceinline__ void group_issue(int (&ch)[2][4], int (&cl)[2][4], const uint32_t* wa,
                                            const uint32_t* wb, const uint4* xd, int t0, int M,
                                            int g, int c, int pitch4, bool xrow) {
#pragma unroll
  for (int j = 0; j < KPG; ++j) {
    const int t = t0 + j;
    const uint4 xb = xrow ? xd[(t * M + g) * 4 + c] : make_uint4(0u, 0u, 0u, 0u);
    const uint32_t w0 = wa[t * pitch4];
    const uint32_t lo_a = w0 & 0x0F0F0F0Fu, hi_a = (w0 >> 4) & 0x0F0F0F0Fu;
    uint32_t lo_b = 0u, hi_b = 0u;
    if (HB) {
      const uint32_t w1 = wb[t * pitch4];
      lo_b = w1 & 0x0F0F0F0Fu;
      hi_b = (w1 >> 4) & 0x0F0F0F0Fu;
    }
    const int q = j & 1;
    if (j < 2) {
#pragma unroll
      for (int i = 0; i < 4; ++i) ch[q][i] = cl[q][i] = 0;
    }
    imma_us(ch[q], lo_a, lo_b, hi_a, hi_b, xb.x, xb.y);
    imma_uu(cl[q], lo_a, lo_b, hi_a, hi_b, xb.z, xb.w);
  }
  if (KPG == 1) {
#pragma unroll
    for (int i = 0; i < 4; ++i) ch[1][i] = cl[1][i] = 0;
  }
}

// Group correction for the lane's two columns (units ua, ub; ub absent when
// !hb) and batch rows 2c, 2c+1: acc += s 2^(E-14) (C - z sum X).
__device__ __forceinline__ void group_correct(float (&acc)[4], const int (&ch)[2][4],
                                              const int (&cl)[2][4], int gi, int ua, int ub, bool hb,
                                              int g, int c, int M, int PITCH, int NB,
                                              const __half* sch, const uint32_t* zqw,
                                              const __half* zqh, const int2* xsum, int zeros_packed,
                                              int zero_offset) {
  int cv[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) cv[i] = 256 * (ch[0][i] + ch[1][i]) + (cl[0][i] + cl[1][i]);
  const float s0 = __half2float(sch[gi * PITCH + ua * 8 + g]);
  const float s1 = hb ? __half2float(sch[gi * PITCH + ub * 8 + g]) : 0.f;
  const int2 xr0 = 2 * c < M ? xsum[gi * M + 2 * c] : make_int2(0, 0);
  const int2 xr1 = 2 * c + 1 < M ? xsum[gi * M + 2 * c + 1] : make_int2(0, 0);
  const float e0 = __int_as_float(xr0.y), e1 = __int_as_float(xr1.y);
  if (zeros_packed) {  // integer zero points: C - z sum X exactly in int32
    const int z0 = int((zqw[gi * NB + ua] >> (4 * g)) & 0xFu) + zero_offset;
    const int z1 = hb ? int((zqw[gi * NB + ub] >> (4 * g)) & 0xFu) + zero_offset : 0;
    acc[0] = fmaf(s0 * e0, float(cv[0] - z0 * xr0.x), acc[0]);
    acc[1] = fmaf(s0 * e1, float(cv[1] - z0 * xr1.x), acc[1]);
    acc[2] = fmaf(s1 * e0, float(cv[2] - z1 * xr0.x), acc[2]);
    acc[3] = fmaf(s1 * e1, float(cv[3] - z1 * xr1.x), acc[3]);
  } else {  // fp16 zero points (reference kernel format, may be fractional)
    const float z0 = __half2float(zqh[gi * PITCH + ua * 8 + g]);
    const float z1 = hb ? __half2float(zqh[gi * PITCH + ub * 8 + g]) : 0.f;
    acc[0] = fmaf(s0 * e0, fmaf(-z0, float(xr0.x), float(cv[0])), acc[0]);
    acc[1] = fmaf(s0 * e1, fmaf(-z0, float(xr1.x), float(cv[1])), acc[1]);
    acc[2] = fmaf(s1 * e0, fmaf(-z1, float(xr0.x), float(cv[2])), acc[2]);
    acc[3] = fmaf(s1 * e1, fmaf(-z1, float(xr1.x), float(cv[3])), acc[3]);
  }
}

// KPG = k-steps per quantisation group (group_size / 32); MR = the largest
// batch row count of the instance (1, or MAX_M).
template <int KPG, int MR>
__global__ void __launch_bounds__(THREADS, 2) w4a16_gemv_res_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(128) unsigned char smem[];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int M = MR == 1 ? 1 : p.M, K = p.K, N = p.N, R = p.rank;
  const int PR = K / 8;              // packed rows
  const int Gt = K / (KPG * KSTEP);  // quantisation groups
  const int NB = p.nb, PITCH = NB * 8;  // words per staged packed row
  const int cta = blockIdx.x;
  const int u0 = int((long long)cta * p.U / p.P);
  const int nu = int((long long)(cta + 1) * p.U / p.P) - u0;
  const int col0 = u0 * 8;
  const int C = p.C;
  uint32_t crank = 0;
  if (C > 1) asm("mov.u32 %0, %%cluster_ctarank;" : "=r"(crank));

  const Layout& L = p.lay;
  const uint32_t bar_w0 = smem_u32(smem + L.bars);  // weight chunk i: bar_w0 + 8 i
  const uint32_t bar_st = bar_w0 + 8 * MAX_CHUNKS;  // scales, fp16 zeros, LoRA B
  const uint32_t bar_h = bar_st + 8;                // h parts from the cluster
  const uint32_t* wsm = reinterpret_cast<const uint32_t*>(smem + L.w);
  uint4* xd = reinterpret_cast<uint4*>(smem + L.xd);
  __half* xh = reinterpret_cast<__half*>(smem + L.xh);
  int2* xsum = reinterpret_cast<int2*>(smem + L.xsum);
  float* red = reinterpret_cast<float*>(smem + L.red);

  // the next kernel in the stream may launch as soon as every CTA of this one
  // is resident: before its own wait it only reads its weights
  asm volatile("griddepcontrol.launch_dependents;");

  if (tid == WARPS * 32) {
    for (int i = 0; i < p.nchunk; ++i) mbar_init(bar_w0 + 8 * i, 1);
    mbar_init(bar_st, 1);
    mbar_init(bar_h, 1);
    asm volatile("fence.mbarrier_init.release.cluster;\nfence.proxy.async.shared::cta;" ::: "memory");
  }
  __syncthreads();
  // peers send h parts only after every CTA of the cluster has initialised
  // its receive barrier (arrive now, wait before sending)
  if (C > 1) asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");

  // LoRA A rows of this CTA's part of K, into registers before the wait
  // (static operand): thread t takes rank block jc = t % (R/8) of rows
  // t / (R/8) + i * (256 / (R/8))
  const int RJ = R >> 3;
  const int krows = K / C, ka = int(crank) * krows;
  uint4 areg[NI_MAX];
  int rstep = 1, rfirst = 0;
  if (R > 0 && warp < WARPS) {
    const int jc = tid % RJ;
    rstep = (WARPS * 32) / RJ;
    rfirst = tid / RJ;
#pragma unroll
    for (int i = 0; i < NI_MAX; ++i) {
      const int r = rfirst + i * rstep;
      areg[i] = (i < p.ni && r < krows) ? ldg_nc_v4(p.A + size_t(ka + r) * R + 8 * jc)
                                        : make_uint4(0u, 0u, 0u, 0u);
    }
    // consume the loads before the wait (a shared-memory store of their XOR):
    // otherwise the compiler may sink them to their use after the wait
    uint32_t fold = 0u;
#pragma unroll
    for (int i = 0; i < NI_MAX; ++i) fold ^= areg[i].x ^ areg[i].y ^ areg[i].z ^ areg[i].w;
    asm volatile("st.shared.u32 [%0], %1;" ::"r"(smem_u32(smem + L.hs)), "r"(fold) : "memory");
  }

  if (warp == WARPS) {
    // ---------------- producer warp ----------------
    if (lane == 0) {
      prefetch_tmap(&p.tw);
      const uint64_t pol = evict_first_policy();
      const uint32_t wdst = smem_u32(smem + L.w);
      for (int ch = 0; ch < p.nchunk; ++ch) {
        mbar_expect_tx(bar_w0 + 8 * ch, uint32_t(p.rows_box) * PITCH * 4);
        tma_2d_hint(wdst + uint32_t(ch * p.rows_box * PITCH * 4), &p.tw, col0, ch * p.rows_box,
                    bar_w0 + 8 * ch, pol);
      }
      uint32_t st_bytes = uint32_t(Gt) * NB * 16;
      if (!p.zeros_packed) st_bytes += uint32_t(Gt) * NB * 16;
      if (R > 0) st_bytes += uint32_t(R) * NB * 16;
      mbar_expect_tx(bar_st, st_bytes);
      tma_2d(smem_u32(smem + L.sc), &p.ts, col0, 0, bar_st);
      if (!p.zeros_packed) tma_2d(smem_u32(smem + L.zq), &p.tz, col0, 0, bar_st);
      if (R > 0) tma_2d(smem_u32(smem + L.bl), &p.tb, col0, 0, bar_st);
      if (R > 0 && C > 1) mbar_expect_tx(bar_h, uint32_t(C * M * R) * 4u);
    }
    if (p.zeros_packed) {  // GPTQ qzeros words of the CTA's units (plain loads; read after __syncthreads)
      uint32_t* zq = reinterpret_cast<uint32_t*>(smem + L.zq);
      const int zw = N >> 3;
      for (int it = lane; it < Gt * nu; it += 32) {
        const int gi = it / nu, u = it - gi * nu;
        zq[gi * NB + u] = __ldg(p.qz + size_t(gi) * zw + u0 + u);
      }
    }
  } else {
    // column partials start at zero: warps add only the tiles they cover
    for (int i = tid; i < WARPS * PITCH * M; i += WARPS * 32) red[i] = 0.f;
    // the cluster barrier completes while the previous kernel finishes
    if (C > 1) asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
  }

  // ---- the activations come from the previous kernel in the stream ----
  if (p.pdl) asm volatile("griddepcontrol.wait;" ::: "memory");

  // activations: natural fp16 copy (LoRA) and, per packed row, the fixed-point
  // digits in MMA-B order (H of the even rows, H of the odd rows, L even, L
  // odd; 4 bytes each); per (group, row) sum X and 2^(E-14).  A group of a row
  // is an aligned block of 4*KPG consecutive items, inside one warp.
  for (int base = warp * 32; base < M * PR; base += THREADS) {
    const int it = base + lane;
    const bool ok = it < M * PR;
    const int m = ok ? it / PR : 0, pr = it - m * PR;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (ok) {
      v = *reinterpret_cast<const uint4*>(p.x + size_t(m) * K + size_t(pr) * 8);
      *reinterpret_cast<uint4*>(xh + size_t(m) * K + size_t(pr) * 8) = v;
    }
    const float2 f0 = h2_to_f2(v.x), f1 = h2_to_f2(v.y), f2 = h2_to_f2(v.z), f3 = h2_to_f2(v.w);
    const float xv[8] = {f0.x, f0.y, f1.x, f1.y, f2.x, f2.y, f3.x, f3.y};
    float mx = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) mx = fmaxf(mx, fabsf(xv[i]));
#pragma unroll
    for (int w = 1; w < 4 * KPG; w <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, w));
    // 2^E >= mx with mx = f 2^E, f in [0.5, 1): scale x by 2^(14-E) (exact)
    const int E = mx > 0.f ? int((__float_as_uint(mx) >> 23) & 0xFFu) - 126 : 0;
    const float up = __int_as_float((127 + 14 - E) << 23);
    int X[8], sx = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      X[i] = __float2int_rn(xv[i] * up);
      sx += X[i];
    }
#pragma unroll
    for (int w = 1; w < 4 * KPG; w <<= 1) sx += __shfl_xor_sync(0xffffffffu, sx, w);
    if (ok) {
      uint32_t he = 0u, ho = 0u, le = 0u, lo = 0u;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        he |= (uint32_t(X[2 * e] >> 8) & 0xFFu) << (8 * e);
        ho |= (uint32_t(X[2 * e + 1] >> 8) & 0xFFu) << (8 * e);
        le |= (uint32_t(X[2 * e]) & 0xFFu) << (8 * e);
        lo |= (uint32_t(X[2 * e + 1]) & 0xFFu) << (8 * e);
      }
      xd[((pr >> 2) * M + m) * 4 + (pr & 3)] = make_uint4(he, ho, le, lo);
      if ((pr & (4 * KPG - 1)) == 0)
        xsum[(pr / (4 * KPG)) * M + m] = make_int2(sx, __float_as_int(__int_as_float((127 - 14 + E) << 23)));
    }
  }
  __syncthreads();  // activations, group sums, packed zero points, zeroed partials
  if (warp == WARPS) return;

  // ---------------- compute warps ----------------
  float* hr = reinterpret_cast<float*>(smem + L.hr);
  if (R > 0) {
    // LoRA down-projection over this CTA's K / C rows, fp32
    float hacc[MR][8];
#pragma unroll
    for (int m = 0; m < MR; ++m)
#pragma unroll
      for (int e = 0; e < 8; ++e) hacc[m][e] = 0.f;
#pragma unroll
    for (int i = 0; i < NI_MAX; ++i) {
      const int r = rfirst + i * rstep;
      if (i < p.ni && r < krows) {
        const int k = ka + r;
        const float2 a0 = h2_to_f2(areg[i].x), a1 = h2_to_f2(areg[i].y);
        const float2 a2 = h2_to_f2(areg[i].z), a3 = h2_to_f2(areg[i].w);
        const float av[8] = {a0.x, a0.y, a1.x, a1.y, a2.x, a2.y, a3.x, a3.y};
#pragma unroll
        for (int m = 0; m < MR; ++m) {
          if (m < M) {
            const float xv = __half2float(xh[size_t(m) * K + k]);
#pragma unroll
            for (int e = 0; e < 8; ++e) hacc[m][e] = fmaf(xv, av[e], hacc[m][e]);
          }
        }
      }
    }
    // lanes holding the same rank block: lane % RJ (RJ divides 32)
    for (int off = RJ; off < 32; off <<= 1)
#pragma unroll
      for (int m = 0; m < MR; ++m)
        if (m < M)
#pragma unroll
          for (int e = 0; e < 8; ++e) hacc[m][e] += __shfl_xor_sync(0xffffffffu, hacc[m][e], off);
    float* hw = reinterpret_cast<float*>(smem + L.hw);
    if (lane < RJ) {
#pragma unroll
      for (int m = 0; m < MR; ++m)
        if (m < M)
#pragma unroll
          for (int e = 0; e < 8; ++e) hw[(warp * M + m) * R + 8 * lane + e] = hacc[m][e];
    }
    asm volatile("bar.sync 1, %0;" ::"n"(WARPS * 32) : "memory");
    // this CTA's part of h (warps in order), sent to every CTA of the cluster
    for (int o = tid; o < M * R; o += WARPS * 32) {
      float hp = 0.f;
      for (int w = 0; w < WARPS; ++w) hp += hw[w * M * R + o];
      if (C > 1) {
        const uint32_t la = smem_u32(hr + crank * M * R + o);
        for (int q = 0; q < C; ++q) st_async_f32(map_rank(la, q), hp, map_rank(bar_h, q));
      } else {
        hr[o] = hp;
      }
    }
  }

  // ---- main loop: (tile, group) items [it0, it1) of this warp, tile-major;
  // two groups in flight: the MMAs of group i+1 issue before group i's
  // correction waits for its results ----
  const int ntl = (nu + 1) >> 1;
  const int I = ntl * Gt;
  const int it0 = (warp * I) / WARPS, it1 = ((warp + 1) * I) / WARPS;
  const __half* sch = reinterpret_cast<const __half*>(smem + L.sc);
  const uint32_t* zqw = reinterpret_cast<const uint32_t*>(smem + L.zq);
  const __half* zqh = reinterpret_cast<const __half*>(smem + L.zq);
  const bool xrow = g < M;
  const int gpc = p.rows_box / (4 * KPG);  // quantisation groups per weight chunk
  const int pitch4 = 4 * PITCH;            // words per k-step
  const int zp = p.zeros_packed, zo = p.zero_offset;
  int waited = -1;                         // weight chunks [0, waited] have landed
  mbar_wait(bar_st, 0);                    // scales, zero points, LoRA B
  for (int tl = it0 / Gt; tl * Gt < it1; ++tl) {
    const int gl = max(it0 - tl * Gt, 0), gh = min(it1 - tl * Gt, Gt);
    if (gl >= gh) continue;
    for (; waited < (gh - 1) / gpc; ++waited) mbar_wait(bar_w0 + 8 * (waited + 1), 0);
    const int ua = 2 * tl, ub = 2 * tl + 1;
    const bool hb = ub < nu;
    const uint32_t* wa = wsm + c * PITCH + ua * 8 + g;
    const uint32_t* wb = wa + 8;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    int ha[2][4], la[2][4], hb2[2][4], lb2[2][4];
    if (hb) {
      group_issue<KPG, true>(ha, la, wa, wb, xd, gl * KPG, M, g, c, pitch4, xrow);
      for (int gi = gl; gi < gh; gi += 2) {
        if (gi + 1 < gh) group_issue<KPG, true>(hb2, lb2, wa, wb, xd, (gi + 1) * KPG, M, g, c, pitch4, xrow);
        group_correct(acc, ha, la, gi, ua, ub, true, g, c, M, PITCH, NB, sch, zqw, zqh, xsum, zp, zo);
        if (gi + 1 >= gh) break;
        if (gi + 2 < gh) group_issue<KPG, true>(ha, la, wa, wb, xd, (gi + 2) * KPG, M, g, c, pitch4, xrow);
        group_correct(acc, hb2, lb2, gi + 1, ua, ub, true, g, c, M, PITCH, NB, sch, zqw, zqh, xsum, zp, zo);
      }
    } else {
      group_issue<KPG, false>(ha, la, wa, wb, xd, gl * KPG, M, g, c, pitch4, xrow);
      for (int gi = gl; gi < gh; gi += 2) {
        if (gi + 1 < gh) group_issue<KPG, false>(hb2, lb2, wa, wb, xd, (gi + 1) * KPG, M, g, c, pitch4, xrow);
        group_correct(acc, ha, la, gi, ua, ub, false, g, c, M, PITCH, NB, sch, zqw, zqh, xsum, zp, zo);
        if (gi + 1 >= gh) break;
        if (gi + 2 < gh) group_issue<KPG, false>(ha, la, wa, wb, xd, (gi + 2) * KPG, M, g, c, pitch4, xrow);
        group_correct(acc, hb2, lb2, gi + 1, ua, ub, false, g, c, M, PITCH, NB, sch, zqw, zqh, xsum, zp, zo);
      }
    }
    // this warp's partial of the tile: red[warp][col][m]
    float* rw = red + size_t(warp) * PITCH * M;
    const bool row0 = 2 * c < M, row1 = 2 * c + 1 < M;
    if (row0) rw[(ua * 8 + g) * M + 2 * c] = acc[0];
    if (row1) rw[(ua * 8 + g) * M + 2 * c + 1] = acc[1];
    if (hb) {
      if (row0) rw[(ub * 8 + g) * M + 2 * c] = acc[2];
      if (row1) rw[(ub * 8 + g) * M + 2 * c + 1] = acc[3];
    }
  }

  // h = the cluster's parts summed in rank order, times the LoRA scale
  float* hs = reinterpret_cast<float*>(smem + L.hs);
  if (R > 0 && warp == 0) {
    if (C > 1) mbar_wait(bar_h, 0);
    for (int o = lane; o < M * R; o += 32) {
      float h = 0.f;
      for (int q = 0; q < C; ++q) h += hr[q * M * R + o];
      hs[o] = p.lora_scale * h;
    }
  }
  asm volatile("bar.sync 1, %0;" ::"n"(WARPS * 32) : "memory");  // partials and h

  const __half* blh = reinterpret_cast<const __half*>(smem + L.bl);
  for (int o = tid; o < nu * 8 * M; o += WARPS * 32) {
    const int col = o / M, m = o - col * M;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) v += red[(w * PITCH + col) * M + m];  // warps in order
    if (R > 0) {
      float l0 = 0.f, l1 = 0.f;
      const float* hm = hs + m * R;
      for (int j = 0; j < R; j += 8) {
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
          l0 = fmaf(hm[j + e], __half2float(blh[(j + e) * PITCH + col]), l0);
          l1 = fmaf(hm[j + e + 1], __half2float(blh[(j + e + 1) * PITCH + col]), l1);
        }
      }
      v += l0 + l1;
    }
    p.y[size_t(m) * N + col0 + col] = __float2half_rn(v);
  }
}

struct Plan {
  int P, C, nb, rows_box, nchunk, ni;
  size_t smem;
  bool ok;
};

template <int KPG>
static int prepare(int dev) {
  static std::mutex mu;
  static bool done[64] = {};
  std::lock_guard<std::mutex> lk(mu);
  if (dev >= 0 && dev < 64 && done[dev]) return QX_OK;
  QX_CUDA_TRY(cudaFuncSetAttribute(w4a16_gemv_res_kernel<KPG, 1>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, int(SMEM_BUDGET)),
              "w4a16_gemv_res: set smem limit");
  QX_CUDA_TRY(cudaFuncSetAttribute(w4a16_gemv_res_kernel<KPG, MAX_M>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, int(SMEM_BUDGET)),
              "w4a16_gemv_res: set smem limit");
  if (dev >= 0 && dev < 64) done[dev] = true;
  return QX_OK;
}

// P = one CTA per SM (at most one unit each); C = the smallest cluster
// (1, 2, 4, 8, dividing P) whose LoRA A share fits the per-thread registers;
// the shared-memory layout must leave room for a second CTA on the SM.
template <int KPG>
static Plan make_plan(int M, int K, int N, int rank, int group, int zeros_packed) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, int, int, int, int>, Plan> cache;
  Plan pl{};
  pl.ok = false;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return pl;
  }
  const auto key = std::make_tuple(dev, M, K, N, rank, group, zeros_packed);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  auto remember = [&](const Plan& v) {
    std::lock_guard<std::mutex> lk(mu);
    cache[key] = v;
    return v;
  };
  if (M < 1 || M > MAX_M || prepare<KPG>(dev) != QX_OK) return remember(pl);
  const int U = N / 8, G = K / group, PR = K / 8;
  if (G > 256 || rank > 256) return remember(pl);
  const int sms = device_sm_count();
  int P = std::min(sms, U);
  int C = 1;
  int ni = 0;
  if (rank > 0) {
    const int RJ = rank / 8;
    if ((WARPS * 32) % RJ != 0) return remember(pl);
    bool found = false;
    for (int cc : {1, 2, 4, 8}) {
      const int Pc = P - P % cc;
      if (Pc < cc || K % (8 * cc) != 0) continue;
      const int krows = K / cc;
      const int need = (krows * RJ + WARPS * 32 - 1) / (WARPS * 32);
      if (need <= NI_MAX) {
        C = cc;
        P = Pc;
        ni = need;
        found = true;
        break;
      }
    }
    if (!found) return remember(pl);
  }
  int nb = (U + P - 1) / P;
  if (!(nb & 1)) ++nb;
  if (nb > MAX_NB) return remember(pl);
  int nchunk = (PR + 255) / 256;
  while (nchunk <= MAX_CHUNKS && (PR % nchunk != 0 || (PR / nchunk) % (4 * KPG) != 0)) ++nchunk;
  if (nchunk > MAX_CHUNKS) return remember(pl);
  const Layout L = layout(M, K, group, rank, C, nb, zeros_packed);
  if (L.total > SMEM_BUDGET) return remember(pl);
  if (C > 1) {  // every cluster must fit at once
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(P, 1, 1);
    cfg.blockDim = dim3(THREADS, 1, 1);
    cfg.dynamicSmemBytes = L.total;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = C;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int clusters = 0;
    const cudaError_t oe =
        M == 1 ? cudaOccupancyMaxActiveClusters(&clusters, w4a16_gemv_res_kernel<KPG, 1>, &cfg)
               : cudaOccupancyMaxActiveClusters(&clusters, w4a16_gemv_res_kernel<KPG, MAX_M>, &cfg);
    if (oe != cudaSuccess) {
      cudaGetLastError();
      return remember(pl);
    }
    if (clusters * C < P) return remember(pl);
  }
  pl.P = P;
  pl.C = C;
  pl.nb = nb;
  pl.rows_box = PR / nchunk;
  pl.nchunk = nchunk;
  pl.ni = ni;
  pl.smem = L.total;
  pl.ok = true;
  return remember(pl);
}

static PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    else
      cudaGetLastError();
  });
  return fn;
}

static int encode_2d(CUtensorMap* map, CUtensorMapDataType type, const void* base, uint64_t cols,
                     uint64_t rows, uint64_t row_stride_bytes, uint32_t box_cols, uint32_t box_rows,
                     const char* what) {
  const auto enc = tmap_encoder();
  if (!enc) return fail(QX_ERR_CUDA, "w4a16_gemv_res: cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {row_stride_bytes};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, type, 2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(QX_ERR_CUDA, "w4a16_gemv_res: tensor map for %s (CUresult %d)", what, int(r));
  return QX_OK;
}

template <int KPG>
static int run(const void* x, const int32_t* qweight, const void* scales, const void* zeros,
               int zeros_packed, int zero_offset, const void* lora_A, const void* lora_B, void* y,
               int M, int K, int N, int rank, int group, float lora_scale, cudaStream_t st) {
  const Plan pl = make_plan<KPG>(M, K, N, rank, group, zeros_packed);
  if (!pl.ok) return QX_ERR_UNSUPPORTED;
  Params prm{};
  prm.x = static_cast<const __half*>(x);
  prm.qz = static_cast<const uint32_t*>(zeros);
  prm.A = static_cast<const __half*>(lora_A);
  prm.y = static_cast<__half*>(y);
  prm.M = M;
  prm.K = K;
  prm.N = N;
  prm.rank = rank;
  prm.zeros_packed = zeros_packed;
  prm.zero_offset = zero_offset;
  prm.lora_scale = rank > 0 ? lora_scale : 0.f;
  prm.U = N / 8;
  prm.P = pl.P;
  prm.C = pl.C;
  prm.nb = pl.nb;
  prm.rows_box = pl.rows_box;
  prm.nchunk = pl.nchunk;
  prm.ni = pl.ni;
  prm.pdl = g_pdl_enabled.load(std::memory_order_relaxed);
  prm.lay = layout(M, K, group, rank, pl.C, pl.nb, zeros_packed);
  const uint32_t bw = uint32_t(pl.nb) * 8;
  const uint64_t G = uint64_t(K / group);
  int rc = encode_2d(&prm.tw, CU_TENSOR_MAP_DATA_TYPE_INT32, qweight, uint64_t(N), uint64_t(K) / 8,
                     uint64_t(N) * 4, bw, uint32_t(pl.rows_box), "qweight");
  if (rc != QX_OK) return rc;
  rc = encode_2d(&prm.ts, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, scales, uint64_t(N), G, uint64_t(N) * 2, bw,
                 uint32_t(G), "scales");
  if (rc != QX_OK) return rc;
  if (!zeros_packed) {
    rc = encode_2d(&prm.tz, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, zeros, uint64_t(N), G, uint64_t(N) * 2,
                   bw, uint32_t(G), "zeros");
    if (rc != QX_OK) return rc;
  }
  if (rank > 0) {
    rc = encode_2d(&prm.tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, lora_B, uint64_t(N), uint64_t(rank),
                   uint64_t(N) * 2, bw, uint32_t(rank), "lora_B");
    if (rc != QX_OK) return rc;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.P, 1, 1);
  cfg.blockDim = dim3(THREADS, 1, 1);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = st;
  cudaLaunchAttribute attrs[2];
  int na = 0;
  if (pl.C > 1) {
    attrs[na].id = cudaLaunchAttributeClusterDimension;
    attrs[na].val.clusterDim.x = pl.C;
    attrs[na].val.clusterDim.y = 1;
    attrs[na].val.clusterDim.z = 1;
    ++na;
  }
  if (prm.pdl) {
    attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = na;
  if (M == 1)
    QX_CUDA_TRY(cudaLaunchKernelEx(&cfg, w4a16_gemv_res_kernel<KPG, 1>, prm), "w4a16_gemv_res: launch");
  else
    QX_CUDA_TRY(cudaLaunchKernelEx(&cfg, w4a16_gemv_res_kernel<KPG, MAX_M>, prm), "w4a16_gemv_res: launch");
  return check_launch("w4a16_gemv_res");
}

}  // namespace gres

// off by default until it beats the clustered split-K kernel at the decode shape
std::atomic<int> g_gemv_resident{0};

// QX_ERR_UNSUPPORTED (nothing launched) when the shape does not suit the
// resident kernel; the caller then runs the clustered split-K GEMV.
int gemv_resident(const void* x, const int32_t* qweight, const void* scales, const void* zeros,
                  int zeros_packed, int zero_offset, const void* lora_A, const void* lora_B, void* y,
                  int M, int K, int N, int rank, int group, float lora_scale, cudaStream_t st) {
  if (!g_gemv_resident.load(std::memory_order_relaxed)) return QX_ERR_UNSUPPORTED;
  if (M > gres::MAX_M || N % 8 != 0 || rank % 8 != 0) return QX_ERR_UNSUPPORTED;
  if (!aligned(zeros, zeros_packed ? 4 : 16)) return QX_ERR_UNSUPPORTED;
  switch (group) {
    case 32: return gres::run<1>(x, qweight, scales, zeros, zeros_packed, zero_offset, lora_A, lora_B, y, M, K, N, rank, group, lora_scale, st);
    case 64: return gres::run<2>(x, qweight, scales, zeros, zeros_packed, zero_offset, lora_A, lora_B, y, M, K, N, rank, group, lora_scale, st);
    case 128: return gres::run<4>(x, qweight, scales, zeros, zeros_packed, zero_offset, lora_A, lora_B, y, M, K, N, rank, group, lora_scale, st);
    case 256: return gres::run<8>(x, qweight, scales, zeros, zeros_packed, zero_offset, lora_A, lora_B, y, M, K, N, rank, group, lora_scale, st);
    default: return QX_ERR_UNSUPPORTED;
  }
}

int gemv_res_device_error(unsigned* code, int reset) {
  QX_CUDA_TRY(cudaMemcpyFromSymbol(code, gres::g_res_error, sizeof(unsigned)),
              "get_device_error: read (resident GEMV)");
  if (reset) {
    const unsigned zero = 0;
    QX_CUDA_TRY(cudaMemcpyToSymbol(gres::g_res_error, &zero, sizeof(unsigned)),
                "get_device_error: reset (resident GEMV)");
  }
  return QX_OK;
}

}  // namespace qx

// Which GEMV kernel a call of this shape runs: 1 = resident, 0 = clustered
// split-K (also for shapes the resident kernel does not take).
extern "C" int qx_w4a16_gemv_route(int M, int K, int N, int rank, int group_size, int zeros_packed,
                                   int* kernel) {
  QX_REQUIRE(kernel, "w4a16_gemv_route: null output");
  *kernel = 0;
  if (!qx::g_gemv_resident.load() || M < 1 || M > qx::gres::MAX_M || N % 8 != 0 || rank % 8 != 0 ||
      K % 32 != 0)
    return QX_OK;
  qx::gres::Plan pl{};
  switch (group_size) {
    case 32: pl = qx::gres::make_plan<1>(M, K, N, rank, group_size, zeros_packed); break;
    case 64: pl = qx::gres::make_plan<2>(M, K, N, rank, group_size, zeros_packed); break;
    case 128: pl = qx::gres::make_plan<4>(M, K, N, rank, group_size, zeros_packed); break;
    case 256: pl = qx::gres::make_plan<8>(M, K, N, rank, group_size, zeros_packed); break;
    default: return QX_OK;
  }
  *kernel = pl.ok ? 1 : 0;
  return QX_OK;
}

extern "C" int qx_set_gemv_resident(int enable) {
  qx::g_gemv_resident.store(enable ? 1 : 0);
  return QX_OK;
}
