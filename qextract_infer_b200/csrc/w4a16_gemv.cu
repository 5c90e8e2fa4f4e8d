// W4A16 (GPTQ int4, group-wise scale/zero) + LoRA decode GEMV for sm_100a.
//
// Replaces the reference's two-launch path (lora_down_gemv_kernel +
// w4a16_lora_fused_gemv_kernel, csrc/kernels/w4a16_lora_gemv.cu:112-226):
// one launch streams every weight byte once from HBM and the LoRA terms ride
// along.  Math reproduced: y = fp16(x.W + (alpha/r)(x.A).B) with
// W = s (q - z) and fp32 accumulation (w4a16_lora_gemv.cu:183-224).
//
// Work decomposition
//   tile    = 256 output columns (8 compute warps x 32 columns).
//   cluster = the S CTAs (S <= 16, any size) that split one tile's K range
//             into whole quantisation groups as evenly as possible: grid
//             (tiles, S), cluster dims (1, S, 1); the host picks S so that the
//             grid runs in one wave with the fewest groups per CTA.
//   warps   = 8 compute warps and one helper warp.  The helper initialises
//             the barriers, starts every copy, stages the zero points, and
//             computes the LoRA down-projection while the compute warps
//             stream the weights.
//   weights = one 2-D TMA copy per quantisation group (KPG*4 packed rows x
//             1056 B: the qweight viewed as 64-bit elements, so the 1 KB tile
//             row plus 32 B of the next tile land as one box row); every
//             group of the CTA is in flight at once when shared memory allows
//             (else a ring with full/empty mbarriers refilled by thread 0).
//             The 1056 B row pitch lets lane (g = lane/4, c = lane%4) read
//             packed row 4*ks + c, columns 4g..4g+3 of its warp, with
//             conflict-free 128-bit loads.
//   dot     = one LOP3 per nibble pair builds exact fp16 operands with the
//             magic-number trick (Kim et al., "Who Says Elephants Can't Run",
//             2022): (v & 0x000F000F) | 0x64006400 is the half2
//             (1024 + q_i, 1024 + q_{i+4}) and (v & 0x00F000F0) | 0x54005400
//             is (64 + q_{i+1}, 64 + q_{i+5}) (the nibble lands four bits up
//             in the mantissa of 64).  They feed mma.sync m16n8k16 with fp32
//             accumulation, the activations of each packed row permuted to
//             (x0, x4 | x1, x5 | x2, x6 | x3, x7) in registers.  The offsets
//             leave with the zero point once per group:
//               sum (q - z) x = C - Off - z Sx,  Off = 1024 Xa + 64 Xb,
//               Sx = Xa + Xb,  Xa / Xb = sums of x over the two nibble classes,
//             and Off / Sx come from a second MMA of the same activation
//             fragments against a constant matrix (rows 1024|64 and 1|1).
//   LoRA    = h_s = x[:, Ks] A[Ks, :] on the tensor cores (ldmatrix.trans
//             of A): each ring stage carries its group's LoRA A rows beside
//             the weights (one bulk copy), so h_s accumulates group by group
//             and no CTA holds an A slice the size of its K range (which at
//             ranks 32-48 and deep K cost whole CTAs of occupancy); by the
//             helper warp for up to 8 rows and ranks below 32, else by the
//             compute warps (16 x 8 tiles spread over the warps).  The LoRA
//             product is linear in K, so each CTA adds (alpha/r) h_s B[:, tile]
//             into its own partial sums and no h is exchanged: at one row the
//             helper warp forms that term in fp32 as soon as h_s is complete,
//             while the compute warps still stream; otherwise the compute
//             warps add it with a hi/lo fp16 MMA pair after their loop.
//   reduce  = each CTA sends its fp32 partial of the columns owned by CTA j
//             straight into CTA j's shared memory with st.async, which
//             completes on CTA j's receive mbarrier; CTA j waits for its
//             expected bytes, sums the S slices in rank order (deterministic)
//             and rounds once.  No global scratch, no atomics.
// Programmatic dependent launch (on by default, qx_set_pdl(0) turns it off):
// the kernel lets the next kernel in the stream launch at once, and waits for
// the previous one only before it reads the activations.  Weights, scales,
// zero points and LoRA factors are therefore read before that wait: they must
// not be written by the kernel issued just before on the same stream.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstring>
#include <map>
#include <unordered_map>
#include <mutex>
#include <tuple>
#include <type_traits>

#include "qx_b200.h"
#include "qx_common.cuh"

namespace qx {

std::atomic<int> g_pdl_enabled{1};
// split-K plan pinned by qx_w4a16_gemv_pin_plan (0: chosen per shape)
std::atomic<int> g_pin_S{0}, g_pin_nst{0};

// Sticky device-side error word (QX_DEVERR_* bits), read by qx_get_device_error.
static __device__ unsigned g_device_error = 0;

namespace gemv {

constexpr int WARPS = 8;                 // compute warps
constexpr int THREADS = (WARPS + 1) * 32;  // + the helper warp
constexpr int COLS = WARPS * 32;         // output columns per tile
constexpr int KSTEP = 32;                // K rows per step (4 packed rows)
constexpr int ROWB = 1056;               // smem bytes per staged packed row (1 KB + 32 B: no bank conflicts)
constexpr int MAX_NST = 4;               // weight stages (quantisation groups) in flight per CTA
constexpr int MROWS = 32;                // batch rows per launch (4 n-tiles of 8)
constexpr int MAX_S = 16;                // largest cluster (non-portable size)
constexpr size_t SMEM_LIMIT = 226 * 1024;  // dynamic; 1 KB left for the static arrays

__host__ __device__ constexpr int ctas_per_sm(int nt) { return nt == 1 ? 3 : (nt == 2 ? 2 : 1); }

// Shared-memory carve-up (byte offsets), identical on host and device.
struct Layout {
  unsigned bars, ring, sz_s, sz_z, sf, xraw, xs, xks, Bs, hs, lu, recv, total;
};

struct alignas(64) Params {
  CUtensorMap tw;  // qweight as u64 [K/8][N/2], box {132, KPG*4}
  CUtensorMap tb;  // LoRA B fp16 [r][N], box {256, r}
  CUtensorMap ts;  // scales fp16 [K/g][N], box {256, gmax}
  CUtensorMap tz;  // fp16 zeros [K/g][N], box {256, gmax}; packed qzeros int32 [K/g][N/8], box {32, gmax}
  const __half* x;
  const uint32_t* qw;
  const __half* scales;
  const void* zeros;
  const __half* A;
  const __half* B;
  __half* y;
  int M, K, N, rank, group, zeros_packed, zero_offset;
  int zeros_tma;  // zero points by TMA (fp16 always; packed when rows are 16 B multiples)
  float lora_scale;
  int T, S, cpr, Ts_max, gmax, nst, pdl;
  int act;                      // 1: SwiGLU epilogue over column blocks (8 gate, 8 up), y [M][N/2]
  int x_early;                  // x is not written by the previous kernel (host rows): read it
                                // before the dependency wait, wait before the output stores
  // residual add + RMSNorm prologue (qx_w4a16_lora_gemv_addnorm, up to 8 rows):
  // x = fp16((r rsqrt(mean(r^2) + eps)) w) with r = fp16(res + delta) over the
  // whole row; the CTAs of tile 0 write r (their K ranges) to res_out
  int addnorm;
  const __half* res;
  const __half* delta;
  const __half* nw;
  __half* res_out;
  float eps;
  int stage;                    // bytes per ring stage: a group's packed weights, then its LoRA A rows
  uint32_t s_magic, cpr_magic;  // ceil(2^32 / S) (S > 1), ceil(2^32 / cpr): exact floor division of small values
  Layout lay;                   // shared-memory carve-up, computed on the host
  unsigned long long* trace;    // profiling build only (qx_trace_launches): phase timestamps
  int trace_launch;
};

// Trace slots of a GEMV CTA (profiling build): 0 entry, 1 dependency wait
// passed, 2 first weight group landed, 3 weight loop done, 4 helper's LoRA
// down-projection done, 5 LoRA up-projection done, 6 partials sent to the
// owners, 7 partials received (owners), 8 exit (owners)
enum GemvTrace { TR_ENTRY, TR_WAITED, TR_GROUP0, TR_LOOP, TR_LORA_DOWN, TR_LORA_UP, TR_SENT, TR_RECEIVED, TR_EXIT };


__host__ __device__ inline unsigned take(unsigned& o, size_t bytes) {
  const unsigned r = o;
  o += unsigned((bytes + 127) & ~size_t(127));
  return r;
}

// row stride of the staged activations (halves): +8 puts consecutive rows
// 4 banks apart, so 8 rows x 4 words of an MMA fragment hit distinct banks
__host__ __device__ inline int xstride(int Ts_max) { return Ts_max * KSTEP + 8; }

// columns each CTA of an S-cluster finalises: 256 / S rounded up to 8 (to 16
// with the SwiGLU epilogue: an owner holds whole gate|up column-block pairs)
__host__ __device__ inline int owner_cols(int S, int act = 0) {
  const int q = act ? 16 : 8;
  return ((COLS + S - 1) / S + q - 1) / q * q;
}

// silu(g) * u with the fast exponential and divide (the formula of
// qx_fused_swiglu)
__device__ __forceinline__ float silu_mul(float g, float u) {
  return __fdividef(g, 1.0f + __expf(-g)) * u;
}
// the fp16 rounding of a column's sum, as the unfused GEMV stores it
__device__ __forceinline__ float round_h(float v) { return __half2float(__float2half_rn(v)); }

// LoRA down-projection, one quantisation group at a time as its ring stage
// lands (the stage holds the group's LoRA A rows beside its weights, so no
// CTA keeps an A slice the size of its K range): on the compute warps for
// batches above 8 rows or ranks of 32 and more, as (16-row block, 8-rank
// block) tiles spread over the warps; else on the helper warp while the
// compute warps stream the weights.
__host__ __device__ inline bool lora_on_warps(int M, int rank) { return rank > 0 && (M > 8 || rank >= 32); }
__host__ __device__ inline int lora_tiles(int M, int rank) { return ((M + 15) / 16) * (rank / 8); }
// one-row launches with the helper's down-projection: the helper also forms the
// up-projection (alpha/r) h_s B[:, tile] in fp32 while the compute warps still
// stream weights (measured at the Qwen3-4B gate_proj shape: 6.29 -> 6.11 us per
// call; at 2-8 rows the compute warps' MMA pair after the loop stays faster)
__host__ __device__ inline bool lora_up_on_helper(int M, int rank) {
  return M == 1 && rank > 0 && !lora_on_warps(M, rank);
}
// tiles per compute warp (registers of the kernel instance: NT batch tiles)
__host__ __device__ constexpr int lora_items(int nt) { return nt == 4 ? 4 : 2; }
// bytes of one ring stage: KPG*4 packed rows of 1056 B, then KPG*32 rows of A
__host__ __device__ inline int stage_bytes(int KPG, int rank) {
  return (KPG * 4 * ROWB + KPG * KSTEP * rank * 2 + 127) & ~127;
}

// M = batch rows of this launch (<= 32).
__host__ __device__ inline Layout layout(int M, int KPG, int Ts_max, int rank, int S, int nst,
                                         int zeros_packed, int act = 0) {
  const int gmax = Ts_max / KPG;
  const size_t Mp = M <= 8 ? 8 : (M <= 16 ? 16 : 32);  // NT * 8 of the kernel instance
  Layout L;
  unsigned o = 0;
  L.bars = take(o, size_t(4 + 2 * nst) * 8);  // statics, B, h, recv, full[nst], empty[nst]
  L.ring = take(o, size_t(nst) * stage_bytes(KPG, rank));  // weight (+ LoRA A) stages
  L.sz_s = take(o, size_t(gmax) * COLS * 2);          // scales [gmax][256]
  L.sz_z = take(o, size_t(gmax) * (zeros_packed ? COLS / 2 : COLS * 2));  // [gmax][32] u32 or [gmax][256] fp16
  L.sf = take(o, size_t(gmax) * COLS * 8);            // (s, s*z) as floats [gmax][256]
  L.xraw = take(o, size_t(M) * xstride(Ts_max) * 2);  // activations [M][Ks(+8)]
  L.xs = take(o, size_t(Ts_max) * M * 4 * 16 + 64);   // in MMA-B order [t][M][c], then a zero block
  L.xks = take(o, size_t(gmax) * Mp * 2 * 4);         // per group (Off, Sx) per row [g][Mp]
  L.Bs = take(o, size_t(rank) * COLS * 2);            // LoRA B tile [r][256]
  L.hs = take(o, size_t(M) * rank * 4);                // h_s [M][r]
  L.lu = take(o, lora_up_on_helper(M, rank) ? COLS * 4 : 0);  // the helper's LoRA term [256]
  L.recv = take(o, size_t(S) * M * owner_cols(S, act) * 4);  // partials from the cluster [S][M][cpr]
  L.total = o;
  return L;
}

struct Plan {
  int tiles, S, T, Ts_max, NT, nst;
  size_t smem;
};

__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;"); }
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  const unsigned a = static_cast<unsigned>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t (&r)[2], const void* p) {
  const unsigned a = static_cast<unsigned>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];"
               : "=r"(r[0]), "=r"(r[1])
               : "r"(a));
}
__device__ __forceinline__ void ldsm_x2(uint32_t (&r)[2], const void* p) {
  const unsigned a = static_cast<unsigned>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
               : "=r"(r[0]), "=r"(r[1])
               : "r"(a));
}
__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
// Weights are read once per call: an L2 evict-first policy keeps the stream
// from pushing activations, scales or code out of L2.
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
               "r"(bytes)
               : "memory");
}
// try_wait suspends the thread for a system-dependent time while the phase is
// incomplete (measured: without a suspend-time hint the GEMV runs 2-3 % faster
// than with a 1 ms hint, e.g. 6.02 vs 6.17 us at the Qwen3-4B gate_proj shape).
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred P; mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 P, [%1], %2; "
      "selp.u32 %0, 1, 0, P; }"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Waits at most kWaitLimitNs (2 s) for the phase; on timeout records QX_DEVERR_MBAR_TIMEOUT
// in the device error word (read with qx_get_device_error) and returns false.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (!mbar_try(bar, parity)) {
    if (global_ns() - t0 > kWaitLimitNs) {
      atomicOr(&g_device_error, QX_DEVERR_MBAR_TIMEOUT);
      return false;
    }
  }
  return true;
}
// 1-D bulk copies global -> this CTA's shared memory, completion counted on `bar`
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}
// 2-D tensor copy global -> this CTA's shared memory; coordinates in elements,
// x innermost (x * element size is a multiple of 16 B at every call site)
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
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
// st.async of two floats into a peer CTA's shared memory; completion counted
// in bytes on the peer's mbarrier (both addresses already mapped with mapa)
__device__ __forceinline__ void st_async_f4(uint32_t raddr, float a, float b, float c, float d,
                                            uint32_t rbar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
          raddr),
      "f"(a), "f"(b), "f"(c), "f"(d), "r"(rbar)
      : "memory");
}
__device__ __forceinline__ uint32_t map_rank(uint32_t addr, int rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

// KPG = k-steps per quantisation group (group_size / 32); LW = the LoRA
// down-projection on the compute warps (lora_on_warps), else on the helper.
template <int NT, int KPG, bool LW>
__global__ void __launch_bounds__(THREADS, ctas_per_sm(NT))
    w4a16_gemv_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ float s_ss[WARPS + 1][8];  // addnorm: per-warp sums of squares of the rows
  __shared__ float s_rs[8];         // addnorm: rsqrt(mean(r^2) + eps) per row

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int tile = blockIdx.x;
  const int s = blockIdx.y;  // == rank in the (1, S, 1) cluster
  const int S = p.S;
  const int Gt = p.T / KPG;  // quantisation groups along K
  // floor(s * Gt / S) and floor((s + 1) * Gt / S) (S == 1: one CTA takes all)
  const int gr0 = S == 1 ? 0 : int(__umulhi(uint32_t(s * Gt), p.s_magic));
  const int gr1 = S == 1 ? Gt : int(__umulhi(uint32_t((s + 1) * Gt), p.s_magic));
  const int ngrp = gr1 - gr0;
  const int ks0 = gr0 * KPG;
  const int Ks = ngrp * KPG * KSTEP;
  const int XS = xstride(p.Ts_max);
  const int M = p.M, N = p.N, R = p.rank;
  constexpr int WBYTES = KPG * 4 * ROWB;  // the weights of a stage (full box, zero-filled past N)
  constexpr int GROUPK = KPG * KSTEP;      // rows of a quantisation group
  constexpr int Mp = NT * 8;
  const int STAGE = p.stage;
  const uint32_t ABYTES = uint32_t(GROUPK * p.rank) * 2u;  // the group's LoRA A rows
  const uint32_t STAGE_TX = uint32_t(WBYTES) + ABYTES;
  const int nst = p.nst;
  const int n_tile0 = tile * COLS;
  const int k0 = ks0 * KSTEP;
  const int CPR = p.cpr;  // columns each CTA of the cluster finalises
  const int own_cols = max(0, min(min(CPR, COLS - s * CPR), N - (n_tile0 + s * CPR)));

  const Layout& L = p.lay;
  __half* xraw = reinterpret_cast<__half*>(smem + L.xraw);
  const float* recv = reinterpret_cast<const float*>(smem + L.recv);
  const uint32_t bar_st = smem_addr(smem + L.bars);  // scales, zeros, LoRA A
  const uint32_t bar_b = bar_st + 8;                 // LoRA B
  const uint32_t bar_h = bar_st + 16;                // h_s computed
  const uint32_t bar_rv = bar_st + 24;               // partials from the cluster
  const uint32_t full0 = bar_st + 32;                // full[i]  = full0 + 8 i
  const uint32_t empty0 = full0 + 8 * nst;           // empty[i] = empty0 + 8 i
  const int wx = n_tile0 / 2;  // tile origin in 64-bit elements (x * 8 B = tile * 1 KB)
  const uint32_t ring_s = smem_addr(smem + L.ring);

  // The next kernel in the stream may launch as soon as every CTA of this one
  // is resident: it only streams its own weights until it waits for us.
  grid_dep_launch();
  unsigned long long* const trc = trace_base(p.trace, p.trace_launch);
  trace_stamp(trc, TR_ENTRY, tid == 0);

  if (warp == WARPS && lane == 0) {
    prefetch_tmap(&p.tw);
    mbar_init(bar_st, p.zeros_tma ? 1 : 33);  // + one arrival per helper lane (plain-loaded zeros)
    mbar_init(bar_b, 1);
    mbar_init(bar_h, 32);
    mbar_init(bar_rv, 1);
    // a stage is free once every compute warp, and the helper when it takes
    // the group's LoRA A rows, has read it
    const int readers = WARPS + ((p.rank > 0 && !lora_on_warps(p.M, p.rank)) ? 1 : 0);
    for (int i = 0; i < nst; ++i) {
      mbar_init(full0 + 8 * i, 1);
      mbar_init(empty0 + 8 * i, readers);
    }
    asm volatile("fence.mbarrier_init.release.cluster;\nfence.proxy.async.shared::cta;" :::
                     "memory");
  }
  __syncthreads();  // barriers initialised
  // Peers send partial sums only after every CTA of the cluster has
  // initialised its receive barrier (arrive now, wait before sending).
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");

  if (warp == WARPS) {
    // ---------------- helper warp ----------------
    if (lane == 0) {
      // bytes the S CTAs of the cluster will send for this CTA's columns
      mbar_expect_tx(bar_rv, uint32_t(S * M * own_cols) * 4u);
      const uint32_t sz_bytes =
          uint32_t(p.gmax) * (COLS * 2 + (p.zeros_tma ? (p.zeros_packed ? COLS / 2 : COLS * 2) : 0));
      mbar_expect_tx(bar_st, sz_bytes);
      // scales / fp16 zero points of this CTA's groups (gmax rows; rows past
      // the CTA's range are read but unused) first: they are converted before
      // the dependency wait; then the LoRA B tile and the weight groups with
      // their LoRA A rows
      tma_2d(smem_addr(smem + L.sz_s), &p.ts, n_tile0, gr0, bar_st);
      if (p.zeros_tma)
        tma_2d(smem_addr(smem + L.sz_z), &p.tz, p.zeros_packed ? n_tile0 / 8 : n_tile0, gr0, bar_st);
      if (R > 0) {
        mbar_expect_tx(bar_b, uint32_t(R * COLS) * 2);
        tma_2d(smem_addr(smem + L.Bs), &p.tb, n_tile0, 0, bar_b);
      }
      const uint64_t pol = evict_first_policy();
      for (int i = 0; i < min(ngrp, nst); ++i) {
        mbar_expect_tx(full0 + 8 * i, STAGE_TX);
        tma_2d_hint(ring_s + i * STAGE, &p.tw, wx, (ks0 + i * KPG) * 4, full0 + 8 * i, pol);
        if (R > 0)
          bulk_g2s(ring_s + i * STAGE + WBYTES, p.A + size_t(k0 + i * GROUPK) * R, ABYTES, full0 + 8 * i);
      }
    }
    // GPTQ qzeros rows of N/2 bytes that are not a 16 B multiple: plain loads
    if (!p.zeros_tma) {
      const int zwords = N >> 3;
      const uint32_t* zsrc = static_cast<const uint32_t*>(p.zeros);
      uint32_t* zdst = reinterpret_cast<uint32_t*>(smem + L.sz_z);
      for (int it = lane; it < p.gmax * (COLS / 8); it += 32) {
        const int row = gr0 + (it >> 5), col = (n_tile0 >> 3) + (it & 31);
        zdst[it] = (row < Gt && col < zwords) ? __ldg(zsrc + size_t(row) * zwords + col) : 0u;
      }
      mbar_arrive(bar_st);
    }
  }

  // scales and zero points of the CTA's groups as floats (s, s * z), by every
  // thread before the dependency wait: they do not depend on the previous
  // kernel and their copy is the first one issued (measured: 6.34 -> 6.23 us
  // per call at the Qwen3-4B gate_proj shape against converting them after
  // the activations are staged)
  mbar_wait(bar_st, 0);
  {
    float2* sfw = reinterpret_cast<float2*>(smem + L.sf);
    const __half* szs = reinterpret_cast<const __half*>(smem + L.sz_s);
    for (int it = tid; it < ngrp * COLS; it += THREADS) {
      const int gi = it >> 8, col = it & (COLS - 1);
      const float sc = __half2float(szs[it]);
      float z;
      if (p.zeros_packed)
        z = float(((reinterpret_cast<const uint32_t*>(smem + L.sz_z)[gi * (COLS / 8) + (col >> 3)] >>
                    (4 * (col & 7))) & 0xFu) + unsigned(p.zero_offset));
      else
        z = __half2float(reinterpret_cast<const __half*>(smem + L.sz_z)[it]);
      sfw[it] = make_float2(sc, sc * z);
    }
  }
  // activations (plain 128-bit loads) in MMA-B order (x0,x4 | x1,x5 | x2,x6 | x3,x7) per packed row,
  // and per group the sums over the two nibble classes:
  // (Off, Sx) = (1024 Xa + 64 Xb, Xa + Xb), by the whole CTA.  A group of a
  // row is an aligned block of 4*KPG lanes (whole warps join the shuffles).
  {
    const int Ts = ngrp * KPG;
    uint4* xsw = reinterpret_cast<uint4*>(smem + L.xs);
    float* xksw = reinterpret_cast<float*>(smem + L.xks);
    // work in chunks of 32 items (8 k-steps, whole groups) of one row, spread over the warps
    const int TB = (Ts + 7) >> 3;  // chunks per row
    // rows M..Mp-1 of every B fragment read one zero block past the rows
    if (tid < 4) xsw[size_t(p.Ts_max) * M * 4 + tid] = make_uint4(0u, 0u, 0u, 0u);
    // the activations may come from the previous kernel in the stream: wait
    // for it here, after every weight and static copy has been started
    if (p.pdl && !p.x_early) grid_dep_wait();
    trace_stamp(trc, TR_WAITED, tid == 0);
    if (p.addnorm) {
      // the residual add over whole rows (the norm needs every column), sums
      // of squares in fp32; r of this CTA's K range goes to xraw (normalised
      // in place below), and tile 0's CTAs store it as the new residual
      const int K8 = p.K >> 3;
      for (int m = 0; m < M; ++m) {
        float acc = 0.f;
        for (int cix = tid; cix < K8; cix += THREADS) {
          // plain loads: the previous kernels wrote these rows
          const uint4 a = *reinterpret_cast<const uint4*>(p.res + size_t(m) * p.K + cix * 8);
          const uint4 b = *reinterpret_cast<const uint4*>(p.delta + size_t(m) * p.K + cix * 8);
          const uint32_t ad[4] = {a.x, a.y, a.z, a.w}, bd[4] = {b.x, b.y, b.z, b.w};
          uint32_t od[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 fa = h2_to_f2(ad[j]), fb = h2_to_f2(bd[j]);
            const __half2 s2 = __floats2half2_rn(fa.x + fb.x, fa.y + fb.y);  // the fp16 residual add
            od[j] = *reinterpret_cast<const uint32_t*>(&s2);
            const float2 f = __half22float2(s2);
            acc = fmaf(f.x, f.x, acc);
            acc = fmaf(f.y, f.y, acc);
          }
          const int kl = cix * 8 - k0;
          if (kl >= 0 && kl < Ks) {
            const uint4 r8 = make_uint4(od[0], od[1], od[2], od[3]);
            *reinterpret_cast<uint4*>(xraw + m * XS + kl) = r8;
            if (tile == 0) *reinterpret_cast<uint4*>(p.res_out + size_t(m) * p.K + cix * 8) = r8;
          }
        }
        acc = warp_sum(acc);
        if (lane == 0) s_ss[warp][m] = acc;
      }
      __syncthreads();  // every warp of the CTA stages (the helper warp too)
      if (tid < M) {
        float t = 0.f;
#pragma unroll
        for (int w = 0; w <= WARPS; ++w) t += s_ss[w][tid];
        s_rs[tid] = 1.0f / sqrtf(t * (1.0f / float(p.K)) + p.eps);
      }
      __syncthreads();
    }
    const __half* xg = p.x + k0;
    // more than one 512-byte chunk per warp (wide batches): every chunk's
    // global read is issued at once (cp.async into xraw, one wait), so the
    // loop below runs on shared memory instead of one load round trip per
    // chunk
    const bool bulk = !p.addnorm && !p.x_early && M * TB > WARPS + 1;
    if (bulk) {
      for (int id = warp; id < M * TB; id += WARPS + 1) {
        const int m = id / TB, it = (id - m * TB) * 32 + lane, t = it >> 2, cc = it & 3;
        if (it < Ts * 4) {
          const uint32_t dst = smem_addr(xraw + m * XS + t * KSTEP + cc * 8);
          asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst),
                       "l"(xg + size_t(m) * p.K + t * KSTEP + cc * 8)
                       : "memory");
        }
      }
      asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
      __syncthreads();
    }
    for (int id = warp; id < M * TB; id += WARPS + 1) {
      const int m = id / TB, it = (id - m * TB) * 32 + lane, t = it >> 2, cc = it & 3;
      const bool ok = it < Ts * 4;  // Ts * 4 is a multiple of 4 * KPG: groups never straddle
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (ok) {
        if (p.addnorm) {  // x = fp16((r * rs) * w) from the staged r, as qx_add_rmsnorm rounds it
          const uint4 r8 = *reinterpret_cast<const uint4*>(xraw + m * XS + t * KSTEP + cc * 8);
          const uint4 w8 = ldg_v4(p.nw + k0 + t * KSTEP + cc * 8);
          const uint32_t rd[4] = {r8.x, r8.y, r8.z, r8.w}, wd[4] = {w8.x, w8.y, w8.z, w8.w};
          const float rs = s_rs[m];
          uint32_t od[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 f = h2_to_f2(rd[j]), gw = h2_to_f2(wd[j]);
            const __half2 o = __floats2half2_rn((f.x * rs) * gw.x, (f.y * rs) * gw.y);
            od[j] = *reinterpret_cast<const uint32_t*>(&o);
          }
          v = make_uint4(od[0], od[1], od[2], od[3]);
        } else if (bulk) {
          v = *reinterpret_cast<const uint4*>(xraw + m * XS + t * KSTEP + cc * 8);
        } else {
          v = *reinterpret_cast<const uint4*>(xg + size_t(m) * p.K + t * KSTEP + cc * 8);
        }
        if (!bulk) *reinterpret_cast<uint4*>(xraw + m * XS + t * KSTEP + cc * 8) = v;  // natural order, LoRA-down
        xsw[(t * M + m) * 4 + cc] = make_uint4(prmt(v.x, v.z, 0x5410u), prmt(v.x, v.z, 0x7632u),
                                                prmt(v.y, v.w, 0x5410u), prmt(v.y, v.w, 0x7632u));
      }
      const float2 a0 = h2_to_f2(v.x), a1 = h2_to_f2(v.y), a2 = h2_to_f2(v.z), a3 = h2_to_f2(v.w);
      float xa = (a0.x + a1.x) + (a2.x + a3.x);  // x0 + x2 + x4 + x6
      float xb = (a0.y + a1.y) + (a2.y + a3.y);  // x1 + x3 + x5 + x7
#pragma unroll
      for (int w = 1; w < 4 * KPG; w <<= 1) {  // the 4*KPG lanes of one group
        xa += __shfl_xor_sync(0xffffffffu, xa, w);
        xb += __shfl_xor_sync(0xffffffffu, xb, w);
      }
      if (ok && (it & (4 * KPG - 1)) == 0)
        *reinterpret_cast<float2*>(xksw + ((t / KPG) * Mp + m) * 2) =
            make_float2(fmaf(1024.f, xa, 64.f * xb), xa + xb);
    }
  }
  __syncthreads();  // permuted activations, group sums, scales ready

  constexpr bool lora_warps = LW;  // == lora_on_warps(M, R), chosen by the host
  if (warp == WARPS) {  // helper: the LoRA down-projection of small batches and ranks
    if (R == 0 || lora_warps) return;
    float* hs = reinterpret_cast<float*>(smem + L.hs);
    // h_s^T[r][m] = A^T[r][Ks] . x^T[Ks][m] as one 16 x 8 tile (rank rows x
    // batch rows; ranks 8 and 16, at most 8 rows), two accumulators (even /
    // odd k blocks), one group per ring stage as it lands
    const int mi = lane >> 3, ri = lane & 7;
    const __half* xrow = xraw + g * XS + 2 * c;  // batch row g of the B fragment
    const int j = 8 * (mi & 1);
    float h4[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    int hst = 0, huse = 0;
    for (int gi = 0; gi < ngrp; ++gi) {
      mbar_wait(full0 + 8 * hst, huse & 1);
      const __half* Ag = reinterpret_cast<const __half*>(smem + L.ring + hst * STAGE + WBYTES);
#pragma unroll
      for (int kb = 0; kb < 2 * KPG; kb += 2) {
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int k = (kb + u) * 16 + ri + 8 * (mi >> 1);
          uint32_t a[4];
          if (R >= 16) {
            ldsm_x4_t(a, Ag + k * R + j);
          } else {  // rank 8: rows 8..15 of the tile are zero
            ldsm_x4_t(a, Ag + k * R + (j & 7));
            a[1] = 0u;
            a[3] = 0u;
          }
          uint32_t b0 = 0u, b1 = 0u;
          if (g < M) {
            b0 = *reinterpret_cast<const uint32_t*>(xrow + gi * GROUPK + (kb + u) * 16);
            b1 = *reinterpret_cast<const uint32_t*>(xrow + gi * GROUPK + (kb + u) * 16 + 8);
          }
          mma_16816(h4[u], a[0], a[1], a[2], a[3], b0, b1);
        }
      }
      if (gi + nst < ngrp) {  // the compute warps refill this stage
        __syncwarp();
        if (lane == 0) mbar_arrive(empty0 + 8 * hst);
      }
      if (++hst == nst) {
        hst = 0;
        ++huse;
      }
    }
    const int j0 = g, m0 = 2 * c;
    if (m0 < M) hs[m0 * R + j0] = h4[0][0] + h4[1][0];
    if (m0 + 1 < M) hs[(m0 + 1) * R + j0] = h4[0][1] + h4[1][1];
    if (j0 + 8 < R) {
      if (m0 < M) hs[m0 * R + j0 + 8] = h4[0][2] + h4[1][2];
      if (m0 + 1 < M) hs[(m0 + 1) * R + j0 + 8] = h4[0][3] + h4[1][3];
    }
    trace_stamp(trc, TR_LORA_DOWN, lane == 0);
    if (lora_up_on_helper(M, R)) {
      // one row: the up-projection in fp32 here, while the compute warps still
      // stream weights (it then costs them one shared-memory read after their
      // loop instead of a chain of MMAs); lane owns columns 8 lane..8 lane + 7
      __syncwarp();  // every rank of h_s in shared memory
      mbar_wait(bar_b, 0);
      const __half* Bs = reinterpret_cast<const __half*>(smem + L.Bs) + lane * 8;
      float* lu = reinterpret_cast<float*>(smem + L.lu) + lane * 8;
      float a8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int jr = 0; jr < R; ++jr) {
        const float hv = p.lora_scale * hs[jr];
        const uint4 b8 = *reinterpret_cast<const uint4*>(Bs + jr * COLS);
        const uint32_t bw[4] = {b8.x, b8.y, b8.z, b8.w};
#pragma unroll
        for (int q2 = 0; q2 < 4; ++q2) {
          const float2 f = h2_to_f2(bw[q2]);
          a8[2 * q2] = fmaf(hv, f.x, a8[2 * q2]);
          a8[2 * q2 + 1] = fmaf(hv, f.y, a8[2 * q2 + 1]);
        }
      }
      *reinterpret_cast<float4*>(lu) = make_float4(a8[0], a8[1], a8[2], a8[3]);
      *reinterpret_cast<float4*>(lu + 4) = make_float4(a8[4], a8[5], a8[6], a8[7]);
    }
    mbar_arrive(bar_h);  // every lane: its h_s (and LoRA-term) stores are released
    return;
  }

  // ---------------- compute warps ----------------
  // LoRA down-projection items of this warp (batches above 8 rows, ranks of
  // 32 and more): (16-row block, 8-rank block) tiles warp, warp + 8, ...,
  // accumulated over the groups in registers
  constexpr int LITEMS = LW ? lora_items(NT) : 1;
  float hl[LITEMS][4];
#pragma unroll
  for (int ii = 0; ii < LITEMS; ++ii) hl[ii][0] = hl[ii][1] = hl[ii][2] = hl[ii][3] = 0.f;
  const int lcol = warp * 32 + 4 * g;  // first of this lane's 4 columns (tile-local)
  const bool col_ok = n_tile0 + lcol < N;  // N % 8 == 0: all 4 columns valid or none
  const uint4* xs = reinterpret_cast<const uint4*>(smem + L.xs);
  // B fragment rows nt*8 + g: the staged row, or the zero block (stride 0) past M
  const uint4* xrow[NT];
  int xstep[NT];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int row = nt * 8 + g;
    xrow[nt] = row < M ? xs + row * 4 + c : xs + size_t(p.Ts_max) * M * 4 + c;
    xstep[nt] = row < M ? M * 4 : 0;
  }
  const float* xks = reinterpret_cast<const float*>(smem + L.xks);

  // acc[pp][nt][i] holds column lcol + 2 pp + (i >> 1), row nt*8 + 2c + (i & 1)
  float acc[2][NT][4], cgr[2][NT][4];
#pragma unroll
  for (int pp = 0; pp < 2; ++pp)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[pp][nt][i] = 0.f;

  int st = 0, use = 0;  // ring stage and wrap count
  const unsigned char* wlane = smem + L.ring + c * ROWB + lcol * 4;
  for (int gi = 0; gi < ngrp; ++gi) {
    mbar_wait(full0 + 8 * st, use & 1);
    trace_stamp(trc, TR_GROUP0, tid == 0 && gi == 0);
#pragma unroll
    for (int j = 0; j < KPG; ++j) {
      const int t = gi * KPG + j;
      const uint4 wq = col_ok ? *reinterpret_cast<const uint4*>(wlane + st * STAGE + j * 4 * ROWB)
                              : make_uint4(0u, 0u, 0u, 0u);
      const uint32_t wv[4] = {wq.x, wq.y, wq.z, wq.w};
      uint32_t q[4][4];
#pragma unroll
      for (int jw = 0; jw < 4; ++jw) {
        const uint32_t hi = wv[jw] >> 8;
        q[jw][0] = lop3_and_or(wv[jw], 0x000F000Fu, 0x64006400u);  // (1024+q0, 1024+q4)
        q[jw][1] = lop3_and_or(wv[jw], 0x00F000F0u, 0x54005400u);  // (64+q1, 64+q5)
        q[jw][2] = lop3_and_or(hi, 0x000F000Fu, 0x64006400u);      // (1024+q2, 1024+q6)
        q[jw][3] = lop3_and_or(hi, 0x00F000F0u, 0x54005400u);      // (64+q3, 64+q7)
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        // activations of row nt*8 + g, packed row c: (x0,x4 | x1,x5 | x2,x6 | x3,x7)
        const uint4 bx = xrow[nt][t * xstep[nt]];
#pragma unroll
        for (int pp = 0; pp < 2; ++pp) {
          if (j == 0)  // the group's first products start from zero
            mma_16816_zc(cgr[pp][nt], q[2 * pp][0], q[2 * pp + 1][0], q[2 * pp][1],
                         q[2 * pp + 1][1], bx.x, bx.y);
          else
            mma_16816(cgr[pp][nt], q[2 * pp][0], q[2 * pp + 1][0], q[2 * pp][1], q[2 * pp + 1][1],
                      bx.x, bx.y);
          mma_16816(cgr[pp][nt], q[2 * pp][2], q[2 * pp + 1][2], q[2 * pp][3], q[2 * pp + 1][3],
                    bx.z, bx.w);
        }
      }
    }
    if (lora_warps) {  // this group's part of the warp's LoRA tiles, A rows from the stage
      const __half* Ag = reinterpret_cast<const __half*>(smem + L.ring + st * STAGE + WBYTES);
      const int RT8 = R >> 3, ntl = lora_tiles(M, R);
#pragma unroll
      for (int ii = 0; ii < LITEMS; ++ii) {
        const int tl = warp + WARPS * ii;
        if (tl < ntl) {
          const int mt = tl / RT8, rt = tl - mt * RT8;
          const int m0 = mt * 16 + g, m1 = m0 + 8;
          const __half* x0 = xraw + (m0 < M ? m0 : 0) * XS + gi * GROUPK + 2 * c;
          const __half* x1 = xraw + (m1 < M ? m1 : 0) * XS + gi * GROUPK + 2 * c;
#pragma unroll
          for (int kb = 0; kb < 2 * KPG; ++kb) {
            const uint32_t a0 = m0 < M ? *reinterpret_cast<const uint32_t*>(x0 + kb * 16) : 0u;
            const uint32_t a2 = m0 < M ? *reinterpret_cast<const uint32_t*>(x0 + kb * 16 + 8) : 0u;
            const uint32_t a1 = m1 < M ? *reinterpret_cast<const uint32_t*>(x1 + kb * 16) : 0u;
            const uint32_t a3 = m1 < M ? *reinterpret_cast<const uint32_t*>(x1 + kb * 16 + 8) : 0u;
            uint32_t bf[2];
            ldsm_x2_t(bf, Ag + (kb * 16 + (lane & 15)) * R + rt * 8);
            mma_16816(hl[ii], a0, a1, a2, a3, bf[0], bf[1]);
          }
        }
      }
    }
    if (gi + nst < ngrp) {  // every reader has read this stage: refill it with group gi + nst
      __syncwarp();
      if (lane == 0) mbar_arrive(empty0 + 8 * st);
      if (tid == 0) {
        mbar_wait(empty0 + 8 * st, use & 1);
        mbar_expect_tx(full0 + 8 * st, STAGE_TX);
        tma_2d_hint(ring_s + st * STAGE, &p.tw, wx, (ks0 + (gi + nst) * KPG) * 4, full0 + 8 * st,
                    evict_first_policy());
        if (R > 0)
          bulk_g2s(ring_s + st * STAGE + WBYTES, p.A + size_t(k0 + (gi + nst) * GROUPK) * R, ABYTES,
                   full0 + 8 * st);
      }
      __syncwarp();
    }
    {  // group correction: acc += s (C - Off) - (s z) Sx
      const float2* sf = reinterpret_cast<const float2*>(smem + L.sf) + gi * COLS + lcol;
      const float4 c01 = *reinterpret_cast<const float4*>(sf);      // (s, sz) of cols 0, 1
      const float4 c23 = *reinterpret_cast<const float4*>(sf + 2);  // cols 2, 3
      const float sv[4] = {c01.x, c01.z, c23.x, c23.z}, zv[4] = {c01.y, c01.w, c23.y, c23.w};
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        // (Off, Sx) of rows nt*8 + 2c, + 1 (rows >= M hold stale values that
        // only reach discarded accumulators)
        const float4 xv = *reinterpret_cast<const float4*>(xks + (gi * Mp + nt * 8 + 2 * c) * 2);
        const float off0 = xv.x, sx0 = xv.y, off1 = xv.z, sx1 = xv.w;
#pragma unroll
        for (int pp = 0; pp < 2; ++pp) {
          const float s0 = sv[2 * pp], s1 = sv[2 * pp + 1];
          const float z0 = zv[2 * pp], z1 = zv[2 * pp + 1];
          acc[pp][nt][0] = fmaf(-z0, sx0, fmaf(s0, cgr[pp][nt][0] - off0, acc[pp][nt][0]));
          acc[pp][nt][1] = fmaf(-z0, sx1, fmaf(s0, cgr[pp][nt][1] - off1, acc[pp][nt][1]));
          acc[pp][nt][2] = fmaf(-z1, sx0, fmaf(s1, cgr[pp][nt][2] - off0, acc[pp][nt][2]));
          acc[pp][nt][3] = fmaf(-z1, sx1, fmaf(s1, cgr[pp][nt][3] - off1, acc[pp][nt][3]));
        }
      }
    }
    if (++st == nst) {
      st = 0;
      ++use;
    }
  }

  trace_stamp(trc, TR_LOOP, tid == 0);
  if (lora_warps) {  // the warps' LoRA tiles into h_s [M][r]
    float* hp = reinterpret_cast<float*>(smem + L.hs);
    const int RT8 = R >> 3, ntl = lora_tiles(M, R);
#pragma unroll
    for (int ii = 0; ii < LITEMS; ++ii) {
      const int tl = warp + WARPS * ii;
      if (tl < ntl) {
        const int mt = tl / RT8, rt = tl - mt * RT8;
        const int m0 = mt * 16 + g, m1 = m0 + 8;
        float* dst = hp + rt * 8 + 2 * c;
        if (m0 < M) *reinterpret_cast<float2*>(dst + m0 * R) = make_float2(hl[ii][0], hl[ii][1]);
        if (m1 < M) *reinterpret_cast<float2*>(dst + m1 * R) = make_float2(hl[ii][2], hl[ii][3]);
      }
    }
  }
  const bool up_helper = !lora_warps && lora_up_on_helper(M, R);
  if (up_helper) {
    // the helper's LoRA term of this lane's 4 columns (row 0: lanes with c == 0)
    mbar_wait(bar_h, 0);
    if (c == 0) {
      const float4 u = *reinterpret_cast<const float4*>(smem + L.lu + lcol * 4);
      acc[0][0][0] += u.x;
      acc[0][0][2] += u.y;
      acc[1][0][0] += u.z;
      acc[1][0][2] += u.w;
    }
  }
  // otherwise this CTA's LoRA term (alpha/r) h_s B[:, tile] joins its partial
  // sums on the tensor cores: A = B^T (rows = this lane's columns), B operand
  // = (alpha/r) h_s^T split into fp16 high and low parts (~22-bit product)
  if (R > 0 && !up_helper) {
    const int RT = R >= 16 ? R / 16 : 1;
    if (lora_warps)
      asm volatile("bar.sync 1, %0;" ::"n"(WARPS * 32) : "memory");  // every warp's h_s partials
    else
      mbar_wait(bar_h, 0);
    mbar_wait(bar_b, 0);
    const float* hs = reinterpret_cast<const float*>(smem + L.hs);
    const __half* Bs = reinterpret_cast<const __half*>(smem + L.Bs);
    for (int kt = 0; kt < RT; ++kt) {
      const int j = kt * 16 + 2 * c;  // this lane's k (rank) pair; j + 8 for the upper half
      uint32_t bh[NT][2], bl[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int m = nt * 8 + g;
        float2 h0 = make_float2(0.f, 0.f), h1 = make_float2(0.f, 0.f);
        if (m < M) {
          {
            const float* hk = hs + size_t(m) * R + j;
            const float2 u = *reinterpret_cast<const float2*>(hk);
            h0.x += u.x;
            h0.y += u.y;
            if (R >= 16) {
              const float2 u8 = *reinterpret_cast<const float2*>(hk + 8);
              h1.x += u8.x;
              h1.y += u8.y;
            }
          }
        }
        const float ls = p.lora_scale;
        const __half2 h0h = __floats2half2_rn(ls * h0.x, ls * h0.y);
        const __half2 h1h = __floats2half2_rn(ls * h1.x, ls * h1.y);
        const float2 h0r = __half22float2(h0h), h1r = __half22float2(h1h);
        const __half2 h0l = __floats2half2_rn(ls * h0.x - h0r.x, ls * h0.y - h0r.y);
        const __half2 h1l = __floats2half2_rn(ls * h1.x - h1r.x, ls * h1.y - h1r.y);
        bh[nt][0] = *reinterpret_cast<const uint32_t*>(&h0h);
        bh[nt][1] = *reinterpret_cast<const uint32_t*>(&h1h);
        bl[nt][0] = *reinterpret_cast<const uint32_t*>(&h0l);
        bl[nt][1] = *reinterpret_cast<const uint32_t*>(&h1l);
      }
#pragma unroll
      for (int pp = 0; pp < 2; ++pp) {
        // (B[j][col], B[j+1][col]) for col = lcol + 2pp (row g) and + 1 (row g + 8)
        const __half* bcol = Bs + lcol + 2 * pp;
        const uint32_t w0 = *reinterpret_cast<const uint32_t*>(bcol + j * COLS);
        const uint32_t w1 = *reinterpret_cast<const uint32_t*>(bcol + (j + 1) * COLS);
        uint32_t w2 = 0u, w3 = 0u;
        if (R >= 16) {
          w2 = *reinterpret_cast<const uint32_t*>(bcol + (j + 8) * COLS);
          w3 = *reinterpret_cast<const uint32_t*>(bcol + (j + 9) * COLS);
        }
        const uint32_t a0 = prmt(w0, w1, 0x5410u), a1 = prmt(w0, w1, 0x7632u);
        const uint32_t a2 = prmt(w2, w3, 0x5410u), a3 = prmt(w2, w3, 0x7632u);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          mma_16816(acc[pp][nt], a0, a1, a2, a3, bh[nt][0], bh[nt][1]);
          mma_16816(acc[pp][nt], a0, a1, a2, a3, bl[nt][0], bl[nt][1]);
        }
      }
    }
  }

  trace_stamp(trc, TR_LORA_UP, tid == 0);
  // host-resident activations were read before the dependency wait: the
  // previous kernel may still write the output (a previous call's y)
  if (p.pdl && p.x_early) grid_dep_wait();
  // send the partial of the columns owned by CTA j into j's receive area
  // [S][M][CPR] (rows nt*8 + 2c (+1), columns lcol + 2pp (+1))
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
  // (the lane's 4 columns lcol..lcol+3 lie in one 8-column block, so in one
  // owner's range: one 16-byte st.async per row)
  if (col_ok) {
    const int owner = __umulhi(uint32_t(lcol), p.cpr_magic), cc = lcol - owner * CPR;
    const uint32_t rbase = map_rank(smem_addr(recv + size_t(s) * M * CPR + cc), owner);
    const uint32_t rbar = map_rank(bar_rv, owner);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int m0 = nt * 8 + 2 * c;
      if (m0 < M)
        st_async_f4(rbase + m0 * CPR * 4, acc[0][nt][0], acc[0][nt][2], acc[1][nt][0], acc[1][nt][2], rbar);
      if (m0 + 1 < M)
        st_async_f4(rbase + (m0 + 1) * CPR * 4, acc[0][nt][1], acc[0][nt][3], acc[1][nt][1], acc[1][nt][3],
                    rbar);
    }
  }

  trace_stamp(trc, TR_SENT, tid == 0);
  // this CTA's columns: wait for the S partials, sum in rank order, round
  if (own_cols > 0) {
    mbar_wait(bar_rv, 0);
    trace_stamp(trc, TR_RECEIVED, tid == 0);
    const int cb = n_tile0 + s * CPR;
    if (p.act) {
      // SwiGLU: output j of the block pair (gate cols 16b..16b+7, up cols
      // 16b+8..16b+15) = silu(g) u from the fp16-rounded sums, at y[m][cb/2 + j]
      const int nout = own_cols >> 1, N2 = N >> 1;
      for (int it = tid; it < M * nout; it += WARPS * 32) {
        const int m = it / nout, j = it - m * nout;
        const int cg = (j >> 3) * 16 + (j & 7);
        float gs = 0.f, us = 0.f;
        for (int r2 = 0; r2 < S; ++r2) {
          const float* rv = recv + (size_t(r2) * M + m) * CPR;
          gs += rv[cg];
          us += rv[cg + 8];
        }
        p.y[size_t(m) * N2 + (cb >> 1) + j] = __float2half_rn(silu_mul(round_h(gs), round_h(us)));
      }
      trace_stamp(trc, TR_EXIT, tid == 0);
      return;
    }
    if (M == 1) {
      for (int cc = tid; cc < own_cols; cc += WARPS * 32) {
        float v = 0.f;
        for (int r2 = 0; r2 < S; ++r2) v += recv[r2 * CPR + cc];
        p.y[cb + cc] = __float2half_rn(v);
      }
      trace_stamp(trc, TR_EXIT, tid == 0);
      return;
    }
    // the compute threads as (row, 4-column group) pairs: rpi rows per pass,
    // 16-byte reads of the partials (own_cols and CPR are multiples of 8)
    const int ov = own_cols >> 2;
    const int rpi = ov >= WARPS * 32 ? 1 : (WARPS * 32) / ov;
    const int mi = tid / ov, c0 = tid - mi * ov;
    for (int m0 = 0; m0 < M; m0 += rpi) {
      const int m = m0 + mi;
      if (mi < rpi && m < M) {
        for (int cv = c0; cv < ov; cv += WARPS * 32) {
          float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
          for (int r2 = 0; r2 < S; ++r2) {
            const float4 u = *reinterpret_cast<const float4*>(recv + (size_t(r2) * M + m) * CPR + 4 * cv);
            v.x += u.x;
            v.y += u.y;
            v.z += u.z;
            v.w += u.w;
          }
          __half* yo = p.y + size_t(m) * N + cb + 4 * cv;
          yo[0] = __float2half_rn(v.x);
          yo[1] = __float2half_rn(v.y);
          yo[2] = __float2half_rn(v.z);
          yo[3] = __float2half_rn(v.w);
        }
      }
    }
    trace_stamp(trc, TR_EXIT, tid == 0);
  }
}

template <int NT, int KPG, bool LW>
static int prepare(int dev) {
  static std::mutex mu;
  static bool done[64] = {};
  std::lock_guard<std::mutex> lk(mu);
  if (dev >= 0 && dev < 64 && done[dev]) return QX_OK;
  auto kern = w4a16_gemv_kernel<NT, KPG, LW>;
  QX_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(SMEM_LIMIT)),
              "w4a16_gemv: set smem limit");
  QX_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1),
              "w4a16_gemv: allow clusters of up to 16 CTAs");
  if (dev >= 0 && dev < 64) done[dev] = true;
  return QX_OK;
}

// Among the cluster sizes and ring depths whose shared memory fits (occupancy
// API for the co-resident clusters), pick one that keeps every SM busy with
// two or more CTAs if any does, then the fewest waves, then the fewest
// quantisation groups per CTA, then the deeper ring.
template <int NT, int KPG, bool LW>
static int make_plan(int M, int K, int N, int rank, int group, int zeros_packed, Plan* out) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, int, int, int, int, int>, Plan> cache;
  int dev = 0;
  QX_CUDA_TRY(cudaGetDevice(&dev), "w4a16_gemv: cudaGetDevice");
  const int pin_S = g_pin_S.load(), pin_nst = g_pin_nst.load();
  const auto key = std::make_tuple(dev, M, K, N, rank, group, zeros_packed, pin_S * 64 + pin_nst);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto itc = cache.find(key);
    if (itc != cache.end()) {
      if (itc->second.tiles == 0)  // remembered: no cluster size fits
        return fail(QX_ERR_UNSUPPORTED, "w4a16_gemv: no cluster size fits M=%d K=%d N=%d rank=%d", M, K,
                    N, rank);
      *out = itc->second;
      return QX_OK;
    }
  }
  const int rc = prepare<NT, KPG, LW>(dev);
  if (rc != QX_OK) return rc;
  const int tiles = (N + COLS - 1) / COLS, T = K / KSTEP, Gt = K / group;
  Plan best{};
  long best_key = -1;
  for (int S = 1; S <= MAX_S && S <= Gt; ++S) {
    if (pin_S > 0 && S != pin_S) continue;
    Plan pl{};
    pl.NT = NT;
    pl.tiles = tiles;
    pl.T = T;
    pl.S = S;
    const int gmax = (Gt + S - 1) / S;
    if (gmax > 256) continue;  // one tensor-map box covers a CTA's scale rows
    if (pin_S == 0 && S > 1 && (Gt + S - 2) / (S - 1) == gmax) continue;  // a smaller cluster is as short
    pl.Ts_max = gmax * KPG;
    // a shallower weight ring (down to 2 stages) buys shared memory for more
    // CTAs per SM, hence wider clusters in one wave on deep-K shapes
    for (int nst = std::min(gmax, MAX_NST); nst >= std::min(gmax, 2); --nst) {
    if (pin_nst > 0 && nst != pin_nst) continue;
    pl.nst = nst;
    pl.smem = layout(M, KPG, pl.Ts_max, rank, S, pl.nst, zeros_packed).total;
    if (pl.smem > SMEM_LIMIT) continue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(tiles, S, 1);
    cfg.blockDim = dim3(THREADS, 1, 1);
    cfg.dynamicSmemBytes = pl.smem;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 1;
    at[0].val.clusterDim.y = S;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, w4a16_gemv_kernel<NT, KPG, LW>, &cfg) != cudaSuccess ||
        clusters <= 0) {
      cudaGetLastError();
      continue;
    }
    const long waves = (long(tiles) + clusters - 1) / clusters;
    // order: single-row plans that keep every SM busy with at least two CTAs
    // first, then fewer waves, then fewer groups per
    // CTA, then the deeper ring.  (Fewest waves alone ran a 4096 x 24576
    // single-row GEMV as 96 one-per-SM CTAs: 35 us, against 24 us for 384
    // CTAs two per SM.  Models of the busiest SM's streaming time that
    // favoured one CTA per SM with a deep ring measured slower: with 9 warps
    // an SM's int4 arithmetic bounds it.)
    int resident = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&resident, w4a16_gemv_kernel<NT, KPG, LW>, THREADS,
                                                      pl.smem) != cudaSuccess) {
      cudaGetLastError();
      resident = 0;
    }
    // (single-row instances: wider batches are bounded by their arithmetic and
    // keep the fewest-waves order, which measured best for them)
    const bool fills = NT > 1 || (long(tiles) * S >= device_sm_count() && resident >= 2);
    const long key2 = (fills ? 0L : 1000000000000L) + waves * 1000000L + long(gmax) * 1000L + (MAX_NST - nst);
    if (best_key < 0 || key2 < best_key) {
      best = pl;
      best_key = key2;
    }
    }
  }
  if (best_key < 0) {
    std::lock_guard<std::mutex> lk(mu);
    cache[key] = Plan{};
    return fail(QX_ERR_UNSUPPORTED, "w4a16_gemv: no cluster size fits M=%d K=%d N=%d rank=%d", M, K, N,
                rank);
  }
  {
    std::lock_guard<std::mutex> lk(mu);
    cache[key] = best;
  }
  *out = best;
  return QX_OK;
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

// 2-D tiled tensor map, no swizzle, zero fill outside the tensor.
static int encode_2d(CUtensorMap* map, CUtensorMapDataType type, const void* base, uint64_t cols,
                     uint64_t rows, uint64_t row_stride_bytes, uint32_t box_cols, uint32_t box_rows,
                     const char* what) {
  const auto enc = tmap_encoder();
  if (!enc) return fail(QX_ERR_CUDA, "w4a16_gemv: cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {row_stride_bytes};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, type, 2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(QX_ERR_CUDA, "w4a16_gemv: tensor map for %s (CUresult %d)", what, int(r));
  return QX_OK;
}

template <int NT, int KPG, bool LW>
static int build_params(Params& prm, Plan* plo);
template <int NT, int KPG, bool LW>
static int launch(const Params& prm, const Plan& pl, cudaStream_t st);

// Launch parameters (plan and tensor maps) of recent calls, keyed by every
// input that shapes them except the activations and the output: a decode loop
// calls the same weights again and again, so the host work per call is a
// lookup.  A tensor map only encodes an address, sizes and strides, so an
// entry stays valid for whatever tensor later occupies the same address with
// the same sizes.
struct ParamKey {
  const void *qw, *sc, *z, *A, *B;
  int dev, M, K, N, rank, group, zp, zo, pdl, nt, kpg;
  uint32_t ls;
  bool operator==(const ParamKey& o) const {
    return qw == o.qw && sc == o.sc && z == o.z && A == o.A && B == o.B && dev == o.dev && M == o.M &&
           K == o.K && N == o.N && rank == o.rank && group == o.group && zp == o.zp && zo == o.zo &&
           pdl == o.pdl && nt == o.nt && kpg == o.kpg && ls == o.ls;
  }
};
struct ParamKeyHash {
  size_t operator()(const ParamKey& k) const {
    size_t h = 1469598103934665603ull;
    auto mix = [&h](uint64_t v) { h = (h ^ v) * 1099511628211ull; };
    mix(reinterpret_cast<uintptr_t>(k.qw));
    mix(reinterpret_cast<uintptr_t>(k.sc));
    mix(reinterpret_cast<uintptr_t>(k.z));
    mix(reinterpret_cast<uintptr_t>(k.A));
    mix(reinterpret_cast<uintptr_t>(k.B));
    mix((uint64_t(k.M) << 32) ^ uint64_t(k.N) ^ (uint64_t(k.dev) << 56));
    mix((uint64_t(k.K) << 32) ^ uint64_t(k.rank) ^ (uint64_t(k.nt) << 48) ^ (uint64_t(k.kpg) << 56));
    mix((uint64_t(k.ls) << 32) ^ uint64_t(k.group) ^ (uint64_t(k.zp) << 16) ^ (uint64_t(k.zo) << 24) ^
        (uint64_t(k.pdl) << 28));
    return h;
  }
};
struct ParamEntry {
  Params prm;
  Plan pl;
};
static std::mutex g_param_mu;
static std::unordered_map<ParamKey, ParamEntry, ParamKeyHash> g_params;
constexpr size_t PARAM_CACHE_MAX = 1024;

template <int NT, int KPG, bool LW>
static int run(Params prm, cudaStream_t st) {
  int dev = 0;
  QX_CUDA_TRY(cudaGetDevice(&dev), "w4a16_gemv: cudaGetDevice");
  uint32_t ls_bits;
  std::memcpy(&ls_bits, &prm.lora_scale, 4);
  const ParamKey key{prm.qw, prm.scales, prm.zeros, prm.A, prm.B, dev, prm.M, prm.K, prm.N, prm.rank,
                     prm.group, prm.zeros_packed, prm.zero_offset,
                     prm.pdl + 2 * prm.act + 4 * prm.x_early + 8 * prm.addnorm, NT, KPG * 2 + (LW ? 1 : 0),
                     ls_bits};
  Plan pl;
  bool hit = false;
  {
    std::lock_guard<std::mutex> lk(g_param_mu);
    auto it = g_params.find(key);
    if (it != g_params.end()) {  // the cached plan and maps; this call's rows and output
      const Params call = prm;
      prm = it->second.prm;
      prm.x = call.x;
      prm.y = call.y;
      prm.res = call.res;
      prm.delta = call.delta;
      prm.nw = call.nw;
      prm.res_out = call.res_out;
      prm.eps = call.eps;
      pl = it->second.pl;
      hit = true;
    }
  }
  if (!hit) {
    const int rc = build_params<NT, KPG, LW>(prm, &pl);
    if (rc != QX_OK) return rc;
    std::lock_guard<std::mutex> lk(g_param_mu);
    if (g_params.size() >= PARAM_CACHE_MAX) g_params.clear();
    g_params.emplace(key, ParamEntry{prm, pl});
  }
  prm.trace = trace_next(QX_TRACE_GEMV, &prm.trace_launch);
  return launch<NT, KPG, LW>(prm, pl, st);
}

// Plan and tensor maps of one call (everything but the activations and output).
template <int NT, int KPG, bool LW>
static int build_params(Params& prm, Plan* plo) {
  Plan pl;
  int rc = make_plan<NT, KPG, LW>(prm.M, prm.K, prm.N, prm.rank, prm.group, prm.zeros_packed, &pl);
  if (rc != QX_OK) return rc;
  prm.T = pl.T;
  prm.S = pl.S;
  prm.s_magic = pl.S > 1 ? uint32_t((0x100000000ull + pl.S - 1) / pl.S) : 0u;
  // the SwiGLU epilogue keeps the plan of the plain GEMV (the same split of K,
  // hence the same sums) with owners of whole 16-column block pairs
  const int ocols = owner_cols(pl.S, prm.act);
  prm.cpr_magic = uint32_t((0x100000000ull + ocols - 1) / ocols);
  prm.lay = layout(prm.M, KPG, pl.Ts_max, prm.rank, pl.S, pl.nst, prm.zeros_packed, prm.act);
  if (prm.lay.total > SMEM_LIMIT)
    return fail(QX_ERR_UNSUPPORTED, "w4a16_gemv_swiglu: shared memory %u over the limit", prm.lay.total);
  pl.smem = prm.lay.total;
  prm.cpr = ocols;
  prm.Ts_max = pl.Ts_max;
  prm.gmax = pl.Ts_max / KPG;
  prm.nst = pl.nst;
  prm.stage = stage_bytes(KPG, prm.rank);
  // qweight as 64-bit elements [K/8][N/2]; one box = a group of packed rows x
  // (256 + 8) columns, i.e. 1056 B rows
  rc = encode_2d(&prm.tw, CU_TENSOR_MAP_DATA_TYPE_UINT64, prm.qw, uint64_t(prm.N) / 2,
                 uint64_t(prm.K) / 8, uint64_t(prm.N) * 4, ROWB / 8, uint32_t(KPG) * 4, "qweight");
  if (rc != QX_OK) return rc;
  const uint64_t Gt = uint64_t(prm.K / prm.group);
  rc = encode_2d(&prm.ts, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, prm.scales, uint64_t(prm.N), Gt,
                 uint64_t(prm.N) * 2, COLS, uint32_t(prm.gmax), "scales");
  if (rc != QX_OK) return rc;
  prm.zeros_tma = !prm.zeros_packed || (prm.N % 32 == 0 && aligned(prm.zeros, 16));
  if (prm.zeros_packed && prm.zeros_tma)
    rc = encode_2d(&prm.tz, CU_TENSOR_MAP_DATA_TYPE_INT32, prm.zeros, uint64_t(prm.N) / 8, Gt,
                   uint64_t(prm.N) / 2, COLS / 8, uint32_t(prm.gmax), "qzeros");
  else if (!prm.zeros_packed)
    rc = encode_2d(&prm.tz, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, prm.zeros, uint64_t(prm.N), Gt,
                   uint64_t(prm.N) * 2, COLS, uint32_t(prm.gmax), "zeros");
  if (rc != QX_OK) return rc;
  if (prm.rank > 0) {
    rc = encode_2d(&prm.tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, prm.B, uint64_t(prm.N),
                   uint64_t(prm.rank), uint64_t(prm.N) * 2, COLS, uint32_t(prm.rank), "lora_B");
    if (rc != QX_OK) return rc;
  }
  *plo = pl;
  return QX_OK;
}

template <int NT, int KPG, bool LW>
static int launch(const Params& prm, const Plan& pl, cudaStream_t st) {
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
  if (prm.pdl) {
    attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = na;
  QX_CUDA_TRY(cudaLaunchKernelEx(&cfg, w4a16_gemv_kernel<NT, KPG, LW>, prm), "w4a16_gemv: launch");
  return check_launch("w4a16_gemv");
}

template <int NT, bool LW>
static int dispatch_kpg(const Params& prm, int kpg, cudaStream_t st) {
  switch (kpg) {
    case 1: return run<NT, 1, LW>(prm, st);
    case 2: return run<NT, 2, LW>(prm, st);
    case 4: return run<NT, 4, LW>(prm, st);
    default: return run<NT, 8, LW>(prm, st);
  }
}

static int dispatch(const Params& prm, int kpg, cudaStream_t st) {
  const bool lw = lora_on_warps(prm.M, prm.rank);
  if (prm.M <= 8) return lw ? dispatch_kpg<1, true>(prm, kpg, st) : dispatch_kpg<1, false>(prm, kpg, st);
  if (prm.M <= 16) return lw ? dispatch_kpg<2, true>(prm, kpg, st) : dispatch_kpg<2, false>(prm, kpg, st);
  return lw ? dispatch_kpg<4, true>(prm, kpg, st) : dispatch_kpg<4, false>(prm, kpg, st);
}

}  // namespace gemv
}  // namespace qx

using namespace qx;

namespace qx {
int gemm_device_error(unsigned* code, int reset);      // w4a16_gemm.cu
int nvar_device_error(unsigned* code, int reset);      // nvlink_allreduce.cu
int attn_device_error(unsigned* code, int reset);      // decode_attn.cu
}

extern "C" int qx_get_device_error(unsigned* code, int reset) {
  QX_REQUIRE(code, "get_device_error: null output");
  QX_CUDA_TRY(cudaMemcpyFromSymbol(code, g_device_error, sizeof(unsigned)),
              "get_device_error: read");
  if (reset) {
    const unsigned zero = 0;
    QX_CUDA_TRY(cudaMemcpyToSymbol(g_device_error, &zero, sizeof(unsigned)),
                "get_device_error: reset");
  }
  unsigned other = 0;
  int rc = qx::gemm_device_error(&other, reset);
  if (rc != QX_OK) return rc;
  *code |= other;
  rc = qx::nvar_device_error(&other, reset);
  if (rc != QX_OK) return rc;
  *code |= other;
  rc = qx::attn_device_error(&other, reset);
  if (rc != QX_OK) return rc;
  *code |= other;
  return QX_OK;
}

namespace qx {
namespace gemv {
// The device address of host memory the device can access (pinned / mapped),
// else null.
static void* device_view(const void* host) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, host) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return a.type == cudaMemoryTypeHost ? a.devicePointer : nullptr;
}
}  // namespace gemv
}  // namespace qx

namespace qx {
namespace gemv {
struct AddNorm {  // the residual add + RMSNorm prologue's operands
  const void* res;
  const void* delta;
  const void* nw;
  void* res_out;
  float eps;
};
}  // namespace gemv
}  // namespace qx

static int w4a16_gemv_entry(const void* x, const int32_t* qweight, const void* scales, const void* zeros,
                            int zeros_packed, int zero_offset, const void* lora_A, const void* lora_B, void* y,
                            int M, int K, int N, int rank, int group_size, float lora_scale,
                            qx_stream_t stream, int act, int x_early, const gemv::AddNorm* an = nullptr);

extern "C" int qx_w4a16_lora_gemv_host(const void* x_host, void* y_host, void* x_dev, void* y_dev,
                                       const int32_t* qweight, const void* scales, const void* zeros,
                                       int zeros_packed, int zero_offset, const void* lora_A,
                                       const void* lora_B, int M, int K, int N, int rank, int group_size,
                                       float lora_scale, qx_stream_t stream) {
  QX_REQUIRE(x_host && y_host && x_dev && y_dev, "w4a16_gemv_host: null buffer");
  QX_REQUIRE(M >= 0 && K > 0 && N > 0, "w4a16_gemv_host: bad sizes M=%d K=%d N=%d", M, K, N);
  if (M == 0) return QX_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const size_t xbytes = size_t(M) * K * 2;
  // pinned (device-mapped) host rows: the GEMV reads x_host itself, before
  // its dependency wait (the host wrote x before this call), so the read
  // overlaps the previous kernel; pageable rows: a copy into x_dev
  // (unless x_host overlaps the y_host of the previous call made here, which
  // that call's GEMV may still be writing: then the read waits)
  static std::mutex last_mu;
  static uintptr_t last_y0 = 0, last_y1 = 0;
  const uintptr_t x0 = reinterpret_cast<uintptr_t>(x_host), x1 = x0 + xbytes;
  const uintptr_t y0 = reinterpret_cast<uintptr_t>(y_host), y1 = y0 + size_t(M) * N * 2;
  bool early;
  {
    std::lock_guard<std::mutex> lk(last_mu);
    early = x1 <= last_y0 || last_y1 <= x0;
    last_y0 = y0;
    last_y1 = y1;
  }
  const void* xh = gemv::device_view(x_host);
  if (!xh)
    QX_CUDA_TRY(cudaMemcpyAsync(x_dev, x_host, xbytes, cudaMemcpyHostToDevice, st),
                "w4a16_gemv_host: copy x to the device");
  // y: written by the GEMV straight into pinned host memory; else a copy
  void* yh = gemv::device_view(y_host);
  const int rc = w4a16_gemv_entry(xh ? xh : x_dev, qweight, scales, zeros, zeros_packed, zero_offset, lora_A,
                                  lora_B, yh ? yh : y_dev, M, K, N, rank, group_size, lora_scale, stream, 0,
                                  xh && early ? 1 : 0);
  if (rc != QX_OK) return rc;
  if (!yh)
    QX_CUDA_TRY(cudaMemcpyAsync(y_host, y_dev, size_t(M) * N * 2, cudaMemcpyDeviceToHost, st),
                "w4a16_gemv_host: copy y to the host");
  return QX_OK;
}

extern "C" int qx_w4a16_gemv_plan(int M, int K, int N, int rank, int group_size, int zeros_packed,
                                  int* out) {
  QX_REQUIRE(out, "w4a16_gemv_plan: null output");
  QX_REQUIRE(M >= 1 && K > 0 && K % gemv::KSTEP == 0 && N > 0 && N % 8 == 0 &&
                 (group_size == 32 || group_size == 64 || group_size == 128 || group_size == 256) &&
                 K % group_size == 0,
             "w4a16_gemv_plan: bad shape M=%d K=%d N=%d group=%d", M, K, N, group_size);
  const int mc = std::min(M, gemv::MROWS);
  const int kpg = group_size / gemv::KSTEP;
  const bool lw = gemv::lora_on_warps(mc, rank);
  gemv::Plan pl{};
  int rc = QX_OK;
  auto pick = [&](auto nt_tag) {
    constexpr int NT = decltype(nt_tag)::value;
    switch (kpg) {
      case 1: rc = lw ? gemv::make_plan<NT, 1, true>(mc, K, N, rank, group_size, zeros_packed, &pl)
                      : gemv::make_plan<NT, 1, false>(mc, K, N, rank, group_size, zeros_packed, &pl); break;
      case 2: rc = lw ? gemv::make_plan<NT, 2, true>(mc, K, N, rank, group_size, zeros_packed, &pl)
                      : gemv::make_plan<NT, 2, false>(mc, K, N, rank, group_size, zeros_packed, &pl); break;
      case 4: rc = lw ? gemv::make_plan<NT, 4, true>(mc, K, N, rank, group_size, zeros_packed, &pl)
                      : gemv::make_plan<NT, 4, false>(mc, K, N, rank, group_size, zeros_packed, &pl); break;
      default: rc = lw ? gemv::make_plan<NT, 8, true>(mc, K, N, rank, group_size, zeros_packed, &pl)
                       : gemv::make_plan<NT, 8, false>(mc, K, N, rank, group_size, zeros_packed, &pl); break;
    }
  };
  if (mc <= 8) pick(std::integral_constant<int, 1>{});
  else if (mc <= 16) pick(std::integral_constant<int, 2>{});
  else pick(std::integral_constant<int, 4>{});
  if (rc != QX_OK) return rc;
  out[0] = pl.tiles;
  out[1] = pl.S;
  out[2] = pl.nst;
  out[3] = pl.Ts_max / kpg;
  out[4] = int(pl.smem);
  return QX_OK;
}

extern "C" int qx_w4a16_gemv_pin_plan(int S, int nst) {
  QX_REQUIRE(S >= 0 && S <= gemv::MAX_S && nst >= 0 && nst <= gemv::MAX_NST,
             "w4a16_gemv_pin_plan: S=%d (0..%d), stages=%d (0..%d)", S, gemv::MAX_S, nst, gemv::MAX_NST);
  g_pin_S.store(S);
  g_pin_nst.store(nst);
  {
    std::lock_guard<std::mutex> lk(gemv::g_param_mu);
    gemv::g_params.clear();  // cached launch parameters carry the old plan
  }
  return QX_OK;
}

extern "C" int qx_set_pdl(int enable) {
  g_pdl_enabled.store(enable ? 1 : 0);
  return QX_OK;
}

static int w4a16_gemv_entry(const void* x, const int32_t* qweight, const void* scales,
                                  const void* zeros, int zeros_packed, int zero_offset,
                                  const void* lora_A, const void* lora_B, void* y, int M, int K,
                                  int N, int rank, int group_size, float lora_scale,
                                  qx_stream_t stream, int act, int x_early, const gemv::AddNorm* an) {
  QX_REQUIRE(M >= 0 && K > 0 && N > 0, "w4a16_gemv: bad sizes M=%d K=%d N=%d", M, K, N);
  if (M == 0) return QX_OK;
  QX_REQUIRE(K % gemv::KSTEP == 0, "w4a16_gemv: K=%d must be a multiple of 32", K);
  QX_REQUIRE((group_size == 32 || group_size == 64 || group_size == 128 || group_size == 256) &&
                 K % group_size == 0,
             "w4a16_gemv: group_size=%d must be 32, 64, 128 or 256 and divide K=%d", group_size, K);
  QX_REQUIRE(N % 8 == 0, "w4a16_gemv: N=%d must be a multiple of 8", N);
  QX_REQUIRE(rank == 0 || rank == 8 || rank == 16 || rank == 32 || rank == 48 || rank == 64 ||
                 rank == 128,
             "w4a16_gemv: LoRA rank %d unsupported (0, 8, 16, 32, 48, 64 or 128)", rank);
  QX_REQUIRE(x && qweight && scales && zeros && y, "w4a16_gemv: null tensor pointer");
  QX_REQUIRE(rank == 0 || (lora_A && lora_B), "w4a16_gemv: rank=%d but lora_A/lora_B missing",
             rank);
  QX_REQUIRE(aligned(x, 16) && aligned(qweight, 16) && aligned(scales, 16) &&
                 (rank == 0 || (aligned(lora_A, 16) && aligned(lora_B, 16))),
             "w4a16_gemv: x, qweight, scales, lora_A and lora_B must be 16-byte aligned");
  QX_REQUIRE(aligned(zeros, zeros_packed ? 4 : 16) && aligned(y, 2),
             "w4a16_gemv: misaligned zeros/y");
  QX_REQUIRE(zeros_packed == 0 || zeros_packed == 1, "w4a16_gemv: zeros_packed must be 0 or 1");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // up to 32 rows per launch; fewer when the activations of 32 rows and the
  // kernel's weight stages do not fit in shared memory together
  int mrows = gemv::MROWS;
  for (int m0 = 0; m0 < M;) {
    const int mc = std::min(mrows, M - m0);
    gemv::Params prm{};
    prm.x = static_cast<const __half*>(x) + size_t(m0) * K;
    prm.qw = reinterpret_cast<const uint32_t*>(qweight);
    prm.scales = static_cast<const __half*>(scales);
    prm.zeros = zeros;
    prm.A = static_cast<const __half*>(lora_A);
    prm.B = static_cast<const __half*>(lora_B);
    prm.y = static_cast<__half*>(y) + size_t(m0) * (act ? N / 2 : N);
    prm.M = mc;
    prm.K = K;
    prm.N = N;
    prm.rank = rank;
    prm.group = group_size;
    prm.zeros_packed = zeros_packed;
    prm.zero_offset = zero_offset;
    prm.lora_scale = rank > 0 ? lora_scale : 0.f;
    prm.pdl = g_pdl_enabled.load(std::memory_order_relaxed);
    prm.act = act;
    prm.x_early = x_early;
    if (an) {  // a single launch (the host keeps M <= 8)
      prm.addnorm = 1;
      prm.res = static_cast<const __half*>(an->res);
      prm.delta = static_cast<const __half*>(an->delta);
      prm.nw = static_cast<const __half*>(an->nw);
      prm.res_out = static_cast<__half*>(an->res_out);
      prm.eps = an->eps;
    }
    const int rc = gemv::dispatch(prm, group_size / gemv::KSTEP, st);
    if (rc == QX_ERR_UNSUPPORTED && mc > 8) {
      mrows = mc > 16 ? 16 : 8;
      continue;
    }
    if (rc != QX_OK) return rc;
    m0 += mc;
  }
  return QX_OK;
}

extern "C" int qx_w4a16_lora_gemv(const void* x, const int32_t* qweight, const void* scales,
                                  const void* zeros, int zeros_packed, int zero_offset,
                                  const void* lora_A, const void* lora_B, void* y, int M, int K,
                                  int N, int rank, int group_size, float lora_scale,
                                  qx_stream_t stream) {
  return w4a16_gemv_entry(x, qweight, scales, zeros, zeros_packed, zero_offset, lora_A, lora_B, y, M, K, N,
                          rank, group_size, lora_scale, stream, 0, 0);
}

extern "C" int qx_w4a16_lora_gemv_addnorm(const void* residual, const void* delta, const void* norm_weight,
                                          float eps, void* residual_out, const int32_t* qweight,
                                          const void* scales, const void* zeros, int zeros_packed,
                                          int zero_offset, const void* lora_A, const void* lora_B, void* y,
                                          int M, int K, int N, int rank, int group_size, float lora_scale,
                                          int swiglu, qx_stream_t stream) {
  QX_REQUIRE(M >= 0 && M <= 8, "w4a16_gemv_addnorm: M=%d rows (1..8)", M);
  QX_REQUIRE(K > 0 && K % 8 == 0, "w4a16_gemv_addnorm: K=%d must be a multiple of 8", K);
  QX_REQUIRE(swiglu == 0 || swiglu == 1, "w4a16_gemv_addnorm: swiglu must be 0 or 1");
  QX_REQUIRE(!swiglu || (N > 0 && N % 16 == 0), "w4a16_gemv_addnorm: N=%d must be a multiple of 16 with SwiGLU",
             N);
  QX_REQUIRE(residual && delta && norm_weight && residual_out, "w4a16_gemv_addnorm: null pointer");
  QX_REQUIRE(aligned(residual, 16) && aligned(delta, 16) && aligned(norm_weight, 16) && aligned(residual_out, 16),
             "w4a16_gemv_addnorm: residual, delta, norm_weight and residual_out must be 16-byte aligned");
  const size_t rb = size_t(M) * K * 2;
  const uintptr_t o0 = reinterpret_cast<uintptr_t>(residual_out);
  auto overlaps = [&](const void* t) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(t);
    return a < o0 + rb && o0 < a + rb;
  };
  QX_REQUIRE(!overlaps(residual) && !overlaps(delta),
             "w4a16_gemv_addnorm: residual_out must not overlap residual or delta (other CTAs still read them)");
  if (M == 0) return QX_OK;
  const gemv::AddNorm an{residual, delta, norm_weight, residual_out, eps};
  return w4a16_gemv_entry(residual, qweight, scales, zeros, zeros_packed, zero_offset, lora_A, lora_B, y, M, K,
                          N, rank, group_size, lora_scale, stream, swiglu, 0, &an);
}

extern "C" int qx_w4a16_lora_gemv_swiglu(const void* x, const int32_t* qweight, const void* scales,
                                         const void* zeros, int zeros_packed, int zero_offset,
                                         const void* lora_A, const void* lora_B, void* y, int M, int K,
                                         int N, int rank, int group_size, float lora_scale,
                                         qx_stream_t stream) {
  QX_REQUIRE(N > 0 && N % 16 == 0, "w4a16_gemv_swiglu: N=%d must be a multiple of 16 (gate|up blocks of 8)",
             N);
  return w4a16_gemv_entry(x, qweight, scales, zeros, zeros_packed, zero_offset, lora_A, lora_B, y, M, K, N,
                          rank, group_size, lora_scale, stream, 1, 0);
}
