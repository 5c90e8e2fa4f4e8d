// W4A16 + LoRA prefill GEMM for sm_100a on the 5th-generation tensor cores.
//
// The large-M form of w4a16_lora_gemv (csrc/kernels/w4a16_lora_gemv.cu:268-323,
// which the reference runs one output element per thread block):
//   y[M, N] = fp16( x[M, K] . dequant(W)[K, N] + (alpha/r) (x . A) . B )
// with W = s (q - z) per quantisation group, fp32 accumulation.
//
// Two launches:
//   lora_down_kernel   (alpha/r) h = (alpha/r) x . A in fp32 (mma.sync; r <= 64,
//                      ~1.6 % of the FLOPs), stored as fp16 high and low parts
//                      [M][64] (zero-padded ranks) for the GEMM's TMA
//   w4a16_gemm_kernel  one CTA per 128 x 256 output tile:
//     warp 0      TMA producers: lane 0 the int4 weight tile [8 packed rows x
//                 256 columns], scales and zero points of each K block (a
//                 6-stage ring freed by the dequant warps), lane 1 the x tile
//                 [128 x 64] (128B swizzle, K-major; a 4-stage ring freed by
//                 the MMA commits)
//     warp 1      TMEM allocation (256 columns: a 128 x 256 fp32 accumulator)
//                 and, from one thread, tcgen05.mma kind::f16 (M=128, N=256,
//                 K=16) on shared-memory descriptors; tcgen05.commit releases
//                 the x and B stages
//     warps 2-17  dequantise the weight tile into the K-major, 128B-swizzled fp16
//                 B operand (2 stages): per packed word, PRMT + LOP3 put
//                 (1024 + q_2i | 64 + q_2i+1) in a half2 (the nibble lands in
//                 the mantissa of 1024 and, four bits up, of 64), HSUB2 removes
//                 (1024 + z | 64 + z) exactly and HMUL2 applies the scale:
//                 fp16(s (q - z)), as the reference dequantises
//                 (tests/test_w4a16_gemv.py:68-90); then the epilogue
//                 (tcgen05.ld 32x32b, fp32 -> fp16, 16-byte stores)
//   The LoRA term enters the same accumulator first: A = the high and low
//   parts of (alpha/r) h (two MMAs, ~22-bit product) and the LoRA B tile, both
//   by TMA before the weight stream; the dequant warps transpose the B tile into the
//   K-major swizzled layout in shared memory.
// Every wait is bounded (2 s, then QX_DEVERR_MBAR_TIMEOUT in the device
// error word); every copy targets this CTA only.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "qx_b200.h"
#include "qx_common.cuh"

namespace qx {
namespace gemm {

constexpr int BM = 128, BN = 256, BK = 64;
// Three rings, each as deep as its producer's latency needs: x tiles (the MMA
// A operand, mostly L2 hits; a stage is freed by the MMA commit), packed
// weights with their scales and zero points (from HBM; freed as soon as the
// dequant warps have read them, so they run furthest ahead) and dequantised
// B tiles (dequant warps -> MMA).  Measured with one ring of 3 stages for
// x + weights and 3 for B: 666 TFLOP/s over the 7 Qwen3-8B shapes (2 stages:
// 549): the weights' stage stayed busy until the MMA of its k-block retired.
#ifndef QX_GEMM_XS
#define QX_GEMM_XS 4
#define QX_GEMM_WS 6
#define QX_GEMM_BS 2
#endif
constexpr int XS = QX_GEMM_XS;  // x-tile stages
constexpr int WS = QX_GEMM_WS;  // packed-weight stages
constexpr int BS = QX_GEMM_BS;  // dequantised-B stages (>= 2: the LoRA B tile is staged raw in slot 1)
static_assert(BS >= 2, "the raw LoRA B tile uses B slot 1");
// Dequantisation is the kernel's issue-bound part (per 8 weights: LDS, 4 x
// PRMT/LOP3/HSUB2/HMUL2, STS): 16 warps (two threads per tile column, each
// half of the K block's packed rows) give every scheduler four warps of
// independent chains (measured with 8 warps: 44 % issue-active, the top
// stall a fixed-latency dependency).
#ifndef QX_GEMM_DQ_WARPS
#define QX_GEMM_DQ_WARPS 16
#endif
constexpr int DQ_WARPS = QX_GEMM_DQ_WARPS;
constexpr int DQ_PARTS = DQ_WARPS / 8;           // threads per tile column
constexpr int THREADS = 64 + DQ_WARPS * 32;      // warp 0 TMA, warp 1 MMA, warps 2.. dequant + epilogue
static_assert(DQ_WARPS == 8 || DQ_WARPS == 16, "8 or 16 dequant warps");
constexpr int A_BYTES = BM * BK * 2;   // 16 KB
constexpr int BF_BYTES = BN * BK * 2;  // 32 KB
constexpr int WQ_BYTES = 8 * BN * 4;   // 8 KB
constexpr int SZ_BYTES = 2048;         // scales + zeros of up to 2 groups
constexpr int MAX_RANK = 64;

// shared-memory carve-up (bytes from a 1024-aligned base)
constexpr int OFF_A = 0;                            // x tiles [XS]
constexpr int OFF_BF = OFF_A + XS * A_BYTES;        // dequantised B [BS]
constexpr int OFF_LH = OFF_BF + BS * BF_BYTES;      // LoRA h (hi | lo), 2 x 16 KB
constexpr int OFF_WQ = OFF_LH + 2 * A_BYTES;        // packed weights [WS]
constexpr int OFF_SZ = OFF_WQ + WS * WQ_BYTES;      // scales + zero points [WS]
constexpr int OFF_BAR = OFF_SZ + WS * SZ_BYTES;
// full_x, empty_x [XS], full_w, empty_w [WS], full_b, empty_b [BS], tmem_full, lora
constexpr int NBARS = 2 * (XS + WS + BS) + 2;
constexpr int OFF_TMEM = OFF_BAR + NBARS * 8;
constexpr int SMEM_BYTES = OFF_TMEM + 16 + 1024;  // + alignment slack
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory of the GEMM rings");
static_assert(OFF_BF % 1024 == 0 && OFF_LH % 1024 == 0, "128B-swizzled operands on 1 KB boundaries");

struct alignas(64) GemmParams {
  CUtensorMap tx;  // x fp16 [M][K], box {64, 128}, 128B swizzle
  CUtensorMap tw;  // qweight u64 [K/8][N/2], box {128, 8}
  CUtensorMap ts;  // scales fp16 [K/g][N], box {256, grows}
  CUtensorMap tz;  // zeros: packed u32 [K/g][N/8] box {32, grows}, or fp16 [K/g][N] box {256, grows}
  CUtensorMap th;  // (alpha/r) h, fp16 high then low parts, [2M][64], box {64, 128}, 128B swizzle
  CUtensorMap tb;  // LoRA B fp16 [r][N], box {256, kp}
  __half* y;
  int M, K, N, rank, group, zeros_packed, zero_offset, grows;
};

// Sticky device-side error word of this file's kernels (QX_DEVERR_* bits),
// merged into qx_get_device_error.
static __device__ unsigned g_gemm_error = 0;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void bar_init(uint32_t b, uint32_t n) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(b), "r"(n) : "memory");
}
__device__ __forceinline__ void bar_arrive(uint32_t b) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(b) : "memory");
}
__device__ __forceinline__ void bar_expect(uint32_t b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(b),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool bar_try(uint32_t b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred P; mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 P, [%1], %2; "
      "selp.u32 %0, 1, 0, P; }"
      : "=r"(ok)
      : "r"(b), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void bar_wait(uint32_t b, uint32_t parity) {
  if (bar_try(b, parity)) return;
  uint64_t t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  while (!bar_try(b, parity)) {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (t - t0 > kWaitLimitNs) {
      atomicOr(&g_gemm_error, QX_DEVERR_MBAR_TIMEOUT);
      return;
    }
  }
}
__device__ __forceinline__ void tma2d(uint32_t dst, const CUtensorMap* m, int x, int y, uint32_t b) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(b)
      : "memory");
}
__device__ __forceinline__ void tma2d_ef(uint32_t dst, const CUtensorMap* m, int x, int y,
                                         uint32_t b) {  // weights: L2 evict-first
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(b), "l"(pol)
      : "memory");
}

// K-major operand with 128-byte swizzle: rows of 128 B, 8-row atoms 1024 B apart
// (SBO), LBO unused (1), descriptor version 1, layout type 2.
__device__ __forceinline__ uint64_t kmajor_sw128_desc(uint32_t saddr) {
  return uint64_t((saddr >> 4) & 0x3FFF) | (uint64_t(1) << 16) | (uint64_t(64) << 32) |
         (uint64_t(1) << 46) | (uint64_t(2) << 61);
}
// kind::f16 instruction descriptor: D f32, A/B f16, both K-major, N=256, M=128
constexpr uint32_t IDESC = (1u << 4) | (uint32_t(BN >> 3) << 17) | (uint32_t(BM >> 4) << 24);

__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t acc,
                                     uint32_t idesc = IDESC) {  // one thread issues
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t b) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(b)
      : "memory");
}

// byte i of v holds (q_2i | q_2i+1 << 4): half2 (q_2i - z, q_2i+1 - z) * s
__device__ __forceinline__ uint32_t dq_pair(uint32_t v, uint32_t sel, uint32_t zz, uint32_t ss) {
  uint32_t r = prmt(v, 0u, sel);
  r = lop3_and_or(r, 0x00F0000Fu, 0x54006400u);  // (1024 + q_2i, 64 + q_2i+1)
  r = hsub2_u32(r, zz);                           // exact: (q - z) in [-16, 15]
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(r), "r"(ss));
  return d;
}

__global__ void __launch_bounds__(THREADS, 1) w4a16_gemm_kernel(const __grid_constant__ GemmParams p) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
  const int KB = p.K / BK;
  const int R = p.rank;
  const int lora_items = R > 0 ? 1 : 0;

  const uint32_t sb = smem_u32(smem);
  const uint32_t full_x = sb + OFF_BAR, empty_x = full_x + 8 * XS;
  const uint32_t full_w = empty_x + 8 * XS, empty_w = full_w + 8 * WS;
  const uint32_t full_b = empty_w + 8 * WS, empty_b = full_b + 8 * BS;
  const uint32_t tmem_full = empty_b + 8 * BS;
  const uint32_t lora_full = tmem_full + 8;
  const int kp = ((R + 15) / 16) * 16;  // LoRA K extent of the MMAs
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_TMEM);

  if (warp == 0 && lane == 0) {
    for (int i = 0; i < XS; ++i) {
      bar_init(full_x + 8 * i, 1);
      bar_init(empty_x + 8 * i, 1);  // MMA commit
    }
    for (int i = 0; i < WS; ++i) {
      bar_init(full_w + 8 * i, 1);
      bar_init(empty_w + 8 * i, DQ_WARPS);  // the dequant warps have read the stage
    }
    for (int i = 0; i < BS; ++i) {
      bar_init(full_b + 8 * i, DQ_WARPS);
      bar_init(empty_b + 8 * i, 1);
    }
    bar_init(tmem_full, 1);
    bar_init(lora_full, 1);
    asm volatile("fence.mbarrier_init.release.cluster;\nfence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {  // 256 TMEM columns: the 128 x 256 fp32 accumulator
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(256)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  const int w_bytes = WQ_BYTES + p.grows * BN * 2 + p.grows * (p.zeros_packed ? BN / 2 : BN * 2);

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producers
    if (lane == 0) {  // packed weights, scales and zero points (released by the dequant warps)
      for (int kb = 0; kb < KB; ++kb) {
        const int s = kb % WS;
        if (kb >= WS) bar_wait(empty_w + 8 * s, ((kb / WS) - 1) & 1);
        bar_expect(full_w + 8 * s, uint32_t(w_bytes));
        tma2d_ef(sb + OFF_WQ + s * WQ_BYTES, &p.tw, n0 / 2, kb * 8, full_w + 8 * s);
        const int grow = (kb * BK) / p.group;
        unsigned char* sz = smem + OFF_SZ + s * SZ_BYTES;
        tma2d(smem_u32(sz), &p.ts, n0, grow, full_w + 8 * s);
        tma2d(smem_u32(sz + 1024), &p.tz, p.zeros_packed ? n0 / 8 : n0, grow, full_w + 8 * s);
      }
    } else if (lane == 1) {  // the LoRA tiles, then the x tiles (released by the MMA)
      if (lora_items) {  // (alpha/r) h hi / lo tiles; the LoRA B tile [kp][256] (raw) into B slot 1
        bar_expect(lora_full, uint32_t(2 * A_BYTES + kp * BN * 2));
        tma2d(sb + OFF_LH, &p.th, 0, m0, lora_full);
        tma2d(sb + OFF_LH + A_BYTES, &p.th, 0, p.M + m0, lora_full);
        tma2d(sb + OFF_BF + BF_BYTES, &p.tb, n0, 0, lora_full);
      }
      for (int kb = 0; kb < KB; ++kb) {
        const int s = kb % XS;
        if (kb >= XS) bar_wait(empty_x + 8 * s, ((kb / XS) - 1) & 1);
        bar_expect(full_x + 8 * s, uint32_t(A_BYTES));
        tma2d(sb + OFF_A + s * A_BYTES, &p.tx, kb * BK, m0, full_x + 8 * s);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      if (lora_items) {  // accumulator = (alpha/r) h B first (hi and lo parts)
        bar_wait(lora_full, 0);
        bar_wait(full_b, 0);  // the transposed B tile
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        for (int part = 0; part < 2; ++part)
          for (int k = 0; k < kp / 16; ++k)
            umma(tmem, kmajor_sw128_desc(sb + OFF_LH + part * A_BYTES + k * 32),
                 kmajor_sw128_desc(sb + OFF_BF + k * 32), (part | k) != 0);
        umma_commit(empty_b);
      }
      for (int kb = 0; kb < KB; ++kb) {
        const int s = kb % XS, i = kb + lora_items, t = i % BS;
        bar_wait(full_x + 8 * s, (kb / XS) & 1);
        bar_wait(full_b + 8 * t, (i / BS) & 1);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
        for (int k = 0; k < BK / 16; ++k)
          umma(tmem, kmajor_sw128_desc(sb + OFF_A + s * A_BYTES + k * 32),
               kmajor_sw128_desc(sb + OFF_BF + t * BF_BYTES + k * 32),
               (lora_items | kb | k) != 0);
        umma_commit(empty_b + 8 * t);
        umma_commit(empty_x + 8 * s);
      }
      umma_commit(tmem_full);
    }
  } else {
    // ------------------------------------------------------------ dequant warps
    const int dt = (tid - 64) & (BN - 1);  // the tile column this thread dequantises
    const int part = (tid - 64) >> 8;       // which packed rows of the K block: [part * PPR, + PPR)
    constexpr int PPR = 8 / DQ_PARTS;
    if (lora_items) {  // transpose the raw LoRA B tile (ring slot 1) into K-major ring slot 0
      if (lane == 0) bar_wait(lora_full, 0);
      __syncwarp();
      bar_wait(lora_full, 0);
      const __half* braw = reinterpret_cast<const __half*>(smem + OFF_BF + BF_BYTES);
      unsigned char* bf = smem + OFF_BF;
      const int nch = kp / 8 / DQ_PARTS;  // 16-byte chunks of the column per thread
      for (int ch = part * nch; ch < (part + 1) * nch; ++ch) {
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e)
          w[e] = uint32_t(__half_as_ushort(braw[(ch * 8 + 2 * e) * BN + dt])) |
                 (uint32_t(__half_as_ushort(braw[(ch * 8 + 2 * e + 1) * BN + dt])) << 16);
        *reinterpret_cast<uint4*>(bf + dt * 128 + ((ch ^ (dt & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      asm volatile("bar.sync 1, %0;" ::"n"(DQ_WARPS * 32) : "memory");  // every warp is done reading slot 1
      if (lane == 0) bar_arrive(full_b);
    }
    for (int kb = 0; kb < KB; ++kb) {
      const int s = kb % WS, i = kb + lora_items, t = i % BS;
      if (i >= BS) bar_wait(empty_b + 8 * t, ((i / BS) - 1) & 1);
      bar_wait(full_w + 8 * s, (kb / WS) & 1);
      const uint32_t* wq = reinterpret_cast<const uint32_t*>(smem + OFF_WQ + s * WQ_BYTES);
      const unsigned char* sz = smem + OFF_SZ + s * SZ_BYTES;
      unsigned char* bf = smem + OFF_BF + t * BF_BYTES;
      uint32_t zz[2], ss[2];
#pragma unroll
      for (int gl = 0; gl < 2; ++gl) {
        if (gl < p.grows) {
          const __half sc = reinterpret_cast<const __half*>(sz)[gl * BN + dt];
          float z;
          if (p.zeros_packed)
            z = float(((reinterpret_cast<const uint32_t*>(sz + 1024)[gl * (BN / 8) + (dt >> 3)] >>
                        (4 * (dt & 7))) & 0xFu) + unsigned(p.zero_offset));
          else
            z = __half2float(reinterpret_cast<const __half*>(sz + 1024)[gl * BN + dt]);
          const __half2 z2 = __floats2half2_rn(1024.f + z, 64.f + z);
          zz[gl] = *reinterpret_cast<const uint32_t*>(&z2);
          const __half2 s2 = __halves2half2(sc, sc);
          ss[gl] = *reinterpret_cast<const uint32_t*>(&s2);
        }
      }
      if (p.zeros_packed) {  // integer zero points: exact half2 arithmetic
#pragma unroll
        for (int r = 0; r < PPR; ++r) {
          const int pr = part * PPR + r;
          const uint32_t v = wq[pr * BN + dt];
          const int gl = p.grows > 1 ? (pr * 8) / p.group : 0;  // groups of 32: two per K block
          const uint32_t z2 = gl ? zz[1] : zz[0], s2 = gl ? ss[1] : ss[0];
          const uint4 o = make_uint4(dq_pair(v, 0x0000u, z2, s2), dq_pair(v, 0x1111u, z2, s2),
                                     dq_pair(v, 0x2222u, z2, s2), dq_pair(v, 0x3333u, z2, s2));
          *reinterpret_cast<uint4*>(bf + dt * 128 + ((pr ^ (dt & 7)) << 4)) = o;
        }
      } else {  // fp16 zero points may be fractional: fp16((q - z) * s) in fp32, as the oracle
        for (int r = 0; r < PPR; ++r) {
          const int pr = part * PPR + r;
          const uint32_t v = wq[pr * BN + dt];
          const int gl = p.grows > 1 ? (pr * 8) / p.group : 0;
          const float sf = __half2float(reinterpret_cast<const __half*>(sz)[gl * BN + dt]);
          const float zf = __half2float(reinterpret_cast<const __half*>(sz + 1024)[gl * BN + dt]);
          uint32_t o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float w0 = (float((v >> (8 * e)) & 0xFu) - zf) * sf;
            const float w1 = (float((v >> (8 * e + 4)) & 0xFu) - zf) * sf;
            const __half2 hv = __floats2half2_rn(w0, w1);
            o[e] = *reinterpret_cast<const uint32_t*>(&hv);
          }
          *reinterpret_cast<uint4*>(bf + dt * 128 + ((pr ^ (dt & 7)) << 4)) =
              make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) {
        bar_arrive(full_b + 8 * t);
        bar_arrive(empty_w + 8 * s);
      }
    }
    // ------------------------------------------------------------ epilogue
    if (lane == 0) bar_wait(tmem_full, 0);
    __syncwarp();
    bar_wait(tmem_full, 0);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    constexpr int CW = BN / (DQ_WARPS / 4);  // columns per warp
    const int q = warp & 3, cpart = (warp - 2) >> 2;  // TMEM lane quarter, column block
    const int row = q * 32 + lane, m = m0 + row;
    for (int cb = 0; cb < CW / 32; ++cb) {
      const int col = cpart * CW + cb * 32;
      uint32_t r[32];
      const uint32_t taddr = tmem + (uint32_t(q * 32) << 16) + uint32_t(col);
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
          "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
          : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
            "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
            "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
            "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
            "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
          : "r"(taddr));
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      if (m < p.M) {
        uint4* dst = reinterpret_cast<uint4*>(p.y + size_t(m) * p.N + n0 + col);
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          uint32_t o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const __half2 hv = __floats2half2_rn(__uint_as_float(r[v * 8 + 2 * e]),
                                                 __uint_as_float(r[v * 8 + 2 * e + 1]));
            o[e] = *reinterpret_cast<const uint32_t*>(&hv);
          }
          dst[v] = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256)
                 : "memory");
  }
}

// (alpha/r) h = (alpha/r) x[M][K] . A[K][r] in fp32, split over K so that the
// grid covers the GPU: CTA (128-row block, K slice) runs 8 warps of mma.sync
// m16n8k16 (16 rows each, one accumulator per 8 ranks) over 32-wide k steps
// whose x and A tiles are double-buffered by cp.async; fp32 partials go to
// part[split][M][64].  A second kernel sums the splits in order and writes the
// scaled result as fp16 high parts hl[m][0..63] and low parts hl[M + m][0..63]
// (ranks r..63 zero), the tiles the GEMM's LoRA MMAs read.
constexpr int LS_ROWS = 128, LS_K = 32, LS_THREADS = 256;
constexpr int LS_STAGES = 3;  // x / A tiles in flight per CTA (two steps ahead of the MMAs)

__host__ __device__ inline int lora_splits(int M) {  // K splits: about two CTAs per SM of 148
  const int rb = (M + LS_ROWS - 1) / LS_ROWS;
  const int ks = (2 * 148 + rb - 1) / rb;
  return ks < 1 ? 1 : (ks > 64 ? 64 : ks);
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(src_bytes)
               : "memory");
}

__global__ void __launch_bounds__(LS_THREADS) lora_down_split_kernel(const __half* __restrict__ x,
                                                                     const __half* __restrict__ A,
                                                                     float* __restrict__ part, int M,
                                                                     int K, int R, int kchunk) {
  __shared__ __align__(128) __half xs[LS_STAGES][LS_ROWS][LS_K + 8];
  __shared__ __align__(128) __half as[LS_STAGES][LS_K][MAX_RANK + 8];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int r0 = blockIdx.x * LS_ROWS;
  const int k0 = blockIdx.y * kchunk, k1 = min(K, k0 + kchunk);
  const int nsteps = (k1 - k0) / LS_K;
  const int NT = R / 8;
  float acc[MAX_RANK / 8][4];
#pragma unroll
  for (int i = 0; i < MAX_RANK / 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  auto load = [&](int step, int buf) {
    const int kb = k0 + step * LS_K;
    for (int it = tid; it < LS_ROWS * (LS_K / 8); it += LS_THREADS) {
      const int rr = it >> 2, ch = it & 3, row = r0 + rr;  // rows past M are zero-filled
      cp_async16(&xs[buf][rr][ch * 8], x + size_t(row < M ? row : 0) * K + kb + ch * 8, row < M ? 16 : 0);
    }
    for (int it = tid; it < LS_K * NT; it += LS_THREADS) {
      const int kk = it / NT, ch = it - kk * NT;
      cp_async16(&as[buf][kk][ch * 8], A + size_t(kb + kk) * R + ch * 8, 16);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  // LS_STAGES - 1 steps in flight ahead of the one computed (an empty commit
  // group where no step is left, so the wait count stays fixed)
#pragma unroll
  for (int sp = 0; sp < LS_STAGES - 1; ++sp) {
    if (sp < nsteps) load(sp, sp);
    else asm volatile("cp.async.commit_group;" ::: "memory");
  }
  for (int st = 0; st < nsteps; ++st) {
    const int nx = st + LS_STAGES - 1;
    if (nx < nsteps) load(nx, nx % LS_STAGES);
    else asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("cp.async.wait_group %0;" ::"n"(LS_STAGES - 1) : "memory");  // step st landed
    __syncthreads();
    const int b = st % LS_STAGES;
#pragma unroll
    for (int kk = 0; kk < LS_K; kk += 16) {
      uint32_t a[4];
      {
        const unsigned sa = smem_u32(&xs[b][warp * 16 + (lane & 15)][kk + 8 * (lane >> 4)]);
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                     : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3])
                     : "r"(sa));
      }
#pragma unroll
      for (int nt = 0; nt < MAX_RANK / 8; ++nt) {
        if (nt < NT) {
          uint32_t bb[2];
          const unsigned sb2 = smem_u32(&as[b][kk + (lane & 15)][nt * 8]);
          asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];"
                       : "=r"(bb[0]), "=r"(bb[1])
                       : "r"(sb2));
          mma_16816(acc[nt], a[0], a[1], a[2], a[3], bb[0], bb[1]);
        }
      }
    }
    __syncthreads();  // the next load overwrites this buffer
  }
  float* dst = part + size_t(blockIdx.y) * M * MAX_RANK;
#pragma unroll
  for (int nt = 0; nt < MAX_RANK / 8; ++nt) {
    const bool v = nt < NT;
    const int row = r0 + warp * 16 + g, col = nt * 8 + 2 * c;
    if (row < M)
      *reinterpret_cast<float2*>(dst + size_t(row) * MAX_RANK + col) =
          make_float2(v ? acc[nt][0] : 0.f, v ? acc[nt][1] : 0.f);
    if (row + 8 < M)
      *reinterpret_cast<float2*>(dst + size_t(row + 8) * MAX_RANK + col) =
          make_float2(v ? acc[nt][2] : 0.f, v ? acc[nt][3] : 0.f);
  }
}

__global__ void __launch_bounds__(256) lora_down_finalize_kernel(const float* __restrict__ part,
                                                                 __half* __restrict__ hl, int M,
                                                                 int splits, float scale) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;  // (row, column pair)
  if (i >= M * (MAX_RANK / 2)) return;
  const int row = i / (MAX_RANK / 2), col = (i - row * (MAX_RANK / 2)) * 2;
  float v0 = 0.f, v1 = 0.f;
  for (int sp = 0; sp < splits; ++sp) {  // in split order: deterministic
    const float2 pv = *reinterpret_cast<const float2*>(part + (size_t(sp) * M + row) * MAX_RANK + col);
    v0 += pv.x;
    v1 += pv.y;
  }
  const __half2 hi = __floats2half2_rn(scale * v0, scale * v1);
  const float2 hr = __half22float2(hi);
  const __half2 lo = __floats2half2_rn(scale * v0 - hr.x, scale * v1 - hr.y);
  *reinterpret_cast<__half2*>(hl + size_t(row) * MAX_RANK + col) = hi;
  *reinterpret_cast<__half2*>(hl + (size_t(M) + row) * MAX_RANK + col) = lo;
}

static PFN_cuTensorMapEncodeTiled_v12000 encoder() {
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

static int encode(CUtensorMap* map, CUtensorMapDataType type, const void* base, uint64_t cols,
                  uint64_t rows, uint64_t stride, uint32_t bc, uint32_t br, CUtensorMapSwizzle sw,
                  const char* what) {
  const auto enc = encoder();
  if (!enc) return fail(QX_ERR_CUDA, "w4a16_gemm: cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {stride};
  const cuuint32_t box[2] = {bc, br};
  const cuuint32_t es[2] = {1, 1};
  const CUresult r = enc(map, type, 2, const_cast<void*>(base), dims, strides, box, es,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(QX_ERR_CUDA, "w4a16_gemm: tensor map for %s (CUresult %d)", what, int(r));
  return QX_OK;
}

}  // namespace gemm

int gemm_device_error(unsigned* code, int reset) {
  QX_CUDA_TRY(cudaMemcpyFromSymbol(code, gemm::g_gemm_error, sizeof(unsigned)), "get_device_error: read");
  if (reset) {
    const unsigned zero = 0;
    QX_CUDA_TRY(cudaMemcpyToSymbol(gemm::g_gemm_error, &zero, sizeof(unsigned)), "get_device_error: reset");
  }
  return QX_OK;
}

}  // namespace qx

using namespace qx;

extern "C" size_t qx_w4a16_lora_gemm_sm100_workspace_size(int M, int rank) {
  // (alpha/r) h as fp16 high and low parts [2M][64], then the fp32 partial sums
  // of the K splits [splits][M][64]
  if (rank <= 0 || M <= 0) return 0;
  return size_t(2) * size_t(M) * gemm::MAX_RANK * 2 +
         size_t(gemm::lora_splits(M)) * size_t(M) * gemm::MAX_RANK * 4;
}

extern "C" int qx_w4a16_lora_gemm_sm100(const void* x, const int32_t* qweight, const void* scales,
                                        const void* zeros, int zeros_packed, int zero_offset,
                                        const void* lora_A, const void* lora_B, void* y, int M, int K,
                                        int N, int rank, int group_size, float lora_scale,
                                        void* workspace, size_t workspace_bytes, qx_stream_t stream) {
  using namespace gemm;
  QX_REQUIRE(M > 0 && K > 0 && N > 0, "w4a16_gemm: bad sizes M=%d K=%d N=%d", M, K, N);
  QX_REQUIRE(N % BN == 0, "w4a16_gemm: N=%d must be a multiple of %d", N, BN);
  QX_REQUIRE(K % BK == 0, "w4a16_gemm: K=%d must be a multiple of %d", K, BK);
  QX_REQUIRE((group_size == 32 || group_size == 64 || group_size == 128 || group_size == 256) &&
                 K % group_size == 0,
             "w4a16_gemm: group_size=%d must be 32, 64, 128 or 256 and divide K=%d", group_size, K);
  QX_REQUIRE(rank == 0 || rank == 8 || rank == 16 || rank == 32 || rank == 48 || rank == 64,
             "w4a16_gemm: LoRA rank %d unsupported (0, 8, 16, 32, 48 or 64)", rank);
  QX_REQUIRE(x && qweight && scales && zeros && y, "w4a16_gemm: null tensor pointer");
  QX_REQUIRE(rank == 0 || (lora_A && lora_B), "w4a16_gemm: rank=%d but lora_A/lora_B missing", rank);
  QX_REQUIRE(aligned(x, 16) && aligned(qweight, 16) && aligned(scales, 16) && aligned(zeros, 16) &&
                 aligned(y, 16) && (rank == 0 || (aligned(lora_A, 16) && aligned(lora_B, 16))),
             "w4a16_gemm: every tensor must be 16-byte aligned");
  QX_REQUIRE(zeros_packed == 0 || zeros_packed == 1, "w4a16_gemm: zeros_packed must be 0 or 1");
  const size_t need = qx_w4a16_lora_gemm_sm100_workspace_size(M, rank);
  QX_REQUIRE(workspace_bytes >= need && (need == 0 || (workspace && aligned(workspace, 16))),
             "w4a16_gemm: workspace of %zu bytes needed, %zu given", need, workspace_bytes);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);

  GemmParams prm{};
  const int grows = group_size >= BK ? 1 : BK / group_size;
  const uint64_t G = uint64_t(K / group_size);
  int rc = encode(&prm.tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, x, uint64_t(K), uint64_t(M),
                  uint64_t(K) * 2, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B, "x");
  if (rc == QX_OK)
    rc = encode(&prm.tw, CU_TENSOR_MAP_DATA_TYPE_UINT64, qweight, uint64_t(N) / 2, uint64_t(K) / 8,
                uint64_t(N) * 4, BN / 2, 8, CU_TENSOR_MAP_SWIZZLE_NONE, "qweight");
  if (rc == QX_OK)
    rc = encode(&prm.ts, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, scales, uint64_t(N), G, uint64_t(N) * 2, BN,
                uint32_t(grows), CU_TENSOR_MAP_SWIZZLE_NONE, "scales");
  if (rc == QX_OK) {
    if (zeros_packed)
      rc = encode(&prm.tz, CU_TENSOR_MAP_DATA_TYPE_INT32, zeros, uint64_t(N) / 8, G, uint64_t(N) / 2,
                  BN / 8, uint32_t(grows), CU_TENSOR_MAP_SWIZZLE_NONE, "qzeros");
    else
      rc = encode(&prm.tz, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, zeros, uint64_t(N), G, uint64_t(N) * 2, BN,
                  uint32_t(grows), CU_TENSOR_MAP_SWIZZLE_NONE, "zeros");
  }
  if (rc != QX_OK) return rc;
  if (rank > 0) {
    const int kp = ((rank + 15) / 16) * 16;
    rc = encode(&prm.th, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, workspace, uint64_t(MAX_RANK),
                uint64_t(2) * uint64_t(M), uint64_t(MAX_RANK) * 2, MAX_RANK, BM,
                CU_TENSOR_MAP_SWIZZLE_128B, "lora h");
    if (rc == QX_OK)
      rc = encode(&prm.tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, lora_B, uint64_t(N), uint64_t(rank),
                  uint64_t(N) * 2, BN, uint32_t(kp), CU_TENSOR_MAP_SWIZZLE_NONE, "lora_B");
    if (rc != QX_OK) return rc;
  }
  prm.y = static_cast<__half*>(y);
  prm.M = M;
  prm.K = K;
  prm.N = N;
  prm.rank = rank;
  prm.group = group_size;
  prm.zeros_packed = zeros_packed;
  prm.zero_offset = zero_offset;
  prm.grows = grows;

  static std::once_flag attr_once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(attr_once, [] {
    attr_err = cudaFuncSetAttribute(w4a16_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    SMEM_BYTES);
  });
  QX_CUDA_TRY(attr_err, "w4a16_gemm: set smem limit");

  if (rank > 0) {
    // K slices of whole 32-wide steps, at most lora_splits(M) of them (the workspace size)
    const int ks_max = lora_splits(M);
    const int kchunk = ((K + ks_max - 1) / ks_max + LS_K - 1) / LS_K * LS_K;
    const int splits = (K + kchunk - 1) / kchunk;
    __half* hl = static_cast<__half*>(workspace);
    float* part = reinterpret_cast<float*>(static_cast<char*>(workspace) + size_t(2) * M * MAX_RANK * 2);
    lora_down_split_kernel<<<dim3((M + LS_ROWS - 1) / LS_ROWS, splits), LS_THREADS, 0, st>>>(
        static_cast<const __half*>(x), static_cast<const __half*>(lora_A), part, M, K, rank, kchunk);
    QX_CUDA_TRY(cudaGetLastError(), "w4a16_gemm: lora_down launch");
    lora_down_finalize_kernel<<<(M * (MAX_RANK / 2) + 255) / 256, 256, 0, st>>>(part, hl, M, splits,
                                                                             lora_scale);
    QX_CUDA_TRY(cudaGetLastError(), "w4a16_gemm: lora_down finalize launch");
  }
  dim3 grid(N / BN, (M + BM - 1) / BM);
  w4a16_gemm_kernel<<<grid, THREADS, SMEM_BYTES, st>>>(prm);
  return check_launch("w4a16_gemm");
}
