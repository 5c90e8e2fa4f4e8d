// GQA decode attention read in place from the StreamingLLM ring (sm_100a).
//
// New component: the reference has no attention kernel; it only materialises
// K/V in logical order (get_kv, csrc/kv_cache/ring_buffer.cu:143-200) for an
// external attention.  Softmax is order-independent, and the valid slots of
// the ring are always the physical prefix [0, valid_length(count)) (sinks
// fill 0..S-1, the window fills S..S+W-1 in order before it wraps), so this
// kernel streams that prefix directly: no index list, no gather copy.
//
// Math (HF Qwen3 eager attention, transformers models/qwen3/modeling_qwen3.py:
// repeat_kv + softmax(q k^T / sqrt(D)) v):  query head h reads KV head
// h / (Hq / Hkv).  The G = Hq / Hkv query heads of one KV head are the 16
// rows of an mma.sync m16n8k16 tile (rows >= G are zero padding), so every K/V
// byte is read once per (sequence, KV head).
//
// Work decomposition (flash-decoding): grid = (chunks, batch * Hkv); a CTA
// (4 warps) owns a chunk of slots, each warp takes 16-slot tiles staged by
// cp.async into XOR-swizzled shared memory (double buffered), computes
// S = Q K^T and O += P V on the tensor cores with an online softmax in fp32,
// the warps merge in shared memory.  The chunks of one (sequence, KV head) are
// then merged one of two ways:
//  * cluster merge (when a sequence's slots are split into 2..16 chunks): the
//    chunk CTAs form one thread-block cluster; each CTA owns a slice of the
//    output and every chunk pushes its (max, sum) rows and O elements for that
//    slice into the owner's shared memory with st.async (completion counted
//    in bytes on the owner's mbarrier, a bounded wait), so no CTA reads a
//    peer and there is no cluster barrier after the tile loop;
//  * global merge (more chunks, or the cluster form pinned off): each CTA
//    writes (max, sum, O) to the workspace and the last CTA of the
//    (sequence, KV head), found with an atomic counter, merges them.
// Both merges sum the chunks in a fixed order (deterministic).
#include <algorithm>
#include <atomic>
#include <cmath>
#include <mutex>

#include "qx_b200.h"
#include "qx_common.cuh"

namespace qx {
namespace attn {

constexpr int D = 128;
constexpr int WARPS = 4;
constexpr int THREADS = WARPS * 32;
constexpr int TILE = 16;
constexpr int ROW_BYTES = D * 2;                 // 256
constexpr int TILE_BYTES = TILE * ROW_BYTES;     // 4 KB
constexpr int WARP_SMEM = 2 * 2 * TILE_BYTES;    // 2 stages x (K, V)
constexpr int SMEM = WARPS * WARP_SMEM;          // 64 KB
constexpr int CHUNK_ALIGN = WARPS * TILE;        // 64 slots: every warp has a tile (16-slot chunks,
                                                 // 52 per head at one sequence, measured slower:
                                                 // 15.7 vs 11.1 us, tiny CTAs and a longer merge)
constexpr int CTAS_PER_SM = 3;
constexpr int PSTRIDE = D + 4;                   // floats per (row) partial: m, l, pad, pad, O[D]
constexpr int COUNTER_SLOTS = 4096;              // fixed counter region at the workspace start
constexpr int MAX_CHUNKS = 64;                   // bounds the merge's shared memory
constexpr int MAX_CLUSTER = 16;                  // chunks merged through distributed shared memory
constexpr int OSTRIDE = D + 8;                   // floats per row of the warp merge (conflict-free float2 stores)
constexpr int QS_BYTES = 16 * D * 2;             // fused form: the G <= 16 rotated query heads
// deep form: 4 tile stages per warp (every tile of a 256-slot chunk in flight at
// once), for grids of at most one CTA per SM
constexpr int SMEM4 = 2 * SMEM;
// cluster merge: every chunk CTA pushes its (max, sum) rows and O vectors into
// the owners' receive areas (O [nch][per][4] floats, then (max, sum) [nch][RMAX]
// rows), past the tiles and the fused q heads: at most (G D / 4 + nch) O
// vectors and nch (per / 32 + 2) rows for G <= 16, nch <= 16
constexpr int RECV_BYTES = 9216;
__host__ __device__ constexpr int smem_bytes(int nb, bool fused, bool cluster = false) {
  return (nb == 4 ? SMEM4 : SMEM) + (fused ? QS_BYTES : 0) + (cluster ? RECV_BYTES : 0);
}
static_assert(THREADS == D, "one thread per head dimension in the merges");
static_assert(WARPS == 4, "the chunk merge interleaves 4 chunk subsets, one per warp");
static_assert(2 * 16 * MAX_CHUNKS * 4 + 32 * 4 + 4 * 16 * D * 4 <= SMEM, "merge fits the tile smem");

// Sticky device-side error word of this file's kernel (QX_DEVERR_* bits),
// merged into qx_get_device_error.
static __device__ unsigned g_attn_error = 0;

struct Params {
  const __half* q;
  const __half* k;
  const __half* v;
  __half* out;
  int Hq, Hkv, G, cap, valid, chunk, nch;
  float scale_log2;
  float* part;          // [B*Hkv][nch][G][PSTRIDE], O 16-byte aligned
  unsigned* counters;   // [B*Hkv]
  int early;            // launched early: the K/V tiles of the first two rounds load before the
                        // dependency wait, and slot `fresh` (the one the previous kernel wrote,
                        // or this kernel's own append) is reloaded after it
  int fresh;
  // fused q/k head norm + RoPE + ring append (qkv: the fused projection
  // output [B][(Hq + 2 Hkv) D]; k / v of the new token go to slot `fresh`)
  int fused;
  const __half* qkv;
  const __half* qnw;
  const __half* knw;
  const float* cosr;
  const float* sinr;
  float eps;
  unsigned long long* trace;  // profiling build only (qx_trace_launches): phase timestamps
  int trace_launch;
};

// Trace slots of an attention CTA (profiling build): 0 entry, 1 dependency
// wait passed, 2 first K/V tile landed, 3 tile loop done, 4 warps merged,
// 5 chunk barrier passed (cluster merge), 6 exit
enum AttnTrace { TR_ENTRY, TR_WAITED, TR_TILE0, TR_LOOP, TR_WARP_MERGE, TR_CHUNK_SYNC, TR_EXIT };

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(src_bytes));
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
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
// byte offset of 16-byte chunk `ch` of tile row `r` (XOR swizzle: conflict-free ldmatrix)
__device__ __forceinline__ uint32_t swz(int r, int ch) {
  return uint32_t(r * ROW_BYTES + ((ch ^ (r & 7)) << 4));
}

__device__ __forceinline__ uint32_t cluster_map(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_async_f32(uint32_t raddr, float a, uint32_t rbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(raddr),
               "r"(__float_as_uint(a)), "r"(rbar)
               : "memory");
}
__device__ __forceinline__ void st_async_f2(uint32_t raddr, float a, float b, uint32_t rbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];" ::"r"(
                   raddr),
               "f"(a), "f"(b), "r"(rbar)
               : "memory");
}
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

// CLUSTER: the grid's x extent (the chunks of one sequence and KV head) is one
// thread-block cluster and the chunks are merged through distributed shared
// memory; otherwise through the workspace by the last CTA.
// NB: K/V tile stages per warp (2, or 4 for grids of at most one CTA per SM)
template <bool CLUSTER, int NB>
__global__ void __launch_bounds__(THREADS) decode_attn_kernel(const Params p) {
  pdl_trigger();
  unsigned long long* const trc = trace_base(p.trace, p.trace_launch);
  trace_stamp(trc, TR_ENTRY, threadIdx.x == 0);
  if (!p.early) pdl_wait();  // no-op unless launched with programmatic dependent launch
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ unsigned s_is_last;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int bh = blockIdx.y, ci = blockIdx.x;
  const int b = bh / p.Hkv, kvh = bh - b * p.Hkv;
  const int c0 = ci * p.chunk;
  const int c1 = min(p.valid, c0 + p.chunk);
  const int ntiles = (c1 - c0 + TILE - 1) / TILE;

  // cluster merge: this CTA owns output vectors [ci per, ci per + own_v) of the
  // G x D block; its receive barrier expects every chunk's share of them
  __shared__ __align__(8) unsigned long long s_rbar;
  const int per = (p.G * (D / 4) + p.nch - 1) / p.nch;
  const int rmax = per / (D / 4) + 2;
  if constexpr (CLUSTER) {
    if (tid == 0) {
      const int own_v = max(0, min(per, p.G * (D / 4) - ci * per));
      const int own_r = own_v ? (ci * per + own_v - 1) / (D / 4) - (ci * per) / (D / 4) + 1 : 0;
      const uint32_t rb = smem_u32(&s_rbar);
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(rb) : "memory");
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
      asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(rb),
                   "r"(uint32_t(p.nch * (own_v * 16 + own_r * 8)))
                   : "memory");
    }
    __syncthreads();
    // peers push only after every CTA of the cluster initialised its barrier
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
  }

  const size_t slot_stride = size_t(p.Hkv) * D;  // halves between consecutive slots
  const __half* kb = p.k + (size_t(b) * p.cap * p.Hkv + kvh) * D;
  const __half* vb = p.v + (size_t(b) * p.cap * p.Hkv + kvh) * D;
  unsigned char* wsm = smem + warp * (NB * 2 * TILE_BYTES);
  const uint32_t wsm_u = smem_u32(wsm);

  auto issue_tile = [&](int t, int stage) {
    const uint32_t ks = wsm_u + stage * 2 * TILE_BYTES;
    const uint32_t vs = ks + TILE_BYTES;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int idx = i * 32 + lane;
      const int r = idx >> 4, ch = idx & 15;
      const int slot = c0 + t * TILE + r;
      const bool ok = slot < c1;
      const size_t off = ok ? size_t(slot) * slot_stride + ch * 8 : 0;
      cp_async16(ks + swz(r, ch), kb + off, ok ? 16 : 0);
      cp_async16(vs + swz(r, ch), vb + off, ok ? 16 : 0);
    }
    cp_async_commit();
  };

  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};

  // NB tiles in flight per warp (an empty commit group where no tile is left)
#pragma unroll
  for (int k = 0; k < NB; ++k) {
    if (warp + k * WARPS < ntiles) issue_tile(warp + k * WARPS, k);
    else cp_async_commit();
  }
  if (p.early) pdl_wait();  // q (and slot `fresh`) come from the previous kernel
  trace_stamp(trc, TR_WAITED, threadIdx.x == 0);

  const __half* qsrc = p.q + (size_t(b) * p.Hq + size_t(kvh) * p.G) * D;
  if (p.fused) {
    // the G query heads of this KV head: head norm + RoPE into shared memory;
    // the CTA whose chunk holds the new token's slot appends its k and v
    __half* qs = reinterpret_cast<__half*>(smem + (NB == 4 ? SMEM4 : SMEM));
    const int heads = p.Hq + 2 * p.Hkv;
    const __half* row = p.qkv + size_t(b) * heads * D;
    for (int i = warp; i < p.G; i += WARPS)
      head_norm_rope<4>(row + size_t(kvh * p.G + i) * D, p.qnw, p.eps, p.cosr, p.sinr, qs + i * D, lane);
    if (p.fresh >= c0 && p.fresh < c1) {
      const size_t dst = ((size_t(b) * p.cap + p.fresh) * p.Hkv + kvh) * D;
      if (warp == 0) {
        head_norm_rope<4>(row + size_t(p.Hq + kvh) * D, p.knw, p.eps, p.cosr, p.sinr,
                          const_cast<__half*>(p.k) + dst, lane);
      } else if (warp == 1) {
        const uint2 v = reinterpret_cast<const uint2*>(row + size_t(p.Hq + p.Hkv + kvh) * D)[lane];
        reinterpret_cast<uint2*>(const_cast<__half*>(p.v) + dst)[lane] = v;
      }
    }
    __syncthreads();  // rotated q in shared memory; the appended slot visible to this CTA
    qsrc = qs;
  }
  // Q fragments (rows = query heads of this KV head, k = head dim)
  uint32_t qa[8][4];
  {
    const __half* qb = qsrc;
    const bool r0 = g < p.G, r1 = g + 8 < p.G;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int d0 = kk * 16 + 2 * c;
      qa[kk][0] = r0 ? *reinterpret_cast<const uint32_t*>(qb + g * D + d0) : 0u;
      qa[kk][1] = r1 ? *reinterpret_cast<const uint32_t*>(qb + (g + 8) * D + d0) : 0u;
      qa[kk][2] = r0 ? *reinterpret_cast<const uint32_t*>(qb + g * D + d0 + 8) : 0u;
      qa[kk][3] = r1 ? *reinterpret_cast<const uint32_t*>(qb + (g + 8) * D + d0 + 8) : 0u;
    }
  }


  for (int it = 0, t = warp; t < ntiles; ++it, t += WARPS) {
    cp_async_wait<NB - 1>();  // tile `it` landed; the NB - 1 after it may still be in flight
    trace_stamp(trc, TR_TILE0, threadIdx.x == 0 && it == 0);
    __syncwarp();
    const int stage = it % NB;
    const uint32_t ks = wsm_u + stage * 2 * TILE_BYTES;
    const uint32_t vs = ks + TILE_BYTES;
    if ((p.early || p.fused) && it < NB) {
      // the tiles of the first NB rounds were requested before the previous
      // kernel finished (or before this kernel appended): reload that slot
      const int r = p.fresh - (c0 + t * TILE);
      if (r >= 0 && r < TILE && p.fresh < c1) {
        const int ch = lane & 15;
        const __half* src = (lane < 16 ? kb : vb) + size_t(p.fresh) * slot_stride + ch * 8;
        const uint4 v = __ldcg(reinterpret_cast<const uint4*>(src));
        const uint32_t dst = (lane < 16 ? ks : vs) + swz(r, ch);
        asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(v.x), "r"(v.y),
                     "r"(v.z), "r"(v.w)
                     : "memory");
        __syncwarp();
      }
    }

    // S = Q K^T : two n-tiles of 8 slots
    float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    {
      const int mi = lane >> 3, ri = lane & 7;
      const int row = 8 * (mi >> 1) + ri;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        uint32_t bk[4];
        ldsm_x4(bk, ks + swz(row, 2 * kk + (mi & 1)));
        mma_16816(s[0], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], bk[0], bk[1]);
        mma_16816(s[1], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], bk[2], bk[3]);
      }
    }
    // scale (log2 domain) and mask slots beyond the chunk
    const int sbase = c0 + t * TILE;
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int slot = sbase + 8 * j + 2 * c + (e & 1);
        s[j][e] = slot < c1 ? s[j][e] * p.scale_log2 : -INFINITY;
      }
    // online softmax: rows g (e = 0,1) and g + 8 (e = 2,3)
    float mx0 = fmaxf(fmaxf(s[0][0], s[0][1]), fmaxf(s[1][0], s[1][1]));
    float mx1 = fmaxf(fmaxf(s[0][2], s[0][3]), fmaxf(s[1][2], s[1][3]));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m_r[0], mx0), mn1 = fmaxf(m_r[1], mx1);
    const float al0 = exp2f(m_r[0] - mn0), al1 = exp2f(m_r[1] - mn1);
    m_r[0] = mn0;
    m_r[1] = mn1;
    float pr[2][4];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      pr[j][0] = exp2f(s[j][0] - mn0);
      pr[j][1] = exp2f(s[j][1] - mn0);
      pr[j][2] = exp2f(s[j][2] - mn1);
      pr[j][3] = exp2f(s[j][3] - mn1);
    }
    l_r[0] = l_r[0] * al0 + ((pr[0][0] + pr[0][1]) + (pr[1][0] + pr[1][1]));
    l_r[1] = l_r[1] * al1 + ((pr[0][2] + pr[0][3]) + (pr[1][2] + pr[1][3]));
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      o[j][0] *= al0;
      o[j][1] *= al0;
      o[j][2] *= al1;
      o[j][3] *= al1;
    }
    const uint32_t pa0 = pack_h2(pr[0][0], pr[0][1]);
    const uint32_t pa1 = pack_h2(pr[0][2], pr[0][3]);
    const uint32_t pa2 = pack_h2(pr[1][0], pr[1][1]);
    const uint32_t pa3 = pack_h2(pr[1][2], pr[1][3]);
    // O += P V : 16 n-tiles of 8 head dims
    {
      const int mi = lane >> 3, ri = lane & 7;
      const int row = 8 * (mi & 1) + ri;
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        uint32_t bv[4];
        ldsm_x4_t(bv, vs + swz(row, 2 * jj + (mi >> 1)));
        mma_16816(o[2 * jj], pa0, pa1, pa2, pa3, bv[0], bv[1]);
        mma_16816(o[2 * jj + 1], pa0, pa1, pa2, pa3, bv[2], bv[3]);
      }
    }
    __syncwarp();
    // the stage is free: request tile it + NB into it
    if (t + NB * WARPS < ntiles) issue_tile(t + NB * WARPS, stage);
    else cp_async_commit();
  }
  cp_async_wait<0>();
  trace_stamp(trc, TR_LOOP, threadIdx.x == 0);
  l_r[0] += __shfl_xor_sync(0xffffffffu, l_r[0], 1);
  l_r[0] += __shfl_xor_sync(0xffffffffu, l_r[0], 2);
  l_r[1] += __shfl_xor_sync(0xffffffffu, l_r[1], 1);
  l_r[1] += __shfl_xor_sync(0xffffffffu, l_r[1], 2);

  // merge the warps of this CTA in shared memory (reuses the tile buffers)
  __syncthreads();
  float* Os = reinterpret_cast<float*>(smem);            // [WARPS][16][OSTRIDE]
  float* ms = Os + WARPS * 16 * OSTRIDE;                  // [WARPS][16]
  float* ls = ms + WARPS * 16;                            // [WARPS][16]
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int d = 8 * j + 2 * c;
    *reinterpret_cast<float2*>(Os + (warp * 16 + g) * OSTRIDE + d) = make_float2(o[j][0], o[j][1]);
    *reinterpret_cast<float2*>(Os + (warp * 16 + g + 8) * OSTRIDE + d) = make_float2(o[j][2], o[j][3]);
  }
  if (c == 0) {
    ms[warp * 16 + g] = m_r[0];
    ms[warp * 16 + g + 8] = m_r[1];
    ls[warp * 16 + g] = l_r[0];
    ls[warp * 16 + g + 8] = l_r[1];
  }
  __syncthreads();
  float* mypart = p.part + (size_t(bh) * p.nch + ci) * p.G * PSTRIDE;
  // cluster form: the receive areas (past the tiles and the fused q heads)
  const int roff = (NB == 4 ? SMEM4 : SMEM) + (p.fused ? QS_BYTES : 0);
  const uint32_t recv_o = smem_u32(smem + roff);                       // [nch][per][4]
  const uint32_t recv_ml = recv_o + uint32_t(p.nch * per * 16);         // [nch][rmax][2]
  if constexpr (CLUSTER) asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
  {
    const int d = tid;  // THREADS == D
    for (int r = 0; r < p.G; ++r) {
      float mx = -INFINITY;
#pragma unroll
      for (int w = 0; w < WARPS; ++w) mx = fmaxf(mx, ms[w * 16 + r]);
      float L = 0.f, O = 0.f;
#pragma unroll
      for (int w = 0; w < WARPS; ++w) {
        const float f = ms[w * 16 + r] == -INFINITY ? 0.f : exp2f(ms[w * 16 + r] - mx);
        L = fmaf(ls[w * 16 + r], f, L);
        O = fmaf(Os[(w * 16 + r) * OSTRIDE + d], f, O);
      }
      if constexpr (CLUSTER) {
        // O of vector v = r * 32 + d / 4 to its owner; (max, sum) of row r to
        // every owner whose vectors cover part of the row
        const int v = r * (D / 4) + (d >> 2);
        const int j = v / per, lv = v - j * per;
        st_async_f32(cluster_map(recv_o + uint32_t((ci * per + lv) * 4 + (d & 3)) * 4u, uint32_t(j)), O,
                     cluster_map(smem_u32(&s_rbar), uint32_t(j)));
        const int jlo = (r * (D / 4)) / per, jhi = min(p.nch - 1, (r * (D / 4) + D / 4 - 1) / per);
        if (d <= jhi - jlo) {
          const int jj = jlo + d, rr = r - (jj * per) / (D / 4);
          st_async_f2(cluster_map(recv_ml + uint32_t(ci * rmax + rr) * 8u, uint32_t(jj)), mx, L,
                      cluster_map(smem_u32(&s_rbar), uint32_t(jj)));
        }
      } else {
        mypart[r * PSTRIDE + 4 + d] = O;
        if (d == 0) {
          mypart[r * PSTRIDE] = mx;
          mypart[r * PSTRIDE + 1] = L;
        }
      }
    }
  }

  trace_stamp(trc, TR_WARP_MERGE, threadIdx.x == 0);
  if constexpr (CLUSTER) {
    // every chunk pushed its share of this CTA's output vectors [v0, v1) and
    // the (max, sum) of their rows: wait for all of it (bounded), then merge
    // the chunks in order (deterministic) from local shared memory
    const int nch = p.nch, G = p.G;
    const int v0 = ci * per, own_v = max(0, min(per, G * (D / 4) - v0));
    if (own_v > 0) {
      const uint32_t rb = smem_u32(&s_rbar);
      if (!mbar_try(rb, 0)) {
        unsigned long long t0, t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
        while (!mbar_try(rb, 0)) {
          asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
          if (t - t0 > kWaitLimitNs) {
            if (tid == 0) atomicOr(&g_attn_error, QX_DEVERR_MBAR_TIMEOUT);
            break;
          }
        }
      }
      trace_stamp(trc, TR_CHUNK_SYNC, threadIdx.x == 0);
      const float* ro = reinterpret_cast<const float*>(smem + roff);
      const float* rml = ro + nch * per * 4;
      const int r0 = v0 / (D / 4);
      for (int e = tid; e < own_v * 4; e += THREADS) {
        const int v = v0 + (e >> 2), r = v / (D / 4), d = (v - r * (D / 4)) * 4 + (e & 3);
        float mx = -INFINITY;
        for (int k = 0; k < nch; ++k) mx = fmaxf(mx, rml[(k * rmax + r - r0) * 2]);
        float L = 0.f, O = 0.f;
        for (int k = 0; k < nch; ++k) {
          const float mk = rml[(k * rmax + r - r0) * 2];
          const float f = mk == -INFINITY ? 0.f : exp2f(mk - mx);
          L = fmaf(rml[(k * rmax + r - r0) * 2 + 1], f, L);
          O = fmaf(ro[(k * per) * 4 + e], f, O);
        }
        p.out[(size_t(b) * p.Hq + size_t(kvh) * G + r) * D + d] = __float2half_rn(O / L);
      }
    }
    trace_stamp(trc, TR_EXIT, threadIdx.x == 0);
    return;
  }

  // the last CTA of this (sequence, KV head) merges the chunks
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned prev = atomicAdd(p.counters + bh, 1u);
    s_is_last = (prev == unsigned(p.nch - 1)) ? 1u : 0u;
  }
  __syncthreads();
  if (!s_is_last) return;
  __threadfence();
  {
    // Merge the chunks: (1) one warp per query row loads its chunks' (max,
    // sum) pairs, reduces the max and the weighted sum with shuffles (fixed
    // butterfly order: deterministic) and stores the chunk weights; (2) O by 4
    // interleaved chunk subsets with 16-byte loads, two rows per pass so their
    // loads are in flight together; (3) fixed-order sum of the subsets.
    const int G = p.G, nch = p.nch;
    const float* pb = p.part + size_t(bh) * nch * G * PSTRIDE;
    float* sm_m = reinterpret_cast<float*>(smem);  // [G][nch] chunk weights
    float* sm_L = sm_m + 2 * G * nch;              // [16]
    // [4][G][D], 16-byte aligned for the float4 stores
    float* sm_o = sm_m + ((2 * G * nch + 16 + 3) & ~3);
    for (int r = warp; r < G; r += WARPS) {
      float mk[MAX_CHUNKS / 32], lk[MAX_CHUNKS / 32];
#pragma unroll
      for (int i = 0; i < MAX_CHUNKS / 32; ++i) {
        const int k = lane + 32 * i;
        const float* pk = pb + (size_t(k) * G + r) * PSTRIDE;
        mk[i] = k < nch ? __ldcg(pk) : -INFINITY;
        lk[i] = k < nch ? __ldcg(pk + 1) : 0.f;
      }
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < MAX_CHUNKS / 32; ++i) mx = fmaxf(mx, mk[i]);
      mx = warp_max(mx);
      float L = 0.f;
#pragma unroll
      for (int i = 0; i < MAX_CHUNKS / 32; ++i) {
        const int k = lane + 32 * i;
        const float f = mk[i] == -INFINITY ? 0.f : exp2f(mk[i] - mx);
        if (k < nch) sm_m[r * nch + k] = f;
        L = fmaf(lk[i], f, L);
      }
      L = warp_sum(L);
      if (lane == 0) sm_L[r] = L;
    }
    __syncthreads();
    const int d4 = tid & 31, kq = tid >> 5;
    for (int r = 0; r < G; r += 2) {
      const bool two = r + 1 < G;
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b2 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
      for (int k = kq; k < nch; k += 4) {
        const float4 v =
            __ldcg(reinterpret_cast<const float4*>(pb + (size_t(k) * G + r) * PSTRIDE + 4) + d4);
        const float4 w = two ? __ldcg(reinterpret_cast<const float4*>(
                                   pb + (size_t(k) * G + r + 1) * PSTRIDE + 4) + d4)
                             : make_float4(0.f, 0.f, 0.f, 0.f);
        const float f = sm_m[r * nch + k];
        const float f2 = two ? sm_m[(r + 1) * nch + k] : 0.f;
        a.x = fmaf(f, v.x, a.x);
        a.y = fmaf(f, v.y, a.y);
        a.z = fmaf(f, v.z, a.z);
        a.w = fmaf(f, v.w, a.w);
        b2.x = fmaf(f2, w.x, b2.x);
        b2.y = fmaf(f2, w.y, b2.y);
        b2.z = fmaf(f2, w.z, b2.z);
        b2.w = fmaf(f2, w.w, b2.w);
      }
      *reinterpret_cast<float4*>(sm_o + (kq * G + r) * D + 4 * d4) = a;
      if (two) *reinterpret_cast<float4*>(sm_o + (kq * G + r + 1) * D + 4 * d4) = b2;
    }
    __syncthreads();
    const int d = tid;
    for (int r = 0; r < G; ++r) {
      const float O = ((sm_o[(0 * G + r) * D + d] + sm_o[(1 * G + r) * D + d]) +
                       sm_o[(2 * G + r) * D + d]) + sm_o[(3 * G + r) * D + d];
      p.out[(size_t(b) * p.Hq + size_t(kvh) * G + r) * D + d] = __float2half_rn(O / sm_L[r]);
    }
  }
  if (tid == 0) p.counters[bh] = 0u;
  trace_stamp(trc, TR_EXIT, tid == 0);
}

struct Plan {
  int chunk, nch, nch_max;
  bool cluster;  // merge the chunks through distributed shared memory
  int nb;        // tile stages per warp (2, or 4 when the grid holds at most one CTA per SM)
  size_t off_part, total;
};

// 0 (default): the cluster merge whenever a sequence has more than one chunk
// and every (sequence, KV head) cluster of the grid is resident at once (one
// wave: measured 10.9 vs 11.7 us at one sequence, while 32 clusters of 13
// CTAs that took two waves ran 26.9 vs 20.7 us); 1: always the workspace
// merge (qx_decode_attention_pin_merge)
static std::atomic<int> g_merge_mode{0};

// fit[n] (n <= MAX_CLUSTER): clusters of n CTAs the device holds at once
// with 2 tile stages per warp, fit[MAX_CLUSTER + 1 + n] with 4 (0: not
// schedulable); null: no cluster merge, 2 stages
static Plan make_plan(int batch, int kv_heads, int G, int cap, int valid, int sms,
                      const int* fit = nullptr) {
  Plan pl{};
  const int bh = batch * kv_heads;
  const int target = std::min(MAX_CHUNKS, std::max(1, sms * CTAS_PER_SM / std::max(1, bh)));
  const int max_by_cap = std::max(1, (cap + CHUNK_ALIGN - 1) / CHUNK_ALIGN);
  pl.nch_max = std::min(target, max_by_cap);
  const int v = std::max(valid, 1);
  const int nch0 = std::max(1, std::min(target, (v + CHUNK_ALIGN - 1) / CHUNK_ALIGN));
  int chunk = (v + nch0 - 1) / nch0;
  chunk = (chunk + CHUNK_ALIGN - 1) / CHUNK_ALIGN * CHUNK_ALIGN;
  pl.chunk = chunk;
  pl.nch = (v + chunk - 1) / chunk;
  pl.off_part = size_t(COUNTER_SLOTS) * 4;
  pl.total = pl.off_part + size_t(bh) * pl.nch_max * G * PSTRIDE * 4;
  pl.cluster = false;
  const int mode = g_merge_mode.load(std::memory_order_relaxed);
  if (fit && pl.nch >= 2 && mode != 1) {
    // fewer, longer chunks so that one cluster holds a whole sequence's chunks
    int maxc = 0;
    for (int n = 2; n <= MAX_CLUSTER; ++n)
      if (fit[n] > 0) maxc = n;
    const int nc = std::min(pl.nch, maxc);
    int ch = (v + std::max(nc, 1) - 1) / std::max(nc, 1);
    ch = (ch + CHUNK_ALIGN - 1) / CHUNK_ALIGN * CHUNK_ALIGN;
    const int n = (v + ch - 1) / ch;
    if (nc >= 2 && n >= 2 && n <= maxc && fit[n] >= bh) {
      pl.chunk = ch;
      pl.nch = n;
      pl.cluster = true;
    }
  }
  // 4 stages per warp when every CTA gets an SM of its own and each warp has
  // at least 3 tiles: the whole chunk is requested at once (one HBM round trip)
  pl.nb = 2;
  if (fit && long(pl.nch) * bh <= sms && pl.chunk >= 3 * CHUNK_ALIGN &&
      (!pl.cluster || fit[MAX_CLUSTER + 1 + pl.nch] >= bh))
    pl.nb = 4;
  return pl;
}

// Raises the kernels' dynamic shared-memory limits once per device (both
// entry points; the per-device state is guarded by a mutex) and records, per
// cluster size n <= 16, how many chunk clusters the device holds at once.
static int prepare_kernel(const int** fit_out) {
  static std::mutex mu;
  static bool done[64] = {};
  static int fit[64][2 * (MAX_CLUSTER + 1)] = {};
  int dev = 0;
  QX_CUDA_TRY(cudaGetDevice(&dev), "decode_attention: cudaGetDevice");
  QX_REQUIRE(dev >= 0 && dev < 64, "decode_attention: device index %d unsupported", dev);
  std::lock_guard<std::mutex> lk(mu);
  if (!done[dev]) {
    QX_CUDA_TRY(cudaFuncSetAttribute(decode_attn_kernel<false, 2>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes(2, true)),
                "decode_attention: set smem limit");
    QX_CUDA_TRY(cudaFuncSetAttribute(decode_attn_kernel<true, 2>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes(2, true, true)),
                "decode_attention: set smem limit");
    QX_CUDA_TRY(cudaFuncSetAttribute(decode_attn_kernel<false, 4>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes(4, true)),
                "decode_attention: set smem limit");
    QX_CUDA_TRY(cudaFuncSetAttribute(decode_attn_kernel<true, 4>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes(4, true, true)),
                "decode_attention: set smem limit");
    QX_CUDA_TRY(cudaFuncSetAttribute(decode_attn_kernel<true, 2>,
                                     cudaFuncAttributeNonPortableClusterSizeAllowed, 1),
                "decode_attention: allow 16-CTA clusters");
    QX_CUDA_TRY(cudaFuncSetAttribute(decode_attn_kernel<true, 4>,
                                     cudaFuncAttributeNonPortableClusterSizeAllowed, 1),
                "decode_attention: allow 16-CTA clusters");
    for (int nbi = 0; nbi < 2; ++nbi) {
      for (int cs = 2; cs <= MAX_CLUSTER; ++cs) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(cs, 1, 1);
        cfg.blockDim = dim3(THREADS, 1, 1);
        cfg.dynamicSmemBytes = smem_bytes(nbi ? 4 : 2, true, true);
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = cs;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        int n = 0;
        const cudaError_t e = nbi ? cudaOccupancyMaxActiveClusters(&n, decode_attn_kernel<true, 4>, &cfg)
                                  : cudaOccupancyMaxActiveClusters(&n, decode_attn_kernel<true, 2>, &cfg);
        if (e != cudaSuccess) {
          cudaGetLastError();
          n = 0;
        }
        fit[dev][nbi * (MAX_CLUSTER + 1) + cs] = n;
      }
    }
    done[dev] = true;
  }
  *fit_out = fit[dev];
  return QX_OK;
}

// Launches the kernel of plan `pl`: clusters of pl.nch CTAs along x for the
// cluster merge, a plain grid otherwise (measured: launched early, its CTAs
// wait resident and the grid lands less evenly, 82 vs 89 us at 32 sequences;
// it still triggers at entry, so the GEMV after it streams its weights
// meanwhile).
static int launch(const Plan& pl, const Params& prm, int batch, int kv_heads, cudaStream_t st,
                  const char* what) {
  const dim3 grid(pl.nch, batch * kv_heads), block(THREADS);
  const int smem = smem_bytes(pl.nb, prm.fused != 0, pl.cluster);
  auto kern = pl.cluster ? (pl.nb == 4 ? decode_attn_kernel<true, 4> : decode_attn_kernel<true, 2>)
                         : (pl.nb == 4 ? decode_attn_kernel<false, 4> : decode_attn_kernel<false, 2>);
  Params pt = prm;
  pt.trace = trace_next(QX_TRACE_DECODE_ATTENTION, &pt.trace_launch);
  if (!pl.cluster && !prm.early) {
    kern<<<grid, block, smem, st>>>(pt);
    return check_launch(what);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  int na = 0;
  if (pl.cluster) {
    at[na].id = cudaLaunchAttributeClusterDimension;
    at[na].val.clusterDim.x = pl.nch;
    at[na].val.clusterDim.y = 1;
    at[na].val.clusterDim.z = 1;
    ++na;
  }
  if (prm.early) {
    at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = at;
  cfg.numAttrs = na;
  QX_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, pt), what);
  return check_launch(what);
}

}  // namespace attn

int attn_device_error(unsigned* code, int reset) {
  QX_CUDA_TRY(cudaMemcpyFromSymbol(code, attn::g_attn_error, sizeof(unsigned)), "get_device_error: read");
  if (reset) {
    const unsigned zero = 0;
    QX_CUDA_TRY(cudaMemcpyToSymbol(attn::g_attn_error, &zero, sizeof(unsigned)), "get_device_error: reset");
  }
  return QX_OK;
}

}  // namespace qx

using namespace qx;

extern "C" size_t qx_decode_attention_workspace_size(int batch, int q_heads, int kv_heads,
                                                     int head_dim, int sink, int window) {
  if (batch <= 0 || kv_heads <= 0 || q_heads <= 0 || q_heads % kv_heads || window < 1 || sink < 0)
    return 0;
  (void)head_dim;
  return attn::make_plan(batch, kv_heads, q_heads / kv_heads, sink + window, sink + window,
                         device_sm_count())
      .total;
}

extern "C" int qx_decode_attention_ex(const void* q, const void* k_cache, const void* v_cache,
                                      void* out, int batch, int q_heads, int kv_heads, int head_dim,
                                      int sink, int window, int64_t count, float softmax_scale,
                                      void* workspace, size_t workspace_bytes, int flags,
                                      qx_stream_t stream) {
  QX_REQUIRE((flags & ~QX_ATTN_AFTER_APPEND) == 0, "decode_attention: unknown flags %d", flags);
  QX_REQUIRE(batch > 0 && q_heads > 0 && kv_heads > 0 && q_heads % kv_heads == 0,
             "decode_attention: bad heads q=%d kv=%d", q_heads, kv_heads);
  QX_REQUIRE(head_dim == attn::D, "decode_attention: head_dim=%d unsupported (128)", head_dim);
  QX_REQUIRE(q_heads / kv_heads <= 16, "decode_attention: GQA group %d > 16",
             q_heads / kv_heads);
  QX_REQUIRE(sink >= 0 && window >= 1, "decode_attention: sink=%d window=%d", sink, window);
  QX_REQUIRE(count > 0, "decode_attention: empty cache (count=%lld)", (long long)count);
  QX_REQUIRE(batch * kv_heads <= attn::COUNTER_SLOTS, "decode_attention: batch*kv_heads > %d",
             attn::COUNTER_SLOTS);
  QX_REQUIRE(q && k_cache && v_cache && out, "decode_attention: null pointer");
  QX_REQUIRE(aligned(k_cache, 16) && aligned(v_cache, 16) && aligned(q, 4) && aligned(out, 2),
             "decode_attention: misaligned tensors");
  const int cap = sink + window;
  const int64_t valid64 = count <= sink ? count : sink + std::min<int64_t>(count - sink, window);
  const int valid = int(valid64);
  const int G = q_heads / kv_heads;
  const int* fit = nullptr;
  {
    const int rc = attn::prepare_kernel(&fit);
    if (rc != QX_OK) return rc;
  }
  const attn::Plan pl =
      attn::make_plan(batch, kv_heads, G, cap, valid, device_sm_count(), fit);
  if (!workspace || workspace_bytes < pl.total || !aligned(workspace, 256))
    return fail(QX_ERR_WORKSPACE, "decode_attention: workspace needs %zu bytes, 256-byte aligned",
                pl.total);
  attn::Params prm{};
  prm.q = static_cast<const __half*>(q);
  prm.k = static_cast<const __half*>(k_cache);
  prm.v = static_cast<const __half*>(v_cache);
  prm.out = static_cast<__half*>(out);
  prm.Hq = q_heads;
  prm.Hkv = kv_heads;
  prm.G = G;
  prm.cap = cap;
  prm.valid = valid;
  prm.chunk = pl.chunk;
  prm.nch = pl.nch;
  const float scale = softmax_scale > 0.f ? softmax_scale : 1.0f / sqrtf(float(head_dim));
  prm.scale_log2 = scale * 1.4426950408889634f;
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  prm.counters = reinterpret_cast<unsigned*>(ws);
  prm.part = reinterpret_cast<float*>(ws + pl.off_part);
  // after an append of position count - 1 (its physical slot is `fresh`) by
  // the previous kernel: load the other slots while it finishes
  // (small grids only: measured on the append + attention pair, one sequence
  // 12.4 vs 12.7 us, while 32 sequences' waiting CTAs landed unevenly, 95.7
  // vs 85.0 us)
  prm.early = (flags & QX_ATTN_AFTER_APPEND) && g_pdl_enabled.load(std::memory_order_relaxed) &&
                      long(pl.nch) * batch * kv_heads <= 2L * device_sm_count()
                  ? 1
                  : 0;
  const int64_t last = count - 1;
  prm.fresh = int(last < sink ? last : sink + (last - sink) % window);
  return attn::launch(pl, prm, batch, kv_heads, reinterpret_cast<cudaStream_t>(stream),
                      "decode_attention");
}

extern "C" int qx_decode_attention(const void* q, const void* k_cache, const void* v_cache,
                                   void* out, int batch, int q_heads, int kv_heads, int head_dim,
                                   int sink, int window, int64_t count, float softmax_scale,
                                   void* workspace, size_t workspace_bytes, qx_stream_t stream) {
  return qx_decode_attention_ex(q, k_cache, v_cache, out, batch, q_heads, kv_heads, head_dim, sink, window,
                                count, softmax_scale, workspace, workspace_bytes, 0, stream);
}

extern "C" int qx_decode_attention_qkv(const void* qkv, const void* q_norm_w, const void* k_norm_w,
                                       float eps, const float* cos_row, const float* sin_row,
                                       void* k_cache, void* v_cache, void* out, int batch, int q_heads,
                                       int kv_heads, int head_dim, int sink, int window, int64_t pos,
                                       float softmax_scale, void* workspace, size_t workspace_bytes,
                                       qx_stream_t stream) {
  QX_REQUIRE(batch > 0 && q_heads > 0 && kv_heads > 0 && q_heads % kv_heads == 0,
             "decode_attention_qkv: bad heads q=%d kv=%d", q_heads, kv_heads);
  QX_REQUIRE(head_dim == attn::D, "decode_attention_qkv: head_dim=%d unsupported (128)", head_dim);
  QX_REQUIRE(q_heads / kv_heads <= 16, "decode_attention_qkv: GQA group %d > 16", q_heads / kv_heads);
  QX_REQUIRE(sink >= 0 && window >= 1 && pos >= 0, "decode_attention_qkv: sink=%d window=%d pos=%lld",
             sink, window, (long long)pos);
  QX_REQUIRE(batch * kv_heads <= attn::COUNTER_SLOTS, "decode_attention_qkv: batch*kv_heads > %d",
             attn::COUNTER_SLOTS);
  QX_REQUIRE(qkv && q_norm_w && k_norm_w && cos_row && sin_row && k_cache && v_cache && out,
             "decode_attention_qkv: null pointer");
  QX_REQUIRE(aligned(qkv, 16) && aligned(k_cache, 16) && aligned(v_cache, 16) && aligned(out, 2),
             "decode_attention_qkv: misaligned tensors");
  const int cap = sink + window;
  const int64_t count = pos + 1;
  const int64_t valid64 = count <= sink ? count : sink + std::min<int64_t>(count - sink, window);
  const int G = q_heads / kv_heads;
  const int* fit = nullptr;
  {
    const int rc = attn::prepare_kernel(&fit);
    if (rc != QX_OK) return rc;
  }
  const attn::Plan pl = attn::make_plan(batch, kv_heads, G, cap, int(valid64), device_sm_count(), fit);
  if (!workspace || workspace_bytes < pl.total || !aligned(workspace, 256))
    return fail(QX_ERR_WORKSPACE, "decode_attention_qkv: workspace needs %zu bytes, 256-byte aligned",
                pl.total);
  attn::Params prm{};
  prm.q = static_cast<const __half*>(qkv);  // unused: the rotated q is built in shared memory
  prm.k = static_cast<const __half*>(k_cache);
  prm.v = static_cast<const __half*>(v_cache);
  prm.out = static_cast<__half*>(out);
  prm.Hq = q_heads;
  prm.Hkv = kv_heads;
  prm.G = G;
  prm.cap = cap;
  prm.valid = int(valid64);
  prm.chunk = pl.chunk;
  prm.nch = pl.nch;
  const float scale = softmax_scale > 0.f ? softmax_scale : 1.0f / sqrtf(float(head_dim));
  prm.scale_log2 = scale * 1.4426950408889634f;
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  prm.counters = reinterpret_cast<unsigned*>(ws);
  prm.part = reinterpret_cast<float*>(ws + pl.off_part);
  prm.fresh = int(pos < sink ? pos : sink + (pos - sink) % window);  // the new token's slot
  prm.fused = 1;
  prm.qkv = static_cast<const __half*>(qkv);
  prm.qnw = static_cast<const __half*>(q_norm_w);
  prm.knw = static_cast<const __half*>(k_norm_w);
  prm.cosr = cos_row;
  prm.sinr = sin_row;
  prm.eps = eps;
  // the previous kernel (the projection) writes no cache slot: with a small
  // grid every tile may load while it finishes
  prm.early = g_pdl_enabled.load(std::memory_order_relaxed) &&
                      long(pl.nch) * batch * kv_heads <= 2L * device_sm_count()
                  ? 1
                  : 0;
  return attn::launch(pl, prm, batch, kv_heads, reinterpret_cast<cudaStream_t>(stream),
                      "decode_attention_qkv");
}

extern "C" int qx_decode_attention_pin_merge(int mode) {
  QX_REQUIRE(mode == 0 || mode == 1, "decode_attention_pin_merge: mode %d (0 auto, 1 workspace)", mode);
  attn::g_merge_mode.store(mode);
  return QX_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free variant of qx_decode_attention.
//
// Some callers cannot allocate device memory when they run attention: a host
// framework that owns the device heap and forbids side allocations, a plugin
// of an inference server that is handed only its input and output buffers, or
// a latency-critical path where cudaMalloc/cudaFree would synchronise the
// device.  This entry point keeps the kernel's scratch (the per-(sequence, KV
// head) counters and the per-chunk partial results) in one array compiled into
// the library instead of a caller workspace.
namespace qx {
namespace attn {

// Every GPU that loads the library holds this array until the process exits.
static __device__ __align__(256) unsigned char g_noalloc_scratch[QX_DECODE_ATTN_NOALLOC_SCRATCH_BYTES];

static std::mutex g_noalloc_mu;
static void* g_noalloc_ptr[64] = {};

// Device address of the array on the current device, looked up once per device
// (the host-side name is only a stand-in and must never reach a kernel).
static int noalloc_scratch(void** out) {
  int dev = 0;
  QX_CUDA_TRY(cudaGetDevice(&dev), "decode_attention_noalloc: cudaGetDevice");
  QX_REQUIRE(dev >= 0 && dev < 64, "decode_attention_noalloc: device index %d unsupported", dev);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    QX_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch),
                "decode_attention_noalloc: cudaGetSymbolAddress");
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return QX_OK;
}

}  // namespace attn
}  // namespace qx

extern "C" int qx_decode_attention_noalloc(const void* q, const void* k_cache,
                                           const void* v_cache, void* out, int batch, int q_heads,
                                           int kv_heads, int head_dim, int sink, int window,
                                           int64_t count, float softmax_scale,
                                           qx_stream_t stream) {
  QX_REQUIRE(batch > 0 && q_heads > 0 && kv_heads > 0 && q_heads % kv_heads == 0,
             "decode_attention_noalloc: bad heads q=%d kv=%d", q_heads, kv_heads);
  QX_REQUIRE(head_dim == attn::D, "decode_attention_noalloc: head_dim=%d unsupported (128)",
             head_dim);
  QX_REQUIRE(q_heads / kv_heads <= 16, "decode_attention_noalloc: GQA group %d > 16",
             q_heads / kv_heads);
  QX_REQUIRE(sink >= 0 && window >= 1, "decode_attention_noalloc: sink=%d window=%d", sink,
             window);
  QX_REQUIRE(count > 0, "decode_attention_noalloc: empty cache (count=%lld)", (long long)count);
  QX_REQUIRE(batch * kv_heads <= attn::COUNTER_SLOTS,
             "decode_attention_noalloc: batch*kv_heads > %d", attn::COUNTER_SLOTS);
  QX_REQUIRE(q && k_cache && v_cache && out, "decode_attention_noalloc: null pointer");
  QX_REQUIRE(aligned(k_cache, 16) && aligned(v_cache, 16) && aligned(q, 4) && aligned(out, 2),
             "decode_attention_noalloc: misaligned tensors");
  const int cap = sink + window;
  const int64_t valid64 = count <= sink ? count : sink + std::min<int64_t>(count - sink, window);
  const int valid = int(valid64);
  const int G = q_heads / kv_heads;
  const int* fit = nullptr;
  {
    const int rc = attn::prepare_kernel(&fit);
    if (rc != QX_OK) return rc;
  }
  const attn::Plan pl =
      attn::make_plan(batch, kv_heads, G, cap, valid, device_sm_count(), fit);
  if (pl.total > size_t(QX_DECODE_ATTN_NOALLOC_SCRATCH_BYTES))
    return fail(QX_ERR_UNSUPPORTED,
                "decode_attention_noalloc: this shape needs %zu bytes of scratch, more than the "
                "%d-byte built-in array; use qx_decode_attention with a workspace",
                pl.total, QX_DECODE_ATTN_NOALLOC_SCRATCH_BYTES);
  void* scratch = nullptr;
  const int src = attn::noalloc_scratch(&scratch);
  if (src != QX_OK) return src;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // the counters must start at zero; the array keeps whatever the last call left
  QX_CUDA_TRY(cudaMemsetAsync(scratch, 0, size_t(batch) * kv_heads * sizeof(unsigned), st),
              "decode_attention_noalloc: clear counters");
  attn::Params prm{};
  prm.q = static_cast<const __half*>(q);
  prm.k = static_cast<const __half*>(k_cache);
  prm.v = static_cast<const __half*>(v_cache);
  prm.out = static_cast<__half*>(out);
  prm.Hq = q_heads;
  prm.Hkv = kv_heads;
  prm.G = G;
  prm.cap = cap;
  prm.valid = valid;
  prm.chunk = pl.chunk;
  prm.nch = pl.nch;
  const float scale = softmax_scale > 0.f ? softmax_scale : 1.0f / sqrtf(float(head_dim));
  prm.scale_log2 = scale * 1.4426950408889634f;
  unsigned char* ws = static_cast<unsigned char*>(scratch);
  prm.counters = reinterpret_cast<unsigned*>(ws);
  prm.part = reinterpret_cast<float*>(ws + pl.off_part);
  return attn::launch(pl, prm, batch, kv_heads, st, "decode_attention_noalloc");
}
