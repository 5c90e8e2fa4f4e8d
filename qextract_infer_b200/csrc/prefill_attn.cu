// Prefill attention over the StreamingLLM ring: the queries of one prompt
// chunk attend to the tokens the ring already holds (the sink slots and the
// previous window, read in place) and to the chunk's own keys, causally, with
// the sink + window mask
//   key kp is visible to query p  <=>  kp <= p  and  (kp < sink or kp > p - window)
// (the rule HF Qwen3 + the reference's cache apply when a chunk is attended
// before it is appended: qextract/kv_cache.py:96-112, ring_buffer.cu:143-200
// give the cache's logical order; the positions of its slots follow from the
// ring's write rule, ring_buffer.cu:115-141).
//
// Flash-attention form: one CTA = 4 warps = 64 query positions of one query
// head; each warp owns 16 of them.  Key tiles of 64 (cache slots first, then
// the chunk's keys up to the block's last position) are staged by cp.async
// into XOR-swizzled shared memory, double buffered and shared by the warps;
// S = Q K^T and O += P V run on the tensor cores (mma.sync m16n8k16, fp32
// accumulation) with an online softmax in the log2 domain.  GQA: the query
// heads of one KV head read the same K/V tiles (from L2 after the first).
#include <algorithm>
#include <cmath>
#include <mutex>

#include "qx_b200.h"
#include "qx_common.cuh"

namespace qx {
namespace pattn {

constexpr int D = 128;
constexpr int WARPS = 4;
constexpr int THREADS = WARPS * 32;
constexpr int QROWS = WARPS * 16;          // query positions per CTA
constexpr int KT = 64;                     // keys per tile
constexpr int ROW_BYTES = D * 2;           // 256
constexpr int TILE_BYTES = KT * ROW_BYTES;  // 16 KB
constexpr int SMEM = 2 * 2 * TILE_BYTES;   // 2 stages x (K, V) = 64 KB

struct Params {
  const __half* q;      // [B][n][Hq][D]
  const __half* kn;     // [B][n][Hkv][D]  the chunk's keys
  const __half* vn;
  const __half* kc;     // [B][cap][Hkv][D]  the ring before the chunk
  const __half* vc;
  __half* out;          // [B][n][Hq][D]
  int n, Hq, Hkv, G, cap, sink, window;
  int valid;            // ring slots holding tokens (a physical prefix)
  long long count;      // tokens written before the chunk: the chunk's first position
  float scale_log2;
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
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
// byte offset of 16-byte chunk `ch` of tile row `r` (XOR swizzle over 8 rows)
__device__ __forceinline__ uint32_t swz(int r, int ch) {
  return uint32_t(r * ROW_BYTES + ((ch ^ (r & 7)) << 4));
}

__global__ void __launch_bounds__(THREADS, 3) prefill_attn_kernel(const Params p) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int h = blockIdx.y, b = blockIdx.z, kvh = h / p.G;
  const int r0 = blockIdx.x * QROWS;
  const int rowA = r0 + warp * 16 + g, rowB = rowA + 8;  // this lane's query rows in the chunk
  const int c0 = int(p.count);
  const int posA = c0 + rowA, posB = c0 + rowB;
  const int last = min(p.n, r0 + QROWS) - 1;  // the CTA's last query row
  const int ncache = (p.valid + KT - 1) / KT;
  const int ntiles = ncache + last / KT + 1;  // cache tiles, then the chunk's keys up to `last`
  const uint32_t sbase = smem_u32(smem);

  auto issue = [&](int t, int stage) {
    const uint32_t ks = sbase + stage * 2 * TILE_BYTES, vs = ks + TILE_BYTES;
    const bool cache = t < ncache;
    const int base = cache ? t * KT : (t - ncache) * KT;
    const int lim = cache ? p.valid : p.n;
    const __half* kb = cache ? p.kc : p.kn;
    const __half* vb = cache ? p.vc : p.vn;
    const size_t rows_b = cache ? size_t(p.cap) : size_t(p.n);
#pragma unroll
    for (int i = 0; i < (KT * 16) / THREADS; ++i) {
      const int idx = i * THREADS + tid, r = idx >> 4, ch = idx & 15;
      const int key = base + r;
      const bool ok = key < lim;
      const size_t off = ok ? ((size_t(b) * rows_b + key) * p.Hkv + kvh) * D + ch * 8 : 0;
      cp_async16(ks + swz(r, ch), kb + off, ok ? 16 : 0);
      cp_async16(vs + swz(r, ch), vb + off, ok ? 16 : 0);
    }
    cp_async_commit();
  };

  issue(0, 0);
  if (ntiles > 1) issue(1, 1);
  else cp_async_commit();

  // Q fragments of rows A and B (rows past the chunk read as zero)
  uint32_t qa[8][4];
  {
    const bool okA = rowA < p.n, okB = rowB < p.n;
    const __half* qA = p.q + ((size_t(b) * p.n + (okA ? rowA : 0)) * p.Hq + h) * D;
    const __half* qB = p.q + ((size_t(b) * p.n + (okB ? rowB : 0)) * p.Hq + h) * D;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int d0 = kk * 16 + 2 * c;
      qa[kk][0] = okA ? *reinterpret_cast<const uint32_t*>(qA + d0) : 0u;
      qa[kk][1] = okB ? *reinterpret_cast<const uint32_t*>(qB + d0) : 0u;
      qa[kk][2] = okA ? *reinterpret_cast<const uint32_t*>(qA + d0 + 8) : 0u;
      qa[kk][3] = okB ? *reinterpret_cast<const uint32_t*>(qB + d0 + 8) : 0u;
    }
  }

  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  const int mi = lane >> 3, ri = lane & 7;

  for (int t = 0; t < ntiles; ++t) {
    cp_async_wait<1>();
    __syncthreads();  // tile t is in shared memory for every warp
    const uint32_t ks = sbase + (t & 1) * 2 * TILE_BYTES, vs = ks + TILE_BYTES;

    // S = Q K^T over the tile's 64 keys (8 n-tiles of 8)
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
      for (int j2 = 0; j2 < 4; ++j2) {
        uint32_t bk[4];
        ldsm_x4(bk, ks + swz(j2 * 16 + 8 * (mi >> 1) + ri, 2 * kk + (mi & 1)));
        mma_16816(s[2 * j2], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], bk[0], bk[1]);
        mma_16816(s[2 * j2 + 1], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], bk[2], bk[3]);
      }
    }
    // positions of this lane's 16 keys and the mask.  A window slot s holds
    // position (c0-1) - ((c0-1-s) mod window): ascending with s except past
    // the newest token, where it drops by `window`.  One modulo per tile: the
    // position of the tile's first window slot, the others stepped from it
    // (a division only for slots past the drop).
    const bool cache = t < ncache;
    const int sb = max(t * KT, p.sink);  // the tile's first window slot (if any)
    const int kpb = cache && sb < p.valid ? (c0 - 1) - ((c0 - 1 - sb) % p.window) : 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e1 = 0; e1 < 2; ++e1) {
        const int kj = j * 8 + 2 * c + e1;
        int kp;
        bool okk;
        if (cache) {
          const int slot = t * KT + kj;
          okk = slot < p.valid;
          int kw = kpb + (slot - sb);
          if (kw > c0 - 1) kw -= p.window * ((kw - (c0 - 1) + p.window - 1) / p.window);
          kp = slot < p.sink ? slot : kw;
        } else {
          const int idx = (t - ncache) * KT + kj;
          okk = idx < p.n;
          kp = c0 + idx;
        }
        const bool vA = okk && kp <= posA && (kp < p.sink || kp > posA - p.window);
        const bool vB = okk && kp <= posB && (kp < p.sink || kp > posB - p.window);
        s[j][e1] = vA ? s[j][e1] * p.scale_log2 : -INFINITY;
        s[j][2 + e1] = vB ? s[j][2 + e1] * p.scale_log2 : -INFINITY;
      }
    }
    // online softmax (rows A: e = 0, 1; rows B: e = 2, 3)
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      mx0 = fmaxf(mx0, fmaxf(s[j][0], s[j][1]));
      mx1 = fmaxf(mx1, fmaxf(s[j][2], s[j][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m_r[0], mx0), mn1 = fmaxf(m_r[1], mx1);
    // a row with no visible key so far keeps zero weights (no inf - inf)
    const float mb0 = mn0 == -INFINITY ? 0.f : mn0, mb1 = mn1 == -INFINITY ? 0.f : mn1;
    const float al0 = exp2f(m_r[0] - mb0), al1 = exp2f(m_r[1] - mb1);
    m_r[0] = mn0;
    m_r[1] = mn1;
    float ls0 = 0.f, ls1 = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      s[j][0] = exp2f(s[j][0] - mb0);
      s[j][1] = exp2f(s[j][1] - mb0);
      s[j][2] = exp2f(s[j][2] - mb1);
      s[j][3] = exp2f(s[j][3] - mb1);
      ls0 += s[j][0] + s[j][1];
      ls1 += s[j][2] + s[j][3];
    }
    l_r[0] = l_r[0] * al0 + ls0;
    l_r[1] = l_r[1] * al1 + ls1;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      o[j][0] *= al0;
      o[j][1] *= al0;
      o[j][2] *= al1;
      o[j][3] *= al1;
    }
    // O += P V: 4 k-steps of 16 keys x 16 n-tiles of 8 head dims
#pragma unroll
    for (int kq = 0; kq < 4; ++kq) {
      const uint32_t pa0 = pack_h2(s[2 * kq][0], s[2 * kq][1]);
      const uint32_t pa1 = pack_h2(s[2 * kq][2], s[2 * kq][3]);
      const uint32_t pa2 = pack_h2(s[2 * kq + 1][0], s[2 * kq + 1][1]);
      const uint32_t pa3 = pack_h2(s[2 * kq + 1][2], s[2 * kq + 1][3]);
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        uint32_t bv[4];
        ldsm_x4_t(bv, vs + swz(kq * 16 + 8 * (mi & 1) + ri, 2 * jj + (mi >> 1)));
        mma_16816(o[2 * jj], pa0, pa1, pa2, pa3, bv[0], bv[1]);
        mma_16816(o[2 * jj + 1], pa0, pa1, pa2, pa3, bv[2], bv[3]);
      }
    }
    __syncthreads();  // every warp is done with this stage: refill it
    if (t + 2 < ntiles) issue(t + 2, t & 1);
    else cp_async_commit();
  }
  cp_async_wait<0>();

  l_r[0] += __shfl_xor_sync(0xffffffffu, l_r[0], 1);
  l_r[0] += __shfl_xor_sync(0xffffffffu, l_r[0], 2);
  l_r[1] += __shfl_xor_sync(0xffffffffu, l_r[1], 1);
  l_r[1] += __shfl_xor_sync(0xffffffffu, l_r[1], 2);
  const float inv0 = 1.f / l_r[0], inv1 = 1.f / l_r[1];
  if (rowA < p.n) {
    __half* oA = p.out + ((size_t(b) * p.n + rowA) * p.Hq + h) * D;
#pragma unroll
    for (int j = 0; j < 16; ++j)
      *reinterpret_cast<uint32_t*>(oA + 8 * j + 2 * c) = pack_h2(o[j][0] * inv0, o[j][1] * inv0);
  }
  if (rowB < p.n) {
    __half* oB = p.out + ((size_t(b) * p.n + rowB) * p.Hq + h) * D;
#pragma unroll
    for (int j = 0; j < 16; ++j)
      *reinterpret_cast<uint32_t*>(oB + 8 * j + 2 * c) = pack_h2(o[j][2] * inv1, o[j][3] * inv1);
  }
}

}  // namespace pattn
}  // namespace qx

using namespace qx;

extern "C" int qx_prefill_attention(const void* q, const void* k_new, const void* v_new,
                                    const void* k_cache, const void* v_cache, void* out, int batch,
                                    int n, int q_heads, int kv_heads, int head_dim, int sink,
                                    int window, int64_t count, float softmax_scale,
                                    qx_stream_t stream) {
  QX_REQUIRE(batch > 0 && n > 0 && q_heads > 0 && kv_heads > 0 && q_heads % kv_heads == 0,
             "prefill_attention: bad sizes batch=%d n=%d heads q=%d kv=%d", batch, n, q_heads, kv_heads);
  QX_REQUIRE(head_dim == pattn::D, "prefill_attention: head_dim=%d unsupported (128)", head_dim);
  QX_REQUIRE(sink >= 0 && window >= 1, "prefill_attention: sink=%d window=%d", sink, window);
  QX_REQUIRE(count >= 0 && count + n < (int64_t(1) << 31), "prefill_attention: positions past 2^31");
  QX_REQUIRE(batch <= 65535 && q_heads <= 65535, "prefill_attention: batch or heads too large");
  QX_REQUIRE(q && k_new && v_new && k_cache && v_cache && out, "prefill_attention: null pointer");
  QX_REQUIRE(aligned(k_new, 16) && aligned(v_new, 16) && aligned(k_cache, 16) && aligned(v_cache, 16) &&
                 aligned(q, 4) && aligned(out, 4),
             "prefill_attention: misaligned tensors");
  pattn::Params prm{};
  prm.q = static_cast<const __half*>(q);
  prm.kn = static_cast<const __half*>(k_new);
  prm.vn = static_cast<const __half*>(v_new);
  prm.kc = static_cast<const __half*>(k_cache);
  prm.vc = static_cast<const __half*>(v_cache);
  prm.out = static_cast<__half*>(out);
  prm.n = n;
  prm.Hq = q_heads;
  prm.Hkv = kv_heads;
  prm.G = q_heads / kv_heads;
  prm.cap = sink + window;
  prm.sink = sink;
  prm.window = window;
  prm.valid = int(count <= sink ? count : sink + std::min<int64_t>(count - sink, window));
  prm.count = count;
  const float scale = softmax_scale > 0.f ? softmax_scale : 1.0f / sqrtf(float(head_dim));
  prm.scale_log2 = scale * 1.4426950408889634f;
  {
    static std::mutex mu;
    static bool done[64] = {};
    int dev = 0;
    QX_CUDA_TRY(cudaGetDevice(&dev), "prefill_attention: cudaGetDevice");
    QX_REQUIRE(dev >= 0 && dev < 64, "prefill_attention: device index %d unsupported", dev);
    std::lock_guard<std::mutex> lk(mu);
    if (!done[dev]) {
      QX_CUDA_TRY(cudaFuncSetAttribute(pattn::prefill_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       pattn::SMEM),
                  "prefill_attention: set smem limit");
      done[dev] = true;
    }
  }
  const dim3 grid((n + pattn::QROWS - 1) / pattn::QROWS, q_heads, batch);
  pattn::prefill_attn_kernel<<<grid, pattn::THREADS, pattn::SMEM, reinterpret_cast<cudaStream_t>(stream)>>>(prm);
  return check_launch("prefill_attention");
}
