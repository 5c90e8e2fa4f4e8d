// One-shot all-reduce over NVLink peer memory, fused with the residual add and
// RMSNorm that follow the row-parallel o and down projections of the
// tensor-parallel decode step (new component: the reference has no tensor
// parallelism; NCCL's all-reduce is the baseline it replaces for small rows).
//
//   x[r] <- fp16(x[r] + fp16(sum over ranks of partial[r]))   (in place)
//   y[r]  = fp16((x[r] * rsqrt(mean(x[r]^2) + eps)) * w)
//
// Push protocol with the epoch carried in every word.  Every rank owns an
// inbox shared with its peers through CUDA IPC:
//   inbox[2][world][max_rows][hidden / 2] u64   (parity, source rank, row)
// whose words are (two fp16 of a partial row) | (epoch << 32).  One CTA per
// row r, per call, with e = counter[r] + 1:
//   1. the CTA reads its partial row and stores it, tagged with e, straight
//      into every peer's inbox[e & 1][rank][r] (relaxed system-scope 64-bit
//      stores over NVLink: no fence, no separate flag);
//   2. it polls its own, local inbox[e & 1][src][r] for every peer src until
//      each word carries e (a 64-bit access is single-copy atomic, so a word
//      with the right tag holds that epoch's data), bounded by the wait limit
//      (2 s by %globaltimer unless qx_nvlink_ar_set_timeout says otherwise; on
//      timeout the device error word gets QX_DEVERR_PEER_TIMEOUT and the row is
//      reduced with whatever is there, so that call's output is undefined);
//   3. it sums the world rows in rank order (fp32; its own from registers),
//      rounds once, adds the residual and RMS-normalises: every rank computes
//      identical bits.
// Only one-way NVLink writes sit on the critical path (the pull form it
// replaces paid a system fence, a remote flag poll and remote data loads).
// Parity makes an inbox slot reusable: a rank writes epoch e + 2 of row r into
// a peer's slot only after its own call with epoch e + 1 finished, which needed
// that peer's epoch e + 1 words, which the peer sends only after its call with
// epoch e (the reader of the slot) completed.  Calls must not overlap on one
// rank (stream order: each call waits for the previous kernel's completion
// before it touches the inbox or the counters) and every rank makes the same
// sequence of calls.
#include <algorithm>
#include <cstring>
#include <vector>

#include "qx_b200.h"
#include "qx_common.cuh"

namespace qx {
namespace nvar {

constexpr int MAX_WORLD = 8;
constexpr int THREADS = 256;

struct Ctx {
  int world = 0, rank = 0, max_rows = 0, hidden = 0, device = -1;
  size_t data_bytes = 0;  // one parity half of the inbox
  char* own = nullptr;    // this rank's inbox
  uint32_t* counter = nullptr;  // private: epochs per row
  char* peer[MAX_WORLD] = {};   // every rank's inbox as mapped here (own included)
  bool opened[MAX_WORLD] = {};  // peer[r] is an IPC mapping to close at destroy
  uint64_t timeout_ns = 2000000000ull;  // limit of each wait for a peer's words
};

struct Params {
  const __half* partial;
  __half* x;
  const __half* w;
  __half* y;
  char* buf[MAX_WORLD];
  uint32_t* counter;
  size_t data_bytes, src_bytes;  // parity half; one source rank's block
  uint64_t timeout_ns;
  int world, rank, hidden;
  float eps;
};

static __device__ unsigned g_ar_error = 0;

__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t gtime() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// VPT: 32-bit words (two fp16) of the row per thread, hidden / 2 <= VPT * THREADS
template <int VPT>
__global__ void __launch_bounds__(THREADS) ar_add_rmsnorm_kernel(const Params p) {
  // the next kernel may launch now; it waits for this one's completion before
  // it reads x or y.  This kernel waits for its predecessor (the projection
  // that wrote `partial`, and transitively the previous call) before it reads
  // anything.
  pdl_trigger();
  pdl_wait();
  __shared__ float s_part[THREADS / 32];
  __shared__ float s_r;
  const int row = blockIdx.x, tid = threadIdx.x;
  const int h2 = p.hidden / 2;
  const uint32_t e = p.counter[row] + 1;
  const uint64_t tag = uint64_t(e) << 32;
  const size_t slot = size_t(e & 1) * p.data_bytes + size_t(row) * h2 * 8;

  // 1. this rank's partial row, pushed into every peer's inbox
  uint32_t mine[VPT];
  {
    const uint32_t* src = reinterpret_cast<const uint32_t*>(p.partial + size_t(row) * p.hidden);
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      const int i = tid + v * THREADS;
      mine[v] = i < h2 ? src[i] : 0u;
    }
  }
  for (int r = 0; r < p.world; ++r) {
    if (r == p.rank) continue;
    uint64_t* dst = reinterpret_cast<uint64_t*>(p.buf[r] + slot + size_t(p.rank) * p.src_bytes);
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      const int i = tid + v * THREADS;
      if (i < h2) st_relaxed_sys_u64(dst + i, tag | mine[v]);
    }
  }

  // 2./3. every peer's words from the local inbox, summed in rank order
  float acc[VPT][2];
#pragma unroll
  for (int v = 0; v < VPT; ++v) acc[v][0] = acc[v][1] = 0.f;
  uint64_t t0 = 0;
  bool late = false;  // this thread's wait ran out: stop waiting
  for (int r = 0; r < p.world; ++r) {
    uint32_t d[VPT];
    if (r == p.rank) {
#pragma unroll
      for (int v = 0; v < VPT; ++v) d[v] = mine[v];
    } else {
      const uint64_t* in = reinterpret_cast<const uint64_t*>(p.buf[p.rank] + slot + size_t(r) * p.src_bytes);
      uint64_t wv[VPT];
#pragma unroll
      for (int v = 0; v < VPT; ++v) {
        const int i = tid + v * THREADS;
        wv[v] = i < h2 ? ld_relaxed_sys_u64(in + i) : tag;
      }
#pragma unroll
      for (int v = 0; v < VPT; ++v) {
        const int i = tid + v * THREADS;
        while (!late && uint32_t(wv[v] >> 32) != e) {
          const uint64_t now = gtime();
          if (t0 == 0) t0 = now;
          if (now - t0 > p.timeout_ns) {
            atomicOr(&g_ar_error, QX_DEVERR_PEER_TIMEOUT);
            late = true;
            break;
          }
          wv[v] = ld_relaxed_sys_u64(in + i);
        }
        d[v] = uint32_t(wv[v]);
      }
    }
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      const float2 f = h2_to_f2(d[v]);
      acc[v][0] += f.x;
      acc[v][1] += f.y;
    }
  }

  // residual add (the all-reduced value rounded once, then the add rounded)
  uint32_t xv[VPT];
  float ss = 0.f;
  uint32_t* xrow = reinterpret_cast<uint32_t*>(p.x + size_t(row) * p.hidden);
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int i = tid + v * THREADS;
    xv[v] = 0u;
    if (i < h2) {
      const float2 fx = h2_to_f2(xrow[i]);
      const float2 fs = __half22float2(__floats2half2_rn(acc[v][0], acc[v][1]));
      const __half2 n2 = __floats2half2_rn(fx.x + fs.x, fx.y + fs.y);
      xv[v] = *reinterpret_cast<const uint32_t*>(&n2);
      xrow[i] = xv[v];
      const float2 fn = __half22float2(n2);
      ss = fmaf(fn.x, fn.x, ss);
      ss = fmaf(fn.y, fn.y, ss);
    }
  }
  ss = warp_sum(ss);
  if ((tid & 31) == 0) s_part[tid >> 5] = ss;
  __syncthreads();
  if (tid < 32) {
    float t = tid < THREADS / 32 ? s_part[tid] : 0.f;
    t = warp_sum(t);
    if (tid == 0) s_r = 1.0f / sqrtf(t * (1.0f / p.hidden) + p.eps);
  }
  __syncthreads();
  const float rr = s_r;
  const uint32_t* wrow = reinterpret_cast<const uint32_t*>(p.w);
  uint32_t* yrow = reinterpret_cast<uint32_t*>(p.y + size_t(row) * p.hidden);
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int i = tid + v * THREADS;
    if (i < h2) {
      const float2 f = h2_to_f2(xv[v]), g = h2_to_f2(wrow[i]);
      const __half2 o = __floats2half2_rn((f.x * rr) * g.x, (f.y * rr) * g.y);
      yrow[i] = *reinterpret_cast<const uint32_t*>(&o);
    }
  }
  if (tid == 0) p.counter[row] = e;
}

}  // namespace nvar

int nvar_device_error(unsigned* code, int reset) {
  QX_CUDA_TRY(cudaMemcpyFromSymbol(code, nvar::g_ar_error, sizeof(unsigned)), "get_device_error: read");
  if (reset) {
    const unsigned zero = 0;
    QX_CUDA_TRY(cudaMemcpyToSymbol(nvar::g_ar_error, &zero, sizeof(unsigned)), "get_device_error: reset");
  }
  return QX_OK;
}

}  // namespace qx

using namespace qx;

extern "C" size_t qx_nvlink_ar_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

extern "C" int qx_nvlink_ar_create(int world, int rank, int max_rows, int hidden, void** ctx_out,
                                   void* handle_out) {
  QX_REQUIRE(ctx_out && handle_out, "nvlink_ar_create: null output");
  QX_REQUIRE(world >= 2 && world <= nvar::MAX_WORLD && rank >= 0 && rank < world,
             "nvlink_ar_create: world=%d rank=%d (2..8 ranks)", world, rank);
  QX_REQUIRE(max_rows >= 1 && max_rows <= 1024 && hidden % 8 == 0 && hidden >= 8 && hidden <= 8192,
             "nvlink_ar_create: max_rows=%d hidden=%d (hidden %% 8 == 0, <= 8192)", max_rows, hidden);
  auto* c = new nvar::Ctx();
  c->world = world;
  c->rank = rank;
  c->max_rows = max_rows;
  c->hidden = hidden;
  // inbox: [2 parities][world sources][max_rows][hidden / 2] tagged 64-bit words
  c->data_bytes = size_t(world) * max_rows * (hidden / 2) * 8;
  cudaError_t e = cudaGetDevice(&c->device);
  if (e == cudaSuccess) e = cudaMalloc(&c->own, 2 * c->data_bytes);
  if (e == cudaSuccess) e = cudaMemset(c->own, 0, 2 * c->data_bytes);  // epoch 0: never a live tag
  if (e == cudaSuccess) e = cudaMalloc(&c->counter, size_t(max_rows) * 4);
  if (e == cudaSuccess) e = cudaMemset(c->counter, 0, size_t(max_rows) * 4);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, c->own);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    if (c->own) cudaFree(c->own);
    if (c->counter) cudaFree(c->counter);
    delete c;
    return fail(QX_ERR_CUDA, "nvlink_ar_create: %s", cudaGetErrorString(e));
  }
  std::memcpy(handle_out, &h, sizeof(h));
  c->peer[rank] = c->own;
  *ctx_out = c;
  return QX_OK;
}

extern "C" int qx_nvlink_ar_open(void* ctx, const void* handles) {
  QX_REQUIRE(ctx && handles, "nvlink_ar_open: null argument");
  auto* c = static_cast<nvar::Ctx*>(ctx);
  const char* hb = static_cast<const char*>(handles);
  for (int r = 0; r < c->world; ++r) {
    if (r == c->rank || c->opened[r]) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, hb + size_t(r) * sizeof(h), sizeof(h));
    void* ptr = nullptr;
    QX_CUDA_TRY(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess),
                "nvlink_ar_open: cudaIpcOpenMemHandle");
    c->peer[r] = static_cast<char*>(ptr);
    c->opened[r] = true;
  }
  return QX_OK;
}

extern "C" int qx_nvlink_ar_open_local(void* ctx, void* const* ctxs) {
  QX_REQUIRE(ctx && ctxs, "nvlink_ar_open_local: null argument");
  auto* c = static_cast<nvar::Ctx*>(ctx);
  for (int r = 0; r < c->world; ++r) {
    if (r == c->rank) continue;
    const auto* o = static_cast<const nvar::Ctx*>(ctxs[r]);
    QX_REQUIRE(o && o->world == c->world && o->rank == r && o->max_rows == c->max_rows &&
                   o->hidden == c->hidden,
               "nvlink_ar_open_local: context %d is not rank %d of the same communicator", r, r);
    if (o->device != c->device) {
      int can = 0;
      QX_CUDA_TRY(cudaDeviceCanAccessPeer(&can, c->device, o->device), "nvlink_ar_open_local: peer query");
      QX_REQUIRE(can, "nvlink_ar_open_local: device %d cannot reach device %d", c->device, o->device);
      const cudaError_t e = cudaDeviceEnablePeerAccess(o->device, 0);
      if (e == cudaErrorPeerAccessAlreadyEnabled)
        cudaGetLastError();
      else
        QX_CUDA_TRY(e, "nvlink_ar_open_local: enable peer access");
    }
    c->peer[r] = o->own;
  }
  return QX_OK;
}

extern "C" int qx_nvlink_ar_set_timeout(void* ctx, int64_t timeout_ns) {
  QX_REQUIRE(ctx, "nvlink_ar_set_timeout: null context");
  QX_REQUIRE(timeout_ns > 0, "nvlink_ar_set_timeout: timeout must be positive (ns)");
  static_cast<nvar::Ctx*>(ctx)->timeout_ns = uint64_t(timeout_ns);
  return QX_OK;
}

extern "C" int qx_nvlink_ar_destroy(void* ctx) {
  if (!ctx) return QX_OK;
  auto* c = static_cast<nvar::Ctx*>(ctx);
  cudaDeviceSynchronize();
  for (int r = 0; r < c->world; ++r)
    if (c->opened[r]) cudaIpcCloseMemHandle(c->peer[r]);
  if (c->own) cudaFree(c->own);
  if (c->counter) cudaFree(c->counter);
  delete c;
  return QX_OK;
}

extern "C" int qx_nvlink_ar_add_rmsnorm(void* ctx, const void* partial, void* x, const void* weight,
                                        void* y, int rows, float eps, qx_stream_t stream) {
  QX_REQUIRE(ctx, "nvlink_ar_add_rmsnorm: null context");
  auto* c = static_cast<nvar::Ctx*>(ctx);
  QX_REQUIRE(rows >= 0 && rows <= c->max_rows, "nvlink_ar_add_rmsnorm: rows=%d > max_rows=%d", rows,
             c->max_rows);
  if (rows == 0) return QX_OK;
  QX_REQUIRE(partial && x && weight && y, "nvlink_ar_add_rmsnorm: null tensor pointer");
  QX_REQUIRE(aligned(partial, 16) && aligned(x, 16) && aligned(weight, 16) && aligned(y, 16),
             "nvlink_ar_add_rmsnorm: tensors must be 16-byte aligned");
  for (int r = 0; r < c->world; ++r)
    QX_REQUIRE(c->peer[r], "nvlink_ar_add_rmsnorm: peer %d not opened (qx_nvlink_ar_open)", r);
  nvar::Params p{};
  p.partial = static_cast<const __half*>(partial);
  p.x = static_cast<__half*>(x);
  p.w = static_cast<const __half*>(weight);
  p.y = static_cast<__half*>(y);
  for (int r = 0; r < c->world; ++r) p.buf[r] = c->peer[r];
  p.counter = c->counter;
  p.data_bytes = c->data_bytes;
  p.src_bytes = size_t(c->max_rows) * (c->hidden / 2) * 8;
  p.timeout_ns = c->timeout_ns;
  p.world = c->world;
  p.rank = c->rank;
  p.hidden = c->hidden;
  p.eps = eps;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int h2 = c->hidden / 2;
  const dim3 grid(rows), block(nvar::THREADS);
  cudaError_t le;
  if (h2 <= 2 * nvar::THREADS)
    le = launch_pdl(nvar::ar_add_rmsnorm_kernel<2>, grid, block, 0, st, p);
  else if (h2 <= 4 * nvar::THREADS)
    le = launch_pdl(nvar::ar_add_rmsnorm_kernel<4>, grid, block, 0, st, p);
  else if (h2 <= 8 * nvar::THREADS)
    le = launch_pdl(nvar::ar_add_rmsnorm_kernel<8>, grid, block, 0, st, p);
  else
    le = launch_pdl(nvar::ar_add_rmsnorm_kernel<16>, grid, block, 0, st, p);
  QX_CUDA_TRY(le, "nvlink_ar_add_rmsnorm: launch");
  return check_launch("nvlink_ar_add_rmsnorm");
}
