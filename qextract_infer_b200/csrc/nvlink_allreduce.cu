// One-shot all-reduce over NVLink peer memory, fused with the residual add and
// RMSNorm that follow the row-parallel o and down projections of the
// tensor-parallel decode step (new component: the reference has no tensor
// parallelism; NCCL's all-reduce is the baseline it replaces for small rows).
//
//   x[r] <- fp16(x[r] + fp16(sum over ranks of partial[r]))   (in place)
//   y[r]  = fp16((x[r] * rsqrt(mean(x[r]^2) + eps)) * w)
//
// Every rank owns a buffer shared with its peers through CUDA IPC:
//   data[2][max_rows][hidden] fp16   (double-buffered by epoch parity)
//   flags[max_rows] u32              (epoch of the row last published)
// and a private counter per row (CTA).  One CTA per row r, per call:
//   1. e = counter[r] + 1; copy partial[r] into data[e & 1][r] (local stores),
//      then one thread: fence.sys + st.release.sys flags[r] = e;
//   2. one thread per peer polls the peer's flags[r] (ld.acquire.sys over
//      NVLink) until it reaches e, bounded (2 s by %globaltimer unless
//      qx_nvlink_ar_set_timeout says otherwise; on timeout the device error
//      word gets QX_DEVERR_PEER_TIMEOUT and the row is reduced with whatever is
//      there, so the output of that call is undefined);
//   3. every rank sums the world rows in rank order (fp32, L2-only loads of
//      peer memory), rounds once, adds the residual, RMS-normalises; all ranks
//      compute identical bits.
// Parity makes a buffer reusable: a rank overwrites data[p] for epoch e + 2
// only after finishing e + 1, which needed every peer's flag e + 1, which each
// peer sets only after it finished reading epoch e.  Calls must not overlap on
// one rank (plain stream order, no programmatic dependent launch) and every
// rank must make the same sequence of calls.
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
  size_t data_bytes = 0;  // one parity half
  char* own = nullptr;    // this rank's shared buffer (data[2] then flags)
  uint32_t* counter = nullptr;  // private: epochs per row
  char* peer[MAX_WORLD] = {};   // every rank's buffer as mapped here (own included)
  bool opened[MAX_WORLD] = {};  // peer[r] is an IPC mapping to close at destroy
  uint64_t timeout_ns = 2000000000ull;  // limit of each wait for a peer's flag
};

struct Params {
  const __half* partial;
  __half* x;
  const __half* w;
  __half* y;
  const char* buf[MAX_WORLD];
  uint32_t* own_flags;
  uint32_t* counter;
  size_t data_bytes;
  uint64_t timeout_ns;
  int world, rank, hidden, flags_off;
  float eps;
};

static __device__ unsigned g_ar_error = 0;

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint64_t gtime() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

template <int VPT>
__global__ void __launch_bounds__(THREADS) ar_add_rmsnorm_kernel(const Params p) {
  // the next GEMV may start streaming its weights now; it waits for this
  // kernel's completion before reading x (calls of this kernel still never
  // overlap: the kernels between two of them wait for their predecessors)
  pdl_trigger();
  __shared__ float s_part[THREADS / 32];
  __shared__ float s_r;
  const int row = blockIdx.x, tid = threadIdx.x;
  const int h8 = p.hidden / 8;
  const uint32_t e = p.counter[row] + 1;
  const size_t off = size_t(e & 1) * p.data_bytes + size_t(row) * p.hidden * 2;
  // 1. publish this rank's partial row
  {
    const uint4* src = reinterpret_cast<const uint4*>(p.partial + size_t(row) * p.hidden);
    uint4* dst = reinterpret_cast<uint4*>(const_cast<char*>(p.buf[p.rank]) + off);
    for (int i = tid; i < h8; i += THREADS) dst[i] = src[i];
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence_system();
    st_release_sys(p.own_flags + row, e);
  }
  // 2. wait for every peer's row of this epoch
  if (tid < p.world && tid != p.rank) {
    const uint32_t* f = reinterpret_cast<const uint32_t*>(p.buf[tid] + p.flags_off) + row;
    if (ld_acquire_sys(f) < e) {
      const uint64_t t0 = gtime();
      while (ld_acquire_sys(f) < e) {
        if (gtime() - t0 > p.timeout_ns) {
          atomicOr(&g_ar_error, QX_DEVERR_PEER_TIMEOUT);
          break;
        }
      }
    }
  }
  __syncthreads();
  // 3. sum in rank order, residual add, RMSNorm
  uint4 xv[VPT];
  float ss = 0.f;
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int i = tid + v * THREADS;
    xv[v] = make_uint4(0u, 0u, 0u, 0u);
    if (i < h8) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      // every rank's 16 bytes requested at once (NVLink round trips overlap),
      // then summed in rank order
      uint4 d[MAX_WORLD];
#pragma unroll
      for (int r = 0; r < MAX_WORLD; ++r)
        d[r] = r < p.world ? __ldcg(reinterpret_cast<const uint4*>(p.buf[r] + off) + i)
                           : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
      for (int r = 0; r < MAX_WORLD; ++r) {
        if (r >= p.world) break;
        const uint32_t dd[4] = {d[r].x, d[r].y, d[r].z, d[r].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = h2_to_f2(dd[j]);
          acc[2 * j] += f.x;
          acc[2 * j + 1] += f.y;
        }
      }
      const uint4 xo = reinterpret_cast<const uint4*>(p.x + size_t(row) * p.hidden)[i];
      const uint32_t xd[4] = {xo.x, xo.y, xo.z, xo.w};
      uint32_t od[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 fx = h2_to_f2(xd[j]);
        const __half2 s2 = __floats2half2_rn(acc[2 * j], acc[2 * j + 1]);  // the all-reduced value
        const float2 fs = __half22float2(s2);
        const __half2 n2 = __floats2half2_rn(fx.x + fs.x, fx.y + fs.y);    // the residual add
        od[j] = *reinterpret_cast<const uint32_t*>(&n2);
        const float2 fn = __half22float2(n2);
        ss = fmaf(fn.x, fn.x, ss);
        ss = fmaf(fn.y, fn.y, ss);
      }
      xv[v] = make_uint4(od[0], od[1], od[2], od[3]);
      reinterpret_cast<uint4*>(p.x + size_t(row) * p.hidden)[i] = xv[v];
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
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int i = tid + v * THREADS;
    if (i < h8) {
      const uint4 wv = reinterpret_cast<const uint4*>(p.w)[i];
      const uint32_t vd[4] = {xv[v].x, xv[v].y, xv[v].z, xv[v].w}, wd[4] = {wv.x, wv.y, wv.z, wv.w};
      uint32_t od[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = h2_to_f2(vd[j]), g = h2_to_f2(wd[j]);
        const __half2 o = __floats2half2_rn((f.x * rr) * g.x, (f.y * rr) * g.y);
        od[j] = *reinterpret_cast<const uint32_t*>(&o);
      }
      reinterpret_cast<uint4*>(p.y + size_t(row) * p.hidden)[i] = make_uint4(od[0], od[1], od[2], od[3]);
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
  c->data_bytes = (size_t(max_rows) * hidden * 2 + 255) & ~size_t(255);
  const size_t flags_bytes = (size_t(max_rows) * 4 + 255) & ~size_t(255);
  cudaError_t e = cudaGetDevice(&c->device);
  if (e == cudaSuccess) e = cudaMalloc(&c->own, 2 * c->data_bytes + flags_bytes);
  if (e == cudaSuccess) e = cudaMemset(c->own, 0, 2 * c->data_bytes + flags_bytes);
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
  p.flags_off = int(2 * c->data_bytes);
  p.own_flags = reinterpret_cast<uint32_t*>(c->own + 2 * c->data_bytes);
  p.counter = c->counter;
  p.data_bytes = c->data_bytes;
  p.timeout_ns = c->timeout_ns;
  p.world = c->world;
  p.rank = c->rank;
  p.hidden = c->hidden;
  p.eps = eps;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int h8 = c->hidden / 8;
  if (h8 <= nvar::THREADS)
    nvar::ar_add_rmsnorm_kernel<1><<<rows, nvar::THREADS, 0, st>>>(p);
  else if (h8 <= 2 * nvar::THREADS)
    nvar::ar_add_rmsnorm_kernel<2><<<rows, nvar::THREADS, 0, st>>>(p);
  else
    nvar::ar_add_rmsnorm_kernel<4><<<rows, nvar::THREADS, 0, st>>>(p);
  return check_launch("nvlink_ar_add_rmsnorm");
}
