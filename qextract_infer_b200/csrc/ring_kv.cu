// StreamingLLM ring KV cache: multi-token / batched append, logical slot
// list and materialising gather.
//
// Index rules are the reference's (csrc/kv_cache/ring_buffer.cu:115-123,
// 149-173; qextract/kv_cache.py:114-152):
//   write_pos(c)    = c < S ? c : S + (c - S) % W
//   valid_length(c) = c <= S ? c : S + min(c - S, W)
//   logical order   = sinks 0..min(c,S)-1, then ring slots S + (start + i) % W
//                     with start = 0 if c - S <= W else (c - S) % W.
// The reference appends one token per launch with the slot computed on the
// host, and gathers through a host-built index list copied with a blocking
// cudaMemcpy.  Here the slot math runs on the device: one launch appends a
// whole chunk for a whole batch, and the gather needs no host round trip.
// For a chunk of T tokens only the last writer of each slot is stored
// (token j of the ring region survives iff j >= T - W), which leaves the
// cache byte-identical to T sequential single-token appends.
#include <algorithm>

#include "qx_b200.h"
#include "qx_common.cuh"

namespace qx {
namespace ring {

__host__ __device__ __forceinline__ int64_t write_pos(int64_t c, int sink, int window) {
  return c < sink ? c : sink + (c - sink) % window;
}

__host__ __device__ __forceinline__ int64_t valid_length(int64_t c, int sink, int window) {
  return c <= sink ? c : sink + ((c - sink) < window ? (c - sink) : int64_t(window));
}

// logical index i (0 <= i < valid_length) -> physical slot
__device__ __forceinline__ int32_t logical_slot(int64_t i, int64_t c, int sink, int window) {
  const int64_t ns = c < sink ? c : sink;
  if (i < ns) return int32_t(i);
  const int64_t f = c - sink;
  const int64_t start = f <= window ? 0 : f % window;
  return int32_t(sink + (start + (i - ns)) % window);
}

// Vectorised append: one work item = one 16-byte chunk of one kept token.
__global__ void append_vec_kernel(uint4* __restrict__ kc, uint4* __restrict__ vc,
                                  const uint4* __restrict__ nk, const uint4* __restrict__ nv,
                                  int batch, int tokens, int first_kept_ring, int row8, int sink,
                                  int window, int64_t count, int64_t items) {
  const int cap = sink + window;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t it = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; it < items; it += stride) {
    const int64_t e = it % row8;
    const int64_t bt = it / row8;  // (b, j) over all tokens of the chunk
    const int j = int(bt % tokens);
    const int b = int(bt / tokens);
    const int64_t cj = count + j;
    if (cj >= sink && j < first_kept_ring) continue;  // overwritten later in this chunk
    const int64_t slot = write_pos(cj, sink, window);
    const int64_t dst = (int64_t(b) * cap + slot) * row8 + e;
    const int64_t src = (int64_t(b) * tokens + j) * row8 + e;
    kc[dst] = __ldg(nk + src);
    vc[dst] = __ldg(nv + src);
  }
}

__global__ void append_scalar_kernel(__half* __restrict__ kc, __half* __restrict__ vc,
                                     const __half* __restrict__ nk, const __half* __restrict__ nv,
                                     int batch, int tokens, int first_kept_ring, int row, int sink,
                                     int window, int64_t count, int64_t items) {
  const int cap = sink + window;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t it = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; it < items; it += stride) {
    const int64_t e = it % row;
    const int64_t bt = it / row;
    const int j = int(bt % tokens);
    const int b = int(bt / tokens);
    const int64_t cj = count + j;
    if (cj >= sink && j < first_kept_ring) continue;
    const int64_t slot = write_pos(cj, sink, window);
    kc[(int64_t(b) * cap + slot) * row + e] = nk[(int64_t(b) * tokens + j) * row + e];
    vc[(int64_t(b) * cap + slot) * row + e] = nv[(int64_t(b) * tokens + j) * row + e];
  }
}

__global__ void slot_indices_kernel(int32_t* __restrict__ out, int64_t n, int sink, int window,
                                    int64_t count) {
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
    out[i] = logical_slot(i, count, sink, window);
}

__global__ void gather_vec_kernel(const uint4* __restrict__ kc, const uint4* __restrict__ vc,
                                  uint4* __restrict__ ko, uint4* __restrict__ vo, int row8,
                                  int sink, int window, int64_t count, int64_t valid,
                                  int64_t items) {
  const int cap = sink + window;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t it = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; it < items; it += stride) {
    const int64_t e = it % row8;
    const int64_t bi = it / row8;
    const int64_t i = bi % valid;
    const int64_t b = bi / valid;
    const int64_t slot = logical_slot(i, count, sink, window);
    ko[it] = __ldg(kc + (b * cap + slot) * row8 + e);
    vo[it] = __ldg(vc + (b * cap + slot) * row8 + e);
  }
}

__global__ void gather_scalar_kernel(const __half* __restrict__ kc, const __half* __restrict__ vc,
                                     __half* __restrict__ ko, __half* __restrict__ vo, int row,
                                     int sink, int window, int64_t count, int64_t valid,
                                     int64_t items) {
  const int cap = sink + window;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t it = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; it < items; it += stride) {
    const int64_t e = it % row;
    const int64_t bi = it / row;
    const int64_t i = bi % valid;
    const int64_t b = bi / valid;
    const int64_t slot = logical_slot(i, count, sink, window);
    ko[it] = kc[(b * cap + slot) * row + e];
    vo[it] = vc[(b * cap + slot) * row + e];
  }
}

static inline unsigned grid_for(int64_t items) {
  const int64_t maxb = int64_t(device_sm_count()) * 8;
  return unsigned(std::max<int64_t>(1, std::min<int64_t>((items + 255) / 256, maxb)));
}

}  // namespace ring
}  // namespace qx

using namespace qx;

extern "C" int qx_ring_append(void* k_cache, void* v_cache, const void* new_k, const void* new_v,
                              int batch, int tokens, int kv_heads, int head_dim, int sink,
                              int window, int64_t count, qx_stream_t stream) {
  QX_REQUIRE(batch > 0 && tokens >= 0 && kv_heads > 0 && head_dim > 0,
             "ring_append: bad sizes batch=%d tokens=%d kv_heads=%d head_dim=%d", batch, tokens,
             kv_heads, head_dim);
  QX_REQUIRE(sink >= 0 && window >= 1, "ring_append: sink=%d window=%d", sink, window);
  QX_REQUIRE(count >= 0, "ring_append: negative count");
  if (tokens == 0) return QX_OK;
  QX_REQUIRE(k_cache && v_cache && new_k && new_v, "ring_append: null pointer");
  // ring-region tokens j < T - W are overwritten by later tokens of the same chunk
  const int first_kept_ring = std::max(0, tokens - window);
  const int row = kv_heads * head_dim;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (row % 8 == 0 && aligned(k_cache, 16) && aligned(v_cache, 16) && aligned(new_k, 16) &&
      aligned(new_v, 16)) {
    const int row8 = row / 8;
    const int64_t items = int64_t(batch) * tokens * row8;
    ring::append_vec_kernel<<<ring::grid_for(items), 256, 0, st>>>(
        static_cast<uint4*>(k_cache), static_cast<uint4*>(v_cache),
        static_cast<const uint4*>(new_k), static_cast<const uint4*>(new_v), batch, tokens,
        first_kept_ring, row8, sink, window, count, items);
  } else {
    const int64_t items = int64_t(batch) * tokens * row;
    ring::append_scalar_kernel<<<ring::grid_for(items), 256, 0, st>>>(
        static_cast<__half*>(k_cache), static_cast<__half*>(v_cache),
        static_cast<const __half*>(new_k), static_cast<const __half*>(new_v), batch, tokens,
        first_kept_ring, row, sink, window, count, items);
  }
  return check_launch("ring_append");
}

extern "C" int64_t qx_ring_slot_indices(int32_t* slots, int sink, int window, int64_t count,
                                        qx_stream_t stream) {
  QX_REQUIRE(sink >= 0 && window >= 1 && count >= 0, "ring_slot_indices: sink=%d window=%d",
             sink, window);
  const int64_t n = ring::valid_length(count, sink, window);
  if (n == 0) return 0;
  QX_REQUIRE(slots, "ring_slot_indices: null output");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  ring::slot_indices_kernel<<<ring::grid_for(n), 256, 0, st>>>(slots, n, sink, window, count);
  const int rc = check_launch("ring_slot_indices");
  return rc == QX_OK ? n : rc;
}

extern "C" int qx_ring_gather(const void* k_cache, const void* v_cache, void* k_out, void* v_out,
                              int batch, int kv_heads, int head_dim, int sink, int window,
                              int64_t count, qx_stream_t stream) {
  QX_REQUIRE(batch > 0 && kv_heads > 0 && head_dim > 0 && sink >= 0 && window >= 1 && count >= 0,
             "ring_gather: bad arguments");
  const int64_t valid = ring::valid_length(count, sink, window);
  if (valid == 0) return QX_OK;
  QX_REQUIRE(k_cache && v_cache && k_out && v_out, "ring_gather: null pointer");
  const int row = kv_heads * head_dim;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (row % 8 == 0 && aligned(k_cache, 16) && aligned(v_cache, 16) && aligned(k_out, 16) &&
      aligned(v_out, 16)) {
    const int row8 = row / 8;
    const int64_t items = int64_t(batch) * valid * row8;
    ring::gather_vec_kernel<<<ring::grid_for(items), 256, 0, st>>>(
        static_cast<const uint4*>(k_cache), static_cast<const uint4*>(v_cache),
        static_cast<uint4*>(k_out), static_cast<uint4*>(v_out), row8, sink, window, count, valid,
        items);
  } else {
    const int64_t items = int64_t(batch) * valid * row;
    ring::gather_scalar_kernel<<<ring::grid_for(items), 256, 0, st>>>(
        static_cast<const __half*>(k_cache), static_cast<const __half*>(v_cache),
        static_cast<__half*>(k_out), static_cast<__half*>(v_out), row, sink, window, count, valid,
        items);
  }
  return check_launch("ring_gather");
}
