/*
 * qx_b200.h -- C ABI of libqx_b200.so, the sm_100a (B200) kernels behind the
 * QExtract-Infer operator API.
 *
 * Conventions
 *   - All pointers are device pointers unless stated otherwise; fp16 data is
 *     passed as `const void*` / `void*` holding IEEE binary16 values.
 *   - Every tensor is dense row-major (C-contiguous).
 *   - `stream` is a cudaStream_t (NULL = legacy default stream).  All work is
 *     enqueued on it; nothing synchronises the host.
 *   - Nothing here allocates device memory.  Ops that need scratch take a
 *     caller-owned `workspace`; its required size comes from the matching
 *     `*_workspace_size` function.
 *   - Return value: 0 on success, negative on error (QX_ERR_*); the message
 *     of the last error on the calling thread is returned by qx_last_error().
 *
 * The reference interface each entry point replaces is cited as
 * path:line within the QExtract-Infer project.
 */
#ifndef QX_B200_H_
#define QX_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* qx_stream_t; /* == cudaStream_t */

#define QX_OK 0
#define QX_ERR_INVALID (-1)
#define QX_ERR_CUDA (-2)
#define QX_ERR_WORKSPACE (-3)
#define QX_ERR_UNSUPPORTED (-4)

/* Message of the last failed call on this thread ("" if none). */
const char* qx_last_error(void);

/* Device-side failures that a kernel cannot return as a status: a bounded
 * wait inside a kernel that timed out sets a bit here instead of hanging the
 * GPU (the kernel then finishes with undefined output).  New component: the
 * reference has no device-side error reporting. */
#define QX_DEVERR_MBAR_TIMEOUT 1u
/* a peer rank's row did not arrive within the wait limit (qx_nvlink_ar_add_rmsnorm) */
#define QX_DEVERR_PEER_TIMEOUT 2u
/* Reads (and with reset != 0 clears) the sticky error bits of the current
 * device; synchronises with the device. */
int qx_get_device_error(unsigned* code, int reset);
/* Library version string. */
const char* qx_version(void);
/* Profiling: per-CTA phase timestamps (%globaltimer, ns) of the next
 * `launches` launches of one kernel family into `buf` (device memory,
 * launches x grid x 16 uint64; launch i, CTA c at (i * grid + c) * 16; slot 15
 * holds the SM id; which slot is which phase is listed beside each kernel's
 * trace points).  Only the profiling build of the library
 * (libqx_b200_trace.so, compiled with -DQX_TRACE) records; the product library
 * returns QX_ERR_UNSUPPORTED and carries no trace code in its kernels.
 * buf = NULL stops tracing.  No counterpart in the reference. */
#define QX_TRACE_GEMV 0
#define QX_TRACE_DECODE_ATTENTION 1
#define QX_TRACE_SLOTS 16
int qx_trace_launches(int kernel, void* buf, int launches);
/* Host plumbing for callers without their own CUDA runtime binding (ctypes,
 * cgo, JNI): one cudaMemcpyAsync of `bytes` from src to dst on `stream`, the
 * direction taken from the pointers (pinned host or device).  No counterpart
 * in the reference (its pybind layer moves data with torch). */
int qx_copy_async(void* dst, const void* src, size_t bytes, qx_stream_t stream);

/* ------------------------------------------------------------------------
 * W4A16(-LoRA) GEMV.
 * Replaces w4a16_lora_gemv() (csrc/kernels/w4a16_lora_gemv.cu:268-323) and
 * w4a16_gemv() (:233-265), bound at csrc/binding.cpp:44-56.
 *
 *   y[M, N] = fp16( x[M, K] . dequant(qweight) + lora_scale * (x . A) . B )
 *
 *   x        fp16  [M, K]           (M = product of the leading dims)
 *   qweight  int32 [K/8, N]         nibble i of qweight[p, n] = W_q[8p+i, n]
 *   scales   fp16  [K/group, N]
 *   zeros    zeros_packed == 0: fp16 [K/group, N]  (reference kernel format)
 *            zeros_packed == 1: int32 [K/group, N/8] GPTQ qzeros, z = nibble + zero_offset
 *   lora_A   fp16  [K, rank]   lora_B fp16 [rank, N]   (rank == 0: no LoRA; A, B may be NULL)
 *   lora_scale  = lora_alpha / rank   (the reference computes it at w4a16_lora_gemv.cu:221)
 *   y        fp16  [M, N]
 * Constraints: K % 32 == 0, group_size % 32 == 0, K % group_size == 0,
 * N % 8 == 0, rank in {0, 8, 16, 32, 48, 64, 128}; x, qweight, scales, lora_A,
 * lora_B (and fp16 zeros) 16-byte aligned.
 * Any M >= 1 (rows are processed 32 at a time).
 * No workspace: each group of CTAs that splits K forms a thread-block cluster
 * and reduces through distributed shared memory (st.async into the CTA that
 * owns the columns).
 * ---------------------------------------------------------------------- */
int qx_w4a16_lora_gemv(const void* x, const int32_t* qweight, const void* scales,
                       const void* zeros, int zeros_packed, int zero_offset,
                       const void* lora_A, const void* lora_B, void* y,
                       int M, int K, int N, int rank, int group_size, float lora_scale,
                       qx_stream_t stream);

/* The gate|up projection of an MLP followed by SwiGLU, in one launch: the
 * GEMV above over N = 2I columns laid out in blocks of 16 (8 gate columns,
 * then the 8 up columns of the same outputs), each owner CTA rounding its
 * gate and up sums to fp16 and writing y[m][i] = fp16(silu(g) u) ([M, I]) with
 * the formula of qx_fused_swiglu.  Bit-identical to qx_w4a16_lora_gemv on the
 * interleaved weights followed by SwiGLU on the matching columns.  N % 16 == 0.
 * Replaces the reference's gate/up projections and fused_swiglu call
 * (qextract/patch.py:94-113) with one kernel: the [M, 2I] intermediate never
 * reaches memory. */
int qx_w4a16_lora_gemv_swiglu(const void* x, const int32_t* qweight, const void* scales,
                              const void* zeros, int zeros_packed, int zero_offset,
                              const void* lora_A, const void* lora_B, void* y,
                              int M, int K, int N, int rank, int group_size, float lora_scale,
                              qx_stream_t stream);

/* The decode step's residual add + RMSNorm as the GEMV's prologue (one launch
 * instead of qx_add_rmsnorm + the GEMV): every CTA forms r = fp16(residual +
 * delta) over whole rows, x = fp16((r * rsqrt(mean(r^2) + eps)) * norm_weight)
 * with the rounding of qx_add_rmsnorm, and runs the GEMV (swiglu = 1: the
 * SwiGLU form of qx_w4a16_lora_gemv_swiglu) on x; r is written to
 * residual_out (the new residual stream).  residual / delta / residual_out fp16
 * [M, K], norm_weight fp16 [K]; M <= 8 rows (each CTA reads the whole rows);
 * residual_out must not overlap residual or delta (callers alternate two
 * residual buffers).  Matches qx_add_rmsnorm followed by the GEMV up to the
 * order of the sum of squares.  Replaces the patched layer's RMSNorm
 * (qextract/patch.py:73-87) together with the residual add that the HF decoder
 * layer runs before it, ahead of the MLP / attention projections. */
int qx_w4a16_lora_gemv_addnorm(const void* residual, const void* delta, const void* norm_weight,
                               float eps, void* residual_out, const int32_t* qweight,
                               const void* scales, const void* zeros, int zeros_packed,
                               int zero_offset, const void* lora_A, const void* lora_B, void* y,
                               int M, int K, int N, int rank, int group_size, float lora_scale,
                               int swiglu, qx_stream_t stream);

/* Programmatic dependent launch for the GEMV (on by default; 0 turns it
 * off).  When on, a GEMV launches as soon as every CTA of the GEMV before it
 * in the stream is running: it streams its weights and stages scales /
 * zeros / LoRA factors while that kernel finishes, and waits for it only
 * before reading x (and so before writing y).  The library's RMSNorm, SwiGLU,
 * decode-step and decode-attention kernels trigger at their start too, so a
 * GEMV after them streams its weights while they run; kernels that do not
 * trigger early (every kernel outside this library) still complete first.  The
 * weight operands must therefore not be written by a GEMV issued just
 * before on the same stream (true for model weights).  Returns 0. */
int qx_set_pdl(int enable);

/* qx_w4a16_lora_gemv for callers whose activations and outputs live in host
 * memory (a cgo / JNI / ctypes plugin): moves x_host [M, K] into x_dev, runs
 * the GEMV, and delivers y [M, N] into y_host, all enqueued on `stream` in one
 * call; the caller synchronises before reading y_host.  Pinned (device-mapped)
 * host buffers take the fast form: the GEMV reads x_host over the bus itself,
 * as soon as it launches (while the previous kernel on the stream still runs:
 * x_host must hold this call's rows when the call is made, and must not be
 * written by kernels still pending on the stream, except the previous call of
 * this function, whose y_host is detected), and writes y straight into y_host
 * (x_dev and y_dev unused).  Pageable buffers go through cudaMemcpyAsync into
 * x_dev and out of y_dev.  New entry point: the reference's op takes device
 * tensors only. */
int qx_w4a16_lora_gemv_host(const void* x_host, void* y_host, void* x_dev, void* y_dev,
                            const int32_t* qweight, const void* scales, const void* zeros,
                            int zeros_packed, int zero_offset, const void* lora_A, const void* lora_B,
                            int M, int K, int N, int rank, int group_size, float lora_scale,
                            qx_stream_t stream);

/* The split-K plan qx_w4a16_lora_gemv uses for a shape (at most 32 rows of M
 * per launch): out[0] = 256-column tiles, out[1] = CTAs splitting K per tile
 * (the cluster size S), out[2] = weight stages in flight per CTA, out[3] =
 * quantisation groups of the longest CTA, out[4] = shared memory per CTA in
 * bytes.  Plans are chosen on the current device.  New component (the
 * reference has one launch shape).  Returns 0 or an error status. */
int qx_w4a16_gemv_plan(int M, int K, int N, int rank, int group_size, int zeros_packed, int* out);
/* Pins the split-K plan of every later qx_w4a16_lora_gemv call whose shape
 * admits it: S CTAs per tile and nst weight stages (0 = chosen per shape);
 * shapes the pinned plan does not fit fail with QX_ERR_UNSUPPORTED.  For
 * tuning; process-wide.  Returns 0 or QX_ERR_INVALID. */
int qx_w4a16_gemv_pin_plan(int S, int nst);


/* ------------------------------------------------------------------------
 * W4A16-LoRA GEMM on the tcgen05 tensor cores (prefill, large M).
 * Same math and operand formats as qx_w4a16_lora_gemv (the reference runs
 * every M through w4a16_lora_gemv(), csrc/kernels/w4a16_lora_gemv.cu:268-323);
 * new component: the reference has no tensor-core path.  Launches the LoRA
 * down-projection (h = x . A, fp32, into the workspace) and the GEMM
 * (128 x 256 output tiles, TMA-fed, int4 dequantised in shared memory,
 * accumulator in TMEM, LoRA term added on the tensor cores).
 * Constraints: N % 256 == 0, K % 64 == 0, group_size in {32, 64, 128, 256},
 * rank in {0, 8, 16, 32, 48, 64}; every tensor and the workspace 16-byte aligned.
 * workspace: qx_w4a16_lora_gemm_sm100_workspace_size(M, rank) bytes (the scaled
 * LoRA down-projection as fp16 high and low parts);
 * its contents need no initialisation.
 * ---------------------------------------------------------------------- */
size_t qx_w4a16_lora_gemm_sm100_workspace_size(int M, int rank);
int qx_w4a16_lora_gemm_sm100(const void* x, const int32_t* qweight, const void* scales,
                             const void* zeros, int zeros_packed, int zero_offset,
                             const void* lora_A, const void* lora_B, void* y, int M, int K, int N,
                             int rank, int group_size, float lora_scale, void* workspace,
                             size_t workspace_bytes, qx_stream_t stream);

/* ------------------------------------------------------------------------
 * Fused kernels of the tensor-parallel decode step (new components; the
 * reference's patched Qwen3 layer, qextract/patch.py, runs each as
 * separate torch ops).  Rounding points equal the unfused sequence.
 *
 * qx_add_rmsnorm: x <- fp16(x + delta) in place (the residual add), then
 *   y = fp16((x * rsqrt(mean(x^2) + eps)) * w) as qx_fused_rmsnorm.
 *   x, delta, y fp16 [rows, hidden]; w fp16 [hidden]; hidden % 8 == 0,
 *   hidden <= 8192; 16-byte aligned.
 * qx_qk_norm_rope_append: qkv fp16 [batch, q_heads + 2 kv_heads, head_dim]
 *   (the fused q|k|v projection of one decode position); q and k heads are
 *   RMSNorm'd over head_dim with q_norm_w / k_norm_w (fp16 result) and
 *   rotated (rotate-half RoPE; cos_row / sin_row fp32 [head_dim] of the
 *   position); q heads go to q_out fp16 [batch, q_heads, head_dim], k and v
 *   heads to slot (pos < sink ? pos : sink + (pos - sink) % window) of the
 *   ring caches k_cache / v_cache fp16 [batch, sink + window, kv_heads,
 *   head_dim].  head_dim in {64, 128, 256}.
 * qx_swiglu_packed: gate_up fp16 [rows, 2 inter] (gate columns, then up);
 *   y fp16 [rows, inter] = fp16(silu(gate) * up) as qx_fused_swiglu;
 *   inter % 8 == 0, 16-byte aligned.
 * ---------------------------------------------------------------------- */
int qx_add_rmsnorm(void* x, const void* delta, const void* weight, void* y, int64_t rows, int hidden,
                   float eps, qx_stream_t stream);
int qx_qk_norm_rope_append(const void* qkv, int batch, int q_heads, int kv_heads, int head_dim,
                           const void* q_norm_w, const void* k_norm_w, float eps,
                           const float* cos_row, const float* sin_row, void* q_out, void* k_cache,
                           void* v_cache, int sink, int window, int64_t pos, qx_stream_t stream);
int qx_swiglu_packed(const void* gate_up, void* y, int64_t rows, int inter, qx_stream_t stream);

/* ------------------------------------------------------------------------
 * One-shot all-reduce over NVLink peer memory fused with the residual add and
 * RMSNorm after the row-parallel projections of the tensor-parallel decode
 * step (new component; NCCL's all-reduce is the baseline it replaces):
 *   x[r] <- fp16(x[r] + fp16(sum over ranks of partial[r]))  (in place)
 *   y[r]  = fp16((x[r] * rsqrt(mean(x[r]^2) + eps)) * w)
 * Every rank computes identical bits (rank-ordered fp32 sum).
 * Setup, on every rank of one node (one GPU per rank): qx_nvlink_ar_create
 * allocates this rank's inbox (2 x world x max_rows x hidden x 4 bytes: every
 * peer's rows pushed in with their epoch; the only allocation in the library) and writes its IPC handle
 * (qx_nvlink_ar_handle_bytes() bytes) to handle_out; exchange the handles
 * (all-gather, rank order) and call qx_nvlink_ar_open with all of them; then
 * a barrier before the first call.  Calls: every rank makes the same sequence
 * of calls; calls on one rank must not overlap (stream order).  A peer that
 * does not arrive within the wait limit (2 s unless qx_nvlink_ar_set_timeout
 * sets another) sets QX_DEVERR_PEER_TIMEOUT and that call's output is
 * undefined; the rank that timed out is then one epoch ahead, so its later
 * calls time out too until the communicator is rebuilt.
 * ---------------------------------------------------------------------- */
size_t qx_nvlink_ar_handle_bytes(void);
int qx_nvlink_ar_create(int world, int rank, int max_rows, int hidden, void** ctx, void* handle_out);
int qx_nvlink_ar_open(void* ctx, const void* handles);
/* Alternative to qx_nvlink_ar_open when every rank's context lives in this
 * process (one process driving several GPUs, or several ranks on one GPU):
 * ctxs[r] is rank r's context; peer access is enabled between distinct
 * devices. */
int qx_nvlink_ar_open_local(void* ctx, void* const* ctxs);
/* Limit of each wait for a peer's row, in nanoseconds (default 2e9). */
int qx_nvlink_ar_set_timeout(void* ctx, int64_t timeout_ns);
int qx_nvlink_ar_add_rmsnorm(void* ctx, const void* partial, void* x, const void* weight, void* y,
                             int rows, float eps, qx_stream_t stream);
int qx_nvlink_ar_destroy(void* ctx);

/* ------------------------------------------------------------------------
 * Fused RMSNorm.  Replaces fused_rmsnorm() (csrc/kernels/rmsnorm.cu:162-210,
 * bound at csrc/binding.cpp:36-38).
 *   y[r, :] = fp16( (x[r, :] * rsqrt(mean(x[r, :]^2) + eps)) * w )
 * x, y fp16 [rows, H]; w fp16 [H].  Any H >= 1; H % 8 == 0 and 16-byte
 * aligned rows take the vector path.
 * ---------------------------------------------------------------------- */
int qx_fused_rmsnorm(const void* x, const void* weight, void* y, int64_t rows, int hidden,
                     float eps, qx_stream_t stream);

/* ------------------------------------------------------------------------
 * Fused SwiGLU.  Replaces fused_swiglu() (csrc/kernels/swiglu.cu:94-135,
 * bound at csrc/binding.cpp:40-42).
 *   y[i] = fp16( g[i] * sigmoid(g[i]) * u[i] ),  i < n
 * ---------------------------------------------------------------------- */
int qx_fused_swiglu(const void* gate, const void* up, void* y, int64_t n, qx_stream_t stream);

/* ------------------------------------------------------------------------
 * StreamingLLM ring KV cache (sink + circular window).
 * Replaces RingBufferKVCache::append / get_kv / get_valid_length
 * (csrc/kv_cache/ring_buffer.cu:109-209, bound at csrc/binding.cpp:59-74)
 * and the Python twins in qextract/kv_cache.py:75-152.
 *
 * Layer storage: k_cache, v_cache fp16 [batch, sink + window, kv_heads, head_dim].
 * `count` is the number of tokens written before this call (write_count in
 * the reference).  Token j of the chunk goes to slot write_pos(count + j):
 *   write_pos(c) = c < sink ? c : sink + (c - sink) % window.
 * Appending T tokens at once leaves the cache exactly as T single-token
 * appends would (later tokens win a slot).  Advancing `count` (after the
 * last layer) is the caller's job, as in the reference.
 * ---------------------------------------------------------------------- */
int qx_ring_append(void* k_cache, void* v_cache, const void* new_k, const void* new_v,
                   int batch, int tokens, int kv_heads, int head_dim, int sink, int window,
                   int64_t count, qx_stream_t stream);

/* Logical-order slot list (sinks, then the ring from its oldest token) for
 * `count` written tokens; writes valid_length(count) int32 indices to
 * `slots` (device) and returns that length (>= 0) or a negative status. */
int64_t qx_ring_slot_indices(int32_t* slots, int sink, int window, int64_t count,
                             qx_stream_t stream);

/* Materialise K and V in logical order, the reference get_kv():
 * out fp16 [batch, valid_length(count), kv_heads, head_dim]. */
int qx_ring_gather(const void* k_cache, const void* v_cache, void* k_out, void* v_out,
                   int batch, int kv_heads, int head_dim, int sink, int window, int64_t count,
                   qx_stream_t stream);

/* ------------------------------------------------------------------------
 * GQA decode attention read in place from the ring (no gather).  New
 * component (the reference has no attention kernel); semantics: HF Qwen3
 * eager attention over the cache's valid slots (qextract/kv_cache.py:121-142
 * order is irrelevant to the result).
 *   q fp16 [batch, q_heads, head_dim] (post-RoPE), caches as above,
 *   out fp16 [batch, q_heads, head_dim];  q_heads % kv_heads == 0,
 *   head_dim == 128, q_heads / kv_heads <= 16.
 * softmax_scale <= 0 selects 1/sqrt(head_dim).
 * workspace: >= qx_decode_attention_workspace_size(...) bytes, 256-byte
 * aligned, zero-filled before first use, left zero-filled by every call.
 * ---------------------------------------------------------------------- */
size_t qx_decode_attention_workspace_size(int batch, int q_heads, int kv_heads, int head_dim,
                                          int sink, int window);

int qx_decode_attention(const void* q, const void* k_cache, const void* v_cache, void* out,
                        int batch, int q_heads, int kv_heads, int head_dim, int sink,
                        int window, int64_t count, float softmax_scale, void* workspace,
                        size_t workspace_bytes, qx_stream_t stream);

/* Prefill attention of one prompt chunk over the StreamingLLM ring, before the
 * chunk is appended: q [batch, n, q_heads, 128] (the chunk's queries, at
 * positions count .. count + n - 1), k_new / v_new [batch, n, kv_heads, 128]
 * (the chunk's keys and values), k_cache / v_cache [batch, sink + window,
 * kv_heads, 128] (the ring after `count` tokens: its valid slots are read in
 * place, each at the position the ring's write rule gives it).  Key kp is
 * visible to query p iff kp <= p and (kp < sink or kp > p - window).  out
 * [batch, n, q_heads, 128] fp16; softmax_scale <= 0 means 1/sqrt(128).  Replaces
 * the reference's gather (QExtractKVCache.get_kv, qextract/kv_cache.py:96-112)
 * followed by an attention over the gathered copy. */
int qx_prefill_attention(const void* q, const void* k_new, const void* v_new, const void* k_cache,
                         const void* v_cache, void* out, int batch, int n, int q_heads,
                         int kv_heads, int head_dim, int sink, int window, int64_t count,
                         float softmax_scale, qx_stream_t stream);

/* qx_decode_attention with flags.  QX_ATTN_AFTER_APPEND: the kernel just
 * before this call on `stream` wrote q and position count - 1 of every
 * sequence into the cache (a decode step's append) and nothing else this call
 * reads; when its grid is small (at most two CTAs per SM: one or a few
 * sequences) the attention is then launched early (programmatic dependent
 * launch) and loads its first K/V tiles while that kernel finishes, reloading
 * the appended slot once it has.  Without flags it equals qx_decode_attention.
 * New component (no counterpart in the reference). */
#define QX_ATTN_AFTER_APPEND 1
int qx_decode_attention_ex(const void* q, const void* k_cache, const void* v_cache, void* out,
                           int batch, int q_heads, int kv_heads, int head_dim, int sink,
                           int window, int64_t count, float softmax_scale, void* workspace,
                           size_t workspace_bytes, int flags, qx_stream_t stream);

/* One decode position in one kernel: the q/k head RMSNorm, RoPE and ring
 * append of qx_qk_norm_rope_append followed by qx_decode_attention over the
 * ring including the new token, bit-identical to that pair.  qkv: the fused
 * projection output [batch, (q_heads + 2 kv_heads) * 128] fp16 (16-byte
 * aligned); the new token's k and v go to the ring slot of position `pos`; out
 * [batch, q_heads, 128].  Every CTA rotates the query heads of its KV head
 * itself; the one whose slot chunk holds the new slot appends k and v.  When
 * the grid is small it is launched early and loads its K/V tiles while the
 * projection finishes.  Workspace as qx_decode_attention.  New component
 * (the reference runs these as separate torch ops). */
int qx_decode_attention_qkv(const void* qkv, const void* q_norm_w, const void* k_norm_w, float eps,
                            const float* cos_row, const float* sin_row, void* k_cache, void* v_cache,
                            void* out, int batch, int q_heads, int kv_heads, int head_dim, int sink,
                            int window, int64_t pos, float softmax_scale, void* workspace,
                            size_t workspace_bytes, qx_stream_t stream);

/* Greedy head: logits = h W for h [batch, hidden] fp16 and W [hidden, vocab]
 * fp16 (a rank's vocabulary slice, vocab contiguous), rounded to fp16, and per
 * row the largest logit (as fp32) and its index + vocab_offset (the smallest
 * index among equal maxima).  batch <= 32, hidden % 64 == 0, vocab % 8 == 0.
 * Workspace: qx_lm_head_argmax_workspace_size(vocab) bytes, no
 * initialisation.  New component (the reference leaves the lm_head to HF). */
size_t qx_lm_head_argmax_workspace_size(int vocab);
int qx_lm_head_argmax(const void* h, const void* weight, int batch, int hidden, int vocab,
                      int64_t vocab_offset, float* out_val, int64_t* out_idx, void* workspace,
                      size_t workspace_bytes, qx_stream_t stream);

/* How both decode-attention entry points merge the slot chunks of one
 * sequence and KV head (process-wide; results agree within fp32 rounding):
 * 0 (default) through distributed shared memory, the chunk CTAs forming one
 * thread-block cluster (up to 16 chunks; longer chunks when needed),
 * 1 through the workspace (partials written, the last CTA merges them). */
int qx_decode_attention_pin_merge(int mode);

/* ------------------------------------------------------------------------
 * Allocation-free decode attention.  No counterpart in the reference.
 * For callers that cannot allocate device memory when attention runs (a host
 * framework that owns the device heap, a server plugin handed only its
 * input/output buffers, or a path where cudaMalloc would synchronise the
 * device): same arguments and results as qx_decode_attention, but the
 * scratch is one array of QX_DECODE_ATTN_NOALLOC_SCRATCH_BYTES built into the
 * library (held by every GPU that loads it until the process exits) instead
 * of a caller workspace.  Shapes whose scratch exceeds that size are rejected
 * with QX_ERR_UNSUPPORTED and a message (Qwen3-8B geometry, 32 query / 8 KV
 * heads, 4 + 4092 slots, fits every batch up to 247 on a 148-SM B200; the
 * need is qx_decode_attention_workspace_size for the same shape).
 * The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress) for that device; make that first call before any
 * stream capture.  Each call clears the counters it needs with
 * cudaMemsetAsync on `stream` and allocates nothing.  All calls share the
 * one array: calls that overlap on the GPU (different streams, or different
 * host threads) race on it and must be serialised by the caller.
 * ---------------------------------------------------------------------- */
#define QX_DECODE_ATTN_NOALLOC_SCRATCH_BYTES (4 << 20)

int qx_decode_attention_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                void* out, int batch, int q_heads, int kv_heads, int head_dim,
                                int sink, int window, int64_t count, float softmax_scale,
                                qx_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* QX_B200_H_ */
