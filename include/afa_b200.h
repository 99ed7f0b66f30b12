/*
 * afa_b200.h -- C ABI of the B200 (sm_100a) Algebraic FlashAttention library
 * (libafa_b200.so).
 *
 * The reference (tasmaikeni13/algebraic-intelligence) is a JAX repository;
 * its hot path is the Python functions below. Each entry point here is what a
 * foreign-function binding of that path (ctypes, or an XLA FFI custom-call
 * handler) calls, with plain pointers and sizes:
 *
 *   afa_fwd               <- pallas_afa_forward  (src/kernels/pallas_afa.py:154-264)
 *                            also the math of tiled_afa_forward (:330-406) and,
 *                            through valid_len, algebraic_flash_attention (:695-739)
 *   afa_fwd_hop           <- one hop of distributed_ring_afa (pallas_afa.py:634-654)
 *   afa_finalize          <- the ring's final divide (pallas_afa.py:661)
 *   afa_ring_export/open/pull/close
 *                         <- the K/V transport of the ring, lax.ppermute
 *                            (pallas_afa.py:651-652)
 *   afa_bwd               <- tiled_afa_backward (pallas_afa.py:409-522), the VJP
 *                            of pallas_afa (:555-615)
 *   afa_ago_table         <- build_cayley_rotary_matrix (src/attention.py:156-207)
 *   afa_ago_rotate        <- apply_ago_rotations (src/attention.py:210-240)
 *   afa_decode            <- no reference counterpart: exact AFA for one query
 *                            token over a KV cache (pallas_afa_forward with Lq=1)
 *   algebraic_softmax_fwd <- algebraic_softmax   (src/attention.py:88-91, :59-67)
 *   algebraic_softmax_bwd <- its custom VJP      (src/attention.py:70-85)
 *   afa_octic(_bwd)       <- octic_kernel and its VJP (src/attention.py:38-50) and
 *                            _vmu_octic_kernel   (pallas_afa.py:32-49)
 *
 * Conventions
 *   - Tensors are contiguous, row-major; attention tensors are (B, H, L, D).
 *   - All buffers are device memory owned by the caller; no entry point
 *     allocates. Launches are ordered on `stream` (a cudaStream_t; NULL = the
 *     legacy default stream) and return as soon as the work is queued.
 *   - dtype codes: AFA_F32, AFA_BF16, AFA_F16, AFA_F64. Accumulators and the
 *     denominator output (d_total) are float32, or float64 for AFA_F64 inputs.
 *   - Every entry point returns AFA_OK or an error code and never aborts; the
 *     message of the last failure on the calling thread is afa_last_error().
 *   - Kernels that wait on on-chip barriers give up after a bounded time and
 *     record a non-zero device status; afa_device_status() reads it.
 */
#ifndef AFA_B200_H_
#define AFA_B200_H_

#include <stddef.h>

#if defined(__GNUC__)
#define AFA_API __attribute__((visibility("default")))
#else
#define AFA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define AFA_F32 0
#define AFA_BF16 1
#define AFA_F16 2
#define AFA_F64 3

#define AFA_OK 0
#define AFA_ERR_INVALID 1     /* bad shape, pointer or hyperparameter (ValueError in Python) */
#define AFA_ERR_DTYPE 2       /* dtype not supported (TypeError in Python) */
#define AFA_ERR_CUDA 3        /* a CUDA runtime call failed */
#define AFA_ERR_DEVICE 4      /* a kernel reported a device-side failure (bounded wait ran out) */

/* Library version string. */
AFA_API const char* afa_version(void);

/* Message of the last error returned on the calling thread ("" if none). */
AFA_API const char* afa_last_error(void);

/*
 * AFA forward, pallas_afa_forward (pallas_afa.py:154-264).
 *   q, k, v     (B, H, L, D) in `dtype` (AFA_F32, AFA_BF16 or AFA_F64).
 *   out         (B, H, L, D) in `dtype`: rho(QK^T/sqrt(D))^8 V / (rowsum + sink).
 *   d_total     (B, H, L) accumulation dtype: rowsum + sink; may be NULL
 *               (return_denominator=False).
 *   causal      key j visible from query i iff j <= i (pallas_afa.py:121-124).
 *   valid_len   keys with index >= valid_len are dropped (pallas_afa.py:116-118);
 *               0 means all L keys. Must be in [0, L].
 * AFA_BF16 with D in {64, 128} runs on the tcgen05 tensor cores; other cases on
 * the CUDA cores. AFA_F16 returns AFA_ERR_DTYPE: the reference casts P to the
 * value dtype (pallas_afa.py:133), and rho^8 exceeds the float16 range for
 * scores above about 2.4.
 */
AFA_API int afa_fwd(const void* q, const void* k, const void* v, void* out, void* d_total, int B, int H, int L, int D,
            int dtype, float sink_omega, int causal, int valid_len, void* stream);

/*
 * One ring hop (distributed_ring_afa body, pallas_afa.py:634-654), or any
 * grouped partial forward over up to 4 problems.
 *   q           (B, H, Lq, D); k, v (B, H, Lk, D).
 *   o_acc       (B, H, Lq, D) accumulation dtype; d_acc (B, H, Lq): the running
 *               unnormalised numerator sum P V and row sum sum P.
 *   out         (B, H, Lq, D) in `dtype`; d_total (B, H, Lq) accumulation dtype
 *               (may be NULL) -- written by the FINALIZE and ONLY modes.
 *   problems    host array of nproblems x 10 ints:
 *                 q_row0, q_len, q_pos0, nk, k0_row0, k0_len, k0_pos0,
 *                 k1_row0, k1_len, k1_pos0
 *               A problem maps query rows [q_row0, q_row0+q_len) (global
 *               positions from q_pos0) onto nk (1 or 2) key segments of K/V.
 *               With causal, key position <= query position decides
 *               visibility (pallas_afa.py:640-646); a segment may be wholly
 *               invisible (no tiles run, the epilogue still does). Query ranges
 *               of different problems must not overlap, except in
 *               AFA_HOP_ACCUMULATE on the tensor cores (bf16, D 64 or 128,
 *               at most 1024 query pairs of 256 rows per (b, h)), where the
 *               partial sums of shared rows add (two ring hops in one launch);
 *               with two key segments and causal, the first must be visible to
 *               every query row.
 *   mode        AFA_HOP_STORE      o_acc = O, d_acc = d          (first hop)
 *               AFA_HOP_ACCUMULATE o_acc += O, d_acc += d        (middle hops)
 *               AFA_HOP_FINALIZE   out = (o_acc + O) / (d_acc + d + sink),
 *                                  d_total = d_acc + d + sink    (last hop,
 *                                  the divide of pallas_afa.py:661 fused in)
 *               AFA_HOP_ONLY       out = O / (d + sink)          (single hop)
 *   Rows outside every problem are not touched.
 */
#define AFA_HOP_STORE 0
#define AFA_HOP_ACCUMULATE 1
#define AFA_HOP_FINALIZE 2
#define AFA_HOP_ONLY 3
AFA_API int afa_fwd_hop(const void* q, const void* k, const void* v, void* o_acc, void* d_acc, void* out,
                        void* d_total, int B, int H, int Lq, int Lk, int D, int dtype, const int* problems,
                        int nproblems, int causal, int mode, float sink_omega, void* stream);

/*
 * Ring epilogue (pallas_afa.py:661): out = o_acc / (d_acc + sink) in `dtype`,
 * d_total = d_acc + sink (may be NULL). rows = B*H*L.
 */
AFA_API int afa_finalize(const void* o_acc, const void* d_acc, void* out, void* d_total, long long rows, int D, int dtype,
                 float sink_omega, void* stream);

/*
 * Ring K/V exchange between the processes of one node (the transport that
 * replaces lax.ppermute in distributed_ring_afa, pallas_afa.py:651-652).
 *
 * Each rank publishes its K/V shard in a device buffer that every other rank
 * maps with CUDA IPC; a hop then pulls the shard it needs straight from the
 * owning rank with the copy engines over NVLink, so the transfer uses no SMs
 * and overlaps the previous hop's kernel. Ordering between ranks (publish
 * before pull, pull before overwrite or free) is the caller's: the Python ring
 * inserts two stream-ordered barriers per call, after publishing and at the
 * end.
 *
 *   afa_ring_export  IPC handle (AFA_RING_HANDLE_BYTES bytes, written to
 *                    handle_out) of the device allocation that holds ptr, and
 *                    ptr's byte offset in it. ptr must come from cudaMalloc (or
 *                    an allocator built on it, like PyTorch's default one).
 *   afa_ring_open    maps a peer's handle into this process on the current
 *                    device; *base_out is the mapping's base (add the offset).
 *   afa_ring_close   unmaps a base returned by afa_ring_open.
 *   afa_ring_pull    stream-ordered copy of `bytes` from src (a peer mapping
 *                    or local memory) to dst on the copy engines.
 *   afa_ring_pull2d  the same for `rows` rows of `row_bytes` bytes, src rows
 *                    `src_pitch` bytes apart and dst rows `dst_pitch` apart:
 *                    a shard pulled into half of every (batch, head) block of
 *                    a receive buffer that holds two hops' shards, so one
 *                    kernel launch computes both hops.
 */
#define AFA_RING_HANDLE_BYTES 64
AFA_API int afa_ring_export(const void* ptr, void* handle_out, unsigned long long* offset_out);
AFA_API int afa_ring_open(const void* handle, void** base_out);
AFA_API int afa_ring_close(void* base);
AFA_API int afa_ring_pull(void* dst, const void* src, size_t bytes, void* stream);
AFA_API int afa_ring_pull2d(void* dst, size_t dst_pitch, const void* src, size_t src_pitch, size_t row_bytes,
                            size_t rows, void* stream);

/*
 * Backward (tiled_afa_backward, pallas_afa.py:409-522; the VJP of pallas_afa,
 * :555-575): dq, dk, dv of sum(out * g_out) for out = afa_fwd(q, k, v).
 *   q, k, v, out, g_out, dq, dk, dv  (B, H, L, D) in `dtype` (bf16, f32, f64)
 *   d_total   (B, H, L) from afa_fwd: row sum + sink, float32 (float64 for f64)
 *   sink_omega the forward's sink (tiled_afa_backward's sink_omega argument).
 *             The gradient math uses the sink only through d_total, as in the
 *             reference (:429); d_total - sink_omega, a row's weight sum, tells
 *             the bf16 tensor-core kernels which rows lie wholly in the
 *             negative tail of rho^8 and need its cancellation-free branch.
 *   causal, valid_len as afa_fwd (valid_len 0 = L)
 *   workspace afa_bwd_workspace_bytes(B, H, L, D, dtype) bytes of device
 *             scratch (the per-row E = sum(g_out * out)), caller-owned.
 */
AFA_API int afa_bwd(const void* q, const void* k, const void* v, const void* out, const void* d_total,
                    const void* g_out, void* dq, void* dk, void* dv, int B, int H, int L, int D, int dtype,
                    float sink_omega, int causal, int valid_len, void* workspace, size_t workspace_bytes,
                    void* stream);
AFA_API size_t afa_bwd_workspace_bytes(int B, int H, int L, int D, int dtype);

/*
 * AGO rotary position rotations, the Q/K prologue of the attention layer
 * (src/model.py:262-264).
 *   afa_ago_table   build_cayley_rotary_matrix (src/attention.py:156-207):
 *                   c, s = (max_seq_len, dim/2) tables in `dtype`, computed in
 *                   float32 (float64 for AFA_F64). freqs: optional HOST array of
 *                   dim/2 doubles (the explicit rational frequencies); NULL uses
 *                   the default ladder from `base`. dim even, at most 512.
 *   afa_ago_rotate  apply_ago_rotations (src/attention.py:210-240): rotates q and
 *                   k (contiguous, same shape, last axis = dim) into q_out and k_out
 *                   (which may alias them). Row r (of rows = elements / dim) sits
 *                   at sequence position (r / inner) % seq_len; inner is the
 *                   product of the axes between the sequence axis and the last.
 *                   c, s: (>= seq_len, dim/2) tables in table_dtype, cast to
 *                   `dtype` before use as in the reference.
 */
AFA_API int afa_ago_table(void* c, void* s, int dim, int max_seq_len, const double* freqs, double base, int dtype,
                          void* stream);
AFA_API int afa_ago_rotate(const void* q, const void* k, void* q_out, void* k_out, const void* c, const void* s,
                           int table_dtype, long long rows, int dim, int seq_len, long long inner, int dtype,
                           void* stream);

/*
 * Decode step (no reference counterpart; the math of pallas_afa_forward with a
 * single query row, non-causal).
 *   q           (B, H, D) -- one token per (batch, head)
 *   k_cache, v_cache  (B, H, Lkv, D)
 *   out         (B, H, D); d_total (B, H) float32, may be NULL.
 *   kv_lens     optional device int32[B]: visible cache length per batch row,
 *               clamped to [0, Lkv]; a row of length 0 gives output 0 and
 *               d_total = sink_omega. NULL uses kv_len for all rows (0 = Lkv).
 *   workspace   device scratch of afa_decode_workspace_bytes(B, H, Lkv, D)
 *               bytes (may be NULL when that size is 0).
 * AFA_BF16 (D in 64/128/256) and AFA_F32 (D in 64/128) use the split-KV
 * streaming kernel; other supported shapes fall back to the CUDA-core
 * forward kernel.
 */
AFA_API int afa_decode(const void* q, const void* k_cache, const void* v_cache, void* out, void* d_total, int B, int H,
               int Lkv, int D, int dtype, float sink_omega, const int* kv_lens, int kv_len, void* workspace,
               size_t workspace_bytes, void* stream);
AFA_API size_t afa_decode_workspace_bytes(int B, int H, int Lkv, int D);

/*
 * Allocation-free decode step. No counterpart in the reference: it is
 * afa_decode for callers that cannot hand over device scratch memory --
 * plugin hosts whose allocator belongs to another runtime, serving loops that
 * forbid allocation per token. Same arguments and results as afa_decode minus
 * the workspace. The split-KV scratch instead lives in a fixed 1 MiB array
 * that every GPU loading the library keeps until exit. Shapes whose split-KV
 * scratch exceeds that (afa_decode_workspace_bytes > 1 MiB for a dtype and
 * head dim afa_decode streams with split-KV) return AFA_ERR_INVALID. All calls
 * share the array, so calls that overlap on the GPU race; serialise them on
 * one stream. The first call on a device resolves the array's device address
 * (cudaGetSymbolAddress); make it before any stream capture. That address is
 * cached for the process: do not use the library across cudaDeviceReset.
 */
AFA_API int afa_decode_noalloc(const void* q, const void* k_cache, const void* v_cache, void* out, void* d_total,
                               int B, int H, int Lkv, int D, int dtype, float sink_omega, const int* kv_lens,
                               int kv_len, void* stream);

/*
 * algebraic_softmax (src/attention.py:88-91): rows x cols, last axis
 * normalised. dtype AFA_F32, AFA_BF16, AFA_F16 (fp32 accumulation) or AFA_F64.
 * Errors mirror the reference: sink_omega must be finite and >= 0, eps finite
 * and > 0 (attention.py:60-63), cols > 0 (primitives.py:58-59).
 */
AFA_API int algebraic_softmax_fwd(const void* x, void* y, long long rows, int cols, int dtype, double sink_omega,
                          double eps, void* stream);

/* octic_kernel (src/attention.py:47-50): y = rho(x)^8 elementwise, n elements. */
AFA_API int afa_octic(const void* x, void* y, long long n, int dtype, void* stream);
/* The VJP of octic_kernel (src/attention.py:38-44): dx = 8 r rho(x)^8 g, r = rsqrt(1 + x^2). */
AFA_API int afa_octic_bwd(const void* x, const void* g, void* dx, long long n, int dtype, void* stream);

/*
 * algebraic_softmax backward: the custom VJP of algebraic_softmax
 * (src/attention.py:70-85 with the AVN VJP, src/primitives.py:73-79). x: the
 * forward's input scores, g: the upstream gradient, dx: the input gradient,
 * all (rows, cols) in `dtype`; the same sink_omega / eps as the forward. The
 * forward quantities are recomputed from x.
 */
AFA_API int algebraic_softmax_bwd(const void* x, const void* g, void* dx, long long rows, int cols, int dtype,
                                  double sink_omega, double eps, void* stream);

/*
 * Synchronises `stream`, then reads the calling device's status word (0 = no
 * kernel reported a failure) into *status; clears it when `clear` is non-zero.
 */
AFA_API int afa_device_status(void* stream, int* status, int clear);

/*
 * Failure-detection self-test (no reference counterpart): launches one thread
 * that waits on an on-chip barrier nothing ever releases, with a wait budget of
 * budget_ns (at most 2 s). The wait gives up, records status 0x1ff and the
 * kernel returns; afa_device_status() then reports 0x1ff. Exercises the same
 * bounded wait every pipelined kernel uses, without faulting or hanging a GPU.
 */
AFA_API int afa_selftest_bounded_wait(long long budget_ns, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* AFA_B200_H_ */
