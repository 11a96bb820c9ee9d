/*
 * fp8attn -- B200 (sm_100a) FP8 PagedAttention hot path behind a plain C ABI.
 *
 * Three entry points replace the three GPU kernels of nano-vLLM's FP8 KV-cache attention path
 * (Lin-so/my-nano-vllm); the Python signatures they sit behind are kept verbatim by the
 * `nanovllm_b200` package:
 *
 *   fp8attn_store_kvcache  <- store_kvcache          nanovllm/layers/attention.py:33-40
 *                             (kernel store_kvcache_kernel, :11-31)
 *   fp8attn_decode         <- fp8_decode_attention   nanovllm/kernels/fp8_attention.py:173-207
 *                             (kernel fp8_paged_attention_decode_kernel, :88-171)
 *   fp8attn_prefill        <- fp8_prefill_attention  nanovllm/kernels/fp8_attention.py:314-353
 *                             (kernel fp8_paged_attention_prefill_kernel, :209-312)
 *
 * Conventions
 *   - All pointers are device pointers; `stream` is a cudaStream_t (NULL = legacy stream).
 *     Nothing synchronises the stream or reads device memory on the host, so every call can be
 *     captured into a CUDA graph.
 *   - bf16 tensors are passed as raw 16-bit patterns, e4m3 caches as bytes.  head_dim must be 128.
 *   - Paged caches are [num_blocks, block_size, num_kv_heads, 128] e4m3, contiguous; block_size is
 *     a multiple of 16.  Optional scales are fp32 [num_blocks * block_size, num_kv_heads]; NULL
 *     means unit scale, which is the reference's behaviour (its cache has no scales).
 *   - Return value: 0 on success, otherwise an FP8ATTN_E* code; fp8attn_last_error() gives a
 *     message (thread-local).  Launch errors are reported, device-side problems (a bounded wait
 *     that timed out, a workspace overflow) are recorded in the workspace's error word
 *     (int32 at byte offset FP8ATTN_WS_ERROR_OFFSET) and never trap.
 */
#ifndef FP8ATTN_H_
#define FP8ATTN_H_

#include <stdint.h>

#if defined(__GNUC__)
#define FP8ATTN_API __attribute__((visibility("default")))
#else
#define FP8ATTN_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define FP8ATTN_OK 0
#define FP8ATTN_EINVAL 1     /* invalid argument (null pointer, shape, stride, alignment) */
#define FP8ATTN_EWORKSPACE 2 /* workspace missing or smaller than fp8attn_workspace_bytes() */
#define FP8ATTN_ECUDA 3      /* CUDA error while preparing or launching */

#define FP8ATTN_WS_ERROR_OFFSET 0

/* Library version (major * 10000 + minor * 100 + patch). */
FP8ATTN_API int fp8attn_version(void);

/* Message for the last non-zero status returned on this thread. */
FP8ATTN_API const char* fp8attn_last_error(void);

/*
 * KV store / quantise.  Replaces store_kvcache (nanovllm/layers/attention.py:33-40).
 * For every token i < num_tokens with slot = slot_mapping[i] != -1:
 *   k_cache[slot] = e4m3(key[i]),  v_cache[slot] = e4m3(value[i])      (cache rows of KVH*128)
 * key/value rows are KVH*128 bf16 values, row i at key + i*key_row_stride (elements).
 * scaled == 0: round-to-nearest-even cast with finite overflow saturating to +-448; scale arrays
 *              (if given) receive 1.0.
 * scaled == 1: per (token, kv head) scale = amax/448 (0 -> 1); bytes = e4m3(clamp(x/scale)).
 * Slots outside [0, num_slots) are skipped like -1.
 */
FP8ATTN_API int fp8attn_store_kvcache(const void* key, int64_t key_row_stride, const void* value,
                          int64_t value_row_stride, void* k_cache, void* v_cache, float* k_scale,
                          float* v_scale, const int32_t* slot_mapping, int64_t num_tokens,
                          int num_kv_heads, int head_dim, int64_t num_slots, int scaled,
                          void* stream);

/*
 * Fused attention-input epilogue: q_norm / k_norm (RMSNorm over each head's 128 values), rotary
 * embedding of q and k, and the K/V store of fp8attn_store_kvcache, in one kernel.  Replaces, for
 * the q, k, v split of the QKV projection's output, the chain RMSNorm.rms_forward
 * (nanovllm/layers/layernorm.py:16-26) -> RotaryEmbedding.forward
 * (nanovllm/layers/rotary_embedding.py:37-47) -> store_kvcache (nanovllm/layers/attention.py:33-40)
 * that Qwen3Attention.forward runs (nanovllm/models/qwen3.py:102-111).
 * qkv: bf16 [num_tokens, row] (row = qkv_row_stride elements): num_heads q heads, then
 *      num_kv_heads k heads, then num_kv_heads v heads, 128 values each.
 * positions: int64 [num_tokens] (clamped to [0, max_position)); q_weight, k_weight: bf16 [128];
 * cos_sin: fp32 [max_position, 128], per position the cos of the 64 rotary frequencies, then
 *      their sin (the reference's cos_sin_cache).
 * q_out: bf16 [num_tokens, num_heads, 128] (normalised, rotated q); k_out: the same for k
 *      ([num_tokens, num_kv_heads, 128]) or NULL.
 * Caches, scales, slot_mapping, num_slots and scaled as in fp8attn_store_kvcache: the rotated K and
 * the raw V rows of tokens with a valid slot go to the caches.
 * Arithmetic: r = rsqrt(sum(x^2)/128 + eps), n = bf16((x r) w), then the rotation of n in fp32
 * rounded to bf16, then the e4m3 cast.
 */
FP8ATTN_API int fp8attn_qk_norm_rope_store(const void* qkv, int64_t qkv_row_stride,
                               const int64_t* positions, const void* q_weight,
                               const void* k_weight, float eps, const float* cos_sin,
                               int64_t max_position, void* q_out, void* k_out, void* k_cache,
                               void* v_cache, float* k_scale, float* v_scale,
                               const int32_t* slot_mapping, int64_t num_tokens, int num_heads,
                               int num_kv_heads, int head_dim, int64_t num_slots, int scaled,
                               void* stream);

/*
 * Workspace needed by fp8attn_decode (max_seqlen_q = 1) or fp8attn_prefill (its max_seqlen_q)
 * on the current device.  The workspace must be zero-filled before its first use; every call
 * leaves its counters at zero again.  One workspace must not be used by two calls that can run
 * at the same time.
 */
FP8ATTN_API int64_t fp8attn_workspace_bytes(int num_seqs, int num_heads, int num_kv_heads, int max_seqlen_q);

/*
 * Paged decode.  Replaces fp8_decode_attention (nanovllm/kernels/fp8_attention.py:173-207).
 * q: [num_seqs, num_heads, 128] bf16, rows q_row_stride elements apart; out: contiguous
 * [num_seqs, num_heads, 128] bf16.  Sequence b attends key positions < context_lens[b] (clamped
 * to max_num_blocks * block_size) of kv head h / (num_heads / num_kv_heads), position j in
 * cache block block_tables[b * block_tables_stride + j / block_size].  context_lens[b] <= 0
 * gives zeros.  Block ids outside [0, num_blocks) mask their positions out.
 */
FP8ATTN_API int fp8attn_decode(void* out, const void* q, int64_t q_row_stride, const void* k_cache,
                   const void* v_cache, const float* k_scale, const float* v_scale,
                   const int32_t* block_tables, int64_t block_tables_stride, int max_num_blocks,
                   const int32_t* context_lens, int num_seqs, int num_heads, int num_kv_heads,
                   int head_dim, int64_t num_blocks, int block_size, float softmax_scale,
                   void* workspace, int64_t workspace_bytes, void* stream);

/*
 * Varlen causal prefill / chunked prefill / speculative verify.  Replaces fp8_prefill_attention
 * (nanovllm/kernels/fp8_attention.py:314-353).
 * q: [Tq, num_heads, 128] bf16 (rows q_row_stride elements apart); out: contiguous like q.
 * Sequence s has query rows cu_seqlens_q[s]..cu_seqlens_q[s+1] and nk = cu_seqlens_k[s+1] -
 * cu_seqlens_k[s] key positions; query row i attends key positions j <= i + (nk - nq).
 *   block_tables != NULL: k/v are paged caches (as in fp8attn_decode), num_blocks = cache blocks.
 *   block_tables == NULL: k/v are contiguous [Tk, num_kv_heads, 128] e4m3 with token rows
 *                         kv_row_stride bytes apart, num_blocks = Tk, key rows from
 *                         cu_seqlens_k[s]; block_size is ignored.
 * Short query sequences (speculative verification, 1 + k rows) are served by the split-KV
 * decode engine inside this call; longer ones by the tensor-core prefill engine.
 */
FP8ATTN_API int fp8attn_prefill(void* out, const void* q, int64_t q_row_stride, const void* k, const void* v,
                    int64_t kv_row_stride, const float* k_scale, const float* v_scale,
                    const int32_t* block_tables, int64_t block_tables_stride, int max_num_blocks,
                    const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k, int num_seqs,
                    int max_seqlen_q, int max_seqlen_k, int num_heads, int num_kv_heads,
                    int head_dim, int64_t num_blocks, int block_size, float softmax_scale,
                    void* workspace, int64_t workspace_bytes, void* stream);

/* Persistent CTAs a decode (max_seqlen_q = 1) or prefill call of this shape launches on the
 * current device for its split-KV engine (diagnostics and benchmarking). */
FP8ATTN_API int fp8attn_decode_ctas(int num_seqs, int num_heads, int num_kv_heads, int max_seqlen_q);

/*
 * No counterpart in the reference.  fp8attn_decode without a caller-supplied workspace: the
 * split-KV scratch is a file-scope device array of FP8ATTN_NOALLOC_SCRATCH_BYTES inside the
 * library, so a call allocates no device memory (no cudaMalloc / cudaFree, no caching allocator).
 * For hosts that cannot allocate on the decode path: a C / cgo / ctypes host without a device
 * allocator of its own, or one that has handed all free HBM to the KV cache (the reference sizes
 * its cache from mem_get_info, nanovllm/engine/model_runner.py:104-122) and has none left for a
 * workspace.  Arguments, results and errors are those of fp8attn_decode.
 *   - Limit: a shape whose workspace (fp8attn_workspace_bytes(num_seqs, num_heads,
 *     num_kv_heads, 1)) exceeds FP8ATTN_NOALLOC_SCRATCH_BYTES is rejected with
 *     FP8ATTN_EWORKSPACE (on a 148-SM B200 this admits up to ~3200 (sequence, kv head) pairs
 *     for GQA groups <= 8; wider groups need fp8attn_decode).
 *   - Setup: the first call on a device resolves the array's address with cudaGetSymbolAddress
 *     (which loads the library's module on that device); make it outside any stream capture,
 *     with the device current.
 *   - Zero state: the array starts zeroed; its work counters (bytes 4..11) must be zero when a
 *     launch starts, and every launch leaves them zero.  Device error codes are recorded in its
 *     first word, which this call does not read (it never synchronises): read it with
 *     fp8attn_noalloc_read_error.
 *   - One scratch per device: calls whose kernels may overlap (other streams, other host threads,
 *     other processes sharing the context) race on it and give wrong results.  Serialise them.
 *   - The resolved address is kept for the life of the process: after cudaDeviceReset (or any
 *     other teardown of the device's primary context) this entry point must not be called again
 *     on that device.
 */
#define FP8ATTN_NOALLOC_SCRATCH_BYTES (32LL << 20)
FP8ATTN_API int fp8attn_decode_noalloc(void* out, const void* q, int64_t q_row_stride,
                   const void* k_cache, const void* v_cache, const float* k_scale,
                   const float* v_scale, const int32_t* block_tables, int64_t block_tables_stride,
                   int max_num_blocks, const int32_t* context_lens, int num_seqs, int num_heads,
                   int num_kv_heads, int head_dim, int64_t num_blocks, int block_size,
                   float softmax_scale, void* stream);

/* Device error word of fp8attn_decode_noalloc's scratch on the current device, copied into *dst
 * (host or device memory) in stream order: *dst holds it once `stream` has reached this point
 * (synchronise the stream, or wait on an event recorded after this call, before reading it).
 * clear != 0 also zeroes the word, after the copy.  Diagnostics: no counterpart in the reference. */
FP8ATTN_API int fp8attn_noalloc_read_error(int32_t* dst, int clear, void* stream);

/* Device error word of a workspace (the int32 at FP8ATTN_WS_ERROR_OFFSET: 0 = none, 1 = a bounded
 * wait timed out, 2 = bad block, 3 = tensor-memory allocation, 4 = workspace too small), copied
 * into *dst in stream order as above, so a host can check a step without a blocking read on the
 * hot path; clear != 0 zeroes it after the copy.  Diagnostics: no counterpart in the reference. */
FP8ATTN_API int fp8attn_read_error(const void* workspace, int32_t* dst, int clear, void* stream);

/* Tuning knob (process-wide, atomic): minimum key positions per split-KV work item, a multiple of
 * 128 (default 128).  Returns the previous value; other values are rejected with -1.  Calls that
 * are already launched keep the value they were planned with. */
FP8ATTN_API int fp8attn_set_decode_min_chunk(int tokens);

/*
 * FP8 block-scaled linear layer (replaces fp8_block_linear, nanovllm/kernels/fp8_linear.py:93-139,
 * called by nanovllm/layers/linear.py:58 for checkpoints quantised in 128 x 128 weight blocks).
 * Types: x and out bf16, xq and w e4m3 (one byte), x_scale and w_scale bf16.  Shapes: x [M, K],
 * w [N, K] (contiguous), w_scale [N / 128, K / 128] (contiguous), out [M, N]; N and K positive
 * multiples of 128, M >= 0 (M = 0 is a no-op).  Row strides are in elements of each tensor.
 *   fp8attn_fp8_dyn_quant (fp8_dyn_quant_kernel, :11-31): per token m and 128-column group g,
 *     s = max|x[m, g]| / 448 (1 for an all-zero group), xq = e4m3(clamp(x / s, -448, 448)),
 *     x_scale[m, g] = bf16(s).  xq [M, K] (row stride a multiple of 4), x_scale [M, K / 128]
 *     (contiguous).  x 16-byte aligned, its row stride a multiple of 8.
 *   fp8attn_fp8_block_gemm (fp8_block_gemm_kernel, :34-71): out[m, n] = bf16(sum over groups g,
 *     in order, of (xq[m, g] . w[n, g]) * (x_scale[m, g] * w_scale[n / 128, g])), each group's
 *     dot exact (fp32 tensor-core accumulation of e4m3 products) and the sum kept in fp32.
 *     xq, w and out 16-byte aligned, xq's row stride a multiple of 16 and out's a multiple of
 *     8.  workspace: at least
 *     fp8attn_fp8_gemm_workspace_bytes(M, N, K) bytes, 16-byte aligned; its first int32 is the
 *     device error word (fp8attn_read_error reads it), the rest holds split-K partial sums.
 *   fp8attn_fp8_block_linear: both, with xq and x_scale placed in the workspace after the GEMM's
 *     part; workspace of fp8attn_fp8_linear_workspace_bytes(M, N, K) bytes.
 * The workspace sizes depend on the current device's SM count (split-K ranges); they return -1
 * for invalid sizes.  Errors: FP8ATTN_EINVAL for shapes, strides, alignment and null pointers,
 * FP8ATTN_EWORKSPACE for a missing or small workspace.  Launches are asynchronous on `stream`.
 */
FP8ATTN_API int64_t fp8attn_fp8_gemm_workspace_bytes(int64_t M, int N, int K);
FP8ATTN_API int64_t fp8attn_fp8_linear_workspace_bytes(int64_t M, int N, int K);
FP8ATTN_API int fp8attn_fp8_dyn_quant(const void* x, int64_t x_row_stride, void* xq,
                   int64_t xq_row_stride, void* x_scale, int64_t M, int K, void* stream);
FP8ATTN_API int fp8attn_fp8_block_gemm(const void* xq, int64_t xq_row_stride, const void* x_scale,
                   const void* w, const void* w_scale, void* out, int64_t out_row_stride,
                   int64_t M, int N, int K, void* workspace, int64_t workspace_bytes, void* stream);
FP8ATTN_API int fp8attn_fp8_block_linear(const void* x, int64_t x_row_stride, const void* w,
                   const void* w_scale, void* out, int64_t out_row_stride, int64_t M, int N, int K,
                   void* workspace, int64_t workspace_bytes, void* stream);

/*
 * Row-parallel FP8 linear with its tensor-parallel all-reduce in one launch (replaces
 * RowParallelLinear.forward, nanovllm/layers/linear.py:235-239, for block-quantised weights:
 * y = fp8_block_linear(x_r, w_r, w_scale_r) on each rank, then dist.all_reduce(y)).
 *   Rank r passes its K slice: x [M, K] bf16 (K = in_features / world), w [N, K] e4m3 and
 *   w_scale [N / 128, K / 128] bf16 (the slices RowParallelLinear's loaders keep).  Each rank's
 *   output rows of a 128 x 128 tile are rounded to bf16 (the reference's local result), written
 *   over NVLink into the tile owner's receive buffer (owner = tile % world) and stamped; the owner
 *   adds the world partials in rank order in fp32, rounds to bf16 and writes the tile into every
 *   rank's output.  No host synchronisation and no collective library call.
 *   buffers[r]: rank r's buffer of fp8attn_tp_linear_layout(max_tokens, N, world) bytes, as
 *   mapped in this process (peer-accessible, e.g. torch symmetric memory), 256-byte aligned,
 *   zero-filled before the first call; the same allocation on every rank.  The result is at
 *   buffers[rank] + *out_offset, bf16 [M, N] rows N apart, complete when the launch ends and
 *   valid until this rank's next call on the buffers.
 *   epoch: this call's stamp, the same on every rank and larger than any earlier call's on the
 *   buffers (1, 2, 3, ...).  Every rank must make the same calls in the same order; a rank whose
 *   peers do not arrive gives up after 5 s and records 1 (wait timed out) in the workspace's
 *   error word (fp8attn_read_error).
 *   workspace: fp8attn_fp8_tp_linear_workspace_bytes(M, K) bytes, 16-byte aligned.
 *   Sizes: N and K multiples of 128, 0 <= M <= max_tokens, 1 <= world <= 8.
 */
FP8ATTN_API int64_t fp8attn_tp_linear_layout(int64_t max_tokens, int N, int world,
                   int64_t* out_offset, int64_t* recv_offset);
FP8ATTN_API int64_t fp8attn_fp8_tp_linear_workspace_bytes(int64_t M, int K);
FP8ATTN_API int fp8attn_fp8_tp_linear(const void* x, int64_t x_row_stride, const void* w,
                   const void* w_scale, void* const* buffers, int rank, int world, uint64_t epoch,
                   int64_t max_tokens, int64_t M, int N, int K, void* workspace,
                   int64_t workspace_bytes, void* stream);

/*
 * Self-checks of device-side mechanisms (no counterpart in the reference; used by the tests).
 *   fp8attn_diag_wait_timeout: num_ctas CTAs each claim one work item from the control block at
 *     `workspace` (ints: [0] error word, [1] next item, [2] CTAs finished, zeroed by the caller)
 *     and wait on an mbarrier that nothing arrives on, with the library's bounded wait given a
 *     limit of limit_ns: every wait must give up, record 1 (wait timed out) in the error word and
 *     let the launch finish with [1] and [2] back at zero.
 *   fp8attn_diag_exp2: poly[i] = the prefill softmax's FMA-pipe 2^x(i), mufu[i] = ex2.approx(x[i]).
 */
FP8ATTN_API int fp8attn_diag_wait_timeout(void* workspace, int64_t limit_ns, int num_ctas, void* stream);
FP8ATTN_API int fp8attn_diag_exp2(const float* x, float* poly, float* mufu, int64_t n, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FP8ATTN_H_ */
