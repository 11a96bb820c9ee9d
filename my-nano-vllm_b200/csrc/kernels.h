// Host-side launch interface between the C-ABI layer (capi.cu) and the kernels.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace fp8attn {

// ------------------------------------------------------------------ store
struct StoreParams {
  const uint16_t* key;  // bf16 [N, KVH, 128], rows `key_row_stride` elements apart
  int64_t key_row_stride;
  const uint16_t* value;
  int64_t value_row_stride;
  uint8_t* k_cache;  // e4m3 [num_slots, KVH, 128]
  uint8_t* v_cache;
  float* k_scale;  // fp32 [num_slots, KVH] or null
  float* v_scale;
  const int32_t* slot_mapping;  // [N]
  int64_t num_tokens;
  int64_t num_slots;
  int num_kv_heads;
  int scaled;  // 0: plain RNE cast (scale 1.0); 1: amax/448 per (token, kv head)
};
cudaError_t launch_store(const StoreParams& p, cudaStream_t stream);

// ------------------------------------------------------------------ q/k norm + rope + store
struct QkNormParams {
  const uint16_t* qkv;  // bf16 [N, row stride]: q heads, k heads, v heads of 128 each
  int64_t qkv_row_stride;  // elements
  const int64_t* positions;  // [N], clamped to [0, max_position)
  const uint16_t* q_weight;  // bf16 [128] (q_norm), [128] (k_norm)
  const uint16_t* k_weight;
  const float* cos_sin;  // fp32 [max_position, 128]: cos of the 64 frequencies, then sin
  int64_t max_position;
  float eps;
  uint16_t* q_out;  // bf16 [N, Hq, 128]
  uint16_t* k_out;  // bf16 [N, KVH, 128] or null
  uint8_t* k_cache;  // e4m3 [num_slots, KVH, 128]
  uint8_t* v_cache;
  float* k_scale;  // fp32 [num_slots, KVH] or null
  float* v_scale;
  const int32_t* slot_mapping;  // [N]; -1 (or out of range): not stored
  int64_t num_tokens;
  int64_t num_slots;
  int num_heads;
  int num_kv_heads;
  int scaled;
};
cudaError_t launch_qk_norm_rope_store(const QkNormParams& p, cudaStream_t stream);

// ------------------------------------------------------------------ FP8 block-scaled linear
// Dynamic quantisation of the activations: per token and 128-column group, scale = amax / 448
// (1 for an all-zero group), e4m3 = RNE(clamp(x / scale, +-448)), the scale stored as bf16.
struct Fp8QuantParams {
  const uint16_t* x;  // bf16 [M, K], rows x_row_stride elements apart
  int64_t x_row_stride;
  uint8_t* xq;        // e4m3 [M, K], rows xq_row_stride bytes apart
  int64_t xq_row_stride;
  uint16_t* x_scale;  // bf16 [M, K / 128]
  int64_t M;
  int K;
};
cudaError_t launch_fp8_dyn_quant(const Fp8QuantParams& p, cudaStream_t stream);

// out[M, N] = sum over 128-column blocks kb of (xq[:, kb] . w[:, kb]^T) * x_scale[m, kb] *
// w_scale[n / 128, kb], in fp32, rounded once to bf16.
struct Fp8GemmParams {
  const uint8_t* xq;        // e4m3 [M, K], rows xq_row_stride bytes apart (multiple of 16)
  int64_t xq_row_stride;
  const uint16_t* x_scale;  // bf16 [M, K / 128]
  const uint8_t* w;         // e4m3 [N, K], contiguous
  const uint16_t* w_scale;  // bf16 [N / 128, K / 128]
  uint16_t* out;            // bf16 [M, N], rows out_row_stride elements apart
  int64_t out_row_stride;
  float* partials;          // fp32 [splits, M, N] (split-K), from the workspace
  int* err;                 // device error word (workspace head)
  int64_t M;
  int N, K;
  int splits;               // K blocks are divided into this many ranges (one unit each)
};
constexpr int kFp8GemmTokens = 128;  // tokens per work unit (the MMA's N)
int fp8_gemm_splits(int64_t M, int N, int K, int num_sms);
int64_t fp8_gemm_workspace_bytes(int64_t M, int N, int K, int num_sms);
cudaError_t launch_fp8_block_gemm(const Fp8GemmParams& p, int num_sms, cudaStream_t stream);

// Row-parallel FP8 linear with the tensor-parallel all-reduce over peer memory (one kernel).
// Every rank computes y_r = x_r . w_r^T on its K slice; output tile t (128 tokens x 128 features,
// t = token tile * N/128 + feature block) belongs to rank t % world.  Pointers are each rank's
// buffers as mapped in this process (index = rank).  Per rank:
//   recv  bf16 [world][M][N]: the partial tile of source s at rows s * M + m;
//   out   bf16 [M][N]: the all-reduced output;
//   flags u64 [world + 1][tiles_cap]: row s < world = the call's stamp once source s's partial of
//         tile t has landed here; row world = the stamp once tile t's final values are in `out`.
constexpr int kMaxTpRanks = 8;
struct Fp8TpParams {
  uint16_t* recv[kMaxTpRanks];
  uint16_t* out[kMaxTpRanks];
  unsigned long long* flags[kMaxTpRanks];
  unsigned long long epoch;  // this call's stamp: larger than every earlier call's on the buffers
  int64_t tiles_cap;         // flags per row
  int rank, world;
};
cudaError_t launch_fp8_tp_gemm(const Fp8GemmParams& p, const Fp8TpParams& tp, int num_sms,
                               cudaStream_t stream);

// ------------------------------------------------------------------ decode engine
// Control block at the head of the decode workspace (ints):
//   [0] sticky device error code, [1] next work item, [2] CTAs finished.
constexpr int kCtrlInts = 64;  // 256 bytes
constexpr int kMaxSeqs = 2048;  // per launch (the published plan below has room for this many)
// Plan published by the decode kernel for its combine kernel, right after the control block:
// [0] chunk size, [1] item count, [2 + b] item prefix of sequence b (b = 0 .. num_seqs).
constexpr int kPlanInts = kMaxSeqs + 8;
constexpr int kDecodeTile = 128;  // key positions per decode pipeline stage

struct DecodeParams {
  uint16_t* out;  // bf16
  int64_t out_row_stride;  // elements per query token row
  const uint16_t* q;  // bf16
  int64_t q_row_stride;
  const float* k_scale;  // per (slot, kv head) or null
  const float* v_scale;
  const int32_t* block_tables;
  int64_t bt_stride;
  int max_blocks;
  const int32_t* context_lens;  // decode mode
  const int32_t* cu_q;  // spec mode (prefill entry point, short query sequences)
  const int32_t* cu_k;
  int num_seqs;
  int num_heads;
  int num_kv_heads;
  int group;  // num_heads / num_kv_heads
  int block_size;
  int box_rows;  // TMA box height: 128, 64, 32 or 16 (divides block_size and kDecodeTile)
  int64_t num_blocks;
  int spec_mode;
  int spec_q_max;  // spec mode: sequences with 1 <= nq <= spec_q_max are handled here
  int max_rowgroups;
  int min_chunk;  // minimum tokens per work item (multiple of 64)
  float scale_log2;  // softmax_scale * log2(e)
  int* ctrl;
  int* plan;      // kPlanInts ints, written by the decode kernel, read by its combine kernel
  float* partials;
  int max_items;
};

// Rows (query rows of one kv head) per work item for the two engine widths.
inline int decode_rows(int nt) { return 8 * nt; }
int64_t decode_workspace_bytes(int num_seqs, int num_kv_heads, int max_rowgroups, int rows,
                               int grid);
int64_t decode_max_items(int64_t pairs, int grid);
// Grid (persistent CTAs) the decode engine uses on the current device for the given width.
int decode_grid(int nt);
// Engine variants: nt = 8-row planes per row group (R = 8 nt rows, 1..3), rv = rows the
// softmax processes (4 or R).
// Grid an actual launch uses (persistent CTAs resident at once) for this batch size.
int decode_launch_grid(int nt, int rv, int num_seqs);
cudaError_t launch_decode(const DecodeParams& p, int nt, int rv, const CUtensorMap& tmk,
                          const CUtensorMap& tmv, cudaStream_t stream);

// ------------------------------------------------------------------ prefill engine
struct PrefillParams {
  uint16_t* out;
  int64_t out_row_stride;
  const uint16_t* q;
  int64_t q_row_stride;
  const uint8_t* k;  // paged cache [nb, BS, KVH, 128] or contiguous [Tk, KVH, 128]
  const uint8_t* v;
  int64_t kv_row_stride;  // bytes between consecutive token rows (contiguous layout)
  const float* k_scale;
  const float* v_scale;
  const int32_t* block_tables;  // null: contiguous layout
  int64_t bt_stride;
  int max_blocks;
  const int32_t* cu_q;
  const int32_t* cu_k;
  int num_seqs;
  int max_seqlen_q;
  int num_heads;
  int num_kv_heads;
  int group;
  int block_size;
  int64_t num_blocks;  // paged: blocks in the cache; contiguous: token rows
  int min_q;  // sequences with nq < min_q are left to the decode engine
  float scale_log2;
  int* err;
};
cudaError_t launch_prefill(const PrefillParams& p, cudaStream_t stream);

}  // namespace fp8attn
