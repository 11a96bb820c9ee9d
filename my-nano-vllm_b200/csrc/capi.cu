// C-ABI layer: argument validation, TMA descriptor encoding, engine selection and launches.
// See include/fp8attn.h for the contract of every entry point.
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <atomic>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/fp8attn.h"
#include "common.cuh"
#include "kernels.h"

namespace {

thread_local std::string g_last_error;
std::atomic<int> g_min_chunk{128};

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(FP8ATTN_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// The paged cache viewed as a 2-D byte tensor [num_blocks * block_size, KVH * 128]; one box is
// `box_rows` token rows x the 128 bytes of one kv head, 128-byte swizzled.  L2 fills are promoted
// to 128 bytes, the row a box reads: 256 would pull in the next kv head's row, which another
// CTA's item reads, often after it was evicted (measured 0.4-3 % slower on the decode shapes).
int make_cache_map(CUtensorMap* map, const void* cache, int64_t rows, int kvh, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return fail(FP8ATTN_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(kvh) * fp8attn::kHeadDim,
                              static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(kvh) * fp8attn::kHeadDim};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(fp8attn::kHeadDim),
                             static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(cache), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FP8ATTN_ECUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
  return FP8ATTN_OK;
}

// Query sequences with at most this many rows go to the split-KV decode engine inside the
// prefill entry point (speculative verification: 1 + k rows).
int spec_q_max(int group) {
  int m = 64 / group;
  if (m > 16) m = 16;
  if (m < 1) m = 1;
  return m;
}

struct EnginePlan {
  int nt;             // 8-row planes per row group: R = 8 nt rows (1..3)
  int rv;             // rows the softmax processes per row group (4, or R)
  int rows;
  int max_rowgroups;
};

EnginePlan plan_engine(int group, int max_q) {
  EnginePlan e;
  const int r = group * (max_q < 1 ? 1 : max_q);
  e.nt = r <= 8 ? 1 : (r <= 16 ? 2 : 3);
  e.rows = fp8attn::decode_rows(e.nt);
  e.rv = r <= 4 ? 4 : e.rows;
  e.max_rowgroups = (r + e.rows - 1) / e.rows;
  return e;
}

// TMA box height of the decode engine: divides both its 32-token tile and the block size.
int box_rows_for(int block_size) {
  static_assert(fp8attn::kDecodeTile == 128, "box heights below assume 128-token tiles");
  for (int r = 128; r > 16; r >>= 1)
    if (block_size % r == 0) return r;
  return 16;
}

int check_common(int num_seqs, int num_heads, int num_kv_heads, int head_dim) {
  if (head_dim != fp8attn::kHeadDim)
    return fail(FP8ATTN_EINVAL, "head_dim must be 128 (got %d)", head_dim);
  if (num_heads <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads != 0)
    return fail(FP8ATTN_EINVAL, "num_heads (%d) must be a positive multiple of num_kv_heads (%d)",
                num_heads, num_kv_heads);
  if (num_seqs < 0 || num_seqs > fp8attn::kMaxSeqs)
    return fail(FP8ATTN_EINVAL, "num_seqs must be in [0, %d] (got %d)", fp8attn::kMaxSeqs,
                num_seqs);
  return FP8ATTN_OK;
}

int check_paged(const void* k, const void* v, const int32_t* bt, int64_t bt_stride,
                int max_blocks, int64_t num_blocks, int block_size) {
  if (k == nullptr || v == nullptr || bt == nullptr)
    return fail(FP8ATTN_EINVAL, "null cache or block_tables pointer");
  if (!aligned16(k) || !aligned16(v))
    return fail(FP8ATTN_EINVAL, "caches must be 16-byte aligned");
  if (block_size <= 0 || block_size % 16 != 0)
    return fail(FP8ATTN_EINVAL, "block_size must be a positive multiple of 16 (got %d)",
                block_size);
  if (max_blocks < 0 || bt_stride < max_blocks)
    return fail(FP8ATTN_EINVAL, "bad block table geometry (max_num_blocks %d, stride %lld)",
                max_blocks, static_cast<long long>(bt_stride));
  if (static_cast<int64_t>(max_blocks) * block_size >= (1 << 24))
    return fail(FP8ATTN_EINVAL, "max_num_blocks * block_size must be < 2^24");
  if (num_blocks <= 0 || num_blocks * block_size > INT32_MAX)
    return fail(FP8ATTN_EINVAL, "num_blocks * block_size must be in (0, 2^31)");
  return FP8ATTN_OK;
}

}  // namespace

extern "C" {

int fp8attn_version(void) { return 100; }

const char* fp8attn_last_error(void) { return g_last_error.c_str(); }

int fp8attn_decode_ctas(int num_seqs, int num_heads, int num_kv_heads, int max_seqlen_q) {
  if (num_seqs < 0 || num_heads <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads) return -1;
  const int group = num_heads / num_kv_heads;
  const int mq = max_seqlen_q <= 1 ? 1 : (max_seqlen_q < spec_q_max(group) ? max_seqlen_q
                                                                           : spec_q_max(group));
  const EnginePlan e = plan_engine(group, mq);
  return fp8attn::decode_launch_grid(e.nt, e.rv, num_seqs);
}

int fp8attn_set_decode_min_chunk(int tokens) {
  if (tokens < fp8attn::kDecodeTile || tokens % fp8attn::kDecodeTile != 0) return -1;
  return g_min_chunk.exchange(tokens);
}

int fp8attn_store_kvcache(const void* key, int64_t key_row_stride, const void* value,
                          int64_t value_row_stride, void* k_cache, void* v_cache, float* k_scale,
                          float* v_scale, const int32_t* slot_mapping, int64_t num_tokens,
                          int num_kv_heads, int head_dim, int64_t num_slots, int scaled,
                          void* stream) {
  if (head_dim != fp8attn::kHeadDim)
    return fail(FP8ATTN_EINVAL, "head_dim must be 128 (got %d)", head_dim);
  if (num_tokens < 0 || num_kv_heads <= 0 || num_slots < 0)
    return fail(FP8ATTN_EINVAL, "bad sizes");
  if (num_tokens == 0) return FP8ATTN_OK;
  if (!key || !value || !k_cache || !v_cache || !slot_mapping)
    return fail(FP8ATTN_EINVAL, "null pointer argument");
  if (!aligned16(k_cache) || !aligned16(v_cache))
    return fail(FP8ATTN_EINVAL, "caches must be 16-byte aligned");
  if ((reinterpret_cast<uintptr_t>(key) & 1) || (reinterpret_cast<uintptr_t>(value) & 1))
    return fail(FP8ATTN_EINVAL, "key/value must be 2-byte aligned");
  if ((k_scale == nullptr) != (v_scale == nullptr))
    return fail(FP8ATTN_EINVAL, "k_scale and v_scale must both be given or both be null");
  if (scaled && k_scale == nullptr)
    return fail(FP8ATTN_EINVAL, "scaled mode needs scale arrays");
  fp8attn::StoreParams p;
  p.key = static_cast<const uint16_t*>(key);
  p.key_row_stride = key_row_stride;
  p.value = static_cast<const uint16_t*>(value);
  p.value_row_stride = value_row_stride;
  p.k_cache = static_cast<uint8_t*>(k_cache);
  p.v_cache = static_cast<uint8_t*>(v_cache);
  p.k_scale = k_scale;
  p.v_scale = v_scale;
  p.slot_mapping = slot_mapping;
  p.num_tokens = num_tokens;
  p.num_slots = num_slots;
  p.num_kv_heads = num_kv_heads;
  p.scaled = scaled ? 1 : 0;
  const cudaError_t e = fp8attn::launch_store(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "store launch");
  return FP8ATTN_OK;
}

int64_t fp8attn_workspace_bytes(int num_seqs, int num_heads, int num_kv_heads,
                                int max_seqlen_q) {
  if (num_seqs < 0 || num_heads <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads) return -1;
  const int group = num_heads / num_kv_heads;
  const int mq = max_seqlen_q <= 1 ? 1 : (max_seqlen_q < spec_q_max(group) ? max_seqlen_q
                                                                           : spec_q_max(group));
  const EnginePlan e = plan_engine(group, mq);
  return fp8attn::decode_workspace_bytes(num_seqs, num_kv_heads, e.max_rowgroups, e.rows,
                                         fp8attn::decode_grid(e.nt));
}

static int run_decode_engine(fp8attn::DecodeParams& p, const EnginePlan& e, const void* k_cache,
                             const void* v_cache, void* workspace, int64_t workspace_bytes,
                             cudaStream_t stream) {
  const int grid = fp8attn::decode_grid(e.nt);
  const int64_t need =
      fp8attn::decode_workspace_bytes(p.num_seqs, p.num_kv_heads, e.max_rowgroups, e.rows, grid);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(FP8ATTN_EWORKSPACE, "workspace of %lld bytes is smaller than the %lld needed",
                static_cast<long long>(workspace_bytes), static_cast<long long>(need));
  if (!aligned16(workspace)) return fail(FP8ATTN_EINVAL, "workspace must be 16-byte aligned");
  const int64_t pairs = static_cast<int64_t>(p.num_seqs) * p.num_kv_heads * e.max_rowgroups;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  p.ctrl = reinterpret_cast<int*>(ws);
  p.plan = reinterpret_cast<int*>(ws + fp8attn::kCtrlInts * 4);
  p.partials = reinterpret_cast<float*>(ws + fp8attn::kCtrlInts * 4 + fp8attn::kPlanInts * 4);
  p.max_items = static_cast<int>(fp8attn::decode_max_items(pairs, grid));
  p.max_rowgroups = e.max_rowgroups;
  p.min_chunk = g_min_chunk.load();
  p.box_rows = box_rows_for(p.block_size);
  CUtensorMap tmk, tmv;
  const int64_t rows = p.num_blocks * p.block_size;
  int rc = make_cache_map(&tmk, k_cache, rows, p.num_kv_heads, p.box_rows);
  if (rc) return rc;
  rc = make_cache_map(&tmv, v_cache, rows, p.num_kv_heads, p.box_rows);
  if (rc) return rc;
  const cudaError_t err = fp8attn::launch_decode(p, e.nt, e.rv, tmk, tmv, stream);
  if (err != cudaSuccess) return cuda_fail(err, "decode launch");
  return FP8ATTN_OK;
}

static int launch_prefill_engine(void* out, const void* q, int64_t q_row_stride, const void* k,
                                 const void* v, int64_t kv_row_stride, const float* k_scale,
                                 const float* v_scale, const int32_t* block_tables,
                                 int64_t block_tables_stride, int max_num_blocks,
                                 const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k,
                                 int num_seqs, int max_seqlen_q, int num_heads, int num_kv_heads,
                                 int group, bool paged, int64_t num_blocks, int block_size,
                                 int min_q, float scale_log2, void* workspace, cudaStream_t st) {
  const int head_dim = fp8attn::kHeadDim;
  fp8attn::PrefillParams pp{};
  pp.out = static_cast<uint16_t*>(out);
  pp.out_row_stride = static_cast<int64_t>(num_heads) * head_dim;
  pp.q = static_cast<const uint16_t*>(q);
  pp.q_row_stride = q_row_stride;
  pp.k = static_cast<const uint8_t*>(k);
  pp.v = static_cast<const uint8_t*>(v);
  pp.kv_row_stride = paged ? static_cast<int64_t>(num_kv_heads) * head_dim : kv_row_stride;
  pp.k_scale = k_scale;
  pp.v_scale = v_scale;
  pp.block_tables = block_tables;
  pp.bt_stride = block_tables_stride;
  pp.max_blocks = max_num_blocks;
  pp.cu_q = cu_seqlens_q;
  pp.cu_k = cu_seqlens_k;
  pp.num_seqs = num_seqs;
  pp.max_seqlen_q = max_seqlen_q;
  pp.num_heads = num_heads;
  pp.num_kv_heads = num_kv_heads;
  pp.group = group;
  pp.block_size = paged ? block_size : 1;
  pp.num_blocks = num_blocks;
  pp.min_q = min_q;
  pp.scale_log2 = scale_log2;
  pp.err = static_cast<int*>(workspace);
  const cudaError_t e = fp8attn::launch_prefill(pp, st);
  if (e != cudaSuccess) return cuda_fail(e, "prefill launch");
  return FP8ATTN_OK;
}

int fp8attn_qk_norm_rope_store(const void* qkv, int64_t qkv_row_stride, const int64_t* positions,
                               const void* q_weight, const void* k_weight, float eps,
                               const float* cos_sin, int64_t max_position, void* q_out, void* k_out,
                               void* k_cache, void* v_cache, float* k_scale, float* v_scale,
                               const int32_t* slot_mapping, int64_t num_tokens, int num_heads,
                               int num_kv_heads, int head_dim, int64_t num_slots, int scaled,
                               void* stream) {
  if (head_dim != fp8attn::kHeadDim)
    return fail(FP8ATTN_EINVAL, "head_dim must be 128 (got %d)", head_dim);
  if (num_tokens < 0 || num_heads <= 0 || num_kv_heads <= 0 || num_slots < 0 || max_position <= 0)
    return fail(FP8ATTN_EINVAL, "bad sizes");
  if (num_tokens == 0) return FP8ATTN_OK;
  if (!qkv || !positions || !q_weight || !k_weight || !cos_sin || !q_out || !k_cache ||
      !v_cache || !slot_mapping)
    return fail(FP8ATTN_EINVAL, "null pointer argument");
  if ((reinterpret_cast<uintptr_t>(qkv) & 7) || qkv_row_stride % 4 != 0 ||
      qkv_row_stride < static_cast<int64_t>(num_heads + 2 * num_kv_heads) * head_dim)
    return fail(FP8ATTN_EINVAL, "qkv must be 8-byte aligned with rows of (Hq + 2 KVH) * 128");
  if ((reinterpret_cast<uintptr_t>(q_out) & 7) || (k_out && (reinterpret_cast<uintptr_t>(k_out) & 7)) ||
      (reinterpret_cast<uintptr_t>(q_weight) & 7) || (reinterpret_cast<uintptr_t>(k_weight) & 7) ||
      (reinterpret_cast<uintptr_t>(cos_sin) & 15) || (reinterpret_cast<uintptr_t>(k_cache) & 3) ||
      (reinterpret_cast<uintptr_t>(v_cache) & 3))
    return fail(FP8ATTN_EINVAL, "misaligned pointer argument");
  if ((k_scale == nullptr) != (v_scale == nullptr))
    return fail(FP8ATTN_EINVAL, "k_scale and v_scale must both be given or both be null");
  if (scaled && k_scale == nullptr) return fail(FP8ATTN_EINVAL, "scaled mode needs scale arrays");
  fp8attn::QkNormParams p;
  p.qkv = static_cast<const uint16_t*>(qkv);
  p.qkv_row_stride = qkv_row_stride;
  p.positions = positions;
  p.q_weight = static_cast<const uint16_t*>(q_weight);
  p.k_weight = static_cast<const uint16_t*>(k_weight);
  p.cos_sin = cos_sin;
  p.max_position = max_position;
  p.eps = eps;
  p.q_out = static_cast<uint16_t*>(q_out);
  p.k_out = static_cast<uint16_t*>(k_out);
  p.k_cache = static_cast<uint8_t*>(k_cache);
  p.v_cache = static_cast<uint8_t*>(v_cache);
  p.k_scale = k_scale;
  p.v_scale = v_scale;
  p.slot_mapping = slot_mapping;
  p.num_tokens = num_tokens;
  p.num_slots = num_slots;
  p.num_heads = num_heads;
  p.num_kv_heads = num_kv_heads;
  p.scaled = scaled ? 1 : 0;
  const cudaError_t e = fp8attn::launch_qk_norm_rope_store(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "q/k norm + rope + store launch");
  return FP8ATTN_OK;
}

int fp8attn_read_error(const void* workspace, int32_t* dst, int clear, void* stream) {
  if (workspace == nullptr || dst == nullptr) return fail(FP8ATTN_EINVAL, "null pointer argument");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* word = static_cast<uint8_t*>(const_cast<void*>(workspace)) + FP8ATTN_WS_ERROR_OFFSET;
  cudaError_t e = cudaMemcpyAsync(dst, word, sizeof(int32_t), cudaMemcpyDefault, st);
  if (e != cudaSuccess) return cuda_fail(e, "error word copy");
  if (clear) {
    e = cudaMemsetAsync(word, 0, sizeof(int32_t), st);
    if (e != cudaSuccess) return cuda_fail(e, "error word clear");
  }
  return FP8ATTN_OK;
}

int fp8attn_decode(void* out, const void* q, int64_t q_row_stride, const void* k_cache,
                   const void* v_cache, const float* k_scale, const float* v_scale,
                   const int32_t* block_tables, int64_t block_tables_stride, int max_num_blocks,
                   const int32_t* context_lens, int num_seqs, int num_heads, int num_kv_heads,
                   int head_dim, int64_t num_blocks, int block_size, float softmax_scale,
                   void* workspace, int64_t workspace_bytes, void* stream) {
  int rc = check_common(num_seqs, num_heads, num_kv_heads, head_dim);
  if (rc) return rc;
  if (num_seqs == 0) return FP8ATTN_OK;
  rc = check_paged(k_cache, v_cache, block_tables, block_tables_stride, max_num_blocks,
                   num_blocks, block_size);
  if (rc) return rc;
  if (!out || !q || !context_lens) return fail(FP8ATTN_EINVAL, "null pointer argument");
  if (!aligned16(out) || !aligned16(q) || q_row_stride % 8 != 0 ||
      q_row_stride < static_cast<int64_t>(num_heads) * head_dim)
    return fail(FP8ATTN_EINVAL, "q/out must be 16-byte aligned with rows of num_heads*128");
  if ((k_scale == nullptr) != (v_scale == nullptr))
    return fail(FP8ATTN_EINVAL, "k_scale and v_scale must both be given or both be null");
  const int group = num_heads / num_kv_heads;
  const EnginePlan e = plan_engine(group, 1);
  if (e.max_rowgroups > 127) return fail(FP8ATTN_EINVAL, "too many query heads per kv head");
  fp8attn::DecodeParams p{};
  p.out = static_cast<uint16_t*>(out);
  p.out_row_stride = static_cast<int64_t>(num_heads) * head_dim;
  p.q = static_cast<const uint16_t*>(q);
  p.q_row_stride = q_row_stride;
  p.k_scale = k_scale;
  p.v_scale = v_scale;
  p.block_tables = block_tables;
  p.bt_stride = block_tables_stride;
  p.max_blocks = max_num_blocks;
  p.context_lens = context_lens;
  p.num_seqs = num_seqs;
  p.num_heads = num_heads;
  p.num_kv_heads = num_kv_heads;
  p.group = group;
  p.block_size = block_size;
  p.num_blocks = num_blocks;
  p.spec_mode = 0;
  p.spec_q_max = 1;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  return run_decode_engine(p, e, k_cache, v_cache, workspace, workspace_bytes,
                           static_cast<cudaStream_t>(stream));
}

int fp8attn_prefill(void* out, const void* q, int64_t q_row_stride, const void* k, const void* v,
                    int64_t kv_row_stride, const float* k_scale, const float* v_scale,
                    const int32_t* block_tables, int64_t block_tables_stride, int max_num_blocks,
                    const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k, int num_seqs,
                    int max_seqlen_q, int max_seqlen_k, int num_heads, int num_kv_heads,
                    int head_dim, int64_t num_blocks, int block_size, float softmax_scale,
                    void* workspace, int64_t workspace_bytes, void* stream) {
  (void)max_seqlen_k;  // the reference does not use it either (fp8_attention.py:314-353)
  int rc = check_common(num_seqs, num_heads, num_kv_heads, head_dim);
  if (rc) return rc;
  if (num_seqs == 0 || max_seqlen_q <= 0) return FP8ATTN_OK;
  if (!out || !q || !k || !v || !cu_seqlens_q || !cu_seqlens_k)
    return fail(FP8ATTN_EINVAL, "null pointer argument");
  if (!aligned16(out) || !aligned16(q) || q_row_stride % 8 != 0 ||
      q_row_stride < static_cast<int64_t>(num_heads) * head_dim)
    return fail(FP8ATTN_EINVAL, "q/out must be 16-byte aligned with rows of num_heads*128");
  if ((k_scale == nullptr) != (v_scale == nullptr))
    return fail(FP8ATTN_EINVAL, "k_scale and v_scale must both be given or both be null");
  const int group = num_heads / num_kv_heads;
  const bool paged = block_tables != nullptr;
  if (paged) {
    rc = check_paged(k, v, block_tables, block_tables_stride, max_num_blocks, num_blocks,
                     block_size);
    if (rc) return rc;
  } else {
    if (kv_row_stride < static_cast<int64_t>(num_kv_heads) * head_dim || kv_row_stride % 16 != 0 ||
        !aligned16(k) || !aligned16(v) || num_blocks < 0)
      return fail(FP8ATTN_EINVAL, "bad contiguous k/v layout");
  }
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const float scale_log2 = softmax_scale * 1.4426950408889634f;
  int min_q = 1;
  // speculative-verify sized sequences (paged layout) go to the split-KV decode engine, the
  // rest to the prefill engine.  The prefill kernel is launched first and the decode engine
  // after it as a programmatic dependent, so when no sequence is short the engine's set-up and
  // empty plan overlap the prefill kernel's tail instead of delaying its start.
  fp8attn::DecodeParams p{};
  EnginePlan e{};
  if (paged) {
    const int sq = spec_q_max(group);
    const int mq = max_seqlen_q < sq ? max_seqlen_q : sq;
    e = plan_engine(group, mq);
    const int64_t need = fp8attn::decode_workspace_bytes(num_seqs, num_kv_heads, e.max_rowgroups,
                                                         e.rows, fp8attn::decode_grid(e.nt));
    if (workspace == nullptr || workspace_bytes < need)
      return fail(FP8ATTN_EWORKSPACE, "workspace of %lld bytes is smaller than the %lld needed",
                  static_cast<long long>(workspace_bytes), static_cast<long long>(need));
    p.out = static_cast<uint16_t*>(out);
    p.out_row_stride = static_cast<int64_t>(num_heads) * head_dim;
    p.q = static_cast<const uint16_t*>(q);
    p.q_row_stride = q_row_stride;
    p.k_scale = k_scale;
    p.v_scale = v_scale;
    p.block_tables = block_tables;
    p.bt_stride = block_tables_stride;
    p.max_blocks = max_num_blocks;
    p.cu_q = cu_seqlens_q;
    p.cu_k = cu_seqlens_k;
    p.num_seqs = num_seqs;
    p.num_heads = num_heads;
    p.num_kv_heads = num_kv_heads;
    p.group = group;
    p.block_size = block_size;
    p.num_blocks = num_blocks;
    p.spec_mode = 1;
    p.spec_q_max = mq;
    p.scale_log2 = scale_log2;
    min_q = mq + 1;
  } else if (workspace == nullptr || workspace_bytes < 256) {
    return fail(FP8ATTN_EWORKSPACE, "workspace missing");
  }
  if (max_seqlen_q >= min_q) {
    rc = launch_prefill_engine(out, q, q_row_stride, k, v, kv_row_stride, k_scale, v_scale,
                               block_tables, block_tables_stride, max_num_blocks, cu_seqlens_q,
                               cu_seqlens_k, num_seqs, max_seqlen_q, num_heads, num_kv_heads,
                               group, paged, num_blocks, block_size, min_q, scale_log2,
                               workspace, st);
    if (rc) return rc;
  }
  if (paged) return run_decode_engine(p, e, k, v, workspace, workspace_bytes, st);
  return FP8ATTN_OK;
}

}  // extern "C"

// ---------------------------------------------------------------- decode without allocation
// The split-KV scratch of fp8attn_decode_noalloc: control words, plan and partials, laid out as
// a caller workspace.  Zero at module load; the decode kernel returns its counters to zero at
// the end of every launch.
static __device__ __align__(256) uint8_t g_noalloc_scratch[FP8ATTN_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_addr[kMaxDevices] = {};

int noalloc_scratch(void** addr) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(FP8ATTN_EINVAL, "device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(no-alloc scratch)");
    g_noalloc_addr[dev] = p;
  }
  *addr = g_noalloc_addr[dev];
  return FP8ATTN_OK;
}
}  // namespace

extern "C" {

int fp8attn_decode_noalloc(void* out, const void* q, int64_t q_row_stride, const void* k_cache,
                           const void* v_cache, const float* k_scale, const float* v_scale,
                           const int32_t* block_tables, int64_t block_tables_stride,
                           int max_num_blocks, const int32_t* context_lens, int num_seqs,
                           int num_heads, int num_kv_heads, int head_dim, int64_t num_blocks,
                           int block_size, float softmax_scale, void* stream) {
  int rc = check_common(num_seqs, num_heads, num_kv_heads, head_dim);
  if (rc) return rc;
  if (num_seqs == 0) return FP8ATTN_OK;
  const int64_t need = fp8attn_workspace_bytes(num_seqs, num_heads, num_kv_heads, 1);
  if (need > FP8ATTN_NOALLOC_SCRATCH_BYTES)
    return fail(FP8ATTN_EWORKSPACE,
                "decode of %d sequences x %d kv heads (%d q heads) needs %lld bytes of scratch; "
                "the static scratch of fp8attn_decode_noalloc holds %lld: use fp8attn_decode "
                "with a workspace",
                num_seqs, num_kv_heads, num_heads, static_cast<long long>(need),
                static_cast<long long>(FP8ATTN_NOALLOC_SCRATCH_BYTES));
  void* scratch = nullptr;
  rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  return fp8attn_decode(out, q, q_row_stride, k_cache, v_cache, k_scale, v_scale, block_tables,
                        block_tables_stride, max_num_blocks, context_lens, num_seqs, num_heads,
                        num_kv_heads, head_dim, num_blocks, block_size, softmax_scale, scratch,
                        FP8ATTN_NOALLOC_SCRATCH_BYTES, stream);
}

int fp8attn_noalloc_read_error(int32_t* dst, int clear, void* stream) {
  if (dst == nullptr) return fail(FP8ATTN_EINVAL, "null destination");
  void* scratch = nullptr;
  const int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  return fp8attn_read_error(scratch, dst, clear, stream);
}

}  // extern "C"

// ---------------------------------------------------------------- FP8 block-scaled linear
namespace {

int64_t round16(int64_t v) { return (v + 15) & ~int64_t{15}; }

int device_sms() {
  static int sms[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  if (sms[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    sms[dev] = n > 0 ? n : 148;
  }
  return sms[dev];
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

int check_linear_sizes(int64_t M, int N, int K) {
  if (M < 0 || N <= 0 || K <= 0 || N % 128 != 0 || K % 128 != 0)
    return fail(FP8ATTN_EINVAL, "fp8 linear needs M >= 0 and N, K positive multiples of 128 "
                "(got M=%lld N=%d K=%d)", static_cast<long long>(M), N, K);
  if ((M + fp8attn::kFp8GemmTokens - 1) / fp8attn::kFp8GemmTokens * (N / 128) > (1LL << 26))
    return fail(FP8ATTN_EINVAL, "fp8 linear: M=%lld x N=%d is more than 2^26 output tiles",
                static_cast<long long>(M), N);
  return FP8ATTN_OK;
}

int run_quant(const void* x, int64_t x_row_stride, void* xq, int64_t xq_row_stride,
              void* x_scale, int64_t M, int K, cudaStream_t st) {
  if (M == 0) return FP8ATTN_OK;
  if (x == nullptr || xq == nullptr || x_scale == nullptr)
    return fail(FP8ATTN_EINVAL, "fp8 quant: null pointer argument");
  if (!aligned(x, 16) || x_row_stride < K || x_row_stride % 8 != 0)
    return fail(FP8ATTN_EINVAL, "fp8 quant: x must be 16-byte aligned with a row stride >= K "
                "that is a multiple of 8 elements");
  if (!aligned(xq, 4) || xq_row_stride < K || xq_row_stride % 4 != 0)
    return fail(FP8ATTN_EINVAL, "fp8 quant: xq must be 4-byte aligned with a row stride >= K "
                "that is a multiple of 4 bytes");
  if (!aligned(x_scale, 2)) return fail(FP8ATTN_EINVAL, "fp8 quant: x_scale must be 2-byte aligned");
  fp8attn::Fp8QuantParams p;
  p.x = static_cast<const uint16_t*>(x);
  p.x_row_stride = x_row_stride;
  p.xq = static_cast<uint8_t*>(xq);
  p.xq_row_stride = xq_row_stride;
  p.x_scale = static_cast<uint16_t*>(x_scale);
  p.M = M;
  p.K = K;
  const cudaError_t e = fp8attn::launch_fp8_dyn_quant(p, st);
  return e == cudaSuccess ? FP8ATTN_OK : cuda_fail(e, "fp8 quant launch");
}

int run_gemm(const void* xq, int64_t xq_row_stride, const void* x_scale, const void* w,
             const void* w_scale, void* out, int64_t out_row_stride, int64_t M, int N, int K,
             void* workspace, int64_t workspace_bytes, cudaStream_t st) {
  if (M == 0) return FP8ATTN_OK;
  if (xq == nullptr || x_scale == nullptr || w == nullptr || w_scale == nullptr || out == nullptr)
    return fail(FP8ATTN_EINVAL, "fp8 gemm: null pointer argument");
  if (!aligned(xq, 16) || !aligned(w, 16) || xq_row_stride < K || xq_row_stride % 16 != 0)
    return fail(FP8ATTN_EINVAL, "fp8 gemm: xq and w must be 16-byte aligned, xq's row stride "
                ">= K and a multiple of 16 bytes");
  if (!aligned(x_scale, 2) || !aligned(w_scale, 2) || !aligned(out, 16) || out_row_stride < N ||
      out_row_stride % 8 != 0)
    return fail(FP8ATTN_EINVAL, "fp8 gemm: scales must be 2-byte aligned, out 16-byte aligned "
                "with a row stride >= N that is a multiple of 8");
  const int sms = device_sms();
  const int64_t need = fp8attn::fp8_gemm_workspace_bytes(M, N, K, sms);
  if (workspace == nullptr || workspace_bytes < need || !aligned(workspace, 16))
    return fail(FP8ATTN_EWORKSPACE, "fp8 gemm: workspace of %lld bytes (16-byte aligned) needed, "
                "got %lld", static_cast<long long>(need), static_cast<long long>(workspace_bytes));
  fp8attn::Fp8GemmParams p;
  p.xq = static_cast<const uint8_t*>(xq);
  p.xq_row_stride = xq_row_stride;
  p.x_scale = static_cast<const uint16_t*>(x_scale);
  p.w = static_cast<const uint8_t*>(w);
  p.w_scale = static_cast<const uint16_t*>(w_scale);
  p.out = static_cast<uint16_t*>(out);
  p.out_row_stride = out_row_stride;
  p.err = static_cast<int*>(workspace);
  p.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + fp8attn::kCtrlInts * 4);
  p.M = M;
  p.N = N;
  p.K = K;
  p.splits = fp8attn::fp8_gemm_splits(M, N, K, sms);
  const cudaError_t e = fp8attn::launch_fp8_block_gemm(p, sms, st);
  if (e == cudaErrorInvalidValue) return fail(FP8ATTN_EINVAL, "fp8 gemm: tensor map rejected");
  return e == cudaSuccess ? FP8ATTN_OK : cuda_fail(e, "fp8 gemm launch");
}

}  // namespace

extern "C" {

int64_t fp8attn_fp8_gemm_workspace_bytes(int64_t M, int N, int K) {
  if (M < 0 || N <= 0 || K <= 0) return -1;
  return fp8attn::fp8_gemm_workspace_bytes(M, N, K, device_sms());
}

int64_t fp8attn_fp8_linear_workspace_bytes(int64_t M, int N, int K) {
  if (M < 0 || N <= 0 || K <= 0) return -1;
  return round16(fp8attn_fp8_gemm_workspace_bytes(M, N, K)) + round16(M * K) +
         round16(M * (K / 128) * 2);
}

int fp8attn_fp8_dyn_quant(const void* x, int64_t x_row_stride, void* xq, int64_t xq_row_stride,
                          void* x_scale, int64_t M, int K, void* stream) {
  if (M < 0 || K <= 0 || K % 128 != 0)
    return fail(FP8ATTN_EINVAL, "fp8 quant needs M >= 0 and K a positive multiple of 128 "
                "(got M=%lld K=%d)", static_cast<long long>(M), K);
  return run_quant(x, x_row_stride, xq, xq_row_stride, x_scale, M, K,
                   static_cast<cudaStream_t>(stream));
}

int fp8attn_fp8_block_gemm(const void* xq, int64_t xq_row_stride, const void* x_scale,
                           const void* w, const void* w_scale, void* out, int64_t out_row_stride,
                           int64_t M, int N, int K, void* workspace, int64_t workspace_bytes,
                           void* stream) {
  const int rc = check_linear_sizes(M, N, K);
  if (rc) return rc;
  return run_gemm(xq, xq_row_stride, x_scale, w, w_scale, out, out_row_stride, M, N, K, workspace,
                  workspace_bytes, static_cast<cudaStream_t>(stream));
}

int fp8attn_fp8_block_linear(const void* x, int64_t x_row_stride, const void* w,
                             const void* w_scale, void* out, int64_t out_row_stride, int64_t M,
                             int N, int K, void* workspace, int64_t workspace_bytes,
                             void* stream) {
  int rc = check_linear_sizes(M, N, K);
  if (rc) return rc;
  if (M == 0) return FP8ATTN_OK;
  const int64_t need = fp8attn_fp8_linear_workspace_bytes(M, N, K);
  if (workspace == nullptr || workspace_bytes < need || !aligned(workspace, 16))
    return fail(FP8ATTN_EWORKSPACE, "fp8 linear: workspace of %lld bytes (16-byte aligned) "
                "needed, got %lld", static_cast<long long>(need),
                static_cast<long long>(workspace_bytes));
  const int64_t gemm_ws = round16(fp8attn_fp8_gemm_workspace_bytes(M, N, K));
  uint8_t* base = static_cast<uint8_t*>(workspace);
  uint8_t* xq = base + gemm_ws;
  uint8_t* xs = xq + round16(M * K);
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  rc = run_quant(x, x_row_stride, xq, K, xs, M, K, st);
  if (rc) return rc;
  return run_gemm(xq, K, xs, w, w_scale, out, out_row_stride, M, N, K, workspace, gemm_ws, st);
}

}  // extern "C"

// ---------------------------------------------------------------- row-parallel FP8 linear
namespace {
int64_t round256(int64_t v) { return (v + 255) & ~int64_t{255}; }

struct TpLayout {
  int64_t tiles_cap, flags_bytes, out_offset, recv_offset, total;
};
bool tp_layout(int64_t max_tokens, int N, int world, TpLayout* l) {
  if (max_tokens <= 0 || N <= 0 || N % 128 != 0 || world < 1 || world > fp8attn::kMaxTpRanks)
    return false;
  l->tiles_cap = (max_tokens + fp8attn::kFp8GemmTokens - 1) / fp8attn::kFp8GemmTokens * (N / 128);
  l->flags_bytes = round256(static_cast<int64_t>(world + 1) * l->tiles_cap * 8);
  l->out_offset = l->flags_bytes;
  l->recv_offset = l->out_offset + round256(max_tokens * N * 2);
  l->total = l->recv_offset + round256(static_cast<int64_t>(world) * max_tokens * N * 2);
  return true;
}
}  // namespace

extern "C" {

int64_t fp8attn_tp_linear_layout(int64_t max_tokens, int N, int world, int64_t* out_offset,
                                 int64_t* recv_offset) {
  TpLayout l;
  if (!tp_layout(max_tokens, N, world, &l)) return -1;
  if (out_offset) *out_offset = l.out_offset;
  if (recv_offset) *recv_offset = l.recv_offset;
  return l.total;
}

int64_t fp8attn_fp8_tp_linear_workspace_bytes(int64_t M, int K) {
  if (M < 0 || K <= 0 || K % 128 != 0) return -1;
  return round16(fp8attn::kCtrlInts * 4) + round16(M * K) + round16(M * (K / 128) * 2);
}

int fp8attn_fp8_tp_linear(const void* x, int64_t x_row_stride, const void* w, const void* w_scale,
                          void* const* buffers, int rank, int world, uint64_t epoch,
                          int64_t max_tokens, int64_t M, int N, int K, void* workspace,
                          int64_t workspace_bytes, void* stream) {
  int rc = check_linear_sizes(M, N, K);
  if (rc) return rc;
  TpLayout l;
  if (!tp_layout(max_tokens, N, world, &l))
    return fail(FP8ATTN_EINVAL, "tp linear: world must be 1..%d and max_tokens positive (got "
                "world=%d max_tokens=%lld)", fp8attn::kMaxTpRanks, world,
                static_cast<long long>(max_tokens));
  if (rank < 0 || rank >= world)
    return fail(FP8ATTN_EINVAL, "tp linear: rank %d outside 0..%d", rank, world - 1);
  if (M > max_tokens)
    return fail(FP8ATTN_EINVAL, "tp linear: M=%lld exceeds the buffers' max_tokens=%lld",
                static_cast<long long>(M), static_cast<long long>(max_tokens));
  if (epoch == 0) return fail(FP8ATTN_EINVAL, "tp linear: epoch must be >= 1");
  if (buffers == nullptr) return fail(FP8ATTN_EINVAL, "tp linear: null buffer table");
  for (int r = 0; r < world; ++r)
    if (buffers[r] == nullptr || !aligned(buffers[r], 256))
      return fail(FP8ATTN_EINVAL, "tp linear: buffer of rank %d is null or not 256-byte aligned",
                  r);
  if (M == 0) return FP8ATTN_OK;
  const int64_t need = fp8attn_fp8_tp_linear_workspace_bytes(M, K);
  if (workspace == nullptr || workspace_bytes < need || !aligned(workspace, 16))
    return fail(FP8ATTN_EWORKSPACE, "tp linear: workspace of %lld bytes (16-byte aligned) "
                "needed, got %lld", static_cast<long long>(need),
                static_cast<long long>(workspace_bytes));
  if (w == nullptr || w_scale == nullptr || !aligned(w, 16) || !aligned(w_scale, 2))
    return fail(FP8ATTN_EINVAL, "tp linear: w (16-byte aligned) and w_scale must be given");
  uint8_t* base = static_cast<uint8_t*>(workspace);
  uint8_t* xq = base + round16(fp8attn::kCtrlInts * 4);
  uint8_t* xs = xq + round16(M * K);
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  rc = run_quant(x, x_row_stride, xq, K, xs, M, K, st);
  if (rc) return rc;
  fp8attn::Fp8GemmParams p;
  p.xq = xq;
  p.xq_row_stride = K;
  p.x_scale = reinterpret_cast<const uint16_t*>(xs);
  p.w = static_cast<const uint8_t*>(w);
  p.w_scale = static_cast<const uint16_t*>(w_scale);
  p.out = nullptr;
  p.out_row_stride = N;
  p.err = static_cast<int*>(workspace);
  p.partials = nullptr;
  p.M = M;
  p.N = N;
  p.K = K;
  p.splits = 1;
  fp8attn::Fp8TpParams tp = {};
  for (int r = 0; r < world; ++r) {
    uint8_t* b = static_cast<uint8_t*>(buffers[r]);
    tp.flags[r] = reinterpret_cast<unsigned long long*>(b);
    tp.out[r] = reinterpret_cast<uint16_t*>(b + l.out_offset);
    tp.recv[r] = reinterpret_cast<uint16_t*>(b + l.recv_offset);
  }
  tp.epoch = epoch;
  tp.tiles_cap = l.tiles_cap;
  tp.rank = rank;
  tp.world = world;
  const cudaError_t e = fp8attn::launch_fp8_tp_gemm(p, tp, device_sms(), st);
  if (e == cudaErrorInvalidValue) return fail(FP8ATTN_EINVAL, "tp linear: tensor map rejected");
  return e == cudaSuccess ? FP8ATTN_OK : cuda_fail(e, "tp linear launch");
}

}  // extern "C"
