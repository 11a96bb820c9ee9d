// Fused attention-input epilogue: per-head RMSNorm of q and k, rotary embedding of both, and the
// FP8 K/V store, in one pass over the QKV projection's output.
//
// Replaces the chain the reference runs between the QKV projection and the attention kernels
// (nanovllm/models/qwen3.py:102-111):
//   q = q_norm(q); k = k_norm(k)              RMSNorm.rms_forward   nanovllm/layers/layernorm.py:16-26
//   q, k = rotary_emb(positions, q, k)        RotaryEmbedding        nanovllm/layers/rotary_embedding.py:6-47
//   store_kvcache(k, v, k_cache, v_cache, slot_mapping)             nanovllm/layers/attention.py:11-40
// so K makes one HBM round trip instead of three (norm out, rope out, store in), and V one.
//
// Arithmetic, as the reference's compiled functions compute it (torch.compile, inductor):
//   RMSNorm: r = rsqrt(sum(x^2) / 128 + eps) in fp32, out = bf16((x * r) * w) -- one rounding (the
//            compiled function keeps x * r in fp32 before the weight multiply);
//   RoPE on the normalised bf16 values, fp32, cos/sin from the fp32 cos_sin cache row of the
//            token's position: y1 = x1 cos - x2 sin, y2 = x2 cos + x1 sin, each as one fused
//            multiply-add of its first product and the rounded second, then bf16;
//   store: the roped bf16 K (and the raw V) as e4m3, round to nearest even, finite overflow
//            saturating to +-448 (the store kernel's cast), or amax/448-scaled.
// The fp32 sum of squares follows the compiled reference's reduction order (4 elements per lane
// as a multiply and three fused multiply-adds, then a butterfly over the lanes from offset 16 down
// to 1): on seeded inputs of six shapes (q, k and cache bytes of 20M values) the outputs are
// identical to the reference's, bit for bit.
//
// Work: one warp task per token and group of up to 8 heads (rows of 128 values, 4 per lane; lane
// l holds elements 4l .. 4l + 3, whose rotary partners -- the other half of the head -- sit in
// lane l ^ 16), with all of the task's loads issued before the first is used.
#include "common.cuh"
#include "kernels.h"

namespace fp8attn {
namespace {

constexpr int kQkThreads = 256;

__device__ __forceinline__ float bf16_to_f32(uint32_t bits16) { return __uint_as_float(bits16 << 16); }

__device__ __forceinline__ uint32_t f32_to_bf16_bits(float x) {
  __nv_bfloat16 b = __float2bfloat16_rn(x);
  return static_cast<uint32_t>(*reinterpret_cast<uint16_t*>(&b));
}

__device__ __forceinline__ void widen4(uint2 raw, float (&x)[4]) {
  x[0] = bf16_to_f32(raw.x & 0xFFFFu);
  x[1] = bf16_to_f32(raw.x >> 16);
  x[2] = bf16_to_f32(raw.y & 0xFFFFu);
  x[3] = bf16_to_f32(raw.y >> 16);
}

__device__ __forceinline__ uint2 pack4(const float (&y)[4]) {
  return make_uint2(f32_to_bf16_bits(y[0]) | (f32_to_bf16_bits(y[1]) << 16),
                    f32_to_bf16_bits(y[2]) | (f32_to_bf16_bits(y[3]) << 16));
}

// One warp task: up to kRowsPerTask heads (rows of 128 values) of one token.  The token's
// position, slot and cos/sin row and the task's rows are all loaded before any is used.
template <int kRowsPerTask>
__global__ void __launch_bounds__(kQkThreads) qk_norm_rope_store_kernel(const QkNormParams p) {
  // launched as a programmatic dependent of the previous kernel (the QKV projection): nothing is
  // read before it ends
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int64_t task = (static_cast<int64_t>(blockIdx.x) * kQkThreads + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int heads = p.num_heads + 2 * p.num_kv_heads;
  const int tasks_per_token = (heads + kRowsPerTask - 1) / kRowsPerTask;
  if (task >= p.num_tokens * tasks_per_token) return;  // whole warps leave together
  const int64_t token = task / tasks_per_token;
  const int h0 = static_cast<int>(task - token * tasks_per_token) * kRowsPerTask;
  const int nrows = min(kRowsPerTask, heads - h0);
  int64_t pos = p.positions[token];
  const int64_t slot = p.slot_mapping[token];
  const uint16_t* src = p.qkv + token * p.qkv_row_stride + static_cast<int64_t>(h0) * kHeadDim + 4 * lane;
  uint2 raw[kRowsPerTask];
#pragma unroll
  for (int i = 0; i < kRowsPerTask; ++i)
    raw[i] = i < nrows ? *reinterpret_cast<const uint2*>(src + i * kHeadDim) : make_uint2(0, 0);
  const bool any_qk = h0 < p.num_heads + p.num_kv_heads;
  float c[4] = {0.f, 0.f, 0.f, 0.f}, s[4] = {0.f, 0.f, 0.f, 0.f};
  float wq[4] = {0.f, 0.f, 0.f, 0.f}, wk[4] = {0.f, 0.f, 0.f, 0.f};
  if (any_qk) {
    pos = pos < 0 ? 0 : (pos >= p.max_position ? p.max_position - 1 : pos);  // stay in the table
    const float* cs = p.cos_sin + pos * kHeadDim + 4 * (lane & 15);
    const float4 c4 = *reinterpret_cast<const float4*>(cs);
    const float4 s4 = *reinterpret_cast<const float4*>(cs + kHeadDim / 2);
    c[0] = c4.x; c[1] = c4.y; c[2] = c4.z; c[3] = c4.w;
    s[0] = s4.x; s[1] = s4.y; s[2] = s4.z; s[3] = s4.w;
    widen4(*reinterpret_cast<const uint2*>(p.q_weight + 4 * lane), wq);
    widen4(*reinterpret_cast<const uint2*>(p.k_weight + 4 * lane), wk);
  }
  const bool store_ok = slot >= 0 && slot < p.num_slots;
  const int kvh = p.num_kv_heads;
#pragma unroll
  for (int i = 0; i < kRowsPerTask; ++i) {
    if (i >= nrows) break;
    const int h = h0 + i;
    const bool is_q = h < p.num_heads;
    const bool is_k = !is_q && h < p.num_heads + kvh;
    float x[4], y[4];
    widen4(raw[i], x);
    if (is_q || is_k) {
      // ---- RMSNorm over the head's 128 values.  Per lane: x0^2, then three fused multiply-adds;
      // across lanes: butterfly from offset 16 down to 1 -- the order of the compiled
      // reference's reduction (its output matches this kernel's bit for bit on seeded inputs)
      float ss = x[0] * x[0];
      ss = fmaf(x[1], x[1], ss);
      ss = fmaf(x[2], x[2], ss);
      ss = fmaf(x[3], x[3], ss);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
      const float r = rsqrtf(ss / 128.0f + p.eps);
      float n[4];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        n[k] = bf16_to_f32(f32_to_bf16_bits((x[k] * r) * (is_q ? wq[k] : wk[k])));
      // ---- rotary embedding: this lane's 4 values and their partners in the other half
      const bool first_half = lane < 16;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float other = __shfl_xor_sync(0xffffffffu, n[k], 16);
        // first half (x1 = n, x2 = other): x1 cos - x2 sin; second half (x2 = n, x1 = other):
        // x2 cos + x1 sin -- each a fused multiply-add of the first product and the rounded
        // second
        y[k] = first_half ? fmaf(n[k], c[k], -__fmul_rn(other, s[k]))
                          : fmaf(n[k], c[k], __fmul_rn(other, s[k]));
        y[k] = bf16_to_f32(f32_to_bf16_bits(y[k]));
      }
      if (is_q) {
        *reinterpret_cast<uint2*>(p.q_out + (token * p.num_heads + h) * kHeadDim + 4 * lane) = pack4(y);
        continue;
      }
      if (p.k_out != nullptr)
        *reinterpret_cast<uint2*>(p.k_out + (token * kvh + (h - p.num_heads)) * kHeadDim + 4 * lane) =
            pack4(y);
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k) y[k] = x[k];
    }
    // ---- K (rotated) or V (raw) row into the paged e4m3 cache
    const int head = h - p.num_heads - (is_k ? 0 : kvh);
    float scale = 1.0f;
    if (p.scaled) {
      float amax = fmaxf(fmaxf(fabsf(y[0]), fabsf(y[1])), fmaxf(fabsf(y[2]), fabsf(y[3])));
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
      scale = __fdiv_rn(amax, 448.0f);
      if (!(scale > 0.f)) scale = 1.0f;
#pragma unroll
      for (int k = 0; k < 4; ++k) y[k] = fminf(fmaxf(__fdiv_rn(y[k], scale), -448.0f), 448.0f);
    }
    if (!store_ok) continue;
    const uint32_t lo = static_cast<uint32_t>(
        __nv_cvt_float2_to_fp8x2(make_float2(y[0], y[1]), __NV_SATFINITE, __NV_E4M3));
    const uint32_t hi = static_cast<uint32_t>(
        __nv_cvt_float2_to_fp8x2(make_float2(y[2], y[3]), __NV_SATFINITE, __NV_E4M3));
    uint8_t* cache = is_k ? p.k_cache : p.v_cache;
    *reinterpret_cast<uint32_t*>(cache + (slot * kvh + head) * kHeadDim + 4 * lane) = lo | (hi << 16);
    float* sc = is_k ? p.k_scale : p.v_scale;
    if (sc != nullptr && lane == 0) sc[slot * kvh + head] = scale;
  }
}

}  // namespace

cudaError_t launch_qk_norm_rope_store(const QkNormParams& p, cudaStream_t stream) {
  if (p.num_tokens == 0) return cudaSuccess;
  // 8 heads per task for large batches (measured 42.5 us for 5,561 tokens of 32 + 2 x 8 heads,
  // against 50.2 with 4 and 57.3 with 16); 4 for small ones, whose tasks would not fill the GPU
  // (256 tokens: 4.6 us against 5.6 with 8)
  const int heads = p.num_heads + 2 * p.num_kv_heads;
  const bool small = p.num_tokens <= 1024;
  const int rows = small ? 4 : 8;
  const int64_t tasks = p.num_tokens * ((heads + rows - 1) / rows);
  const int64_t blocks = (tasks * 32 + kQkThreads - 1) / kQkThreads;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(blocks));
  cfg.blockDim = dim3(kQkThreads);
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (small) return cudaLaunchKernelEx(&cfg, qk_norm_rope_store_kernel<4>, p);
  return cudaLaunchKernelEx(&cfg, qk_norm_rope_store_kernel<8>, p);
}

}  // namespace fp8attn
