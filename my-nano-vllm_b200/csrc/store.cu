// KV store / quantise kernel: scatter new bf16 K/V rows through slot_mapping into the paged
// e4m3 caches (and their optional per-(slot, kv-head) fp32 scales).
//
// Replaces store_kvcache_kernel (nanovllm/layers/attention.py:11-31).  Same contract: row i of
// key/value goes to cache row slot_mapping[i] (a cache row is KVH*128 e4m3 bytes), rows with
// slot -1 are skipped.  The cast is round-to-nearest-even with finite overflow saturating to
// +-448 (the hardware conversion the reference's Triton store lowers to on the GPU).
//
// Layout of the work: a unit is 16 consecutive elements (two 16-byte bf16 loads, one 16-byte
// e4m3 store).  Eight consecutive units cover one (token, kv head) row of 128, so the scaled
// mode's amax is a 3-step shuffle, and a warp's 32 units cover 4 heads of one token's K or V
// row: both the loads and the stores of a warp are contiguous 512-byte / 256-byte runs.  Each
// thread takes kUnits units a whole grid apart and issues all their loads before converting any,
// so one wave keeps every byte of a typical batch in flight.
#include "common.cuh"
#include "kernels.h"

namespace fp8attn {
namespace {

constexpr int kStoreThreads = 256;
constexpr int kUnits = 4;

struct Unit {
  const uint16_t* src;
  uint8_t* dst;
  float* scale_dst;  // scale of the unit's (slot, head) row, written by the row's first unit
  bool in_range, active;
};

__device__ __forceinline__ Unit unit_at(const StoreParams& p, int64_t u) {
  const int kvh = p.num_kv_heads;
  const int chunks_per_row = kvh * 8;  // 16-element chunks per (token, K or V) row
  const int64_t units = p.num_tokens * 2 * chunks_per_row;
  Unit t;
  t.in_range = u < units;
  const int64_t uu = t.in_range ? u : 0;
  const int64_t token = uu / (2 * chunks_per_row);
  const int rem = static_cast<int>(uu - token * 2 * chunks_per_row);
  const int is_v = rem >= chunks_per_row;
  const int chunk = rem - is_v * chunks_per_row;  // 0 .. KVH*8-1
  const int64_t slot = t.in_range ? static_cast<int64_t>(__ldg(p.slot_mapping + token)) : -1;
  t.active = t.in_range && slot >= 0 && slot < p.num_slots;
  t.src = (is_v ? p.value + token * p.value_row_stride : p.key + token * p.key_row_stride) + chunk * 16;
  t.dst = (is_v ? p.v_cache : p.k_cache) + slot * static_cast<int64_t>(kvh) * kHeadDim + chunk * 16;
  float* sc = is_v ? p.v_scale : p.k_scale;
  t.scale_dst = (sc != nullptr && (chunk & 7) == 0) ? sc + slot * kvh + (chunk >> 3) : nullptr;
  return t;
}

template <bool kVec>
__global__ void __launch_bounds__(kStoreThreads)
    store_kernel(const StoreParams p) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kStoreThreads;
  const int64_t u0 = static_cast<int64_t>(blockIdx.x) * kStoreThreads + threadIdx.x;
  Unit t[kUnits];
  uint32_t w[kUnits][8];  // raw bf16 pairs, all loads in flight before any conversion
#pragma unroll
  for (int k = 0; k < kUnits; ++k) {
    t[k] = unit_at(p, u0 + k * stride);
    if (t[k].active) {
      if (kVec) {
        const uint4 a = __ldg(reinterpret_cast<const uint4*>(t[k].src));
        const uint4 b = __ldg(reinterpret_cast<const uint4*>(t[k].src) + 1);
        w[k][0] = a.x; w[k][1] = a.y; w[k][2] = a.z; w[k][3] = a.w;
        w[k][4] = b.x; w[k][5] = b.y; w[k][6] = b.z; w[k][7] = b.w;
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i)
          w[k][i] = static_cast<uint32_t>(__ldg(t[k].src + 2 * i)) |
                    (static_cast<uint32_t>(__ldg(t[k].src + 2 * i + 1)) << 16);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) w[k][i] = 0u;
    }
  }
#pragma unroll
  for (int k = 0; k < kUnits; ++k) {
    float x[16];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      x[2 * i] = __uint_as_float(w[k][i] << 16);
      x[2 * i + 1] = __uint_as_float(w[k][i] & 0xFFFF0000u);
    }
    float scale = 1.0f;
    if (p.scaled) {  // every lane of the warp takes part in the shuffles
      float amax = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(x[i]));
      // the 8 lanes of one (token, head) row are consecutive and 8-aligned within the warp
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
      scale = __fdiv_rn(amax, 448.0f);
      if (!(scale > 0.f)) scale = 1.0f;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float y = __fdiv_rn(x[i], scale);
        x[i] = fminf(fmaxf(y, -448.0f), 448.0f);
      }
    }
    if (!t[k].active) continue;
    uint32_t packed[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __nv_fp8x2_storage_t lo =
          __nv_cvt_float2_to_fp8x2(make_float2(x[4 * i], x[4 * i + 1]), __NV_SATFINITE, __NV_E4M3);
      const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(
          make_float2(x[4 * i + 2], x[4 * i + 3]), __NV_SATFINITE, __NV_E4M3);
      packed[i] = static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
    }
    *reinterpret_cast<uint4*>(t[k].dst) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    if (t[k].scale_dst != nullptr) *t[k].scale_dst = scale;
  }
}

}  // namespace

cudaError_t launch_store(const StoreParams& p, cudaStream_t stream) {
  if (p.num_tokens == 0) return cudaSuccess;
  const int64_t units = p.num_tokens * 2 * p.num_kv_heads * 8;
  const int64_t blocks = (units + kStoreThreads * kUnits - 1) / (kStoreThreads * kUnits);
  const bool vec = (reinterpret_cast<uintptr_t>(p.key) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(p.value) % 16 == 0) &&
                   (p.key_row_stride % 8 == 0) && (p.value_row_stride % 8 == 0);
  if (vec)
    store_kernel<true><<<static_cast<unsigned>(blocks), kStoreThreads, 0, stream>>>(p);
  else
    store_kernel<false><<<static_cast<unsigned>(blocks), kStoreThreads, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace fp8attn
