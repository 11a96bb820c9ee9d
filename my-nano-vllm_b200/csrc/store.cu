// KV store / quantise kernel: scatter new bf16 K/V rows through slot_mapping into the paged
// e4m3 caches (and their optional per-(slot, kv-head) fp32 scales).
//
// Replaces store_kvcache_kernel (nanovllm/layers/attention.py:11-31).  Same contract: row i of
// key/value goes to cache row slot_mapping[i] (a cache row is KVH*128 e4m3 bytes), rows with
// slot -1 are skipped.  The cast is round-to-nearest-even with finite overflow saturating to
// +-448 (the hardware conversion the reference's Triton store lowers to on the GPU).
//
// Layout of the work: one thread converts 16 consecutive elements (two 16-byte bf16 loads, one
// 16-byte e4m3 store).  Eight consecutive threads cover one (token, kv head) row of 128, so the
// scaled mode's amax is a 3-step shuffle.  A warp covers 4 heads of one token's K or V row, so
// both the loads and the stores of a warp are contiguous 512-byte / 256-byte runs.
#include "common.cuh"
#include "kernels.h"

namespace fp8attn {
namespace {

constexpr int kStoreThreads = 256;

template <bool kVec>
__global__ void __launch_bounds__(kStoreThreads)
    store_kernel(const StoreParams p) {
  const int kvh = p.num_kv_heads;
  const int chunks_per_row = kvh * 8;  // 16-element chunks per (token, K or V) row
  const int64_t units = p.num_tokens * 2 * chunks_per_row;
  const int64_t u = static_cast<int64_t>(blockIdx.x) * kStoreThreads + threadIdx.x;
  // every lane of a warp stays in the shuffle below; out-of-range lanes just do no memory work
  const bool in_range = u < units;
  const int64_t uu = in_range ? u : 0;
  const int64_t token = uu / (2 * chunks_per_row);
  const int rem = static_cast<int>(uu - token * 2 * chunks_per_row);
  const int is_v = rem >= chunks_per_row;
  const int chunk = rem - is_v * chunks_per_row;  // 0 .. KVH*8-1
  const int head = chunk >> 3;

  int64_t slot = in_range ? static_cast<int64_t>(__ldg(p.slot_mapping + token)) : -1;
  const bool active = in_range && slot >= 0 && slot < p.num_slots;

  const uint16_t* src = is_v ? p.value + token * p.value_row_stride
                             : p.key + token * p.key_row_stride;
  src += chunk * 16;
  float x[16];
  if (active) {
    if (kVec) {
      const uint4 a = __ldg(reinterpret_cast<const uint4*>(src));
      const uint4 b = __ldg(reinterpret_cast<const uint4*>(src) + 1);
      const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        x[2 * i] = __uint_as_float(w[i] << 16);
        x[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) x[i] = __uint_as_float(static_cast<uint32_t>(__ldg(src + i)) << 16);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) x[i] = 0.f;
  }

  float scale = 1.0f;
  if (p.scaled) {
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
  if (!active) return;

  uint32_t packed[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_fp8x2_storage_t lo =
        __nv_cvt_float2_to_fp8x2(make_float2(x[4 * i], x[4 * i + 1]), __NV_SATFINITE, __NV_E4M3);
    const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(
        make_float2(x[4 * i + 2], x[4 * i + 3]), __NV_SATFINITE, __NV_E4M3);
    packed[i] = static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
  }
  uint8_t* cache = is_v ? p.v_cache : p.k_cache;
  uint8_t* dst = cache + slot * static_cast<int64_t>(kvh) * kHeadDim + chunk * 16;
  *reinterpret_cast<uint4*>(dst) = make_uint4(packed[0], packed[1], packed[2], packed[3]);

  float* sc = is_v ? p.v_scale : p.k_scale;
  if (sc != nullptr && (chunk & 7) == 0) sc[slot * kvh + head] = scale;
}

}  // namespace

cudaError_t launch_store(const StoreParams& p, cudaStream_t stream) {
  if (p.num_tokens == 0) return cudaSuccess;
  const int64_t units = p.num_tokens * 2 * p.num_kv_heads * 8;
  const int64_t blocks = (units + kStoreThreads - 1) / kStoreThreads;
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
