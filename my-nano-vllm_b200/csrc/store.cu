// KV store / quantise kernel: scatter new bf16 K/V rows through slot_mapping into the paged
// e4m3 caches (and their optional per-(slot, kv-head) fp32 scales).
//
// Replaces store_kvcache_kernel (nanovllm/layers/attention.py:11-31).  Same contract: row i of
// key/value goes to cache row slot_mapping[i] (a cache row is KVH*128 e4m3 bytes), rows with
// slot -1 are skipped.  The cast is round-to-nearest-even with finite overflow saturating to
// +-448 (the hardware conversion the reference's Triton store lowers to on the GPU).
//
// Layout of the work: one thread converts 8 consecutive elements of a token's K row and the same 8
// of its V row (one 16-byte bf16 load each, one 8-byte e4m3 store each) and loads the token's
// slot once for both.  Sixteen consecutive threads cover one (token, kv head) row of 128, so the
// scaled mode's amax is a 4-step shuffle, and a warp's loads and stores are contiguous 512-byte /
// 256-byte runs.  This is the reference Triton kernel's granularity (8 elements per thread of a
// 4-warp program per token); larger units per thread measured slower on B200 (fewer loads in
// flight per SM for the same residency).
#include "common.cuh"
#include "kernels.h"

namespace fp8attn {
namespace {

constexpr int kStoreThreads = 256;

// 8 bf16 (one 16-byte load); read-only, not kept in L1 (each byte is read once).
__device__ __forceinline__ uint4 load8(const uint16_t* src) {
  uint4 a;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(a.x), "=r"(a.y), "=r"(a.z), "=r"(a.w) : "l"(src));
  return a;
}

// Thread t: token t / (KVH * 16), 8-element chunk c = t % (KVH * 16) of both its K and its V row.
// The slot load and both row loads are issued before any is used (the row addresses do not
// depend on the slot).
template <bool kVec>
__global__ void __launch_bounds__(kStoreThreads)
    store_kernel(const StoreParams p) {
  // launched as a programmatic dependent of the previous kernel on the stream (the producer of
  // key/value): the launch and the CTAs' start overlap its tail; nothing is read before it ends
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int kvh = p.num_kv_heads;
  const int per_tok = kvh * 16;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * kStoreThreads + threadIdx.x;
  const bool in_range = t < p.num_tokens * per_tok;
  const int64_t token = in_range ? t / per_tok : 0;
  const int c = static_cast<int>(t - token * per_tok);
  const int slot_raw = in_range ? ldg_keep(p.slot_mapping + token) : -1;
  const uint16_t* ks = p.key + token * p.key_row_stride + c * 8;
  const uint16_t* vs = p.value + token * p.value_row_stride + c * 8;
  uint4 a = make_uint4(0, 0, 0, 0), b = make_uint4(0, 0, 0, 0);
  if (in_range) {
    if (kVec) {
      a = load8(ks);
      b = load8(vs);
    } else {
      uint32_t w[8];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        w[k] = static_cast<uint32_t>(__ldg(ks + 2 * k)) |
               (static_cast<uint32_t>(__ldg(ks + 2 * k + 1)) << 16);
        w[4 + k] = static_cast<uint32_t>(__ldg(vs + 2 * k)) |
                   (static_cast<uint32_t>(__ldg(vs + 2 * k + 1)) << 16);
      }
      a = make_uint4(w[0], w[1], w[2], w[3]);
      b = make_uint4(w[4], w[5], w[6], w[7]);
    }
  }
  const int64_t slot = slot_raw;
  const bool active = in_range && slot >= 0 && slot < p.num_slots;
#pragma unroll
  for (int kv = 0; kv < 2; ++kv) {
    const uint4 u = kv ? b : a;
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
    float x[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      x[2 * k] = active ? __uint_as_float(w[k] << 16) : 0.f;
      x[2 * k + 1] = active ? __uint_as_float(w[k] & 0xFFFF0000u) : 0.f;
    }
    float scale = 1.0f;
    if (p.scaled) {
      // every lane stays in the shuffle: the 16 lanes of one (token, head) row are consecutive
      // and 16-aligned within the warp
      float amax = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) amax = fmaxf(amax, fabsf(x[k]));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 8));
      scale = __fdiv_rn(amax, 448.0f);
      if (!(scale > 0.f)) scale = 1.0f;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float y = __fdiv_rn(x[k], scale);
        x[k] = fminf(fmaxf(y, -448.0f), 448.0f);
      }
    }
    if (!active) continue;
    uint32_t packed[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(
          make_float2(x[4 * k], x[4 * k + 1]), __NV_SATFINITE, __NV_E4M3);
      const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(
          make_float2(x[4 * k + 2], x[4 * k + 3]), __NV_SATFINITE, __NV_E4M3);
      packed[k] = static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
    }
    uint8_t* cache = kv ? p.v_cache : p.k_cache;
    *reinterpret_cast<uint2*>(cache + slot * static_cast<int64_t>(kvh) * kHeadDim + c * 8) =
        make_uint2(packed[0], packed[1]);
    float* sc = kv ? p.v_scale : p.k_scale;
    if (sc != nullptr && (c & 15) == 0) sc[slot * kvh + (c >> 4)] = scale;
  }
}

}  // namespace

cudaError_t launch_store(const StoreParams& p, cudaStream_t stream) {
  if (p.num_tokens == 0) return cudaSuccess;
  const int64_t threads = p.num_tokens * p.num_kv_heads * 16;
  const bool vec = (reinterpret_cast<uintptr_t>(p.key) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(p.value) % 16 == 0) &&
                   (p.key_row_stride % 8 == 0) && (p.value_row_stride % 8 == 0);
  const int64_t blocks = (threads + kStoreThreads - 1) / kStoreThreads;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(blocks));
  cfg.blockDim = dim3(kStoreThreads);
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (vec) return cudaLaunchKernelEx(&cfg, store_kernel<true>, p);
  return cudaLaunchKernelEx(&cfg, store_kernel<false>, p);
}

}  // namespace fp8attn
