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

#ifndef STORE_UNITS
#define STORE_UNITS 2
#endif

namespace fp8attn {
namespace {

constexpr int kStoreThreads = 256;

// 16 bf16 (two 16-byte loads) of one unit; read-only, not kept in L1 (each byte is read once).
__device__ __forceinline__ void load_unit(const uint16_t* src, uint4& a, uint4& b) {
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(a.x), "=r"(a.y), "=r"(a.z), "=r"(a.w) : "l"(src));
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(b.x), "=r"(b.y), "=r"(b.z), "=r"(b.w) : "l"(src + 8));
}

// kU units per thread, unit u = blockIdx.x * kU * kStoreThreads + i * kStoreThreads + threadIdx.x
// (consecutive threads take consecutive units for every i, so every load and store of a warp is
// one contiguous run).  Every global load of the thread -- the slot of each unit and its row data
// -- is issued before any of them is used: the data address does not depend on the slot, so the
// slot load's latency is not paid in front of the data loads.
template <bool kVec, int kU>
__global__ void __launch_bounds__(kStoreThreads)
    store_kernel(const StoreParams p) {
  // launched as a programmatic dependent of the previous kernel on the stream (the producer of
  // key/value): the launch and the CTAs' start overlap its tail; nothing is read before it ends
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int kvh = p.num_kv_heads;
  const int chunks_per_row = kvh * 8;  // 16-element chunks per (token, K or V) row
  const int64_t units = p.num_tokens * 2 * chunks_per_row;
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kU * kStoreThreads + threadIdx.x;
  int64_t token[kU];
  int chunk[kU], is_v[kU];
  bool in_range[kU];
  int slot_raw[kU];
  uint4 wa[kU], wb[kU];
#pragma unroll
  for (int i = 0; i < kU; ++i) {
    const int64_t u = base + static_cast<int64_t>(i) * kStoreThreads;
    in_range[i] = u < units;
    const int64_t uu = in_range[i] ? u : 0;
    token[i] = uu / (2 * chunks_per_row);
    const int rem = static_cast<int>(uu - token[i] * 2 * chunks_per_row);
    is_v[i] = rem >= chunks_per_row;
    chunk[i] = rem - is_v[i] * chunks_per_row;  // 0 .. KVH*8-1
    slot_raw[i] = in_range[i] ? ldg_keep(p.slot_mapping + token[i]) : -1;
    const uint16_t* src = (is_v[i] ? p.value + token[i] * p.value_row_stride
                                   : p.key + token[i] * p.key_row_stride) + chunk[i] * 16;
    if (kVec) {
      if (in_range[i]) {
        load_unit(src, wa[i], wb[i]);
      } else {
        wa[i] = wb[i] = make_uint4(0, 0, 0, 0);
      }
    } else {
      uint32_t w[8];
#pragma unroll
      for (int k = 0; k < 8; ++k)
        w[k] = in_range[i] ? (static_cast<uint32_t>(__ldg(src + 2 * k)) |
                              (static_cast<uint32_t>(__ldg(src + 2 * k + 1)) << 16)) : 0u;
      wa[i] = make_uint4(w[0], w[1], w[2], w[3]);
      wb[i] = make_uint4(w[4], w[5], w[6], w[7]);
    }
  }
#pragma unroll
  for (int i = 0; i < kU; ++i) {
    const int64_t slot = slot_raw[i];
    const bool active = in_range[i] && slot >= 0 && slot < p.num_slots;
    const uint32_t w[8] = {wa[i].x, wa[i].y, wa[i].z, wa[i].w, wb[i].x, wb[i].y, wb[i].z, wb[i].w};
    float x[16];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      x[2 * k] = active ? __uint_as_float(w[k] << 16) : 0.f;
      x[2 * k + 1] = active ? __uint_as_float(w[k] & 0xFFFF0000u) : 0.f;
    }
    float scale = 1.0f;
    if (p.scaled) {
      // every lane stays in the shuffle: the 8 lanes of one (token, head) row are consecutive
      // and 8-aligned within the warp, for every i
      float amax = 0.f;
#pragma unroll
      for (int k = 0; k < 16; ++k) amax = fmaxf(amax, fabsf(x[k]));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
      scale = __fdiv_rn(amax, 448.0f);
      if (!(scale > 0.f)) scale = 1.0f;
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const float y = __fdiv_rn(x[k], scale);
        x[k] = fminf(fmaxf(y, -448.0f), 448.0f);
      }
    }
    if (!active) continue;
    uint32_t packed[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(
          make_float2(x[4 * k], x[4 * k + 1]), __NV_SATFINITE, __NV_E4M3);
      const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(
          make_float2(x[4 * k + 2], x[4 * k + 3]), __NV_SATFINITE, __NV_E4M3);
      packed[k] = static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
    }
    uint8_t* cache = is_v[i] ? p.v_cache : p.k_cache;
    uint8_t* dst = cache + slot * static_cast<int64_t>(kvh) * kHeadDim + chunk[i] * 16;
    *reinterpret_cast<uint4*>(dst) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    float* sc = is_v[i] ? p.v_scale : p.k_scale;
    if (sc != nullptr && (chunk[i] & 7) == 0) sc[slot * kvh + (chunk[i] >> 3)] = scale;
  }
}

}  // namespace

cudaError_t launch_store(const StoreParams& p, cudaStream_t stream) {
  if (p.num_tokens == 0) return cudaSuccess;
  const int64_t units = p.num_tokens * 2 * p.num_kv_heads * 8;
  const bool vec = (reinterpret_cast<uintptr_t>(p.key) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(p.value) % 16 == 0) &&
                   (p.key_row_stride % 8 == 0) && (p.value_row_stride % 8 == 0);
  constexpr int U = STORE_UNITS;
  const int64_t blocks = (units + U * kStoreThreads - 1) / (U * kStoreThreads);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(blocks));
  cfg.blockDim = dim3(kStoreThreads);
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (vec)
    return cudaLaunchKernelEx(&cfg, store_kernel<true, U>, p);
  return cudaLaunchKernelEx(&cfg, store_kernel<false, U>, p);
}

}  // namespace fp8attn
