// Shared device helpers for the FP8 PagedAttention kernels (sm_100a).
//
// Everything here is a thin wrapper over one PTX instruction (mbarrier, TMA, cp.async,
// conversions, packed f32x2 arithmetic) or a small numeric helper.  Every wait on an mbarrier is
// bounded by wall-clock time (%globaltimer): when the bound is hit the waiter records an error
// code in a global flag and gives up, so a logic error cannot hang the GPU.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

namespace fp8attn {

constexpr int kHeadDim = 128;
// Wall-clock bound for any single mbarrier wait (ns): a healthy wait is < 100 us.
constexpr unsigned long long kWaitLimitNs = 1000000000ull;  // 1 s

// Error codes written into the control block's error word by device code.
enum DeviceError : int {
  kDevErrNone = 0,
  kDevErrWaitTimeout = 1,
  kDevErrBadBlock = 2,
  kDevErrTmemAlloc = 3,
  kDevErrWorkspace = 4,
};

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
          smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity to complete.  Returns false (and records
// kDevErrWaitTimeout in *err) when more than limit_ns of wall-clock time pass.  The clock is read
// only every 1024 polls: reading %globaltimer is slow, and a wait that completes must not pay
// for it.
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, int* err,
                                              unsigned long long limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  unsigned long long t0 = 0;
  for (uint32_t polls = 1;; ++polls) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((polls & 1023u) == 0) {
      const unsigned long long now = globaltimer_ns();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > limit_ns) {
        if (err) atomicExch(err, kDevErrWaitTimeout);
        return false;
      }
    }
  }
}

// The library's waits: bounded by kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  return mbar_wait_for(bar, parity, err, kWaitLimitNs);
}

// End of a persistent launch that claimed work from the control block (ctrl[1] = next work item,
// ctrl[2] = CTAs finished): the last CTA to finish returns both counters to zero, so the next
// launch on the same workspace starts from a clean state.  Called by one thread per CTA, after
// every thread of the CTA is done with the counters.
__device__ __forceinline__ void release_work_counters(int* ctrl) {
  __threadfence();
  const int done = atomicAdd(ctrl + 2, 1);
  if (done == static_cast<int>(gridDim.x) - 1) {
    atomicExch(ctrl + 1, 0);
    atomicExch(ctrl + 2, 0);
  }
}

// ---------------------------------------------------------------------------------------------
// TMA (no multicast anywhere in this library)
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Order this thread's generic-proxy shared-memory writes before later async-proxy reads
// (tensor-core operand fetches).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Two e4m3 bytes (low byte -> low half) to f16x2; exact.
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t two_bytes) {
  __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(two_bytes & 0xFFFFu),
                                             __NV_E4M3);
  return static_cast<uint32_t>(h.x) | (static_cast<uint32_t>(h.y) << 16);
}

// f16x2 -> two e4m3 bytes (low half -> low byte), round to nearest even, saturating.
__device__ __forceinline__ uint32_t f16x2_to_e4m3x2(uint32_t h) {
  __half2_raw r;
  r.x = static_cast<unsigned short>(h & 0xFFFFu);
  r.y = static_cast<unsigned short>(h >> 16);
  return static_cast<uint32_t>(__nv_cvt_halfraw2_to_fp8x2(r, __NV_SATFINITE, __NV_E4M3));
}

// Two floats -> two e4m3 bytes (a -> low byte), round to nearest even, saturating.
__device__ __forceinline__ uint32_t f32x2_to_e4m3x2(float a, float b) {
  return static_cast<uint32_t>(
      __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3));
}

// x (f16x2) ~= hi + lo with hi, lo e4m3 pairs: hi = e4m3(x), lo = e4m3(x - hi).  The pair carries
// about 8 significant bits (the residual is at most 2^-4 of x).
__device__ __forceinline__ void split_f16x2_e4m3(uint32_t x, uint32_t& hi, uint32_t& lo) {
  hi = f16x2_to_e4m3x2(x);
  const uint32_t back = e4m3x2_to_f16x2(hi);
  const __half2 r = __hsub2(*reinterpret_cast<const __half2*>(&x),
                            *reinterpret_cast<const __half2*>(&back));
  lo = f16x2_to_e4m3x2(*reinterpret_cast<const uint32_t*>(&r));
}

// Value of a non-negative e4m3 byte (bits 0-6 of b; the sign bit must be clear) as fp32, with
// integer and one multiply instead of a conversion: the 7 exponent+mantissa bits placed at
// fp32 bits 20-26 read as 2^(e-127)(1 + m/8) (or m 2^-130 for e = 0), and 2^120 rebiases that
// to e4m3's 2^(e-7)(1 + m/8) (m 2^-9): exact for normals and subnormals (mul.rn, no flush).
__device__ __forceinline__ float e4m3_pos_to_f32(uint32_t b) {
  float y;
  asm("mul.rn.f32 %0, %1, 0f7B800000;" : "=f"(y) : "f"(__uint_as_float((b & 0x7Fu) << 20)));
  return y;
}

// Two non-negative floats -> e4m3 hi and lo pairs (a -> low bytes) with a ~= hi + lo: hi =
// e4m3(a), lo = e4m3(a - hi), about 8 significant bits; two conversions per pair.
__device__ __forceinline__ void split_pos_f32x2_e4m3(float a, float b, uint32_t& hi, uint32_t& lo) {
  hi = f32x2_to_e4m3x2(a, b);
  lo = f32x2_to_e4m3x2(a - e4m3_pos_to_f32(hi), b - e4m3_pos_to_f32(hi >> 8));
}

// (lo, hi) floats -> f16x2 with lo in the low half; round to nearest even.
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float lg2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ---- packed fp32 pairs (sm_100 f32x2 arithmetic: one instruction for two lanes of work)
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// 2^x for two values on the FMA pipe instead of the MUFU unit (whose ex2 rate bounds the
// attention softmax): relative error < 1e-4 for x >= -125 (smaller x gives ~2^-125).  x = n + f
// with n = round(x) from the 1.5 * 2^23 shifter (round to nearest), 2^f on [-0.5, 0.5] by a
// degree-3 polynomial fitted here for relative error, and n added into the exponent field.
__device__ __forceinline__ void exp2_poly_x2(float x0, float x1, float& r0, float& r1) {
  const uint64_t x = f2_pack(fmaxf(x0, -125.f), fmaxf(x1, -125.f));
  const uint64_t shifter = f2_pack(12582912.f, 12582912.f);
  const uint64_t t = f2_add(x, shifter);
  const uint64_t f = f2_sub(x, f2_sub(t, shifter));
  uint64_t p = f2_fma(f, f2_pack(0.05517098f, 0.05517098f), f2_pack(0.24260971f, 0.24260971f));
  p = f2_fma(p, f, f2_pack(0.69326097f, 0.69326097f));
  p = f2_fma(p, f, f2_pack(0.99992818f, 0.99992818f));
  float p0, p1, t0, t1;
  f2_unpack(p, p0, p1);
  f2_unpack(t, t0, t1);
  r0 = __uint_as_float(__float_as_uint(p0) + (__float_as_uint(t0) << 23));
  r1 = __uint_as_float(__float_as_uint(p1) + (__float_as_uint(t1) << 23));
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// fp32 -> fp16 -> bf16, the reference output path (.to(tl.float16) stored into bf16).
__device__ __forceinline__ __nv_bfloat16 out_round(float x) {
  return __float2bfloat16_rn(__half2float(__float2half_rn(x)));
}

// Read-only global loads that stay where they are written: the compiler may not sink them to
// their first use, so a load issued early (a prefetch) really overlaps with the work after it.
__device__ __forceinline__ int ldg_keep(const int* p) {
  int v;
  asm volatile("ld.global.nc.s32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ uint4 ldg_keep_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// 16-byte global -> shared copy that bypasses registers (zero-filled when !pred); completion
// per thread with cp_async_commit / cp_async_wait<n>.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool pred) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(pred ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

}  // namespace fp8attn
