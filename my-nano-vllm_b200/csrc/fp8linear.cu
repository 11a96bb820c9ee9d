// FP8 block-scaled linear layer on the sm_100a tensor cores: y = x . w^T with e4m3 weights in
// 128 x 128 blocks (one bf16 scale each) and activations quantised per token and 128-column group.
//
// Replaces fp8_block_linear (nanovllm/kernels/fp8_linear.py:93-139) and its two Triton kernels:
//   fp8_dyn_quant_kernel (:11-31): per (token, 128-column group) scale = amax / 448 (1 for an
//     all-zero group), xq = e4m3(clamp(x / scale, +-448)), the scale stored as bf16 (bytes equal
//     to the reference's on the GPU: the same approximate fp32 division);
//   fp8_block_gemm_kernel (:34-71): per 128-column block kb, the fp32 dot of the block times
//     (x_scale[m, kb] * w_scale[n / 128, kb]) accumulated in fp32, the sum rounded once to the
//     output dtype.
//
// The GEMM is computed transposed (out^T = w . xq^T), so that the weight rows fill the MMA's 128
// rows and the tokens are its N.  A work unit is one 128-row block of output features x 128
// tokens x a range of K blocks (split-K, so that thin decode GEMMs still occupy every SM; the
// ranges' fp32 partial sums are added by a second kernel in split order).  The grid is persistent:
// one CTA per SM walks units u = blockIdx.x, + gridDim.x, ..., and its pipelines run on across
// unit boundaries.  Warps:
//   warp 8   producer: per K block, TMA loads of the weight tile (128 rows x 128 bytes) and the
//            token tile (128 rows x 128 bytes; 128B swizzle, rows past M read as zeros) into a
//            5-stage ring;
//   warp 10  scales: per K block, x_scale[m, kb] * w_scale[nb, kb] in fp32 for the unit's 128
//            tokens into the stage's slot, the loads of 4 blocks in flight together (they are
//            strided 2-byte reads, off the producer's path);
//   warps 9, 11  MMA issuers (one thread each, alternate K blocks): D = xq_kb . w_kb^T (tokens are the MMA's 128 rows, the
//            128 features its N), four kind::f8f6f4 products of K = 32 into one of four
//            128-column tensor-memory buffers (all 512 columns), so the tensor cores run up to
//            four blocks ahead of the promotion;
//   warps 0-7  promotion: warp w reads tensor-memory lanes 32 (w % 4) .. + 31 (tokens) and
//            columns 64 (w / 4) .. + 63 (features) of D, so a thread owns 64 consecutive outputs
//            of one token row and one scale product per K block, and accumulates
//            acc += D * scale product in fp32 registers (packed fp32x2 fused multiply-adds),
//            block by block in K order (the reference's per-block scaling, which the tensor cores
//            cannot apply: the scales are arbitrary fp32, not powers of two); at a unit's end it
//            writes its 64 bf16 outputs as 16-byte stores, or, with split-K, its range's fp32
//            partial sums through a shared-memory stage that the 256 threads copy out as whole
//            rows.
// The row-parallel form (kTP) sends each bf16 tile through the same stage to the rank that owns
// it and adds the ranks' tiles there (tp_reduce_gather).
#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace fp8attn {
namespace {

constexpr int kBlk = 128;                 // K block (bytes of e4m3) and weight rows per unit
constexpr int kTok = kFp8GemmTokens;      // tokens per unit (the MMA's N)
constexpr int kGemmStages = 5;
constexpr int kDBufs = 4;                 // D buffers of kTok columns: all 512 of tensor memory
constexpr int kPromoWarps = 8;            // warps 0-7
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kScaleWarp = 10;
constexpr int kMmaWarp2 = 11;             // second MMA issuer: odd K-block positions
constexpr int kGemmThreads = 12 * 32;
constexpr int kScaleBatch = 4;            // K blocks whose scale loads are in flight together

// ------------------------------------------------------------------ dynamic quantisation
// a / b as the reference computes it: Triton's `/` on fp32 tensors is the full-range approximate
// division (div.full.f32), not the IEEE one.  With it the quantised bytes equal the reference's;
// with IEEE division about 0.1 % of them differed by one step (quotients that are exact e4m3
// rounding midpoints, e.g. 0.816406 / 0.00537109 = 152 between 144 and 160, are common with bf16
// inputs and scales).
__device__ __forceinline__ float div_like_reference(float a, float b) {
  float y;
  asm("div.full.f32 %0, %1, %2;" : "=f"(y) : "f"(a), "f"(b));
  return y;
}

// One warp per (token, 128-column group): lane l takes columns 4l .. 4l + 3.
__global__ void __launch_bounds__(256) fp8_dyn_quant_kernel(const Fp8QuantParams p) {
  const int64_t groups = p.M * (p.K / kBlk);
  const int64_t w = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= groups) return;  // uniform per warp
  const int kc = p.K / kBlk;
  const int64_t m = w / kc;
  const int g = static_cast<int>(w - m * kc);
  const uint2 raw = *reinterpret_cast<const uint2*>(p.x + m * p.x_row_stride + g * kBlk + 4 * lane);
  float x[4] = {__uint_as_float(raw.x << 16), __uint_as_float(raw.x & 0xFFFF0000u),
                __uint_as_float(raw.y << 16), __uint_as_float(raw.y & 0xFFFF0000u)};
  float amax = fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3])));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  float scale = div_like_reference(amax, 448.0f);
  if (!(scale > 0.f)) scale = 1.0f;  // an all-zero group
#pragma unroll
  for (int i = 0; i < 4; ++i) x[i] = fminf(fmaxf(div_like_reference(x[i], scale), -448.0f), 448.0f);
  const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(x[0], x[1]), __NV_SATFINITE, __NV_E4M3);
  const uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(x[2], x[3]), __NV_SATFINITE, __NV_E4M3);
  *reinterpret_cast<uint32_t*>(p.xq + m * p.xq_row_stride + g * kBlk + 4 * lane) = lo | (hi << 16);
  if (lane == 0) {
    const __nv_bfloat16 s = __float2bfloat16_rn(scale);
    p.x_scale[m * kc + g] = *reinterpret_cast<const uint16_t*>(&s);
  }
}

// ------------------------------------------------------------------ block-scaled GEMM
struct __align__(1024) GemmSmem {
  uint8_t w[kGemmStages][kBlk * kBlk];  // weight tiles: 128 rows x 128 bytes, 128B swizzle
  uint8_t x[kGemmStages][kTok * kBlk];  // token tiles: 128 rows x 128 bytes, 128B swizzle
  float ss[kGemmStages][kTok];          // x_scale[m, kb] * w_scale[nb, kb] of the stage's block
  uint64_t full[kGemmStages];           // tiles landed
  uint64_t ss_full[kGemmStages];        // the stage's scale products written (32 lanes)
  uint64_t empty[kGemmStages];          // the MMA's commit and every promotion warp
  uint64_t d_full[kDBufs];              // D buffer complete
  uint64_t d_empty[kDBufs];             // D buffer read by every promotion warp
  // the row-parallel launch's bf16 output tile, 128 rows x 16 chunks of 16 bytes, chunk c of row
  // r at r * 16 + (c ^ (r & 15)) (spread over the banks); lets the copy to the owner run as
  // whole rows
  uint4 stage[kTok * 16];
  uint32_t tmem_base;
};
static_assert(sizeof(GemmSmem) + 1024 <= 227 * 1024, "smem");
static_assert(sizeof(GemmSmem) > 114 * 1024, "one CTA per SM: the D ring takes all of TMEM");

// a0 = fma(d0, s, a0), a1 = fma(d1, s, a1): one packed fp32x2 instruction, each half an IEEE
// fused multiply-add.
__device__ __forceinline__ void fma2(float& a0, float& a1, float d0, float d1, float s) {
  asm("{\n\t.reg .b64 a, d, s;\n\t"
      "mov.b64 a, {%0, %1};\n\t"
      "mov.b64 d, {%2, %3};\n\t"
      "mov.b64 s, {%4, %4};\n\t"
      "fma.rn.f32x2 a, d, s, a;\n\t"
      "mov.b64 {%0, %1}, a;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "f"(d0), "f"(d1), "f"(s));
}

__device__ __forceinline__ float bf16_to_f32(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

// Work unit u -> (feature block nb, token tile mt, K range split); feature blocks vary fastest.
struct GemmUnit {
  int nb, split, kb0, nk;
  int64_t m0;
};
__device__ __forceinline__ GemmUnit gemm_unit(const Fp8GemmParams& p, int64_t u) {
  const int tiles_n = p.N / kBlk;
  const int kc = p.K / kBlk;
  const int per = (kc + p.splits - 1) / p.splits;
  GemmUnit g;
  g.nb = static_cast<int>(u % tiles_n);
  const int64_t rest = u / tiles_n;
  g.split = static_cast<int>(rest % p.splits);
  g.m0 = (rest / p.splits) * kTok;
  g.kb0 = g.split * per;
  g.nk = max(0, min(kc, g.kb0 + per) - g.kb0);
  return g;
}

// ---- cross-GPU stamps (peer memory; system scope)
constexpr unsigned long long kPeerWaitLimitNs = 5000000000ull;  // 5 s: ranks launch at skewed times

__device__ __forceinline__ void stamp_release(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long stamp_acquire(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// Wait until *p >= epoch; gives up after kPeerWaitLimitNs, recording kDevErrWaitTimeout.
__device__ __forceinline__ bool wait_stamp(const unsigned long long* p, unsigned long long epoch,
                                           int* err) {
  unsigned long long t0 = 0;
  for (uint32_t polls = 0;; ++polls) {
    if (stamp_acquire(p) >= epoch) return true;
    if ((polls & 63u) == 63u) {
      const unsigned long long now = globaltimer_ns();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > kPeerWaitLimitNs) {
        if (err) atomicExch(err, kDevErrWaitTimeout);
        return false;
      }
    }
    __nanosleep(128);
  }
}
// Barrier of the 256 promotion threads (warps 0-7) only.
__device__ __forceinline__ void promo_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// The promotion threads' tile through shared memory: a thread puts its row's 64 bf16 outputs
// (eight 16-byte chunks, columns 64 h .. + 63) into the stage; after a barrier, every thread
// copies chunks tid, tid + 256, ... out as whole rows (a warp writes two 256-byte rows per
// instruction, where the threads' own row-wise stores would each be a separate 16-byte write).
__device__ __forceinline__ void stage_bf16_row(uint4* stage, int row, int h, const float (&v)[64]) {
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    uint32_t w4[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const __nv_bfloat162 h2 = __floats2bfloat162_rn(v[8 * q + 2 * e], v[8 * q + 2 * e + 1]);
      w4[e] = *reinterpret_cast<const uint32_t*>(&h2);
    }
    stage[row * 16 + ((8 * h + q) ^ (row & 15))] = make_uint4(w4[0], w4[1], w4[2], w4[3]);
  }
}
// rows [0, rows) of the stage (16 chunks of 16 bytes each) to dst, rows pitch_bytes apart
__device__ __forceinline__ void copy_stage_rows(const uint4* stage, uint8_t* dst, int64_t pitch_bytes,
                                                int64_t rows, int tid) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int c = tid + 256 * i, r16 = c >> 4, col = c & 15;
    if (r16 < rows)
      *reinterpret_cast<uint4*>(dst + r16 * pitch_bytes + 16 * col) =
          stage[r16 * 16 + (col ^ (r16 & 15))];
  }
}

// Before a stamp that publishes the promotion threads' stores to other GPUs: one system-scope
// fence per warp, by lane 0 after the warp's lanes have synchronised; the barrier that follows
// and the stamping thread's release carry them on (the fences are cumulative).  A fence in every
// thread cost ~20 us per tile: system-scope fences of an SM's threads run one after another.
__device__ __forceinline__ void publish_fence(int lane) {
  __syncwarp();
  if (lane == 0) __threadfence_system();
}

// Phases 2 and 3 of the row-parallel launch, run by the promotion threads after the GEMM units.
// Phase 2: for each tile this rank owns (tiles rank, rank + world, ...; spread over the CTAs),
// wait for every source's stamp, sum the world bf16 partials in rank order in fp32 (what an
// all-reduce of the ranks' bf16 outputs computes), round to bf16 and write the rows to every
// rank's `out`; then, once for all of the CTA's tiles, fence and stamp them final on every rank
// (a fence waits for the remote writes' acknowledgements: one per tile cost ~30 us each).
// Phase 3: wait until every tile of this rank's `out` is stamped final, so the output is complete
// when the launch ends.
__device__ void tp_reduce_gather(const Fp8GemmParams& p, const Fp8TpParams& tp, int tid) {
  const int tiles_n = p.N / kBlk;
  const int64_t tiles = ((p.M + kTok - 1) / kTok) * tiles_n;
  // after one wait has given up, later waits of the same thread are skipped (the error word is
  // set; the output is not valid), so a missing peer costs one limit, not one per tile
  bool alive = true;
  for (int64_t j = blockIdx.x;; j += gridDim.x) {
    const int64_t t = tp.rank + j * tp.world;
    if (t >= tiles) break;
    if (tid == 0)
      for (int s = 0; s < tp.world && alive; ++s)
        alive = wait_stamp(tp.flags[tp.rank] + s * tp.tiles_cap + t, tp.epoch, p.err);
    promo_sync();
    // thread: 16-byte chunks tid, tid + 256, ... of the tile (row = chunk / 16), so a warp reads
    // and writes two whole 256-byte rows per instruction; sources outermost, so that the eight
    // chunks' loads of one source are in flight together (each element still sums the sources
    // in rank order)
    const int64_t m0 = (t / tiles_n) * kTok;
    const int nbase = static_cast<int>(t % tiles_n) * kBlk;
    float a8[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int e = 0; e < 8; ++e) a8[i][e] = 0.f;
    for (int s = 0; s < tp.world; ++s) {
      uint4 w[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int c = tid + 256 * i, r16 = c >> 4, col = c & 15;
        const int64_t m = m0 + r16;
        // peers wrote these rows: read them from L2 (ld.global.cg), not from a stale L1 line
        w[i] = m < p.M ? __ldcg(reinterpret_cast<const uint4*>(
                             tp.recv[tp.rank] + (static_cast<int64_t>(s) * p.M + m) * p.N + nbase +
                             8 * col))
                       : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t ws[4] = {w[i].x, w[i].y, w[i].z, w[i].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          a8[i][2 * e] += __uint_as_float(ws[e] << 16);
          a8[i][2 * e + 1] += __uint_as_float(ws[e] & 0xFFFF0000u);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int c = tid + 256 * i, r16 = c >> 4, col = c & 15;
      const int64_t m = m0 + r16;
      if (m >= p.M) continue;
      uint32_t v[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const __nv_bfloat162 h2 = __floats2bfloat162_rn(a8[i][2 * e], a8[i][2 * e + 1]);
        v[e] = *reinterpret_cast<const uint32_t*>(&h2);
      }
      for (int r = 0; r < tp.world; ++r)
        *reinterpret_cast<uint4*>(tp.out[r] + m * p.N + nbase + 8 * col) =
            make_uint4(v[0], v[1], v[2], v[3]);
    }
    promo_sync();  // before tid 0 waits for the next tile
  }
  // publish the owned tiles' final rows: one fence per warp, then the stamps on every rank
  publish_fence(tid & 31);
  promo_sync();
  for (int64_t j = blockIdx.x + static_cast<int64_t>(tid) * gridDim.x;; j += 256LL * gridDim.x) {
    const int64_t t = tp.rank + j * tp.world;
    if (t >= tiles) break;
    for (int r = 0; r < tp.world; ++r)
      stamp_release(tp.flags[r] + static_cast<int64_t>(tp.world) * tp.tiles_cap + t, tp.epoch);
  }
  alive = true;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * 256 + tid; t < tiles && alive;
       t += static_cast<int64_t>(gridDim.x) * 256)
    alive = wait_stamp(tp.flags[tp.rank] + static_cast<int64_t>(tp.world) * tp.tiles_cap + t,
                       tp.epoch, p.err);
}

// kTP = false: the block-scaled GEMM.  kTP = true: the row-parallel launch -- each unit's bf16
// tile goes to its owner's receive buffer and is stamped there, then tp_reduce_gather.
template <bool kTP>
__global__ void __launch_bounds__(kGemmThreads, 1)
    fp8_block_gemm_kernel(const __grid_constant__ CUtensorMap tmx,
                          const __grid_constant__ CUtensorMap tmw, const Fp8GemmParams p,
                          const Fp8TpParams tp) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  GemmSmem& sm = *reinterpret_cast<GemmSmem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kc = p.K / kBlk;
  const int64_t units = ((p.M + kTok - 1) / kTok) * (p.N / kBlk) * p.splits;

  if (tid == 0) {
    for (int i = 0; i < kGemmStages; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.ss_full[i], 32);
      mbar_init(&sm.empty[i], 1 + kPromoWarps);
    }
    for (int b = 0; b < kDBufs; ++b) {
      mbar_init(&sm.d_full[b], 1);
      mbar_init(&sm.d_empty[b], kPromoWarps);
    }
    fence_mbar_init();
  }
  if (warp == kProducerWarp && lane == 0) {
    prefetch_tensormap(&tmx);
    prefetch_tensormap(&tmw);
  }
  if (warp == kMmaWarp) {
    tc::tmem_alloc(&sm.tmem_base, kDBufs * kTok);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = sm.tmem_base;
  // launched as a programmatic dependent of the quantisation kernel: nothing it writes is read
  // before it has finished
  asm volatile("griddepcontrol.wait;" ::: "memory");

  // Every role walks the same units and K blocks; r counts this CTA's K blocks (ring position).
  if (warp == kProducerWarp) {
    // ============================================================ producer (TMA)
    if (lane == 0) {
      uint32_t r = 0;
      bool ok = true;
      for (int64_t u = blockIdx.x; u < units && ok; u += gridDim.x) {
        const GemmUnit g = gemm_unit(p, u);
        for (int i = 0; i < g.nk; ++i, ++r) {
          const int stage = r % kGemmStages;
          if (!mbar_wait(&sm.empty[stage], ((r / kGemmStages) & 1) ^ 1, p.err)) { ok = false; break; }
          mbar_arrive_expect_tx(&sm.full[stage], kBlk * kBlk + kTok * kBlk);
          tma_load_2d(&sm.w[stage][0], &tmw, &sm.full[stage], (g.kb0 + i) * kBlk, g.nb * kBlk);
          tma_load_2d(&sm.x[stage][0], &tmx, &sm.full[stage], (g.kb0 + i) * kBlk,
                      static_cast<int>(g.m0));
        }
      }
    }
    __syncwarp();
  } else if (warp == kScaleWarp) {
    // ============================================================ scale products
    // ss[m] = x_scale[m0 + m, kb] * w_scale[nb, kb] in fp32 (the reference's s_act * s_w).  The
    // loads of kScaleBatch blocks are issued together, before the waits for their stages, so
    // their latency overlaps.
    uint32_t r = 0;
    bool ok = true;
    for (int64_t u = blockIdx.x; u < units && ok; u += gridDim.x) {
      const GemmUnit g = gemm_unit(p, u);
      for (int i0 = 0; i0 < g.nk && ok; i0 += kScaleBatch) {
        float xv[kScaleBatch][kTok / 32], sw[kScaleBatch];
#pragma unroll
        for (int t = 0; t < kScaleBatch; ++t) {
          const int kb = g.kb0 + min(i0 + t, g.nk - 1);
          sw[t] = bf16_to_f32(__ldg(p.w_scale + static_cast<int64_t>(g.nb) * kc + kb));
#pragma unroll
          for (int e = 0; e < kTok / 32; ++e) {
            const int64_t m = g.m0 + lane + 32 * e;
            xv[t][e] = m < p.M ? bf16_to_f32(__ldg(p.x_scale + m * kc + kb)) : 0.f;
          }
        }
#pragma unroll
        for (int t = 0; t < kScaleBatch; ++t) {
          if (i0 + t >= g.nk) break;
          const uint32_t rr = r + i0 + t;
          const int stage = rr % kGemmStages;
          if (!mbar_wait(&sm.empty[stage], ((rr / kGemmStages) & 1) ^ 1, p.err)) { ok = false; break; }
#pragma unroll
          for (int e = 0; e < kTok / 32; ++e) sm.ss[stage][lane + 32 * e] = xv[t][e] * sw[t];
          mbar_arrive(&sm.ss_full[stage]);
        }
      }
      r += g.nk;
    }
  } else if (warp == kMmaWarp || warp == kMmaWarp2) {
    // ============================================================ MMA issuers
    // Two threads in warps on different schedulers take alternate K-block positions: an MMA
    // instruction holds its issuing thread for about 100 cycles, more than the tensor core
    // needs for it, so one issuer cannot keep the tensor core busy.  Their blocks go to distinct
    // D buffers, and each thread's commits track its own MMAs only.
    if (lane == 0) {
      const uint32_t idesc = tc::idesc_e4m3(kTok, kBlk, false, false);
      const uint32_t mine = warp == kMmaWarp2 ? 1u : 0u;
      uint32_t r = 0;
      bool ok = true;
      for (int64_t u = blockIdx.x; u < units && ok; u += gridDim.x) {
        const GemmUnit g = gemm_unit(p, u);
        for (int i = 0; i < g.nk; ++i, ++r) {
          if ((r & 1u) != mine) continue;
          const int stage = r % kGemmStages;
          const int buf = r % kDBufs;
          if (!mbar_wait(&sm.full[stage], (r / kGemmStages) & 1, p.err) ||
              !mbar_wait(&sm.d_empty[buf], ((r / kDBufs) & 1) ^ 1, p.err)) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          // K steps of 32 bytes add 2 to the start-address field (address >> 4)
          const uint64_t xd = tc::smem_desc(smem_u32(&sm.x[stage][0]), 16, 1024, tc::kSw128);
          const uint64_t wd = tc::smem_desc(smem_u32(&sm.w[stage][0]), 16, 1024, tc::kSw128);
#pragma unroll
          for (int ks = 0; ks < kBlk / 32; ++ks)
            tc::mma_f8_plain(tmem + buf * kBlk, xd + static_cast<uint64_t>(2 * ks),
                             wd + static_cast<uint64_t>(2 * ks), idesc, ks > 0 ? 1u : 0u);
          tc::commit(&sm.d_full[buf]);
          tc::commit(&sm.empty[stage]);
        }
      }
    }
    __syncwarp();
  } else {
    // ============================================================ promotion
    // warp w: tensor-memory lanes 32 (w % 4) .. + 31 = tokens m0 + 32 (w % 4) + lane, and D
    // columns 64 (w / 4) .. + 63 = output features nb * 128 + 64 (w / 4) + c: a thread owns 64
    // consecutive outputs of one token row, and one scale product per K block.
    const int quad = warp & 3, half = warp >> 2;
    const uint32_t lane_base = static_cast<uint32_t>(32 * quad) << 16;
    uint32_t r = 0;
    bool ok = true;
    // Where the unit's end has barriers (the row-parallel launch, staged split-K partials), every
    // promotion thread walks every unit, also after a failed wait (then without waiting or
    // computing), so that the barriers always see all 256 threads.
    for (int64_t u = blockIdx.x; u < units && (kTP || p.splits > 1 || ok); u += gridDim.x) {
      const GemmUnit g = gemm_unit(p, u);
      const bool active = g.m0 + 32 * quad < p.M;  // warp-uniform: some row of the warp is real
      float acc[64];
#pragma unroll
      for (int j = 0; j < 64; ++j) acc[j] = 0.f;
      for (int i = 0; i < g.nk && ok; ++i, ++r) {
        const int stage = r % kGemmStages;
        const int buf = r % kDBufs;
        if (!mbar_wait(&sm.ss_full[stage], (r / kGemmStages) & 1, p.err) ||
            !mbar_wait(&sm.d_full[buf], (r / kDBufs) & 1, p.err)) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
        if (active) {
          const float sc = sm.ss[stage][32 * quad + lane];
          float d[4][16];
#pragma unroll
          for (int c = 0; c < 4; ++c) tc::ld16(tmem + lane_base + buf * kBlk + 64 * half + 16 * c, d[c]);
          tc::wait_ld();
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int j = 0; j < 16; j += 2)
              fma2(acc[16 * c + j], acc[16 * c + j + 1], d[c][j], d[c][j + 1], sc);
        }
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&sm.d_empty[buf]);
          mbar_arrive(&sm.empty[stage]);
        }
      }
      const int row = 32 * quad + lane;
      const int64_t rows = ok ? min(static_cast<int64_t>(kTok), p.M - g.m0) : 0;
      if constexpr (!kTP) {
        if (p.splits == 1) {
          // bf16 rows straight from the registers: staging them (two more barriers a unit) was
          // measured 9 % slower at 8,192 tokens; the row-wise stores stay within this GPU's L2
          if (row < rows) {
            uint4* d = reinterpret_cast<uint4*>(p.out + (g.m0 + row) * p.out_row_stride +
                                                g.nb * kBlk + 64 * half);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              uint32_t w4[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const __nv_bfloat162 h2 =
                    __floats2bfloat162_rn(acc[8 * q + 2 * e], acc[8 * q + 2 * e + 1]);
                w4[e] = *reinterpret_cast<const uint32_t*>(&h2);
              }
              d[q] = make_uint4(w4[0], w4[1], w4[2], w4[3]);
            }
          }
        } else {
          // fp32 partial sums through the stage, as whole rows (17 % faster at 256 tokens than the
          // threads' row-wise stores); the tile is 64 KB, the stage 32 KB: one half at a time
          float* dst = p.partials + (static_cast<int64_t>(g.split) * p.M + g.m0) * p.N + g.nb * kBlk;
#pragma unroll 1
          for (int h = 0; h < 2; ++h) {
            if (ok && half == h)
#pragma unroll
              for (int q = 0; q < 16; ++q)
                sm.stage[row * 16 + (q ^ (row & 15))] = make_uint4(
                    __float_as_uint(acc[4 * q]), __float_as_uint(acc[4 * q + 1]),
                    __float_as_uint(acc[4 * q + 2]), __float_as_uint(acc[4 * q + 3]));
            promo_sync();
            copy_stage_rows(sm.stage, reinterpret_cast<uint8_t*>(dst + 64 * h), p.N * 4, rows, tid);
            promo_sync();
          }
        }
      } else {
        // this rank's bf16 tile (the reference's local output) into the owner's receive buffer
        const int64_t t = (g.m0 / kTok) * (p.N / kBlk) + g.nb;
        const int owner = static_cast<int>(t % tp.world);
        // through shared memory, so that the copy to the owner (often over NVLink) runs as whole
        // 256-byte rows: a thread's row-wise 16-byte stores would each be a separate small write
        if (ok) stage_bf16_row(sm.stage, row, half, acc);
        promo_sync();
        uint16_t* dst = tp.recv[owner] + (static_cast<int64_t>(tp.rank) * p.M + g.m0) * p.N +
                        g.nb * kBlk;
        copy_stage_rows(sm.stage, reinterpret_cast<uint8_t*>(dst), p.N * 2, rows, tid);
        promo_sync();  // the stage is rewritten by the next unit
      }
    }
    if constexpr (kTP) {
      // publish this CTA's tiles: one fence per warp, then the stamps, one thread a unit
      publish_fence(lane);
      promo_sync();
      if (ok) {
        for (int64_t u = blockIdx.x + static_cast<int64_t>(tid) * gridDim.x; u < units;
             u += static_cast<int64_t>(256) * gridDim.x) {
          const GemmUnit g = gemm_unit(p, u);
          const int64_t t = (g.m0 / kTok) * (p.N / kBlk) + g.nb;
          stamp_release(tp.flags[t % tp.world] + static_cast<int64_t>(tp.rank) * tp.tiles_cap + t,
                        tp.epoch);
        }
      }
      tp_reduce_gather(p, tp, tid);
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == kMmaWarp) tc::tmem_dealloc(tmem, kDBufs * kTok);
}

// out[m, n] = bf16(sum over the splits, in order, of partials[s, m, n]); four values a thread.
__global__ void __launch_bounds__(256) fp8_split_reduce_kernel(const Fp8GemmParams p) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int64_t quads = p.M * (p.N / 4);
  const int64_t q = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x;
  if (q >= quads) return;
  const int64_t m = q / (p.N / 4);
  const int n = static_cast<int>(q - m * (p.N / 4)) * 4;
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int k = 0; k < p.splits; ++k) {
    const float4 v = *reinterpret_cast<const float4*>(p.partials + (static_cast<int64_t>(k) * p.M + m) * p.N + n);
    s.x += v.x;
    s.y += v.y;
    s.z += v.z;
    s.w += v.w;
  }
  uint16_t* dst = p.out + m * p.out_row_stride + n;
  const __nv_bfloat16 a = __float2bfloat16_rn(s.x), b = __float2bfloat16_rn(s.y);
  const __nv_bfloat16 c = __float2bfloat16_rn(s.z), d = __float2bfloat16_rn(s.w);
  dst[0] = *reinterpret_cast<const uint16_t*>(&a);
  dst[1] = *reinterpret_cast<const uint16_t*>(&b);
  dst[2] = *reinterpret_cast<const uint16_t*>(&c);
  dst[3] = *reinterpret_cast<const uint16_t*>(&d);
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// [rows, row_bytes] e4m3 (row stride `stride` bytes) in boxes of 128 bytes x box_rows rows, 128B
// swizzle; rows past the end read as zeros.
bool make_rows_map(CUtensorMap* map, const void* base, int64_t rows, int64_t row_bytes,
                   int64_t stride, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(row_bytes), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(stride)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kBlk), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

cudaError_t launch_fp8_dyn_quant(const Fp8QuantParams& p, cudaStream_t stream) {
  const int64_t groups = p.M * (p.K / kBlk);
  if (groups == 0) return cudaSuccess;
  const int64_t blocks = (groups + 7) / 8;
  fp8_dyn_quant_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(p);
  return cudaGetLastError();
}

// Split-K, only when there are fewer output tiles than SMs (else its partial sums cost more
// traffic than the last wave's imbalance): the number of K ranges s (1 .. 16) that minimises the
// persistent grid's time in K-block steps, ceil(units(s) / num_sms) * ceil(kc / s), the smaller s
// on ties.
int fp8_gemm_splits(int64_t M, int N, int K, int num_sms) {
  const int64_t base = static_cast<int64_t>(N / kBlk) * ((M + kTok - 1) / kTok);
  const int kc = K / kBlk;
  if (base <= 0 || kc <= 0 || num_sms <= 0 || base >= num_sms) return 1;
  int best = 1;
  int64_t best_cost = ((base + num_sms - 1) / num_sms) * kc;
  for (int s = 2; s <= 16 && s <= kc; ++s) {
    const int per = (kc + s - 1) / s;
    if ((kc + per - 1) / per != s) continue;  // s ranges of `per` blocks, none empty
    const int64_t cost = ((base * s + num_sms - 1) / num_sms) * per;
    if (cost < best_cost) {
      best = s;
      best_cost = cost;
    }
  }
  return best;
}

int64_t fp8_gemm_workspace_bytes(int64_t M, int N, int K, int num_sms) {
  const int s = fp8_gemm_splits(M, N, K, num_sms);
  return kCtrlInts * 4 + (s > 1 ? static_cast<int64_t>(s) * M * N * 4 : 0);
}

namespace {
template <bool kTP>
cudaError_t launch_gemm_impl(const Fp8GemmParams& p, const Fp8TpParams& tp, int num_sms,
                             cudaStream_t stream) {
  CUtensorMap tmx, tmw;
  if (!make_rows_map(&tmx, p.xq, p.M, p.K, p.xq_row_stride, kTok) ||
      !make_rows_map(&tmw, p.w, p.N, p.K, p.K, kBlk))
    return cudaErrorInvalidValue;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  const size_t smem = sizeof(GemmSmem) + 1024;
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaFuncSetAttribute(fp8_block_gemm_kernel<kTP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(smem));
    configured[dev] = true;
  }
  const int64_t units = ((p.M + kTok - 1) / kTok) * (p.N / kBlk) * p.splits;
  const int64_t ctas = units < num_sms ? units : num_sms;
  // both kernels are programmatic dependents of the kernel before them on the stream
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(ctas));
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, fp8_block_gemm_kernel<kTP>, tmx, tmw, p, tp);
  if (e != cudaSuccess || p.splits == 1) return e;
  const int64_t quads = p.M * (p.N / 4);
  cudaLaunchConfig_t rcfg = {};
  rcfg.gridDim = dim3(static_cast<unsigned>((quads + 255) / 256));
  rcfg.blockDim = dim3(256);
  rcfg.stream = stream;
  rcfg.attrs = attr;
  rcfg.numAttrs = 1;
  return cudaLaunchKernelEx(&rcfg, fp8_split_reduce_kernel, p);
}
}  // namespace

cudaError_t launch_fp8_block_gemm(const Fp8GemmParams& p, int num_sms, cudaStream_t stream) {
  if (p.M == 0) return cudaSuccess;
  return launch_gemm_impl<false>(p, Fp8TpParams{}, num_sms, stream);
}

cudaError_t launch_fp8_tp_gemm(const Fp8GemmParams& p, const Fp8TpParams& tp, int num_sms,
                               cudaStream_t stream) {
  if (p.M == 0) return cudaSuccess;
  if (p.splits != 1 || tp.world < 1 || tp.world > kMaxTpRanks) return cudaErrorInvalidValue;
  return launch_gemm_impl<true>(p, tp, num_sms, stream);
}

}  // namespace fp8attn
