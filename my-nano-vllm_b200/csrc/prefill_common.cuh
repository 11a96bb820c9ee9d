// Shared parts of the two varlen causal prefill kernels (prefill.cu: one CTA per work item;
// prefill_persistent.cu: one CTA per SM claiming work items): constants, the ring's tile header,
// the CTA's shared memory, per-sequence geometry, the q / P conversions to e4m3 hi + lo, and the
// K/V tensor maps.
//
// Both replace fp8_paged_attention_prefill_kernel (nanovllm/kernels/fp8_attention.py:209-312) for
// query sequences too long for the split-KV decode engine (which the prefill entry point uses for
// speculative-verify sized sequences).  Same contract: sequence s has query rows
// cu_q[s]..cu_q[s+1] and nk = cu_k[s+1] - cu_k[s] key positions; query row i attends key
// positions j <= i + (nk - nq) (:267-268, :297-298); K/V come from the paged cache through
// block_tables (first max_num_blocks columns visited, :281) or from contiguous [Tk, KVH, 128]
// rows starting at cu_k[s] (:254-263); rows with no visible key give 0 (:311).
//
// A work item is one (q tile of 128 rows, NG q heads of one kv head, sequence): NG = 2 when the
// GQA group is even, so two softmax groups share every K/V tile and take turns on the tensor
// cores (while one computes its P, the MMAs of the other run).  Warps of a CTA:
//   warps 8g..8g+7  softmax group g: warp (g, half, quadrant) owns query rows 32 quadrant .. +31
//             of head g and key columns 64 half .. +63 of every tile.  A thread converts its half
//             of a q row to e4m3 hi + lo (power-of-two row scale, shared by both halves), then per
//             key tile reads its S columns from tensor memory twice (max, then P), writes
//             P = 16 * 2^(s - m) as e4m3 hi + lo back into the S columns already read, and
//             finally divides its half of the tensor-memory O row by the row sum.  O is rescaled
//             only when a row maximum grows by more than 2^4 (P <= 256);
//   warp 8 NG       TMA producer: 128-token K and V tiles (128-byte rows, 128B swizzle) into the
//             ring; key tiles past the causal limit of the q tile's last row are never loaded;
//   warp 8 NG + 1   MMA issuer (one thread), per tile and group:
//               O_g += [Phi_g; Plo_g] . V   two accumulating kind::f8f6f4 chains, P_g read from
//                                           tensor memory, V MN-major straight from its TMA tile
//               S_g  = [Qhi_g; Qlo_g] . K^T  two accumulating kind::f8f6f4 chains, M = N = 128
//             in that order: P_g occupies S_g's columns until its PV has read it.
#pragma once

#include <climits>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace fp8attn {
namespace {

constexpr int kBM = 128;      // query rows per work item
constexpr int kBN = 128;      // key positions per tile
constexpr int kMaxBoxes = kBN / 16;
constexpr float kRescaleLog2 = 4.f;  // lazy rescale threshold (log2 units)
constexpr float kPScaleLog2 = 4.f;   // P is quantised as 16 * 2^(s - m_ref) <= 16 * 2^4

// Tile header, written by the producer for every ring stage it fills.  In the persistent kernel
// the item's geometry travels with every tile, so the softmax threads keep none of it live across
// the tiles; the per-item kernel uses only the tile's own fields (j0, boxmask, blk).
struct PrefillTile {
  int item;                   // work item (< 0: no more work)
  int j, ntiles;              // this tile of the item's ntiles (ntiles 0: rows see no key)
  int j0;                     // first key position of the tile
  uint32_t boxmask;           // boxes whose block is valid (contiguous layout: all)
  int vis;                    // key positions that can be read
  int lim0;                   // largest visible key position of the tile's first q row
  int rows;                   // q rows of the tile
  int kvh;                    // kv head
  int k_begin;                // contiguous layout: the sequence's first key row
  int64_t q_off, out_off;     // element offsets of (first row, first head of the pair) in q / out
  int blk[kMaxBoxes];         // paged: physical block of each box (-1: masked)
};

template <int NG>
struct PrefillCfg {
  static constexpr int kStages = 2;
  static constexpr int kNH = 2;                      // warps per row quadrant (column halves)
  static constexpr int kGroupThreads = 128 * kNH;    // softmax threads of one group
  static constexpr int kProducerWarp = 4 * kNH * NG;
  static constexpr int kMmaWarp = kProducerWarp + 1;
  static constexpr int kThreads = (kProducerWarp + 2) * 32;
  // tensor memory: group g's S (and its P, written over the columns already read) at 256 g,
  // its O at 256 g + 128
  static constexpr uint32_t kTmemCols = NG == 2 ? 512 : 256;
};

template <int NG>
struct __align__(1024) PrefillSmem {
  static constexpr int kStages = PrefillCfg<NG>::kStages;
  uint8_t qhi[NG][kBM * 128];           // A operand of S: K-major SW128
  uint8_t qlo[NG][kBM * 128];
  uint8_t k[kStages][kBN * 128];        // TMA tiles, 128-byte rows, 128B swizzle
  uint8_t v[kStages][kBN * 128];
  // the V tile as f16, the PV B operand (MN-major, 128B swizzle): two 64-dim halves of kBN key
  // rows x 128 bytes (per-item kernel)
  uint8_t vh[kStages][2 * kBN * 128];
  PrefillTile tile[kStages];
  // general-path column table of the group's current tile (thread r fills column r): key and
  // value scales, and a validity bit per column
  float colk[NG][kBN];
  float colv[NG][kBN];
  uint32_t colok[NG][kBN / 32];
  uint64_t kv_full[kStages];
  uint64_t vh_full[kStages];   // the stage's f16 V written (every softmax thread; per-item kernel)
  uint64_t kv_empty[kStages];  // K and V read by every group's MMAs (one commit), header by the
                               // softmax threads
  // per-row values the two column halves of a group exchange (q amax, tile max, row sum)
  float xq[NG][2][kBM];
  float xmax[NG][2][kBM];
  float xl[NG][2][kBM];
  uint64_t q_full[NG];
  uint64_t s_full[NG];         // S_g(j) ready
  uint64_t o_full[NG];         // an item's last PV_g done: O_g final
  uint64_t p_full[NG];         // P_g(j) in tensor memory, O_g rescaled, invalid V rows zeroed
  uint64_t xch[NG];            // the group's exchanges (all its softmax threads)
  uint64_t xpair[NG][4];       // exchanges of one row quadrant's two column-half warps
  uint64_t o_free[NG];         // the group's read-out of an item's O is done
  uint32_t tmem_base;
  int scratch[32];
  // persistent kernel: followed in shared memory by the plan, int prefix[num_seqs + 1] (the work
  // items before each sequence)
};
static_assert(sizeof(PrefillSmem<2>) + 1024 + (kMaxSeqs + 1) * 4 <= 227 * 1024, "smem");
static_assert(sizeof(PrefillSmem<1>) + 1024 + (kMaxSeqs + 1) * 4 <= 227 * 1024, "smem");

struct SeqInfo {
  int q_begin, nq, k_begin, nk;
  int vis;        // key positions that can be read (paged: capped by the table width)
  int ntiles;     // key tiles this q tile needs
};

__device__ __forceinline__ bool seq_info(const PrefillParams& p, int s, int qt, SeqInfo& si) {
  si.q_begin = __ldg(p.cu_q + s);
  si.nq = __ldg(p.cu_q + s + 1) - si.q_begin;
  si.k_begin = __ldg(p.cu_k + s);
  si.nk = __ldg(p.cu_k + s + 1) - si.k_begin;
  if (si.nq < p.min_q || qt * kBM >= si.nq) return false;
  si.vis = si.nk;
  if (p.block_tables != nullptr) si.vis = min(si.vis, p.max_blocks * p.block_size);
  if (si.vis < 0) si.vis = 0;
  const int q_last = min(si.nq, qt * kBM + kBM) - 1;
  const int lim = q_last + (si.nk - si.nq);  // largest key position any row of the tile sees
  const int kv_end = min(si.vis, lim + 1);
  si.ntiles = kv_end > 0 ? (kv_end + kBN - 1) / kBN : 0;
  return true;
}

// Power-of-two scale so that |x| / s < 256 for the largest element (same rule as the decode
// engine's query rows); returns 1/s and writes s.
__device__ __forceinline__ float pow2_inv_scale(float amax, float* s) {
  int ex = 0;
  if (amax > 0.f && amax < INFINITY) ex = ((__float_as_uint(amax) >> 23) & 0xFF) - 127;
  ex = max(-100, min(ex, 120));
  *s = __uint_as_float(static_cast<uint32_t>(127 - 7 + ex) << 23);
  return __uint_as_float(static_cast<uint32_t>(127 + 7 - ex) << 23);
}

// 16 floats -> e4m3 hi (16 bytes) and lo (16 bytes) such that x ~= hi + lo.
__device__ __forceinline__ void split16(const float* x, uint4& hi, uint4& lo) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const float x0 = x[4 * w], x1 = x[4 * w + 1], x2 = x[4 * w + 2], x3 = x[4 * w + 3];
    const uint32_t h01 = f32x2_to_e4m3x2(x0, x1), h23 = f32x2_to_e4m3x2(x2, x3);
    const uint32_t r01 = e4m3x2_to_f16x2(h01), r23 = e4m3x2_to_f16x2(h23);
    const __half2 b01 = *reinterpret_cast<const __half2*>(&r01);
    const __half2 b23 = *reinterpret_cast<const __half2*>(&r23);
    const uint32_t l01 = f32x2_to_e4m3x2(x0 - __low2float(b01), x1 - __high2float(b01));
    const uint32_t l23 = f32x2_to_e4m3x2(x2 - __low2float(b23), x3 - __high2float(b23));
    h[w] = h01 | (h23 << 16);
    l[w] = l01 | (l23 << 16);
  }
  hi = make_uint4(h[0], h[1], h[2], h[3]);
  lo = make_uint4(l[0], l[1], l[2], l[3]);
}

// 32x32b.x32: thread reads 32 consecutive columns of its lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  float a[16], b[16];
  tc::ld16(taddr, a);
  tc::ld16(taddr + 16, b);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    v[i] = a[i];
    v[16 + i] = b[i];
  }
}

__host__ __device__ constexpr int box_rows_of(bool paged, int bs) {
  return paged ? (bs % 128 == 0 ? 128 : bs % 64 == 0 ? 64 : bs % 32 == 0 ? 32 : 16) : kBN;
}

// Tensor-memory column of the 16 P words of the 32-key chunk at key column c0 (f16 pairs in key
// order, or e4m3 hi: 8 columns then lo: 8): inside the 64 S columns of the chunk's half, over the
// first 32, which that half has already read when it writes P.
__device__ __forceinline__ constexpr uint32_t p_col(int c0) {
  return static_cast<uint32_t>((c0 & ~63) + ((c0 & 63) >> 1));
}


using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn() {
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

inline bool make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t row_bytes, int kvh,
              int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(kvh) * 128, static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
  const cuuint32_t box[2] = {128, static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}


}  // namespace

// The persistent kernel's launch (prefill_persistent.cu), for launch_prefill's choice.
cudaError_t launch_prefill_persistent(const PrefillParams& p, const CUtensorMap& tmk,
                                      const CUtensorMap& tmv, cudaStream_t stream);

}  // namespace fp8attn
