// Split-KV paged decode engine (HBM-bound), on the sm_100a tensor cores.
//
// Replaces fp8_paged_attention_decode_kernel (nanovllm/kernels/fp8_attention.py:88-171) and,
// inside the prefill entry point, serves the short query sequences of speculative verification
// (1 + k rows per sequence, causal among themselves).
//
// Work decomposition.  A work item is (sequence, kv head, row group, chunk of key positions).
// A row group is up to R = 8*NT query rows that share one kv head (GQA: the group's q heads,
// times the sequence's query tokens in spec mode), so each K/V byte is read from HBM once per
// row group -- once in total for decode.  Every CTA first computes the same plan from the
// sequence lengths (chunk size, item prefix sums in shared memory: per sequence, or for large
// batches per range of sequences), then a persistent grid pulls items from an atomic counter.
// An item whose (sequence, kv head, row group) has more than one chunk writes an unnormalised
// partial (O, reference max, row sum); a combine kernel, launched after, merges them using the
// plan CTA 0 publishes.
//
// Two CTAs per SM, eight warps each (warps 6-7 have no role; they balance the register file
// across the four schedulers):
//   warp 4  producer: walks the items (the next one claimed and its block-table window and query
//           rows prefetched one item ahead), writes a 16-word tile header one word per lane,
//           and issues TMA loads of 128-token K and V tiles (128-byte rows, 128B swizzle; one
//           lane per box) into a 3-deep ring (2-deep for wider row groups); per item it prepares
//           the query rows as e4m3 hi + lo pairs (q scaled by a power of two per row, about 8
//           significant bits in total);
//   warp 5  MMA issuer (one thread), per tile j:
//             S^T[128 tok x 2R]  = K_j . [Qhi; Qlo]^T          tcgen05.mma kind::f8f6f4 (e4m3)
//             O^T[128 dim x 2R] += V_{j-1}^T . [Phi; Plo]^T    (V read MN-major from its tile)
//           S double-buffered and O accumulated in tensor memory, P double-buffered in shared
//           memory;
//   warps 0-3 softmax: thread = token row of S^T (and dim row of O^T): online softmax with the
//           column max from redux.sync + a 4-warp exchange.  P = 16 * 2^(s - m_ref) (e4m3 hi +
//           lo) against a reference max that moves only when a row max grows by more than 2^4;
//           O is then rescaled in tensor memory (rare), so no per-tile work touches O.  Only the
//           RV live rows of the row group are processed (4 for the GQA-4 decode).
// K and V bytes go to the tensor cores untouched: no per-byte conversion anywhere.
#include <climits>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace fp8attn {
namespace {

constexpr int kTile = kDecodeTile;  // key positions per stage
constexpr int kMaxCtasPerSm = 2;  // single-plane engines: two CTAs share an SM
// Warp roles.  Single-plane engines (NT = 1): softmax warps 0-3, producer warp 4, MMA warp 5;
// warps 6-7 have no role (two warps per scheduler, which balances the register file so that two
// CTAs share an SM).  Wide engines (NT > 1: 16 or 24 query rows per item): softmax warps 0-7, two
// per tensor-memory lane quadrant, each with half of the rows; producer warp 8, MMA warp 9.
template <int NT>
struct Roles {
  static constexpr int kSoftmaxWarps = NT == 1 ? 4 : 8;
  static constexpr int kProducerWarp = kSoftmaxWarps;
  static constexpr int kMmaWarp = kSoftmaxWarps + 1;
  // the PV products are issued by their own thread (warp 6 of the single-plane engines, warp 10
  // of the wide ones), the S products by the MMA warp.  Wide engines: 11 warps put three on one
  // scheduler, whose 16K registers then allow at most 168 per thread (the kernel uses 160)
  static constexpr int kPvWarp = kSoftmaxWarps + 2;
  static constexpr int kWarps = NT == 1 ? 8 : 11;
  static constexpr int kThreads = 32 * kWarps;
  static constexpr int kSoftmaxThreads = 32 * kSoftmaxWarps;
};
constexpr int kMaxBoxes = kTile / 16;
// Plan target: work items per CTA, at most kItemsPerCta (the bound the workspace is sized for).
// An item costs about kItemCostTokens key positions of fixed work (claim, query operand, first
// tile's exact max, read-out, a partial to combine), so with W key positions per CTA the
// finishing time ~ W + items * kItemCostTokens + one item's length is least near
// sqrt(W / kItemCostTokens) items: 16 on 32k-token contexts, 10 on 256 sequences of 512-4096, and
// at least 6.  Wide row groups have costly item epilogues (24 rows of sums and partials), so
// they split less.
constexpr int kItemsPerCta = 16;
constexpr float kMinItemsPerCta = 6.f;
constexpr float kItemCostTokens = 160.f;
template <int NT>
__host__ __device__ constexpr int items_per_cta() { return NT == 1 ? kItemsPerCta : 2; }

enum : int { kFirst = 1, kLast = 2 };

// Per-tile header, written by the producer one word per lane: item (< 0: no more work), key
// position of the tile's first row, rows inside the chunk, flags | q slot << 4, then per box the
// cache row of its first token (-1: masked block or no box).
enum : int { kHdrItem = 0, kHdrTok0 = 1, kHdrValid = 2, kHdrFlags = 3, kHdrSlot0 = 4,
             kHdrWords = 16 };
static_assert(kHdrSlot0 + kMaxBoxes <= kHdrWords, "header");

// Per-item facts the softmax epilogue needs, by q slot (written with the item's Q operand).
struct ItemInfo {
  int kvh, rg, nchunks, qrow0, rows;
  int mbase;  // spec mode: nk - nq (row q sees key positions <= mbase + its token index)
};

template <int NT>
struct __align__(1024) DecodeSmem {
  static constexpr int R = 8 * NT;  // query rows per item
  static constexpr int N = 2 * R;   // S / O columns: rows 0..R-1 hi, R..2R-1 lo
  // single-plane engines: 3 stages, two CTAs per SM; wide engines: one CTA per SM (10 warps at
  // up to 204 registers) with 5 stages, which keeps more K/V bytes in flight per SM than two
  // CTAs with 2 stages each could (measured on 192 verify sequences of 5 rows: 0.86 -> 0.78 ms)
  static constexpr int STAGES = NT == 1 ? 3 : 5;
  uint8_t k[STAGES][kTile * kHeadDim];  // 16 KB each, 1024-aligned
  uint8_t v[STAGES][kTile * kHeadDim];
  uint8_t q2[2][N * kHeadDim];            // K-major SW128 query operand, by item parity
  uint8_t p2[2][NT][kTile * 16];          // P^T planes of 16 columns, MN-major, by tile parity
  float qscale[2][R];                     // per-row score multiplier (scale * log2 e * 2^k)
  uint8_t qstage[R * 256];                // raw bf16 query rows of the next item (cp.async)
  float alpha[4][R];                      // per-warp copy of a tile's rescale factors (rare)
  float red[2][4][R];                     // cross-warp row maxima, double-buffered by tile
  alignas(16) int vote[2][8];             // per warp: a score above its row's reference + 2^4
  float redl[2][4][R];                    // an item's per-warp row sums, by item parity
  float mfin[2][R];                       // an item's final reference maxima, by item parity
  alignas(16) int hdr[STAGES][kHdrWords];
  ItemInfo iinfo[2];
  uint64_t kv_full[STAGES];
  uint64_t kv_empty[STAGES];
  uint64_t s_full[2];
  uint64_t s_empty[2];
  uint64_t p_full[2];
  uint64_t pv_done[2];
  uint64_t q_full[2];
  uint64_t q_empty[2];
  uint64_t sync128[2];  // bounded barriers of 128 softmax threads (the wide engines' halves)
  uint32_t tmem_base;
  int scratch[16];
  unsigned long long total_work;
  // followed in shared memory by the plan, sized per launch:
  //   per sequence: int prefix[num_seqs + 1] (item prefix sums) and int info[num_seqs]
  //                 ((L << 7) | row groups); on the wide engines, up to kThreads sequences
  //                 also int perm[num_seqs]: the sequences in claim order (shortest chunks
  //                 first), prefix in that order;
  //   sampled (batches whose per-sequence arrays would leave room for one CTA per SM only):
  //                 the same two arrays over the kThreads ranges of `per` sequences that the plan
  //                 threads own -- prefix[kThreads + 1] at each range's first sequence, and info
  //                 of that sequence -- so the size no longer grows with the batch
};

// Two CTAs share an SM (228 KB of shared memory, 1 KB reserved per CTA) with the sorted plan
// arrays of up to 256 sequences, and at any batch size with the sampled plan.
static_assert(sizeof(DecodeSmem<1>) + 2 * 1024 + (2 * Roles<1>::kThreads + 1) * 4 <= 228 * 1024 / 2,
              "smem");
// The wide engines run one CTA per SM: their ring and the largest plan fit one CTA's limit.
static_assert(sizeof(DecodeSmem<2>) + 1024 + (3 * kMaxSeqs + 1) * 4 <= 227 * 1024, "smem");
static_assert(sizeof(DecodeSmem<3>) + 1024 + (3 * kMaxSeqs + 1) * 4 <= 227 * 1024, "smem");
// Claim order of a batch of up to kThreads sequences on the wide (spec-verify) engines: by the
// length of their chunks, in tiles (capped at kSortKeys), shortest first, ties by index; with
// chunks of about the same length at the end of the work, the CTAs finish together.  Measured:
// 192 verify sequences of 5 rows, 4 % faster.  The single-plane decode engines keep index order:
// the same order, permuted on the host, made 256 sequences of 512-4096 tokens 3.4 % faster, but
// the sort in the plan cost about as much as it saved there.
constexpr int kSortKeys = 32;
static_assert(kSortKeys * Roles<1>::kWarps == Roles<1>::kThreads &&
              kSortKeys * Roles<2>::kWarps == Roles<2>::kThreads, "one (key, warp) count per thread");
// sequences per range of the sampled plan, at most (for the smaller CTA): they fit the lanes of
// the producer warp
constexpr int kMaxPlanPer = (kMaxSeqs + Roles<1>::kThreads - 1) / Roles<1>::kThreads;
static_assert(kMaxPlanPer <= 32, "sampled plan");

__device__ __forceinline__ int seq_len_clamped(const DecodeParams& p, int b, int* nq_out) {
  int L, nq;
  if (p.spec_mode) {
    nq = __ldg(p.cu_q + b + 1) - __ldg(p.cu_q + b);
    L = __ldg(p.cu_k + b + 1) - __ldg(p.cu_k + b);
    if (nq < 1 || nq > p.spec_q_max) L = 0, nq = 0;  // not routed here
  } else {
    nq = 1;
    L = __ldg(p.context_lens + b);
  }
  const int cap = p.max_blocks * p.block_size;
  L = L < 0 ? 0 : (L > cap ? cap : L);
  *nq_out = nq;
  return L;
}

// Row groups of R query rows of a sequence with nq query tokens and L key positions.
__device__ __forceinline__ int seq_rowgroups(int L, int nq, int group, int R) {
  return L > 0 ? (nq * group + R - 1) / R : 0;
}

// Block-wide exclusive scan of one int per thread (kThreads threads).
template <int kThreads>
__device__ __forceinline__ int block_exclusive_scan(int v, int* smem, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) smem[warp] = x;
  __syncthreads();
  int base = 0, tot = 0;
#pragma unroll
  for (int w = 0; w < kThreads / 32; ++w) {
    const int s = smem[w];
    if (w < warp) base += s;
    tot += s;
  }
  __syncthreads();
  *total = tot;
  return base + x - v;
}

// Order-preserving float <-> int maps (for redux.sync max).
__device__ __forceinline__ int f2ord(float f) {
  const int i = __float_as_int(f);
  return i >= 0 ? i : i ^ 0x7FFFFFFF;
}
__device__ __forceinline__ float ord2f(int i) { return __int_as_float(i >= 0 ? i : i ^ 0x7FFFFFFF); }

// Producer cursor: the item whose tiles are being issued.  Warp-uniform.
template <int NT>
struct Cursor {
  int item;  // >= total_items: exhausted
  int next;  // prefetched id of the following item (lane 0 holds the atomic's result)
  int b, kvh, rg, c, nchunks, t0, t1, t;
  int qrow0, rows, lim_base, row0;
  int nth;           // items started (selects the q buffer)
  int ebase, myent;  // block-table entries ebase .. ebase+31, one per lane
};

// Claims `item` for the cursor and starts the load of its first 32 block-table entries (one
// per lane).  Called by the whole producer warp.  With the sampled plan, a search finds the
// item's range of `per` sequences and the lanes read that range's lengths (one sequence each)
// to find its sequence.
template <int NT, bool kSampled>
__device__ __forceinline__ void cursor_set(Cursor<NT>& P, int item, const DecodeParams& p,
                                           const int* prefix, const int* info, const int* perm,
                                           int per, int total_items, int CT, int B) {
  constexpr int R = DecodeSmem<NT>::R;
  P.item = item;
  if (item >= total_items) return;
  const int nranges = kSampled ? (B + per - 1) / per : B;
  int lo = 0, hi = nranges - 1;  // largest range (or sequence) with prefix <= item
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (prefix[mid] <= item) lo = mid; else hi = mid - 1;
  }
  int b, L, nrg, r;
  if (!kSampled || per == 1) {  // the range is one sequence
    b = kSampled || perm == nullptr ? lo : perm[lo];
    const int inf = info[b];
    L = inf >> 7;
    nrg = inf & 127;
    r = item - prefix[lo];
  } else {
    const int lane = threadIdx.x & 31;
    const int bl = lo * per + lane;
    int Ll = 0, nql = 0;
    if (lane < per && bl < B) Ll = seq_len_clamped(p, bl, &nql);
    const int rgl = seq_rowgroups(Ll, nql, p.group, R);
    const int cnt = (Ll + CT - 1) / CT * p.num_kv_heads * rgl;
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < kMaxPlanPer; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    const int first = prefix[lo] + incl - cnt;
    const unsigned hit = __ballot_sync(0xffffffffu, cnt > 0 && item >= first && item < first + cnt);
    if (hit == 0) {  // cannot happen with a consistent plan: report it, take no work
      if (lane == 0) atomicExch(p.ctrl, kDevErrWorkspace);
      P.item = total_items;
      return;
    }
    const int src = __ffs(hit) - 1;
    b = lo * per + src;
    L = __shfl_sync(0xffffffffu, Ll, src);
    nrg = __shfl_sync(0xffffffffu, rgl, src);
    r = item - __shfl_sync(0xffffffffu, first, src);
  }
  const int nchunks = (L + CT - 1) / CT;
  // items of sequence b: chunk-major, then kv head, then row group, so the CTAs that start
  // at about the same time read the same token rows (neighbouring heads share DRAM pages)
  const int npairs = p.num_kv_heads * nrg;
  const int c = r / npairs;
  const int pair_local = r - c * npairs;
  P.b = b;
  P.kvh = pair_local / nrg;
  P.rg = pair_local - P.kvh * nrg;
  P.c = c;
  P.nchunks = nchunks;
  // the sequence's chunks are balanced (equal up to one tile) instead of CT, CT, ..., remainder,
  // so no item is a short tail; the chunk count, which the combine uses, stays ceil(L / CT)
  const int cts = ((L + nchunks - 1) / nchunks + kTile - 1) / kTile * kTile;
  P.t0 = c * cts;
  P.t1 = min(L, P.t0 + cts);
  P.t = P.t0;
  int nq = 1;
  P.qrow0 = b;
  P.lim_base = INT_MAX / 2;
  if (p.spec_mode) {
    P.qrow0 = __ldg(p.cu_q + b);
    nq = __ldg(p.cu_q + b + 1) - P.qrow0;
    const int nk = __ldg(p.cu_k + b + 1) - __ldg(p.cu_k + b);
    P.lim_base = nk - nq;
  }
  P.row0 = P.rg * R;
  P.rows = min(R, nq * p.group - P.row0);
  if (p.spec_mode) P.lim_base += P.row0 / p.group;
  // start the loads the item will need: its first 32 block-table entries and its q rows
  const int lane = threadIdx.x & 31;
  P.ebase = P.t0 / p.block_size;
  const int idx = P.ebase + lane;
  P.myent = idx < p.max_blocks
                ? ldg_keep(p.block_tables + static_cast<int64_t>(b) * p.bt_stride + idx) : -1;
}

// Starts copying the cursor's query rows (bf16) into qstage with cp.async; prepare_q consumes
// them one item later, so the load latency is never waited on.
template <int NT>
__device__ __forceinline__ void stage_q(const Cursor<NT>& P, const DecodeParams& p, uint8_t* qstage) {
  const int lane = threadIdx.x & 31;
  const int G = p.group;
  // lane l: row (l >> 2) + 8 pass, dims 32 (l & 3) .. +32 (64 bytes), the slice prepare_q reads
#pragma unroll
  for (int pass = 0; pass < NT; ++pass) {
    const int rq = pass * 8 + (lane >> 2);
    const bool ok = rq < P.rows;
    const int rr = P.row0 + rq;
    const int j = rr / G, h = P.kvh * G + (rr - j * G);
    const uint16_t* src = ok ? p.q + static_cast<int64_t>(P.qrow0 + j) * p.q_row_stride +
                                   static_cast<int64_t>(h) * kHeadDim + 32 * (lane & 3)
                             : p.q;
    const uint32_t dst = smem_u32(qstage + rq * 256 + 64 * (lane & 3));
#pragma unroll
    for (int i = 0; i < 4; ++i) cp_async16(dst + 16 * i, src + 8 * i, ok);
  }
  cp_async_commit();
}

// The item's query rows -> K-major SW128 [hi rows | lo rows] operand + per-row multipliers.
// Lane l handles row (l >> 2) (+ 8 per pass) and dims 32 (l & 3) .. +32, from P.qraw.
template <int NT>
__device__ __forceinline__ void prepare_q(const Cursor<NT>& P, int slot, const DecodeParams& p,
                                          DecodeSmem<NT>& sm, int lane) {
  constexpr int R = DecodeSmem<NT>::R;
  const int quarter = lane & 3;
  cp_async_wait<0>();  // this item's rows (the only copy in flight)
#pragma unroll
  for (int pass = 0; pass < NT; ++pass) {
    const int r = pass * 8 + (lane >> 2);
    float q[32];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 w = *reinterpret_cast<const uint4*>(&sm.qstage[r * 256 + 64 * quarter + 16 * i]);
      const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        q[8 * i + 2 * k] = __uint_as_float(ww[k] << 16);
        q[8 * i + 2 * k + 1] = __uint_as_float(ww[k] & 0xFFFF0000u);
      }
    }
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(q[i]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    int ex = 0;  // |q| / 2^(ex-7) < 256 for the row's largest element
    if (amax > 0.f && amax < INFINITY) ex = ((__float_as_uint(amax) >> 23) & 0xFF) - 127;
    ex = max(-100, min(ex, 120));
    const float inv_s = __uint_as_float(static_cast<uint32_t>(127 + 7 - ex) << 23);
    const float s_row = __uint_as_float(static_cast<uint32_t>(127 - 7 + ex) << 23);
    uint32_t hi[8], lo[8];
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const float x0 = q[4 * w] * inv_s, x1 = q[4 * w + 1] * inv_s;
      const float x2 = q[4 * w + 2] * inv_s, x3 = q[4 * w + 3] * inv_s;
      const uint32_t h01 = f32x2_to_e4m3x2(x0, x1), h23 = f32x2_to_e4m3x2(x2, x3);
      const uint32_t r01 = e4m3x2_to_f16x2(h01), r23 = e4m3x2_to_f16x2(h23);
      const __half2 b01 = *reinterpret_cast<const __half2*>(&r01);
      const __half2 b23 = *reinterpret_cast<const __half2*>(&r23);
      const uint32_t l01 = f32x2_to_e4m3x2(x0 - __low2float(b01), x1 - __high2float(b01));
      const uint32_t l23 = f32x2_to_e4m3x2(x2 - __low2float(b23), x3 - __high2float(b23));
      hi[w] = h01 | (h23 << 16);
      lo[w] = l01 | (l23 << 16);
    }
    // rows r (hi) and R + r (lo), 16-byte chunks 2*quarter and 2*quarter + 1, 128B swizzle
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int chunk = 2 * quarter + half;
      const int rh = r, rl = R + r;
      *reinterpret_cast<uint4*>(&sm.q2[slot][rh * 128 + ((chunk ^ (rh & 7)) << 4)]) =
          make_uint4(hi[4 * half], hi[4 * half + 1], hi[4 * half + 2], hi[4 * half + 3]);
      *reinterpret_cast<uint4*>(&sm.q2[slot][rl * 128 + ((chunk ^ (rl & 7)) << 4)]) =
          make_uint4(lo[4 * half], lo[4 * half + 1], lo[4 * half + 2], lo[4 * half + 3]);
    }
    if (quarter == 0) sm.qscale[slot][r] = s_row * p.scale_log2;
  }
}

template <int NT, int RV, bool kSampled>
__global__ void __launch_bounds__(Roles<NT>::kThreads, NT == 1 ? kMaxCtasPerSm : 1)
    decode_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                  const DecodeParams p) {
  constexpr int kThreads = Roles<NT>::kThreads;
  constexpr int kWarps = Roles<NT>::kWarps;
  constexpr int kProducerWarp = Roles<NT>::kProducerWarp;
  constexpr int kMmaWarp = Roles<NT>::kMmaWarp;
  constexpr int kPvWarp = Roles<NT>::kPvWarp;
  constexpr int kSoftmaxThreads = Roles<NT>::kSoftmaxThreads;
  using Smem = DecodeSmem<NT>;
  constexpr int R = Smem::R;
  constexpr int N = Smem::N;
  constexpr int kStages = Smem::STAGES;
  static_assert(RV >= 1 && RV <= R && RV % 4 == 0, "live rows");
  constexpr uint32_t kTmemCols = 4 * N <= 64 ? 64 : (4 * N <= 128 ? 128 : 256);  // S x2, O x2
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int G = p.group;
  const int B = p.num_seqs;
  int* prefix = reinterpret_cast<int*>(&sm + 1);
  int* info = prefix + (kSampled ? kThreads : B) + 1;
  // per-sequence plan of up to kThreads sequences on the wide (spec-verify) engines: claim order
  // sorted (perm after info)
  const bool sorted_plan = !kSampled && NT > 1 && B <= kThreads;
  int* perm = sorted_plan ? info + B : nullptr;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.kv_full[s], 1);
      mbar_init(&sm.kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.s_full[i], 1);
      mbar_init(&sm.s_empty[i], kSoftmaxThreads);
      mbar_init(&sm.q_full[i], 32);
      mbar_init(&sm.q_empty[i], kSoftmaxThreads);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.p_full[i], kSoftmaxThreads);
      mbar_init(&sm.pv_done[i], 1);
    }
    mbar_init(&sm.sync128[0], 128);
    mbar_init(&sm.sync128[1], 128);
    fence_mbar_init();
    sm.total_work = 0;
  }
  if (warp == kProducerWarp && lane == 0) {
    prefetch_tensormap(&tmk);
    prefetch_tensormap(&tmv);
  }
  if (warp == kMmaWarp) {
    tc::tmem_alloc(&sm.tmem_base, kTmemCols);
    tc::tmem_relinquish();
  }

  // launched as a programmatic dependent of the previous kernel on the stream: everything above
  // overlaps its tail; no input is read before it has finished
  asm volatile("griddepcontrol.wait;" ::: "memory");

  // ---------------------------------------------------------------- plan (every CTA, same result)
  const int per = (B + kThreads - 1) / kThreads;
  const int s0 = min(B, tid * per), s1 = min(B, s0 + per);
  long long my_work = 0;
  // sampled plan: the thread's lengths and row groups, read once and kept in registers
  int len_r[kSampled ? kMaxPlanPer : 1], rg_r[kSampled ? kMaxPlanPer : 1];
  if constexpr (kSampled) {
#pragma unroll
    for (int i = 0; i < kMaxPlanPer; ++i) {
      int nq = 0;
      len_r[i] = s0 + i < s1 ? seq_len_clamped(p, s0 + i, &nq) : 0;
      rg_r[i] = seq_rowgroups(len_r[i], nq, G, R);
      my_work += static_cast<long long>(len_r[i]) * rg_r[i];
    }
  } else {
    for (int b = s0; b < s1; ++b) {
      int nq;
      const int L = seq_len_clamped(p, b, &nq);
      const int rg = seq_rowgroups(L, nq, G, R);
      info[b] = (L << 7) | rg;
      my_work += static_cast<long long>(L) * rg;
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (my_work) atomicAdd(&sm.total_work, static_cast<unsigned long long>(my_work));
  __syncthreads();
  const uint32_t tmem = sm.tmem_base;
  const unsigned long long total_work =
      sm.total_work * static_cast<unsigned long long>(p.num_kv_heads);
  long long ct;
  if constexpr (NT == 1) {
    const float per_cta = static_cast<float>(total_work) / static_cast<float>(gridDim.x);
    const float items = fminf(fmaxf(sqrtf(per_cta / kItemCostTokens), kMinItemsPerCta),
                              static_cast<float>(kItemsPerCta));
    ct = static_cast<long long>(ceilf(per_cta / items));
  } else {
    const unsigned long long target =
        static_cast<unsigned long long>(items_per_cta<NT>()) * gridDim.x;
    ct = static_cast<long long>((total_work + target - 1) / target);
  }
  if (ct < p.min_chunk) ct = p.min_chunk;
  ct = (ct + kTile - 1) / kTile * kTile;
  const int CT = static_cast<int>(ct > (1 << 24) ? (1 << 24) : ct);

  int my_items = 0;
  if constexpr (kSampled) {
#pragma unroll
    for (int i = 0; i < kMaxPlanPer; ++i)
      my_items += (len_r[i] + CT - 1) / CT * p.num_kv_heads * rg_r[i];
  } else {
    for (int b = s0; b < s1; ++b) {
      const int inf = info[b];
      my_items += (((inf >> 7) + CT - 1) / CT) * p.num_kv_heads * (inf & 127);
    }
  }
  int total_items = 0, base = 0;
  if (!sorted_plan) base = block_exclusive_scan<kThreads>(my_items, sm.scratch, &total_items);
  if constexpr (kSampled) {
    prefix[tid] = base;
    if (tid == kThreads - 1) prefix[kThreads] = total_items;
    info[tid] = (len_r[0] << 7) | rg_r[0];
    if (blockIdx.x == 0) {  // the combine kernel reads each sequence's item prefix after this launch
      int acc = base;
#pragma unroll
      for (int i = 0; i < kMaxPlanPer; ++i) {
        if (s0 + i < s1) p.plan[2 + s0 + i] = acc;
        acc += (len_r[i] + CT - 1) / CT * p.num_kv_heads * rg_r[i];
      }
      if (tid == 0) {
        p.plan[0] = CT;
        p.plan[1] = total_items;
        p.plan[2 + B] = total_items;
      }
    }
    __syncthreads();
  } else if (sorted_plan) {
    // sequence tid (one per thread): its key and items; stable counting sort by key through
    // per-warp ranks and a (key, warp) count table in the K ring (unused until the producer
    // starts), scanned key-major so that every CTA derives the same order
    const bool valid = tid < B;
    int key = kSortKeys;  // past every valid key: threads without a sequence
    if (valid) {
      const int inf = info[tid];
      const int L = inf >> 7;
      const int nch = (L + CT - 1) / CT;
      key = L > 0 ? min(((L + nch - 1) / nch + kTile - 1) / kTile, kSortKeys) - 1 : 0;
    }
    const unsigned peers = __match_any_sync(0xffffffffu, key);
    const int rank = __popc(peers & ((1u << lane) - 1));
    int* counts = reinterpret_cast<int*>(&sm.k[0][0]);
    counts[tid] = 0;
    __syncthreads();
    if (valid && rank == 0) counts[key * kWarps + warp] = __popc(peers);
    __syncthreads();
    int nseq;
    const int first = block_exclusive_scan<kThreads>(counts[tid], sm.scratch, &nseq);
    counts[tid] = first;
    __syncthreads();
    if (valid) perm[counts[key * kWarps + warp] + rank] = tid;
    __syncthreads();
    // item prefix in claim order: thread tid holds sorted position tid
    int sb = 0, scnt = 0;
    if (valid) {
      sb = perm[tid];
      const int inf = info[sb];
      scnt = ((inf >> 7) + CT - 1) / CT * p.num_kv_heads * (inf & 127);
    }
    const int sbase = block_exclusive_scan<kThreads>(scnt, sm.scratch, &total_items);
    if (valid) prefix[tid] = sbase;
    if (tid == kThreads - 1) prefix[B] = total_items;
    if (blockIdx.x == 0) {  // the combine kernel reads each sequence's first item after this launch
      if (valid) p.plan[2 + sb] = sbase;
      if (tid == 0) {
        p.plan[0] = CT;
        p.plan[1] = total_items;
        p.plan[2 + B] = total_items;
      }
    }
    fence_proxy_async_smem();  // the count table's stores come before the ring's TMA writes
    __syncthreads();
  } else {
    {
      int acc = base;
      for (int b = s0; b < s1; ++b) {
        prefix[b] = acc;
        const int inf = info[b];
        acc += (((inf >> 7) + CT - 1) / CT) * p.num_kv_heads * (inf & 127);
      }
      if (tid == kThreads - 1) prefix[B] = total_items;
    }
    __syncthreads();
    if (blockIdx.x == 0) {  // the combine kernel reads the same plan after this launch
      for (int b = tid; b <= B; b += kThreads) p.plan[2 + b] = prefix[b];
      if (tid == 0) {
        p.plan[0] = CT;
        p.plan[1] = total_items;
      }
    }
  }
  // partial results are indexed by item id; a workspace sized by decode_workspace_bytes always
  // has room, and a TMA box must fit its stage: anything else is reported, never overrun
  const bool fits = total_items <= p.max_items && p.box_rows >= 16 && p.box_rows <= kTile &&
                    kTile % p.box_rows == 0;
  if (!fits && tid == 0 && blockIdx.x == 0) atomicExch(p.ctrl, kDevErrWorkspace);

  // zero the outputs of routed sequences without key positions (reference: acc / max(s, 1e-10))
  for (int b = blockIdx.x; b < B; b += gridDim.x) {
    int nq = 1, qrow0 = b;
    if constexpr (kSampled) {
      if (per == 1 ? (info[b] >> 7) != 0 : seq_len_clamped(p, b, &nq) != 0) continue;
      nq = 1;
    } else {
      if ((info[b] >> 7) != 0) continue;
    }
    if (p.spec_mode) {
      qrow0 = __ldg(p.cu_q + b);
      nq = __ldg(p.cu_q + b + 1) - qrow0;
      if (nq < 1 || nq > p.spec_q_max) continue;
    }
    const int per_row = p.num_heads * kHeadDim / 8;  // uint4 per token row
    for (int j = 0; j < nq; ++j) {
      uint4* dst = reinterpret_cast<uint4*>(p.out + static_cast<int64_t>(qrow0 + j) * p.out_row_stride);
      for (int i = tid; i < per_row; i += kThreads) dst[i] = make_uint4(0, 0, 0, 0);
    }
  }

  if (fits && warp == kProducerWarp) {
    // ============================================================ producer
    // P: the item whose tiles are being issued; Pn: the next item, claimed and prefetching
    Cursor<NT> P, Pn;
    P.nth = 0;
    P.next = 0;
    {
      int ids[2] = {0, 0};
      if (lane == 0) {
        ids[0] = atomicAdd(p.ctrl + 1, 1);
        ids[1] = atomicAdd(p.ctrl + 1, 1);
        Pn.next = atomicAdd(p.ctrl + 1, 1);
      }
      ids[0] = __shfl_sync(0xffffffffu, ids[0], 0);
      ids[1] = __shfl_sync(0xffffffffu, ids[1], 0);
      cursor_set<NT, kSampled>(P, ids[0], p, prefix, info, perm, per, total_items, CT, B);
      cursor_set<NT, kSampled>(Pn, ids[1], p, prefix, info, perm, per, total_items, CT, B);
      if (P.item < total_items) stage_q<NT>(P, p, sm.qstage);
    }
    int stage = 0;
    uint32_t phase = 0;
    const int box_rows = p.box_rows;
    const int box_shift = 31 - __clz(box_rows);
    // lane l: cache row of the current item's box boxbase + l (-1: masked block / past the end),
    // computed once per 32 boxes from the block-table window the cursor prefetched
    int myslot = -1, boxbase = 0;
    auto compute_boxes = [&](int base) {
      const int e0 = (P.t0 + (base << box_shift)) / p.block_size;
      if (e0 != P.ebase) {  // beyond the prefetched window (items of more than 32 boxes)
        P.ebase = e0;
        const int idx = e0 + lane;
        P.myent = idx < p.max_blocks
                      ? __ldg(p.block_tables + static_cast<int64_t>(P.b) * p.bt_stride + idx) : -1;
      }
      const int pos = P.t0 + ((base + lane) << box_shift);
      const int e = pos / p.block_size;
      const int blk = __shfl_sync(0xffffffffu, P.myent, (e - P.ebase) & 31);
      myslot = (pos >= P.t1 || blk < 0 || blk >= p.num_blocks) ? -1
                                                               : blk * p.block_size + (pos - e * p.block_size);
      boxbase = base;
    };
    while (true) {
      if (P.item >= total_items) {
        if (mbar_wait(&sm.kv_empty[stage], phase ^ 1, p.ctrl) && lane == 0) {
          sm.hdr[stage][kHdrItem] = -1;
          mbar_arrive(&sm.kv_full[stage]);
        }
        break;
      }
      const int slot = P.nth & 1;
      if (P.t == P.t0) {
        if (!mbar_wait(&sm.q_empty[slot], ((P.nth >> 1) & 1) ^ 1, p.ctrl)) break;
        prepare_q<NT>(P, slot, p, sm, lane);
        if (lane < 6) {
          const int v = lane == 0 ? P.kvh : lane == 1 ? P.rg : lane == 2 ? P.nchunks
                        : lane == 3 ? P.qrow0 : lane == 4 ? P.rows : P.lim_base - P.row0 / p.group;
          reinterpret_cast<int*>(&sm.iinfo[slot])[lane] = v;
        }
        fence_proxy_async_smem();
        mbar_arrive(&sm.q_full[slot]);
        // the staging rows were read into registers above (their uses are issued): reuse it
        if (Pn.item < total_items) stage_q<NT>(Pn, p, sm.qstage);
        compute_boxes(0);
      }
      if (!mbar_wait(&sm.kv_empty[stage], phase ^ 1, p.ctrl)) break;
      const int t = P.t;
      const int nvalid = min(kTile, P.t1 - t);
      const int nbox = (nvalid + box_rows - 1) >> box_shift;
      const int ib0 = (t - P.t0) >> box_shift;
      if (ib0 + nbox > boxbase + 32) compute_boxes(ib0);
      // header, one word per lane; lane 4 + j carries box j
      const int jb = lane - kHdrSlot0;
      const int bslot = __shfl_sync(0xffffffffu, myslot, (ib0 + jb - boxbase) & 31);
      const bool boxok = jb >= 0 && jb < nbox && bslot >= 0;
      const uint32_t okmask = __ballot_sync(0xffffffffu, boxok);
      const int flags = (t == P.t0 ? kFirst : 0) | (t + kTile >= P.t1 ? kLast : 0) | (slot << 4);
      const int hv = lane == kHdrItem ? P.item : lane == kHdrTok0 ? t : lane == kHdrValid ? nvalid
                     : lane == kHdrFlags ? flags : (boxok ? bslot : -1);
      if (lane < kHdrSlot0 + kMaxBoxes) sm.hdr[stage][lane] = hv;
      if (lane == 0)
        mbar_arrive_expect_tx(&sm.kv_full[stage], __popc(okmask) * 2u * box_rows * kHeadDim);
      __syncwarp();
      // lane 2j loads K box j, lane 2j + 1 V box j
      {
        const int tj = lane >> 1;
        const int tslot = __shfl_sync(0xffffffffu, hv, (kHdrSlot0 + tj) & 31);
        if (tj < nbox && tj < kMaxBoxes && tslot >= 0) {
          const bool is_v = lane & 1;
          tma_load_2d((is_v ? &sm.v[stage][0] : &sm.k[stage][0]) + tj * box_rows * kHeadDim,
                      is_v ? &tmv : &tmk, &sm.kv_full[stage], P.kvh * kHeadDim, tslot);
        }
      }
      __syncwarp();
      if (++stage == kStages) { stage = 0; phase ^= 1; }
      P.t += kTile;
      if (P.t >= P.t1) {
        const int nth = P.nth + 1;
        const int nxt = __shfl_sync(0xffffffffu, Pn.next, 0);
        P = Pn;
        P.nth = nth;
        if (lane == 0) Pn.next = atomicAdd(p.ctrl + 1, 1);
        if (P.item < total_items) cursor_set<NT, kSampled>(Pn, nxt, p, prefix, info, perm, per, total_items, CT, B);
        else Pn.item = total_items;
      }
    }
  } else if (fits && warp == kMmaWarp) {
    // ============================================================ MMA issuer (lane 0)
    // tile j: S_j into S buffer j%2.  The PV products have their own issuing thread (kPvWarp):
    // an MMA costs its issuing thread about 100 cycles and these products are small (N = 16 per
    // plane), so one thread issuing both paced the tile loop.  The two threads' products touch
    // disjoint state (S buffers; P in shared memory and O), and each thread's commits track its
    // own products.
    if (lane == 0) {
      const uint32_t idesc_s = tc::idesc_e4m3(128, N, false, false);
      int stage = 0, j = 0;
      uint32_t phase = 0;
      int qcount[2] = {0, 0};
      while (true) {
        if (!mbar_wait(&sm.kv_full[stage], phase, p.ctrl)) break;
        if (sm.hdr[stage][kHdrItem] < 0) break;
        const int hflags = sm.hdr[stage][kHdrFlags];
        const int slot = hflags >> 4;
        if (hflags & kFirst) {
          if (!mbar_wait(&sm.q_full[slot], qcount[slot] & 1, p.ctrl)) break;
          qcount[slot]++;
        }
        const int sb = j & 1;
        if (!mbar_wait(&sm.s_empty[sb], ((j >> 1) & 1) ^ 1, p.ctrl)) break;
        tc::fence_after_sync();
        const uint32_t ka = smem_u32(&sm.k[stage][0]);
        const uint32_t qa = smem_u32(&sm.q2[slot][0]);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const uint64_t ad = tc::smem_desc(ka + ks * 32, 16, 1024, tc::kSw128);
          const uint64_t bd = tc::smem_desc(qa + ks * 32, 16, 1024, tc::kSw128);
          tc::mma_f8(tmem + sb * N, ad, bd, idesc_s, ks > 0 ? 1u : 0u);
        }
        tc::commit(&sm.s_full[sb]);
        ++j;
        if (++stage == kStages) { stage = 0; phase ^= 1; }
      }
    }
    __syncwarp();
  } else if (fits && warp == kPvWarp) {
    // ============================================================ PV issuer (lane 0)
    // PV_j as soon as P_j is written, accumulated into the O buffer of the item's parity (an
    // item's first tile starts it afresh); its commit releases the stage
    if (lane == 0) {
      // P^T's NT planes of 16 columns lie 2 KB apart, the descriptor's stride between 16-column
      // blocks (SBO): one MMA of N = 16 NT per 32-key step covers them all
      const uint32_t idesc_pv = tc::idesc_e4m3(128, 16 * NT, true, true);
      int stage = 0, j = 0;
      uint32_t phase = 0;
      int items = 0;
      while (true) {
        if (!mbar_wait(&sm.kv_full[stage], phase, p.ctrl)) break;
        if (sm.hdr[stage][kHdrItem] < 0) break;
        const int first = sm.hdr[stage][kHdrFlags] & kFirst;
        if (first) ++items;
        const int b = j & 1;
        if (!mbar_wait(&sm.p_full[b], (j >> 1) & 1, p.ctrl)) break;
        tc::fence_after_sync();
        const uint32_t va = smem_u32(&sm.v[stage][0]);
        const int ob = (items - 1) & 1;
        const uint32_t pa = smem_u32(&sm.p2[b][0][0]);
        static_assert(sizeof(sm.p2[0][0]) == 2048, "plane stride = SBO");
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const uint64_t ad = tc::smem_desc(va + ks * 32 * 128, 0, 1024, tc::kSw128);
          const uint64_t bd = tc::smem_desc(pa + ks * 32 * 16, 128, 2048, tc::kSwNone);
          tc::mma_f8(tmem + (2 + ob) * N, ad, bd, idesc_pv, (ks > 0 || !first) ? 1u : 0u);
        }
        tc::commit(&sm.kv_empty[stage]);
        tc::commit(&sm.pv_done[b]);
        ++j;
        if (++stage == kStages) { stage = 0; phase ^= 1; }
      }
    }
    __syncwarp();
  } else if (fits && warp < Roles<NT>::kSoftmaxWarps) {
    if constexpr (NT == 1) {
      // ============================================================ softmax warps 0-3
      // thread r: token row r of S^T and dim row r of O^T.  Per row q of the row group (the first
      // RV are live): m_ref[q] = reference max (log2 units, uniform over the 128 threads), l_part[q]
      // = this thread's share of the row sum, both relative to m_ref.
      const int r = tid;
      const uint32_t lane_base = static_cast<uint32_t>(32 * warp) << 16;
      const bool kscaled = p.k_scale != nullptr;
      const bool vscaled = p.v_scale != nullptr;
      const int box_shift = 31 - __clz(p.box_rows);
      constexpr float kRescaleLog2 = 4.f;  // P = 16 * 2^(s - m_ref) <= 256 < 448 (e4m3 max)
      constexpr float kPScale = 16.f;
      float m_ref[RV], l_part[RV];
      // up to 8 live rows keep their score multiplier and causal limit in registers
      constexpr bool kRowRegs = RV <= 8;
      float cs_r[kRowRegs ? RV : 1];
      int rows_i = 0, qrow_lo = 0;  // the item's live rows; spec mode: (nk - nq) G + rg R
      int kvh = 0;
      int stage = 0, j = 0, sync_uses = 0, item_first_tile = 0;
      uint32_t phase = 0;
      int qcount[2] = {0, 0};
      auto sync = [&]() -> bool {
        mbar_arrive(&sm.sync128[0]);
        return mbar_wait(&sm.sync128[0], (sync_uses++) & 1, p.ctrl);
      };
      auto wait_pv = [&](int t) -> bool {
        const int b = t & 1;
        if (!mbar_wait(&sm.pv_done[b], (t >> 1) & 1, p.ctrl)) return false;
        tc::fence_after_sync();
        return true;
      };
      const uint32_t o_base = tmem + lane_base + 2 * N;  // O of an item: o_base + (item parity) N
      int nitem = 0;  // items started
      // the item whose read-out is deferred to the next tile (its last PV is then normally done,
      // and its row-sum exchange rides on that tile's barrier)
      bool pend_ep = false;
      int pend_j = 0, pend_ob = 0, pend_slot = 0, pend_item = 0;
      auto finish = [&]() -> bool {
        if (!wait_pv(pend_j)) return false;
        float o[RV];
  #pragma unroll
        for (int q = 0; q < RV; ++q) o[q] = 0.f;
  #pragma unroll
        for (int c = 0; c < N; c += 16) {
          float o16[16];
          tc::ld16(o_base + pend_ob * N + c, o16);
          tc::wait_ld();
  #pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int q = (c + i) % R;
            if (q < RV) o[q] += o16[i];
          }
        }
        tc::fence_before_sync();
        const ItemInfo ii = sm.iinfo[pend_slot];
        const int rows = ii.rows, nchunks = ii.nchunks, rg = ii.rg, qrow0 = ii.qrow0;
        const int d = r;  // output dim
  #pragma unroll
        for (int q = 0; q < RV; ++q) {
          if (q >= rows) break;
          const float lsum = sm.redl[pend_ob][0][q] + sm.redl[pend_ob][1][q] +
                             sm.redl[pend_ob][2][q] + sm.redl[pend_ob][3][q];
          if (nchunks == 1) {
            const int rr = rg * R + q;
            const int jj = rr / G, hh = ii.kvh * G + (rr - jj * G);
            __nv_bfloat16 v = out_round(o[q] / fmaxf(lsum, 1e-10f));
            p.out[static_cast<int64_t>(qrow0 + jj) * p.out_row_stride + hh * kHeadDim + d] =
                *reinterpret_cast<uint16_t*>(&v);
          } else {
            float* part = p.partials + (static_cast<int64_t>(pend_item) * R + q) * (kHeadDim + 4);
            part[d] = o[q];
            if (d == 0) {
              // a chunk whose rows saw no key position carries no weight in the combine
              part[kHeadDim] = lsum > 0.f ? sm.mfin[pend_ob][q] : -INFINITY;
              part[kHeadDim + 1] = lsum;
            }
          }
        }
        mbar_arrive(&sm.q_empty[pend_slot]);
        pend_ep = false;
        return true;
      };
      while (true) {
        if (!mbar_wait(&sm.kv_full[stage], phase, p.ctrl)) break;
        // everything this tile needs from its header, read now: once P is handed over, the PV
        // completes, the stage is released and the producer rewrites the header
        const int4 hw = *reinterpret_cast<const int4*>(&sm.hdr[stage][0]);
        const int item = hw.x;
        if (item < 0) break;
        const int tok0 = hw.y, nvalid = hw.z, flags = hw.w & 15, slot = hw.w >> 4;
        const int slot0 = sm.hdr[stage][kHdrSlot0 + (r >> box_shift)];
        const bool valid = r < nvalid && slot0 >= 0;
        if (flags & kFirst) {
          if (!mbar_wait(&sm.q_full[slot], qcount[slot] & 1, p.ctrl)) break;
          qcount[slot]++;
          ++nitem;
          item_first_tile = j;
          kvh = sm.iinfo[slot].kvh;
          rows_i = sm.iinfo[slot].rows;
          // spec mode: row q = rg R + q of the sequence (token (rg R + q) / G) sees key positions
          // <= mbase + token, i.e. position pos is visible to rows q >= (pos - mbase) G - rg R
          qrow_lo = p.spec_mode ? sm.iinfo[slot].mbase * G + sm.iinfo[slot].rg * R : 0;
  #pragma unroll
          for (int q = 0; q < RV; ++q) {
            m_ref[q] = -INFINITY;
            l_part[q] = 0.f;
            if constexpr (kRowRegs) cs_r[q] = sm.qscale[slot][q];
          }
        }
        float ks = 1.f, lv = 0.f;
        if ((kscaled || vscaled) && valid) {
          const int64_t idx = (static_cast<int64_t>(slot0) + (r & (p.box_rows - 1))) * p.num_kv_heads + kvh;
          if (kscaled) ks = __ldg(p.k_scale + idx);
          if (vscaled) lv = lg2(__ldg(p.v_scale + idx));
        }
        // ---------------------------------------------------- scores of this token row
        const int sb = j & 1;
        if (!mbar_wait(&sm.s_full[sb], (j >> 1) & 1, p.ctrl)) break;
        tc::fence_after_sync();
        float x[N];
  #pragma unroll
        for (int c = 0; c < N; c += 16) {
          float v16[16];
          tc::ld16(tmem + lane_base + sb * N + c, v16);
  #pragma unroll
          for (int i = 0; i < 16; ++i) x[c + i] = v16[i];
        }
        tc::wait_ld();
        tc::fence_before_sync();
        mbar_arrive(&sm.s_empty[sb]);
        const int pos = tok0 + r;
        // rows [qmin, rows_i) see this thread's key position (all live rows outside spec mode)
        const int qmin = !valid ? INT_MAX : (p.spec_mode ? pos * G - qrow_lo : INT_MIN);
        float xs[RV];  // score (log2 units) + log2 of the value scale: P's exponent
        bool over = false;  // a score the current reference cannot take (P would pass 256)
  #pragma unroll
        for (int q = 0; q < RV; ++q) {
          float csq;
          if constexpr (kRowRegs) {
            csq = cs_r[kRowRegs ? q : 0];
          } else {
            const float4 c4 = *reinterpret_cast<const float4*>(&sm.qscale[slot][q & ~3]);
            csq = (q & 3) == 0 ? c4.x : (q & 3) == 1 ? c4.y : (q & 3) == 2 ? c4.z : c4.w;
          }
          float sc = (x[q] + x[R + q]) * csq * ks;
          if (!(q >= qmin && q < rows_i)) sc = -INFINITY;
          xs[q] = sc + lv;
          over |= xs[q] > m_ref[q] + kRescaleLog2;
        }
        // one vote per warp; the exact per-row maxima are exchanged only when some warp needs a
        // new reference (an item's first tile, and rare growth after it)
        const bool wover = __any_sync(0xffffffffu, over);
        if (lane == 0) sm.vote[sb][warp] = wover ? 1 : 0;
        if (!sync()) break;
        const int4 votes = *reinterpret_cast<const int4*>(&sm.vote[sb][0]);
        uint32_t resc = 0;  // rows whose reference moved (uniform); factors in this warp's alpha row
        if (votes.x | votes.y | votes.z | votes.w) {
  #pragma unroll
          for (int q = 0; q < RV; ++q) {
            const int wm = __reduce_max_sync(0xffffffffu, f2ord(xs[q]));
            if (lane == 0) sm.red[sb][warp][q] = ord2f(wm);
          }
          if (!sync()) break;
  #pragma unroll
          for (int q = 0; q < RV; ++q) {
            const float tmax = fmaxf(fmaxf(sm.red[sb][0][q], sm.red[sb][1][q]),
                                     fmaxf(sm.red[sb][2][q], sm.red[sb][3][q]));
            if (tmax > m_ref[q] + kRescaleLog2) {
              const float a = m_ref[q] == -INFINITY ? 0.f : ex2(m_ref[q] - tmax);
              m_ref[q] = tmax;
              l_part[q] *= a;
              resc |= 1u << q;
              if (lane == 0) sm.alpha[warp][q] = a;
            }
          }
        }
        // ---------------------------------------------------- P and row sums
  #pragma unroll
        for (int q = 0; q < RV; ++q) {
          const float m_use = m_ref[q] == -INFINITY ? 0.f : m_ref[q];
          const float pe = kPScale * ex2(xs[q] - m_use);
          l_part[q] += vscaled ? kPScale * ex2(xs[q] - lv - m_use) : pe;
          xs[q] = pe;
        }
        // P^T row r: 2R bytes, hi rows then lo rows, as 16-byte planes of 16 columns
        uint32_t words[R / 2];
  #pragma unroll
        for (int w = 0; w < R / 2; ++w) words[w] = 0u;
  #pragma unroll
        for (int w = 0; w < RV / 4; ++w) {
          const uint32_t a = pack_f16x2(xs[4 * w], xs[4 * w + 1]);
          const uint32_t b = pack_f16x2(xs[4 * w + 2], xs[4 * w + 3]);
          uint32_t ah, al, bh, bl;
          split_f16x2_e4m3(a, ah, al);
          split_f16x2_e4m3(b, bh, bl);
          words[w] = ah | (bh << 16);
          words[R / 4 + w] = al | (bl << 16);
        }
        // O rescale (rare): O must be quiescent, i.e. the previous tile's PV done
        if (resc && j > item_first_tile) {
          __syncwarp();
          if (!wait_pv(j - 1)) break;
  #pragma unroll
          for (int c = 0; c < N; c += 16) {
            float o16[16];
            const uint32_t o_cur = o_base + ((nitem - 1) & 1) * N;
            tc::ld16(o_cur + c, o16);
            tc::wait_ld();
  #pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int q = (c + i) % R;
              if (q < RV && ((resc >> q) & 1u)) o16[i] *= sm.alpha[warp][q];
            }
            tc::st16(o_cur + c, o16);
          }
          tc::wait_st();
        }
        // P buffer sb was last read by PV_{j-2}
        if (j >= 2 && !wait_pv(j - 2)) break;
  #pragma unroll
        for (int plane = 0; plane < NT; ++plane)
          *reinterpret_cast<uint4*>(&sm.p2[sb][plane][r * 16]) =
              make_uint4(words[4 * plane], words[4 * plane + 1], words[4 * plane + 2], words[4 * plane + 3]);
        if (!valid) {  // masked rows may hold any bytes (NaN codes): zero V's row
          uint4* vrow = reinterpret_cast<uint4*>(&sm.v[stage][r * 128]);
  #pragma unroll
          for (int i = 0; i < 8; ++i) vrow[i] = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async_smem();
        tc::fence_before_sync();
        mbar_arrive(&sm.p_full[sb]);

        // the previous item's read-out (its sums were exchanged at this tile's barrier)
        if (pend_ep && !finish()) break;
        if (flags & kLast) {
          // park the item: per-warp row sums and the final maxima, read out one tile later
          const int ob = (nitem - 1) & 1;
  #pragma unroll
          for (int q = 0; q < RV; ++q) {
            float l = l_part[q];
  #pragma unroll
            for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
            if (lane == 0) sm.redl[ob][warp][q] = l;
            if (tid == 0) sm.mfin[ob][q] = m_ref[q];
          }
          pend_ep = true;
          pend_j = j;
          pend_ob = ob;
          pend_slot = slot;
          pend_item = item;
          if constexpr (NT > 1) {  // wide row groups: read out at once (registers are scarce)
            if (!sync() || !finish()) break;
          }
        }
        ++j;
        if (++stage == kStages) { stage = 0; phase ^= 1; }
      }
      // the last item's read-out (a barrier first: every warp has parked its sums)
      if (pend_ep && sync()) finish();
  
    } else {
      // ============================================================ softmax, wide row groups
      // NT > 1 (16 or 24 query rows per item): 8 warps.  Warp w owns token rows 32 (w & 3) .. + 31
      // of S^T (and dim rows of O^T: its tensor-memory lane quadrant) and the query rows
      // [h RH, (h + 1) RH) of the row group, h = w >> 2, so every thread handles RH = RV / 2 rows.
      // The two halves never exchange anything: each has its own 128-thread barrier, its own
      // rows' maxima, sums and read-out; they meet only on the tile barriers of the pipeline.
      constexpr int RH = RV / 2;
      static_assert(RH == 8 || RH == 12, "rows per half");
      const int quad = warp & 3, half = warp >> 2;
      const int qb = half * RH;  // this half's first row
      const int r = tid & 127;
      const uint32_t lane_base = static_cast<uint32_t>(32 * quad) << 16;
      const bool kscaled = p.k_scale != nullptr;
      const bool vscaled = p.v_scale != nullptr;
      const int box_shift = 31 - __clz(p.box_rows);
      constexpr float kRescaleLog2 = 4.f;  // P = 16 * 2^(s - m_ref) <= 256 < 448 (e4m3 max)
      constexpr float kPScale = 16.f;
      float m_ref[RH], l_part[RH];
      int rows_i = 0, qrow_lo = 0, kvh = 0;
      int stage = 0, j = 0, sync_uses = 0, item_first_tile = 0, nitem = 0;
      uint32_t phase = 0;
      int qcount[2] = {0, 0};
      auto sync = [&]() -> bool {  // the 128 threads of this half
        mbar_arrive(&sm.sync128[half]);
        return mbar_wait(&sm.sync128[half], (sync_uses++) & 1, p.ctrl);
      };
      auto wait_pv = [&](int t) -> bool {
        const int b = t & 1;
        if (!mbar_wait(&sm.pv_done[b], (t >> 1) & 1, p.ctrl)) return false;
        tc::fence_after_sync();
        return true;
      };
      // RH consecutive tensor-memory columns of this thread's lane: one 8-column access (RH = 8,
      // columns at multiples of 8) or three 4-column ones (RH = 12, columns at multiples of 4)
      auto ld_rows = [&](uint32_t taddr, float (&v)[RH]) {
        if constexpr (RH == 8) {
          tc::ld8(taddr, v);
        } else {
#pragma unroll
          for (int k = 0; k < RH / 4; ++k) {
            float a[4];
            tc::ld4(taddr + 4 * k, a);
#pragma unroll
            for (int i = 0; i < 4; ++i) v[4 * k + i] = a[i];
          }
        }
      };
      auto st_rows = [&](uint32_t taddr, const float (&v)[RH]) {
        if constexpr (RH == 8) {
          tc::st8(taddr, v);
        } else {
#pragma unroll
          for (int k = 0; k < RH / 4; ++k) {
            const float a[4] = {v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]};
            tc::st4(taddr + 4 * k, a);
          }
        }
      };
      const uint32_t o_base = tmem + lane_base + 2 * N;  // O of an item: o_base + (item parity) N
      while (true) {
        if (!mbar_wait(&sm.kv_full[stage], phase, p.ctrl)) break;
        const int4 hw = *reinterpret_cast<const int4*>(&sm.hdr[stage][0]);
        const int item = hw.x;
        if (item < 0) break;
        const int tok0 = hw.y, nvalid = hw.z, flags = hw.w & 15, slot = hw.w >> 4;
        const int slot0 = sm.hdr[stage][kHdrSlot0 + (r >> box_shift)];
        const bool valid = r < nvalid && slot0 >= 0;
        if (flags & kFirst) {
          if (!mbar_wait(&sm.q_full[slot], qcount[slot] & 1, p.ctrl)) break;
          qcount[slot]++;
          ++nitem;
          item_first_tile = j;
          kvh = sm.iinfo[slot].kvh;
          rows_i = sm.iinfo[slot].rows;
          qrow_lo = p.spec_mode ? sm.iinfo[slot].mbase * G + sm.iinfo[slot].rg * R : 0;
#pragma unroll
          for (int i = 0; i < RH; ++i) {
            m_ref[i] = -INFINITY;
            l_part[i] = 0.f;
          }
        }
        float ks = 1.f, lv = 0.f;
        if ((kscaled || vscaled) && valid) {
          const int64_t idx = (static_cast<int64_t>(slot0) + (r & (p.box_rows - 1))) * p.num_kv_heads + kvh;
          if (kscaled) ks = __ldg(p.k_scale + idx);
          if (vscaled) lv = lg2(__ldg(p.v_scale + idx));
        }
        // ---------------------------------------------------- scores of this half's rows
        const int sb = j & 1;
        if (!mbar_wait(&sm.s_full[sb], (j >> 1) & 1, p.ctrl)) break;
        tc::fence_after_sync();
        float xs[RH];
        {
          float xh[RH], xl[RH];
          ld_rows(tmem + lane_base + sb * N + qb, xh);
          ld_rows(tmem + lane_base + sb * N + R + qb, xl);
          tc::wait_ld();
          tc::fence_before_sync();
          mbar_arrive(&sm.s_empty[sb]);
          const int pos = tok0 + r;
          // rows [qmin, rows_i) see this thread's key position (all live rows outside spec mode)
          const int qmin = !valid ? INT_MAX : (p.spec_mode ? pos * G - qrow_lo : INT_MIN);
#pragma unroll
          for (int i = 0; i < RH; i += 4) {
            const float4 c4 = *reinterpret_cast<const float4*>(&sm.qscale[slot][qb + i]);
            const float cs4[4] = {c4.x, c4.y, c4.z, c4.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const int q = qb + i + k;
              float sc = (xh[i + k] + xl[i + k]) * cs4[k] * ks;
              if (!(q >= qmin && q < rows_i)) sc = -INFINITY;
              xs[i + k] = sc + lv;
            }
          }
        }
        bool over = false;  // a score the current reference cannot take (P would pass 256)
#pragma unroll
        for (int i = 0; i < RH; ++i) over |= xs[i] > m_ref[i] + kRescaleLog2;
        // one vote per warp; this half's exact per-row maxima are exchanged only when one of its
        // warps needs a new reference (an item's first tile, and rare growth after it)
        const bool wover = __any_sync(0xffffffffu, over);
        if (lane == 0) sm.vote[sb][warp] = wover ? 1 : 0;
        if (!sync()) break;
        const int4 votes = *reinterpret_cast<const int4*>(&sm.vote[sb][4 * half]);
        uint32_t resc = 0;  // this half's rows whose reference moved (bit i: row qb + i)
        if (votes.x | votes.y | votes.z | votes.w) {
#pragma unroll
          for (int i = 0; i < RH; ++i) {
            const int wm = __reduce_max_sync(0xffffffffu, f2ord(xs[i]));
            if (lane == 0) sm.red[sb][quad][qb + i] = ord2f(wm);
          }
          if (!sync()) break;
#pragma unroll
          for (int i = 0; i < RH; ++i) {
            const int q = qb + i;
            const float tmax = fmaxf(fmaxf(sm.red[sb][0][q], sm.red[sb][1][q]),
                                     fmaxf(sm.red[sb][2][q], sm.red[sb][3][q]));
            if (tmax > m_ref[i] + kRescaleLog2) {
              const float a = m_ref[i] == -INFINITY ? 0.f : ex2(m_ref[i] - tmax);
              m_ref[i] = tmax;
              l_part[i] *= a;
              resc |= 1u << i;
              if (lane == 0) sm.alpha[quad][q] = a;
            }
          }
        }
        // ---------------------------------------------------- P and row sums
#pragma unroll
        for (int i = 0; i < RH; ++i) {
          const float m_use = m_ref[i] == -INFINITY ? 0.f : m_ref[i];
          const float pe = kPScale * ex2(xs[i] - m_use);
          l_part[i] += vscaled ? kPScale * ex2(xs[i] - lv - m_use) : pe;
          xs[i] = pe;
        }
        uint32_t whi[RH / 4], wlo[RH / 4];  // this half's hi and lo bytes of P^T row r
#pragma unroll
        for (int w = 0; w < RH / 4; ++w) {
          const uint32_t a = pack_f16x2(xs[4 * w], xs[4 * w + 1]);
          const uint32_t b = pack_f16x2(xs[4 * w + 2], xs[4 * w + 3]);
          uint32_t ah, al, bh, bl;
          split_f16x2_e4m3(a, ah, al);
          split_f16x2_e4m3(b, bh, bl);
          whi[w] = ah | (bh << 16);
          wlo[w] = al | (bl << 16);
        }
        // O rescale (rare): O must be quiescent, i.e. the previous tile's PV done; this thread's
        // dim row, this half's hi and lo columns
        if (__any_sync(0xffffffffu, resc != 0) && j > item_first_tile) {
          if (!wait_pv(j - 1)) break;
          const uint32_t o_cur = o_base + ((nitem - 1) & 1) * N;
#pragma unroll
          for (int plane = 0; plane < 2; ++plane) {
            float o[RH];
            ld_rows(o_cur + plane * R + qb, o);
            tc::wait_ld();
#pragma unroll
            for (int i = 0; i < RH; ++i)
              if ((resc >> i) & 1u) o[i] *= sm.alpha[quad][qb + i];
            st_rows(o_cur + plane * R + qb, o);
          }
          tc::wait_st();
        }
        // P buffer sb was last read by PV_{j-2}
        if (j >= 2 && !wait_pv(j - 2)) break;
#pragma unroll
        for (int w = 0; w < RH / 4; ++w) {
          const int bh = qb + 4 * w, bl = R + qb + 4 * w;  // byte offsets in the 2R-byte row
          *reinterpret_cast<uint32_t*>(&sm.p2[sb][bh >> 4][r * 16 + (bh & 15)]) = whi[w];
          *reinterpret_cast<uint32_t*>(&sm.p2[sb][bl >> 4][r * 16 + (bl & 15)]) = wlo[w];
        }
        if (!valid && half == 0) {  // masked rows may hold any bytes (NaN codes): zero V's row
          uint4* vrow = reinterpret_cast<uint4*>(&sm.v[stage][r * 128]);
#pragma unroll
          for (int i = 0; i < 8; ++i) vrow[i] = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async_smem();
        tc::fence_before_sync();
        mbar_arrive(&sm.p_full[sb]);

        if (flags & kLast) {
          // the item's read-out, at once: this half's row sums (per quadrant) and final maxima,
          // a barrier, then its rows of O once the last PV is done
          const int ob = (nitem - 1) & 1;
#pragma unroll
          for (int i = 0; i < RH; ++i) {
            float l = l_part[i];
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
            if (lane == 0) sm.redl[ob][quad][qb + i] = l;
            if (r == 0) sm.mfin[ob][qb + i] = m_ref[i];
          }
          if (!sync() || !wait_pv(j)) break;
          const ItemInfo ii = sm.iinfo[slot];
          float oh[RH], ol[RH];
          ld_rows(o_base + ob * N + qb, oh);
          ld_rows(o_base + ob * N + R + qb, ol);
          tc::wait_ld();
          tc::fence_before_sync();
          const int d = r;  // output dim
#pragma unroll
          for (int i = 0; i < RH; ++i) {
            const int q = qb + i;
            if (q >= ii.rows) break;
            const float o = oh[i] + ol[i];
            const float lsum = sm.redl[ob][0][q] + sm.redl[ob][1][q] + sm.redl[ob][2][q] +
                               sm.redl[ob][3][q];
            if (ii.nchunks == 1) {
              const int rr = ii.rg * R + q;
              const int jj = rr / G, hh = ii.kvh * G + (rr - jj * G);
              __nv_bfloat16 v = out_round(o / fmaxf(lsum, 1e-10f));
              p.out[static_cast<int64_t>(ii.qrow0 + jj) * p.out_row_stride + hh * kHeadDim + d] =
                  *reinterpret_cast<uint16_t*>(&v);
            } else {
              float* part = p.partials + (static_cast<int64_t>(item) * R + q) * (kHeadDim + 4);
              part[d] = o;
              if (d == 0) {
                // a chunk whose rows saw no key position carries no weight in the combine
                part[kHeadDim] = lsum > 0.f ? sm.mfin[ob][q] : -INFINITY;
                part[kHeadDim + 1] = lsum;
              }
            }
          }
          mbar_arrive(&sm.q_empty[slot]);
        }
        ++j;
        if (++stage == kStages) { stage = 0; phase ^= 1; }
      }
    }
  }

  // ---------------------------------------------------------------- teardown
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == kMmaWarp) tc::tmem_dealloc(tmem, kTmemCols);
  if (tid == 0) release_work_counters(p.ctrl);
}

// Combines the split-KV partials of every (sequence, kv head, row group) with more than one
// chunk, using the plan the decode kernel published.  Single-plane engines (many chunks per
// pair): one warp per (pair, row), grid-strided.
// Partial rows hold O (unnormalised, 128 floats), then the reference max (log2 units) and the
// row sum.  Lane c takes the (max, sum) of chunks c, c + 32, ...: the row's largest max M comes
// from a warp reduction and chunk c's weight is 2^(m_c - M); lane l then accumulates output dims
// 4l .. 4l + 3 over the chunks (one 16-byte load per chunk, all independent), so a pair costs
// about two L2 round trips.  Launched as a programmatic dependent of the decode kernel: it waits
// for the decode grid before touching the partials.
constexpr int kCombineWarps = 8;
template <int NT>
__global__ void __launch_bounds__(32 * kCombineWarps)
    combine_rows_kernel(const DecodeParams p) {
  constexpr int R = 8 * NT;
  // a following decode launch may start its setup now; it waits for this grid before any read
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the decode grid has finished
  const int G = p.group;
  const int CT = p.plan[0];
  const int lane = threadIdx.x & 31;
  const int64_t nrows = static_cast<int64_t>(p.num_seqs) * p.num_kv_heads * p.max_rowgroups * R;
  const int64_t w0 = static_cast<int64_t>(blockIdx.x) * kCombineWarps + (threadIdx.x >> 5);
  const int64_t wstride = static_cast<int64_t>(gridDim.x) * kCombineWarps;
  for (int64_t w = w0; w < nrows; w += wstride) {
    const int64_t pi = w / R;
    const int q = static_cast<int>(w - pi * R);
    const int b = static_cast<int>(pi / (p.num_kv_heads * p.max_rowgroups));
    const int rem = static_cast<int>(pi - static_cast<int64_t>(b) * p.num_kv_heads * p.max_rowgroups);
    const int kvh = rem / p.max_rowgroups, rg = rem - kvh * p.max_rowgroups;
    int nq;
    const int L = seq_len_clamped(p, b, &nq);
    if (L <= 0) continue;
    const int nrg = (nq * G + R - 1) / R;
    const int nchunks = (L + CT - 1) / CT;
    if (rg >= nrg || nchunks <= 1 || q >= min(R, nq * G - rg * R)) continue;
    const int qrow0 = p.spec_mode ? __ldg(p.cu_q + b) : b;
    const int64_t first = p.plan[2 + b] + kvh * nrg + rg;
    const int64_t stride = static_cast<int64_t>(p.num_kv_heads) * nrg;
    auto part = [&](int c) -> const float* {
      return p.partials + ((first + c * stride) * R + q) * (kHeadDim + 4);
    };
    // the row's largest reference max over its chunks (-inf: no chunk saw a key position)
    float m_lane = -INFINITY;  // chunk `lane`'s max, kept for the common case of <= 32 chunks
    float M = -INFINITY;
    for (int c = lane; c < nchunks; c += 32) {
      const float m = __ldcg(part(c) + kHeadDim);
      if (c == lane) m_lane = m;
      M = fmaxf(M, m);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
    float lsum = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int c0 = 0; c0 < nchunks; c0 += 32) {
      const int c = c0 + lane;
      float wl = 0.f;
      if (c < nchunks) {
        const float m = c0 == 0 ? m_lane : __ldcg(part(c) + kHeadDim);
        wl = m == -INFINITY ? 0.f : ex2(m - M);
        lsum += wl * __ldcg(part(c) + kHeadDim + 1);
      }
      const int n = min(32, nchunks - c0);
#pragma unroll 4
      for (int i = 0; i < n; ++i) {
        const float wi = __shfl_sync(0xffffffffu, wl, i);
        const float4 o = __ldcg(reinterpret_cast<const float4*>(part(c0 + i)) + lane);
        acc.x += wi * o.x;
        acc.y += wi * o.y;
        acc.z += wi * o.z;
        acc.w += wi * o.w;
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, off);
    const float inv = 1.f / fmaxf(lsum, 1e-10f);
    const int rr = rg * R + q;
    const int jj = rr / G, hh = kvh * G + (rr - jj * G);
    const __nv_bfloat16 v0 = out_round(acc.x * inv), v1 = out_round(acc.y * inv);
    const __nv_bfloat16 v2 = out_round(acc.z * inv), v3 = out_round(acc.w * inv);
    // 2-byte stores: the output row stride carries no alignment guarantee beyond bf16
    uint16_t* dst = p.out + static_cast<int64_t>(qrow0 + jj) * p.out_row_stride + hh * kHeadDim + 4 * lane;
    dst[0] = *reinterpret_cast<const uint16_t*>(&v0);
    dst[1] = *reinterpret_cast<const uint16_t*>(&v1);
    dst[2] = *reinterpret_cast<const uint16_t*>(&v2);
    dst[3] = *reinterpret_cast<const uint16_t*>(&v3);
  }
}

// Wide engines' combine (few chunks per pair, many rows): one CTA per pair (grid-strided);
// thread = output dim.  Partial rows hold O (unnormalised, 128 floats), then the reference max (log2
// units) and the row sum.  Per pair: the (max, sum) of every (row, chunk) are gathered in parallel
// (per-row maxima by shared-memory atomics on order-preserving ints), their weights computed once,
// then each thread's partial-O loads are all independent.  Launched as a programmatic dependent
// of the decode kernel: it waits for the decode grid before touching the partials.
constexpr int kCombineSlots = 1024;  // (row, chunk) weights staged per round
template <int NT>
__global__ void __launch_bounds__(kHeadDim)
    combine_pairs_kernel(const DecodeParams p) {
  constexpr int R = 8 * NT;
  __shared__ int smax[R];
  __shared__ float ssum[R];
  __shared__ float swt[kCombineSlots];
  // a following decode launch may start its setup now; it waits for this grid before any read
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the decode grid has finished
  const int G = p.group;
  const int CT = p.plan[0];
  const int64_t npairs = static_cast<int64_t>(p.num_seqs) * p.num_kv_heads * p.max_rowgroups;
  const int d = threadIdx.x;
  for (int64_t pi = blockIdx.x; pi < npairs; pi += gridDim.x) {
    const int b = static_cast<int>(pi / (p.num_kv_heads * p.max_rowgroups));
    const int rem = static_cast<int>(pi - static_cast<int64_t>(b) * p.num_kv_heads * p.max_rowgroups);
    const int kvh = rem / p.max_rowgroups, rg = rem - kvh * p.max_rowgroups;
    int nq;
    const int L = seq_len_clamped(p, b, &nq);
    if (L <= 0) continue;
    const int nrg = (nq * G + R - 1) / R;
    const int nchunks = (L + CT - 1) / CT;
    if (rg >= nrg || nchunks <= 1) continue;
    const int qrow0 = p.spec_mode ? __ldg(p.cu_q + b) : b;
    const int rows = min(R, nq * G - rg * R);
    const int64_t first = p.plan[2 + b] + kvh * nrg + rg;
    const int64_t stride = static_cast<int64_t>(p.num_kv_heads) * nrg;
    auto part = [&](int q, int c) -> const float* {
      return p.partials + ((first + c * stride) * R + q) * (kHeadDim + 4);
    };
    if (d < R) { smax[d] = f2ord(-INFINITY); ssum[d] = 0.f; }
    __syncthreads();
    const int n = rows * nchunks;
    for (int i = d; i < n; i += kHeadDim) {
      const int q = i / nchunks, c = i - q * nchunks;
      atomicMax(&smax[q], f2ord(__ldcg(part(q, c) + kHeadDim)));
    }
    __syncthreads();
    float o[R];
#pragma unroll
    for (int q = 0; q < R; ++q) o[q] = 0.f;
    for (int base = 0; base < n; base += kCombineSlots) {
      const int m = min(kCombineSlots, n - base);
      for (int i = d; i < m; i += kHeadDim) {
        const int q = (base + i) / nchunks, c = (base + i) - q * nchunks;
        const float M = ord2f(smax[q]);
        const float* pr = part(q, c);
        const float w = ex2(__ldcg(pr + kHeadDim) - (M == -INFINITY ? 0.f : M));
        swt[i] = w;
        atomicAdd(&ssum[q], w * __ldcg(pr + kHeadDim + 1));
      }
      __syncthreads();
#pragma unroll
      for (int q = 0; q < R; ++q) {
        if (q >= rows) break;
        const int c0 = max(0, base - q * nchunks), c1 = min(nchunks, base + m - q * nchunks);
#pragma unroll 4
        for (int c = c0; c < c1; ++c) o[q] += swt[q * nchunks + c - base] * __ldcg(part(q, c) + d);
      }
      __syncthreads();
    }
#pragma unroll
    for (int q = 0; q < R; ++q) {
      if (q >= rows) break;
      const int rr = rg * R + q;
      const int jj = rr / G, hh = kvh * G + (rr - jj * G);
      __nv_bfloat16 v = out_round(o[q] / fmaxf(ssum[q], 1e-10f));
      p.out[static_cast<int64_t>(qrow0 + jj) * p.out_row_stride + hh * kHeadDim + d] =
          *reinterpret_cast<uint16_t*>(&v);
    }
    __syncthreads();
  }
}

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && cached[dev]) return cached[dev];
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (sms < 1) sms = 1;
  if (dev >= 0 && dev < 64) cached[dev] = sms;
  return sms;
}

template <int NT>
size_t decode_smem_bytes(int num_seqs, bool sampled) {
  // + alignment slack, + the per-launch plan arrays (prefix, info)
  constexpr int kThreads = Roles<NT>::kThreads;
  const int plan_ints = sampled ? 2 * kThreads + 1
                                : (NT > 1 && num_seqs <= kThreads ? 3 : 2) * num_seqs + 1;
  return sizeof(DecodeSmem<NT>) + 1024 + static_cast<size_t>(plan_ints) * sizeof(int);
}

using DecodeKernelFn = void (*)(CUtensorMap, CUtensorMap, DecodeParams);

struct DecodeShape {
  DecodeKernelFn fn;
  int grid;
  size_t smem;
};

// The launch of this batch: the per-sequence plan while the engine's CTAs per SM (two for the
// single-plane engines, one for the wide ones) still fit with it, else the sampled one; a
// persistent grid of as many CTAs as fit on every SM (at most kMaxCtasPerSm; tensor memory per
// CTA is at most 256 columns, so it never limits).
template <int NT, int RV>
DecodeShape decode_shape(int num_seqs) {
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaFuncSetAttribute(decode_kernel<NT, RV, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(decode_smem_bytes<NT>(kMaxSeqs, false)));
    cudaFuncSetAttribute(decode_kernel<NT, RV, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(decode_smem_bytes<NT>(0, true)));
    // all of the unified L1/shared storage as shared memory: two CTAs' rings must fit
    cudaFuncSetAttribute(decode_kernel<NT, RV, false>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    cudaFuncSetAttribute(decode_kernel<NT, RV, true>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    configured[dev] = true;
  }
  // The occupancy calculator reports 1 for every kernel that allocates tensor memory, so the
  // CTAs per SM are counted from the resources themselves: shared memory (with the per-block
  // reservation) and registers.  Tensor memory (at most 256 of 512 columns per CTA) never limits.
  // Were fewer CTAs resident, the extra ones would find the work counter exhausted and leave.
  int smem_sm = 0, resv = 0;
  cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
  cudaDeviceGetAttribute(&resv, cudaDevAttrReservedSharedMemoryPerBlock, dev);
  const bool sampled = static_cast<int>(decode_smem_bytes<NT>(num_seqs, false)) + resv >
                       smem_sm / (NT == 1 ? kMaxCtasPerSm : 1);
  DecodeShape sh;
  sh.fn = sampled ? decode_kernel<NT, RV, true> : decode_kernel<NT, RV, false>;
  sh.smem = decode_smem_bytes<NT>(num_seqs, sampled);
  cudaFuncAttributes fa;
  cudaFuncGetAttributes(&fa, sh.fn);
  const int per_cta_smem = static_cast<int>(sh.smem) + resv;
  int occ = per_cta_smem > 0 ? smem_sm / per_cta_smem : 1;
  const int by_regs = fa.numRegs > 0 ? 65536 / (fa.numRegs * Roles<NT>::kThreads) : 1;
  occ = occ < by_regs ? occ : by_regs;
  occ = occ < 1 ? 1 : (occ > kMaxCtasPerSm ? kMaxCtasPerSm : occ);
  sh.grid = sm_count() * occ;
  return sh;
}

}  // namespace

int decode_grid(int nt) {
  (void)nt;
  return sm_count() * kMaxCtasPerSm;  // upper bound of any launch's grid (workspace sizing)
}

int decode_launch_grid(int nt, int rv, int num_seqs) {
  switch (nt) {
    case 1: return (rv <= 4 ? decode_shape<1, 4>(num_seqs) : decode_shape<1, 8>(num_seqs)).grid;
    case 2: return decode_shape<2, 16>(num_seqs).grid;
    default: return decode_shape<3, 24>(num_seqs).grid;
  }
}

int64_t decode_max_items(int64_t pairs, int grid) {
  return static_cast<int64_t>(kItemsPerCta) * grid + pairs;
}

int64_t decode_workspace_bytes(int num_seqs, int num_kv_heads, int max_rowgroups, int rows,
                               int grid) {
  const int64_t pairs = static_cast<int64_t>(num_seqs) * num_kv_heads * max_rowgroups;
  int64_t bytes = kCtrlInts * 4 + kPlanInts * 4;
  bytes += decode_max_items(pairs, grid) * rows * (kHeadDim + 4) * 4;
  return bytes;
}

namespace {
template <int NT, int RV>
void launch_variant(const DecodeParams& p, const CUtensorMap& tmk, const CUtensorMap& tmv,
                    int cgrid, cudaStream_t stream) {
  const DecodeShape sh = decode_shape<NT, RV>(p.num_seqs);
  // programmatic dependent launch: the CTAs' setup (barriers, tensor memory) overlaps the tail of
  // the previous kernel; the kernel waits for it (griddepcontrol.wait) before reading any input
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t dcfg = {};
  dcfg.gridDim = dim3(sh.grid);
  dcfg.blockDim = dim3(Roles<NT>::kThreads);
  dcfg.dynamicSmemBytes = sh.smem;
  dcfg.stream = stream;
  dcfg.attrs = attr;
  dcfg.numAttrs = 1;
  cudaLaunchKernelEx(&dcfg, sh.fn, tmk, tmv, p);
  if (cgrid > 0) {
    // programmatic dependent launch: the combine CTAs may be scheduled as decode CTAs retire;
    // each waits (griddepcontrol.wait) for the whole decode grid before reading the partials
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cgrid);
    cfg.blockDim = dim3(NT == 1 ? 32 * kCombineWarps : kHeadDim);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if constexpr (NT == 1) cudaLaunchKernelEx(&cfg, combine_rows_kernel<NT>, p);
    else cudaLaunchKernelEx(&cfg, combine_pairs_kernel<NT>, p);
  }
}
}  // namespace

cudaError_t launch_decode(const DecodeParams& p, int nt, int rv, const CUtensorMap& tmk,
                          const CUtensorMap& tmv, cudaStream_t stream) {
  const int64_t pairs = static_cast<int64_t>(p.num_seqs) * p.num_kv_heads * p.max_rowgroups;
  // combine CTAs, at most 16 per SM: single-plane engines one warp per (pair, row),
  // kCombineWarps per CTA; wide engines one CTA per pair
  const int64_t cblocks = nt == 1 ? (pairs * decode_rows(nt) + kCombineWarps - 1) / kCombineWarps
                                  : pairs;
  const int cgrid = static_cast<int>(cblocks < 16LL * sm_count() ? cblocks : 16LL * sm_count());
  switch (nt) {
    case 1:
      if (rv <= 4) launch_variant<1, 4>(p, tmk, tmv, cgrid, stream);
      else launch_variant<1, 8>(p, tmk, tmv, cgrid, stream);
      break;
    case 2: launch_variant<2, 16>(p, tmk, tmv, cgrid, stream); break;
    default: launch_variant<3, 24>(p, tmk, tmv, cgrid, stream); break;
  }
  return cudaGetLastError();
}

}  // namespace fp8attn
