// Split-KV paged decode engine (HBM-bound).
//
// Replaces fp8_paged_attention_decode_kernel (nanovllm/kernels/fp8_attention.py:88-171) and,
// inside the prefill entry point, serves the short query sequences of speculative verification
// (1 + k rows per sequence, causal among themselves).
//
// Work decomposition.  A work item is (sequence, kv head, row group, chunk of key positions).
// A row group is up to ROWS = 8*NT query rows that share one kv head (GQA: the group's q heads,
// times the sequence's query tokens in spec mode), so each K/V byte is loaded from HBM once per
// row group -- once in total for decode, where all q heads of a kv head fit one group.  Every CTA
// first computes the same plan from the sequence lengths (chunk size, item prefix sums in shared
// memory); then a persistent grid pulls items from an atomic counter.  Chunks of one
// (sequence, kv head, row group) are consecutive items, so the split-KV partial results are
// combined by whichever CTA finishes the pair's last chunk (atomic ticket), with no second
// launch and no spinning.
//
// CTA = 4 consumer warps + 1 producer warp.  The producer walks the items, looks block ids up in
// block_tables and issues TMA loads of 64-token K and V tiles (128-byte rows, 128B swizzle) into
// a STAGES-deep ring, plus a 1-D bulk copy of the item's query rows.  Each consumer warp takes
// 16 of the 64 tokens of a tile:
//   S^T[16 tok x 8 rows] = K[16 x 128] . Q^T   mma.sync m16n8k16, K dequantised e4m3 -> f16 in
//                                              registers (exact), Q bf16 -> f16
//   online softmax per query row (exp2 domain), P^T moved into B-fragment layout by movmatrix
//   O^T[128 dims x 8 rows] += V^T . P^T        V transposed in registers by byte permutes
// The contraction index permutations (dims inside QK, output dims inside PV) are chosen so every
// shared-memory read is a conflict-free 16-byte load; outputs are un-permuted at the store.
#include <climits>

#include "common.cuh"
#include "kernels.h"

namespace fp8attn {
namespace {

constexpr int kTile = 64;            // tokens per pipeline stage
constexpr int kConsumerWarps = 4;
constexpr int kDecodeThreads = (kConsumerWarps + 1) * 32;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kMaxBoxes = kTile / 16;

enum : int { kFirst = 1, kLast = 2 };

struct StageHeader {
  int item;  // < 0: no more work
  int seq, kvh, rg;
  int tok0;    // key position of the tile's first row
  int nvalid;  // rows of the tile inside the chunk
  int flags;
  int nchunks;
  int pair_first;  // item id of the pair's chunk 0
  int nq;
  int qrow0;  // first query token row of the sequence
  int rows;   // valid query rows in this row group
  int qslot;
  int lim_base;  // causal limit of the row group's token 0: key positions <= lim_base + j
  int blk[kMaxBoxes];  // physical block of each box (-1: invalid)
};

template <int NT>
struct DecodeCfg {
  static constexpr int ROWS = 8 * NT;
  static constexpr int STAGES = NT == 1 ? 4 : 3;
};

template <int NT>
struct __align__(1024) DecodeSmem {
  static constexpr int ROWS = DecodeCfg<NT>::ROWS;
  static constexpr int STAGES = DecodeCfg<NT>::STAGES;
  uint8_t k[STAGES][kTile * kHeadDim];  // each stage 1024-aligned (8 KB)
  uint8_t v[STAGES][kTile * kHeadDim];
  uint16_t qbuf[2][ROWS][kHeadDim];  // bf16 query rows, double-buffered by item
  float mrg_o[kConsumerWarps][ROWS][kHeadDim + 4];
  float mrg_m[kConsumerWarps][ROWS];
  float mrg_l[kConsumerWarps][ROWS];
  int prefix[kMaxSeqs + 1];  // item prefix sums over sequences
  int info[kMaxSeqs];        // (L << 7) | rowgroups, per sequence
  StageHeader hdr[STAGES];
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t qempty[2];
  int scratch[8];
};

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

// Block-wide exclusive scan of one int per thread (all kDecodeThreads threads participate).
__device__ __forceinline__ int block_exclusive_scan(int v, int* smem8, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) smem8[warp] = x;
  __syncthreads();
  int base = 0, tot = 0;
#pragma unroll
  for (int w = 0; w < kDecodeThreads / 32; ++w) {
    const int s = smem8[w];
    if (w < warp) base += s;
    tot += s;
  }
  __syncthreads();
  *total = tot;
  return base + x - v;
}

template <int NT>
__global__ void __launch_bounds__(kDecodeThreads, NT == 1 ? 2 : 2)
    decode_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                  const DecodeParams p) {
  using Smem = DecodeSmem<NT>;
  constexpr int ROWS = Smem::ROWS;
  constexpr int STAGES = Smem::STAGES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int G = p.group;
  const int B = p.num_seqs;

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], kConsumerWarps);
    }
    mbar_init(&sm.qempty[0], kConsumerWarps);
    mbar_init(&sm.qempty[1], kConsumerWarps);
    fence_mbar_init();
  }
  if (warp == kConsumerWarps && lane == 0) {
    prefetch_tensormap(&tmk);
    prefetch_tensormap(&tmv);
  }

  // ---------------------------------------------------------------- plan (every CTA, same result)
  // Each thread owns a contiguous run of sequences.
  const int per = (B + kDecodeThreads - 1) / kDecodeThreads;
  const int s0 = min(B, tid * per), s1 = min(B, s0 + per);
  const int max_rows_pass = ROWS;
  long long my_work = 0;
  for (int b = s0; b < s1; ++b) {
    int nq;
    const int L = seq_len_clamped(p, b, &nq);
    const int rows = nq * G;
    const int rg = L > 0 ? (rows + max_rows_pass - 1) / max_rows_pass : 0;
    sm.info[b] = (L << 7) | rg;
    my_work += static_cast<long long>(L) * rg;
  }
  // total key-position passes (x kv heads) -> chunk size targeting ~32 items per CTA
  __shared__ unsigned long long s_total;
  if (tid == 0) s_total = 0;
  __syncthreads();
  if (my_work) atomicAdd(&s_total, static_cast<unsigned long long>(my_work));
  __syncthreads();
  const unsigned long long total_work = s_total * static_cast<unsigned long long>(p.num_kv_heads);
  const unsigned long long target = 32ull * gridDim.x;
  long long ct = static_cast<long long>((total_work + target - 1) / target);
  ct = (ct + kTile - 1) / kTile * kTile;
  if (ct < p.min_chunk) ct = p.min_chunk;
  const int CT = static_cast<int>(ct > (1 << 24) ? (1 << 24) : ct);

  int my_items = 0;
  for (int b = s0; b < s1; ++b) {
    const int inf = sm.info[b];
    const int L = inf >> 7, rg = inf & 127;
    my_items += ((L + CT - 1) / CT) * p.num_kv_heads * rg;
  }
  int total_items;
  const int base = block_exclusive_scan(my_items, sm.scratch, &total_items);
  {
    int acc = base;
    for (int b = s0; b < s1; ++b) {
      sm.prefix[b] = acc;
      const int inf = sm.info[b];
      const int L = inf >> 7, rg = inf & 127;
      acc += ((L + CT - 1) / CT) * p.num_kv_heads * rg;
    }
    if (tid == kDecodeThreads - 1) sm.prefix[B] = total_items;
  }
  __syncthreads();
  // partial results are indexed by item id; a workspace sized by decode_workspace_bytes always
  // has room, anything else is reported instead of overrunning it
  const bool fits = total_items <= p.max_items;
  if (!fits && tid == 0 && blockIdx.x == 0) atomicExch(p.ctrl, kDevErrWorkspace);

  if (!fits) {
    // nothing to do
  } else if (warp == kConsumerWarps) {
    // ============================================================ producer warp
    int stage = 0;
    uint32_t phase = 0;
    int nth = 0;  // items taken by this CTA
    int item = 0;
    if (lane == 0) item = atomicAdd(p.ctrl + 1, 1);
    item = __shfl_sync(0xffffffffu, item, 0);
    bool ok = true;
    while (ok && item < total_items) {
      int nxt = 0;
      if (lane == 0) nxt = atomicAdd(p.ctrl + 1, 1);
      // locate the sequence: largest b with prefix[b] <= item
      int lo = 0, hi = B - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (sm.prefix[mid] <= item) lo = mid; else hi = mid - 1;
      }
      const int b = lo;
      const int inf = sm.info[b];
      const int L = inf >> 7, nrg = inf & 127;
      const int nchunks = (L + CT - 1) / CT;
      const int r = item - sm.prefix[b];
      const int pair_local = r / nchunks;
      const int c = r - pair_local * nchunks;
      const int kvh = pair_local / nrg;
      const int rg = pair_local - kvh * nrg;
      int nq = 1, qrow0 = b, lim_base = INT_MAX / 2;
      if (p.spec_mode) {
        qrow0 = __ldg(p.cu_q + b);
        nq = __ldg(p.cu_q + b + 1) - qrow0;
        const int nk = __ldg(p.cu_k + b + 1) - __ldg(p.cu_k + b);
        lim_base = nk - nq;
      }
      const int rows_total = nq * G;
      const int row0 = rg * ROWS;
      const int rows = min(ROWS, rows_total - row0);
      const int t0 = c * CT;
      const int t1 = min(L, t0 + CT);
      const int qslot = nth & 1;
      const uint32_t qbytes = static_cast<uint32_t>(rows) * kHeadDim * 2;

      // the item's query rows go into qbuf[qslot] once the consumers released it
      if (!mbar_wait(&sm.qempty[qslot], ((nth >> 1) & 1) ^ 1, p.ctrl)) { ok = false; break; }

      int ebase = INT_MIN / 2, myent = -1;
      const int64_t bt_row = static_cast<int64_t>(b) * p.bt_stride;
      for (int t = t0; t < t1 && ok; t += kTile) {
        if (!mbar_wait(&sm.empty[stage], phase ^ 1, p.ctrl)) { ok = false; break; }
        const int nvalid = min(kTile, t1 - t);
        const int nbox = (nvalid + p.box_rows - 1) / p.box_rows;
        int blks[kMaxBoxes];
#pragma unroll
        for (int j = 0; j < kMaxBoxes; ++j) {
          blks[j] = -1;
          if (j < nbox) {
            const int pos = t + j * p.box_rows;
            const int e = pos / p.block_size;
            if (e < ebase || e >= ebase + 32) {
              ebase = e;
              const int idx = ebase + lane;
              myent = idx < p.max_blocks ? __ldg(p.block_tables + bt_row + idx) : -1;
            }
            int blk = __shfl_sync(0xffffffffu, myent, e - ebase);
            if (blk < 0 || blk >= p.num_blocks) blk = -1;
            blks[j] = blk;
          }
        }
        if (lane == 0) {
          StageHeader& h = sm.hdr[stage];
          h.item = item;
          h.seq = b;
          h.kvh = kvh;
          h.rg = rg;
          h.tok0 = t;
          h.nvalid = nvalid;
          h.flags = (t == t0 ? kFirst : 0) | (t + kTile >= t1 ? kLast : 0);
          h.nchunks = nchunks;
          h.pair_first = item - c;
          h.nq = nq;
          h.qrow0 = qrow0;
          h.rows = rows;
          h.qslot = qslot;
          h.lim_base = lim_base + (p.spec_mode ? row0 / G : 0);
#pragma unroll
          for (int j = 0; j < kMaxBoxes; ++j) h.blk[j] = blks[j];
          uint32_t bytes = 0;
#pragma unroll
          for (int j = 0; j < kMaxBoxes; ++j)
            if (blks[j] >= 0) bytes += 2u * p.box_rows * kHeadDim;
          if (t == t0) bytes += qbytes;
          mbar_arrive_expect_tx(&sm.full[stage], bytes);
#pragma unroll
          for (int j = 0; j < kMaxBoxes; ++j) {
            if (blks[j] >= 0) {
              const int pos = t + j * p.box_rows;
              const int y = blks[j] * p.block_size + (pos % p.block_size);
              const int x = kvh * kHeadDim;
              tma_load_2d(&sm.k[stage][j * p.box_rows * kHeadDim], &tmk, &sm.full[stage], x, y);
              tma_load_2d(&sm.v[stage][j * p.box_rows * kHeadDim], &tmv, &sm.full[stage], x, y);
            }
          }
          if (t == t0) {
            // query rows row0 .. row0+rows-1: row r is (token r / G, head kvh*G + r % G); rows
            // of one token are contiguous in q
            int r = row0;
            while (r < row0 + rows) {
              const int j = r / G;
              const int g = r - j * G;
              const int run = min(G - g, row0 + rows - r);
              const uint16_t* src = p.q + static_cast<int64_t>(qrow0 + j) * p.q_row_stride +
                                    static_cast<int64_t>(kvh * G + g) * kHeadDim;
              bulk_load(&sm.qbuf[qslot][r - row0][0], src, run * kHeadDim * 2, &sm.full[stage]);
              r += run;
            }
          }
        }
        __syncwarp();
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
      ++nth;
      item = __shfl_sync(0xffffffffu, nxt, 0);
    }
    // termination marker
    if (ok && mbar_wait(&sm.empty[stage], phase ^ 1, p.ctrl)) {
      if (lane == 0) {
        sm.hdr[stage].item = -1;
        mbar_arrive(&sm.full[stage]);
      }
    } else if (lane == 0) {
      // timed out: still release the consumers so they can leave
      sm.hdr[stage].item = -1;
      mbar_arrive(&sm.full[stage]);
    }
  } else {
    // ============================================================ consumer warps
    const int g = lane >> 2, t = lane & 3;
    // zero outputs of routed sequences that have no key positions (reference: acc/max(s,1e-10))
    for (int b = blockIdx.x; b < B; b += gridDim.x) {
      const int inf = sm.info[b];
      if ((inf >> 7) != 0) continue;
      int nq = 1, qrow0 = b;
      if (p.spec_mode) {
        qrow0 = __ldg(p.cu_q + b);
        nq = __ldg(p.cu_q + b + 1) - qrow0;
        if (nq < 1 || nq > p.spec_q_max) continue;
      }
      const int per_row = p.num_heads * kHeadDim / 8;  // uint4 per token row
      for (int j = 0; j < nq; ++j) {
        uint4* dst = reinterpret_cast<uint4*>(p.out + static_cast<int64_t>(qrow0 + j) * p.out_row_stride);
        for (int i = tid; i < per_row; i += kConsumerThreads) dst[i] = make_uint4(0, 0, 0, 0);
      }
    }

    uint32_t qf[NT][2][4][2];  // Q B-fragments [n-tile][chunk half][word][b0b1 / b2b3]
    float o[8][NT][4];         // O^T accumulators [m-tile][n-tile][c0..c3]
    float m_run[NT][2], l_run[NT][2];
    int lim[NT][2];

    int stage = 0;
    uint32_t phase = 0;
    while (true) {
      if (!mbar_wait(&sm.full[stage], phase, p.ctrl)) break;
      const StageHeader h = sm.hdr[stage];
      if (h.item < 0) break;
      const uint32_t kbase = smem_u32(&sm.k[stage][0]);
      const uint32_t vbase = smem_u32(&sm.v[stage][0]);

      if (h.flags & kFirst) {
        // query fragments: n-tile nt row (8nt + g), physical dims [32t, 32t + 32)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const int row = 8 * nt + g;
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            uint4 a = make_uint4(0, 0, 0, 0), bq = make_uint4(0, 0, 0, 0);
            if (row < h.rows) {
              const uint4* src = reinterpret_cast<const uint4*>(&sm.qbuf[h.qslot][row][16 * (2 * t + hh)]);
              a = src[0];
              bq = src[1];
            }
            const uint32_t wv[8] = {a.x, a.y, a.z, a.w, bq.x, bq.y, bq.z, bq.w};
#pragma unroll
            for (int w = 0; w < 4; ++w) {
              qf[nt][hh][w][0] = bf16x2_to_f16x2(wv[2 * w]);      // dims 4w+0, 4w+1
              qf[nt][hh][w][1] = bf16x2_to_f16x2(wv[2 * w + 1]);  // dims 4w+2, 4w+3
            }
          }
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int col = 8 * nt + 2 * t + e;
            lim[nt][e] = col < h.rows ? (p.spec_mode ? h.lim_base + (col + (h.rg * ROWS) % G) / G
                                                      : INT_MAX)
                                      : -1;
            m_run[nt][e] = -INFINITY;
            l_run[nt][e] = 0.f;
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.qempty[h.qslot]);
#pragma unroll
        for (int mt = 0; mt < 8; ++mt)
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int i = 0; i < 4; ++i) o[mt][nt][i] = 0.f;
      }

      const int slice0 = warp * 16;  // my 16 rows of the tile
      if (slice0 < h.nvalid) {
        // ------------------------------------------------ S^T = K . Q^T
        float s[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
        const int rk = slice0 + g;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int cchunk = 2 * t + hh;
          const uint4 k0 = ld_shared_v4(kbase + rk * 128 + ((cchunk ^ g) << 4));
          const uint4 k1 = ld_shared_v4(kbase + (rk + 8) * 128 + ((cchunk ^ g) << 4));
          const uint32_t w0[4] = {k0.x, k0.y, k0.z, k0.w};
          const uint32_t w1[4] = {k1.x, k1.y, k1.z, k1.w};
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            uint32_t a[4];
            a[0] = e4m3x2_to_f16x2(w0[w]);        // row g,   dims 4w+0..1
            a[1] = e4m3x2_to_f16x2(w1[w]);        // row g+8, dims 4w+0..1
            a[2] = e4m3x2_to_f16x2(w0[w] >> 16);  // row g,   dims 4w+2..3
            a[3] = e4m3x2_to_f16x2(w1[w] >> 16);  // row g+8, dims 4w+2..3
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) mma_f16_16816(s[nt], a, qf[nt][hh][w][0], qf[nt][hh][w][1]);
          }
        }
        // ------------------------------------------------ scales, masks, online softmax
        const int box_lo = (slice0 + g) / p.box_rows, box_hi = (slice0 + g + 8) / p.box_rows;
        const bool vlo = (slice0 + g) < h.nvalid && h.blk[box_lo] >= 0;
        const bool vhi = (slice0 + g + 8) < h.nvalid && h.blk[box_hi] >= 0;
        const int pos_lo = h.tok0 + slice0 + g, pos_hi = pos_lo + 8;
        float ks_lo = 1.f, ks_hi = 1.f;
        if (p.k_scale != nullptr) {
          if (vlo) ks_lo = __ldg(p.k_scale + (static_cast<int64_t>(h.blk[box_lo]) * p.block_size + pos_lo % p.block_size) * p.num_kv_heads + h.kvh);
          if (vhi) ks_hi = __ldg(p.k_scale + (static_cast<int64_t>(h.blk[box_hi]) * p.block_size + pos_hi % p.block_size) * p.num_kv_heads + h.kvh);
        }
        float pf[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            float xl = s[nt][e] * ks_lo * p.scale_log2;
            float xh = s[nt][2 + e] * ks_hi * p.scale_log2;
            if (!(vlo && pos_lo <= lim[nt][e])) xl = -INFINITY;
            if (!(vhi && pos_hi <= lim[nt][e])) xh = -INFINITY;
            float mx = fmaxf(xl, xh);
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
            const float m_new = fmaxf(m_run[nt][e], mx);
            const float m_use = m_new == -INFINITY ? 0.f : m_new;
            const float alpha = ex2(m_run[nt][e] - m_use);
            const float pl = ex2(xl - m_use), ph = ex2(xh - m_use);
            l_run[nt][e] = l_run[nt][e] * alpha + pl + ph;
            m_run[nt][e] = m_new;
            pf[nt][e] = pl;
            pf[nt][2 + e] = ph;
#pragma unroll
            for (int mt = 0; mt < 8; ++mt) {
              o[mt][nt][e] *= alpha;
              o[mt][nt][2 + e] *= alpha;
            }
          }
        }
        // P^T as B fragments (tokens 2t,2t+1 | 2t+8,2t+9 for row g)
        uint32_t pb[NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          pb[nt][0] = movmatrix_trans(pack_f16x2(pf[nt][0], pf[nt][1]));
          pb[nt][1] = movmatrix_trans(pack_f16x2(pf[nt][2], pf[nt][3]));
        }
        // ------------------------------------------------ O^T += V^T . P^T
        const int vt[4] = {slice0 + 2 * t, slice0 + 2 * t + 1, slice0 + 2 * t + 8, slice0 + 2 * t + 9};
        uint4 vw[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          vw[i] = ld_shared_v4(vbase + vt[i] * 128 + ((g ^ (vt[i] & 7)) << 4));
          const bool ok = vt[i] < h.nvalid && h.blk[vt[i] / p.box_rows] >= 0;
          if (!ok) vw[i] = make_uint4(0, 0, 0, 0);  // masked rows may hold any bytes (NaN codes)
        }
        uint32_t vsc[2] = {0x3C003C00u, 0x3C003C00u};  // f16x2 scales (1.0) for tokens (2t,2t+1), (2t+8,2t+9)
        if (p.v_scale != nullptr) {
          float f[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            f[i] = 0.f;
            const int bi = vt[i] / p.box_rows;
            if (vt[i] < h.nvalid && h.blk[bi] >= 0) {
              const int pos = h.tok0 + vt[i];
              f[i] = __ldg(p.v_scale + (static_cast<int64_t>(h.blk[bi]) * p.block_size + pos % p.block_size) * p.num_kv_heads + h.kvh);
            }
          }
          vsc[0] = pack_f16x2(f[0], f[1]);
          vsc[1] = pack_f16x2(f[2], f[3]);
        }
        const uint32_t W[4][4] = {{vw[0].x, vw[0].y, vw[0].z, vw[0].w},
                                  {vw[1].x, vw[1].y, vw[1].z, vw[1].w},
                                  {vw[2].x, vw[2].y, vw[2].z, vw[2].w},
                                  {vw[3].x, vw[3].y, vw[3].z, vw[3].w}};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          // 4x4 byte transpose: T[j] = dim (16g + 4i + j) of tokens (2t, 2t+1, 2t+8, 2t+9)
          const uint32_t x0 = prmt(W[0][i], W[1][i], 0x5140);
          const uint32_t x1 = prmt(W[0][i], W[1][i], 0x7362);
          const uint32_t y0 = prmt(W[2][i], W[3][i], 0x5140);
          const uint32_t y1 = prmt(W[2][i], W[3][i], 0x7362);
          const uint32_t T0 = prmt(x0, y0, 0x5410), T1 = prmt(x0, y0, 0x7632);
          const uint32_t T2 = prmt(x1, y1, 0x5410), T3 = prmt(x1, y1, 0x7632);
          uint32_t a0[4] = {e4m3x2_to_f16x2(T0), e4m3x2_to_f16x2(T1), e4m3x2_to_f16x2(T0 >> 16),
                            e4m3x2_to_f16x2(T1 >> 16)};
          uint32_t a1[4] = {e4m3x2_to_f16x2(T2), e4m3x2_to_f16x2(T3), e4m3x2_to_f16x2(T2 >> 16),
                            e4m3x2_to_f16x2(T3 >> 16)};
          if (p.v_scale != nullptr) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint32_t sc = (j < 2) ? vsc[0] : vsc[1];
              __half2 x = *reinterpret_cast<__half2*>(&a0[j]);
              __half2 y = *reinterpret_cast<__half2*>(&a1[j]);
              const __half2 s2 = *reinterpret_cast<const __half2*>(&sc);
              x = __hmul2(x, s2);
              y = __hmul2(y, s2);
              a0[j] = *reinterpret_cast<uint32_t*>(&x);
              a1[j] = *reinterpret_cast<uint32_t*>(&y);
            }
          }
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            mma_f16_16816(o[2 * i][nt], a0, pb[nt][0], pb[nt][1]);
            mma_f16_16816(o[2 * i + 1][nt], a1, pb[nt][0], pb[nt][1]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.empty[stage]);
      if (++stage == STAGES) { stage = 0; phase ^= 1; }

      if (h.flags & kLast) {
        // ------------------------------------------------ merge the 4 warps' partial states
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            float l = l_run[nt][e];
            l += __shfl_xor_sync(0xffffffffu, l, 4);
            l += __shfl_xor_sync(0xffffffffu, l, 8);
            l += __shfl_xor_sync(0xffffffffu, l, 16);
            if (g == 0) {
              sm.mrg_m[warp][8 * nt + 2 * t + e] = m_run[nt][e];
              sm.mrg_l[warp][8 * nt + 2 * t + e] = l;
            }
          }
#pragma unroll
        for (int mt = 0; mt < 8; ++mt)
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              // m-tile mt = 2*ii + jh, row g (+8 if i >= 2) -> dim 16g + 4ii + 2jh + jl
              // stored at k*8 + g (k = dim % 16, g = dim / 16): conflict-free for these writes
              // and for the per-thread reads below
              const int ii = mt >> 1, jh = mt & 1, jl = i >> 1;
              const int kk = 4 * ii + 2 * jh + jl;
              const int col = 8 * nt + 2 * t + (i & 1);
              sm.mrg_o[warp][col][kk * 8 + g] = o[mt][nt][i];
            }
        named_barrier(1, kConsumerThreads);
        const int d = tid;  // consumer thread = permuted dim slot; real dim below
        const int dim_real = 16 * (d & 7) + (d >> 3);
        const bool direct = h.nchunks == 1;
        for (int col = 0; col < h.rows; ++col) {
          float M = -INFINITY;
#pragma unroll
          for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, sm.mrg_m[w][col]);
          const float Mu = M == -INFINITY ? 0.f : M;
          float L = 0.f, O = 0.f;
#pragma unroll
          for (int w = 0; w < kConsumerWarps; ++w) {
            const float wt = ex2(sm.mrg_m[w][col] - Mu);
            L += wt * sm.mrg_l[w][col];
            O += wt * sm.mrg_o[w][col][d];
          }
          if (direct) {
            const int r = h.rg * ROWS + col;
            const int j = r / G, hh = h.kvh * G + (r - j * G);
            __nv_bfloat16 v = out_round(O / fmaxf(L, 1e-10f));
            p.out[static_cast<int64_t>(h.qrow0 + j) * p.out_row_stride + hh * kHeadDim + dim_real] =
                *reinterpret_cast<uint16_t*>(&v);
          } else {
            float* part = p.partials + (static_cast<int64_t>(h.item) * ROWS + col) * (kHeadDim + 2);
            part[d] = O;
            if (d == 0) {
              part[kHeadDim] = M;
              part[kHeadDim + 1] = L;
            }
          }
        }
        if (!direct) {
          __threadfence();
          named_barrier(1, kConsumerThreads);
          int* ticket = p.tickets + (static_cast<int64_t>(h.seq) * p.num_kv_heads + h.kvh) * p.max_rowgroups + h.rg;
          if (tid == 0) {
            const int prev = atomicAdd(ticket, 1);
            const int last = prev == h.nchunks - 1;
            if (last) atomicExch(ticket, 0);
            sm.scratch[0] = last;
          }
          named_barrier(1, kConsumerThreads);
          if (sm.scratch[0]) {
            __threadfence();
            for (int col = 0; col < h.rows; ++col) {
              float M = -INFINITY;
              for (int c = 0; c < h.nchunks; ++c) {
                const float* part = p.partials + (static_cast<int64_t>(h.pair_first + c) * ROWS + col) * (kHeadDim + 2);
                M = fmaxf(M, __ldcg(part + kHeadDim));
              }
              const float Mu = M == -INFINITY ? 0.f : M;
              float L = 0.f, O = 0.f;
              for (int c = 0; c < h.nchunks; ++c) {
                const float* part = p.partials + (static_cast<int64_t>(h.pair_first + c) * ROWS + col) * (kHeadDim + 2);
                const float wt = ex2(__ldcg(part + kHeadDim) - Mu);
                L += wt * __ldcg(part + kHeadDim + 1);
                O += wt * __ldcg(part + d);
              }
              const int r = h.rg * ROWS + col;
              const int j = r / G, hh = h.kvh * G + (r - j * G);
              __nv_bfloat16 v = out_round(O / fmaxf(L, 1e-10f));
              p.out[static_cast<int64_t>(h.qrow0 + j) * p.out_row_stride + hh * kHeadDim + dim_real] =
                  *reinterpret_cast<uint16_t*>(&v);
            }
          }
        }
        // merge buffers are rewritten by the next item only after everyone read them
        named_barrier(1, kConsumerThreads);
      }
    }
  }

  // ---------------------------------------------------------------- last CTA out resets counters
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const int done = atomicAdd(p.ctrl + 2, 1);
    if (done == static_cast<int>(gridDim.x) - 1) {
      atomicExch(p.ctrl + 1, 0);
      atomicExch(p.ctrl + 2, 0);
    }
  }
}

template <int NT>
size_t decode_smem_bytes() {
  return sizeof(DecodeSmem<NT>) + 1024;  // + alignment slack
}

template <int NT>
int decode_grid_impl() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && cached[dev]) return cached[dev];
  int sms = 0, occ = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const size_t smem = decode_smem_bytes<NT>();
  cudaFuncSetAttribute(decode_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       static_cast<int>(smem));
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, decode_kernel<NT>, kDecodeThreads, smem);
  if (occ < 1) occ = 1;
  const int grid = sms * occ;
  if (dev < 64) cached[dev] = grid;
  return grid;
}

}  // namespace

int decode_grid(int nt) { return nt == 1 ? decode_grid_impl<1>() : decode_grid_impl<2>(); }

int64_t decode_workspace_bytes(int num_seqs, int num_kv_heads, int max_rowgroups, int rows,
                               int grid) {
  const int64_t pairs = static_cast<int64_t>(num_seqs) * num_kv_heads * max_rowgroups;
  const int64_t max_items = 32LL * grid + pairs;
  int64_t bytes = kCtrlInts * 4;
  bytes += (pairs * 4 + 255) / 256 * 256;
  bytes += max_items * rows * (kHeadDim + 2) * 4;
  return bytes;
}

cudaError_t launch_decode(const DecodeParams& p, int nt, const CUtensorMap& tmk,
                          const CUtensorMap& tmv, cudaStream_t stream) {
  if (nt == 1) {
    const int grid = decode_grid_impl<1>();
    decode_kernel<1><<<grid, kDecodeThreads, decode_smem_bytes<1>(), stream>>>(tmk, tmv, p);
  } else {
    const int grid = decode_grid_impl<2>();
    decode_kernel<2><<<grid, kDecodeThreads, decode_smem_bytes<2>(), stream>>>(tmk, tmv, p);
  }
  return cudaGetLastError();
}

}  // namespace fp8attn
