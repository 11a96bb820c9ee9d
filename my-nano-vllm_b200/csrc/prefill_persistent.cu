// Persistent varlen causal prefill kernel: one CTA per SM, claiming work items.
//
// Every CTA derives the same list of work items from cu_seqlens on the device (none for the
// sequences the split-KV decode engine serves), so no CTA is launched for a sequence without
// prefill work; launch_prefill picks this kernel when the per-item grid would be mostly such
// empty CTAs (speculative-verify batches).  The roles, the ring and the arithmetic are the
// per-item kernel's (prefill_common.cuh); across items the barrier phases run on, and an item's
// S products may start during the previous item's O read-out.
#include "prefill_common.cuh"

namespace fp8attn {
namespace {
// Block-wide exclusive scan of one int per thread (kThreads threads).
template <int kThreads>
__device__ __forceinline__ int prefill_block_scan(int v, int* smem, int* total) {
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
    const int t = smem[w];
    if (w < warp) base += t;
    tot += t;
  }
  __syncthreads();
  *total = tot;
  return base + x - v;
}

// Work items of sequence s: its q tiles of 128 rows (when it has at least min_q rows) times the
// head pairs; none for the sequences the split-KV engine serves.
__device__ __forceinline__ int seq_items(const PrefillParams& p, int s, int head_pairs) {
  const int nq = __ldg(p.cu_q + s + 1) - __ldg(p.cu_q + s);
  return nq >= p.min_q && nq > 0 ? (nq + kBM - 1) / kBM * head_pairs : 0;
}

// One thread's half of a query row (kCols dims from column cb) -> e4m3 hi / lo in the group's
// 128B-swizzled K-major q planes, scaled by a power of two from the row's amax (both halves
// exchange theirs through xq and the group barrier xch).  Returns the row's score factor, NaN
// when the exchange timed out.  Kept out of line: inlined into the persistent tile loop, its
// registers made the tile code spill.
template <int kNH>
__device__ __noinline__ float load_q_row(const uint16_t* __restrict__ src, bool row_ok, int r, int cb,
                                         int half, uint8_t* qhi, uint8_t* qlo, float* xq,
                                         uint64_t* xch, uint32_t xphase, int* err, float scale_log2) {
  constexpr int kW = 16 / kNH;  // 16-byte loads of this half (8 bf16 each)
  auto load = [&](int i) {
    return row_ok ? ldg_keep_v4(reinterpret_cast<const uint4*>(src) + i) : make_uint4(0, 0, 0, 0);
  };
  auto widen = [](const uint4& v, float* x) {
    const uint32_t ww[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      x[2 * k] = __uint_as_float(ww[k] << 16);
      x[2 * k + 1] = __uint_as_float(ww[k] & 0xFFFF0000u);
    }
  };
  uint4 w[kW];  // all loads in flight at once
#pragma unroll
  for (int i = 0; i < kW; ++i) w[i] = load(i);
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < kW; ++i) {
    float x[8];
    widen(w[i], x);
#pragma unroll
    for (int k = 0; k < 8; ++k) amax = fmaxf(amax, fabsf(x[k]));
  }
  if (kNH > 1) {
    xq[half * kBM + r] = amax;
    mbar_arrive(xch);
    if (!mbar_wait(xch, xphase, err)) return __int_as_float(0x7fc00000);
    amax = fmaxf(xq[r], xq[kBM + r]);
  }
  float srow;
  const float inv = pow2_inv_scale(amax, &srow);
#pragma unroll
  for (int cc = 0; cc < kW / 2; ++cc) {  // 16 dims per 16-byte chunk
    const int c = cb / 16 + cc;
    float x[16];
    widen(w[2 * cc], x);
    widen(w[2 * cc + 1], x + 8);
#pragma unroll
    for (int k = 0; k < 16; ++k) x[k] *= inv;
    uint4 hv, lv;
    split16(x, hv, lv);
    const int off = r * 128 + ((c ^ (r & 7)) << 4);
    *reinterpret_cast<uint4*>(&qhi[off]) = hv;
    *reinterpret_cast<uint4*>(&qlo[off]) = lv;
  }
  return srow * scale_log2;
}

// One thread's half of an output row: kCols O columns from tensor memory (this warp's lane
// quadrant) times inv -> fp16 -> bf16 at out_row (null: the row does not exist; the columns are
// still read, as tcgen05.ld is warp-collective).  Out of line for the same reason as load_q_row.
template <int kCols>
__device__ __noinline__ void store_o_row(uint32_t o_taddr, float inv, uint16_t* out_row) {
#pragma unroll
  for (int c0 = 0; c0 < kCols; c0 += 16) {
    float o16[16];
    tc::ld16(o_taddr + c0, o16);
    tc::wait_ld();
    if (out_row != nullptr) {
      uint32_t pk[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        __nv_bfloat16 a = out_round(o16[2 * i] * inv), b = out_round(o16[2 * i + 1] * inv);
        pk[i] = static_cast<uint32_t>(*reinterpret_cast<uint16_t*>(&a)) |
                (static_cast<uint32_t>(*reinterpret_cast<uint16_t*>(&b)) << 16);
      }
      uint4* dst = reinterpret_cast<uint4*>(out_row + c0);
      dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
    }
  }
}

// Persistent: one CTA per SM.  Every CTA computes the same plan (the work items before each
// sequence, in shared memory); the producer claims items from the workspace's counter, in order
// sequence by sequence, q tiles from the last (which sees the most keys) to the first, and
// streams their K/V tiles through the ring; the MMA issuer and the softmax groups follow the
// tile headers.  Barrier phases run on across items.  At an item's last tile the groups load the
// next item's q rows before reading out this item's O, so the next item's S products overlap the
// read-out; its first PV, which overwrites O, waits for the read-out (o_free).  The last tile's
// stage is held until the read-out, which takes the output rows from its header.
template <int NG>
__global__ void __launch_bounds__(PrefillCfg<NG>::kThreads, 1)
    prefill_persistent_kernel(const __grid_constant__ CUtensorMap tmk,
                              const __grid_constant__ CUtensorMap tmv, const PrefillParams p) {
  using Cfg = PrefillCfg<NG>;
  constexpr int kStages = Cfg::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  PrefillSmem<NG>& sm = *reinterpret_cast<PrefillSmem<NG>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = p.group;
  const int head_pairs = p.num_heads / NG;
  const int S = p.num_seqs;
  int* prefix = reinterpret_cast<int*>(&sm + 1);

  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&sm.kv_full[i], 1);
      mbar_init(&sm.kv_empty[i], 1 + Cfg::kGroupThreads * NG);  // MMA commit, softmax threads
      mbar_init(&sm.vh_full[i], Cfg::kGroupThreads * NG);
    }
    for (int g = 0; g < NG; ++g) {
      mbar_init(&sm.q_full[g], Cfg::kGroupThreads);
      mbar_init(&sm.s_full[g], 1);
      mbar_init(&sm.o_full[g], 1);
      mbar_init(&sm.p_full[g], Cfg::kGroupThreads);
      mbar_init(&sm.xch[g], Cfg::kGroupThreads);
      for (int qd = 0; qd < 4; ++qd) mbar_init(&sm.xpair[g][qd], 64);
      mbar_init(&sm.o_free[g], Cfg::kGroupThreads);
    }
    fence_mbar_init();
  }
  if (warp == Cfg::kProducerWarp && lane == 0) {
    prefetch_tensormap(&tmk);
    prefetch_tensormap(&tmv);
  }
  if (warp == Cfg::kMmaWarp) {
    tc::tmem_alloc(&sm.tmem_base, Cfg::kTmemCols);
    tc::tmem_relinquish();
  }
  // ---------------------------------------------------------------- plan (every CTA, same result)
  const int per = (S + Cfg::kThreads - 1) / Cfg::kThreads;
  const int s0 = min(S, tid * per), s1 = min(S, s0 + per);
  int mine = 0;
  for (int s = s0; s < s1; ++s) mine += seq_items(p, s, head_pairs);
  int total_items = 0;
  int acc = prefill_block_scan<Cfg::kThreads>(mine, sm.scratch, &total_items);
  for (int s = s0; s < s1; ++s) {
    prefix[s] = acc;
    acc += seq_items(p, s, head_pairs);
  }
  if (tid == 0) prefix[S] = total_items;
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = sm.tmem_base;
  const bool kscaled = p.k_scale != nullptr;
  const bool paged = p.block_tables != nullptr;
  const int bs = p.block_size;
  const int box_rows = box_rows_of(paged, bs);
  const int box_shift = 31 - __clz(box_rows);

  if (warp == Cfg::kProducerWarp) {
    // ============================================================ TMA producer
    const int nbox = kBN / box_rows;
    int stage = 0;
    uint32_t phase = 0;
    // The next item is claimed two tiles before this one's last (its seq lookup and first block
    // table loads then overlap the last tiles), i.e. a few tiles before this CTA's consumers run
    // dry: claiming a whole item ahead would let a busy CTA hold a long item that an idle one
    // could run (a tail of up to one item on batches of few long items).
    int next = lane == 0 ? atomicAdd(p.err + 1, 1) : 0;
    while (true) {
      const int item = __shfl_sync(0xffffffffu, next, 0);
      if (item >= total_items) {  // no more work: a last header tells the consumers
        if (mbar_wait(&sm.kv_empty[stage], phase ^ 1, p.err) && lane == 0) {
          sm.tile[stage].item = -1;
          mbar_arrive_expect_tx(&sm.kv_full[stage], 0);
        }
        break;
      }
      // the item's sequence: the last with prefix <= item
      int lo = 0, hi = S - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (prefix[mid] <= item) lo = mid; else hi = mid - 1;
      }
      const int s = lo;
      const int r = item - prefix[s];
      SeqInfo si;
      seq_info(p, s, 0, si);
      const int nqt = (si.nq + kBM - 1) / kBM;
      const int qt = nqt - 1 - r / head_pairs;
      const int hp = r - (r / head_pairs) * head_pairs;
      seq_info(p, s, qt, si);
      const int kvh = hp * NG / G;
      const int64_t bt_row = static_cast<int64_t>(s) * p.bt_stride;
      int ebase = INT_MIN / 2, myent = -1;
      const int nt = si.ntiles;
      bool ok = true;
      const int last = max(nt, 1) - 1;
      for (int j = 0; j <= last; ++j) {  // an item without key tiles still sends a header
        const int j0 = j * kBN;
        if (j == max(0, last - 2) && lane == 0) next = atomicAdd(p.err + 1, 1);
        int blks[kMaxBoxes];
        if (paged) {
#pragma unroll
          for (int b = 0; b < kMaxBoxes; ++b) {
            blks[b] = -1;
            if (b < nbox && nt > 0) {
              const int pos = j0 + b * box_rows;
              const int e = pos / bs;
              if (e < ebase || e >= ebase + 32) {
                ebase = e;
                const int idx = e + lane;
                myent = idx < p.max_blocks ? ldg_keep(p.block_tables + bt_row + idx) : -1;
              }
              int blk = __shfl_sync(0xffffffffu, myent, e - ebase);
              if (blk < 0 || blk >= p.num_blocks || pos >= si.vis) blk = -1;
              blks[b] = blk;
            }
          }
        }
        if (!mbar_wait(&sm.kv_empty[stage], phase ^ 1, p.err)) { ok = false; break; }
        if (lane == 0) {
          PrefillTile& t = sm.tile[stage];
          const int q0 = qt * kBM;
          t.item = item;
          t.j = j;
          t.ntiles = nt;
          t.j0 = j0;
          t.vis = si.vis;
          t.lim0 = q0 + (si.nk - si.nq);
          t.rows = min(kBM, si.nq - q0);
          t.kvh = kvh;
          t.k_begin = si.k_begin;
          t.q_off = static_cast<int64_t>(si.q_begin + q0) * p.q_row_stride + hp * NG * 128;
          t.out_off = static_cast<int64_t>(si.q_begin + q0) * p.out_row_stride + hp * NG * 128;
          uint32_t bytes = 0, mask = 0;
#pragma unroll
          for (int b = 0; b < kMaxBoxes; ++b) {
            t.blk[b] = paged ? blks[b] : 0;
            if (nt > 0 && b < nbox && (!paged || blks[b] >= 0)) {
              bytes += 2u * box_rows * 128;
              mask |= 1u << b;
            }
          }
          t.boxmask = mask;
          mbar_arrive_expect_tx(&sm.kv_full[stage], bytes);
        }
        __syncwarp();
        if (lane < 2 && nt > 0) {  // lane 0: K boxes, lane 1: V boxes
          const CUtensorMap* map = lane == 0 ? &tmk : &tmv;
          uint8_t* dst = lane == 0 ? &sm.k[stage][0] : &sm.v[stage][0];
          for (int b = 0; b < nbox; ++b) {
            int y;
            if (paged) {
              if (blks[b] < 0) continue;
              const int pos = j0 + b * box_rows;
              y = blks[b] * bs + (pos - (pos / bs) * bs);
            } else {
              y = si.k_begin + j0 + b * box_rows;  // rows past the tensor end read as zeros
            }
            tma_load_2d(dst + b * box_rows * 128, map, &sm.kv_full[stage], kvh * 128, y);
          }
        }
        __syncwarp();
        if (++stage == kStages) { stage = 0; phase ^= 1; }
      }
      if (!ok) break;
    }
  } else if (warp == Cfg::kMmaWarp) {
    // ============================================================ MMA issuer
    // per tile j and group g in turn: PV_g(j-1) once P_g(j-1) is written (P lives in S_g's
    // columns, so it must be read before the next S), then S_g(j); the tensor pipe runs one
    // thread's MMAs in order.  A tile's stage is released after every group's PV of it.
    if (lane == 0) {
      const uint32_t idesc_s = tc::idesc_e4m3(128, 128, false, false);
      const uint32_t idesc_pv = tc::idesc_f16(128, 128, false, true);
      int stage = 0, prev_stage = 0;
      uint32_t phase = 0, prev_phase = 0;
      int pv_count[NG];   // PVs issued per group (parity of p_full)
      int items_done = 0;  // items with key tiles whose O was started (parity of q_full / o_free)
      int q_items = 0;     // items whose q rows were loaded (parity of q_full)
#pragma unroll
      for (int g = 0; g < NG; ++g) pv_count[g] = 0;
      bool ok = true;
      // O_g += P_g . V over tile jt of the item (stage st, filled in phase ph): kind::f16, K = 16
      // keys per MMA, P_g (f16 pairs) from S_g's columns, V as f16 (both groups converted their
      // shares: vh_full)
      auto issue_pv = [&](int g, int jt, int st, uint32_t ph) -> bool {
        if (!mbar_wait(&sm.p_full[g], pv_count[g] & 1, p.err)) return false;
        // an item's first PV overwrites O: the previous item's read-out must be done
        if (jt == 0 && items_done > 0 && !mbar_wait(&sm.o_free[g], (items_done - 1) & 1, p.err))
          return false;
        if (g == 0 && !mbar_wait(&sm.vh_full[st], ph, p.err)) return false;
        ++pv_count[g];
        tc::fence_after_sync();
        const uint32_t vb = smem_u32(&sm.vh[st][0]);
        const uint32_t pt = tmem + 256 * g;
#pragma unroll
        for (int ks = 0; ks < kBN / 16; ++ks) {
          // V rows 16 ks .. + 15: two 64-dim blocks kBN * 128 bytes apart, 8-row groups 1 KB apart
          const uint64_t bd = tc::smem_desc(vb + ks * 16 * 128, kBN * 128, 1024, tc::kSw128);
          tc::mma_f16_ts(tmem + 256 * g + 128, pt + p_col(16 * ks & ~31) + ((16 * ks) & 16) / 2, bd,
                         idesc_pv, (jt > 0 || ks > 0) ? 1u : 0u);
        }
        return true;
      };
      while (ok) {
        if (!mbar_wait(&sm.kv_full[stage], phase, p.err)) break;
        const PrefillTile& t = sm.tile[stage];
        if (t.item < 0) break;
        const int j = t.j, nt = t.ntiles;
        if (nt == 0) {  // an item whose rows see no key: nothing to compute
          mbar_arrive(&sm.kv_empty[stage]);
          if (++stage == kStages) { stage = 0; phase ^= 1; }
          continue;
        }
        if (j == 0) {
          // the groups' q rows of this item (its S products only touch S columns, so they may
          // run during the previous item's read-out; its first PV waits for that read-out)
          for (int g = 0; g < NG && ok; ++g) ok = mbar_wait(&sm.q_full[g], q_items & 1, p.err);
          ++q_items;
          if (!ok) break;
        }
        const uint32_t ka = smem_u32(&sm.k[stage][0]);
        for (int g = 0; g < NG && ok; ++g) {
          if (j > 0 && !issue_pv(g, j - 1, prev_stage, prev_phase)) { ok = false; break; }
          const uint32_t qh = smem_u32(&sm.qhi[g][0]), ql = smem_u32(&sm.qlo[g][0]);
#pragma unroll
          for (int plane = 0; plane < 2; ++plane)
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
              const uint64_t ad = tc::smem_desc((plane ? ql : qh) + ks * 32, 16, 1024, tc::kSw128);
              const uint64_t bd = tc::smem_desc(ka + ks * 32, 16, 1024, tc::kSw128);
              tc::mma_f8(tmem + 256 * g, ad, bd, idesc_s, (plane > 0 || ks > 0) ? 1u : 0u);
            }
          tc::commit(&sm.s_full[g]);
        }
        if (!ok) break;
        if (j > 0) tc::commit(&sm.kv_empty[prev_stage]);
        if (j == nt - 1) {  // the item's last PV, then its O is final
          for (int g = 0; g < NG && ok; ++g) {
            ok = issue_pv(g, j, stage, phase);
            if (ok) tc::commit(&sm.o_full[g]);
          }
          if (!ok) break;
          tc::commit(&sm.kv_empty[stage]);
          ++items_done;
        }
        prev_stage = stage;
        prev_phase = phase;
        if (++stage == kStages) { stage = 0; phase ^= 1; }
      }
    }
    __syncwarp();
  } else {
    // ============================================================ softmax group g
    // warp (g, half, quadrant): query rows 32 quadrant .. + 31 of head g, key columns
    // 64 half .. + 63 of every tile (and the same half of each q and O row)
    constexpr int kNH = Cfg::kNH;
    constexpr int kCols = kBN / kNH;
    const int g = warp / (4 * kNH);
    const int half = (warp >> 2) & (kNH - 1);
    const int cb = half * kCols;
    const int r = 32 * (warp & 3) + lane;  // query row within the tile
    const uint32_t lane_base = static_cast<uint32_t>(32 * (warp & 3)) << 16;
    const uint32_t s_tmem = tmem + lane_base + 256 * g;
    const uint32_t o_tmem = s_tmem + 128;
    uint8_t* const qhi = sm.qhi[g];
    uint8_t* const qlo = sm.qlo[g];
    uint32_t xphase = 0;
    int s_waits = 0;  // s_full completions waited for (parity)
    int o_waits = 0;  // o_full completions waited for (parity)
    // the group's exchange: every softmax thread arrives, then waits (bounded) for all
    auto exchange = [&]() -> bool {
      mbar_arrive(&sm.xch[g]);
      const bool done = mbar_wait(&sm.xch[g], xphase, p.err);
      xphase ^= 1;
      return done;
    };
    // the row's exchange: the two warps (column halves) of this row quadrant only
    uint32_t pphase = 0;
    uint64_t* const xpair = &sm.xpair[g][warp & 3];
    auto pair_exchange = [&]() -> bool {
      mbar_arrive(xpair);
      const bool done = mbar_wait(xpair, pphase, p.err);
      pphase ^= 1;
      return done;
    };
    bool ok = true;
    int stage = 0;
    uint32_t phase = 0;
    // the row's state within the current item; the rest of the item is read from the headers
    float cs = 0.f, m_ref = -INFINITY, l = 0.f;
    bool q_ready = false;  // the next item's q rows are loaded already
    // the query row of tile header tn's item -> e4m3 hi / lo, 128B-swizzled K-major rows (this
    // half's dims); the caller has seen the last S product of the previous item, the q planes'
    // last reader, complete
    auto q_rows = [&](const PrefillTile& tn) -> bool {
      const bool row_ok = r < tn.rows;
      cs = load_q_row<kNH>(p.q + tn.q_off + static_cast<int64_t>(row_ok ? r : 0) * p.q_row_stride + g * 128 + cb,
                           row_ok, r, cb, half, qhi, qlo, &sm.xq[g][0][0], &sm.xch[g], xphase,
                           p.err, p.scale_log2);
      if (kNH > 1) xphase ^= 1;
      if (cs != cs) return false;
      fence_proxy_async_smem();
      mbar_arrive(&sm.q_full[g]);
      return true;
    };
    while (ok) {
      if (!mbar_wait(&sm.kv_full[stage], phase, p.err)) break;
      const int tstage = stage;
      const PrefillTile& t = sm.tile[tstage];
      const int item = t.item;
      if (item < 0) break;
      const int j = t.j, nt = t.ntiles;
      const int j0 = t.j0;
      const uint32_t boxmask = t.boxmask;  // boxes whose block is valid
      if (j == 0) {
        // ---- a new item: its query rows (unless loaded during the previous item's read-out)
        if (nt > 0 && !q_ready && !q_rows(t)) { ok = false; break; }
        q_ready = false;
        m_ref = -INFINITY;
        l = 0.f;
      }
      if (nt == 0) {
        // rows that see no key position: zeros (the reference's where(l > 0, acc / l, 0))
        if (r < t.rows) {
          uint4* dst = reinterpret_cast<uint4*>(p.out + t.out_off + static_cast<int64_t>(r) * p.out_row_stride + g * 128 + cb);
          for (int i = 0; i < kCols / 8; ++i) dst[i] = make_uint4(0, 0, 0, 0);
        }
        mbar_arrive(&sm.vh_full[stage]);  // keeps its phases in step with the stage's uses
        mbar_arrive(&sm.kv_empty[stage]);
        if (++stage == kStages) { stage = 0; phase ^= 1; }
        continue;
      }
      // key columns of this tile that can be valid at all (visible, inside this sequence)
      const int col_end = min(kBN, t.vis - j0);
      // ---- this thread's share of the V tile -> f16 (the PV operand): key row r, dims
      // cb + g * kConv .. + kConv - 1 (the groups split each half's 64 dims); keys outside the
      // sequence or in masked blocks, whose bytes may be anything, become zeros
      {
        constexpr int kConv = 64 / NG;
        const bool kv_ok = r < col_end && ((boxmask >> (r >> box_shift)) & 1u);
        const uint8_t* vrow = &sm.v[stage][r * 128];
        uint8_t* hrow = &sm.vh[stage][half * kBN * 128 + r * 128];
#pragma unroll
        for (int c = 0; c < kConv / 16; ++c) {
          const int d = g * kConv + 16 * c;  // first dim of the chunk within the half
          const uint4 x = kv_ok ? *reinterpret_cast<const uint4*>(vrow + ((((cb + d) >> 4) ^ (r & 7)) << 4))
                                : make_uint4(0, 0, 0, 0);
          const uint32_t w[4] = {x.x, x.y, x.z, x.w};
          uint32_t hw[8];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            hw[2 * i] = e4m3x2_to_f16x2(w[i] & 0xFFFFu);
            hw[2 * i + 1] = e4m3x2_to_f16x2(w[i] >> 16);
          }
          const int dc = d >> 3;  // 8-dim (16-byte) chunk of the f16 row
          *reinterpret_cast<uint4*>(hrow + ((dc ^ (r & 7)) << 4)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
          *reinterpret_cast<uint4*>(hrow + (((dc + 1) ^ (r & 7)) << 4)) = make_uint4(hw[4], hw[5], hw[6], hw[7]);
        }
        fence_proxy_async_smem();
        mbar_arrive(&sm.vh_full[stage]);
      }
      // columns [0, vlim) of this tile are visible to this row.  A tile with a masked block, or
      // any tile of a scaled cache, takes the general path through the column table (uniform
      // across the group's warps)
      const int vlim = r < t.rows ? max(0, min(col_end, t.lim0 + r - j0 + 1)) : 0;
      const bool general = kscaled || !(p.scale_log2 > 0.f) || boxmask != (1u << (kBN / box_rows)) - 1u;
      const bool last = j == nt - 1;
      // S_g(j) complete => PV_g(j-1) complete (issued before it): O is quiescent
      if (!mbar_wait(&sm.s_full[g], s_waits & 1, p.err)) { ok = false; break; }
      ++s_waits;
      tc::fence_after_sync();
      if (general) {
        // S_g(j) complete => the group finished tile j-1, the table's last reader; the first
        // column half fills it (thread r: column r)
        const int c = r;
        if (half == 0) {
          const bool cok = c < col_end && ((boxmask >> (c >> box_shift)) & 1u);
          float ks = 1.f, vs = 1.f;
          if (kscaled && cok) {
            const int kv = j0 + c;
            const int64_t slot = paged ? static_cast<int64_t>(t.blk[c >> box_shift]) * bs + (kv % bs)
                                       : static_cast<int64_t>(t.k_begin) + kv;
            ks = __ldg(p.k_scale + slot * p.num_kv_heads + t.kvh);
            vs = __ldg(p.v_scale + slot * p.num_kv_heads + t.kvh);
          }
          sm.colk[g][c] = ks;
          sm.colv[g][c] = vs;
          const uint32_t bal = __ballot_sync(0xffffffffu, cok);
          if (lane == 0) sm.colok[g][warp & 3] = bal;
        }
        if (!exchange()) { ok = false; break; }
      }
      // done with the tile's header and block list; the last tile's header stays until the
      // item's read-out, which takes the output rows from it
      if (!last) mbar_arrive(&sm.kv_empty[stage]);
      // ---- pass 1: row maximum (of the raw scores on the fast path: cs > 0 commutes with max)
      float tmax = -INFINITY;
#pragma unroll 1
      for (int c0 = cb; c0 < cb + kCols; c0 += 32) {
        float v[32];
        tmem_ld32(s_tmem + c0, v);
        tc::wait_ld();
        if (!general && c0 + 32 <= vlim) {  // every column visible: four independent chains
          float a0 = v[0], a1 = v[1], a2 = v[2], a3 = v[3];
#pragma unroll
          for (int i = 4; i < 32; i += 4) {
            a0 = fmaxf(a0, v[i]);
            a1 = fmaxf(a1, v[i + 1]);
            a2 = fmaxf(a2, v[i + 2]);
            a3 = fmaxf(a3, v[i + 3]);
          }
          tmax = fmaxf(tmax, fmaxf(fmaxf(a0, a1), fmaxf(a2, a3)));
        } else if (!general) {
#pragma unroll
          for (int i = 0; i < 32; ++i) tmax = fmaxf(tmax, c0 + i < vlim ? v[i] : -INFINITY);
        } else {
          const uint32_t okw = sm.colok[g][c0 >> 5];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const bool cok = ((okw >> i) & 1u) && c0 + i < vlim;
            tmax = fmaxf(tmax, cok ? v[i] * sm.colk[g][c0 + i] * cs : -INFINITY);
          }
        }
      }
      if (!general && tmax != -INFINITY) tmax *= cs;
      if (kNH > 1) {  // the row's other half (its S reads are done once it arrives)
        sm.xmax[g][half][r] = tmax;
        if (!pair_exchange()) { ok = false; break; }
        tmax = fmaxf(sm.xmax[g][0][r], sm.xmax[g][1][r]);
      }
      // lazy rescale: move the reference max only when it grows by more than 2^4, so that
      // P = 16 * 2^(s - m_ref) <= 256
      float alpha = 1.f;
      if (tmax > m_ref + kRescaleLog2) {
        alpha = m_ref == -INFINITY ? 0.f : ex2(m_ref - tmax);
        m_ref = tmax;
        l *= alpha;
      }
      // ---- pass 2: P as e4m3 hi + lo into this half's S columns already read (chunk c0 of 32
      // keys -> hi in columns p_col(c0) .. + 8, lo in the next 8)
      const float bias = kPScaleLog2 - (m_ref == -INFINITY ? 0.f : m_ref);
      float l_tile = 0.f;
#pragma unroll 1
      for (int c0 = cb; c0 < cb + kCols; c0 += 32) {
        float v[32];
        tmem_ld32(s_tmem + c0, v);
        tc::wait_ld();
        uint32_t pw[16];  // f16 pairs: keys c0 + 2i (low half) and c0 + 2i + 1
        if (!general) {
          // exponent arguments as packed pairs; every third pair (5 of the 16) takes a
          // polynomial on the FMA pipe, the others the MUFU ex2 (whose rate bounds this loop);
          // the row sum adds the fp32 values in four packed partials
          const uint64_t cs2 = f2_pack(cs, cs), bias2 = f2_pack(bias, bias);
          uint64_t la[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) la[k] = f2_pack(0.f, 0.f);
          const bool full = c0 + 32 <= vlim;
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            float a0, a1;
            f2_unpack(f2_fma(f2_pack(v[2 * k], v[2 * k + 1]), cs2, bias2), a0, a1);
            if (!full) {
              a0 = c0 + 2 * k < vlim ? a0 : -INFINITY;
              a1 = c0 + 2 * k + 1 < vlim ? a1 : -INFINITY;
            }
            float e0, e1;
            if (k % 3 == 2) {
              exp2_poly_x2(a0, a1, e0, e1);
            } else {
              e0 = ex2(a0);
              e1 = ex2(a1);
            }
            la[k & 3] = f2_add(la[k & 3], f2_pack(e0, e1));
            pw[k] = pack_f16x2(e0, e1);
          }
          float s0, s1;
          f2_unpack(f2_add(f2_add(la[0], la[1]), f2_add(la[2], la[3])), s0, s1);
          l_tile += s0 + s1;
        } else {
          const uint32_t okw = sm.colok[g][c0 >> 5];
          float la[4] = {0.f, 0.f, 0.f, 0.f};  // independent partial sums
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const bool cok = ((okw >> i) & 1u) && c0 + i < vlim;
            const float e = cok ? ex2(v[i] * sm.colk[g][c0 + i] * cs + bias) : 0.f;
            la[i & 3] += e;
            v[i] = e * sm.colv[g][c0 + i];
          }
          l_tile += (la[0] + la[1]) + (la[2] + la[3]);
#pragma unroll
          for (int k = 0; k < 16; ++k) pw[k] = pack_f16x2(v[2 * k], v[2 * k + 1]);
        }
        tc::st16u(s_tmem + p_col(c0), pw);
      }
      l += l_tile;
      // O (quiescent) follows a moved reference; each warp rescales its own rows
      if (__any_sync(0xffffffffu, alpha != 1.f) && j > 0) {
#pragma unroll
        for (int c0 = cb; c0 < cb + kCols; c0 += 16) {
          float o16[16];
          tc::ld16(o_tmem + c0, o16);
          tc::wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) o16[i] *= alpha;
          tc::st16(o_tmem + c0, o16);
        }
      }
      tc::wait_st();
      tc::fence_before_sync();
      mbar_arrive(&sm.p_full[g]);
      if (++stage == kStages) { stage = 0; phase ^= 1; }
      if (!last) continue;
      // the next item's q rows first: its S(0) then runs during this item's last PV and read-out
      // (the next ring stage holds the next item's first tile, or the end-of-work header)
      if (!mbar_wait(&sm.kv_full[stage], phase, p.err)) { ok = false; break; }
      {
        const PrefillTile& tn = sm.tile[stage];
        if (tn.item >= 0 && tn.ntiles > 0) {
          if (!q_rows(tn)) { ok = false; break; }
          q_ready = true;
        }
      }
      // ---- the item's epilogue: O / l -> fp16 -> bf16 (the reference's output path)
      float lsum = l;
      if (kNH > 1) {  // the row sum over both halves
        sm.xl[g][half][r] = l;
        if (!pair_exchange()) { ok = false; break; }
        lsum = sm.xl[g][0][r] + sm.xl[g][1][r];
      }
      if (!mbar_wait(&sm.o_full[g], o_waits & 1, p.err)) { ok = false; break; }  // O final
      ++o_waits;
      tc::fence_after_sync();
      const float inv = lsum > 0.f ? 1.f / lsum : 0.f;  // O and l carry the same factor 16
      uint16_t* const out_row = r < t.rows ? p.out + t.out_off + static_cast<int64_t>(r) * p.out_row_stride + g * 128 + cb
                                           : nullptr;
      store_o_row<kCols>(o_tmem + cb, inv, out_row);
      tc::fence_before_sync();
      mbar_arrive(&sm.o_free[g]);  // the next item's first PV may overwrite O
      mbar_arrive(&sm.kv_empty[tstage]);
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == Cfg::kMmaWarp) tc::tmem_dealloc(tmem, Cfg::kTmemCols);
  if (tid == 0) release_work_counters(p.err);
}


template <int NG>
cudaError_t launch_groups(const PrefillParams& p, const CUtensorMap& tmk, const CUtensorMap& tmv,
                          cudaStream_t stream) {
  static bool configured[64] = {false};
  static int sms[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaFuncSetAttribute(prefill_persistent_kernel<NG>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(sizeof(PrefillSmem<NG>) + 1024 + (kMaxSeqs + 1) * 4));
    cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    configured[dev] = true;
  }
  const size_t smem = sizeof(PrefillSmem<NG>) + 1024 + static_cast<size_t>(p.num_seqs + 1) * 4;
  // one CTA per SM, fewer when the call cannot have that many work items
  const int64_t bound = static_cast<int64_t>(p.num_seqs) * ((p.max_seqlen_q + kBM - 1) / kBM) *
                        (p.num_heads / NG);
  const int n_sm = dev >= 0 && dev < 64 && sms[dev] > 0 ? sms[dev] : 148;
  const int grid = static_cast<int>(bound < n_sm ? (bound > 0 ? bound : 1) : n_sm);
  prefill_persistent_kernel<NG><<<grid, PrefillCfg<NG>::kThreads, smem, stream>>>(tmk, tmv, p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_prefill_persistent(const PrefillParams& p, const CUtensorMap& tmk,
                                      const CUtensorMap& tmv, cudaStream_t stream) {
  return p.group % 2 == 0 ? launch_groups<2>(p, tmk, tmv, stream)
                          : launch_groups<1>(p, tmk, tmv, stream);
}

}  // namespace fp8attn
