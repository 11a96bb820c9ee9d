// Varlen causal prefill kernel, one CTA per work item: grid (q tiles, head pairs, sequences),
// q tiles from the last (which sees the most keys) to the first; a CTA whose tile or sequence has
// no prefill work returns at once.  Also the entry, launch_prefill, which picks between this
// kernel and the persistent one (prefill_persistent.cu).  Roles, ring and arithmetic:
// prefill_common.cuh.
#include "prefill_common.cuh"

namespace fp8attn {
namespace {

// Per-item grids larger than this (about 14 waves of 148 SMs) go to the persistent kernel.
constexpr int64_t kPersistentCtas = 2048;

template <int NG>
__global__ void __launch_bounds__(PrefillCfg<NG>::kThreads, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                   const PrefillParams p) {
  using Cfg = PrefillCfg<NG>;
  constexpr int kStages = Cfg::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  PrefillSmem<NG>& sm = *reinterpret_cast<PrefillSmem<NG>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // heavy tiles first: later q tiles see more keys
  const int qt = static_cast<int>(gridDim.x) - 1 - static_cast<int>(blockIdx.x);
  const int h0 = blockIdx.y * NG, s = blockIdx.z;  // q heads h0 .. h0 + NG - 1 share a kv head
  SeqInfo si;
  if (!seq_info(p, s, qt, si)) return;  // uniform across the CTA
  const int G = p.group;
  const int kvh = h0 / G;
  const int q0 = qt * kBM;
  const int rows = min(kBM, si.nq - q0);

  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&sm.kv_full[i], 1);
      mbar_init(&sm.kv_empty[i], 1 + Cfg::kGroupThreads * NG);  // MMA commit, softmax threads
      mbar_init(&sm.vh_full[i], Cfg::kGroupThreads * NG);
    }
    for (int g = 0; g < NG; ++g) {
      mbar_init(&sm.q_full[g], Cfg::kGroupThreads);
      mbar_init(&sm.s_full[g], 1);
      mbar_init(&sm.p_full[g], Cfg::kGroupThreads);
      mbar_init(&sm.xch[g], Cfg::kGroupThreads);
      for (int qd = 0; qd < 4; ++qd) mbar_init(&sm.xpair[g][qd], 64);
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
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = sm.tmem_base;
  const int ntiles = si.ntiles;
  const bool kscaled = p.k_scale != nullptr;
  const bool paged = p.block_tables != nullptr;
  const int bs = p.block_size;
  const int box_rows = box_rows_of(paged, bs);
  const int box_shift = 31 - __clz(box_rows);

  if (warp == Cfg::kProducerWarp) {
    // ============================================================ TMA producer
    const int nbox = kBN / box_rows;
    const int64_t bt_row = static_cast<int64_t>(s) * p.bt_stride;
    int ebase = INT_MIN / 2, myent = -1;
    int stage = 0;
    uint32_t phase = 0;
    for (int j = 0; j < ntiles; ++j) {
      const int j0 = j * kBN;
      int blks[kMaxBoxes];
      if (paged) {
#pragma unroll
        for (int b = 0; b < kMaxBoxes; ++b) {
          blks[b] = -1;
          if (b < nbox) {
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
      if (!mbar_wait(&sm.kv_empty[stage], phase ^ 1, p.err)) break;
      if (lane == 0) {
        PrefillTile& t = sm.tile[stage];
        t.j0 = j0;
        uint32_t bytes = 0, mask = 0;
#pragma unroll
        for (int b = 0; b < kMaxBoxes; ++b) {
          t.blk[b] = paged ? blks[b] : 0;
          if (b < nbox && (!paged || blks[b] >= 0)) {
            bytes += 2u * box_rows * 128;
            mask |= 1u << b;
          }
        }
        t.boxmask = mask;
        mbar_arrive_expect_tx(&sm.kv_full[stage], bytes);
      }
      __syncwarp();
      if (lane < 2) {  // lane 0: K boxes, lane 1: V boxes
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
  } else if (warp == Cfg::kMmaWarp) {
    // ============================================================ MMA issuer
    // per tile j and group g in turn: PV_g(j-1) once P_g(j-1) is written (P lives in S_g's
    // columns, so it must be read before the next S), then S_g(j); the tensor pipe runs one
    // thread's MMAs in order.  The stage of tile j-1 is released after every group's PV.
    if (lane == 0 && ntiles > 0) {
      const uint32_t idesc_s = tc::idesc_e4m3(128, 128, false, false);
      const uint32_t idesc_pv = tc::idesc_f16(128, 128, false, true);
      bool ok = true;
      for (int g = 0; g < NG && ok; ++g) ok = mbar_wait(&sm.q_full[g], 0, p.err);
      int stage = 0, prev_stage = 0;
      uint32_t phase = 0;
      // operand descriptors, built once: a K step moves an operand by a multiple of 16 bytes,
      // i.e. adds to the start-address field (bits 0-13, address >> 4), which no operand here
      // carries past its 14 bits
      const uint64_t dk0 = tc::smem_desc(smem_u32(&sm.k[0][0]), 16, 1024, tc::kSw128);
      const uint64_t dk1 = tc::smem_desc(smem_u32(&sm.k[kStages - 1][0]), 16, 1024, tc::kSw128);
      const uint64_t dv0 = tc::smem_desc(smem_u32(&sm.vh[0][0]), kBN * 128, 1024, tc::kSw128);
      const uint64_t dv1 = tc::smem_desc(smem_u32(&sm.vh[kStages - 1][0]), kBN * 128, 1024, tc::kSw128);
      static_assert(kStages == 2, "two descriptor bases per ring");
      // O_g += P_g . V over tile jt (stage st): kind::f16, K = 16 keys per MMA, P_g (f16 pairs)
      // from S_g's columns, V as f16 (both groups converted their shares: vh_full)
      auto issue_pv = [&](int g, int jt, int st) -> bool {
        if (!mbar_wait(&sm.p_full[g], jt & 1, p.err)) return false;
        if (g == 0 && !mbar_wait(&sm.vh_full[st], (jt / kStages) & 1, p.err)) return false;
        tc::fence_after_sync();
        const uint64_t dv = st ? dv1 : dv0;
        const uint32_t pt = tmem + 256 * g;
#pragma unroll
        for (int ks = 0; ks < kBN / 16; ++ks) {
          // V rows 16 ks .. + 15 (2 KB further per step): two 64-dim blocks kBN * 128 bytes
          // apart, 8-row groups 1 KB apart
          tc::mma_f16_ts(tmem + 256 * g + 128, pt + p_col(16 * ks & ~31) + ((16 * ks) & 16) / 2,
                         dv + static_cast<uint64_t>(ks * (16 * 128 >> 4)), idesc_pv,
                         (jt > 0 || ks > 0) ? 1u : 0u);
        }
        return true;
      };
      for (int j = 0; ok && j < ntiles; ++j) {
        const uint64_t dk = stage ? dk1 : dk0;
        for (int g = 0; g < NG && ok; ++g) {
          if (j > 0 && !issue_pv(g, j - 1, prev_stage)) { ok = false; break; }
          if (g == 0 && !mbar_wait(&sm.kv_full[stage], phase, p.err)) { ok = false; break; }
          const uint64_t dqh = tc::smem_desc(smem_u32(&sm.qhi[g][0]), 16, 1024, tc::kSw128);
          const uint64_t dql = tc::smem_desc(smem_u32(&sm.qlo[g][0]), 16, 1024, tc::kSw128);
#pragma unroll
          for (int plane = 0; plane < 2; ++plane)
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)  // 32 bytes further per step
              tc::mma_f8(tmem + 256 * g, (plane ? dql : dqh) + static_cast<uint64_t>(2 * ks),
                         dk + static_cast<uint64_t>(2 * ks), idesc_s, (plane > 0 || ks > 0) ? 1u : 0u);
          tc::commit(&sm.s_full[g]);
        }
        if (!ok) break;
        if (j > 0) tc::commit(&sm.kv_empty[prev_stage]);
        prev_stage = stage;
        if (++stage == kStages) { stage = 0; phase ^= 1; }
      }
      if (ok) {
        for (int g = 0; g < NG && ok; ++g) {
          ok = issue_pv(g, ntiles - 1, prev_stage);
          if (ok) tc::commit(&sm.s_full[g]);  // O_g final
        }
        if (ok) tc::commit(&sm.kv_empty[prev_stage]);
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
    const int h = h0 + g;
    const int r = 32 * (warp & 3) + lane;  // query row within the tile
    const bool row_ok = r < rows;
    const int qi = q0 + r;           // query index within the sequence
    const int lim = qi + (si.nk - si.nq);  // largest visible key position of this row
    const uint32_t lane_base = static_cast<uint32_t>(32 * (warp & 3)) << 16;
    const uint32_t s_tmem = tmem + lane_base + 256 * g;
    const uint32_t o_tmem = s_tmem + 128;
    uint8_t* const qhi = sm.qhi[g];
    uint8_t* const qlo = sm.qlo[g];
    uint32_t xphase = 0;
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
    // ---- query row -> e4m3 hi / lo, 128B-swizzled K-major rows (this half's dims)
    float cs;
    bool ok = true;
    {
      constexpr int kW = 16 / kNH;  // 16-byte loads of this half (8 bf16 each)
      uint4 w[kW];  // all loads in flight at once
      if (row_ok) {
        const uint4* src = reinterpret_cast<const uint4*>(
            p.q + static_cast<int64_t>(si.q_begin + qi) * p.q_row_stride + static_cast<int64_t>(h) * 128 + cb);
#pragma unroll
        for (int i = 0; i < kW; ++i) w[i] = ldg_keep_v4(src + i);
      } else {
#pragma unroll
        for (int i = 0; i < kW; ++i) w[i] = make_uint4(0, 0, 0, 0);
      }
      auto widen = [&](const uint4& v, float* x) {
        const uint32_t ww[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          x[2 * k] = __uint_as_float(ww[k] << 16);
          x[2 * k + 1] = __uint_as_float(ww[k] & 0xFFFF0000u);
        }
      };
      float amax = 0.f;
#pragma unroll
      for (int i = 0; i < kW; ++i) {
        float x[8];
        widen(w[i], x);
#pragma unroll
        for (int k = 0; k < 8; ++k) amax = fmaxf(amax, fabsf(x[k]));
      }
      if (kNH > 1) {
        sm.xq[g][half][r] = amax;
        ok = pair_exchange();
        amax = fmaxf(sm.xq[g][0][r], sm.xq[g][1][r]);
      }
      float srow;
      const float inv = pow2_inv_scale(amax, &srow);
      cs = srow * p.scale_log2;
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
    }
    fence_proxy_async_smem();
    mbar_arrive(&sm.q_full[g]);

    float m_ref = -INFINITY;  // reference max of O and l (log2 units)
    float l = 0.f;
    int stage = 0;
    uint32_t phase = 0;
    for (int j = 0; ok && j < ntiles; ++j) {
      if (!mbar_wait(&sm.kv_full[stage], phase, p.err)) { ok = false; break; }
      const int j0 = sm.tile[stage].j0;
      const uint32_t boxmask = sm.tile[stage].boxmask;  // boxes whose block is valid
      // key columns of this tile that can be valid at all (visible, inside this sequence)
      const int col_end = min(kBN, si.vis - j0);
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
      // across the group's four warps)
      const int vlim = row_ok ? max(0, min(col_end, lim - j0 + 1)) : 0;
      const bool general = kscaled || !(p.scale_log2 > 0.f) || boxmask != (1u << (kBN / box_rows)) - 1u;
      // S_g(j) complete => PV_g(j-1) complete (issued before it): O is quiescent
      if (!mbar_wait(&sm.s_full[g], j & 1, p.err)) { ok = false; break; }
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
            const int64_t slot = paged ? static_cast<int64_t>(sm.tile[stage].blk[c >> box_shift]) * bs + (kv % bs)
                                       : static_cast<int64_t>(si.k_begin) + kv;
            ks = __ldg(p.k_scale + slot * p.num_kv_heads + kvh);
            vs = __ldg(p.v_scale + slot * p.num_kv_heads + kvh);
          }
          sm.colk[g][c] = ks;
          sm.colv[g][c] = vs;
          const uint32_t bal = __ballot_sync(0xffffffffu, cok);
          if (lane == 0) sm.colok[g][warp & 3] = bal;
        }
        if (!exchange()) { ok = false; break; }
      }
      mbar_arrive(&sm.kv_empty[stage]);  // done with the tile's header and block list
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
    }
    // ---- epilogue: O / l -> fp16 -> bf16 (the reference's output path)
    if (ntiles > 0 && ok && kNH > 1) {  // the row sum over both halves
      sm.xl[g][half][r] = l;
      ok = pair_exchange();
      l = sm.xl[g][0][r] + sm.xl[g][1][r];
    }
    if (row_ok) {
      uint16_t* dst = p.out + static_cast<int64_t>(si.q_begin + qi) * p.out_row_stride + h * 128 + cb;
      if (ntiles == 0 || !ok) {
        for (int i = 0; i < kCols / 8; ++i) reinterpret_cast<uint4*>(dst)[i] = make_uint4(0, 0, 0, 0);
      }
    }
    if (ntiles > 0 && ok) {
      if (mbar_wait(&sm.s_full[g], ntiles & 1, p.err)) {
        tc::fence_after_sync();
        const float inv = l > 0.f ? 1.f / l : 0.f;  // O and l carry the same factor 16
#pragma unroll
        for (int c0 = cb; c0 < cb + kCols; c0 += 16) {
          float o16[16];
          tc::ld16(o_tmem + c0, o16);
          tc::wait_ld();
          if (row_ok) {
            uint32_t pk[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              __nv_bfloat16 a = out_round(o16[2 * i] * inv), b = out_round(o16[2 * i + 1] * inv);
              pk[i] = static_cast<uint32_t>(*reinterpret_cast<uint16_t*>(&a)) |
                      (static_cast<uint32_t>(*reinterpret_cast<uint16_t*>(&b)) << 16);
            }
            uint4* dst = reinterpret_cast<uint4*>(
                p.out + static_cast<int64_t>(si.q_begin + qi) * p.out_row_stride + h * 128 + c0);
            dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
          }
        }
      }
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == Cfg::kMmaWarp) tc::tmem_dealloc(tmem, Cfg::kTmemCols);
}

template <int NG>
cudaError_t launch_groups(const PrefillParams& p, const CUtensorMap& tmk, const CUtensorMap& tmv,
                          cudaStream_t stream) {
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  const size_t smem = sizeof(PrefillSmem<NG>) + 1024;
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaFuncSetAttribute(prefill_kernel<NG>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(smem));
    configured[dev] = true;
  }
  const dim3 grid((p.max_seqlen_q + kBM - 1) / kBM, p.num_heads / NG, p.num_seqs);
  prefill_kernel<NG><<<grid, PrefillCfg<NG>::kThreads, smem, stream>>>(tmk, tmv, p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_prefill(const PrefillParams& p, cudaStream_t stream) {
  const bool paged = p.block_tables != nullptr;
  const int box_rows = box_rows_of(paged, p.block_size);
  const int64_t rows = paged ? p.num_blocks * p.block_size : p.num_blocks;
  CUtensorMap tmk, tmv;
  if (!make_map(&tmk, p.k, rows, p.kv_row_stride, p.num_kv_heads, box_rows) ||
      !make_map(&tmv, p.v, rows, p.kv_row_stride, p.num_kv_heads, box_rows))
    return cudaErrorInvalidValue;
  // The per-item grid launches a CTA for every (q tile below max_seqlen_q, head pair, sequence),
  // work or not; an empty CTA still costs its scheduling (about 4.5 ns each, amortised over the
  // SMs: 55 us for the 12k of a 192-sequence verify batch).  Past kPersistentCtas of them the
  // persistent kernel, whose CTAs claim only real items, takes the call; below, the per-item
  // kernel, which has no per-item bookkeeping in its tile loop, is the faster one.
  const int ng = p.group % 2 == 0 ? 2 : 1;
  const int64_t ctas = static_cast<int64_t>(p.num_seqs) * ((p.max_seqlen_q + kBM - 1) / kBM) *
                       (p.num_heads / ng);
  if (ctas > kPersistentCtas) return launch_prefill_persistent(p, tmk, tmv, stream);
  // two q heads of one kv head per CTA when the GQA group is even
  return ng == 2 ? launch_groups<2>(p, tmk, tmv, stream) : launch_groups<1>(p, tmk, tmv, stream);
}

}  // namespace fp8attn
