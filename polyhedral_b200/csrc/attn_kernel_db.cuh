// The 64-row super-tile variant of the block-sparse attention forward (opt-in,
// pa_attn_args.kv_rows = 64).  Same work items, plan, warp roles, masks and epilogue
// as the default kernel in attn_kernel.cuh, but KV super-tiles are 64 rows and each
// half's S is double-buffered in TMEM:
//   TMEM: S/P half 0 buffers [0,64) [64,128), half 1 [128,192) [192,256),
//         O0 [256, 256+D), O1 [256+D, 256+2D)
// so the MMA warp computes S(j+1) while the softmax warps work on S(j).  Per
// super-tile g (buffer g & 1) it issues S_h(g) for both halves, then P_h(g-1).V(g-1)
// from buffer (g-1) & 1; S(g+2) reuses a buffer only after the P.V that reads P from
// it has been issued ahead of it.  The K/V ring has 8 slots of 64-row tiles; K(g)
// sits at ring position 2g and V(g) at 2g + 1.  This removes the per-half chain
// softmax -> P.V + next S -> softmax of the default kernel at the price of an N = 64
// S-MMA (bounded by shared-memory reads of Q) and twice as many per-tile steps; it is
// faster where per-tile mask work is heavy (many partial tiles), slower on mostly
// full tiles.  Each half computes only the super-tiles live for it (the plan's
// per-half status): a band narrower than the item's 256 rows leaves each half tiles
// that only the other half needs, and skipping them gives the same result (a dead
// tile adds exact zeros and never raises the running maximum).
#pragma once
#include "attn_kernel.cuh"

namespace pa {
namespace attn {
namespace db {

constexpr int BN = 64;           // KV rows per super-tile
constexpr int kDescAhead = 2;    // super-tiles of plan descriptors loaded ahead

template <int D>
struct Smem {
  static constexpr int kQTileBytes = BM * D * 2;    // one 128-row Q tile, 16-bit
  static constexpr int kKVTileBytes = BN * D * 2;   // one 64-row K or V tile
  static constexpr int kQRegion = BM * 128;         // one 64-column chunk of a Q tile
  static constexpr int kKVRegion = BN * 128;        // one 64-column chunk of a K/V tile
  static constexpr int kSlots = 8;
  static constexpr int kQOff = 0;
  static constexpr int kKVOff = 2 * kQTileBytes;
  static constexpr int kBarOff = kKVOff + kSlots * kKVTileBytes;
  // barriers: q_full[2] q_empty[2] s_full[2][2] p_full[2][2] pv_done[2] o_full[2] drain
  //           item_full[2] item_empty[2] kv_full[S] kv_empty[S]
  static constexpr int kNumBars = 21 + 2 * kSlots;
  static constexpr int kMiscOff = kBarOff + 8 * kNumBars;    // tmem base, abort
  static constexpr int kSlotOff = kMiscOff + 16;               // item ring: ItemSlot[2]
  // epilogue staging [8 warps][32 rows][128 B], 128-byte swizzled boxes for the O
  // tensor map (1024-byte aligned)
  static constexpr int kEpiOff = (kSlotOff + 2 * (int)sizeof(ItemSlot) + 1023) & ~1023;
  static constexpr int kBytes = kEpiOff + 8 * 32 * 128;
  static constexpr int kAlloc = kBytes + 1024;                 // room to align to 1024
};


struct SegInfo64 {
  int row0;
  int st;
};

template <int L>
__device__ __forceinline__ int num_super64(const FwdParams& P, int cnt) {
  constexpr int S = BN / L;
  if (P.A <= BN) return (cnt + S - 1) / S;
  return cnt * (P.A / BN);
}

template <int L>
__device__ __forceinline__ SegInfo64 seg_info64(const FwdParams& P, const int32_t* ent,
                                            const uint8_t* sts, int cnt, int u, int sg) {
  constexpr int S = BN / L;
  if (P.A <= BN) {
    const int e = u * S + sg;
    if (e < cnt) return SegInfo64{__ldg(ent + e) * P.A, (int)__ldg(sts + e)};
    return SegInfo64{P.N, 0};
  }
  const int sub = P.A / BN;
  const int e = u / sub;
  return SegInfo64{__ldg(ent + e) * P.A + (u - e * sub) * BN, (int)__ldg(sts + e)};
}

template <int D, int L, bool kBf16, bool kRS>
__global__ void __launch_bounds__(kThreads, 1)
attn_fwd_db_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ FwdParams P) {
  using SM = Smem<D>;
  constexpr int S = BN / L;              // segments per super-tile
  constexpr int NS = SM::kSlots;
  constexpr int kChunks = D / 64;        // 128-byte swizzle chunks along D

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sQ = smem + SM::kQOff;
  uint8_t* sKV = smem + SM::kKVOff;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM::kBarOff);
  uint64_t* q_full = bars + 0;
  uint64_t* q_empty = bars + 2;
  uint64_t* s_full = bars + 4;     // [half][buffer]
  uint64_t* p_full = bars + 8;     // [half][buffer]
  uint64_t* pv_done = bars + 12;   // [half]
  uint64_t* o_full = bars + 14;
  uint64_t* drain = bars + 16;
  uint64_t* item_full = bars + 17;
  uint64_t* item_empty = bars + 19;
  uint64_t* kv_full = bars + 21;
  uint64_t* kv_empty = bars + 21 + NS;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + SM::kMiscOff);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + SM::kMiscOff + 4);
  ItemSlot* s_slot = reinterpret_cast<ItemSlot*>(smem + SM::kSlotOff);   // [2]
  uint8_t* sEpi = smem + SM::kEpiOff;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const ErrSink& err = P.err;   // read from the parameter space where used

  if (threadIdx.x == 0) {
    for (int h = 0; h < 2; ++h) {
      mbar_init(&q_full[h], 1);
      mbar_init(&q_empty[h], 1);
      mbar_init(&pv_done[h], 1);
      mbar_init(&o_full[h], 1);
      for (int b = 0; b < 2; ++b) {
        mbar_init(&s_full[h * 2 + b], 1);
        mbar_init(&p_full[h * 2 + b], BM);
      }
    }
    mbar_init(drain, 1);
    for (int r = 0; r < 2; ++r) {
      mbar_init(&item_full[r], 1);
      mbar_init(&item_empty[r], 1 + 8);   // MMA thread + one lane per softmax warp
    }
    for (int s = 0; s < NS; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    *s_abort = 0;
    fence_barrier_init();
  }
  if (warp == kLoadWarp && lane == 0) {
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
  }
  if (warp == kMmaWarp) {
    tmem_alloc(s_tmem, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  if (warp >= 8) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kOtherRegs));
  if (warp == kLoadWarp) {
    // ------------------------------------------------------------ producer
    // K/V ring positions: super-tile g puts K at 2g and V at 2g + 1; position p
    // lives in slot p % NS.
    if (lane == 0) {
      int qi = 0;
      int q_armed[2] = {0, 0};
      uint32_t kv_g = 0;
      uint32_t ring = 0;
      while (true) {
        // fetch the next work item and hand it to the MMA and softmax warps
        int it = atomicAdd(P.pv.sched, 1);
        if (it >= P.total_items || *s_abort) it = -1;
        // the ring entry: the item, its pair and (batch, head), the list length and the
        // first super-tile's plan descriptors
        const uint32_t rs = ring & 1;
        if (ring >= 2 &&
            !mbar_wait(&item_empty[rs], ((ring >> 1) - 1) & 1, s_abort, err, DEV_TIMEOUT_ITEM))
          break;
        ItemSlot& sl = s_slot[rs];
        sl.it = it;
        if (it >= 0) {
          int pp, bb;
          item_coords(P, it, pp, bb);
          const int cc = __ldg(P.pv.pair_cnt + pp);
          sl.p = pp;
          sl.bh = bb;
          sl.cnt = cc;
          if constexpr (S <= 2) {
            const uint2* desc = P.pv.desc + (size_t)pp * P.pv.cap;
#pragma unroll
            for (int sg = 0; sg < S; ++sg) {
              const int e = P.A <= BN ? sg : 0;
              sl.d0[sg] = e < cc ? __ldg(desc + e) : make_uint2(0u, 0u);
            }
          }
        }
        mbar_arrive(&item_full[rs]);
        ++ring;
        if (it < 0) break;
        const int p = sl.p, bh = sl.bh, cnt = sl.cnt;
        const int nsup = num_super64<L>(P, cnt);
        if (nsup == 0) continue;
        const int32_t* ent = P.pv.entries + (size_t)p * P.pv.cap;
        const uint8_t* sts = P.pv.status + (size_t)p * P.pv.cap;
        bool ok = true;
        for (int h = 0; h < 2 && ok; ++h) {
          if (qi > 0) ok = mbar_wait(&q_empty[h], (qi - 1) & 1, s_abort, err, DEV_TIMEOUT_Q);
          if (!ok) break;
          // test hook (pa_attn_fwd_withheld): the first item's half-0 Q tile is never
          // loaded, so the MMA warp's bounded wait on it runs out
          if (qi == 0 && h == 0 && P.withhold_q) continue;
          mbar_arrive_expect_tx(&q_full[h], SM::kQTileBytes);
          ++q_armed[h];
          const int qr = p * 2 * BM + h * BM;
          for (int c = 0; c < kChunks; ++c) {
            if constexpr (kRS)
              tma_load_4d(sQ + h * SM::kQTileBytes + c * SM::kQRegion, &tm_q, &q_full[h], c * 64,
                          qr / P.nb, qr % P.nb, bh);
            else
              tma_load_3d(sQ + h * SM::kQTileBytes + c * SM::kQRegion, &tm_q, &q_full[h], c * 64,
                          qr, bh);
          }
        }
        if (!ok) break;
        for (int u = 0; u < nsup && ok; ++u) {
          SegInfo64 si[S];
#pragma unroll
          for (int sg = 0; sg < S; ++sg) si[sg] = seg_info64<L>(P, ent, sts, cnt, u, sg);
          for (int kv = 0; kv < 2; ++kv) {
            const uint32_t slot = kv_g % NS;
            if (kv_g >= (uint32_t)NS) {
              ok = mbar_wait(&kv_empty[slot], ((kv_g / NS) - 1) & 1, s_abort, err,
                             DEV_TIMEOUT_KV);
              if (!ok) break;
            }
            ++kv_g;
            uint8_t* dst = sKV + slot * SM::kKVTileBytes;
            mbar_arrive_expect_tx(&kv_full[slot], SM::kKVTileBytes);
            const void* tm = kv == 0 ? (const void*)&tm_k : (const void*)&tm_v;
#pragma unroll
            for (int sg = 0; sg < S; ++sg) {
              const int r0 = si[sg].row0;
              for (int c = 0; c < kChunks; ++c) {
                if constexpr (kRS)
                  tma_load_4d(dst + c * SM::kKVRegion + sg * L * 128, tm, &kv_full[slot], c * 64,
                              r0 / P.nb, r0 % P.nb, bh);
                else
                  tma_load_3d(dst + c * SM::kKVRegion + sg * L * 128, tm, &kv_full[slot], c * 64,
                              r0, bh);
              }
            }
          }
        }
        ++qi;
      }
      // Teardown: let every copy this thread issued land before the CTA can exit.
      // A phase that completed long ago also satisfies the parity test, so this
      // only ever waits on copies still in flight.
      const uint64_t t0 = globaltimer();
      for (uint32_t s = 0; s < (uint32_t)NS && s < kv_g; ++s) {
        const uint32_t uses = (kv_g - s + NS - 1) / NS;   // loads issued into slot s
        while (!mbar_try_wait(&kv_full[s], (uses - 1) & 1)) {
          if (globaltimer() - t0 > kDrainLimitNs) { err.record(DEV_TIMEOUT_DRAIN); break; }
        }
      }
      for (int h = 0; h < 2; ++h) {
        if (q_armed[h] == 0) continue;
        while (!mbar_try_wait(&q_full[h], (q_armed[h] - 1) & 1)) {
          if (globaltimer() - t0 > kDrainLimitNs) { err.record(DEV_TIMEOUT_DRAIN); break; }
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    // Per super-tile g: S_h(g) for each half h it is live for, into that half's S
    // buffer gh[h] & 1 (gh[h] counts half h's live super-tiles), then the P.V of
    // super-tile g - 1 for the halves live in it.  S_h(next) therefore runs while the
    // softmax works on S_h(current); a buffer is rewritten only after the P.V that
    // reads P from it has been issued ahead of it in this thread's order.
    if (lane == 0) {
      int qi = 0;
      uint32_t g = 0;                   // super-tiles issued so far (all items)
      bool ok = true;
      const uint32_t sQa = smem_u32(sQ), sKVa = smem_u32(sKV);
      auto wait_pos = [&](uint32_t pos) -> bool {
        const bool r = mbar_wait(&kv_full[pos % NS], (pos / NS) & 1, s_abort, err, DEV_TIMEOUT_KV);
        tc_fence_after();
        return r;
      };
      const uint64_t q_desc[2] = {smem_desc_sw128(sQa, 16),
                                  smem_desc_sw128(sQa + SM::kQTileBytes, 16)};
      auto issue_s = [&](int h, uint32_t kslot, uint32_t b) {
        const uint32_t d = tmem + h * 128 + b * 64;
        const uint64_t qd = q_desc[h];
        const uint64_t kd = smem_desc_sw128(sKVa + kslot * SM::kKVTileBytes, 16);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t qo = ((kk >> 2) * SM::kQRegion + (kk & 3) * 32) >> 4;
          const uint64_t ko = ((kk >> 2) * SM::kKVRegion + (kk & 3) * 32) >> 4;
          mma_ss(d, qd + qo, kd + ko, P.idesc_qk, kk > 0);
        }
      };
      auto issue_pv = [&](int h, uint32_t vslot, uint32_t b, bool acc) {
        const uint32_t d = tmem + 256 + h * D;
        const uint32_t pa_ = tmem + h * 128 + b * 64 + 32;
        const uint64_t vd = smem_desc_sw128(sKVa + vslot * SM::kKVTileBytes, SM::kKVRegion);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk)
          mma_ts(d, pa_ + kk * 8, vd + (uint64_t)((kk * 16 * 128) >> 4), P.idesc_pv,
                 (acc || kk > 0) ? 1u : 0u);
      };
      // whether any segment of super-tile u is live for half h
      auto live_of = [&](const uint8_t* sts, int cnt, int u, int h) -> bool {
        bool lv = false;
#pragma unroll
        for (int sg = 0; sg < S; ++sg) {
          const int e = P.A <= BN ? u * S + sg : u / (P.A / BN);
          if (e < cnt) lv |= ((__ldg(sts + e) >> (2 * h)) & 3u) != 0;
        }
        return lv;
      };
      // P.V of super-tile gp for the halves live in it (pd); pc = that tile's count
      // among the half's live tiles, pacc = whether it accumulates (not the half's
      // first live tile of the item)
      uint32_t gh[2] = {0, 0};
      auto pv_step = [&](uint32_t gp, const bool (&pd)[2], const uint32_t (&pc)[2],
                         const bool (&pacc)[2]) -> bool {
        if (!wait_pos(2 * gp + 1)) return false;
        const uint32_t vslot = (2 * gp + 1) % NS;
        for (int h = 0; h < 2; ++h) {
          if (!pd[h]) continue;
          const uint32_t b = pc[h] & 1;
          if (!mbar_wait(&p_full[h * 2 + b], (pc[h] >> 1) & 1, s_abort, err, DEV_TIMEOUT_P))
            return false;
          tc_fence_after();
          issue_pv(h, vslot, b, pacc[h]);
          tc_commit(&pv_done[h]);
        }
        tc_commit(&kv_empty[vslot]);
        return true;
      };
      uint32_t ring = 0;
      while (ok) {
        const uint32_t rs = ring & 1;
        if (!(ok = mbar_wait(&item_full[rs], (ring >> 1) & 1, s_abort, err, DEV_TIMEOUT_ITEM)))
          break;
        const int it = s_slot[rs].it, p = s_slot[rs].p, cnt = s_slot[rs].cnt;
        mbar_arrive(&item_empty[rs]);
        ++ring;
        if (it < 0) break;
        const int nsup = num_super64<L>(P, cnt);
        if (nsup == 0) continue;
        const uint8_t* sts = P.pv.status + (size_t)p * P.pv.cap;
        ok = mbar_wait(&q_full[0], qi & 1, s_abort, P.err_q, DEV_TIMEOUT_Q) &&
             mbar_wait(&q_full[1], qi & 1, s_abort, P.err_q, DEV_TIMEOUT_Q);
        tc_fence_after();
        if (!ok) break;
        bool pd[2] = {false, false}, pacc[2] = {false, false}, seen[2] = {false, false};
        uint32_t pc[2] = {0, 0};
        bool lv_next[2] = {live_of(sts, cnt, 0, 0), live_of(sts, cnt, 0, 1)};
        for (int u = 0; u < nsup && ok; ++u, ++g) {
          const bool lv[2] = {lv_next[0], lv_next[1]};
          if (u + 1 < nsup) {   // read a tile ahead, off the issue path
            lv_next[0] = live_of(sts, cnt, u + 1, 0);
            lv_next[1] = live_of(sts, cnt, u + 1, 1);
          }
          if (!(ok = wait_pos(2 * g))) break;
          const uint32_t kslot = (2 * g) % NS;
          for (int h = 0; h < 2; ++h) {
            if (lv[h]) {
              issue_s(h, kslot, gh[h] & 1);
              tc_commit(&s_full[h * 2 + (gh[h] & 1)]);
            }
            if (u == nsup - 1) tc_commit(&q_empty[h]);   // the item's last read of Q_h
          }
          tc_commit(&kv_empty[kslot]);
          if (u > 0 && !(ok = pv_step(g - 1, pd, pc, pacc))) break;
          for (int h = 0; h < 2; ++h) {
            pd[h] = lv[h];
            if (lv[h]) {
              pc[h] = gh[h]++;
              pacc[h] = seen[h];
              seen[h] = true;
            }
          }
        }
        if (!ok) break;
        if (!(ok = pv_step(g - 1, pd, pc, pacc))) break;
        for (int h = 0; h < 2; ++h) tc_commit(&o_full[h]);
        ++qi;
      }
      // drain: the commit lands once every MMA issued above has completed
      tc_commit(drain);
      const uint64_t t0 = globaltimer();
      while (!mbar_try_wait(drain, 0)) {
        if (globaltimer() - t0 > kDrainLimitNs) { err.record(DEV_TIMEOUT_DRAIN); break; }
      }
    }
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kSoftmaxRegs));
    // ------------------------------------------------------------ softmax + epilogue
    const int h = warp >> 2;              // which half
    const int wq = warp & 3;              // TMEM lane quarter
    const int r_in = wq * 32 + lane;      // row within the half
    const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
    const uint32_t tS = tmem + lane_off + h * 128;   // + b * 64 for buffer b
    const uint32_t tO = tmem + lane_off + 256 + h * D;
    uint32_t gh = 0, to = 0;             // this half's live super-tiles so far (all items)
    const float c2 = P.scale_log2;
    uint32_t ring = 0;
    while (true) {
      const uint32_t rs = ring & 1;
      bool got = mbar_wait(&item_full[rs], (ring >> 1) & 1, s_abort, err, DEV_TIMEOUT_ITEM);
      if (!__all_sync(0xffffffffu, got)) break;
      const int it = s_slot[rs].it, p = s_slot[rs].p, bh = s_slot[rs].bh, cnt = s_slot[rs].cnt;
      uint2 d0[S];   // the first super-tile's descriptors, from the ring entry (S <= 2)
#pragma unroll
      for (int sg = 0; sg < S; ++sg) d0[sg] = S <= 2 ? s_slot[rs].d0[sg] : make_uint2(0u, 0u);
      __syncwarp();
      if (lane == 0) mbar_arrive(&item_empty[rs]);
      ++ring;
      if (it < 0) break;
      const int nsup = num_super64<L>(P, cnt);
      const int32_t* ent = P.pv.entries + (size_t)p * P.pv.cap;
      const uint2* desc = P.pv.desc + (size_t)p * P.pv.cap;
      const int row = p * 2 * BM + h * BM + r_in;
      const bool valid = row < P.N;
      const int irow = !valid        ? -(1 << 30)
                       : kRS          ? (row % P.nb) * P.rs + row / P.nb
                       : P.perm_q    ? __ldg(P.perm_q + row)
                                     : row;
      // plan descriptors of super-tile u's segments (the next tile's are loaded one
      // tile ahead)
      // Loads are issued as volatile so that they stay where they are written, a
      // whole tile (or kDescAhead tiles) before their use.
      auto load_desc = [&](int u, uint2 (&d)[S]) {
#pragma unroll
        for (int sg = 0; sg < S; ++sg) {
          const int e = P.A <= BN ? u * S + sg : u / (P.A / BN);
          d[sg] = make_uint2(0u, 0u);
          if (u < nsup && e < cnt)
            asm volatile("ld.global.nc.v2.u32 {%0, %1}, [%2];"
                         : "=r"(d[sg].x), "=r"(d[sg].y) : "l"(desc + e));
        }
      };
      uint2 dnext[kDescAhead][S];
      if constexpr (S <= 2) {
#pragma unroll
        for (int sg = 0; sg < S; ++sg) dnext[0][sg] = d0[sg];
      } else {
        load_desc(0, dnext[0]);
      }
#pragma unroll
      for (int a = 1; a < kDescAhead; ++a) load_desc(a, dnext[a]);
      float m_used = -INFINITY, l = 0.f;
      bool ok = true, first = true;        // first: no live super-tile yet in this item
      // the previous item's box stores have read the staging: waited for here, while
      // the item's first S is still in flight
      if (lane == 0) bulk_wait_read();
      for (int u = 0; u < nsup; ++u) {
        const uint32_t b = gh & 1;
        uint2 dcur[S];
#pragma unroll
        for (int sg = 0; sg < S; ++sg) dcur[sg] = dnext[0][sg];
#pragma unroll
        for (int a = 0; a + 1 < kDescAhead; ++a)
#pragma unroll
          for (int sg = 0; sg < S; ++sg) dnext[a][sg] = dnext[a + 1][sg];
        load_desc(u + kDescAhead, dnext[kDescAhead - 1]);
        // a super-tile dead for this half is not computed for it (the MMA warp skips
        // it from the same status bits)
        {
          bool live = false;
#pragma unroll
          for (int sg = 0; sg < S; ++sg) live |= ((dcur[sg].y >> (24 + 2 * h)) & 3u) != 0;
          if (!live) continue;
        }
        // live bits of this row for the tile's 64 columns
        uint32_t mk[2];
        {
          int sub = 0;
          if (P.A > BN) sub = u - (u / (P.A / BN)) * (P.A / BN);
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            uint32_t w = 0;
#pragma unroll
            for (int part = 0; part < (L >= 32 ? 1 : 2); ++part) {
              const int sg = L >= 32 ? k * 32 / L : 2 * k + part;
              const int base = L >= 32 ? (k * 32) % L : 0;
              const int nb = L >= 32 ? 32 : 16;
              const uint2 d = dcur[sg];
              const int st = (d.y >> (24 + 2 * h)) & 3;
              uint32_t bits = st == 1 ? 0xffffffffu : 0u;
              if (st == 2) {
                const int dj = (int)(d.y & 0xffffu);
                const int sh = (d.y & (1u << 20)) ? (int)((d.y >> 16) & 15u) : -1;
                const int j0 = (int)d.x + sub * BN * dj;
                if (!(((d.y >> 21) & 1u) &&
                      progression_bits(P.pred, irow - j0, j0, dj, sh, base, L, bits))) {
                  const int e = P.A <= BN ? u * S + sg : u / (P.A / BN);
                  const int32_t* cols =
                      P.perm_kv ? P.perm_kv + __ldg(ent + e) * P.A + sub * BN + base : nullptr;
                  bits = element_bits(P.pred, irow, cols, j0, dj, base, nb);
                }
              }
              if (nb == 16) bits &= 0xffffu;
              w |= bits << (16 * part);
            }
            mk[k] = w;
          }
        }
        ok = mbar_wait(&s_full[h * 2 + b], (gh >> 1) & 1, s_abort, err, DEV_TIMEOUT_S);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        tc_fence_after();
        float s[64];
        {
          uint32_t r0[32], r1[32];
          tmem_ld32(tS + b * 64, r0);
          tmem_ld32(tS + b * 64 + 32, r1);
          tmem_wait_ld();
          tmem_regs_ready(r0);
          tmem_regs_ready(r1);
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            s[i] = __uint_as_float(r0[i]);
            s[32 + i] = __uint_as_float(r1[i]);
          }
        }
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          if (mk[k] != 0xffffffffu) {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (!((mk[k] >> i) & 1u)) s[k * 32 + i] = -INFINITY;
          }
        }
        float mx;
        {
          float m8[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) m8[j] = fmaxf(s[2 * j], s[2 * j + 1]);
#pragma unroll
          for (int c = 16; c < 64; c += 16) {
#pragma unroll
            for (int j = 0; j < 8; ++j) m8[j] = fmax3(m8[j], s[c + 2 * j], s[c + 2 * j + 1]);
          }
          mx = fmax3(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]));
        }
        const float m_tile = mx * c2;
        const float m_new = fmaxf(m_used, m_tile);
        bool bump = false;
        float factor = 1.f;
        if (first) {
          m_used = m_new;
        } else if (m_new > m_used + 8.0f) {
          bump = true;
          factor = ex2(m_used - m_new);
          m_used = m_new;
        }
        const bool need_o = bump && l > 0.f;
        if (bump) l *= factor;
        const float msub = m_used == -INFINITY ? 0.f : m_used;
        float r8[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) r8[j] = 0.f;
#pragma unroll
        for (int q2 = 0; q2 < 2; ++q2) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int c = q2 * 32 + 2 * i;
            float x0, x1;
            ffma2(x0, x1, s[c], s[c + 1], c2, -msub);
            float a, b2;
            exp2_pair(i, x0, x1, a, b2);
            const int j = (2 * i) & 7;
            fadd2(r8[j], r8[j + 1], a, b2);
            pk[i] = pack2<kBf16>(a, b2);
          }
          tmem_st16(tS + b * 64 + 32 + q2 * 16, pk);
        }
        l += ((r8[0] + r8[1]) + (r8[2] + r8[3])) + ((r8[4] + r8[5]) + (r8[6] + r8[7]));
        // O rescale (rare: only when the running max grew by more than 2^8).  The
        // previous tile's P.V may still be running: wait for it first.
        if (__any_sync(0xffffffffu, need_o)) {
          ok = mbar_wait(&pv_done[h], (gh - 1) & 1, s_abort, err, DEV_TIMEOUT_P);
          if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
          tc_fence_after();
          const float f = need_o ? factor : 1.f;
#pragma unroll 1
          for (int k = 0; k < D / 32; ++k) {
            uint32_t r[32];
            tmem_ld32(tO + k * 32, r);
            tmem_wait_ld();
            tmem_regs_ready(r);
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * f);
            tmem_st32(tO + k * 32, r);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&p_full[h * 2 + b]);
        first = false;
        ++gh;
      }
      if (!ok) break;
      // epilogue: O / l, LSE
      float inv_l = l > 0.f ? 1.f / l : 0.f;
      const float lse_v = l > 0.f ? (m_used + __log2f(l)) * 0.69314718055994530942f : -INFINITY;
      char* orow = nullptr;
      if (valid) {
        const int orw = kRS          ? (row % P.nb) * P.rs + row / P.nb
                        : P.o_row_map ? __ldg(P.o_row_map + row)
                                      : row;
        if ((unsigned)orw < (unsigned)P.N) {
          orow = static_cast<char*>(P.o) +
                 ((long long)bh * P.o_bh_stride + (long long)orw * P.o_row_stride) * 2;
          if (P.lse) P.lse[(long long)bh * P.lse_bh_stride + orw] = lse_v;
        }
      }
      // O leaves through the warp's staging buffer, 32 rows x 64 columns at a time: the
      // warp writes its rows into a 128-byte-swizzled box and one lane stores it with a
      // TMA instruction through the O tensor map (rows in the kernel's order, or in
      // original order through the residue view).  Rows scattered by o_row_map are
      // written lane by lane, whole 128-byte row segments at a time.
      uint8_t* stage = sEpi + warp * (32 * 128);
      // the MMA warp signals o_full for every item with super-tiles; O holds this
      // half's result only if it had a live one
      const bool have_o = nsup > 0;
      if (have_o) {
        ok = mbar_wait(&o_full[h], to & 1, s_abort, err, DEV_TIMEOUT_O);
        ++to;
        if (!__all_sync(0xffffffffu, ok)) break;
        tc_fence_after();
      }
      if (P.o_row_map == nullptr) {
        const int wrow0 = p * 2 * BM + h * BM + wq * 32;   // the warp's first row
#pragma unroll 1
        for (int dh = 0; dh < D / 64; ++dh) {
          uint32_t r0[32], r1[32];
          if (have_o && !first) {
            tmem_ld32(tO + dh * 64, r0);
            tmem_ld32(tO + dh * 64 + 32, r1);
            tmem_wait_ld();
            tmem_regs_ready(r0);
            tmem_regs_ready(r1);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) r0[i] = r1[i] = 0u;
          }
          if (lane == 0 && dh > 0) bulk_wait_read();   // the previous box store has read it
          __syncwarp();
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            uint32_t w4[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int col = 8 * (c & 3) + 2 * j;
              w4[j] = pack2<kBf16>(__uint_as_float(c < 4 ? r0[col] : r1[col]) * inv_l,
                                   __uint_as_float(c < 4 ? r0[col + 1] : r1[col + 1]) * inv_l);
            }
            *reinterpret_cast<uint4*>(stage + lane * 128 + ((c ^ (lane & 7)) << 4)) =
                make_uint4(w4[0], w4[1], w4[2], w4[3]);
          }
          fence_proxy_async_shared();          // the rows are written before TMA reads them
          __syncwarp();
          if (lane == 0) {
            if constexpr (kRS)
              tma_store_4d(&P.tm_o, stage, dh * 64, wrow0 / P.nb, wrow0 % P.nb, bh);
            else
              tma_store_3d(&P.tm_o, stage, dh * 64, wrow0, bh);
            bulk_commit();
          }
        }
        if (have_o) tc_fence_before();
        continue;
      }
#pragma unroll
      for (int dh = 0; dh < D / 64; ++dh) {
        uint32_t w[32];   // 64 outputs of this row, packed in pairs
        if (have_o && !first) {
          uint32_t r0[32], r1[32];
          tmem_ld32(tO + dh * 64, r0);
          tmem_ld32(tO + dh * 64 + 32, r1);
          tmem_wait_ld();
          tmem_regs_ready(r0);
          tmem_regs_ready(r1);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            w[i] = pack2<kBf16>(__uint_as_float(r0[2 * i]) * inv_l,
                                __uint_as_float(r0[2 * i + 1]) * inv_l);
            w[16 + i] = pack2<kBf16>(__uint_as_float(r1[2 * i]) * inv_l,
                                     __uint_as_float(r1[2 * i + 1]) * inv_l);
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) w[i] = 0u;
        }
        __syncwarp();   // the previous round's readers are done with the buffer
#pragma unroll
        for (int c = 0; c < 8; ++c)
          *reinterpret_cast<uint4*>(stage + lane * 128 + ((c ^ (lane & 7)) << 4)) =
              make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
        __syncwarp();
        const int c = lane & 7;
#pragma unroll
        for (int it = 0; it < 8; ++it) {
          const int rr = it * 4 + (lane >> 3);
          const uint4 v = *reinterpret_cast<const uint4*>(stage + rr * 128 + ((c ^ (rr & 7)) << 4));
          const unsigned long long dst =
              __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(orow), rr);
          if (dst) *reinterpret_cast<uint4*>(reinterpret_cast<char*>(dst) + dh * 128 + c * 16) = v;
        }
      }
      if (have_o) tc_fence_before();
    }
  }

  // ------------------------------------------------------------ teardown
  // every box store has completed before the CTA can exit
  if (warp < 8 && lane == 0) bulk_wait_all();
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp) tmem_dealloc(tmem, kTmemCols);
  if (threadIdx.x == 0) {
    // the last CTA to finish rewinds the work counter for the next launch
    __threadfence();
    if (atomicAdd(P.pv.sched + 1, 1) == (int)gridDim.x - 1) {
      atomicExch(P.pv.sched, 0);
      atomicExch(P.pv.sched + 1, 0);
      atomicExch(P.pv.done, (int32_t)P.err.epoch);   // every CTA has recorded its status
    }
  }
}


template <int D, bool kRS>
int launch_family_db(const Tmap& tq, const Tmap& tk, const Tmap& tv, const FwdParams& P, int grid,
                  int L, bool bf16, cudaStream_t stream) {
  auto go = [&](auto kernel) -> int {
    const int smem = Smem<D>::kAlloc;
    PA_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
            "pa_attn_fwd");
    // the warpgroups' setmaxnreg shares must fit in what the CTA is launched with
    static std::atomic<int> regs_ok{0};   // checked once per instantiation
    cudaFuncAttributes fa;
    fa.numRegs = 1 << 20;
    if (!regs_ok.load(std::memory_order_relaxed))
      PA_CUDA(cudaFuncGetAttributes(&fa, kernel), "pa_attn_fwd");
    if (fa.numRegs * kThreads < 2 * 128 * kSoftmaxRegs + 128 * kOtherRegs)
      return fail(PA_ERR_UNSUPPORTED, "pa_attn_fwd: 64-row kernel built with %d registers per "
                  "thread, below its register split", fa.numRegs);
    regs_ok.store(1, std::memory_order_relaxed);
    kernel<<<grid, kThreads, smem, stream>>>(tq, tk, tv, P);
    return PA_OK;
  };
  switch (L) {
    case 16: return bf16 ? go(attn_fwd_db_kernel<D, 16, true, kRS>) : go(attn_fwd_db_kernel<D, 16, false, kRS>);
    case 32: return bf16 ? go(attn_fwd_db_kernel<D, 32, true, kRS>) : go(attn_fwd_db_kernel<D, 32, false, kRS>);
    default: return bf16 ? go(attn_fwd_db_kernel<D, 64, true, kRS>) : go(attn_fwd_db_kernel<D, 64, false, kRS>);
  }
}

int launch_d128(const Tmap& tq, const Tmap& tk, const Tmap& tv, const FwdParams& P, int grid, int L,
                bool bf16, cudaStream_t stream);
int launch_d128_residue(const Tmap& tq, const Tmap& tk, const Tmap& tv, const FwdParams& P,
                        int grid, int L, bool bf16, cudaStream_t stream);
int launch_d64(const Tmap& tq, const Tmap& tk, const Tmap& tv, const FwdParams& P, int grid, int L,
               bool bf16, cudaStream_t stream);
int launch_d64_residue(const Tmap& tq, const Tmap& tk, const Tmap& tv, const FwdParams& P,
                       int grid, int L, bool bf16, cudaStream_t stream);

}  // namespace db
}  // namespace attn
}  // namespace pa
