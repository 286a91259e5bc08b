// Shared pieces of the block-sparse attention forward: constants, the plan
// layout, the kernel parameters and the kernel template itself.  csrc/attn.cu holds
// the plan kernels, argument checks and C entry points; the kernel's instantiations
// are spread over csrc/attn_k*.cu so they compile in parallel.
#pragma once
#include <cuda.h>
#include <math.h>
#include <atomic>
#include "common.cuh"
#include "capi_util.h"

namespace pa {
namespace attn {


constexpr int kThreads = 384;      // three warpgroups; warps 10-11 complete the third
constexpr int kSoftmaxRegs = 200;  // setmaxnreg split of the 384 x 168 launch registers:
constexpr int kOtherRegs = 104;    //   256 x 200 + 128 x 104 = 64512
constexpr int kLoadWarp = 8;
constexpr int kMmaWarp = 9;

// Warp roles of the forward kernel by column groups per row (kCG): with kCG = 1 one
// softmax thread owns a row of S (8 softmax warps, the constants above); with kCG = 2
// two threads share it, 64 columns each (16 softmax warps, 640 threads; setmaxnreg
// split of the 640 x 96 launch registers: 512 x 104 + 128 x 64 = 61440; the split
// with the fewest spills, ptxas -v).
template <int kCG>
struct Roles {
  static constexpr int kSoftmaxWarps = 8 * kCG;
  static constexpr int kThreads = kCG == 1 ? 384 : 640;
  static constexpr int kLoadWarp = kSoftmaxWarps;
  static constexpr int kMmaWarp = kSoftmaxWarps + 1;
  static constexpr int kSoftmaxRegs = kCG == 1 ? 200 : 104;
  static constexpr int kOtherRegs = kCG == 1 ? 104 : 64;
};
constexpr int BM = 128;   // query rows per half
constexpr int BN = 128;   // KV rows per super-tile
constexpr int kTmemCols = 512;
constexpr uint32_t kDrainLimitNs = 200u * 1000u * 1000u;

// ----------------------------------------------------------------- plan layout
struct PlanView {
  int32_t* err;        // status word: (launch epoch << 8) | DEV_* code of a failed launch
  int32_t* sched;      // [2]: next work item, CTAs finished (reset by the last CTA)
  int32_t* done;       // epoch of the last launch whose CTAs all finished
  int32_t* pair_cnt;   // [npairs] union entries of pair p
  int32_t* order;      // [npairs] pairs sorted by decreasing entry count
  int32_t* entries;    // [npairs * cap] ascending A-tile ids
  uint8_t* status;     // [npairs * cap] bits 0-1 half 0, bits 2-3 half 1: 0 dead 1 full 2 partial
  uint2* desc;         // [npairs * cap] per listed tile: see make_desc below
  int cap;
  int npairs;
};

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

struct PlanSizes {
  size_t off_cnt, off_order, off_entries, off_status, off_desc, total;
  int cap, npairs;
};

inline PlanSizes plan_sizes(int N, int A) {
  PlanSizes s;
  s.npairs = (N + 2 * BM - 1) / (2 * BM);
  s.cap = N / A;
  s.off_cnt = 256;
  s.off_order = align_up(s.off_cnt + 4ull * s.npairs, 256);
  s.off_entries = align_up(s.off_order + 4ull * s.npairs, 256);
  s.off_status = align_up(s.off_entries + 4ull * s.npairs * s.cap, 256);
  s.off_desc = align_up(s.off_status + (size_t)s.npairs * s.cap, 256);
  s.total = align_up(s.off_desc + 8ull * s.npairs * s.cap, 256);
  return s;
}

inline PlanView plan_view(void* ws, int N, int A) {
  const PlanSizes s = plan_sizes(N, A);
  char* b = static_cast<char*>(ws);
  PlanView v;
  v.err = reinterpret_cast<int32_t*>(b);
  v.sched = reinterpret_cast<int32_t*>(b + 64);
  v.done = reinterpret_cast<int32_t*>(b + 128);
  v.pair_cnt = reinterpret_cast<int32_t*>(b + s.off_cnt);
  v.order = reinterpret_cast<int32_t*>(b + s.off_order);
  v.entries = reinterpret_cast<int32_t*>(b + s.off_entries);
  v.status = reinterpret_cast<uint8_t*>(b + s.off_status);
  v.desc = reinterpret_cast<uint2*>(b + s.off_desc);
  v.cap = s.cap;
  v.npairs = s.npairs;
  return v;
}

// Status of the last launch on a workspace from its header words: the failure code
// when the error word carries that launch's epoch, else 0 (the word is older).
inline int32_t launch_status(int32_t err_word, int32_t done_epoch) {
  if (err_word == 0) return 0;
  return ((uint32_t)err_word >> 8) == (uint32_t)done_epoch ? (err_word & 0xff) : 0;
}

// ------------------------------------------------------------- plan kernels
// ------------------------------------------------------------- forward kernel
struct FwdParams {
  // O as a tensor map of boxes of 64 columns x 32 rows (one softmax warp's rows), for
  // the epilogue's TMA loads (merge) and stores; unused when o_row_map scatters rows
  CUtensorMap tm_o;
  int BH, N, A;
  int rs, nb;          // residue stride of a virtual permutation (0 = none), N / rs
  const int32_t* perm_q;
  const int32_t* perm_kv;
  const int32_t* o_row_map;
  void* o;
  float* lse;
  long long o_bh_stride, o_row_stride, lse_bh_stride;
  Pred pred;
  float scale_log2;
  PlanView pv;
  uint32_t idesc_qk, idesc_pv;
  int total_items;
  int hg;              // heads per scheduling group (BH: one group)
  // gathered K/V (gather kernel only): rows per head of the 2-D K / V views, whether
  // K/V rows go through perm_kv, the row multiplier of the K reads (1 = none) and
  // whether the extra rows are scattered
  int g_kbh, g_vbh, g_kv, g_mult, g_scatter;
  ErrSink err;         // status word of the workspace, this launch's 24-bit epoch
                       // (nonzero) and the limit of every bounded barrier wait
  ErrSink err_q;       // the same for the MMA issuer's waits on Q tiles; its limit is a
                       // quarter of the others' under the withheld-Q test hook, so that
                       // wait is the one that runs out first, deterministically
  int withhold_q;      // test hook: never load half 0's Q tile of a CTA's first item
};

// One entry of the work-item ring in shared memory, written by the producer before it
// signals item_full: the item, its pair and (batch, head), the pair's list length and
// the plan descriptors of the first super-tile's segments, so that the MMA and softmax
// warps start an item without a chain of dependent global loads.
struct ItemSlot {
  int it, p, bh, cnt;
  uint2 d0[2];   // kept when a super-tile has at most two segments
};

template <int D, int kCG = 1>
struct Smem {
  static constexpr int kTileBytes = BM * D * 2;               // one 128-row tile, 16-bit
  static constexpr int kSlots = D == 128 ? 4 : 8;
  static constexpr int kQOff = 0;
  static constexpr int kKVOff = 2 * kTileBytes;
  static constexpr int kBarOff = kKVOff + kSlots * kTileBytes;
  // barriers: q_full[2] q_empty[2] s_full[2] p_full[2] o_full[2] drain item_full[2]
  //           item_empty[2] kv_full[S] kv_empty[S]
  // kCG = 1: + epi_bar[8] (a softmax warp's TMA load of the O rows in place, merge)
  static constexpr int kNumBars = 15 + 2 * kSlots + 8;
  static constexpr int kMiscOff = kBarOff + 8 * kNumBars;    // tmem base, abort
  static constexpr int kSlotOff = kMiscOff + 16;               // item ring: ItemSlot[2]
  // kCG = 1: epilogue staging [8 warps][32 rows][128 B], 128-byte swizzled boxes for the
  // O tensor map (1024-byte aligned); kCG = 2: none (the two threads of a row share a
  // warp and exchange through shuffles)
  static constexpr int kEpiOff = (kSlotOff + 2 * (int)sizeof(ItemSlot) + 1023) & ~1023;
  static constexpr int kBytes = kEpiOff + (kCG == 1 ? 8 * 32 * 128 : 0);
  static constexpr int kAlloc = kBytes + 1024;                 // room to align to 1024
  // gathered K/V only: the landing place of the extra rows nobody reads (one
  // four-row gather: 4 rows x 128 bytes)
  static constexpr int kDiscardOff = (kBytes + 1023) & ~1023;
  static constexpr int kAllocGather = kDiscardOff + 512 + 1024;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// d = a * b + c on two lanes at once (f32x2), every operand a pair.
__device__ __forceinline__ void fma2v(float& d0, float& d1, float a0, float a1, float b0,
                                      float b1, float c0, float c1) {
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\t"
      "mov.b64 rb, {%4, %5};\n\t"
      "mov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\t"
      "mov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d0), "=f"(d1) : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}

// Pairs (index i = 0..15 of each 32-column chunk of a row) whose exponentials run on
// the FMA pipe (exp2_fma) instead of the XU pipe.  On B200 ex2 is the softmax's only
// XU instruction, at 8 cycles per warp instruction per scheduler: the exponentials of
// a 128 x 128 tile take the XU as long as the tensor core takes for the tile's two
// MMAs.  Measured on the forward kernels (c2, c3, c4, c5; 4, 5 and 8 of 16 pairs):
// no faster with 4, slower with more -- the per-half chain, not the XU, sets the
// kernel's period -- so no pair is moved by default.
#ifndef PA_FMA_EXP_PAIRS
#define PA_FMA_EXP_PAIRS 0u
#endif
constexpr uint32_t kFmaExpPairs = PA_FMA_EXP_PAIRS;

// 2^x for two values on the FMA and integer pipes, no XU instruction: x = j + f with
// j = rint(x), read from the low mantissa bits of t = x + 1.5 * 2^23 (the add rounds
// to the nearest integer; 1.5 * 2^23 keeps t in [2^23, 2^24) for |x| < 2^22);
// 2^f by a cubic on [-1/2, 1/2] fitted for least maximum relative error (7.5e-5, well
// below the bf16 rounding P gets next); 2^j as the float whose exponent field is
// j + 127, made by one integer multiply-add on t's bits ((j mod 2^9) << 23 plus the
// bits of 1.0f, mod 2^32).  x is clamped to >= -127 first, where that field is 0: the
// scale is exactly 0, so a masked score (-inf) gives exactly 0, as ex2.approx.ftz
// does.  Used for x <= 127 (the softmax's x never exceeds the lazy-rescale margin).
__device__ __forceinline__ void exp2_fma(float x0, float x1, float& y0, float& y1) {
  constexpr float kRound = 12582912.0f;   // 1.5 * 2^23
  constexpr float kC0 = 0.99992811f, kC1 = 0.69326097f, kC2 = 0.24261054f, kC3 = 0.055171322f;
  x0 = fmaxf(x0, -127.0f);
  x1 = fmaxf(x1, -127.0f);
  float t0, t1, j0, j1, f0, f1, p0, p1;
  fma2v(t0, t1, x0, x1, 1.0f, 1.0f, kRound, kRound);        // t = x + R
  fma2v(j0, j1, t0, t1, 1.0f, 1.0f, -kRound, -kRound);      // j = t - R (exact)
  fma2v(f0, f1, j0, j1, -1.0f, -1.0f, x0, x1);              // f = x - j
  fma2v(p0, p1, f0, f1, kC3, kC3, kC2, kC2);
  fma2v(p0, p1, p0, p1, f0, f1, kC1, kC1);
  fma2v(p0, p1, p0, p1, f0, f1, kC0, kC0);
  const float s0 = __uint_as_float(__float_as_uint(t0) * 8388608u + 0x3F800000u);
  const float s1 = __uint_as_float(__float_as_uint(t1) * 8388608u + 0x3F800000u);
  fma2v(y0, y1, p0, p1, s0, s1, 0.0f, 0.0f);               // 2^f * 2^j
}

// The exponentials of pair i of a 32-column chunk (i a compile-time constant after
// unrolling): on the FMA pipe for the pairs in kFmaExpPairs, on the XU otherwise.
__device__ __forceinline__ void exp2_pair(int i, float x0, float x1, float& y0, float& y1) {
  if ((kFmaExpPairs >> i) & 1u) {
    exp2_fma(x0, x1, y0, y1);
  } else {
    y0 = ex2(x0);
    y1 = ex2(x1);
  }
}

template <bool kBf16>
__device__ __forceinline__ void unpack2(uint32_t u, float& lo, float& hi) {
  if constexpr (kBf16) {
    lo = __uint_as_float(u << 16);
    hi = __uint_as_float(u & 0xffff0000u);
  } else {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&u));
    lo = f.x;
    hi = f.y;
  }
}

template <bool kBf16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (kBf16) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}

// Number of super-tiles of pair `p` and, for segment `sg` of super-tile `u`, the
// first KV row (N when past the end) and the 4-bit status.
struct SegInfo {
  int row0;
  int st;
};

// Work item `it` -> (pair, head).  Items run in groups of P.hg heads (the last group
// may have fewer; P.hg = BH by default: one group); inside a group they go pair by
// pair in the plan's longest-first order, every head of the group for one pair.
// With small groups the CTAs in flight read the K/V of a few heads only, which stay
// in L2 while the pairs that share them run.
__device__ __forceinline__ void item_coords(const FwdParams& P, int it, int& p, int& bh) {
  const int gsz = P.hg * P.pv.npairs;          // items of a full group
  const int g = it / gsz;
  const int h0 = g * P.hg;
  const int gh = min(P.hg, P.BH - h0);         // heads of this group
  const int li = it - g * gsz;
  const int q = li / gh;
  p = __ldg(P.pv.order + q);
  bh = h0 + (li - q * gh);
}

template <int L>
__device__ __forceinline__ int num_super(const FwdParams& P, int cnt) {
  constexpr int S = BN / L;
  if (P.A <= BN) return (cnt + S - 1) / S;
  return cnt * (P.A / BN);
}

template <int L>
__device__ __forceinline__ SegInfo seg_info(const FwdParams& P, const int32_t* ent,
                                            const uint8_t* sts, int cnt, int u, int sg) {
  constexpr int S = BN / L;
  if (P.A <= BN) {
    const int e = u * S + sg;
    if (e < cnt) return SegInfo{__ldg(ent + e) * P.A, (int)__ldg(sts + e)};
    return SegInfo{P.N, 0};
  }
  const int sub = P.A / BN;
  const int e = u / sub;
  return SegInfo{__ldg(ent + e) * P.A + (u - e * sub) * BN, (int)__ldg(sts + e)};
}

// d = a * b + c on two lanes at once (f32x2).
__device__ __forceinline__ void ffma2(float& d0, float& d1, float a0, float a1, float b, float c) {
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\t"
      "mov.b64 rb, {%4, %4};\n\t"
      "mov.b64 rc, {%5, %5};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\t"
      "mov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d0), "=f"(d1) : "f"(a0), "f"(a1), "f"(b), "f"(c));
}
// a += b on two lanes at once (f32x2).
__device__ __forceinline__ void fadd2(float& a0, float& a1, float b0, float b1) {
  asm("{\n\t.reg .b64 ra, rb;\n\t"
      "mov.b64 ra, {%0, %1};\n\t"
      "mov.b64 rb, {%2, %3};\n\t"
      "add.rn.f32x2 ra, ra, rb;\n\t"
      "mov.b64 {%0, %1}, ra;\n\t}"
      : "+f"(a0), "+f"(a1) : "f"(b0), "f"(b1));
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

template <int D, int L, bool kBf16, bool kRS, bool kMerge, bool kGather = false, int kCG = 1>
__global__ void __launch_bounds__(Roles<kCG>::kThreads, 1)
attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ FwdParams P) {
  using SM = Smem<D, kCG>;
  using R = Roles<kCG>;
  constexpr int kLoadWarp = R::kLoadWarp;
  constexpr int kMmaWarp = R::kMmaWarp;
  constexpr int S = BN / L;              // segments per super-tile
  // the ring entry carries the first super-tile's descriptors for one segment (more
  // would cost the one-thread softmax registers it spills)
  constexpr int kSlotSegs = 1;
  constexpr int NS = SM::kSlots;
  constexpr int kChunks = D / 64;        // 128-byte swizzle chunks along D
  constexpr uint32_t kRegion = BM * 128; // bytes of one 64-column chunk of a 128-row tile

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sQ = smem + SM::kQOff;
  uint8_t* sKV = smem + SM::kKVOff;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM::kBarOff);
  uint64_t* q_full = bars + 0;
  uint64_t* q_empty = bars + 2;
  uint64_t* s_full = bars + 4;
  uint64_t* p_full = bars + 6;
  uint64_t* o_full = bars + 8;
  uint64_t* drain = bars + 10;
  uint64_t* item_full = bars + 11;
  uint64_t* item_empty = bars + 13;
  uint64_t* kv_full = bars + 15;
  uint64_t* kv_empty = bars + 15 + NS;
  uint64_t* epi_bar = bars + 15 + 2 * NS;    // kCG = 1: [softmax warp], TMA loads of old O
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
      mbar_init(&s_full[h], 1);
      mbar_init(&p_full[h], BM * kCG);
      mbar_init(&o_full[h], 1);
    }
    mbar_init(drain, 1);
    for (int r = 0; r < 2; ++r) {
      mbar_init(&item_full[r], 1);
      mbar_init(&item_empty[r], 1 + R::kSoftmaxWarps);   // MMA thread + a lane per softmax warp
    }
    for (int s = 0; s < NS; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    if constexpr (kCG == 1)
      for (int b = 0; b < 8; ++b) mbar_init(&epi_bar[b], 1);
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


  if (warp >= R::kSoftmaxWarps) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(R::kOtherRegs));
  if (warp == kLoadWarp) {
    // ------------------------------------------------------------ producer
    // Teardown: let every copy issued into the ring and the Q tiles land before the
    // CTA can exit.  A phase that completed long ago also satisfies the parity
    // test, so this only ever waits on copies still in flight.
    auto drain_copies = [&](uint32_t kv_g, const int* q_armed) {
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
    };
    // writes the ring entry of item `it` (or of the end marker, it < 0) into `sl`
    auto fill_slot = [&](ItemSlot& sl, int it) {
      sl.it = it;
      if (it < 0) return;
      int p, bh;
      item_coords(P, it, p, bh);
      const int cnt = __ldg(P.pv.pair_cnt + p);
      sl.p = p;
      sl.bh = bh;
      sl.cnt = cnt;
      if constexpr (S <= kSlotSegs) {
        const uint2* desc = P.pv.desc + (size_t)p * P.pv.cap;
#pragma unroll
        for (int sg = 0; sg < S; ++sg) {
          const int e = P.A <= BN ? sg : 0;
          sl.d0[sg] = e < cnt ? __ldg(desc + e) : make_uint2(0u, 0u);
        }
      }
    };
    if constexpr (kGather) {
      // Gathered K/V rows (the reference's GATHER_KV / GATHER_MULT knobs,
      // gpu/triton_attn.py:99-128): row j of the kernel order is read from row
      // perm_kv[j] of K and V left in original order (row j itself without
      // gather_kv), four rows per tile::gather4 copy.  Every lane issues the copies
      // of its own 4-row group of each super-tile; lane 0 owns the schedule and the
      // barriers and broadcasts its decisions, so the warp stays converged.  With
      // g_mult = R > 1 each K tile also reads (R - 1) more row sets -- rows
      // row(j) + r A (contiguous) or perm_kv[j + r A] (scattered), mod N -- into a
      // discard buffer: the reference weights them by zero, so the result is the
      // same and only their traffic is paid.
      int qi = 0;
      int q_armed[2] = {0, 0};
      uint32_t kv_g = 0;
      uint32_t ring = 0;
      const int grp = lane * 4;                    // this lane's rows of a super-tile
      const int sg_l = grp / L, t_l = grp - (grp / L) * L;
      const uint32_t k_bytes = (uint32_t)P.g_mult * SM::kTileBytes;
      const int32_t* perm = P.perm_kv;
      uint8_t* sDiscard = smem + SM::kDiscardOff;
      auto rows4 = [&](const int32_t* pm, int j) -> int4 {   // pm[j..j+3], identity if null
        if (pm) return __ldg(reinterpret_cast<const int4*>(pm + j));
        return make_int4(j, j + 1, j + 2, j + 3);
      };
      while (true) {
        int it = -1, ok = 1;
        if (lane == 0) {
          it = atomicAdd(P.pv.sched, 1);
          if (it >= P.total_items || *s_abort) it = -1;
          const uint32_t rs = ring & 1;
          if (ring >= 2 &&
              !mbar_wait(&item_empty[rs], ((ring >> 1) - 1) & 1, s_abort, err, DEV_TIMEOUT_ITEM)) {
            ok = 0;
          } else {
            fill_slot(s_slot[rs], it);
            mbar_arrive(&item_full[rs]);
          }
        }
        ++ring;
        ok = __shfl_sync(0xffffffffu, ok, 0);
        it = __shfl_sync(0xffffffffu, it, 0);
        if (!ok || it < 0) break;
        int p, bh;
        item_coords(P, it, p, bh);
        const int cnt = __ldg(P.pv.pair_cnt + p);
        const int nsup = num_super<L>(P, cnt);
        if (nsup == 0) continue;
        const int32_t* ent = P.pv.entries + (size_t)p * P.pv.cap;
        const uint8_t* sts = P.pv.status + (size_t)p * P.pv.cap;
        if (lane == 0) {
          for (int h = 0; h < 2; ++h) {
            if (qi > 0 && !mbar_wait(&q_empty[h], (qi - 1) & 1, s_abort, err, DEV_TIMEOUT_Q)) {
              ok = 0;
              break;
            }
            mbar_arrive_expect_tx(&q_full[h], SM::kTileBytes);
            ++q_armed[h];
            const int qr = p * 2 * BM + h * BM;
            for (int c = 0; c < kChunks; ++c)
              tma_load_3d(sQ + h * SM::kTileBytes + c * kRegion, &tm_q, &q_full[h], c * 64, qr,
                          bh);
          }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        const int kb = bh * P.g_kbh, vb = bh * P.g_vbh;   // row 0 of this head in the 2-D views
        for (int u = 0; u < nsup && ok; ++u) {
          const SegInfo si = seg_info<L>(P, ent, sts, cnt, u, sg_l);
          // a padding segment (past the listed tiles, masked as dead) reads any valid rows
          const int j = si.row0 < P.N ? si.row0 + t_l : t_l % P.N;
          const int4 b = rows4(P.g_kv ? perm : nullptr, j);
          for (int kv = 0; kv < 2; ++kv) {
            const uint32_t slot = kv_g % NS;
            if (lane == 0) {
              if (kv_g >= (uint32_t)NS &&
                  !mbar_wait(&kv_empty[slot], ((kv_g / NS) - 1) & 1, s_abort, err,
                             DEV_TIMEOUT_KV))
                ok = 0;
              else
                mbar_arrive_expect_tx(&kv_full[slot], kv == 0 ? k_bytes : SM::kTileBytes);
            }
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            ++kv_g;
            uint8_t* dst = sKV + slot * SM::kTileBytes + grp * 128;
            const void* tm = kv == 0 ? (const void*)&tm_k : (const void*)&tm_v;
            const int base = kv == 0 ? kb : vb;
            for (int c = 0; c < kChunks; ++c)
              tma_gather4(dst + c * kRegion, tm, &kv_full[slot], c * 64, base + b.x, base + b.y,
                          base + b.z, base + b.w);
            if (kv == 0) {
              for (int r = 1; r < P.g_mult; ++r) {
                int4 e;
                if (P.g_scatter) {
                  e = rows4(perm, (j + r * P.A) % P.N);
                } else {
                  const int sh = r * P.A;
                  e = make_int4((b.x + sh) % P.N, (b.y + sh) % P.N, (b.z + sh) % P.N,
                                (b.w + sh) % P.N);
                }
                for (int c = 0; c < kChunks; ++c)
                  tma_gather4(sDiscard, &tm_k, &kv_full[slot], c * 64, kb + e.x, kb + e.y,
                              kb + e.z, kb + e.w);
              }
            }
          }
        }
        if (!ok) break;
        ++qi;
      }
      if (lane == 0) drain_copies(kv_g, q_armed);
    } else if (lane == 0) {
      int qi = 0;
      int q_armed[2] = {0, 0};
      uint32_t kv_g = 0;
      uint32_t ring = 0;
      while (true) {
        // fetch the next work item and hand it to the MMA and softmax warps
        int it = atomicAdd(P.pv.sched, 1);
        if (it >= P.total_items || *s_abort) it = -1;
        const uint32_t rs = ring & 1;
        if (ring >= 2 &&
            !mbar_wait(&item_empty[rs], ((ring >> 1) - 1) & 1, s_abort, err, DEV_TIMEOUT_ITEM))
          break;
        fill_slot(s_slot[rs], it);
        mbar_arrive(&item_full[rs]);
        ++ring;
        if (it < 0) break;
        const int p = s_slot[rs].p, bh = s_slot[rs].bh, cnt = s_slot[rs].cnt;
        const int nsup = num_super<L>(P, cnt);
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
          mbar_arrive_expect_tx(&q_full[h], SM::kTileBytes);
          ++q_armed[h];
          const int qr = p * 2 * BM + h * BM;
          for (int c = 0; c < kChunks; ++c) {
            if constexpr (kRS)
              tma_load_4d(sQ + h * SM::kTileBytes + c * kRegion, &tm_q, &q_full[h], c * 64,
                          qr / P.nb, qr % P.nb, bh);
            else
              tma_load_3d(sQ + h * SM::kTileBytes + c * kRegion, &tm_q, &q_full[h], c * 64, qr,
                          bh);
          }
        }
        if (!ok) break;
        for (int u = 0; u < nsup && ok; ++u) {
          SegInfo si[S];
#pragma unroll
          for (int sg = 0; sg < S; ++sg) si[sg] = seg_info<L>(P, ent, sts, cnt, u, sg);
          for (int kv = 0; kv < 2; ++kv) {
            const uint32_t slot = kv_g % NS;
            if (kv_g >= (uint32_t)NS) {
              ok = mbar_wait(&kv_empty[slot], ((kv_g / NS) - 1) & 1, s_abort, err,
                             DEV_TIMEOUT_KV);
              if (!ok) break;
            }
            ++kv_g;
            uint8_t* dst = sKV + slot * SM::kTileBytes;
            mbar_arrive_expect_tx(&kv_full[slot], SM::kTileBytes);
            const void* tm = kv == 0 ? (const void*)&tm_k : (const void*)&tm_v;
#pragma unroll
            for (int sg = 0; sg < S; ++sg) {
              const int r0 = si[sg].row0;
              for (int c = 0; c < kChunks; ++c) {
                if constexpr (kRS)
                  tma_load_4d(dst + c * kRegion + sg * L * 128, tm, &kv_full[slot], c * 64,
                              r0 / P.nb, r0 % P.nb, bh);
                else
                  tma_load_3d(dst + c * kRegion + sg * L * 128, tm, &kv_full[slot], c * 64, r0,
                              bh);
              }
            }
          }
        }
        ++qi;
      }
      drain_copies(kv_g, q_armed);
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int qi = 0;
      uint32_t kv_c = 0;
      uint32_t tp[2] = {0, 0};
      bool ok = true;
      const uint32_t sQa = smem_u32(sQ), sKVa = smem_u32(sKV);
      auto wait_kv = [&](uint32_t& slot) -> bool {
        slot = kv_c % NS;
        const bool r = mbar_wait(&kv_full[slot], (kv_c / NS) & 1, s_abort, err, DEV_TIMEOUT_KV);
        ++kv_c;
        tc_fence_after();
        return r;
      };
      // Descriptors are built once per operand tile; stepping K only moves the
      // start-address field (bits 0-13, in 16-byte units), a compile-time offset.
      const uint64_t q_desc[2] = {smem_desc_sw128(sQa, 16),
                                  smem_desc_sw128(sQa + SM::kTileBytes, 16)};
      auto issue_s = [&](int h, uint32_t kslot) {
        const uint32_t d = tmem + h * 128;
        const uint64_t qd = q_desc[h];
        const uint64_t kd = smem_desc_sw128(sKVa + kslot * SM::kTileBytes, 16);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t off = ((kk >> 2) * kRegion + (kk & 3) * 32) >> 4;
          mma_ss(d, qd + off, kd + off, P.idesc_qk, kk > 0);
        }
      };
      auto issue_pv = [&](int h, uint32_t vslot, bool acc) {
        const uint32_t d = tmem + 256 + h * D;
        const uint32_t pa_ = tmem + h * 128 + 64;
        const uint64_t vd = smem_desc_sw128(sKVa + vslot * SM::kTileBytes, kRegion);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk)
          mma_ts(d, pa_ + kk * 8, vd + (uint64_t)((kk * 16 * 128) >> 4), P.idesc_pv,
                 (acc || kk > 0) ? 1u : 0u);
      };
      auto wait_p = [&](int h) -> bool {
        const bool r = mbar_wait(&p_full[h], tp[h] & 1, s_abort, err, DEV_TIMEOUT_P);
        ++tp[h];
        tc_fence_after();
        return r;
      };
      uint32_t ring = 0;
      while (ok) {
        const uint32_t rs = ring & 1;
        if (!(ok = mbar_wait(&item_full[rs], (ring >> 1) & 1, s_abort, err, DEV_TIMEOUT_ITEM)))
          break;
        const int it = s_slot[rs].it, cnt = s_slot[rs].cnt;
        mbar_arrive(&item_empty[rs]);
        ++ring;
        if (it < 0) break;
        const int nsup = num_super<L>(P, cnt);
        if (nsup == 0) continue;
        ok = mbar_wait(&q_full[0], qi & 1, s_abort, P.err_q, DEV_TIMEOUT_Q) &&
             mbar_wait(&q_full[1], qi & 1, s_abort, P.err_q, DEV_TIMEOUT_Q);
        tc_fence_after();
        if (!ok) break;
        uint32_t ks, vs;
        if (!(ok = wait_kv(ks))) break;
        issue_s(0, ks);
        tc_commit(&s_full[0]);
        issue_s(1, ks);
        tc_commit(&s_full[1]);
        tc_commit(&kv_empty[ks]);
        for (int u = 1; u < nsup && ok; ++u) {
          if (!(ok = wait_kv(vs))) break;
          if (!(ok = wait_kv(ks))) break;
          for (int h = 0; h < 2 && ok; ++h) {
            if (!(ok = wait_p(h))) break;
            issue_pv(h, vs, u > 1);
            issue_s(h, ks);
            tc_commit(&s_full[h]);
          }
          tc_commit(&kv_empty[vs]);
          tc_commit(&kv_empty[ks]);
        }
        if (!ok) break;
        tc_commit(&q_empty[0]);
        tc_commit(&q_empty[1]);
        if (!(ok = wait_kv(vs))) break;
        for (int h = 0; h < 2 && ok; ++h) {
          if (!(ok = wait_p(h))) break;
          issue_pv(h, vs, nsup > 1);
          tc_commit(&o_full[h]);
        }
        tc_commit(&kv_empty[vs]);
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
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(R::kSoftmaxRegs));
    if constexpr (kCG == 2) {
      // ------------------------------------------------------------ softmax + epilogue,
      // two threads per row, in one warp: warp w of the 16 handles half h = w / 8 and the
      // 16 TMEM lanes (query rows) 32 (w % 4) + 16 ((w / 4) % 2) + [0, 16); lane t takes
      // row t % 16 of them and its S columns [64 cg, 64 cg + 64), cg = t / 16 (the
      // .16x32bx2 TMEM shape).  The two threads of a row combine their partial row maxima
      // by a shuffle once per super-tile (so both make the same rescaling decisions) and
      // their partial row sums in the epilogue, and each writes its half of the O row.
      // Columns [32 cg, 32 cg + 32) of the packed P overwrite S columns 64-127, which the
      // partner lane loaded in the same warp-wide TMEM load.
      const int h = warp >> 3;
      const int hs = (warp >> 2) & 1;
      const int wq = warp & 3;
      const int cg = lane >> 4;
      const int r_in = wq * 32 + hs * 16 + (lane & 15);
      const uint32_t lane_off = (uint32_t)(wq * 32 + hs * 16) << 16;
      const uint32_t tS = tmem + lane_off + h * 128;
      const uint32_t tO = tmem + lane_off + 256 + h * D;
      uint32_t ts = 0, to = 0;
      const float c2 = P.scale_log2;
      uint32_t ring = 0;
      while (true) {
        const uint32_t rs = ring & 1;
        bool got = mbar_wait(&item_full[rs], (ring >> 1) & 1, s_abort, err, DEV_TIMEOUT_ITEM);
        if (!__all_sync(0xffffffffu, got)) break;
        const int it = s_slot[rs].it, p = s_slot[rs].p, bh = s_slot[rs].bh, cnt = s_slot[rs].cnt;
        __syncwarp();
        if (lane == 0) mbar_arrive(&item_empty[rs]);
        ++ring;
        if (it < 0) break;
        const int nsup = num_super<L>(P, cnt);
        const int32_t* ent = P.pv.entries + (size_t)p * P.pv.cap;
        const uint2* desc = P.pv.desc + (size_t)p * P.pv.cap;
        const int row = p * 2 * BM + h * BM + r_in;
        const bool valid = row < P.N;
        const int irow = !valid        ? -(1 << 30)
                         : kRS          ? (row % P.nb) * P.rs + row / P.nb
                         : P.perm_q    ? __ldg(P.perm_q + row)
                                       : row;
        float lse_prev = -INFINITY;
        if constexpr (kMerge) {
          if (valid) {
            const int orw0 = kRS          ? (row % P.nb) * P.rs + row / P.nb
                             : P.o_row_map ? __ldg(P.o_row_map + row)
                                           : row;
            if ((unsigned)orw0 < (unsigned)P.N) {
              const char* op = static_cast<const char*>(P.o) +
                               ((long long)bh * P.o_bh_stride + (long long)orw0 * P.o_row_stride) * 2 +
                               cg * D;
              asm volatile("prefetch.global.L2 [%0];" ::"l"(op));
              asm volatile("ld.global.f32 %0, [%1];"
                           : "=f"(lse_prev)
                           : "l"(P.lse + (long long)bh * P.lse_bh_stride + orw0));
            }
          }
        }
        float m_used = -INFINITY, l = 0.f;
        bool ok = true;
        for (int u = 0; u < nsup; ++u) {
          // live bits of this row for this thread's 64 columns, while S is in flight
          auto word_bits = [&](int sg, int base, int width) -> uint32_t {
            int e, sub = 0;
            if (P.A <= BN) {
              e = u * S + sg;
            } else {
              const int spt = P.A / BN;
              e = u / spt;
              sub = u - e * spt;
            }
            uint2 d = make_uint2(0u, 0u);
            if (e < cnt) d = __ldg(desc + e);
            const int st = (d.y >> (24 + 2 * h)) & 3;
            uint32_t w = st == 1 ? (width == 32 ? 0xffffffffu : 0xffffu) : 0u;
            if (st == 2) {
              const int dj = (int)(d.y & 0xffffu);
              const int sh = (d.y & (1u << 20)) ? (int)((d.y >> 16) & 15u) : -1;
              const bool ap = (d.y >> 21) & 1u;
              const int j0 = (int)d.x + sub * BN * dj;
              if (!(ap && progression_bits(P.pred, irow - j0, j0, dj, sh, base, L, w))) {
                const int32_t* cols = P.perm_kv ? P.perm_kv + __ldg(ent + e) * P.A + sub * BN + base
                                                : nullptr;
                w = element_bits(P.pred, irow, cols, j0, dj, base, width);
              }
              if (width == 16) w &= 0xffffu;
            }
            return w;
          };
          uint32_t mk[2];
#pragma unroll
          for (int kk = 0; kk < 2; ++kk) {
            const int kw = 2 * cg + kk;          // 32-column word of the super-tile
            if constexpr (L >= 32)
              mk[kk] = word_bits((kw * 32) / L, (kw * 32) % L, 32);
            else
              mk[kk] = word_bits(2 * kw, 0, 16) | (word_bits(2 * kw + 1, 0, 16) << 16);
          }
          ok = mbar_wait(&s_full[h], ts & 1, s_abort, err, DEV_TIMEOUT_S);
          ++ts;
          if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
          tc_fence_after();
          float s[64];
          {
            uint32_t r0[32], r1[32];
            tmem_ld32_pair<64>(tS, r0);
            tmem_ld32_pair<64>(tS + 32, r1);
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
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
          const float m_tile = mx * c2;
          const float m_new = fmaxf(m_used, m_tile);
          const float m_prev = m_used;
          bool bump = false;
          float factor = 1.f;
          if (u == 0) {
            m_used = m_new;
          } else if (m_new > m_used + 8.0f) {
            bump = true;
            factor = ex2(m_used - m_new);
            m_used = m_new;
          }
          // O holds something once any earlier key was live for the row, whichever
          // thread's columns it was in: decided on the shared maximum, not on this
          // thread's partial sum, so both threads of the row rescale together
          const bool need_o = bump && m_prev != -INFINITY;
          if (bump) l *= factor;
          const float msub = m_used == -INFINITY ? 0.f : m_used;
          float r8[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) r8[j] = 0.f;
#pragma unroll
          for (int q4 = 0; q4 < 2; ++q4) {
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int c = q4 * 32 + 2 * i;
              float x0, x1;
              ffma2(x0, x1, s[c], s[c + 1], c2, -msub);
              float a, b;
              exp2_pair(i, x0, x1, a, b);
              const int j = (2 * i) & 7;
              fadd2(r8[j], r8[j + 1], a, b);
              pk[i] = pack2<kBf16>(a, b);
            }
            tmem_st16_pair<32>(tS + 64 + q4 * 16, pk);
          }
          l += ((r8[0] + r8[1]) + (r8[2] + r8[3])) + ((r8[4] + r8[5]) + (r8[6] + r8[7]));
          // O rescale (rare), this thread's half of the row
          if (__any_sync(0xffffffffu, need_o)) {
            const float f = need_o ? factor : 1.f;
#pragma unroll 1
            for (int k = 0; k < D / 64; ++k) {
              uint32_t r[32];
              tmem_ld32_pair<D / 2>(tO + k * 32, r);
              tmem_wait_ld();
              tmem_regs_ready(r);
#pragma unroll
              for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * f);
              tmem_st32_pair<D / 2>(tO + k * 32, r);
            }
          }
          tmem_wait_st();
          tc_fence_before();
          mbar_arrive(&p_full[h]);
        }
        if (!ok) break;
        // epilogue: the row's sum from both threads, O / l, LSE (written by cg 0)
        l += __shfl_xor_sync(0xffffffffu, l, 16);
        float inv_l = l > 0.f ? 1.f / l : 0.f;
        const float lse_v = l > 0.f ? (m_used + __log2f(l)) * 0.69314718055994530942f : -INFINITY;
        float w_old = 0.f;
        char* orow = nullptr;
        if (valid) {
          const int orw = kRS          ? (row % P.nb) * P.rs + row / P.nb
                          : P.o_row_map ? __ldg(P.o_row_map + row)
                                        : row;
          if ((unsigned)orw < (unsigned)P.N) {
            orow = static_cast<char*>(P.o) +
                   ((long long)bh * P.o_bh_stride + (long long)orw * P.o_row_stride) * 2 + cg * D;
            if (P.lse) {
              float* lp = P.lse + (long long)bh * P.lse_bh_stride + orw;
              float lse_out = lse_v;
              if constexpr (kMerge) {
                const float lo = lse_prev;
                const float mm = fmaxf(lo, lse_v);
                float wa = 0.f, wb = 0.f;
                if (mm != -INFINITY) {
                  wa = expf(lo - mm);
                  wb = expf(lse_v - mm);
                }
                const float den = wa + wb;
                const float inv = den > 0.f ? 1.f / den : 0.f;
                w_old = wa * inv;
                inv_l *= wb * inv;
                lse_out = den > 0.f ? mm + logf(den) : -INFINITY;
              }
              if (cg == 0) *lp = lse_out;
            }
          }
        }
        const bool have_o = nsup > 0;
        if (have_o) {
          ok = mbar_wait(&o_full[h], to & 1, s_abort, err, DEV_TIMEOUT_O);
          ++to;
          if (!__all_sync(0xffffffffu, ok)) break;
          tc_fence_after();
        }
        // this thread's D/2 columns of the row, 32 at a time, straight to global memory
#pragma unroll 1
        for (int k = 0; k < D / 64; ++k) {
          uint32_t r[32];
          if (have_o) {
            tmem_ld32_pair<D / 2>(tO + k * 32, r);
            tmem_wait_ld();
            tmem_regs_ready(r);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = 0u;
          }
          if (orow) {
            char* dst = orow + k * 64;
            uint4 ov[4];
            if constexpr (kMerge) {
#pragma unroll
              for (int c = 0; c < 4; ++c)
                asm volatile("ld.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                             : "=r"(ov[c].x), "=r"(ov[c].y), "=r"(ov[c].z), "=r"(ov[c].w)
                             : "l"(dst + c * 16));
            }
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              uint32_t w[4];
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                float a = __uint_as_float(r[8 * c + 2 * j]) * inv_l;
                float b = __uint_as_float(r[8 * c + 2 * j + 1]) * inv_l;
                if constexpr (kMerge) {
                  const uint32_t old = j == 0 ? ov[c].x : j == 1 ? ov[c].y : j == 2 ? ov[c].z : ov[c].w;
                  float oa, ob;
                  unpack2<kBf16>(old, oa, ob);
                  a = fmaf(w_old, oa, a);
                  b = fmaf(w_old, ob, b);
                }
                w[j] = pack2<kBf16>(a, b);
              }
              *reinterpret_cast<uint4*>(dst + c * 16) = make_uint4(w[0], w[1], w[2], w[3]);
            }
          }
        }
        if (have_o) tc_fence_before();
      }
    } else {
    // ------------------------------------------------------------ softmax + epilogue
    const int h = warp >> 2;              // which half
    const int wq = warp & 3;              // TMEM lane quarter
    const int r_in = wq * 32 + lane;      // row within the half
    const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
    const uint32_t tS = tmem + lane_off + h * 128;
    const uint32_t tO = tmem + lane_off + 256 + h * D;
    uint32_t ts = 0, to = 0;
    uint32_t epi_issued = 0, epi_done = 0;   // TMA loads of the staging (merge): issued, awaited
    const float c2 = P.scale_log2;
    uint32_t ring = 0;
    while (true) {
      const uint32_t rs = ring & 1;
      bool got = mbar_wait(&item_full[rs], (ring >> 1) & 1, s_abort, err, DEV_TIMEOUT_ITEM);
      if (!__all_sync(0xffffffffu, got)) break;
      const int it = s_slot[rs].it, p = s_slot[rs].p, bh = s_slot[rs].bh, cnt = s_slot[rs].cnt;
      uint2 d0[S];   // the first super-tile's descriptors, from the ring entry
#pragma unroll
      for (int sg = 0; sg < S; ++sg)
        d0[sg] = S <= kSlotSegs ? s_slot[rs].d0[sg] : make_uint2(0u, 0u);
      __syncwarp();
      if (lane == 0) mbar_arrive(&item_empty[rs]);
      ++ring;
      if (it < 0) break;
      const int nsup = num_super<L>(P, cnt);
      const int32_t* ent = P.pv.entries + (size_t)p * P.pv.cap;
      const uint2* desc = P.pv.desc + (size_t)p * P.pv.cap;
      const int row = p * 2 * BM + h * BM + r_in;
      const bool valid = row < P.N;
      const int irow = !valid        ? -(1 << 30)
                       : kRS          ? (row % P.nb) * P.rs + row / P.nb
                       : P.perm_q    ? __ldg(P.perm_q + row)
                                     : row;
      // merge: the LSE in place is read now (the O row in place is pulled into L2
      // during the last super-tile), so the epilogue does not wait on memory for them
      float lse_prev = -INFINITY;
      if constexpr (kMerge) {
        if (valid) {
          const int orw0 = kRS          ? (row % P.nb) * P.rs + row / P.nb
                           : P.o_row_map ? __ldg(P.o_row_map + row)
                                         : row;
          if ((unsigned)orw0 < (unsigned)P.N) {
            asm volatile("ld.global.f32 %0, [%1];"
                         : "=f"(lse_prev)
                         : "l"(P.lse + (long long)bh * P.lse_bh_stride + orw0));
          }
        }
      }
      float m_used = -INFINITY, l = 0.f;
      bool ok = true;
      // the previous item's box stores have read the staging: waited for here, while
      // the item's first S is still in flight, rather than in the epilogue
      if (lane == 0) bulk_wait_read();
      for (int u = 0; u < nsup; ++u) {
        if constexpr (kMerge) {
          // the O row in place is pulled into L2 during the item's last super-tile,
          // close enough to the epilogue to be still there (an item's K/V stream
          // would have evicted it if fetched at the item's start)
          if (u == nsup - 1 && valid) {
            const int orw0 = kRS          ? (row % P.nb) * P.rs + row / P.nb
                             : P.o_row_map ? __ldg(P.o_row_map + row)
                                           : row;
            if ((unsigned)orw0 < (unsigned)P.N) {
              const char* op = static_cast<const char*>(P.o) +
                               ((long long)bh * P.o_bh_stride + (long long)orw0 * P.o_row_stride) * 2;
              asm volatile("prefetch.global.L2 [%0];" ::"l"(op));
              if constexpr (D == 128) asm volatile("prefetch.global.L2 [%0];" ::"l"(op + 128));
            }
          }
        }
        // this half's view of the super-tile's segments, from the plan descriptors
        int sts_[S], j0s[S], djs[S], shs[S], es[S], subs[S];
        bool aps[S];
#pragma unroll
        for (int sg = 0; sg < S; ++sg) {
          int e, sub = 0;
          if (P.A <= BN) {
            e = u * S + sg;
          } else {
            const int spt = P.A / BN;
            e = u / spt;
            sub = u - e * spt;
          }
          uint2 d = make_uint2(0u, 0u);
          if (S <= kSlotSegs && u == 0) d = d0[sg];
          else if (e < cnt) d = __ldg(desc + e);
          sts_[sg] = (d.y >> (24 + 2 * h)) & 3;
          djs[sg] = (int)(d.y & 0xffffu);
          shs[sg] = (d.y & (1u << 20)) ? (int)((d.y >> 16) & 15u) : -1;
          aps[sg] = (d.y >> 21) & 1u;
          j0s[sg] = (int)d.x + sub * BN * djs[sg];
          es[sg] = e;
          subs[sg] = sub;
        }
        // live bits of this row for the 128 columns, computed while S is in flight
        uint32_t mk[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if constexpr (L >= 32) {
            constexpr int per = L / 32;
            const int sg = k / per, base = (k % per) * 32;
            const int st = sts_[sg];
            uint32_t w = st == 1 ? 0xffffffffu : 0u;
            if (st == 2) {
              if (!(aps[sg] && progression_bits(P.pred, irow - j0s[sg], j0s[sg], djs[sg], shs[sg],
                                                base, L, w))) {
                const int32_t* cols = P.perm_kv ? P.perm_kv + __ldg(ent + es[sg]) * P.A +
                                                      subs[sg] * BN + base
                                                : nullptr;
                w = element_bits(P.pred, irow, cols, j0s[sg], djs[sg], base, 32);
              }
            }
            mk[k] = w;
          } else {
            uint32_t w = 0;
#pragma unroll
            for (int hw = 0; hw < 2; ++hw) {
              const int sg = 2 * k + hw;
              const int st = sts_[sg];
              uint32_t b = st == 1 ? 0xffffu : 0u;
              if (st == 2) {
                if (!(aps[sg] && progression_bits(P.pred, irow - j0s[sg], j0s[sg], djs[sg],
                                                  shs[sg], 0, L, b))) {
                  const int32_t* cols =
                      P.perm_kv ? P.perm_kv + __ldg(ent + es[sg]) * P.A : nullptr;
                  b = element_bits(P.pred, irow, cols, j0s[sg], djs[sg], 0, 16);
                }
                b &= 0xffffu;
              }
              w |= b << (16 * hw);
            }
            mk[k] = w;
          }
        }
        ok = mbar_wait(&s_full[h], ts & 1, s_abort, err, DEV_TIMEOUT_S);
        ++ts;
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        tc_fence_after();
        float s[128];
        {
          uint32_t r0[32], r1[32], r2[32], r3[32];
          tmem_ld32(tS + 0, r0);
          tmem_ld32(tS + 32, r1);
          tmem_ld32(tS + 64, r2);
          tmem_ld32(tS + 96, r3);
          tmem_wait_ld();
          tmem_regs_ready(r0);
          tmem_regs_ready(r1);
          tmem_regs_ready(r2);
          tmem_regs_ready(r3);
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            s[i] = __uint_as_float(r0[i]);
            s[32 + i] = __uint_as_float(r1[i]);
            s[64 + i] = __uint_as_float(r2[i]);
            s[96 + i] = __uint_as_float(r3[i]);
          }
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
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
          for (int c = 16; c < 128; c += 16) {
#pragma unroll
            for (int j = 0; j < 8; ++j) m8[j] = fmax3(m8[j], s[c + 2 * j], s[c + 2 * j + 1]);
          }
          mx = fmax3(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]));
        }
        const float m_tile = mx * c2;
        const float m_new = fmaxf(m_used, m_tile);
        bool bump = false;
        float factor = 1.f;
        if (u == 0) {
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
        for (int q4 = 0; q4 < 4; ++q4) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int c = q4 * 32 + 2 * i;
            float x0, x1;
            ffma2(x0, x1, s[c], s[c + 1], c2, -msub);
            float a, b;
            exp2_pair(i, x0, x1, a, b);
            const int j = (2 * i) & 7;
            fadd2(r8[j], r8[j + 1], a, b);
            pk[i] = pack2<kBf16>(a, b);
          }
          tmem_st16(tS + 64 + q4 * 16, pk);
        }
        l += ((r8[0] + r8[1]) + (r8[2] + r8[3])) + ((r8[4] + r8[5]) + (r8[6] + r8[7]));
        // O rescale (rare: only when the running max grew by more than 2^8)
        if (__any_sync(0xffffffffu, need_o)) {
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
        mbar_arrive(&p_full[h]);
      }
      if (!ok) break;
      // epilogue: O / l, LSE
      float inv_l = l > 0.f ? 1.f / l : 0.f;
      const float lse_v = l > 0.f ? (m_used + __log2f(l)) * 0.69314718055994530942f : -INFINITY;
      float w_old = 0.f;   // weight of the O row already in place (merge)
      char* orow = nullptr;
      if (valid) {
        const int orw = kRS          ? (row % P.nb) * P.rs + row / P.nb
                        : P.o_row_map ? __ldg(P.o_row_map + row)
                                      : row;
        if ((unsigned)orw < (unsigned)P.N) {
          orow = static_cast<char*>(P.o) +
                 ((long long)bh * P.o_bh_stride + (long long)orw * P.o_row_stride) * 2;
          if (P.lse) {
            float* lp = P.lse + (long long)bh * P.lse_bh_stride + orw;
            if constexpr (kMerge) {
              // The row already holds the result (O1, l1) of a disjoint part:
              // O = (e^(l1-m) O1 + e^(l2-m) O2) / (e^(l1-m) + e^(l2-m)), m = max(l1, l2),
              // LSE = m + log(e^(l1-m) + e^(l2-m)); this part's weight folds into 1/l.
              // (exponent and logarithm on the special-function unit: den is in [1, 2],
              // so the approximations' error stays below 1e-6 of the LSE)
              const float lo = lse_prev;
              const float mm = fmaxf(lo, lse_v);
              float wa = 0.f, wb = 0.f;
              if (mm != -INFINITY) {
                wa = ex2((lo - mm) * 1.44269504088896340736f);
                wb = ex2((lse_v - mm) * 1.44269504088896340736f);
              }
              const float den = wa + wb;
              const float inv = den > 0.f ? __fdividef(1.f, den) : 0.f;
              w_old = wa * inv;
              inv_l *= wb * inv;
              *lp = den > 0.f ? mm + __log2f(den) * 0.69314718055994530942f : -INFINITY;
            } else {
              *lp = lse_v;
            }
          }
        }
      }
      // O leaves through the warp's staging buffer, 32 rows x 64 columns at a time.  Rows
      // in the kernel's order (or, with the residue permutation, its original order) make
      // one box of the O tensor map: the warp writes its rows into the 128-byte-swizzled
      // staging and one lane stores the box with a TMA instruction (a merge first has the
      // rows in place loaded into the same staging by TMA, and adds to them there).  Rows
      // scattered by o_row_map are written lane by lane, whole 128-byte row segments at
      // a time.
      uint8_t* stage = sEpi + warp * (32 * 128);
      const bool have_o = nsup > 0;
      if (P.o_row_map == nullptr) {
        const int wrow0 = p * 2 * BM + h * BM + wq * 32;   // the warp's first row
        auto box_load = [&](int dh) {                       // lane 0, merge
          mbar_arrive_expect_tx(&epi_bar[warp], 32 * 128);
          if constexpr (kRS)
            tma_load_4d(stage, &P.tm_o, &epi_bar[warp], dh * 64, wrow0 / P.nb, wrow0 % P.nb, bh);
          else
            tma_load_3d(stage, &P.tm_o, &epi_bar[warp], dh * 64, wrow0, bh);
          ++epi_issued;
        };
        auto box_store = [&](int dh) {                      // lane 0
          if constexpr (kRS)
            tma_store_4d(&P.tm_o, stage, dh * 64, wrow0 / P.nb, wrow0 % P.nb, bh);
          else
            tma_store_3d(&P.tm_o, stage, dh * 64, wrow0, bh);
          bulk_commit();
        };
        if constexpr (kMerge) {
          if (lane == 0) box_load(0);
        }
        if (have_o) {
          ok = mbar_wait(&o_full[h], to & 1, s_abort, err, DEV_TIMEOUT_O);
          ++to;
          if (!__all_sync(0xffffffffu, ok)) break;
          tc_fence_after();
        }
#pragma unroll 1
        for (int dh = 0; dh < D / 64; ++dh) {
          uint32_t r0[32], r1[32];
          if (have_o) {
            tmem_ld32(tO + dh * 64, r0);
            tmem_ld32(tO + dh * 64 + 32, r1);
            tmem_wait_ld();
            tmem_regs_ready(r0);
            tmem_regs_ready(r1);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) r0[i] = r1[i] = 0u;
          }
          if constexpr (kMerge) {
            ok = mbar_wait(&epi_bar[warp], epi_done & 1, s_abort, err, DEV_TIMEOUT_O);
            ++epi_done;
            if (!__all_sync(0xffffffffu, ok)) break;
            // this lane's row of the box: the row in place in, the merged row out
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              uint4* slot = reinterpret_cast<uint4*>(stage + lane * 128 + ((c ^ (lane & 7)) << 4));
              const uint4 v = *slot;
              const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
              uint32_t w4[4];
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const int col = 8 * (c & 3) + 2 * j;
                const float n0 = __uint_as_float(c < 4 ? r0[col] : r1[col]) * inv_l;
                const float n1 = __uint_as_float(c < 4 ? r0[col + 1] : r1[col + 1]) * inv_l;
                float a, b2;
                unpack2<kBf16>(vv[j], a, b2);
                w4[j] = pack2<kBf16>(fmaf(w_old, a, n0), fmaf(w_old, b2, n1));
              }
              *slot = make_uint4(w4[0], w4[1], w4[2], w4[3]);
            }
          } else {
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
          }
          fence_proxy_async_shared();          // the rows are written before TMA reads them
          __syncwarp();
          if (lane == 0) {
            box_store(dh);
            if constexpr (kMerge) {
              if (dh + 1 < D / 64) {
                bulk_wait_read();
                box_load(dh + 1);
              }
            }
          }
        }
        if (!ok) break;
        if (have_o) tc_fence_before();
        continue;
      }
      if (have_o) {
        ok = mbar_wait(&o_full[h], to & 1, s_abort, err, DEV_TIMEOUT_O);
        ++to;
        if (!__all_sync(0xffffffffu, ok)) break;
        tc_fence_after();
      }
      if constexpr (!kMerge) {
#pragma unroll
        for (int dh = 0; dh < D / 64; ++dh) {
          uint32_t w[32];   // 64 outputs of this row, packed in pairs
          if (have_o) {
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
      } else {
        // merge: the rows in place are read through the staging buffer the same way;
        // the loads of every 64-column chunk of the warp's 32 rows are issued before
        // the first is used, so their round trips to memory overlap
        const int cc = lane & 7;
        uint4 ovs[D / 64][8];
#pragma unroll
        for (int dh = 0; dh < D / 64; ++dh) {
#pragma unroll
          for (int it = 0; it < 8; ++it) {
            const int rr = it * 4 + (lane >> 3);
            const unsigned long long src =
                __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(orow), rr);
            ovs[dh][it] = make_uint4(0u, 0u, 0u, 0u);
            if (src)
              asm volatile("ld.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                           : "=r"(ovs[dh][it].x), "=r"(ovs[dh][it].y), "=r"(ovs[dh][it].z),
                             "=r"(ovs[dh][it].w)
                           : "l"(reinterpret_cast<const char*>(src) + dh * 128 + cc * 16));
          }
        }
#pragma unroll
        for (int dh = 0; dh < D / 64; ++dh) {
          __syncwarp();   // the previous round's readers are done with the buffer
#pragma unroll
          for (int it = 0; it < 8; ++it) {
            const int rr = it * 4 + (lane >> 3);
            *reinterpret_cast<uint4*>(stage + rr * 128 + ((cc ^ (rr & 7)) << 4)) = ovs[dh][it];
          }
          __syncwarp();
          uint32_t w[32];
#pragma unroll
          for (int half32 = 0; half32 < 2; ++half32) {
            uint32_t r[32];
            if (have_o) {
              tmem_ld32(tO + dh * 64 + half32 * 32, r);
              tmem_wait_ld();
              tmem_regs_ready(r);
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i) r[i] = 0u;
            }
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4) {
              const int c = half32 * 4 + c4;
              const uint4 v = *reinterpret_cast<const uint4*>(stage + lane * 128 + ((c ^ (lane & 7)) << 4));
              const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                float a, b2;
                unpack2<kBf16>(vv[j], a, b2);
                w[4 * c + j] = pack2<kBf16>(fmaf(w_old, a, __uint_as_float(r[8 * c4 + 2 * j]) * inv_l),
                                            fmaf(w_old, b2, __uint_as_float(r[8 * c4 + 2 * j + 1]) * inv_l));
              }
            }
          }
          __syncwarp();   // every lane has read its old row
#pragma unroll
          for (int c = 0; c < 8; ++c)
            *reinterpret_cast<uint4*>(stage + lane * 128 + ((c ^ (lane & 7)) << 4)) =
                make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
          __syncwarp();
#pragma unroll
          for (int it = 0; it < 8; ++it) {
            const int rr = it * 4 + (lane >> 3);
            const uint4 v = *reinterpret_cast<const uint4*>(stage + rr * 128 + ((cc ^ (rr & 7)) << 4));
            const unsigned long long dst =
                __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(orow), rr);
            if (dst) *reinterpret_cast<uint4*>(reinterpret_cast<char*>(dst) + dh * 128 + cc * 16) = v;
          }
        }
      }
      if (have_o) tc_fence_before();
    }
    // the warp's TMA traffic of the staging is finished before the CTA can exit: a box
    // load still in flight (an aborted merge) lands, every box store completes
    if (lane == 0) {
      if (epi_issued > epi_done) {
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(&epi_bar[warp], (epi_issued - 1) & 1)) {
          if (globaltimer() - t0 > kDrainLimitNs) { err.record(DEV_TIMEOUT_DRAIN); break; }
        }
      }
      bulk_wait_all();
    }
    __syncwarp();
    }   // kCG == 1
  }

  // ------------------------------------------------------------ teardown
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


// Launchers of one instantiation family each (head dim x residue mode), defined in
// csrc/attn_k*.cu so the sixteen-odd kernel instantiations compile in parallel.
using Tmap = CUtensorMap;
#define PA_DECLARE_LAUNCH(name)                                                            \
  int name(const Tmap& tq, const Tmap& tk, const Tmap& tv, const FwdParams& P, int grid, \
           int L, bool bf16, cudaStream_t stream);
PA_DECLARE_LAUNCH(launch_d128)
PA_DECLARE_LAUNCH(launch_d128_residue)
PA_DECLARE_LAUNCH(launch_d64)
PA_DECLARE_LAUNCH(launch_d64_residue)
PA_DECLARE_LAUNCH(launch_d128_merge)
PA_DECLARE_LAUNCH(launch_d128_residue_merge)
PA_DECLARE_LAUNCH(launch_d64_merge)
PA_DECLARE_LAUNCH(launch_d64_residue_merge)
PA_DECLARE_LAUNCH(launch_d128_gather)
PA_DECLARE_LAUNCH(launch_d64_gather)
PA_DECLARE_LAUNCH(launch_d128_pairs)
PA_DECLARE_LAUNCH(launch_d128_residue_pairs)
PA_DECLARE_LAUNCH(launch_d64_pairs)
PA_DECLARE_LAUNCH(launch_d64_residue_pairs)
#undef PA_DECLARE_LAUNCH

// Body of the launchers: pick the instantiation for (L, dtype).
template <int D, bool kRS, bool kMerge, bool kGather = false, int kCG = 1>
int launch_family(const Tmap& tq, const Tmap& tk, const Tmap& tv, const FwdParams& P, int grid,
                  int L, bool bf16, cudaStream_t stream) {
  auto go = [&](auto kernel) -> int {
    const int smem = kGather ? Smem<D, kCG>::kAllocGather : Smem<D, kCG>::kAlloc;
    PA_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
            "pa_attn_fwd");
    // the warpgroups' setmaxnreg shares must fit in the registers the CTA is launched
    // with; a split above them would never complete, so refuse to launch instead
    using R = Roles<kCG>;
    static std::atomic<int> regs_ok{0};   // checked once per instantiation
    cudaFuncAttributes fa;
    fa.numRegs = 1 << 20;
    if (!regs_ok.load(std::memory_order_relaxed))
      PA_CUDA(cudaFuncGetAttributes(&fa, kernel), "pa_attn_fwd");
    if (fa.numRegs * R::kThreads <
        R::kSoftmaxWarps * 32 * R::kSoftmaxRegs + (R::kThreads - R::kSoftmaxWarps * 32) * R::kOtherRegs)
      return fail(PA_ERR_UNSUPPORTED, "pa_attn_fwd: kernel built with %d registers per thread, "
                  "below its register split", fa.numRegs);
    regs_ok.store(1, std::memory_order_relaxed);
    kernel<<<grid, Roles<kCG>::kThreads, smem, stream>>>(tq, tk, tv, P);
    return PA_OK;
  };
  switch (L) {
    case 16: return bf16 ? go(attn_fwd_kernel<D, 16, true, kRS, kMerge, kGather, kCG>)
                         : go(attn_fwd_kernel<D, 16, false, kRS, kMerge, kGather, kCG>);
    case 32: return bf16 ? go(attn_fwd_kernel<D, 32, true, kRS, kMerge, kGather, kCG>)
                         : go(attn_fwd_kernel<D, 32, false, kRS, kMerge, kGather, kCG>);
    case 64: return bf16 ? go(attn_fwd_kernel<D, 64, true, kRS, kMerge, kGather, kCG>)
                         : go(attn_fwd_kernel<D, 64, false, kRS, kMerge, kGather, kCG>);
    default: return bf16 ? go(attn_fwd_kernel<D, 128, true, kRS, kMerge, kGather, kCG>)
                         : go(attn_fwd_kernel<D, 128, false, kRS, kMerge, kGather, kCG>);
  }
}

}  // namespace attn
}  // namespace pa
