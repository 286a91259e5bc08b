// Block-index builder: classifies every BQ x A tile of the (permuted) mask as
// dead / full / partial and writes the reference's BlockIndex arrays
// (gpu/blockindex.py:32-51) without materialising the N x N mask.
//
// One CTA per query block; a column permutation is staged in shared memory first
// when it fits.  Every tile is first decided from bounds alone, one tile per
// thread -- the min/max original coordinate of its rows and columns and, for
// lattice kinds, whether all rows (columns) share one residue modulo the lattice
// stride, which makes the lattice term constant over the tile (the usual case under
// a residue permutation).  Tiles the bounds cannot decide are queued and enumerated
// element by element, one warp per tile.  Live tiles are then compacted in
// ascending column order with a block-wide scan, so kv_idx is bit-identical to
// the reference's np.flatnonzero order.
#include <climits>
#include "common.cuh"
#include "capi_util.h"

namespace pa {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxTilesPerRow = 65536;   // N / A, bounded by the flag array in shared memory
constexpr int kMaxBQ = 4096;

enum : uint8_t { T_DEAD = 0, T_FULL = 1, T_PARTIAL = 2, T_QUEUED = 3, T_OVERFLOW = 4 };
constexpr int kUndCap = 1024;            // undecided tiles queued per row block

// 0 = dead, 1 = full, 3 = undecided.  Exact whenever it decides.
__device__ int classify_bounds(const Pred& p, int imin, int imax, int jmin, int jmax,
                               bool uniform, int dres) {
  const int dmin = imin - jmax, dmax = imax - jmin;
  if (dmax < 0) return 0;
  const bool causal_all = dmin >= 0;
  switch (p.kind) {
    case PA_CAUSAL:
      return causal_all ? 1 : 3;
    case PA_WINDOW:
      if (dmin >= p.p0) return 0;
      if (causal_all && dmax < p.p0) return 1;
      return 3;
    case PA_DILATED:
      if (uniform) {
        if (dres != 0) return 0;
        if (causal_all) return 1;
      }
      return 3;
    case PA_LOCAL_STRIDED:
      if (causal_all && dmax < p.p0) return 1;
      if (uniform) {
        if (dres == 0 && causal_all) return 1;
        if (dres != 0 && dmin >= p.p0) return 0;
      }
      return 3;
    case PA_TWOBAND:
      if (causal_all && dmax < p.p0) return 1;
      if (dmin >= p.p1 && dmin >= 0 && dmax < p.p1 + p.p2) return 1;
      if (dmin >= p.p0 && (dmax < p.p1 || dmin >= p.p1 + p.p2)) return 0;
      return 3;
    case PA_SINKS:
      if (causal_all && (dmax < p.p0 || jmax < p.p1)) return 1;
      if (dmin >= p.p0 && jmin >= p.p1) return 0;
      return 3;
    case PA_FAR_STRIDED:
      if (dmax < p.p0) return 0;
      if (uniform) {
        if (dres != 0) return 0;
        if (dmin >= p.p0) return 1;
      }
      return 3;
  }
  return 3;
}

// Live bits of `n` (<= 32) columns evaluated one by one; column c has original index
// cols[c] when given -- shared memory (the staged permutation) or global memory, so a
// generic load, not element_bits' read-only global load -- else j0 + (base + c) * dj.
__device__ uint32_t element_bits_any(const Pred& p, int i, const int* cols, int j0, int dj,
                                     int base, int n) {
  uint32_t w = 0;
  for (int c = 0; c < n; ++c) {
    const int j = cols ? cols[c] : j0 + (base + c) * dj;
    w |= (uint32_t)pred_live(p, i, j) << c;
  }
  return w;
}

__device__ __forceinline__ int warp_min(int v) {
  for (int o = 16; o; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ int warp_max(int v) {
  for (int o = 16; o; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Exclusive scan of one int per thread across the CTA; returns the total.
__device__ int block_exclusive_scan(int v, int* out, int* s_warp) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_warp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < kWarps ? s_warp[lane] : 0;
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < kWarps) s_warp[lane] = w;   // inclusive warp totals
  }
  __syncthreads();
  const int before = (warp ? s_warp[warp - 1] : 0) + x - v;
  *out = before;
  const int total = s_warp[kWarps - 1];
  __syncthreads();
  return total;
}

__global__ void __launch_bounds__(kThreads)
block_index_kernel(Pred pred, int N, int BQ, int A, const int32_t* __restrict__ perm_q,
                   const int32_t* __restrict__ perm_kv, const uint8_t* __restrict__ dense,
                   int32_t* __restrict__ kv_idx, int kv_stride, int32_t* __restrict__ kv_num,
                   int8_t* __restrict__ kv_partial, unsigned long long* __restrict__ stats,
                   int stage_kv) {
  extern __shared__ __align__(16) uint8_t smem[];
  int* rows_i = reinterpret_cast<int*>(smem);                 // [BQ]
  uint8_t* flags = smem + ((BQ * 4 + 15) & ~15);              // [nk]
  // perm_kv staged once per CTA when it fits: the per-tile column reads below are
  // then shared-memory reads instead of dependent global round trips
  int* cols_s = reinterpret_cast<int*>(flags + ((N / A + 15) & ~15));   // [N] when stage_kv
  __shared__ int s_warp[kWarps];
  __shared__ int s_red[4];
  __shared__ unsigned long long s_live;
  __shared__ int s_nund;                 // tiles the bounds left undecided
  __shared__ int s_und[kUndCap];

  const int nk = N / A;
  const int rb = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int mod = pred.mod;

  if (threadIdx.x == 0) {
    s_red[0] = INT_MAX; s_red[1] = INT_MIN; s_red[2] = 1; s_live = 0ull; s_nund = 0;
  }
  for (int r = threadIdx.x; r < BQ; r += kThreads) {
    const int row = rb * BQ + r;
    rows_i[r] = perm_q ? perm_q[row] : row;
  }
  if (stage_kv) {
    for (int c = threadIdx.x; c < N; c += kThreads) cols_s[c] = perm_kv[c];
  }
  const int32_t* cols = stage_kv ? cols_s : perm_kv;   // NULL: identity columns
  __syncthreads();

  // Row-block summary: min / max original row, and residue uniformity mod `mod`.
  {
    int mn = INT_MAX, mx = INT_MIN, uni = 1;
    const int r0 = mod > 1 ? rows_i[0] % mod : 0;
    for (int r = threadIdx.x; r < BQ; r += kThreads) {
      const int i = rows_i[r];
      mn = min(mn, i); mx = max(mx, i);
      if (mod > 1 && i % mod != r0) uni = 0;
    }
    mn = warp_min(mn); mx = warp_max(mx);
    uni = __all_sync(0xffffffffu, uni);
    if (lane == 0) {
      atomicMin(&s_red[0], mn); atomicMax(&s_red[1], mx);
      if (!uni) s_red[2] = 0;
    }
  }
  __syncthreads();
  const int imin = s_red[0], imax = s_red[1];
  const bool iuni = s_red[2] != 0;
  const int ires = mod > 1 ? rows_i[0] % mod : 0;

  // Pass 1, one tile per thread: every tile the bounds decide.  Column bounds are
  // closed-form for identity columns and read from the (staged) permutation otherwise.
  // Tiles the bounds cannot decide go to a queue the warps then share, so that the
  // few partial tiles of a row block are enumerated by different warps.
  unsigned long long live_t = 0;
  for (int t = threadIdx.x; t < nk; t += kThreads) {
    const int c0 = t * A;
    int cls = 3;
    if (!dense) {
      int mn, mx, uni = 1, jres;
      if (!cols) {
        mn = c0;
        mx = c0 + A - 1;
        jres = mod > 1 ? c0 % mod : 0;
        uni = A == 1;                       // consecutive columns: mixed residues
      } else {
        mn = mx = cols[c0];
        jres = mod > 1 ? mn % mod : 0;
        for (int c = 1; c < A; ++c) {
          const int j = cols[c0 + c];
          mn = min(mn, j);
          mx = max(mx, j);
          if (mod > 1 && j % mod != jres) uni = 0;
        }
      }
      const bool uniform = (mod <= 1) || (iuni && uni);
      const int dres = mod > 1 ? (((ires - jres) % mod) + mod) % mod : 0;
      cls = classify_bounds(pred, imin, imax, mn, mx, uniform, dres);
    }
    uint8_t flag = T_DEAD;
    if (cls == 1) {
      flag = T_FULL;
      live_t += (unsigned long long)BQ * A;
    } else if (cls == 3) {
      const int k = atomicAdd(&s_nund, 1);
      if (k < kUndCap) {
        s_und[k] = t;
        flag = T_QUEUED;
      } else {
        flag = T_OVERFLOW;                  // enumerated by the strided pass below
      }
    }
    flags[t] = flag;
  }
  if (live_t) atomicAdd(&s_live, live_t);
  __syncthreads();

  // Pass 2, one warp per undecided tile, counting live elements.  Mask kinds whose
  // live columns of a row form at most two ranges of a column progression (every
  // kind here, when the tile's columns are j0 + c*dj) are counted a row per lane, 32
  // columns per word in closed form (progression_bits); other tiles element by element.
  unsigned long long live_w = 0;
  auto enumerate = [&](int t) {
    const int c0 = t * A;
    int any = 0, all = 1;
    unsigned long long cnt = 0;
    bool ap = false;
    int j0 = c0, dj = 1;
    if (!dense) {
      ap = true;
      if (cols) {
        j0 = cols[c0];
        dj = A > 1 ? cols[c0 + 1] - j0 : 1;
        int ok = dj >= 1;
        for (int c = lane; c < A && ok; c += 32) ok = cols[c0 + c] == j0 + c * dj;
        ap = __all_sync(0xffffffffu, ok);
      }
    }
    if (ap) {
      const int sh = (dj & (dj - 1)) == 0 ? 31 - __clz(dj) : -1;
      for (int r = lane; r < BQ; r += 32) {
        const int i = rows_i[r];
        for (int base = 0; base < A; base += 32) {
          const int width = min(32, A - base);
          const uint32_t full = width == 32 ? 0xffffffffu : ((1u << width) - 1u);
          uint32_t w;
          if (!progression_bits(pred, i - j0, j0, dj, sh, base, A, w))
            w = element_bits_any(pred, i, cols ? cols + c0 + base : nullptr, j0, dj, base, width);
          w &= full;
          cnt += __popc(w);
          any |= w != 0u;
          all &= w == full;
        }
      }
    } else {
      // element by element (e = r * A + c, lanes stride by 32)
      int r = lane / A, c = lane % A;
      const int total = BQ * A;
      for (int e = lane; e < total; e += 32) {
        bool lv;
        if (dense) {
          lv = dense[(size_t)(rb * BQ + r) * N + c0 + c] != 0;
        } else {
          const int j = cols ? cols[c0 + c] : c0 + c;
          lv = pred_live(pred, rows_i[r], j);
        }
        any |= lv; all &= lv; cnt += lv;
        c += 32;
        while (c >= A) { c -= A; ++r; }
      }
    }
    any = __any_sync(0xffffffffu, any);
    all = __all_sync(0xffffffffu, all);
    for (int o = 16; o; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
    if (lane == 0) flags[t] = any ? (all ? T_FULL : T_PARTIAL) : T_DEAD;
    live_w += cnt;
  };
  const int nund = min(s_nund, kUndCap);
  for (int k = warp; k < nund; k += kWarps) enumerate(s_und[k]);
  if (s_nund > kUndCap)
    for (int t = warp; t < nk; t += kWarps)
      if (flags[t] == T_OVERFLOW) enumerate(t);
  if (lane == 0 && live_w) atomicAdd(&s_live, live_w);
  __syncthreads();

  // Ascending compaction of live tiles.
  const int chunk = (nk + kThreads - 1) / kThreads;
  const int t0 = min(nk, (int)threadIdx.x * chunk), t1 = min(nk, t0 + chunk);
  int mine = 0;
  for (int t = t0; t < t1; ++t) mine += flags[t] != T_DEAD;
  int pos;
  const int total = block_exclusive_scan(mine, &pos, s_warp);
  int32_t* idx_row = kv_idx + (size_t)rb * kv_stride;
  int8_t* par_row = kv_partial + (size_t)rb * kv_stride;
  for (int t = t0; t < t1; ++t) {
    const uint8_t f = flags[t];
    if (f != T_DEAD) {
      idx_row[pos] = t;
      par_row[pos] = f == T_PARTIAL ? 1 : 0;
      ++pos;
    }
  }
  for (int e = total + threadIdx.x; e < kv_stride; e += kThreads) {
    idx_row[e] = 0;
    par_row[e] = 0;
  }
  if (threadIdx.x == 0) {
    kv_num[rb] = total;
    atomicAdd(&stats[0], (unsigned long long)total * BQ * A);
    atomicAdd(&stats[1], s_live);
    atomicMax(&stats[2], (unsigned long long)total);
    atomicAdd(&stats[3], (unsigned long long)total);
  }
}

int launch_block_index(const Pred& pred, const uint8_t* dense, int32_t N, int32_t BQ, int32_t A,
                       const int32_t* perm_q, const int32_t* perm_kv, int32_t* kv_idx,
                       int32_t kv_stride, int32_t* kv_num, int8_t* kv_partial, int64_t* stats,
                       cudaStream_t stream, const char* who) {
  PA_CHECK_ARG(N >= 1 && N < (1 << 24), "%s: N=%d out of range [1, 2^24)", who, N);
  PA_CHECK_ARG(BQ >= 1 && A >= 1, "%s: BQ=%d and A=%d must be positive", who, BQ, A);
  PA_CHECK_ARG(N % BQ == 0 && N % A == 0,
               "%s: N=%d must be a multiple of BQ=%d and A=%d", who, N, BQ, A);
  PA_CHECK_ARG(kv_idx && kv_num && kv_partial && stats, "%s: null output pointer", who);
  PA_CHECK_ARG(kv_stride >= N / A, "%s: kv_stride=%d < N/A=%d", who, kv_stride, N / A);
  if (N / A > kMaxTilesPerRow || BQ > kMaxBQ)
    return fail(PA_ERR_UNSUPPORTED, "%s: N/A=%d (max %d) or BQ=%d (max %d) too large", who,
                N / A, kMaxTilesPerRow, BQ, kMaxBQ);
  PA_CUDA(cudaMemsetAsync(stats, 0, 4 * sizeof(int64_t), stream), who);
  const size_t base = ((size_t)(BQ * 4 + 15) & ~size_t(15)) + (((size_t)(N / A) + 15) & ~size_t(15));
  // stage perm_kv in shared memory when it fits in what a CTA can have
  const int stage_kv = (perm_kv && !dense && base + (size_t)N * 4 <= 200 * 1024) ? 1 : 0;
  const size_t smem = base + (stage_kv ? (size_t)N * 4 : 0);
  if (smem > 48 * 1024) {
    PA_CUDA(cudaFuncSetAttribute(block_index_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem), who);
  }
  block_index_kernel<<<N / BQ, kThreads, smem, stream>>>(
      pred, N, BQ, A, perm_q, perm_kv, dense, kv_idx, kv_stride, kv_num, kv_partial,
      reinterpret_cast<unsigned long long*>(stats), stage_kv);
  return check_launch(who);
}

}  // namespace

int make_pred(const pa_pred* p, Pred* out, const char* who) {
  PA_CHECK_ARG(p != nullptr, "%s: null predicate", who);
  Pred q{p->kind, p->p0, p->p1, p->p2, 0.f, 0};
  switch (p->kind) {
    case PA_CAUSAL:
      break;
    case PA_WINDOW:
      PA_CHECK_ARG(p->p0 >= 0, "%s: WINDOW needs p0 >= 0", who);
      break;
    case PA_DILATED:
      PA_CHECK_ARG(p->p0 >= 1, "%s: DILATED needs p0 >= 1", who);
      q.mod = p->p0;
      break;
    case PA_LOCAL_STRIDED:
      PA_CHECK_ARG(p->p1 >= 1, "%s: LOCAL_STRIDED needs p1 >= 1", who);
      q.mod = p->p1;
      break;
    case PA_TWOBAND:
    case PA_SINKS:
      break;
    case PA_FAR_STRIDED:
      PA_CHECK_ARG(p->p1 >= 1, "%s: FAR_STRIDED needs p1 >= 1", who);
      q.mod = p->p1;
      break;
    default:
      return fail(PA_ERR_ARG, "%s: unknown mask kind %d", who, p->kind);
  }
  q.inv_mod = q.mod > 0 ? 1.0f / (float)q.mod : 0.f;
  *out = q;
  return PA_OK;
}

}  // namespace pa

extern "C" int pa_block_index(const pa_pred* pred, int32_t N, int32_t BQ, int32_t A,
                              const int32_t* perm_q, const int32_t* perm_kv, int32_t* kv_idx,
                              int32_t kv_stride, int32_t* kv_num, int8_t* kv_partial,
                              int64_t* stats, pa_stream_t stream) {
  pa::Pred p;
  int rc = pa::make_pred(pred, &p, "pa_block_index");
  if (rc) return rc;
  return pa::launch_block_index(p, nullptr, N, BQ, A, perm_q, perm_kv, kv_idx, kv_stride,
                                kv_num, kv_partial, stats, (cudaStream_t)stream,
                                "pa_block_index");
}

extern "C" int pa_block_index_dense(const uint8_t* mask, int32_t N, int32_t BQ, int32_t A,
                                    int32_t* kv_idx, int32_t kv_stride, int32_t* kv_num,
                                    int8_t* kv_partial, int64_t* stats, pa_stream_t stream) {
  PA_CHECK_ARG(mask != nullptr, "pa_block_index_dense: null mask");
  pa::Pred p{PA_CAUSAL, 0, 0, 0, 0.f, 0};
  return pa::launch_block_index(p, mask, N, BQ, A, nullptr, nullptr, kv_idx, kv_stride, kv_num,
                                kv_partial, stats, (cudaStream_t)stream, "pa_block_index_dense");
}
