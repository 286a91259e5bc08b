// Block-sparse flash-attention forward for sm_100a (tcgen05 + TMEM + TMA).
//
// Replaces the reference's Triton kernel (gpu/triton_attn.py:62-182) and its
// launcher (:185-241) with the same semantics: per query row, online softmax over
// the KV tiles the block index lists; the mask predicate is evaluated in
// original coordinates (perm_q[i] - perm_kv[j]) on partial tiles only; a row with
// no live key yields O = 0.  In addition it writes LSE (natural log, -inf for a
// dead row).
//
// Work decomposition.  A CTA owns 256 query rows of one (batch, head) at a time
// as two 128-row halves that share one stream of 128-row KV "super-tiles": the
// plan kernel merges the two halves' tile lists into one ascending union and
// records, per tile and half, whether the tile is dead, full or partial for that
// half.  A super-tile is made of 128/L segments of L = min(A, 128) KV rows, each
// fetched by its own TMA box, so KV tiles of 16/32/64 rows are gathered at tile
// granularity while every MMA runs at N = 128.  Segments past the end of the list
// are fetched from row N (out of bounds, zero-filled) and masked.
//
// Warp roles (384 threads):
//   warps 0-3  softmax, half 0 (TMEM lanes 0-127)    warps 4-7  softmax, half 1
//   warp 8     TMA producer (Q tiles, K/V ring)      warp 9     MMA issuer, TMEM owner
//   warps 10-11 idle; they complete the third warpgroup so its registers can be
//   handed to the softmax warpgroups (setmaxnreg)
// TMEM (512 columns): S0 [0,128), S1 [128,256), O0 [256, 256+D), O1 [256+D, 256+2D).
// P (16-bit) is written by the softmax warps into columns [64,128) of its S buffer
// and consumed from TMEM by the P.V MMA.  Per KV super-tile j the MMA warp issues,
// for each half h in turn, PV_h(j-1) then S_h(j); tcgen05 ops of one thread
// complete in order, so the commit that publishes S_h(j) also proves PV_h(j-1)
// complete, which is what lets the softmax warps rescale O_h in place.
//
// Every wait on a barrier is bounded (common.cuh mbar_wait): on expiry the CTA
// records a status in the workspace, stops issuing work, drains what it issued and
// frees TMEM before exiting.
#include <cuda.h>
#include <math.h>
#include <atomic>
#include <cstring>
#include <mutex>
#include "attn_kernel.cuh"
#include "attn_kernel_db.cuh"

namespace pa {
namespace attn {
namespace {

constexpr int kPlanThreads = 256;

// One CTA per 256-row pair: union of the listed tiles of the query blocks that
// cover each 128-row half, with each half's status.  A tile is full for a half
// when every covering block lists it as full, dead when no covering block lists
// it, partial otherwise (the predicate then decides element by element).
// Per listed tile of every pair, the facts the softmax needs to build its live
// bits without touching the permutation: x = original index j0 of the tile's first
// column; y = dj (bits 0-15; the original indices are j0 + c*dj when they form a
// progression), log2(dj) (bits 16-19) when dj is a power of two (bit 20),
// progression flag (bit 21), and the two halves' status (bits 24-27).
__device__ void plan_desc_pair(const PlanView& pv, int p, int cnt,
                               const int32_t* __restrict__ perm_kv, int A, int rs, int nb) {
  const int32_t* ent = pv.entries + (size_t)p * pv.cap;
  const uint8_t* sts = pv.status + (size_t)p * pv.cap;
  uint2* desc = pv.desc + (size_t)p * pv.cap;
  for (int e = threadIdx.x; e < cnt; e += kPlanThreads) {
    const int row0 = ent[e] * A;
    int j0 = row0, dj = 1;
    bool ap = true;
    if (rs > 0) {                 // a residue block holds original rows j0, j0 + rs, ...
      j0 = (row0 % nb) * rs + row0 / nb;
      dj = rs;
    } else if (perm_kv) {
      j0 = perm_kv[row0];
      dj = A >= 2 ? perm_kv[row0 + 1] - j0 : 1;
      ap = dj >= 1 && dj <= 0xffff;
      for (int c = 2; c < A && ap; ++c) ap = perm_kv[row0 + c] == j0 + c * dj;
      if (!ap) dj = 0;
    }
    uint32_t y = (uint32_t)dj & 0xffffu;
    if (ap && (dj & (dj - 1)) == 0) y |= ((uint32_t)(31 - __clz(dj)) << 16) | (1u << 20);
    if (ap) y |= 1u << 21;
    y |= (uint32_t)(sts[e] & 0xf) << 24;
    desc[e] = make_uint2((uint32_t)j0, y);
  }
}

__global__ void __launch_bounds__(kPlanThreads)
plan_pairs_kernel(const int32_t* __restrict__ kv_idx, const int32_t* __restrict__ kv_num,
                  const int8_t* __restrict__ kv_partial, int kv_stride, int N, int BQ,
                  PlanView pv, const int32_t* __restrict__ perm_kv, int A, int rs, int nb) {
  extern __shared__ uint8_t cnt[];   // [4][cap]: present h0, full h0, present h1, full h1
  __shared__ int s_warp[kPlanThreads / 32];
  const int cap = pv.cap;
  const int p = blockIdx.x;
  for (int t = threadIdx.x; t < 4 * cap; t += kPlanThreads) cnt[t] = 0;
  __syncthreads();
  int nblk[2] = {0, 0};
  for (int h = 0; h < 2; ++h) {
    const int r0 = p * 2 * BM + h * BM;
    if (r0 >= N) continue;
    const int r1 = min(r0 + BM, N);
    const int b0 = r0 / BQ, b1 = (r1 - 1) / BQ;
    nblk[h] = b1 - b0 + 1;
    uint8_t* pres = cnt + (2 * h) * cap;
    uint8_t* full = cnt + (2 * h + 1) * cap;
    for (int b = b0; b <= b1; ++b) {
      const int n = kv_num[b];
      for (int e = threadIdx.x; e < n; e += kPlanThreads) {
        const int t = kv_idx[(size_t)b * kv_stride + e];
        if ((unsigned)t < (unsigned)cap) {
          pres[t] += 1;
          full[t] += kv_partial[(size_t)b * kv_stride + e] == 0 ? 1 : 0;
        }
      }
      __syncthreads();   // one block at a time: a tile appears at most once per block
    }
  }
  // ascending compaction of tiles live in either half
  const int chunk = (cap + kPlanThreads - 1) / kPlanThreads;
  const int t0 = min(cap, (int)threadIdx.x * chunk), t1 = min(cap, t0 + chunk);
  auto status_of = [&](int t) -> int {
    int st = 0;
    for (int h = 0; h < 2; ++h) {
      const int pr = cnt[(2 * h) * cap + t], fu = cnt[(2 * h + 1) * cap + t];
      const int s = (nblk[h] == 0 || pr == 0) ? 0 : (fu == nblk[h] ? 1 : 2);
      st |= s << (2 * h);
    }
    return st;
  };
  int mine = 0;
  for (int t = t0; t < t1; ++t) mine += status_of(t) != 0;
  // block exclusive scan
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = mine;
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_warp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < kPlanThreads / 32 ? s_warp[lane] : 0;
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < kPlanThreads / 32) s_warp[lane] = w;
  }
  __syncthreads();
  int pos = (warp ? s_warp[warp - 1] : 0) + x - mine;
  const int total = s_warp[kPlanThreads / 32 - 1];
  int32_t* ent = pv.entries + (size_t)p * cap;
  uint8_t* sts = pv.status + (size_t)p * cap;
  for (int t = t0; t < t1; ++t) {
    const int st = status_of(t);
    if (st) {
      ent[pos] = t;
      sts[pos] = (uint8_t)st;
      ++pos;
    }
  }
  if (threadIdx.x == 0) pv.pair_cnt[p] = total;
  __syncthreads();   // this pair's entries and statuses are written
  plan_desc_pair(pv, p, total, perm_kv, A, rs, nb);
}

// Longest-first order of the pairs (stable on ties); work item `it` of the forward
// is pair order[it / BH] of head it % BH, fetched dynamically by the CTAs.
__global__ void plan_order_kernel(PlanView pv) {
  const int n = pv.npairs;
  for (int p = threadIdx.x; p < n; p += blockDim.x) {
    const int c = pv.pair_cnt[p];
    int rank = 0;
    for (int q = 0; q < n; ++q) {
      const int d = pv.pair_cnt[q];
      rank += (d > c) || (d == c && q < p);
    }
    pv.order[rank] = p;
  }
  if (threadIdx.x == 0) {
    *pv.err = 0;   // a new plan starts with a clean status
    *pv.done = 0;
    pv.sched[0] = 0;
    pv.sched[1] = 0;
  }
}


}  // namespace

// ------------------------------------------------------------- host side
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                              const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                              const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                              CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn get_encode() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  });
  return fn;
}

// [BH][N][D] 16-bit tensor, box = 64 columns x `rows` rows x 1 head, 128-byte swizzle.
// With a residue stride rs > 0 the row axis is viewed as (rs, N/rs) -- original row
// i = j * rs + r sits at coordinates (r, j) -- and a box of `rows` rows walks j, i.e.
// it reads rows r, r + rs, r + 2 rs, ...: one tile of the residue-permuted order.
int make_tmap(CUtensorMap* m, const void* base, int dtype, int BH, int N, int D,
              long long row_stride, long long bh_stride, int rows, int rs, const char* name) {
  EncodeFn enc = get_encode();
  if (!enc) return fail(PA_ERR_CUDA, "pa_attn_fwd: cuTensorMapEncodeTiled unavailable");
  const cuuint32_t rank = rs > 0 ? 4 : 3;
  cuuint64_t dims[4], strides[3];
  cuuint32_t box[4], estr[4] = {1, 1, 1, 1};
  if (rs > 0) {
    dims[0] = D; dims[1] = rs; dims[2] = N / rs; dims[3] = BH;
    strides[0] = (cuuint64_t)row_stride * 2;
    strides[1] = (cuuint64_t)row_stride * 2 * rs;
    strides[2] = (cuuint64_t)bh_stride * 2;
    box[0] = 64; box[1] = 1; box[2] = rows; box[3] = 1;
  } else {
    dims[0] = D; dims[1] = N; dims[2] = BH;
    strides[0] = (cuuint64_t)row_stride * 2;
    strides[1] = (cuuint64_t)bh_stride * 2;
    box[0] = 64; box[1] = rows; box[2] = 1;
  }
  CUresult r = enc(m, dtype == PA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                   rank, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(PA_ERR_ARG, "pa_attn_fwd: tensor map for %s rejected (CUresult %d): check "
                "16-byte alignment of the base and strides", name, (int)r);
  return PA_OK;
}

// The reference's class-B emulation knobs are set (gather_kv, or a row multiplier).
bool gathered(const pa_attn_args* a) { return a->gather_kv || a->gather_mult > 1; }

// Softmax threads per query row the forward runs with.  0 chooses: two where they were
// measured faster -- tiles at most 32 columns wide (several segments per super-tile,
// so more per-tile mask work to share) or D = 64 -- unless the call needs a kernel
// that has only one (merge, 64-row super-tiles, gathered K/V); one otherwise.
int effective_row_threads(const pa_attn_args* a) {
  if (a->row_threads) return a->row_threads;
  if (a->merge || a->kv_rows == 64 || gathered(a)) return 1;
  return (a->A <= 32 || a->D == 64) ? 2 : 1;
}

// [BH * rows_per_head][D] 16-bit view of K or V for four-row gathers: box = 64 columns
// x 1 row, 128-byte swizzle; row j of head b is row b * rows_per_head + j.
int make_tmap_gather(CUtensorMap* m, const void* base, int dtype, int BH, int N, int D,
                     long long row_stride, long long bh_stride, const char* name) {
  EncodeFn enc = get_encode();
  if (!enc) return fail(PA_ERR_CUDA, "pa_attn_fwd: cuTensorMapEncodeTiled unavailable");
  const long long per_head = bh_stride / row_stride;
  cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)((long long)(BH - 1) * per_head + N)};
  cuuint64_t strides[1] = {(cuuint64_t)row_stride * 2};
  cuuint32_t box[2] = {64, 1}, estr[2] = {1, 1};
  CUresult r = enc(m, dtype == PA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                   2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(PA_ERR_ARG, "pa_attn_fwd: gather tensor map for %s rejected (CUresult %d): "
                "check 16-byte alignment of the base and strides", name, (int)r);
  return PA_OK;
}

int check_args(const pa_attn_args* a, const char* who) {
  PA_CHECK_ARG(a != nullptr, "%s: null args", who);
  PA_CHECK_ARG(a->q && a->k && a->v && a->o, "%s: null q/k/v/o", who);
  PA_CHECK_ARG(a->kv_num, "%s: null kv_num", who);
  PA_CHECK_ARG(a->kv_stride >= 0, "%s: kv_stride=%d < 0", who, a->kv_stride);
  PA_CHECK_ARG(a->kv_stride == 0 || (a->kv_idx && a->kv_partial),
               "%s: null kv_idx / kv_partial", who);
  PA_CHECK_ARG(a->BH >= 1 && a->N >= 1 && a->N < (1 << 24), "%s: bad BH=%d N=%d", who, a->BH,
               a->N);
  PA_CHECK_ARG(a->D == 64 || a->D == 128, "%s: D=%d unsupported (64 or 128)", who, a->D);
  PA_CHECK_ARG(a->dtype == PA_BF16 || a->dtype == PA_F16, "%s: bad dtype %d", who, a->dtype);
  PA_CHECK_ARG(a->BQ >= 1 && a->A >= 1, "%s: BQ=%d, A=%d must be positive", who, a->BQ, a->A);
  PA_CHECK_ARG(a->N % a->BQ == 0 && a->N % a->A == 0,
               "%s: N=%d must be a multiple of BQ=%d and A=%d", who, a->N, a->BQ, a->A);
  PA_CHECK_ARG(a->A % 16 == 0 && (a->A <= 128 ? 128 % a->A == 0 : a->A % 128 == 0),
               "%s: A=%d unsupported (16, 32, 64, 128 or a multiple of 128)", who, a->A);
  PA_CHECK_ARG(a->N / a->A <= 65536 / 4, "%s: N/A=%d too many tiles per row", who,
               a->N / a->A);
  PA_CHECK_ARG(a->merge == 0 || a->merge == 1, "%s: merge=%d must be 0 or 1", who, a->merge);
  PA_CHECK_ARG(a->kv_rows == 0 || a->kv_rows == 128 || a->kv_rows == 64,
               "%s: kv_rows=%d must be 0, 128 or 64", who, a->kv_rows);
  if (a->kv_rows == 64 && a->merge)
    return fail(PA_ERR_UNSUPPORTED, "%s: kv_rows=64 cannot be combined with merge", who);
  PA_CHECK_ARG(!a->merge || a->lse, "%s: merge needs the LSE of the result in place (lse)", who);
  PA_CHECK_ARG(a->sched_heads >= 0, "%s: sched_heads=%d < 0", who, a->sched_heads);
  PA_CHECK_ARG(a->row_threads >= 0 && a->row_threads <= 2, "%s: row_threads=%d must be 0, 1 or 2",
               who, a->row_threads);
  if (a->row_threads == 2 && (a->merge || a->kv_rows == 64 || a->gather_kv || a->gather_mult > 1))
    return fail(PA_ERR_UNSUPPORTED, "%s: row_threads=2 cannot be combined with merge, "
                "kv_rows=64 or gathered K/V", who);
  PA_CHECK_ARG(a->gather_kv == 0 || a->gather_kv == 1, "%s: gather_kv=%d must be 0 or 1", who,
               a->gather_kv);
  PA_CHECK_ARG(a->gather_mult >= 0 && a->gather_mult <= 16,
               "%s: gather_mult=%d must be in 1..16", who, a->gather_mult);
  PA_CHECK_ARG(a->gather_scatter == 0 || a->gather_scatter == 1,
               "%s: gather_scatter=%d must be 0 or 1", who, a->gather_scatter);
  if (gathered(a)) {
    if (a->residue_stride || a->merge || a->kv_rows == 64)
      return fail(PA_ERR_UNSUPPORTED, "%s: gather_kv / gather_mult cannot be combined with "
                  "residue_stride, merge or kv_rows=64", who);
    PA_CHECK_ARG(!a->perm_kv || aligned(a->perm_kv, 16),
                 "%s: gathered K/V need a 16-byte aligned perm_kv", who);
    const int64_t ks[2][2] = {{a->k_bh_stride, a->k_row_stride}, {a->v_bh_stride, a->v_row_stride}};
    for (int t = 0; t < 2; ++t) {
      const int64_t bs = ks[t][0], rw = ks[t][1];
      if (rw <= 0 || bs < 0 || bs % rw != 0)
        return fail(PA_ERR_UNSUPPORTED, "%s: gathered K/V need %s head stride %lld to be a "
                    "multiple of its row stride %lld", who, t ? "v" : "k", (long long)bs,
                    (long long)rw);
      if ((int64_t)(a->BH - 1) * (bs / rw) + a->N > INT32_MAX)
        return fail(PA_ERR_UNSUPPORTED, "%s: gathered K/V: %s spans more than 2^31 rows", who,
                    t ? "v" : "k");
    }
  }
  if (a->residue_stride != 0) {
    const int rs = a->residue_stride;
    PA_CHECK_ARG(rs >= 1 && a->N % rs == 0, "%s: residue_stride=%d must divide N=%d", who, rs,
                 a->N);
    const int nb = a->N / rs;
    PA_CHECK_ARG(nb % BM == 0 && nb % a->A == 0,
                 "%s: N/residue_stride=%d must be a multiple of 128 and of A=%d", who, nb, a->A);
    PA_CHECK_ARG(!a->perm_q && !a->perm_kv && !a->o_row_map,
                 "%s: perm_q, perm_kv and o_row_map are implied by residue_stride; pass NULL", who);
  }
  return PA_OK;
}

// Epoch of the next forward launch: 24 bits, never 0 (0 is a clean status word).
uint32_t next_epoch() {
  static std::atomic<uint32_t> counter{0};
  return counter.fetch_add(1, std::memory_order_relaxed) % 0xffffffu + 1u;
}

int launch_fwd(const pa_attn_args* a, const PlanView& pv, cudaStream_t stream,
               uint64_t wait_ns = kWaitLimitNs, int withhold_q = 0) {
  CUtensorMap tq, tk, tv;
  const bool rows64 = a->kv_rows == 64;
  const int bn = rows64 ? db::BN : BN;
  const int L = a->A < bn ? a->A : bn;
  int rc;
  const int rs = a->residue_stride;
  if ((rc = make_tmap(&tq, a->q, a->dtype, a->BH, a->N, a->D, a->q_row_stride, a->q_bh_stride,
                      BM, rs, "q")))
    return rc;
  const bool gather = gathered(a);
  if (gather) {
    if ((rc = make_tmap_gather(&tk, a->k, a->dtype, a->BH, a->N, a->D, a->k_row_stride,
                               a->k_bh_stride, "k")))
      return rc;
    if ((rc = make_tmap_gather(&tv, a->v, a->dtype, a->BH, a->N, a->D, a->v_row_stride,
                               a->v_bh_stride, "v")))
      return rc;
  } else {
    if ((rc = make_tmap(&tk, a->k, a->dtype, a->BH, a->N, a->D, a->k_row_stride,
                        a->k_bh_stride, L, rs, "k")))
      return rc;
    if ((rc = make_tmap(&tv, a->v, a->dtype, a->BH, a->N, a->D, a->v_row_stride,
                        a->v_bh_stride, L, rs, "v")))
      return rc;
  }
  Pred pred;
  if ((rc = make_pred(&a->pred, &pred, "pa_attn_fwd"))) return rc;
  PA_CHECK_ARG(aligned(a->o, 16) && a->o_row_stride % 8 == 0 && a->o_bh_stride % 8 == 0,
               "pa_attn_fwd: o must be 16-byte aligned with strides multiple of 8 elements");
  FwdParams P;
  memset(&P.tm_o, 0, sizeof(P.tm_o));
  if (!a->o_row_map && (rc = make_tmap(&P.tm_o, a->o, a->dtype, a->BH, a->N, a->D,
                                       a->o_row_stride, a->o_bh_stride, 32, rs, "o")))
    return rc;
  P.BH = a->BH;
  P.N = a->N;
  P.A = a->A;
  P.rs = rs;
  P.nb = rs > 0 ? a->N / rs : a->N;
  P.perm_q = a->perm_q;
  P.perm_kv = a->perm_kv;
  P.o_row_map = a->o_row_map;
  P.o = a->o;
  P.lse = a->lse;
  P.o_bh_stride = a->o_bh_stride;
  P.o_row_stride = a->o_row_stride;
  P.lse_bh_stride = a->lse_bh_stride;
  P.pred = pred;
  const float scale = a->scale > 0.f ? a->scale : 1.0f / sqrtf((float)a->D);
  P.scale_log2 = scale * 1.4426950408889634f;
  P.pv = pv;
  const uint32_t fmt = a->dtype == PA_BF16 ? 1u : 0u;
  P.idesc_qk = make_idesc_f16(fmt, BM, bn, 0, 0);
  P.idesc_pv = make_idesc_f16(fmt, BM, a->D, 0, 1);
  P.total_items = pv.npairs * a->BH;
  // heads per scheduling group (all heads unless the caller asks for groups)
  P.hg = a->sched_heads > 0 && a->sched_heads < a->BH ? a->sched_heads : a->BH;
  P.g_kbh = gather ? (int)(a->k_bh_stride / a->k_row_stride) : 0;
  P.g_vbh = gather ? (int)(a->v_bh_stride / a->v_row_stride) : 0;
  P.g_kv = a->gather_kv;
  P.g_mult = a->gather_mult > 1 ? a->gather_mult : 1;
  P.g_scatter = a->gather_scatter;
  P.err.word = pv.err;
  P.err.epoch = next_epoch();
  P.err.limit_ns = wait_ns;
  P.err_q = P.err;
  if (withhold_q) P.err_q.limit_ns = wait_ns / 4;
  P.withhold_q = withhold_q;

  int dev = 0, sms = 148;
  PA_CUDA(cudaGetDevice(&dev), "pa_attn_fwd");
  PA_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "pa_attn_fwd");
  const int grid = P.total_items < sms ? P.total_items : sms;

  const bool bf16 = a->dtype == PA_BF16;
  int rc2;
  if (gather)
    rc2 = a->D == 128 ? launch_d128_gather(tq, tk, tv, P, grid, L, bf16, stream)
                      : launch_d64_gather(tq, tk, tv, P, grid, L, bf16, stream);
  else if (effective_row_threads(a) == 2 && a->D == 128)
    rc2 = rs > 0 ? launch_d128_residue_pairs(tq, tk, tv, P, grid, L, bf16, stream)
                 : launch_d128_pairs(tq, tk, tv, P, grid, L, bf16, stream);
  else if (effective_row_threads(a) == 2)
    rc2 = rs > 0 ? launch_d64_residue_pairs(tq, tk, tv, P, grid, L, bf16, stream)
                 : launch_d64_pairs(tq, tk, tv, P, grid, L, bf16, stream);
  else if (rows64 && a->D == 128)
    rc2 = rs > 0 ? db::launch_d128_residue(tq, tk, tv, P, grid, L, bf16, stream)
                 : db::launch_d128(tq, tk, tv, P, grid, L, bf16, stream);
  else if (rows64)
    rc2 = rs > 0 ? db::launch_d64_residue(tq, tk, tv, P, grid, L, bf16, stream)
                 : db::launch_d64(tq, tk, tv, P, grid, L, bf16, stream);
  else if (a->D == 128)
    rc2 = a->merge ? (rs > 0 ? launch_d128_residue_merge(tq, tk, tv, P, grid, L, bf16, stream)
                             : launch_d128_merge(tq, tk, tv, P, grid, L, bf16, stream))
                   : (rs > 0 ? launch_d128_residue(tq, tk, tv, P, grid, L, bf16, stream)
                             : launch_d128(tq, tk, tv, P, grid, L, bf16, stream));
  else
    rc2 = a->merge ? (rs > 0 ? launch_d64_residue_merge(tq, tk, tv, P, grid, L, bf16, stream)
                             : launch_d64_merge(tq, tk, tv, P, grid, L, bf16, stream))
                   : (rs > 0 ? launch_d64_residue(tq, tk, tv, P, grid, L, bf16, stream)
                             : launch_d64(tq, tk, tv, P, grid, L, bf16, stream));
  if (rc2) return rc2;
  return check_launch("pa_attn_fwd");
}

}  // namespace
}  // namespace pa

extern "C" size_t pa_attn_workspace_size(const pa_attn_args* a) {
  if (!a || a->N < 1 || a->A < 1) return 0;
  return pa::attn::plan_sizes(a->N, a->A).total;
}

extern "C" int pa_attn_plan(const pa_attn_args* a, void* ws, size_t ws_bytes,
                            pa_stream_t stream) {
  using namespace pa;
  using namespace pa::attn;
  int rc = check_args(a, "pa_attn_plan");
  if (rc) return rc;
  const PlanSizes sz = plan_sizes(a->N, a->A);
  PA_CHECK_ARG(ws && ws_bytes >= sz.total && aligned(ws, 256),
               "pa_attn_plan: workspace must be 256-byte aligned and >= %zu bytes", sz.total);
  const PlanView pv = plan_view(ws, a->N, a->A);
  const size_t smem = 4ull * pv.cap;
  if (smem > 48 * 1024)
    PA_CUDA(cudaFuncSetAttribute(plan_pairs_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem), "pa_attn_plan");
  const cudaStream_t s = (cudaStream_t)stream;
  const int rs = a->residue_stride;
  plan_pairs_kernel<<<pv.npairs, kPlanThreads, smem, s>>>(a->kv_idx, a->kv_num, a->kv_partial,
                                                         a->kv_stride, a->N, a->BQ, pv,
                                                         a->perm_kv, a->A, rs,
                                                         rs > 0 ? a->N / rs : a->N);
  if ((rc = check_launch("pa_attn_plan"))) return rc;
  plan_order_kernel<<<1, 256, 0, s>>>(pv);
  return check_launch("pa_attn_plan");
}

extern "C" int pa_attn_fwd(const pa_attn_args* a, void* ws, size_t ws_bytes,
                           pa_stream_t stream) {
  using namespace pa;
  using namespace pa::attn;
  int rc = check_args(a, "pa_attn_fwd");
  if (rc) return rc;
  const PlanSizes sz = plan_sizes(a->N, a->A);
  PA_CHECK_ARG(ws && ws_bytes >= sz.total && aligned(ws, 256),
               "pa_attn_fwd: workspace must be 256-byte aligned and >= %zu bytes", sz.total);
  return launch_fwd(a, plan_view(ws, a->N, a->A), (cudaStream_t)stream);
}

extern "C" int pa_attn_fwd_withheld(const pa_attn_args* a, void* ws, size_t ws_bytes,
                                    int64_t wait_limit_ns, pa_stream_t stream) {
  using namespace pa;
  using namespace pa::attn;
  int rc = check_args(a, "pa_attn_fwd_withheld");
  if (rc) return rc;
  if (gathered(a))
    return fail(PA_ERR_UNSUPPORTED, "pa_attn_fwd_withheld: not for gathered K/V");
  PA_CHECK_ARG(wait_limit_ns >= 1000 && wait_limit_ns <= (int64_t)kWaitLimitNs,
               "pa_attn_fwd_withheld: wait_limit_ns=%lld outside [1 us, 1 s]",
               (long long)wait_limit_ns);
  const PlanSizes sz = plan_sizes(a->N, a->A);
  PA_CHECK_ARG(ws && ws_bytes >= sz.total && aligned(ws, 256),
               "pa_attn_fwd_withheld: workspace must be 256-byte aligned and >= %zu bytes",
               sz.total);
  return launch_fwd(a, plan_view(ws, a->N, a->A), (cudaStream_t)stream,
                    (uint64_t)wait_limit_ns, 1);
}

namespace pa {
namespace attn {
// Status of the last forward on the workspace at `ws` (device memory), synchronising
// `stream`: the error word and the epoch of the last launch that finished.
int read_status(const void* ws, int32_t* status_host, cudaStream_t stream, const char* who) {
  int32_t words[2] = {0, 0};
  const char* b = static_cast<const char*>(ws);
  PA_CUDA(cudaMemcpyAsync(&words[0], b, sizeof(int32_t), cudaMemcpyDeviceToHost, stream), who);
  PA_CUDA(cudaMemcpyAsync(&words[1], b + 128, sizeof(int32_t), cudaMemcpyDeviceToHost, stream),
          who);
  PA_CUDA(cudaStreamSynchronize(stream), who);
  *status_host = launch_status(words[0], words[1]);
  return *status_host ? PA_ERR_DEVICE : PA_OK;
}
}  // namespace attn
}  // namespace pa

extern "C" int pa_attn_status(const void* ws, int32_t* status_host, pa_stream_t stream) {
  PA_CHECK_ARG(ws && status_host, "pa_attn_status: null pointer");
  return pa::attn::read_status(ws, status_host, (cudaStream_t)stream, "pa_attn_status");
}
