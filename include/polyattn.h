/*
 * polyattn.h -- C ABI of libpolyattn_sm100.so, the sm_100a (B200) implementation of
 * the block-sparse attention forward path of GueroudjiAmal/polyhedral.
 *
 * Every entry point:
 *   - takes plain device pointers, sizes and strides (no framework types);
 *   - is stream-ordered on `stream` (NULL = the legacy default stream) and does
 *     no host synchronisation;
 *   - returns PA_OK (0) or a negative PA_ERR_* code, with a message available
 *     from pa_last_error() on the calling thread; argument errors are detected
 *     before any launch;
 *   - is safe to call concurrently from several host threads on distinct streams.
 *
 * Reference interfaces replaced (paths inside the reference repository):
 *   pa_block_index / pa_block_index_dense  <- gpu/blockindex.py:32-51  build()
 *   pa_residue_perm                        <- gpu/permute.py:12-16     residue_perm()
 *   pa_invert_perm                         <- gpu/permute.py:27-31     invert()
 *   pa_permute_rows                        <- gpu/permute.py:22-24     apply_perm(), and the
 *                                             inverse index_select of gpu/test_correctness.py:77
 *   pa_attn_plan / pa_attn_fwd             <- gpu/triton_attn.py:185-241 block_sparse_attention()
 *                                             (kernel body :62-182)
 *   pa_lse_merge                           <- src/polyattn/experiments/compose.py:7-17,107-118
 *                                             (argued and costed there, never executed)
 */
#ifndef POLYATTN_H
#define POLYATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define PA_API __attribute__((visibility("default")))
#else
#define PA_API
#endif

typedef struct CUstream_st* pa_stream_t; /* same type as cudaStream_t */

enum {
  PA_OK = 0,
  PA_ERR_ARG = -1,          /* invalid argument; nothing was launched */
  PA_ERR_CUDA = -2,         /* a CUDA runtime/driver call failed */
  PA_ERR_UNSUPPORTED = -3,  /* valid request outside what the kernels implement */
  PA_ERR_DEVICE = -4        /* a kernel reported a failure (see pa_attn_status) */
};

/* Mask kinds.  Values 0-5 are the reference's (gpu/masks_gpu.py:9); the
 * predicate is on d = i - j in ORIGINAL coordinates (gpu/masks_gpu.py:37-53). */
enum {
  PA_CAUSAL = 0,         /* d >= 0 */
  PA_WINDOW = 1,         /* 0 <= d < p0 */
  PA_DILATED = 2,        /* d >= 0 && d % p0 == 0 */
  PA_LOCAL_STRIDED = 3,  /* d >= 0 && (d < p0 || d % p1 == 0) */
  PA_TWOBAND = 4,        /* d >= 0 && (d < p0 || (p1 <= d && d < p1 + p2)) */
  PA_SINKS = 5,          /* d >= 0 && (d < p0 || j < p1) */
  PA_FAR_STRIDED = 6     /* d >= p0 && d % p1 == 0   (lattice half of a disjoint split) */
};

enum { PA_BF16 = 0, PA_F16 = 1 };

typedef struct pa_pred {
  int32_t kind, p0, p1, p2;
} pa_pred;

/* Message of the last failed call on this host thread ("" if none). */
PA_API const char* pa_last_error(void);
/* ABI revision of this header (8); bumped on any incompatible change. */
PA_API int pa_abi_version(void);

/* ------------------------------------------------------------ block index
 * Replaces gpu/blockindex.py:32-51.  Classifies every BQ x A tile of the mask
 * seen by a kernel whose rows/columns are permuted by perm_q / perm_kv
 * (permuted position -> original index; NULL = identity), i.e. of M[perm_q][:, perm_kv].
 * Outputs, row i = query block i:
 *   kv_idx    [N/BQ, kv_stride] int32: ascending ids of tiles with any live element,
 *             zero-padded to kv_stride (kv_stride >= N/A);
 *   kv_num    [N/BQ] int32;
 *   kv_partial[N/BQ, kv_stride] int8: 1 unless every element of the tile is live;
 *   stats     int64[4]: {elements = tiles*BQ*A, live, max_kv, tiles}; zeroed by the call.
 * Requires N % BQ == 0, N % A == 0, 1 <= BQ, A and N < 2^24.  Bit-exact with the
 * reference on the first max_kv columns. */
PA_API int pa_block_index(const pa_pred* pred, int32_t N, int32_t BQ, int32_t A,
                   const int32_t* perm_q, const int32_t* perm_kv,
                   int32_t* kv_idx, int32_t kv_stride, int32_t* kv_num,
                   int8_t* kv_partial, int64_t* stats, pa_stream_t stream);

/* Same outputs from an explicit row-major N x N byte mask (nonzero = live) already
 * in the kernel's coordinates (the reference's _Dense adapter,
 * gpu/test_correctness.py:90-95). */
PA_API int pa_block_index_dense(const uint8_t* mask, int32_t N, int32_t BQ, int32_t A,
                         int32_t* kv_idx, int32_t kv_stride, int32_t* kv_num,
                         int8_t* kv_partial, int64_t* stats, pa_stream_t stream);

/* ------------------------------------------------------------ permutations
 * perm[p] = original index at permuted position p, positions ordered by
 * (i mod s, i div s) (gpu/permute.py:12-16).  Any N >= 1, s >= 1. */
PA_API int pa_residue_perm(int32_t N, int32_t s, int32_t* perm, pa_stream_t stream);
/* inv[perm[i]] = i (gpu/permute.py:27-31).  perm must be a permutation of [0, N). */
PA_API int pa_invert_perm(const int32_t* perm, int32_t N, int32_t* inv, pa_stream_t stream);

/* One tensor [BH, N, row_bytes] for pa_permute_rows; strides in BYTES. */
typedef struct pa_rows {
  const void* src;
  void* dst;
  int64_t src_bh_stride, src_row_stride;
  int64_t dst_bh_stride, dst_row_stride;
} pa_rows;

/* Row permutation of up to 4 tensors in one launch (gpu/permute.py:22-24 does one
 * index_select per tensor).  scatter == 0: dst[:, p] = src[:, perm[p]] (gather,
 * apply_perm); scatter == 1: dst[:, perm[p]] = src[:, p] (the inverse permutation
 * applied without forming invert(perm)).  Rows are copied bit for bit.  src and
 * dst must not overlap. */
PA_API int pa_permute_rows(const pa_rows* tensors, int32_t count, int32_t BH, int32_t N,
                    int32_t row_bytes, const int32_t* perm, int32_t scatter,
                    pa_stream_t stream);

/* ------------------------------------------------------------ attention
 * Block-sparse flash-attention forward (gpu/triton_attn.py:185-241): for each
 * query block, online-softmax attention over the listed KV tiles, the mask
 * predicate evaluated in original coordinates (perm_q[i] - perm_kv[j]) on partial
 * tiles only, fp32 accumulation, O = acc / l (0 for a row with no live key) and,
 * in addition to the reference, LSE = logsumexp of the live scaled scores
 * (natural log; -inf for a dead row).
 * Strides are in ELEMENTS; the last dimension must be contiguous. */
typedef struct pa_attn_args {
  const void* q;
  const void* k;
  const void* v;
  void* o;
  float* lse;                        /* [BH, N] (lse_bh_stride), or NULL */
  int32_t BH, N, D, dtype;           /* D in {64, 128}; dtype PA_BF16 or PA_F16 */
  int64_t q_bh_stride, q_row_stride;
  int64_t k_bh_stride, k_row_stride;
  int64_t v_bh_stride, v_row_stride;
  int64_t o_bh_stride, o_row_stride;
  int64_t lse_bh_stride;
  const int32_t* kv_idx;             /* block index, as pa_block_index writes it */
  const int32_t* kv_num;
  const int8_t* kv_partial;
  int32_t kv_stride;                 /* row stride of kv_idx / kv_partial */
  int32_t BQ, A;                     /* tile shape the block index was built at */
  const int32_t* perm_q;             /* permuted position -> original row; NULL = identity */
  const int32_t* perm_kv;            /* NULL = identity */
  const int32_t* o_row_map;          /* NULL: row r of O/LSE is written at r; else at
                                        o_row_map[r] (fuses the inverse permutation) */
  pa_pred pred;
  float scale;                       /* softmax scale; <= 0 means D^-0.5 */
  int32_t residue_stride;            /* 0: q/k/v are in kernel order (as the reference).
                                        s >= 1: q/k/v/o/lse are in ORIGINAL row order and the
                                        kernel works on the residue permutation by s
                                        (gpu/permute.py:12-16) without a copy: its row p
                                        reads original row (p mod N/s)*s + p div (N/s), the
                                        predicate uses those original coordinates, O/LSE
                                        rows go back to original order; perm_q, perm_kv and
                                        o_row_map must be NULL and N/s must be a multiple of
                                        128 and of A.  The block index is that of the
                                        permuted mask, as with physically permuted inputs. */
  int32_t merge;                     /* 0: write O and LSE.  1: O and LSE already hold the
                                        result of an attention over a mask disjoint from this
                                        one, on the same rows; the epilogue merges this one's
                                        result into them (log-sum-exp merge, as pa_lse_merge)
                                        instead of overwriting.  Needs lse != NULL.  No
                                        counterpart in the reference, which never executes
                                        the merge (src/polyattn/experiments/compose.py:7-17). */
  int32_t kv_rows;                   /* KV rows per super-tile of the forward: 0 or 128 (the
                                        default kernel), or 64 (S double-buffered in TMEM so
                                        the next S runs during the softmax, and each 128-row
                                        half computes only the tiles live for it; faster on
                                        bands narrower than a 256-row item, e.g. a window of
                                        64).  64 cannot be combined with merge. */
  /* The reference's class-B traffic emulation (gpu/triton_attn.py:99-128); all zero /
     one for the ordinary forward.  Same tiles, same predicate, same result: only the
     way K/V rows are fetched changes. */
  int32_t gather_kv;                 /* 1: k and v are in ORIGINAL order and row j of the
                                        kernel order is read from row perm_kv[j] (NULL =
                                        identity), per tile, by four-row TMA gathers. */
  int32_t gather_mult;               /* R in 1..16 (0 reads as 1): each K tile also reads
                                        (R-1) more sets of its A rows, which the result
                                        does not use (the reference weights them by 0). */
  int32_t gather_scatter;            /* extra rows of set r: 0 = row(j) + r*A (contiguous),
                                        1 = perm_kv[j + r*A] (scattered), both mod N.
                                        The gathered forward needs residue_stride = 0,
                                        merge = 0, kv_rows 0 or 128, k and v head strides
                                        that are multiples of their row strides, and a
                                        16-byte aligned perm_kv. */
  int32_t sched_heads;               /* heads per scheduling group of the forward's work
                                        items (items of one group run pair by pair, all
                                        its heads together, longest pair first; groups
                                        run one after another): 0 or >= BH = one group.
                                        Groups whose K/V fit in L2 cut DRAM re-reads when
                                        all heads' K/V do not. */
  int32_t row_threads;               /* softmax threads per query row of the forward: 1
                                        (one thread takes the row's 128 columns of a
                                        super-tile), 2 (two threads, 64 columns each, 16
                                        softmax warps; not with merge, kv_rows=64 or
                                        gathered K/V), or 0: the library chooses -- 2 when
                                        A <= 32 or D = 64 and the call allows it, else 1
                                        (what measured faster on B200). */
} pa_attn_args;

/* Bytes of device workspace pa_attn_plan / pa_attn_fwd need for these arguments
 * (depends on N, BQ, A, kv layout only). */
PA_API size_t pa_attn_workspace_size(const pa_attn_args* args);

/* Builds, in `workspace`, the per-256-row work list the forward kernel runs on
 * (union of the listed tiles of the two 128-row halves, with each half's
 * full/partial/dead status and the original column indices of every listed tile,
 * ordered longest first).  Depends only on the block index and perm_kv: it can be
 * built once and reused by every pa_attn_fwd with the same index and perm_kv. */
PA_API int pa_attn_plan(const pa_attn_args* args, void* workspace, size_t workspace_bytes,
                 pa_stream_t stream);

/* Runs the forward on a workspace prepared by pa_attn_plan.  A device-side
 * failure (a bounded barrier wait that ran out: every wait gives up after 1 s, and
 * the kernel then stops issuing work, drains its copies and MMAs and frees TMEM)
 * is recorded in the workspace, readable with pa_attn_status. */
PA_API int pa_attn_fwd(const pa_attn_args* args, void* workspace, size_t workspace_bytes,
                pa_stream_t stream);

/* Status of the most recent forward on `workspace`, synchronising `stream`: 0 when it
 * finished cleanly, else one of the device codes (1 = a wait on a Q tile ran out,
 * 2 = K/V ring, 3 = S, 4 = P, 5 = O, 6 = teardown drain, 7 = work-item ring), and the
 * call returns PA_ERR_DEVICE.  Each launch tags what it records with its own epoch, so
 * a failure of an earlier forward on the same workspace does not show in a later
 * clean one.  No counterpart in the reference, whose only failure handling is the
 * Triton launch retry (gpu/triton_attn.py:224-240). */
PA_API int pa_attn_status(const void* workspace, int32_t* status_host, pa_stream_t stream);

/* Test hook for the failure path above, no counterpart in the reference: runs
 * pa_attn_fwd with every bounded wait limited to wait_limit_ns (1 us .. 1 s; the MMA
 * issuer's waits on Q tiles to a quarter of it, so they run out first) and the first
 * work item of every CTA missing one Q tile (its load is never issued), so the MMA
 * issuer's wait on that tile runs out.  The kernel records code 1, stops, drains and
 * frees TMEM; pa_attn_status then reports it.  Outputs are unspecified.  Not for
 * gathered K/V (gather_kv / gather_mult). */
PA_API int pa_attn_fwd_withheld(const pa_attn_args* args, void* workspace,
                                size_t workspace_bytes, int64_t wait_limit_ns,
                                pa_stream_t stream);

/* pa_attn_plan + pa_attn_fwd without a caller workspace.  No counterpart in the
 * reference: it exists for callers that may not allocate device memory (a host
 * embedding that only hands over tensors it already owns, a process working
 * inside a fixed memory budget or another framework's pool).  The work list goes
 * to a 4 MiB array compiled into the library, which every GPU that loads the
 * library holds until exit; a request whose work list would not fit (see
 * pa_attn_workspace_size; about N <= 36096 at A = 16, 51200 at A = 32) is rejected
 * with PA_ERR_ARG.
 * The first call on a device (and the first in a new CUDA context of it, e.g. after
 * a device reset) looks up that array's device address; make that first call before
 * any stream capture.  All calls share the array and each rebuilds what it reads;
 * calls that overlap on the GPU race on it and must be ordered by the caller.  Calls
 * no cudaMalloc, cudaFree or other allocating routine. */
PA_API int pa_attn_fwd_noalloc(const pa_attn_args* args, pa_stream_t stream);

/* Status of the most recent pa_attn_fwd_noalloc on the current device (as
 * pa_attn_status for a caller workspace: 0, or a device code and PA_ERR_DEVICE),
 * read from the library's array, synchronising `stream`.  No counterpart in the
 * reference.  Allocates nothing. */
PA_API int pa_attn_noalloc_status(int32_t* status_host, pa_stream_t stream);

/* ------------------------------------------------------------ LSE merge
 * Attention over a disjoint union M = P1 + P2 from the attentions over P1 and P2
 * (src/polyattn/experiments/compose.py:7-17): per row, m = max(l1, l2),
 * w_i = exp(l_i - m), O = (w1 O1 + w2 O2) / (w1 + w2), LSE = m + log(w1 + w2);
 * a row dead in both parts gives O = 0, LSE = -inf.  Part 2's row r is read
 * from row row_map2[r] of o2/lse2 when row_map2 is non-NULL (part 2 computed on
 * permuted rows: row_map2 = invert(perm)).  o may alias o1 and lse may alias lse1.
 * Strides in elements; lse arrays are [BH, N] with row stride 1. */
typedef struct pa_merge_args {
  const void* o1;
  const float* lse1;
  const void* o2;
  const float* lse2;
  void* o;
  float* lse;
  int32_t BH, N, D, dtype;
  int64_t o1_bh_stride, o1_row_stride;
  int64_t o2_bh_stride, o2_row_stride;
  int64_t o_bh_stride, o_row_stride;
  int64_t lse1_bh_stride, lse2_bh_stride, lse_bh_stride;
  const int32_t* row_map2;
} pa_merge_args;

PA_API int pa_lse_merge(const pa_merge_args* args, pa_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* POLYATTN_H */
