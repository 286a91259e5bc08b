// Shared device helpers for the sm_100a kernels: mbarriers with bounded waits,
// TMA tile loads, tcgen05 (TMEM alloc / MMA / ld / st) wrappers, and the mask
// predicate evaluated in original coordinates.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include "polyattn.h"

#define PA_DEV __device__ __forceinline__

namespace pa {

// Device-side failure codes written to the workspace error word.
enum : int32_t {
  DEV_OK = 0,
  DEV_TIMEOUT_Q = 1,        // a wait on the Q-tile barrier ran out
  DEV_TIMEOUT_KV = 2,       // a wait on a K/V ring slot ran out
  DEV_TIMEOUT_S = 3,        // softmax waited too long for S
  DEV_TIMEOUT_P = 4,        // MMA waited too long for P
  DEV_TIMEOUT_O = 5,        // epilogue waited too long for O
  DEV_TIMEOUT_DRAIN = 6,    // teardown could not drain outstanding copies
  DEV_TIMEOUT_ITEM = 7,     // a wait on the work-item ring ran out
};

// A wait gives up after this many nanoseconds of %globaltimer.  One kernel step
// of this library never waits more than microseconds on a barrier; the limit
// only matters when something is wrong, and then it turns a hang into an error
// status the host can read.
constexpr uint64_t kWaitLimitNs = 1000ull * 1000ull * 1000ull;  // 1 s

PA_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

PA_DEV uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ----------------------------------------------------------------- mbarrier
PA_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
PA_DEV void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
PA_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
PA_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
               ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
PA_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return ok != 0;
}
// Where a kernel launch reports a failure: a status word in global memory, tagged
// with the launch's epoch (bits 8-31) above the failure code (bits 0-7), so that a
// word left by an earlier launch on the same workspace reads as stale, not as this
// launch's status.  Also carries the launch's wait limit.
struct ErrSink {
  int32_t* word;
  uint32_t epoch;      // 24-bit launch epoch
  uint64_t limit_ns;   // bounded waits give up after this long
  // Records `code` for this launch.  A wait that gives up raises the CTA's abort
  // flag, so the CTA's other waits stop without recording: the word holds the
  // failure of whichever CTA recorded last, a word of an earlier launch is replaced.
  PA_DEV void record(int32_t code) const {
    if (word) atomicExch(word, (int32_t)((epoch << 8) | ((uint32_t)code & 0xffu)));
  }
};

// Wait for the phase of `bar` with parity `parity` to complete.  Gives up after
// err.limit_ns, or as soon as another thread of the CTA has raised `*abort`;
// on its own timeout it raises `*abort` and records `code` through `err`.
// Returns false when it gave up.  try_wait itself blocks in hardware for a
// system-defined time before returning false; a suspend-time hint (measured)
// made the attention kernel about 1.5 % slower, so none is given.
PA_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                      const ErrSink& err, int32_t code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (globaltimer() - t0 > err.limit_ns) {
      *abort = 1;
      err.record(code);
      return false;
    }
  }
}

// ------------------------------------------------------------------ TMA
// 3-D tiled load (no multicast): box lands at `dst` (shared), completion is
// reported as transaction bytes on `bar`.  c0 must be a multiple of 8 elements
// (16 bytes) for 16-bit data; callers pass 0 or 64.
PA_DEV void tma_load_3d(void* dst, const void* tmap, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];"
      ::"r"(smem_u32(dst)), "l"(tmap), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
// 4-D tiled load (no multicast), for the residue-strided view (D, s, N/s, BH).
PA_DEV void tma_load_4d(void* dst, const void* tmap, uint64_t* bar, int c0, int c1, int c2,
                        int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];"
      ::"r"(smem_u32(dst)), "l"(tmap), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
// Four-row gather (tile::gather4, no multicast) through a 2-D map whose box is 64
// columns x 1 row: rows r0..r3 at column c0 land as four consecutive 128-byte rows
// at dst (swizzled by the map's mode, which follows the shared-memory address).
PA_DEV void tma_gather4(void* dst, const void* tmap, uint64_t* bar, int c0, int r0, int r1,
                        int r2, int r3) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];"
      ::"r"(smem_u32(dst)), "l"(tmap), "r"(smem_u32(bar)), "r"(c0), "r"(r0), "r"(r1), "r"(r2),
        "r"(r3)
      : "memory");
}
// Tiled stores shared -> global (no multicast), completion tracked as a bulk group of
// the issuing thread; the box is read from `src` (shared) laid out as the map's swizzle
// says.  Never at a negative coordinate; c0 a multiple of 8 elements (16 bytes).
PA_DEV void tma_store_3d(const void* tmap, const void* src, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];"
      ::"l"(tmap), "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2) : "memory");
}
PA_DEV void tma_store_4d(const void* tmap, const void* src, int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];"
      ::"l"(tmap), "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3) : "memory");
}
PA_DEV void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Until every bulk group this thread committed has finished reading shared memory.
PA_DEV void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Until every bulk group this thread committed has completed (written global memory).
PA_DEV void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Orders this thread's ordinary shared-memory writes before later async-proxy (TMA)
// accesses of them.
PA_DEV void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
PA_DEV void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// ------------------------------------------------------------------ tcgen05
PA_DEV void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
               ::"r"(smem_u32(dst_smem)), "r"(ncols) : "memory");
}
PA_DEV void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
PA_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
               ::"r"(taddr), "r"(ncols) : "memory");
}
PA_DEV void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
PA_DEV void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Arrive once on `bar` when every tcgen05 op this thread issued so far is done.
PA_DEV void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
      ::"r"(smem_u32(bar)) : "memory");
}
// D[tmem] (+)= A[smem] * B[smem]
PA_DEV void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                   uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem]
PA_DEV void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                   uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}

// 32 consecutive 32-bit TMEM columns of this thread's lane.
PA_DEV void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32"
      " {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
        "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
        "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]),
        "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
PA_DEV void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0],"
      " {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]),
        "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]),
        "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
        "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
        "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]),
        "r"(r[30]), "r"(r[31])
      : "memory");
}
PA_DEV void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0],"
      " {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]),
        "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]),
        "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
// The .16x32bx2 shape: the warp reads 16 TMEM lanes starting at taddr's lane, twice --
// lanes 0-15 get lane (base + t) at columns [col, col + 32), lanes 16-31 get lane
// (base + t - 16) at columns [col + SPLIT, col + SPLIT + 32).  Two threads of a warp
// thereby share one TMEM lane (one query row), each with its own column range.
template <int SPLIT>
PA_DEV void tmem_ld32_pair(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.16x32bx2.x32.b32"
      " {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32], %33;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
        "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
        "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]),
        "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr), "n"(SPLIT));
}
template <int SPLIT>
PA_DEV void tmem_st32_pair(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.16x32bx2.x32.b32 [%0], %33,"
      " {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]),
        "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]),
        "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
        "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
        "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]),
        "r"(r[30]), "r"(r[31]), "n"(SPLIT)
      : "memory");
}
template <int SPLIT>
PA_DEV void tmem_st16_pair(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.16x32bx2.x16.b32 [%0], %17,"
      " {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]),
        "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]),
        "r"(r[13]), "r"(r[14]), "r"(r[15]), "n"(SPLIT)
      : "memory");
}
PA_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// Ties registers written by tcgen05.ld to a point after tcgen05.wait::ld, so the
// compiler cannot schedule their first use between the load and the wait.
PA_DEV void tmem_regs_ready(uint32_t (&r)[32]) {
#pragma unroll
  for (int i = 0; i < 32; i += 8)
    asm volatile("" : "+r"(r[i]), "+r"(r[i + 1]), "+r"(r[i + 2]), "+r"(r[i + 3]),
                      "+r"(r[i + 4]), "+r"(r[i + 5]), "+r"(r[i + 6]), "+r"(r[i + 7]));
}
PA_DEV void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor, 128-byte swizzle, sm_100 format (version 1).
//   K-major operand: rows of 64 16-bit elements (128 B), 8-row groups 1024 B apart.
//   MN-major operand: `lbo` = bytes between 64-element chunks of the MN axis,
//   8-row groups of the K axis 1024 B apart.
PA_DEV uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((1024u >> 4) & 0x3FFF) << 32;   // SBO: 8 rows x 128 B
  d |= (uint64_t)1 << 46;                           // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                           // SWIZZLE_128B
  return d;
}

// Instruction descriptor for kind::f16 with fp32 accumulation.
//   ab_fmt: 0 = f16, 1 = bf16 (A and B always the same type).
__host__ __device__ constexpr uint32_t make_idesc_f16(uint32_t ab_fmt, uint32_t M, uint32_t N,
                                                      uint32_t a_mn_major, uint32_t b_mn_major) {
  return (1u << 4)                 // D format: f32
       | (ab_fmt << 7)             // A format
       | (ab_fmt << 10)            // B format
       | (a_mn_major << 15)
       | (b_mn_major << 16)
       | ((N >> 3) << 17)
       | ((M >> 4) << 24);
}

// ------------------------------------------------------------------ predicate
struct Pred {
  int kind, p0, p1, p2;
  float inv_mod;   // 1 / (lattice modulus), 0 when the kind has none
  int mod;         // lattice modulus (DILATED: p0; LOCAL_STRIDED / FAR_STRIDED: p1)
};

// Validates a predicate and precomputes its lattice modulus (host side).
int make_pred(const pa_pred* p, Pred* out, const char* who);

// d % m == 0 for 0 <= d < 2^24: round(d/m) times m equals d exactly when m | d.
PA_DEV bool divisible(int d, int m, float inv_m) {
  const int q = __float2int_rn(__int2float_rn(d) * inv_m);
  return q * m == d;
}

// mask[i, j] in original coordinates.  Mirrors the reference's mask_mod
// (gpu/masks_gpu.py:37-53) plus FAR_STRIDED (d >= p0 and d % p1 == 0).
PA_DEV bool pred_live(const Pred& p, int i, int j) {
  const int d = i - j;
  if (d < 0) return false;
  switch (p.kind) {
    case PA_CAUSAL: return true;
    case PA_WINDOW: return d < p.p0;
    case PA_DILATED: return divisible(d, p.mod, p.inv_mod);
    case PA_LOCAL_STRIDED: return d < p.p0 || divisible(d, p.mod, p.inv_mod);
    case PA_TWOBAND: return d < p.p0 || (d >= p.p1 && d < p.p1 + p.p2);
    case PA_SINKS: return d < p.p0 || j < p.p1;
    case PA_FAR_STRIDED: return d >= p.p0 && divisible(d, p.mod, p.inv_mod);
    default: return false;
  }
}

// ------------------------------------------------------------------ live bits
// floor(a / b) for b > 0
__device__ __forceinline__ int floordiv(int a, int b) {
  return a >= 0 ? a / b : -((-a + b - 1) / b);
}

// Bits (c - base) for c in [lo, hi], clipped to the word [base, base + 32).
__device__ __forceinline__ uint32_t range_bits(int lo, int hi, int base) {
  lo = max(lo - base, 0);
  hi = min(hi - base, 31);
  if (hi < lo) return 0u;
  const uint32_t upto = hi == 31 ? 0xffffffffu : ((2u << hi) - 1u);
  return upto & ~((1u << lo) - 1u);
}

// Live bits of columns [base, base + 32) of a segment of `len` columns whose
// original indices form the progression j0 + c*dj (dj >= 1), for the row with
// original index i = j0 + e.  With d = e - c*dj decreasing in c, every kind is a
// union of at most two ranges of c, and a lattice term (d % m == 0) is constant
// over the segment when m divides dj, and every m-th column when dj = 1 and m is a
// power of two.  Returns false otherwise (the caller then evaluates element by
// element).
__device__ __forceinline__ bool progression_bits(const Pred& p, int e, int j0, int dj, int sh,
                                                 int base, int len, uint32_t& out) {
  // floor(a / dj): an arithmetic shift when dj is a power of two (sh >= 0)
  auto fdiv = [&](int a) { return sh >= 0 ? (a >> sh) : floordiv(a, dj); };
  const int cz = fdiv(e);                               // d >= 0  <=>  c <= cz
  int lo1 = 0, hi1 = -1, lo2 = 0, hi2 = -1;
  bool lattice = false;
  if (p.mod > 0) {
    if (!divisible(dj, p.mod, p.inv_mod)) {
      // Unit column step (no permutation) and a power-of-two modulus: the lattice
      // columns are every mod-th one, a shifted periodic pattern.
      if (dj != 1 || p.mod > 32 || (p.mod & (p.mod - 1))) return false;
      const uint32_t pat = p.mod == 2 ? 0x55555555u : p.mod == 4 ? 0x11111111u
                           : p.mod == 8 ? 0x01010101u : p.mod == 16 ? 0x00010001u : 1u;
      const uint32_t lat = e >= 0 ? pat << ((e - base) & (p.mod - 1)) : 0u;
      int hi = cz;
      uint32_t near = 0u;
      switch (p.kind) {
        case PA_DILATED:
          break;
        case PA_FAR_STRIDED:
          hi = min(cz, fdiv(e - p.p0));
          break;
        case PA_LOCAL_STRIDED:
          near = range_bits(fdiv(e - p.p0) + 1, min(cz, len - 1), base);
          break;
        default:
          return false;
      }
      out = (range_bits(0, min(hi, len - 1), base) & lat) | near;
      return true;
    }
    lattice = e >= 0 && divisible(e, p.mod, p.inv_mod);   // only e >= 0 can reach c <= cz
  }
  switch (p.kind) {
    case PA_CAUSAL:
      hi1 = cz;
      break;
    case PA_WINDOW:                                     // d < p0 <=> c > (e - p0) / dj
      lo1 = fdiv(e - p.p0) + 1;
      hi1 = cz;
      break;
    case PA_DILATED:
      hi1 = lattice ? cz : -1;
      break;
    case PA_LOCAL_STRIDED:
      lo1 = fdiv(e - p.p0) + 1;
      hi1 = cz;
      hi2 = lattice ? cz : -1;
      break;
    case PA_TWOBAND:
      lo1 = fdiv(e - p.p0) + 1;
      hi1 = cz;
      lo2 = fdiv(e - p.p1 - p.p2) + 1;
      hi2 = min(cz, fdiv(e - p.p1));
      break;
    case PA_SINKS:                                      // kv < p1 <=> c <= (p1 - j0 - 1) / dj
      lo1 = fdiv(e - p.p0) + 1;
      hi1 = cz;
      hi2 = min(cz, fdiv(p.p1 - j0 - 1));
      break;
    case PA_FAR_STRIDED:                                // d >= p0 <=> c <= (e - p0) / dj
      hi1 = lattice ? min(cz, fdiv(e - p.p0)) : -1;
      break;
    default:
      return false;
  }
  hi1 = min(hi1, len - 1);
  hi2 = min(hi2, len - 1);
  out = range_bits(lo1, hi1, base) | range_bits(lo2, hi2, base);
  return true;
}

// Live bits of `n` (<= 32) columns evaluated one by one; column c has original
// index cols[c] (global memory) when given, else j0 + (base + c) * dj.
__device__ __forceinline__ uint32_t element_bits(const Pred& p, int i, const int* cols, int j0,
                                                 int dj, int base, int n) {
  uint32_t w = 0;
#pragma unroll 1
  for (int c = 0; c < n; ++c) {
    const int j = cols ? __ldg(cols + c) : j0 + (base + c) * dj;
    w |= (uint32_t)pred_live(p, i, j) << c;
  }
  return w;
}

}  // namespace pa
