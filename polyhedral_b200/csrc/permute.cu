// Class A re-indexing on the device: the residue permutation, its inverse, and
// the row permutation of [BH, N, row] tensors (gpu/permute.py:12-31).
//
// The row copy is HBM-bound.  Each CTA copies a band of 64 rows of one tensor /
// head; a row is split into 16-byte vectors (8-byte or 4-byte when the row
// size or alignment does not allow 16), and every thread issues all its loads
// for four rows before the matching stores, so a warp keeps several 512-byte
// requests in flight.  Up to four tensors (Q, K, V, ...) share one launch.
#include "common.cuh"
#include "capi_util.h"

namespace pa {
namespace {

constexpr int kRowsPerCta = 64;
constexpr int kRowUnroll = 4;

struct RowsDesc {
  const char* src;
  char* dst;
  long long sbh, srow, dbh, drow;
};
struct RowsBatch {
  RowsDesc t[4];
};

__global__ void residue_perm_kernel(int N, int s, int32_t* __restrict__ perm) {
  const int p = blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= N) return;
  // class r holds r, r+s, r+2s, ...: the first N % s classes have N/s + 1 members
  const int q = N / s, rem = N % s;
  const int big = rem * (q + 1);
  int r, t;
  if (p < big) {
    r = p / (q + 1);
    t = p - r * (q + 1);
  } else {
    const int pp = p - big;
    r = rem + pp / q;
    t = pp - (r - rem) * q;
  }
  perm[p] = r + t * s;
}

__global__ void invert_perm_kernel(const int32_t* __restrict__ perm, int N,
                                   int32_t* __restrict__ inv) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= N) return;
  const int p = perm[i];
  if ((unsigned)p < (unsigned)N) inv[p] = i;
}

template <typename V>
__global__ void __launch_bounds__(256)
permute_rows_kernel(RowsBatch b, int N, int chunks, const int32_t* __restrict__ perm,
                    int scatter) {
  const RowsDesc d = b.t[blockIdx.z];
  const int bh = blockIdx.y;
  const char* __restrict__ src = d.src + (long long)bh * d.sbh;
  char* __restrict__ dst = d.dst + (long long)bh * d.dbh;
  const int row0 = blockIdx.x * kRowsPerCta;
  const int rows = min(kRowsPerCta, N - row0);
  const int ty = threadIdx.y, ny = blockDim.y;
  for (int base = ty; base < rows; base += ny * kRowUnroll) {
    const V* s[kRowUnroll];
    V* o[kRowUnroll];
    bool ok[kRowUnroll];
#pragma unroll
    for (int u = 0; u < kRowUnroll; ++u) {
      const int r = base + u * ny;
      ok[u] = r < rows;
      const int p = row0 + (ok[u] ? r : 0);
      int q = __ldg(perm + p);
      if ((unsigned)q >= (unsigned)N) {   // not a permutation entry: skip the row
        ok[u] = false;
        q = p;
      }
      const int sr = scatter ? p : q;
      const int dr = scatter ? q : p;
      s[u] = reinterpret_cast<const V*>(src + (long long)sr * d.srow);
      o[u] = reinterpret_cast<V*>(dst + (long long)dr * d.drow);
    }
    for (int c = threadIdx.x; c < chunks; c += blockDim.x) {
      V v[kRowUnroll];
#pragma unroll
      for (int u = 0; u < kRowUnroll; ++u)
        if (ok[u]) v[u] = __ldg(s[u] + c);
#pragma unroll
      for (int u = 0; u < kRowUnroll; ++u)
        if (ok[u]) __stcs(o[u] + c, v[u]);
    }
  }
}

template <typename V>
int launch_rows(const RowsBatch& b, int count, int BH, int N, int row_bytes,
                const int32_t* perm, int scatter, cudaStream_t stream) {
  const int chunks = row_bytes / (int)sizeof(V);
  const int bx = chunks >= 32 ? 32 : chunks;
  const int by = 256 / bx;
  dim3 grid((N + kRowsPerCta - 1) / kRowsPerCta, BH, count);
  permute_rows_kernel<V><<<grid, dim3(bx, by), 0, stream>>>(b, N, chunks, perm, scatter);
  return check_launch("pa_permute_rows");
}

}  // namespace
}  // namespace pa

extern "C" int pa_residue_perm(int32_t N, int32_t s, int32_t* perm, pa_stream_t stream) {
  PA_CHECK_ARG(N >= 1 && s >= 1 && perm, "pa_residue_perm: need N >= 1, s >= 1, perm");
  pa::residue_perm_kernel<<<(N + 255) / 256, 256, 0, (cudaStream_t)stream>>>(N, s, perm);
  return pa::check_launch("pa_residue_perm");
}

extern "C" int pa_invert_perm(const int32_t* perm, int32_t N, int32_t* inv, pa_stream_t stream) {
  PA_CHECK_ARG(N >= 1 && perm && inv, "pa_invert_perm: need N >= 1, perm, inv");
  pa::invert_perm_kernel<<<(N + 255) / 256, 256, 0, (cudaStream_t)stream>>>(perm, N, inv);
  return pa::check_launch("pa_invert_perm");
}

extern "C" int pa_permute_rows(const pa_rows* tensors, int32_t count, int32_t BH, int32_t N,
                               int32_t row_bytes, const int32_t* perm, int32_t scatter,
                               pa_stream_t stream) {
  using namespace pa;
  PA_CHECK_ARG(tensors && perm, "pa_permute_rows: null tensors or perm");
  PA_CHECK_ARG(count >= 1 && count <= 4, "pa_permute_rows: count=%d not in [1, 4]", count);
  PA_CHECK_ARG(BH >= 1 && BH <= 65535 && N >= 1 && row_bytes >= 1,
               "pa_permute_rows: bad BH=%d N=%d row_bytes=%d", BH, N, row_bytes);
  RowsBatch b{};
  int align = 16;
  for (int i = 0; i < count; ++i) {
    const pa_rows& t = tensors[i];
    PA_CHECK_ARG(t.src && t.dst, "pa_permute_rows: tensor %d has a null pointer", i);
    b.t[i] = RowsDesc{static_cast<const char*>(t.src), static_cast<char*>(t.dst),
                      t.src_bh_stride, t.src_row_stride, t.dst_bh_stride, t.dst_row_stride};
    const long long vals[] = {(long long)(uintptr_t)t.src, (long long)(uintptr_t)t.dst,
                              t.src_bh_stride, t.src_row_stride, t.dst_bh_stride,
                              t.dst_row_stride, row_bytes};
    for (long long v : vals) {
      while (align > 1 && (v % align) != 0) align >>= 1;
    }
  }
  const cudaStream_t s = (cudaStream_t)stream;
  switch (align) {
    case 16: return launch_rows<int4>(b, count, BH, N, row_bytes, perm, scatter, s);
    case 8: return launch_rows<int2>(b, count, BH, N, row_bytes, perm, scatter, s);
    case 4: return launch_rows<int>(b, count, BH, N, row_bytes, perm, scatter, s);
    case 2: return launch_rows<short>(b, count, BH, N, row_bytes, perm, scatter, s);
    default: return launch_rows<char>(b, count, BH, N, row_bytes, perm, scatter, s);
  }
}
