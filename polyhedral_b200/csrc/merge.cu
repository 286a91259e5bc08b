// Log-sum-exp merge of two attentions over disjoint masks into the attention
// over their union -- the combine src/polyattn/experiments/compose.py:7-17
// argues for (and costs at :107-118) but never executes.
//
// HBM-bound: each output row reads two O rows and two LSE values and writes one
// O row and one LSE.  A row is handled by D/16 threads, each moving 32 bytes
// (16 elements) per input; a 256-thread CTA takes 64 rows of one head per step of its
// grid-stride loop at D = 128, two per thread, all loads issued before any use.
#include <math.h>
#include "common.cuh"
#include "capi_util.h"

namespace pa {
namespace {

template <typename T>
struct Vec8;
template <>
struct Vec8<__nv_bfloat16> {
  static __device__ __forceinline__ void to_float(const uint4& u, float (&f)[8]) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 x = __bfloat1622float2(h[i]);
      f[2 * i] = x.x;
      f[2 * i + 1] = x.y;
    }
  }
  static __device__ __forceinline__ uint4 from_float(const float (&f)[8]) {
    uint4 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    return u;
  }
};
template <>
struct Vec8<__half> {
  static __device__ __forceinline__ void to_float(const uint4& u, float (&f)[8]) {
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 x = __half22float2(h[i]);
      f[2 * i] = x.x;
      f[2 * i + 1] = x.y;
    }
  }
  static __device__ __forceinline__ uint4 from_float(const float (&f)[8]) {
    uint4 u;
    __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
    return u;
  }
};

// m = max(l1, l2); O = (e^(l1-m) O1 + e^(l2-m) O2) / (e^(l1-m) + e^(l2-m));
// LSE = m + log(e^(l1-m) + e^(l2-m)); both -inf -> O = 0, LSE = -inf.  Returns the
// two weights folded into w1 / w2 and the merged LSE.
__device__ __forceinline__ float merge_weights(float l1, float l2, float& w1, float& w2) {
  const float m = fmaxf(l1, l2);
  w1 = 0.f;
  w2 = 0.f;
  if (m != -INFINITY) {
    w1 = expf(l1 - m);
    w2 = expf(l2 - m);
  }
  const float den = w1 + w2;
  const float inv = den > 0.f ? 1.f / den : 0.f;
  w1 *= inv;
  w2 *= inv;
  return den > 0.f ? m + logf(den) : -INFINITY;
}

constexpr int kThreads = 256;
constexpr int kRows = 2;   // rows per thread per chunk: all their loads are issued first
constexpr int kVecs = 2;   // 16-byte vectors per thread per row (16 columns)

// Grid-stride over chunks of kRows * (256 / tpr) consecutive rows of one (b, h): the
// chunk's head and first row come from one 64-bit division per chunk, its base
// pointers from one multiply.  Thread (slot, part) handles columns
// [16 part, 16 part + 16) of rows slot, slot + rpp, ...: every load of its kRows rows
// is in flight before the first use (kRows x 64 bytes of O plus the LSE values), and
// the per-row work (addresses, weights) is shared by 32 bytes of each input.
template <typename T>
__global__ void __launch_bounds__(kThreads, 3) lse_merge_kernel(pa_merge_args a, int tpr) {
  const int rpp = kThreads / tpr;               // rows per pass of the CTA
  const int part = threadIdx.x % tpr;
  const int slot = threadIdx.x / tpr;
  const int c = part * 8 * kVecs;
  const bool col_ok = c < a.D;
  const int chunk_rows = kRows * rpp;
  const long long cpb = (a.N + chunk_rows - 1) / chunk_rows;   // chunks per (b, h)
  const long long nchunks = cpb * a.BH;
  for (long long ch = blockIdx.x; ch < nchunks; ch += gridDim.x) {
    const int bh = (int)(ch / cpb);
    const int row0 = (int)(ch - (long long)bh * cpb) * chunk_rows;
    const T* o1b = static_cast<const T*>(a.o1) + (long long)bh * a.o1_bh_stride + c;
    const T* o2b = static_cast<const T*>(a.o2) + (long long)bh * a.o2_bh_stride + c;
    T* ob = static_cast<T*>(a.o) + (long long)bh * a.o_bh_stride + c;
    const float* l1b = a.lse1 + (long long)bh * a.lse1_bh_stride;
    const float* l2b = a.lse2 + (long long)bh * a.lse2_bh_stride;
    uint4 x1[kRows][kVecs], x2[kRows][kVecs];
    float l1[kRows], l2[kRows];
#pragma unroll
    for (int k = 0; k < kRows; ++k) {
      const int row = row0 + slot + k * rpp;
      const bool in = row < a.N;
      const int r2 = !in ? -1 : (a.row_map2 ? a.row_map2[row] : row);
      const bool r2_ok = (unsigned)r2 < (unsigned)a.N;
      l1[k] = in ? l1b[row] : -INFINITY;
      l2[k] = r2_ok ? l2b[r2] : -INFINITY;
#pragma unroll
      for (int v = 0; v < kVecs; ++v) x1[k][v] = x2[k][v] = make_uint4(0u, 0u, 0u, 0u);
      if (in && col_ok) {
        const uint4* p1 = reinterpret_cast<const uint4*>(o1b + (long long)row * a.o1_row_stride);
        const uint4* p2 = reinterpret_cast<const uint4*>(o2b + (long long)r2 * a.o2_row_stride);
#pragma unroll
        for (int v = 0; v < kVecs; ++v) {
          if (c + 8 * v < a.D) {            // D a multiple of 8, not always of 16
            x1[k][v] = p1[v];
            if (r2_ok) x2[k][v] = p2[v];
          }
        }
      }
    }
    float lse[kRows];
#pragma unroll
    for (int k = 0; k < kRows; ++k) {
      const int row = row0 + slot + k * rpp;
      float w1, w2;
      lse[k] = merge_weights(l1[k], l2[k], w1, w2);
      if (row < a.N && col_ok) {
        uint4* po = reinterpret_cast<uint4*>(ob + (long long)row * a.o_row_stride);
#pragma unroll
        for (int v = 0; v < kVecs; ++v) {
          if (c + 8 * v >= a.D) break;
          float f1[8], f2[8], y[8];
          Vec8<T>::to_float(x1[k][v], f1);
          Vec8<T>::to_float(x2[k][v], f2);
#pragma unroll
          for (int i = 0; i < 8; ++i) y[i] = w1 * f1[i] + w2 * f2[i];
          po[v] = Vec8<T>::from_float(y);
        }
      }
    }
    __syncwarp();   // every lane of these rows has read lse1 before it may be overwritten
    if (part == 0) {
#pragma unroll
      for (int k = 0; k < kRows; ++k) {
        const int row = row0 + slot + k * rpp;
        if (row < a.N) a.lse[(long long)bh * a.lse_bh_stride + row] = lse[k];
      }
    }
  }
}

}  // namespace
}  // namespace pa

extern "C" int pa_lse_merge(const pa_merge_args* a, pa_stream_t stream) {
  using namespace pa;
  PA_CHECK_ARG(a != nullptr, "pa_lse_merge: null args");
  PA_CHECK_ARG(a->o1 && a->o2 && a->o && a->lse1 && a->lse2 && a->lse,
               "pa_lse_merge: null pointer");
  PA_CHECK_ARG(a->BH >= 1 && a->BH <= 65535 && a->N >= 1, "pa_lse_merge: bad BH=%d N=%d",
               a->BH, a->N);
  PA_CHECK_ARG(a->D >= 8 && a->D % 8 == 0 && a->D <= 256,
               "pa_lse_merge: D=%d must be a multiple of 8 in [8, 256]", a->D);
  PA_CHECK_ARG(a->dtype == PA_BF16 || a->dtype == PA_F16, "pa_lse_merge: bad dtype %d",
               a->dtype);
  const long long strides[] = {a->o1_bh_stride, a->o1_row_stride, a->o2_bh_stride,
                               a->o2_row_stride, a->o_bh_stride, a->o_row_stride};
  for (long long s : strides)
    PA_CHECK_ARG(s % 8 == 0, "pa_lse_merge: O strides must be multiples of 8 elements");
  PA_CHECK_ARG(aligned(a->o1, 16) && aligned(a->o2, 16) && aligned(a->o, 16),
               "pa_lse_merge: O pointers must be 16-byte aligned");
  int tpr = (a->D + 8 * kVecs - 1) / (8 * kVecs);   // threads per row, 16 columns each
  if (tpr > 32) tpr = 32;
  while (kThreads % tpr) ++tpr;                      // a power of two <= 32
  const long long chunk_rows = (long long)kRows * (kThreads / tpr);
  const long long nchunks = (a->N + chunk_rows - 1) / chunk_rows * a->BH;
  int dev = 0, sms = 148, per_sm = 4;
  PA_CUDA(cudaGetDevice(&dev), "pa_lse_merge");
  PA_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "pa_lse_merge");
  PA_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(
              &per_sm, a->dtype == PA_BF16 ? lse_merge_kernel<__nv_bfloat16> : lse_merge_kernel<__half>,
              kThreads, 0), "pa_lse_merge");
  // as many CTAs as are resident at once (grid-stride beyond that), no tail wave
  const long long resident = (long long)sms * (per_sm > 0 ? per_sm : 1);
  const int grid = (int)(nchunks < resident ? nchunks : resident);
  if (a->dtype == PA_BF16)
    lse_merge_kernel<__nv_bfloat16><<<grid, kThreads, 0, (cudaStream_t)stream>>>(*a, tpr);
  else
    lse_merge_kernel<__half><<<grid, kThreads, 0, (cudaStream_t)stream>>>(*a, tpr);
  return check_launch("pa_lse_merge");
}
