// Log-sum-exp merge of two attentions over disjoint masks into the attention
// over their union -- the combine src/polyattn/experiments/compose.py:7-17
// argues for (and costs at :107-118) but never executes.
//
// HBM-bound: each output row reads two O rows and two LSE values and writes one
// O row and one LSE.  A row is handled by D/8 threads, each moving 16 bytes
// (8 elements) per input, so a 256-thread CTA covers 16 rows at D = 128 per step of
// its grid-stride loop (8 CTAs per SM).
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

// One output row as one thread sees it: its 8-column share of O1 and O2 and the
// row's two LSE values (D / 8 <= 32 threads cover a row, one chunk each).
template <typename T>
struct RowIn {
  long long g;      // flattened (bh, row), or >= BH * N when past the end
  int bh, row;
  bool valid, r2_ok;
  float l1, l2;
  uint4 x1, x2;
};

template <typename T>
__device__ __forceinline__ void load_row(const pa_merge_args& a, long long g, long long total,
                                         int c, RowIn<T>& r) {
  r.g = g;
  r.valid = g < total && c < a.D;
  const bool in = g < total;
  r.bh = in ? (int)(g / a.N) : 0;
  r.row = in ? (int)(g - (long long)r.bh * a.N) : 0;
  const int r2 = !in ? -1 : (a.row_map2 ? a.row_map2[r.row] : r.row);
  r.r2_ok = (unsigned)r2 < (unsigned)a.N;
  r.l1 = in ? a.lse1[(long long)r.bh * a.lse1_bh_stride + r.row] : -INFINITY;
  r.l2 = r.r2_ok ? a.lse2[(long long)r.bh * a.lse2_bh_stride + r2] : -INFINITY;
  r.x1 = r.x2 = make_uint4(0u, 0u, 0u, 0u);
  if (r.valid) {
    const T* o1 = static_cast<const T*>(a.o1) + (long long)r.bh * a.o1_bh_stride +
                  (long long)r.row * a.o1_row_stride;
    r.x1 = *reinterpret_cast<const uint4*>(o1 + c);
    if (r.r2_ok) {
      const T* o2 = static_cast<const T*>(a.o2) + (long long)r.bh * a.o2_bh_stride +
                    (long long)r2 * a.o2_row_stride;
      r.x2 = *reinterpret_cast<const uint4*>(o2 + c);
    }
  }
}

// m = max(l1, l2); O = (e^(l1-m) O1 + e^(l2-m) O2) / (e^(l1-m) + e^(l2-m));
// LSE = m + log(e^(l1-m) + e^(l2-m)); both -inf -> O = 0, LSE = -inf.
template <typename T>
__device__ __forceinline__ float store_row(const pa_merge_args& a, int c, const RowIn<T>& r) {
  const float m = fmaxf(r.l1, r.l2);
  float w1 = 0.f, w2 = 0.f;
  if (m != -INFINITY) {
    w1 = expf(r.l1 - m);
    w2 = expf(r.l2 - m);
  }
  const float den = w1 + w2;
  const float inv = den > 0.f ? 1.f / den : 0.f;
  w1 *= inv;
  w2 *= inv;
  if (r.valid) {
    float x1[8], x2[8], y[8];
    Vec8<T>::to_float(r.x1, x1);
    Vec8<T>::to_float(r.x2, x2);
#pragma unroll
    for (int i = 0; i < 8; ++i) y[i] = w1 * x1[i] + w2 * x2[i];
    T* o = static_cast<T*>(a.o) + (long long)r.bh * a.o_bh_stride + (long long)r.row * a.o_row_stride;
    *reinterpret_cast<uint4*>(o + c) = Vec8<T>::from_float(y);
  }
  return den > 0.f ? m + logf(den) : -INFINITY;
}

template <typename T>
__global__ void __launch_bounds__(256) lse_merge_kernel(pa_merge_args a, int tpr) {
  // Grid-stride over the flattened (bh, row) rows, two rows per thread per step
  // with all of both rows' loads issued before any arithmetic, so that each thread
  // keeps four 16-byte loads in flight.  Every thread runs the same number of steps
  // (the warp-level sync stays uniform); rows past the end are masked.
  const int rows_per_cta = 256 / tpr;
  const int part = threadIdx.x % tpr;
  const int c = part * 8;
  const long long total = (long long)a.BH * a.N;
  const long long step = (long long)gridDim.x * rows_per_cta * 2;
  for (long long base = (long long)blockIdx.x * rows_per_cta * 2; base < total; base += step) {
    const long long g0 = base + threadIdx.x / tpr;
    RowIn<T> r0, r1;
    load_row<T>(a, g0, total, c, r0);
    load_row<T>(a, g0 + rows_per_cta, total, c, r1);
    const float lse0 = store_row<T>(a, c, r0);
    const float lse1 = store_row<T>(a, c, r1);
    __syncwarp();   // every lane of these rows has read lse1 before it may be overwritten
    if (part == 0) {
      if (r0.g < total) a.lse[(long long)r0.bh * a.lse_bh_stride + r0.row] = lse0;
      if (r1.g < total) a.lse[(long long)r1.bh * a.lse_bh_stride + r1.row] = lse1;
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
  int tpr = a->D / 8;
  if (tpr > 32) tpr = 32;
  while (256 % tpr) --tpr;
  const int rows_per_cta = 256 / tpr;
  int dev = 0, sms = 148;
  PA_CUDA(cudaGetDevice(&dev), "pa_lse_merge");
  PA_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "pa_lse_merge");
  const long long steps = ((long long)a->BH * a->N + 2 * rows_per_cta - 1) / (2 * rows_per_cta);
  const int grid = (int)(steps < 8LL * sms ? steps : 8LL * sms);
  if (a->dtype == PA_BF16)
    lse_merge_kernel<__nv_bfloat16><<<grid, 256, 0, (cudaStream_t)stream>>>(*a, tpr);
  else
    lse_merge_kernel<__half><<<grid, 256, 0, (cudaStream_t)stream>>>(*a, tpr);
  return check_launch("pa_lse_merge");
}
