// Log-sum-exp merge of two attentions over disjoint masks into the attention
// over their union -- the combine src/polyattn/experiments/compose.py:7-17
// argues for (and costs at :107-118) but never executes.
//
// HBM-bound: each output row reads two O rows and two LSE values and writes one
// O row and one LSE.  A row is handled by D/8 threads, each moving 16 bytes
// (8 elements) per input, so a 256-thread CTA covers 16 rows at D = 128.
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

template <typename T>
__global__ void __launch_bounds__(256) lse_merge_kernel(pa_merge_args a, int tpr) {
  const int rows_per_cta = 256 / tpr;
  const int row = blockIdx.x * rows_per_cta + threadIdx.x / tpr;
  const int part = threadIdx.x % tpr;
  const int bh = blockIdx.y;
  const bool valid = row < a.N;
  const int r2 = !valid ? -1 : (a.row_map2 ? a.row_map2[row] : row);
  const bool r2_ok = (unsigned)r2 < (unsigned)a.N;
  const float l1 = valid ? a.lse1[(long long)bh * a.lse1_bh_stride + row] : -INFINITY;
  const float l2 = r2_ok ? a.lse2[(long long)bh * a.lse2_bh_stride + r2] : -INFINITY;
  const float m = fmaxf(l1, l2);
  float w1 = 0.f, w2 = 0.f;
  if (m != -INFINITY) {
    w1 = expf(l1 - m);
    w2 = expf(l2 - m);
  }
  const float den = w1 + w2;
  const float inv = den > 0.f ? 1.f / den : 0.f;
  w1 *= inv;
  w2 *= inv;

  const T* o1 = static_cast<const T*>(a.o1) + (long long)bh * a.o1_bh_stride + (long long)row * a.o1_row_stride;
  const T* o2 = static_cast<const T*>(a.o2) + (long long)bh * a.o2_bh_stride + (long long)(r2_ok ? r2 : 0) * a.o2_row_stride;
  T* o = static_cast<T*>(a.o) + (long long)bh * a.o_bh_stride + (long long)row * a.o_row_stride;
  for (int c = part * 8; valid && c < a.D; c += tpr * 8) {
    float x1[8], x2[8], y[8];
    Vec8<T>::to_float(*reinterpret_cast<const uint4*>(o1 + c), x1);
    if (r2_ok) {
      Vec8<T>::to_float(*reinterpret_cast<const uint4*>(o2 + c), x2);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) x2[i] = 0.f;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) y[i] = w1 * x1[i] + w2 * x2[i];
    *reinterpret_cast<uint4*>(o + c) = Vec8<T>::from_float(y);
  }
  __syncwarp();   // every lane of this row has read lse1 before it may be overwritten
  if (valid && part == 0)
    a.lse[(long long)bh * a.lse_bh_stride + row] = den > 0.f ? m + logf(den) : -INFINITY;
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
  dim3 grid((a->N + rows_per_cta - 1) / rows_per_cta, a->BH);
  if (a->dtype == PA_BF16)
    lse_merge_kernel<__nv_bfloat16><<<grid, 256, 0, (cudaStream_t)stream>>>(*a, tpr);
  else
    lse_merge_kernel<__half><<<grid, 256, 0, (cudaStream_t)stream>>>(*a, tpr);
  return check_launch("pa_lse_merge");
}
