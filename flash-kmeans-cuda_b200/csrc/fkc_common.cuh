// Device helpers shared by several kernels: element conversions and the
// 32-byte norm-extension rows read by the tcgen05 assignment kernel.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>

namespace fkc {

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) {
  return __half2float(v);
}
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) {
  return __float2half_rn(v);
}
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

constexpr int kNormExtBytes = 32;  // 8 tf32 (fp32 bit patterns) per row

// x rounded to tf32 (the top 19 bits of an fp32: 10 stored mantissa bits),
// to nearest with ties away from zero; returned as an fp32 whose low 13 bits
// are zero, so the tensor cores read it exactly.
__device__ __forceinline__ float round_tf32(float x) {
  return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
}

// v = t1 + t2 + t3 (+ < 2^-33 |v|), each term a tf32 value.
__device__ __forceinline__ void split3_tf32(float v, float& t1, float& t2, float& t3) {
  t1 = round_tf32(v);
  const float r1 = v - t1;  // exact: t1 is v with its low bits rounded
  t2 = round_tf32(r1);
  t3 = round_tf32(r1 - t2);
}

// The norm slice of the tensor-core assignment: one K = 8 tf32 MMA per item
// adds <row_ext, centroid_ext> to x.c, with
//   row side (x):      {t1, t2, t3, 1, 1, 1, -delta, 0}
//   centroid side (c): {1, 1, 1, t1, t2, t3, 1,      0}
// so that the sum is value(row) + value(centroid) - delta(row), value =
// -||.||^2 / 2 and delta = 2^-12 ||x||^2 + 2^-100 a row-constant bias (it does
// not change a row's argmin) that keeps every score -dist/2 - delta strictly
// negative, far above the fp32 rounding of the accumulation.
__device__ __forceinline__ void write_norm_ext(void* dst, float value, bool row_side) {
  float t1, t2, t3;
  split3_tf32(value, t1, t2, t3);
  float4 lo, hi;
  if (row_side) {
    const float delta = fmaf(-value, 0x1p-11f, 0x1p-100f);
    lo = make_float4(t1, t2, t3, 1.f);
    hi = make_float4(1.f, 1.f, round_tf32(-delta), 0.f);
  } else {
    lo = make_float4(1.f, 1.f, 1.f, t1);
    hi = make_float4(t2, t3, 1.f, 0.f);
  }
  float4* d = reinterpret_cast<float4*>(dst);
  d[0] = lo;
  d[1] = hi;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

}  // namespace fkc
