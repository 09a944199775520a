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

constexpr int kNormExtBytes = 32;  // 16 bf16 per row

// v = h1 + h2 + h3 (+ < 2^-24 |v|), each term a bf16.
__device__ __forceinline__ void split3_bf16(float v, uint32_t& h1, uint32_t& h2, uint32_t& h3) {
  const __nv_bfloat16 b1 = __float2bfloat16_rn(v);
  const float r1 = v - __bfloat162float(b1);
  const __nv_bfloat16 b2 = __float2bfloat16_rn(r1);
  const float r2 = r1 - __bfloat162float(b2);
  const __nv_bfloat16 b3 = __float2bfloat16_rn(r2);
  h1 = __bfloat16_as_ushort(b1);
  h2 = __bfloat16_as_ushort(b2);
  h3 = __bfloat16_as_ushort(b3);
}

// Row side (x):        {h1, h2, h3, 1, 1, 1, -delta, 0 x 9}
// Centroid side (c):   {1, 1, 1, h1, h2, h3, 1,      0 x 9}
// so that <row_ext, centroid_ext> = value(row) + value(centroid) - delta(row),
// with value = -||.||^2 / 2 and delta = 2^-12 ||x||^2 + 2^-100 a row-constant
// bias (it does not change a row's argmin) that keeps every score -dist/2 -
// delta strictly negative, far above the fp32 rounding of the accumulation.
__device__ __forceinline__ void write_norm_ext(void* dst, float value, bool row_side) {
  uint32_t h1, h2, h3;
  split3_bf16(value, h1, h2, h3);
  const uint32_t one = 0x3F80u;  // bf16 1.0
  uint4 lo;
  if (row_side) {
    const float delta = fmaf(-value, 0x1p-11f, 0x1p-100f);
    const uint32_t nd = __bfloat16_as_ushort(__float2bfloat16_rn(-delta));
    lo = make_uint4(h1 | (h2 << 16), h3 | (one << 16), one | (one << 16), nd);
  } else {
    lo = make_uint4(one | (one << 16), one | (h1 << 16), h2 | (h3 << 16), one);
  }
  uint4* d = reinterpret_cast<uint4*>(dst);
  d[0] = lo;
  d[1] = make_uint4(0u, 0u, 0u, 0u);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

}  // namespace fkc
