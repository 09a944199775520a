// Norm-extension rows read by the tcgen05 assignment kernel (one extra K=8
// slice of tf32 operands that folds the squared norms into the MMA, see
// assign_tc.cu and write_norm_ext in fkc_common.cuh): per point
// {h1,h2,h3,1,1,1,-delta,0} with h1+h2+h3 = -||x||^2/2, per centroid
// {1,1,1,h1,h2,h3,1,0} with h = -||c||^2/2; 32 bytes per row.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "fkc_common.cuh"
#include "fkc_internal.h"
#include "fkc_launch.cuh"

namespace fkc {
namespace {

constexpr int kExtBytes = kNormExtBytes;

// Sum of squares of one row, one warp. 16-byte vector loads when the row
// length allows it, scalar loads otherwise.
template <typename T>
__device__ __forceinline__ float warp_row_sumsq(const T* row, int D, int lane) {
  constexpr int kVec = 16 / sizeof(T);
  float acc = 0.f;
  if ((D * sizeof(T)) % 16 == 0) {
    for (int v = lane; v * kVec < D; v += 32) {
      const uint4 u = reinterpret_cast<const uint4*>(row)[v];
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int i = 0; i < kVec; ++i) {
        const float f = to_f32<T>(e[i]);
        acc = fmaf(f, f, acc);
      }
    }
  } else {
    for (int d = lane; d < D; d += 32) {
      const float f = to_f32<T>(row[d]);
      acc = fmaf(f, f, acc);
    }
  }
  return warp_sum(acc);
}

template <typename T>
__global__ void xnorm_ext_kernel(const T* __restrict__ x, uint8_t* __restrict__ aext,
                                 int64_t rows, int D) {
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t warps_total = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
       r < rows; r += warps_total) {
    const float s = warp_row_sumsq<T>(x + r * D, D, lane);
    if (lane == 0) write_norm_ext(aext + r * kExtBytes, -0.5f * s, true);
  }
}

// Centroid terms: the norm-extension row (cext, nullable) and ||c||^2 (c_sq_out,
// nullable). The squared norm is taken from c_sq when given (the caller's
// value, as the reference's raw-distance path does), else computed from c.
template <typename T>
__global__ void cnorm_ext_kernel(const T* __restrict__ c, const float* __restrict__ c_sq,
                                 uint8_t* __restrict__ cext, float* __restrict__ c_sq_out,
                                 int64_t rows, int D) {
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t warps_total = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
       r < rows; r += warps_total) {
    const float s = (c_sq != nullptr) ? c_sq[r] : warp_row_sumsq<T>(c + r * D, D, lane);
    if (lane == 0) {
      if (cext != nullptr) write_norm_ext(cext + r * kExtBytes, -0.5f * s, false);
      if (c_sq_out != nullptr) c_sq_out[r] = s;
    }
  }
}

// fp32 rows -> split bf16 rows for the tensor-core assignment of fp32 inputs:
// [hi | 0 | lo | 0], each half Dp = D rounded up to 64 elements, hi = bf16(v),
// lo = bf16(v - hi) (round to nearest even). The assignment kernel accumulates
// three passes, hi.hi + hi.lo + lo.hi, which is x.c up to about 2^-16 |x||c|
// (the lo.lo term and the rounding of lo are dropped). Points and centroids use
// the same layout. One thread per 4 elements of a half.
__global__ void split_bf16_kernel(const float* __restrict__ src, __nv_bfloat16* __restrict__ dst,
                                  int64_t rows, int D, int Dp) {
  pdl_wait();
  const int q = Dp / 4;  // 4-element groups per half
  const int64_t total = rows * q;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += stride) {
    const int64_t r = t / q;
    const int c = static_cast<int>(t - r * q) * 4;
    uint2 H = make_uint2(0u, 0u), Lo = make_uint2(0u, 0u);
    if (c < D) {
      const float4 v = *reinterpret_cast<const float4*>(src + r * D + c);
      const float f[4] = {v.x, v.y, v.z, v.w};
      uint32_t hi[2], lo[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const __nv_bfloat16 h0 = __float2bfloat16_rn(f[2 * e]);
        const __nv_bfloat16 h1 = __float2bfloat16_rn(f[2 * e + 1]);
        const __nv_bfloat16 l0 = __float2bfloat16_rn(f[2 * e] - __bfloat162float(h0));
        const __nv_bfloat16 l1 = __float2bfloat16_rn(f[2 * e + 1] - __bfloat162float(h1));
        hi[e] = __bfloat16_as_ushort(h0) | (static_cast<uint32_t>(__bfloat16_as_ushort(h1)) << 16);
        lo[e] = __bfloat16_as_ushort(l0) | (static_cast<uint32_t>(__bfloat16_as_ushort(l1)) << 16);
      }
      H = make_uint2(hi[0], hi[1]);
      Lo = make_uint2(lo[0], lo[1]);
    }
    __nv_bfloat16* row = dst + r * 2 * Dp + c;
    *reinterpret_cast<uint2*>(row) = H;
    *reinterpret_cast<uint2*>(row + Dp) = Lo;
  }
}

int sm_count_or_default_ne() {
  const DeviceInfo* di = nullptr;
  return current_device_info(&di) == FKC_OK ? di->sm_count : 148;
}

int grid_for_rows(int64_t rows, int warps_per_block) {
  const DeviceInfo* di = nullptr;
  int sms = 148;
  if (current_device_info(&di) == FKC_OK) sms = di->sm_count;
  int64_t blocks = (rows + warps_per_block - 1) / warps_per_block;
  const int64_t cap = static_cast<int64_t>(sms) * 16;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return static_cast<int>(blocks);
}

}  // namespace

int launch_xnorm_ext(const void* x, void* aext, int64_t B, int64_t N, int64_t D, int dtype,
                     cudaStream_t stream) {
  const int64_t rows = B * N;
  const dim3 grid(grid_for_rows(rows, 8));
  if (dtype == FKC_DTYPE_F32)
    return launch_pdl(xnorm_ext_kernel<float>, grid, dim3(256), 0, stream,
                      static_cast<const float*>(x), static_cast<uint8_t*>(aext), rows,
                      static_cast<int>(D));
  if (dtype == FKC_DTYPE_BF16)
    return launch_pdl(xnorm_ext_kernel<__nv_bfloat16>, grid, dim3(256), 0, stream,
                      static_cast<const __nv_bfloat16*>(x), static_cast<uint8_t*>(aext), rows,
                      static_cast<int>(D));
  return launch_pdl(xnorm_ext_kernel<__half>, grid, dim3(256), 0, stream,
                    static_cast<const __half*>(x), static_cast<uint8_t*>(aext), rows,
                    static_cast<int>(D));
}

int launch_cnorm_ext(const void* centroids, const float* c_sq, void* cext, float* c_sq_out,
                     int64_t B, int64_t K, int64_t D, int dtype, cudaStream_t stream) {
  const int64_t rows = B * K;
  const dim3 grid(grid_for_rows(rows, 8));
  uint8_t* ce = static_cast<uint8_t*>(cext);
  const int d = static_cast<int>(D);
  switch (dtype) {
    case FKC_DTYPE_BF16:
      return launch_pdl(cnorm_ext_kernel<__nv_bfloat16>, grid, dim3(256), 0, stream,
                        static_cast<const __nv_bfloat16*>(centroids), c_sq, ce, c_sq_out, rows, d);
    case FKC_DTYPE_F16:
      return launch_pdl(cnorm_ext_kernel<__half>, grid, dim3(256), 0, stream,
                        static_cast<const __half*>(centroids), c_sq, ce, c_sq_out, rows, d);
    case FKC_DTYPE_F32:
      return launch_pdl(cnorm_ext_kernel<float>, grid, dim3(256), 0, stream,
                        static_cast<const float*>(centroids), c_sq, ce, c_sq_out, rows, d);
    default:
      return set_error(FKC_EINVAL, "bad dtype %d", dtype);
  }
}

int64_t split_row_elems(int64_t D) { return 2 * ((D + 63) / 64 * 64); }

int launch_split_bf16(const void* src, void* dst, int64_t rows, int64_t D, cudaStream_t stream) {
  FKC_REQUIRE(D % 4 == 0, "split_bf16: D must be a multiple of 4");
  const int64_t Dp = split_row_elems(D) / 2;
  const int64_t threads = rows * (Dp / 4);
  int64_t blocks = (threads + 255) / 256;
  const int64_t cap = static_cast<int64_t>(sm_count_or_default_ne()) * 16;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return launch_pdl(split_bf16_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, stream,
                    static_cast<const float*>(src), static_cast<__nv_bfloat16*>(dst), rows,
                    static_cast<int>(D), static_cast<int>(Dp));
}

}  // namespace fkc
