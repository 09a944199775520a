// CUDA-core assignment for the shapes the tensor-core kernel does not take:
// fp32 inputs, D not a multiple of 16, D > 384, and devices other than sm_100.
//
// Semantics are those of the reference's safe kernel
// (flash_kmeans_cuda/csrc/assign/assign_safe.cu:38-81 and assign_common.cuh:15-36):
//   dist = max(x_sq + c_sq - 2 * dot, 0), dot accumulated in fp32 in ascending d,
//   strict "<" so ties keep the lowest k.
// x_sq / c_sq come from the caller when given (as in the reference), otherwise
// they are computed here in fp32.
//
// Layout: a CTA owns 128 points (one per thread) and streams the centroids in
// tiles of 32 through shared memory, D in slices of 32; each thread keeps 32
// dot-product accumulators in registers.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cfloat>

#include "fkc_internal.h"

namespace fkc {
namespace {

constexpr int kPts = 128;  // points per CTA (threads)
constexpr int kCt = 32;    // centroids per tile
constexpr int kDt = 32;    // feature slice

template <typename T>
__device__ __forceinline__ float ld_f32(const T* p);
template <>
__device__ __forceinline__ float ld_f32<float>(const float* p) {
  return *p;
}
template <>
__device__ __forceinline__ float ld_f32<__half>(const __half* p) {
  return __half2float(*p);
}
template <>
__device__ __forceinline__ float ld_f32<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}

template <typename T>
__global__ void __launch_bounds__(kPts) assign_simt_kernel(
    const T* __restrict__ x, const T* __restrict__ c, const float* __restrict__ x_sq,
    const float* __restrict__ c_sq, int32_t* __restrict__ ids, int N, int K, int D) {
  __shared__ float xs[kPts][kDt + 1];
  __shared__ float cs[kCt][kDt + 1];
  __shared__ float csq[kCt];

  const int b = blockIdx.y;
  const int n0 = blockIdx.x * kPts;
  const int t = threadIdx.x;
  const int n = n0 + t;
  const T* xb = x + static_cast<size_t>(b) * N * D;
  const T* cb = c + static_cast<size_t>(b) * K * D;

  // ||x||^2 for this thread's point.
  float xsq = 0.f;
  if (n < N) {
    if (x_sq != nullptr) {
      xsq = x_sq[static_cast<size_t>(b) * N + n];
    } else {
      const T* row = xb + static_cast<size_t>(n) * D;
      for (int d = 0; d < D; ++d) {
        const float v = ld_f32<T>(row + d);
        xsq = fmaf(v, v, xsq);
      }
    }
  }

  float best = FLT_MAX;
  int best_k = 0;
  for (int k0 = 0; k0 < K; k0 += kCt) {
    float acc[kCt];
#pragma unroll
    for (int j = 0; j < kCt; ++j) acc[j] = 0.f;
    for (int d0 = 0; d0 < D; d0 += kDt) {
      __syncthreads();
      // x slice: kPts x kDt, coalesced along d.
      for (int i = t; i < kPts * kDt; i += kPts) {
        const int r = i / kDt, dd = i % kDt;
        const int gn = n0 + r, gd = d0 + dd;
        xs[r][dd] = (gn < N && gd < D) ? ld_f32<T>(xb + static_cast<size_t>(gn) * D + gd) : 0.f;
      }
      for (int i = t; i < kCt * kDt; i += kPts) {
        const int r = i / kDt, dd = i % kDt;
        const int gk = k0 + r, gd = d0 + dd;
        cs[r][dd] = (gk < K && gd < D) ? ld_f32<T>(cb + static_cast<size_t>(gk) * D + gd) : 0.f;
      }
      __syncthreads();
      const int dlim = min(kDt, D - d0);
      for (int dd = 0; dd < dlim; ++dd) {
        const float xv = xs[t][dd];
#pragma unroll
        for (int j = 0; j < kCt; ++j) acc[j] = fmaf(xv, cs[j][dd], acc[j]);
      }
    }
    __syncthreads();
    if (t < kCt) {
      const int gk = k0 + t;
      float v = 0.f;
      if (gk < K) {
        if (c_sq != nullptr) {
          v = c_sq[static_cast<size_t>(b) * K + gk];
        } else {
          const T* row = cb + static_cast<size_t>(gk) * D;
          for (int d = 0; d < D; ++d) {
            const float e = ld_f32<T>(row + d);
            v = fmaf(e, e, v);
          }
        }
      }
      csq[t] = v;
    }
    __syncthreads();
    const int jlim = min(kCt, K - k0);
    for (int j = 0; j < jlim; ++j) {
      float dist = xsq + csq[j] - 2.0f * acc[j];
      dist = dist > 0.f ? dist : 0.f;
      if (dist < best) {
        best = dist;
        best_k = k0 + j;
      }
    }
  }
  if (n < N) ids[static_cast<size_t>(b) * N + n] = best_k;
}

}  // namespace

int launch_assign_simt(const void* x, const void* centroids, const float* x_sq,
                       const float* c_sq, int32_t* ids, int64_t B, int64_t N, int64_t K,
                       int64_t D, int dtype, cudaStream_t stream) {
  FKC_REQUIRE(B <= 65535, "assign: B=%lld exceeds the fallback kernel's grid limit",
              static_cast<long long>(B));
  const dim3 grid(static_cast<unsigned>((N + kPts - 1) / kPts), static_cast<unsigned>(B));
  const int n = static_cast<int>(N), k = static_cast<int>(K), d = static_cast<int>(D);
  switch (dtype) {
    case FKC_DTYPE_F32:
      assign_simt_kernel<float><<<grid, kPts, 0, stream>>>(
          static_cast<const float*>(x), static_cast<const float*>(centroids), x_sq, c_sq, ids, n,
          k, d);
      break;
    case FKC_DTYPE_F16:
      assign_simt_kernel<__half><<<grid, kPts, 0, stream>>>(
          static_cast<const __half*>(x), static_cast<const __half*>(centroids), x_sq, c_sq, ids,
          n, k, d);
      break;
    case FKC_DTYPE_BF16:
      assign_simt_kernel<__nv_bfloat16><<<grid, kPts, 0, stream>>>(
          static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(centroids),
          x_sq, c_sq, ids, n, k, d);
      break;
    default:
      return set_error(FKC_EINVAL, "assign: bad dtype %d", dtype);
  }
  FKC_CUDA_TRY(cudaGetLastError());
  count_launches(1);
  return FKC_OK;
}

}  // namespace fkc
