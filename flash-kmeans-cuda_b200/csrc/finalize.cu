// Finalize: new = count > 0 ? dtype(sum / count) : old, one warp per centroid.
//
// Reference: flash_kmeans_cuda/csrc/update/update_finalize.cu:39-66 (one thread
// per element). Fused here, in the same pass over the new centroid:
//   * ||new||^2 of the dtype-rounded values (the reference recomputes it with
//     three torch kernels at the top of the next iteration, kmeans.py:94),
//     written as fp32 and/or as the tcgen05 assignment's norm-extension row;
//   * the centroid shift max ||new - old||_2 (kmeans.py:102-104), reduced
//     with an atomicMax on the bit pattern of a non-negative float.
// Division is IEEE round-to-nearest (the reference builds with --use_fast_math,
// i.e. an approximate division).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "fkc_common.cuh"
#include "fkc_internal.h"

namespace fkc {
namespace {

template <typename T>
__global__ void __launch_bounds__(256) finalize_kernel(
    const float* __restrict__ sums, const int32_t* __restrict__ counts,
    const T* __restrict__ old_c, T* __restrict__ new_c, float* __restrict__ c_sq_out,
    uint8_t* __restrict__ cext_out, float* __restrict__ shift_out, int64_t rows, int D) {
  const int lane = threadIdx.x & 31;
  const int64_t warps_total = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
       r < rows; r += warps_total) {
    const int32_t cnt = counts[r];
    const float fc = static_cast<float>(cnt);
    const float* s = sums + r * D;
    const T* o = old_c + r * D;
    T* n = new_c + r * D;
    float sq = 0.f, sh = 0.f;
    for (int d = lane; d < D; d += 32) {
      const T ov = o[d];
      const T nv = cnt > 0 ? from_f32<T>(__fdiv_rn(s[d], fc)) : ov;
      n[d] = nv;
      const float nf = to_f32<T>(nv);
      const float df = nf - to_f32<T>(ov);
      sq = fmaf(nf, nf, sq);
      sh = fmaf(df, df, sh);
    }
    sq = warp_sum(sq);
    sh = warp_sum(sh);
    if (lane == 0) {
      if (c_sq_out != nullptr) c_sq_out[r] = sq;
      if (cext_out != nullptr) write_norm_ext(cext_out + r * kNormExtBytes, -0.5f * sq, false);
      if (shift_out != nullptr)
        atomicMax(reinterpret_cast<unsigned int*>(shift_out), __float_as_uint(sqrtf(sh)));
    }
  }
}

}  // namespace

int launch_finalize(const float* sums, const int32_t* counts, const void* old_c, void* new_c,
                    float* c_sq_out, void* cext_out, float* shift_out, int64_t B, int64_t K,
                    int64_t D, int dtype, cudaStream_t stream) {
  const int64_t rows = B * K;
  if (shift_out != nullptr) FKC_CUDA_TRY(cudaMemsetAsync(shift_out, 0, sizeof(float), stream));
  const DeviceInfo* di = nullptr;
  FKC_TRY(current_device_info(&di));
  int64_t grid = (rows + 7) / 8;
  const int64_t cap = static_cast<int64_t>(di->sm_count) * 16;
  if (grid > cap) grid = cap;
  if (grid < 1) grid = 1;
  uint8_t* ce = static_cast<uint8_t*>(cext_out);
  const int d = static_cast<int>(D);
  switch (dtype) {
    case FKC_DTYPE_F16:
      finalize_kernel<__half><<<static_cast<unsigned>(grid), 256, 0, stream>>>(
          sums, counts, static_cast<const __half*>(old_c), static_cast<__half*>(new_c), c_sq_out,
          ce, shift_out, rows, d);
      break;
    case FKC_DTYPE_BF16:
      finalize_kernel<__nv_bfloat16><<<static_cast<unsigned>(grid), 256, 0, stream>>>(
          sums, counts, static_cast<const __nv_bfloat16*>(old_c),
          static_cast<__nv_bfloat16*>(new_c), c_sq_out, ce, shift_out, rows, d);
      break;
    case FKC_DTYPE_F32:
      finalize_kernel<float><<<static_cast<unsigned>(grid), 256, 0, stream>>>(
          sums, counts, static_cast<const float*>(old_c), static_cast<float*>(new_c), c_sq_out,
          ce, shift_out, rows, d);
      break;
    default:
      return set_error(FKC_EINVAL, "finalize: bad dtype %d", dtype);
  }
  FKC_CUDA_TRY(cudaGetLastError());
  count_launches(1);
  return FKC_OK;
}

}  // namespace fkc
