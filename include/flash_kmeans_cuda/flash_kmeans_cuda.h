#pragma once

// libtorch C++ API of the B200 flash-kmeans-cuda build (libflash_kmeans_cuda.so).
//
// Same namespace, functions, argument meanings and ownership rules as the
// reference header (OpsiClear/flash-kmeans-cuda flash_kmeans_cuda/csrc/
// flash_kmeans_cuda.h:31-77), so C++ consumers can switch libraries by
// relinking. Every function launches on at::cuda::getCurrentCUDAStream() of
// the input's device through the C-ABI in fkc_capi.h; argument errors throw
// c10::Error (TORCH_CHECK), as in the reference.

#include <ATen/ATen.h>

#if defined(_WIN32)
#if defined(FKC_BUILD_SHARED)
#define FKC_API __declspec(dllexport)
#else
#define FKC_API __declspec(dllimport)
#endif
#else
#define FKC_API __attribute__((visibility("default")))
#endif

namespace fkc {

// (B, N) int32 labels: argmin_k ||x[b,n] - centroids[b,k]||^2, ties -> lowest k.
// x (B, N, D), centroids (B, K, D) fp16/bf16/fp32 CUDA; x_sq (B, N) and c_sq
// (B, K) fp32 (c_sq is used as given; x_sq only by the fp32 / odd-D kernel).
FKC_API at::Tensor euclid_assign(const at::Tensor& x, const at::Tensor& centroids,
                                 const at::Tensor& x_sq, const at::Tensor& c_sq);

// Same, writing into caller-provided (B, N) int32 cluster_ids; returns it.
FKC_API at::Tensor euclid_assign_out(const at::Tensor& x, const at::Tensor& centroids,
                                     const at::Tensor& x_sq, const at::Tensor& c_sq,
                                     at::Tensor cluster_ids);

// Per-cluster sums (B, K, D) fp32 and counts (B, K) int32 from labels sorted
// along N and x gathered in that order. The buffers are zeroed first.
FKC_API void centroid_update_sorted(const at::Tensor& x_sorted,
                                    const at::Tensor& cluster_ids_sorted,
                                    at::Tensor centroid_sums, at::Tensor centroid_counts);

// Same accumulator reading rows x[b, sorted_idx[b, i]] of the original-order x.
FKC_API void centroid_update_sorted_indexed(const at::Tensor& x, const at::Tensor& sorted_idx,
                                            const at::Tensor& cluster_ids_sorted,
                                            at::Tensor centroid_sums,
                                            at::Tensor centroid_counts);

// new = counts > 0 ? sums / counts : old, in old's dtype (allocated).
FKC_API at::Tensor centroid_finalize(const at::Tensor& centroid_sums,
                                     const at::Tensor& centroid_counts,
                                     const at::Tensor& old_centroids);

// Same, written into caller-provided out (may alias old_centroids); returns out.
FKC_API at::Tensor centroid_finalize_out(const at::Tensor& centroid_sums,
                                         const at::Tensor& centroid_counts,
                                         const at::Tensor& old_centroids, at::Tensor out);

}  // namespace fkc
