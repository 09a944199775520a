// libtorch fkc:: API (include/flash_kmeans_cuda/flash_kmeans_cuda.h) over the
// C-ABI of libfkc_b200.so. Mirrors the reference's api.cpp behaviour
// (flash_kmeans_cuda/csrc/api.cpp:27-113): same checks, euclid_assign allocates
// its output, the sorted update entry points zero sums/counts before
// accumulating, finalize allocates or writes into `out`.
#include "flash_kmeans_cuda/flash_kmeans_cuda.h"

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "fkc_capi.h"

namespace fkc {
namespace {

int dtype_code(const at::Tensor& t) {
  switch (t.scalar_type()) {
    case at::kHalf: return FKC_DTYPE_F16;
    case at::kBFloat16: return FKC_DTYPE_BF16;
    case at::kFloat: return FKC_DTYPE_F32;
    default: TORCH_CHECK(false, "unsupported dtype ", t.scalar_type());
  }
  return -1;
}

void check_status(int status, const char* what) {
  TORCH_CHECK(status == FKC_OK, what, ": ", fkc_status_string(status), ": ", fkc_last_error());
}

fkc_stream_t current_stream() {
  return reinterpret_cast<fkc_stream_t>(at::cuda::getCurrentCUDAStream().stream());
}

void validate_assign_inputs(const at::Tensor& x, const at::Tensor& centroids,
                            const at::Tensor& x_sq, const at::Tensor& c_sq,
                            const at::Tensor& cluster_ids) {
  TORCH_CHECK(x.is_cuda(), "x must be a CUDA tensor");
  TORCH_CHECK(centroids.is_cuda(), "centroids must be a CUDA tensor");
  TORCH_CHECK(x.dim() == 3, "x must be (B, N, D)");
  TORCH_CHECK(centroids.dim() == 3, "centroids must be (B, K, D)");
  TORCH_CHECK(x.scalar_type() == centroids.scalar_type(), "x and centroids must share dtype");
  TORCH_CHECK(centroids.size(0) == x.size(0) && centroids.size(2) == x.size(2),
              "centroids must be (B, K, D) matching x");
  TORCH_CHECK(x_sq.scalar_type() == at::kFloat, "x_sq must be fp32");
  TORCH_CHECK(c_sq.scalar_type() == at::kFloat, "c_sq must be fp32");
  TORCH_CHECK(c_sq.numel() == centroids.size(0) * centroids.size(1), "c_sq must be (B, K)");
  TORCH_CHECK(cluster_ids.scalar_type() == at::kInt, "cluster_ids must be int32");
  TORCH_CHECK(cluster_ids.dim() == 2 && cluster_ids.size(0) == x.size(0) &&
                  cluster_ids.size(1) == x.size(1),
              "cluster_ids must be (B, N) int32");
  TORCH_CHECK(x.is_contiguous() && centroids.is_contiguous() && x_sq.is_contiguous() &&
                  c_sq.is_contiguous() && cluster_ids.is_contiguous(),
              "all tensors must be contiguous");
}

void validate_update(const at::Tensor& x, const at::Tensor& ids, const at::Tensor& sums,
                     const at::Tensor& counts) {
  TORCH_CHECK(x.is_cuda(), "x must be CUDA");
  TORCH_CHECK(x.dim() == 3, "x must be (B, N, D)");
  TORCH_CHECK(ids.scalar_type() == at::kInt, "cluster_ids must be int32");
  TORCH_CHECK(sums.scalar_type() == at::kFloat, "centroid_sums must be fp32");
  TORCH_CHECK(counts.scalar_type() == at::kInt, "centroid_counts must be int32");
  TORCH_CHECK(x.is_contiguous() && ids.is_contiguous() && sums.is_contiguous() &&
                  counts.is_contiguous(),
              "all tensors must be contiguous");
  TORCH_CHECK(sums.dim() == 3 && sums.size(0) == x.size(0) && sums.size(2) == x.size(2),
              "centroid_sums must be (B, K, D)");
  TORCH_CHECK(counts.numel() == sums.size(0) * sums.size(1), "centroid_counts must be (B, K)");
  TORCH_CHECK(ids.numel() == x.size(0) * x.size(1), "cluster_ids_sorted must be (B, N)");
}

}  // namespace

at::Tensor euclid_assign(const at::Tensor& x, const at::Tensor& centroids,
                         const at::Tensor& x_sq, const at::Tensor& c_sq) {
  at::Tensor ids =
      at::empty({x.size(0), x.size(1)}, at::TensorOptions().dtype(at::kInt).device(x.device()));
  return euclid_assign_out(x, centroids, x_sq, c_sq, ids);
}

at::Tensor euclid_assign_out(const at::Tensor& x, const at::Tensor& centroids,
                             const at::Tensor& x_sq, const at::Tensor& c_sq,
                             at::Tensor cluster_ids) {
  validate_assign_inputs(x, centroids, x_sq, c_sq, cluster_ids);
  c10::cuda::CUDAGuard guard(x.device());
  const int64_t B = x.size(0), N = x.size(1), D = x.size(2), K = centroids.size(1);
  const int code = dtype_code(x);
  const size_t ws_bytes = fkc_assign_workspace_size(B, N, K, D, code);
  at::Tensor ws = at::empty({static_cast<int64_t>(ws_bytes > 0 ? ws_bytes : 1)},
                            at::TensorOptions().dtype(at::kByte).device(x.device()));
  const float* xsq = x_sq.numel() == B * N ? x_sq.data_ptr<float>() : nullptr;
  check_status(fkc_assign(x.data_ptr(), centroids.data_ptr(), xsq, c_sq.data_ptr<float>(),
                          cluster_ids.data_ptr<int32_t>(), B, N, K, D, code, ws.data_ptr(),
                          ws_bytes, current_stream()),
               "euclid_assign");
  return cluster_ids;
}

void centroid_update_sorted(const at::Tensor& x_sorted, const at::Tensor& cluster_ids_sorted,
                            at::Tensor centroid_sums, at::Tensor centroid_counts) {
  validate_update(x_sorted, cluster_ids_sorted, centroid_sums, centroid_counts);
  c10::cuda::CUDAGuard guard(x_sorted.device());
  centroid_sums.zero_();
  centroid_counts.zero_();
  check_status(fkc_update_sorted(x_sorted.data_ptr(), cluster_ids_sorted.data_ptr<int32_t>(),
                                 centroid_sums.data_ptr<float>(),
                                 centroid_counts.data_ptr<int32_t>(), x_sorted.size(0),
                                 x_sorted.size(1), centroid_sums.size(1), x_sorted.size(2),
                                 dtype_code(x_sorted), current_stream()),
               "centroid_update_sorted");
}

void centroid_update_sorted_indexed(const at::Tensor& x, const at::Tensor& sorted_idx,
                                    const at::Tensor& cluster_ids_sorted,
                                    at::Tensor centroid_sums, at::Tensor centroid_counts) {
  validate_update(x, cluster_ids_sorted, centroid_sums, centroid_counts);
  TORCH_CHECK(sorted_idx.scalar_type() == at::kInt, "sorted_idx must be int32");
  TORCH_CHECK(sorted_idx.is_contiguous() && sorted_idx.numel() == x.size(0) * x.size(1),
              "sorted_idx must be (B, N)");
  c10::cuda::CUDAGuard guard(x.device());
  centroid_sums.zero_();
  centroid_counts.zero_();
  check_status(fkc_update_sorted_indexed(x.data_ptr(), sorted_idx.data_ptr<int32_t>(),
                                         cluster_ids_sorted.data_ptr<int32_t>(),
                                         centroid_sums.data_ptr<float>(),
                                         centroid_counts.data_ptr<int32_t>(), x.size(0),
                                         x.size(1), centroid_sums.size(1), x.size(2),
                                         dtype_code(x), current_stream()),
               "centroid_update_sorted_indexed");
}

at::Tensor centroid_finalize(const at::Tensor& centroid_sums, const at::Tensor& centroid_counts,
                             const at::Tensor& old_centroids) {
  return centroid_finalize_out(centroid_sums, centroid_counts, old_centroids,
                               at::empty_like(old_centroids));
}

at::Tensor centroid_finalize_out(const at::Tensor& centroid_sums,
                                 const at::Tensor& centroid_counts,
                                 const at::Tensor& old_centroids, at::Tensor out) {
  TORCH_CHECK(centroid_sums.is_cuda(), "all tensors must be CUDA");
  TORCH_CHECK(centroid_sums.scalar_type() == at::kFloat, "sums must be fp32");
  TORCH_CHECK(centroid_counts.scalar_type() == at::kInt, "counts must be int32");
  TORCH_CHECK(old_centroids.scalar_type() == out.scalar_type(),
              "old and new centroids must share dtype");
  TORCH_CHECK(centroid_sums.is_contiguous() && centroid_counts.is_contiguous() &&
                  old_centroids.is_contiguous() && out.is_contiguous(),
              "all tensors must be contiguous");
  TORCH_CHECK(centroid_sums.dim() == 3, "sums must be (B, K, D)");
  const int64_t B = centroid_sums.size(0), K = centroid_sums.size(1), D = centroid_sums.size(2);
  TORCH_CHECK(old_centroids.numel() == B * K * D && out.numel() == B * K * D,
              "old/new centroids must be (B, K, D)");
  TORCH_CHECK(centroid_counts.numel() == B * K, "counts must be (B, K)");
  c10::cuda::CUDAGuard guard(centroid_sums.device());
  check_status(fkc_finalize(centroid_sums.data_ptr<float>(), centroid_counts.data_ptr<int32_t>(),
                            old_centroids.data_ptr(), out.data_ptr(), nullptr, nullptr, B, K, D,
                            dtype_code(old_centroids), current_stream()),
               "centroid_finalize");
  return out;
}

}  // namespace fkc
