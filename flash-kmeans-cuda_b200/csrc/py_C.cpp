// flash_kmeans_cuda._C: the compiled Python module of the reference
// (flash_kmeans_cuda/csrc/bindings.cpp:107-127) as a PyTorch extension over the
// C-ABI of libfkc_b200.so. The same four functions, argument names, defaults
// and in-place semantics:
//
//   euclid_assign(x, centroids, x_sq, c_sq, out=None) -> (B, N) int32
//   centroid_update_sorted(x_sorted, cluster_ids_sorted, centroid_sums,
//                          centroid_counts)            adds into sums/counts
//   centroid_update_sorted_indexed(x, sorted_idx, cluster_ids_sorted,
//                                  centroid_sums, centroid_counts)
//   centroid_finalize(centroid_sums, centroid_counts, old_centroids, out=None)
//
// Like the reference module, the update entry points accumulate into the
// caller's sums and counts without zeroing them (bindings.cpp:73-90; the
// libtorch fkc:: API zeroes them first, as the reference's api.cpp does).
// Every call runs on the current PyTorch stream of the inputs' device; argument
// errors and C-ABI failures raise RuntimeError (the reference's TORCH_CHECK).
// Scratch memory comes from PyTorch's caching allocator.
#include <torch/extension.h>

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <optional>
#include <stdexcept>
#include <string>

#include "fkc_capi.h"

namespace {

void require(bool ok, const char* msg) {
  if (!ok) throw std::runtime_error(msg);
}

void check_status(int status, const char* what) {
  if (status != FKC_OK)
    throw std::runtime_error(std::string(what) + ": " + fkc_status_string(status) + ": " +
                             fkc_last_error());
}

int dtype_code(const at::Tensor& t) {
  switch (t.scalar_type()) {
    case at::kHalf: return FKC_DTYPE_F16;
    case at::kBFloat16: return FKC_DTYPE_BF16;
    case at::kFloat: return FKC_DTYPE_F32;
    default:
      throw std::runtime_error(std::string("unsupported dtype ") +
                               c10::toString(t.scalar_type()) +
                               " (expected float16, bfloat16 or float32)");
  }
}

fkc_stream_t stream_of(const at::Tensor& t) {
  return reinterpret_cast<fkc_stream_t>(
      at::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

at::Tensor euclid_assign(const at::Tensor& x, const at::Tensor& centroids,
                         const at::Tensor& x_sq, const at::Tensor& c_sq,
                         std::optional<at::Tensor> out) {
  require(x.is_cuda(), "x must be a CUDA tensor");
  require(centroids.is_cuda(), "centroids must be a CUDA tensor");
  require(x.dim() == 3 && centroids.dim() == 3, "x and centroids must be 3D (B,N,D)/(B,K,D)");
  const int64_t B = x.size(0), N = x.size(1), D = x.size(2), K = centroids.size(1);
  require(x.scalar_type() == centroids.scalar_type(), "x and centroids must share dtype");
  require(centroids.size(0) == B && centroids.size(2) == D,
          "centroids must be (B, K, D) matching x");
  require(x_sq.scalar_type() == at::kFloat && c_sq.scalar_type() == at::kFloat,
          "x_sq and c_sq must be fp32");
  at::Tensor ids;
  if (out.has_value()) {
    ids = *out;
    require(ids.scalar_type() == at::kInt, "out must be int32");
    require(ids.dim() == 2 && ids.size(0) == B && ids.size(1) == N, "out must be (B, N) int32");
  } else {
    ids = at::empty({B, N}, x.options().dtype(at::kInt));
  }
  require(x.is_contiguous() && centroids.is_contiguous() && x_sq.is_contiguous() &&
              c_sq.is_contiguous() && ids.is_contiguous(),
          "all tensors must be contiguous");
  require(c_sq.numel() == B * K, "c_sq must be (B, K)");
  const int code = dtype_code(x);
  const c10::cuda::CUDAGuard guard(x.device());
  const size_t ws_bytes = fkc_assign_workspace_size(B, N, K, D, code);
  const at::Tensor ws =
      at::empty({static_cast<int64_t>(ws_bytes > 0 ? ws_bytes : 1)}, x.options().dtype(at::kByte));
  check_status(fkc_assign(x.data_ptr(), centroids.data_ptr(),
                          x_sq.numel() == B * N ? x_sq.data_ptr<float>() : nullptr,
                          c_sq.data_ptr<float>(), ids.data_ptr<int32_t>(), B, N, K, D, code,
                          ws.data_ptr(), ws_bytes, stream_of(x)),
               "euclid_assign");
  return ids;
}

// Shape and dtype checks shared by the two update entry points; returns K.
int64_t check_update(const at::Tensor& x, const at::Tensor& ids_sorted, const at::Tensor& sums,
                     const at::Tensor& counts, const char* what_cuda, const char* what_dims) {
  require(x.is_cuda(), what_cuda);
  require(x.dim() == 3, what_dims);
  require(ids_sorted.scalar_type() == at::kInt, "cluster_ids must be int32");
  require(sums.scalar_type() == at::kFloat, "centroid_sums must be fp32");
  require(counts.scalar_type() == at::kInt, "centroid_counts must be int32");
  require(x.is_contiguous() && ids_sorted.is_contiguous() && sums.is_contiguous() &&
              counts.is_contiguous(),
          "all tensors must be contiguous");
  const int64_t B = x.size(0), N = x.size(1), D = x.size(2);
  require(sums.dim() == 3 && sums.size(0) == B && sums.size(2) == D,
          "centroid_sums must be (B, K, D)");
  const int64_t K = sums.size(1);
  require(counts.numel() == B * K, "centroid_counts must be (B, K)");
  require(ids_sorted.numel() == B * N, "cluster_ids_sorted must be (B, N)");
  return K;
}

void centroid_update_sorted(const at::Tensor& x_sorted, const at::Tensor& cluster_ids_sorted,
                            at::Tensor centroid_sums, at::Tensor centroid_counts) {
  const int64_t K = check_update(x_sorted, cluster_ids_sorted, centroid_sums, centroid_counts,
                                 "x_sorted must be CUDA", "x_sorted must be (B, N, D)");
  const int code = dtype_code(x_sorted);
  const c10::cuda::CUDAGuard guard(x_sorted.device());
  check_status(fkc_update_sorted(x_sorted.data_ptr(), cluster_ids_sorted.data_ptr<int32_t>(),
                                 centroid_sums.data_ptr<float>(),
                                 centroid_counts.data_ptr<int32_t>(), x_sorted.size(0),
                                 x_sorted.size(1), K, x_sorted.size(2), code,
                                 stream_of(x_sorted)),
               "centroid_update_sorted");
}

void centroid_update_sorted_indexed(const at::Tensor& x, const at::Tensor& sorted_idx,
                                    const at::Tensor& cluster_ids_sorted,
                                    at::Tensor centroid_sums, at::Tensor centroid_counts) {
  require(sorted_idx.scalar_type() == at::kInt, "sorted_idx must be int32");
  const int64_t K = check_update(x, cluster_ids_sorted, centroid_sums, centroid_counts,
                                 "x must be CUDA", "x must be (B, N, D)");
  require(sorted_idx.is_contiguous() && sorted_idx.numel() == x.size(0) * x.size(1),
          "sorted_idx must be (B, N)");
  const int code = dtype_code(x);
  const c10::cuda::CUDAGuard guard(x.device());
  check_status(fkc_update_sorted_indexed(x.data_ptr(), sorted_idx.data_ptr<int32_t>(),
                                         cluster_ids_sorted.data_ptr<int32_t>(),
                                         centroid_sums.data_ptr<float>(),
                                         centroid_counts.data_ptr<int32_t>(), x.size(0),
                                         x.size(1), K, x.size(2), code, stream_of(x)),
               "centroid_update_sorted_indexed");
}

at::Tensor centroid_finalize(const at::Tensor& centroid_sums, const at::Tensor& centroid_counts,
                             const at::Tensor& old_centroids, std::optional<at::Tensor> out) {
  require(centroid_sums.is_cuda(), "all tensors must be CUDA");
  require(centroid_sums.scalar_type() == at::kFloat, "sums must be fp32");
  require(centroid_counts.scalar_type() == at::kInt, "counts must be int32");
  at::Tensor nc = out.has_value() ? *out : at::empty_like(old_centroids);
  require(old_centroids.scalar_type() == nc.scalar_type(),
          "old and new centroids must share dtype");
  require(centroid_sums.is_contiguous() && centroid_counts.is_contiguous() &&
              old_centroids.is_contiguous() && nc.is_contiguous(),
          "all tensors must be contiguous");
  require(centroid_sums.dim() == 3, "sums must be (B, K, D)");
  const int64_t B = centroid_sums.size(0), K = centroid_sums.size(1), D = centroid_sums.size(2);
  require(old_centroids.numel() == B * K * D && nc.numel() == B * K * D,
          "old/new centroids must be (B, K, D)");
  require(centroid_counts.numel() == B * K, "counts must be (B, K)");
  const int code = dtype_code(old_centroids);
  const c10::cuda::CUDAGuard guard(centroid_sums.device());
  check_status(fkc_finalize(centroid_sums.data_ptr<float>(), centroid_counts.data_ptr<int32_t>(),
                            old_centroids.data_ptr(), nc.data_ptr(), nullptr, nullptr, B, K, D,
                            code, stream_of(centroid_sums)),
               "centroid_finalize");
  return nc;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() =
      "flash_kmeans_cuda._C: euclid_assign, centroid_update_sorted, "
      "centroid_update_sorted_indexed and centroid_finalize over the C-ABI of libfkc_b200.so";
  m.def("euclid_assign", &euclid_assign, py::arg("x"), py::arg("centroids"), py::arg("x_sq"),
        py::arg("c_sq"), py::arg("out") = py::none(),
        "argmin_k ||x - c_k||^2 per point; returns (B, N) int32");
  m.def("centroid_update_sorted", &centroid_update_sorted, py::arg("x_sorted"),
        py::arg("cluster_ids_sorted"), py::arg("centroid_sums"), py::arg("centroid_counts"),
        "sorted-run accumulate into the caller's (pre-zeroed) sums and counts");
  m.def("centroid_update_sorted_indexed", &centroid_update_sorted_indexed, py::arg("x"),
        py::arg("sorted_idx"), py::arg("cluster_ids_sorted"), py::arg("centroid_sums"),
        py::arg("centroid_counts"),
        "sorted-run accumulate reading x[b, sorted_idx[b, i]] into sums and counts");
  m.def("centroid_finalize", &centroid_finalize, py::arg("centroid_sums"),
        py::arg("centroid_counts"), py::arg("old_centroids"), py::arg("out") = py::none(),
        "new = counts > 0 ? sums / counts : old, in old's dtype");
}
