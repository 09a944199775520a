// C++ consumer smoke test of libflash_kmeans_cuda.so (the fkc:: libtorch API).
// Checks, per the reference's tests/cpp/smoke.cpp:21-109: assignment against a
// matmul + argmin reference for D in {1,7,16,31,32,48,64,96,128,256,257};
// sorted == indexed update (sums allclose, counts exact); finalize against
// where(count > 0, sums / count, old). Exit code 0 on success.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <iostream>
#include <stdexcept>
#include <vector>

#include "flash_kmeans_cuda/flash_kmeans_cuda.h"

static void check(bool ok, const char* msg) {
  if (!ok) throw std::runtime_error(msg);
}

static void test_assign(int64_t D) {
  const int64_t B = 1, N = 512, K = 64;
  auto opts = at::TensorOptions().device(at::kCUDA).dtype(at::kHalf);
  at::Tensor x = at::randn({B, N, D}, opts);
  at::Tensor c = at::randn({B, K, D}, opts);
  at::Tensor x_sq = x.to(at::kFloat).pow(2).sum(-1).contiguous();
  at::Tensor c_sq = c.to(at::kFloat).pow(2).sum(-1).contiguous();
  at::Tensor ids = fkc::euclid_assign(x, c, x_sq, c_sq);
  at::Tensor cross = at::matmul(x.to(at::kDouble), c.to(at::kDouble).transpose(1, 2));
  at::Tensor dist = x_sq.to(at::kDouble).unsqueeze(-1) + c_sq.to(at::kDouble).unsqueeze(1) - 2.0 * cross;
  at::Tensor ref = std::get<1>(dist.min(-1)).to(at::kInt);
  check(ids.sizes() == at::IntArrayRef({B, N}) && ids.scalar_type() == at::kInt, "assign shape/dtype");
  const double dis = ids.ne(ref).to(at::kFloat).mean().item<double>();
  std::cout << "assign D=" << D << " disagreement=" << dis << "\n";
  check(dis < 0.01, "assign disagreement exceeds 1%");
  at::Tensor out = at::full({B, N}, -1, ids.options());
  at::Tensor r = fkc::euclid_assign_out(x, c, x_sq, c_sq, out);
  check(r.data_ptr() == out.data_ptr() && out.equal(ids), "euclid_assign_out");
}

static void test_update_finalize(int64_t D) {
  const int64_t B = 1, N = 512, K = 16;
  auto f = at::TensorOptions().device(at::kCUDA).dtype(at::kFloat);
  auto i = at::TensorOptions().device(at::kCUDA).dtype(at::kInt);
  at::Tensor x = at::randn({B, N, D}, f);
  at::Tensor ids = at::randint(K, {B, N}, i);
  auto sp = at::sort(ids, 1);
  at::Tensor sorted_ids = std::get<0>(sp).contiguous();
  at::Tensor sorted_idx = std::get<1>(sp).to(at::kInt).contiguous();
  at::Tensor x_sorted =
      x.gather(1, sorted_idx.to(at::kLong).unsqueeze(-1).expand({B, N, D})).contiguous();
  at::Tensor sums = at::full({B, K, D}, 5.0, f), counts = at::full({B, K}, 9, i);
  fkc::centroid_update_sorted(x_sorted, sorted_ids, sums, counts);  // zeroes first
  at::Tensor sums2 = at::empty_like(sums), counts2 = at::empty_like(counts);
  fkc::centroid_update_sorted_indexed(x, sorted_idx, sorted_ids, sums2, counts2);
  check(at::allclose(sums, sums2, 1e-4, 1e-4), "indexed update sums mismatch");
  check(counts.equal(counts2), "indexed update counts mismatch");
  check(counts.sum().item<int64_t>() == N, "counts do not sum to N");
  at::Tensor old = at::randn({B, K, D}, f);
  at::Tensor fin = fkc::centroid_finalize(sums, counts, old);
  at::Tensor ref = at::where(counts.unsqueeze(-1).gt(0),
                             sums / counts.clamp_min(1).to(at::kFloat).unsqueeze(-1), old);
  check(at::allclose(fin, ref, 1e-4, 1e-4), "finalize mismatch");
  std::cout << "update/finalize D=" << D << " passed\n";
}

int main() {
  try {
    check(at::cuda::is_available(), "CUDA is not available");
    c10::cuda::CUDAGuard guard(0);
    at::manual_seed(0);
    for (int64_t D : std::vector<int64_t>{1, 7, 16, 31, 32, 48, 64, 96, 128, 256, 257}) test_assign(D);
    for (int64_t D : std::vector<int64_t>{1, 7, 16, 31, 32, 64, 128, 257}) test_update_finalize(D);
    at::cuda::getCurrentCUDAStream().synchronize();
    std::cout << "fkc:: C++ API smoke test passed\n";
    return 0;
  } catch (const std::exception& e) {
    std::cerr << "fkc:: C++ API smoke test failed: " << e.what() << "\n";
    return 1;
  }
}
