// fkc_assign_noalloc: fkc_assign without a caller workspace and without any
// device allocation.
//
// Who needs it. Some callers hold device pointers but cannot allocate device
// memory: an FFI binding that mirrors the 5-argument euclid_assign(x,
// centroids, x_sq, c_sq, out) signature and receives its tensors from another
// runtime has no device allocator of its own; a host whose device memory is
// reserved up front by a pooling allocator would see a raw cudaMalloc fail;
// and a latency-critical pipeline cannot afford cudaFree, which synchronises
// the whole device. Such callers cannot hand fkc_assign the workspace it needs
// for the tensor-core path.
//
// How. The scratch (the per-point and per-centroid norm slices the tensor-core
// kernel reads, 32 bytes per row) lives in a file-scope __device__ array of
// FKC_ASSIGN_NOALLOC_SCRATCH_BYTES (32 MiB). The CUDA runtime places it when
// this file's module is loaded on a device; nothing here calls cudaMalloc,
// cudaFree or an allocating library routine. The first call on each device
// looks up the array's address on that device with cudaGetSymbolAddress (with
// the device current) and caches it. The call then runs exactly the fkc_assign
// code path with the array as its workspace.
//
// Sharing. Every call on a device uses the same array. Nothing in it has to
// start at zero: each call writes both norm slices in full before the
// assignment kernel reads them, and the kernel's tensor maps end at N and K,
// so it never reads rows of the array beyond this call's slices. Calls that
// overlap on the GPU (different streams with no ordering between them, or
// different host threads) race on the array; order them on one stream or with
// events. Calls on different devices use different instances of the array.
#include <cuda_runtime.h>

#include <array>
#include <mutex>

#include "fkc_internal.h"

static_assert(FKC_ASSIGN_NOALLOC_SCRATCH_BYTES % 256 == 0, "scratch size");

static __device__ __align__(256) uint8_t g_fkc_noalloc_scratch[FKC_ASSIGN_NOALLOC_SCRATCH_BYTES];

namespace fkc {
namespace {

constexpr int kMaxNoallocDevices = 64;
std::mutex g_noalloc_mu;
std::array<void*, kMaxNoallocDevices> g_noalloc_ptr{};

// Address of the scratch array on the current device (looked up once per
// device, with that device current).
int noalloc_scratch(void** out) {
  int dev = -1;
  const cudaError_t de = cudaGetDevice(&dev);
  if (de != cudaSuccess) {
    cudaGetLastError();
    return set_error(FKC_EUNSUPPORTED, "no CUDA device: %s", cudaGetErrorString(de));
  }
  if (dev < 0 || dev >= kMaxNoallocDevices)
    return set_error(FKC_EUNSUPPORTED, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_fkc_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return set_error(FKC_ECUDA, "fkc_assign_noalloc: scratch lookup on device %d failed: %s",
                       dev, cudaGetErrorString(e));
    }
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return FKC_OK;
}

}  // namespace
}  // namespace fkc

extern "C" FKC_CAPI_EXPORT int fkc_assign_noalloc(const void* x, const void* centroids,
                                                  const float* x_sq, const float* c_sq,
                                                  int32_t* ids, int64_t B, int64_t N, int64_t K,
                                                  int64_t D, int dtype, fkc_stream_t stream) {
  fkc::clear_error();
  // The size check comes before any CUDA call. Shapes that do not take the
  // tensor-core path need no scratch (0 here); invalid shapes also give 0 and
  // are reported by fkc_assign's own argument checks.
  size_t need = fkc_assign_workspace_size(B, N, K, D, dtype);
  // fp32 beyond the scratch: the CUDA-core kernel, which needs no scratch.
  if (dtype == FKC_DTYPE_F32 && need > static_cast<size_t>(FKC_ASSIGN_NOALLOC_SCRATCH_BYTES))
    need = 0;
  if (need > static_cast<size_t>(FKC_ASSIGN_NOALLOC_SCRATCH_BYTES))
    return fkc::set_error(
        FKC_EWORKSPACE,
        "fkc_assign_noalloc: B=%lld N=%lld K=%lld needs %zu bytes of scratch, more than the "
        "%u-byte static scratch holds (32 bytes per point and per centroid); use fkc_assign "
        "with a caller workspace",
        static_cast<long long>(B), static_cast<long long>(N), static_cast<long long>(K), need,
        static_cast<unsigned>(FKC_ASSIGN_NOALLOC_SCRATCH_BYTES));
  void* scratch = nullptr;
  size_t scratch_bytes = 0;
  if (need > 0) {
    FKC_TRY(fkc::noalloc_scratch(&scratch));
    scratch_bytes = FKC_ASSIGN_NOALLOC_SCRATCH_BYTES;
  }
  return fkc_assign(x, centroids, x_sq, c_sq, ids, B, N, K, D, dtype, scratch, scratch_bytes,
                    stream);
}
