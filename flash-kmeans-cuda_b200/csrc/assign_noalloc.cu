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
// kernel reads, 32 bytes per row; for fp32 also the split bf16 operand rows)
// lives in a file-scope __device__ array of FKC_ASSIGN_NOALLOC_SCRATCH_BYTES
// (32 MiB). The CUDA runtime places it when this file's module is loaded on a
// device; nothing here calls cudaMalloc, cudaFree or an allocating library
// routine. In host code the array's name is only a host-side stand-in, so
// every call looks up the array's address on the current device with
// cudaGetSymbolAddress (a host-side query that allocates nothing) and passes
// that address on. Looking it up per call rather than caching it keeps the
// address right when the device's context is torn down and created again
// (cudaDeviceReset, a primary-context reset), after which the module is
// loaded anew and the array may sit elsewhere. The first call on a device
// also loads the module there (the runtime loads modules lazily), so that
// first call should come before any stream capture. The call then runs
// exactly the fkc_assign code path with the array as its workspace.
//
// Sharing. Every call on a device uses the same array. Nothing in it has to
// start at zero: each call writes both norm slices (and the split rows) in
// full before the assignment kernel reads them, and the kernel's tensor maps
// end at N and K, so it never reads rows of the array beyond this call's
// slices. The array keeps whatever the last call wrote. Calls that overlap on
// the GPU (different streams with no ordering between them, or different host
// threads) race on the array; order them on one stream or with events. Calls
// on different devices use different instances of the array.
#include <cuda_runtime.h>

#include "fkc_internal.h"

static_assert(FKC_ASSIGN_NOALLOC_SCRATCH_BYTES % 256 == 0, "scratch size");

static __device__ __align__(256) uint8_t g_fkc_noalloc_scratch[FKC_ASSIGN_NOALLOC_SCRATCH_BYTES];

namespace fkc {
namespace {

// Device address of the scratch array in the current context.
int noalloc_scratch(void** out) {
  int dev = -1;
  const cudaError_t de = cudaGetDevice(&dev);
  if (de != cudaSuccess) {
    cudaGetLastError();
    return set_error(FKC_EUNSUPPORTED, "no CUDA device: %s", cudaGetErrorString(de));
  }
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_fkc_noalloc_scratch);
  if (e != cudaSuccess || p == nullptr) {
    cudaGetLastError();
    return set_error(FKC_ECUDA, "fkc_assign_noalloc: scratch lookup on device %d failed: %s",
                     dev, cudaGetErrorString(e));
  }
  *out = p;
  return FKC_OK;
}

}  // namespace
}  // namespace fkc

extern "C" FKC_CAPI_EXPORT int fkc_assign_noalloc(const void* x, const void* centroids,
                                                  const float* x_sq, const float* c_sq,
                                                  int32_t* ids, int64_t B, int64_t N, int64_t K,
                                                  int64_t D, int dtype, fkc_stream_t stream) {
  fkc::clear_error();
  // The size check comes before any CUDA call. A call that fkc_assign would
  // route to the CUDA-core kernel needs no scratch (0 here): a shape or dtype
  // outside the tensor-core path, FKC_ASSIGN_FORCE_SAFE=1, or x / centroids
  // not 16-byte aligned. Invalid shapes also give 0 and are reported by
  // fkc_assign's own argument checks.
  size_t need = fkc::assign_may_use_tc_host(x, centroids, D, dtype)
                    ? fkc_assign_workspace_size(B, N, K, D, dtype)
                    : 0;
  // fp32 beyond the scratch: fkc_assign keeps the CUDA-core kernel when the
  // workspace cannot hold the split operand rows, so no scratch is needed.
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
