// extern "C" entry points of libfkc_b200.so (declared in include/fkc_capi.h),
// plus the host-side services the launchers share: per-thread error text,
// per-device property cache, TMA descriptor encoding and the device error word.
#include <cuda.h>
#include <cuda_runtime.h>

#include <array>
#include <atomic>
#include <cstdarg>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "fkc_internal.h"
#include "fkc_launch.cuh"

// Written (atomicCAS from 0) by kernels whose bounded pipeline waits expired.
__device__ int g_fkc_device_error = 0;

namespace fkc {
namespace {

thread_local char g_last_error[1024] = {0};

constexpr int kMaxDevices = 64;
std::mutex g_dev_mu;
std::array<DeviceInfo, kMaxDevices> g_dev_info{};
std::array<bool, kMaxDevices> g_dev_ready{};
std::array<int*, kMaxDevices> g_err_word{};
std::atomic<uint64_t> g_launches{0};

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;
std::once_flag g_encode_once;

bool env_flag(const char* name) {
  const char* s = std::getenv(name);
  return s != nullptr && (std::strcmp(s, "1") == 0 || std::strcmp(s, "true") == 0);
}

// FKC_ASSIGN_FORCE_SAFE=1 routes every assignment to the CUDA-core kernel
// (reference: flash_kmeans_cuda/csrc/api.cpp:12-19, read once).
bool force_safe_path() {
  static const bool v = env_flag("FKC_ASSIGN_FORCE_SAFE");
  return v;
}

// FKC_DETERMINISTIC=1 (read once) makes the Lloyd update bit-reproducible:
// stable counting sort + span gather + ordered join (update_det.cu) instead of
// the counting sort with atomic slot claims and vector-atomic accumulation,
// which is faster (c3, one B200: 0.90 vs 0.91 ms/iter; c4 0.134 vs 0.159).
bool deterministic_update() {
  static const bool v = env_flag("FKC_DETERMINISTIC");
  return v;
}

}  // namespace

int set_error(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

void clear_error() { g_last_error[0] = '\0'; }

void count_launches(int n) {
  if (count_captured_launch(n)) return;  // recorded into a graph, counted per replay
  g_launches.fetch_add(static_cast<uint64_t>(n));
}

int current_device_info(const DeviceInfo** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(FKC_EUNSUPPORTED, "no CUDA device: %s", cudaGetErrorString(e));
  }
  if (dev < 0 || dev >= kMaxDevices) return set_error(FKC_EUNSUPPORTED, "device %d", dev);
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (!g_dev_ready[dev]) {
    DeviceInfo di;
    di.device = dev;
    FKC_CUDA_TRY(cudaDeviceGetAttribute(&di.sm_count, cudaDevAttrMultiProcessorCount, dev));
    FKC_CUDA_TRY(cudaDeviceGetAttribute(&di.cc_major, cudaDevAttrComputeCapabilityMajor, dev));
    FKC_CUDA_TRY(cudaDeviceGetAttribute(&di.cc_minor, cudaDevAttrComputeCapabilityMinor, dev));
    int smem = 0;
    FKC_CUDA_TRY(cudaDeviceGetAttribute(&smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    di.smem_optin = static_cast<size_t>(smem);
    g_dev_info[dev] = di;
    g_dev_ready[dev] = true;
  }
  *out = &g_dev_info[dev];
  return FKC_OK;
}

int* device_error_word() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (g_err_word[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_fkc_device_error) != cudaSuccess) return nullptr;
    g_err_word[dev] = static_cast<int*>(p);
  }
  return g_err_word[dev];
}

int encode_tmap_3d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t dim0,
                   uint64_t dim1, uint64_t dim2, uint64_t stride1_bytes, uint64_t stride2_bytes,
                   uint32_t box0, uint32_t box1, CUtensorMapSwizzle swizzle) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<EncodeTiledFn>(fn);
    cudaGetLastError();
  });
  if (g_encode == nullptr)
    return set_error(FKC_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t dims[3] = {dim0, dim1, dim2};
  const cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  const cuuint32_t box[3] = {box0, box1, 1};
  const cuuint32_t elem_strides[3] = {1, 1, 1};
  const CUresult r = g_encode(map, dtype, 3, const_cast<void*>(base), dims, strides, box,
                              elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(FKC_ECUDA,
                     "cuTensorMapEncodeTiled failed (%d): dims {%llu,%llu,%llu} box {%u,%u}",
                     static_cast<int>(r), static_cast<unsigned long long>(dim0),
                     static_cast<unsigned long long>(dim1), static_cast<unsigned long long>(dim2),
                     box0, box1);
  return FKC_OK;
}

namespace {

// fp32 inputs on the tensor cores: x and the centroids are split into bf16
// [hi | lo] rows of 2 Dp elements (Dp = D rounded up to 64; the kernel runs the
// hi.hi, hi.lo and lo.hi K steps, see launch_split_bf16). Up to D = 256 the
// rows fit the bf16 kernel's resident row tile; up to D = 384 x is streamed
// through the centroid stages.
bool split_f32(int64_t D, int dtype) {
  return dtype == FKC_DTYPE_F32 && D >= 16 && D <= 384 && D % 16 == 0;
}

// Shape/dtype eligibility of the tensor-core assignment, independent of the
// device (workspace sizes must not depend on which GPU is current).
bool tc_shape_ok(int64_t D, int dtype) {
  return ((dtype == FKC_DTYPE_F16 || dtype == FKC_DTYPE_BF16) && D >= 16 && D <= 512 &&
          D % 16 == 0) ||
         split_f32(D, dtype);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool use_tc(const void* x, const void* c, int64_t D, int dtype) {
  const bool split = split_f32(D, dtype);
  return tc_shape_ok(D, dtype) && !force_safe_path() && aligned16(x) && aligned16(c) &&
         assign_tc_supported(split ? split_row_elems(D) : D, split ? FKC_DTYPE_BF16 : dtype,
                             split);
}

}  // namespace

bool assign_may_use_tc_host(const void* x, const void* c, int64_t D, int dtype) {
  return tc_shape_ok(D, dtype) && !force_safe_path() && aligned16(x) && aligned16(c);
}

namespace {

// Operand rows of the split-fp32 path: x2 (B, N, 2 Dp) and c2 (B, K, 2 Dp) bf16.
size_t split_bytes(int64_t B, int64_t N, int64_t K, int64_t D, int dtype) {
  if (!split_f32(D, dtype)) return 0;
  const int64_t E = split_row_elems(D);
  return align_up(static_cast<size_t>(B * N * E) * 2, 256) +
         align_up(static_cast<size_t>(B * K * E) * 2, 256);
}

int check_dims(int64_t B, int64_t N, int64_t K, int64_t D, int dtype) {
  FKC_REQUIRE(dtype_valid(dtype), "dtype must be FKC_DTYPE_F16/BF16/F32 (got %d)", dtype);
  FKC_REQUIRE(B >= 1 && N >= 1 && K >= 1 && D >= 1,
              "B, N, K, D must be >= 1 (got B=%lld N=%lld K=%lld D=%lld)",
              static_cast<long long>(B), static_cast<long long>(N), static_cast<long long>(K),
              static_cast<long long>(D));
  FKC_REQUIRE(N <= 2147483647ll && K <= 2147483647ll && D <= 65536,
              "N and K must fit int32 and D <= 65536");
  FKC_REQUIRE(B <= (1ll << 31) / 1 && B * K <= (1ll << 31) - 1,
              "B*K must be < 2^31 (got %lld)", static_cast<long long>(B * K));
  return FKC_OK;
}

cudaStream_t as_stream(fkc_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

size_t assign_ws_bytes(int64_t B, int64_t N, int64_t K, int64_t D, int dtype) {
  if (!tc_shape_ok(D, dtype)) return 0;
  return align_up(static_cast<size_t>(B * N) * 32, 256) +
         align_up(static_cast<size_t>(B * K) * 32, 256) + split_bytes(B, N, K, D, dtype);
}

struct LloydWs {
  uint8_t* aext = nullptr;    // (B,N,16) bf16, tensor-core path
  uint8_t* cext = nullptr;    // (B,K,16) bf16, tensor-core path
  float* c_sq = nullptr;      // (B,K) fp32
  UpdateWorkspace upd{};
  UpdatePlan plan{};          // fused update + finalize (single-GPU iteration)
  LoopCtl* ctl = nullptr;     // whole-loop graph control block
  uint8_t* splitk = nullptr;  // assign_splitk_bytes(), tensor-core path
  uint8_t* x3 = nullptr;      // (B,N,2Dp) bf16 [hi|lo], split-fp32 tensor-core path
  uint8_t* c3 = nullptr;      // (B,K,2Dp) bf16 [hi|lo], split-fp32 tensor-core path
  DetWorkspace det{};         // deterministic update (update_det.cu)
};

constexpr size_t kCtlBytes = 256;

size_t lloyd_ws_bytes(int64_t B, int64_t N, int64_t K, int64_t D, int dtype) {
  return assign_ws_bytes(B, N, K, D, dtype) + align_up(static_cast<size_t>(B * K) * 4, 256) +
         update_workspace_bytes(B, N, K) + update_plan_bytes(B, N, K, D) + kCtlBytes +
         (tc_shape_ok(D, dtype) ? assign_splitk_bytes() : 0) +
         det_update_bytes(B, N, K, D, dtype);
}

int carve_lloyd(void* ws, size_t ws_bytes, int64_t B, int64_t N, int64_t K, int64_t D, int dtype,
                LloydWs* out) {
  const size_t need = lloyd_ws_bytes(B, N, K, D, dtype);
  if (ws == nullptr || ws_bytes < need)
    return set_error(FKC_EWORKSPACE, "Lloyd workspace needs %zu bytes (got %zu at %p)", need,
                     ws_bytes, ws);
  FKC_REQUIRE((reinterpret_cast<uintptr_t>(ws) & 255u) == 0,
              "workspace must be 256-byte aligned");
  // Parts that depend only on (B, K, D, dtype) come first, at the same offsets
  // for every N: ranks holding different numbers of points share the layout
  // of the centroid terms (fkc_lloyd_finalize_multimem writes them remotely).
  uint8_t* p = static_cast<uint8_t*>(ws);
  const bool tc = tc_shape_ok(D, dtype);
  if (tc) {
    out->cext = p;
    p += align_up(static_cast<size_t>(B * K) * 32, 256);
  }
  out->c_sq = reinterpret_cast<float*>(p);
  p += align_up(static_cast<size_t>(B * K) * 4, 256);
  out->ctl = reinterpret_cast<LoopCtl*>(p);
  p += kCtlBytes;
  if (tc) {
    out->splitk = p;
    p += assign_splitk_bytes();
    out->aext = p;
    p += align_up(static_cast<size_t>(B * N) * 32, 256);
    if (split_f32(D, dtype)) {
      const int64_t E = split_row_elems(D);
      out->x3 = p;
      p += align_up(static_cast<size_t>(B * N * E) * 2, 256);
      out->c3 = p;
      p += align_up(static_cast<size_t>(B * K * E) * 2, 256);
    }
  }
  out->upd = carve_update_workspace(p, B, N, K);
  p += update_workspace_bytes(B, N, K);
  out->plan = carve_update_plan(p, B, N, K, D);
  p += update_plan_bytes(B, N, K, D);
  out->det = carve_det(p, B, N, K, D, dtype);
  return FKC_OK;
}

// counts_ready: counts already holds the histogram of `ids` (fkc_lloyd_assign),
// whose labels all lie in [0,K).
// zero_scalar (nullable): one float the scatter also zeroes (the step's shift).
int update_from_ids(const void* x, const int32_t* ids, float* sums, int32_t* counts,
                    bool counts_ready, const UpdateWorkspace& uw, int64_t B, int64_t N,
                    int64_t K, int64_t D, int dtype, cudaStream_t st,
                    float* zero_scalar = nullptr) {
  if (!counts_ready) {
    FKC_TRY(launch_zero_fill(counts, static_cast<size_t>(B * K) * 4, st));
    FKC_TRY(launch_histogram(ids, counts, B, N, K, st));
  }
  UpdateWorkspace w = uw;
  w.zero_scalar = zero_scalar;
  if (aligned16(sums)) {
    // the scatter kernel zeroes sums (no separate fill launch)
    w.zero_f32 = sums;
    w.zero_count = B * K * D;
  }
  FKC_TRY(launch_counting_sort(ids, counts, w, B, N, K, counts_ready, st));
  if (w.zero_f32 == nullptr)
    FKC_TRY(launch_zero_fill(sums, static_cast<size_t>(B * K * D) * 4, st));
  return launch_run_accumulate(x, uw.perm, uw.ids_sorted, sums, nullptr, B, N, K, D, dtype, st);
}

}  // namespace
}  // namespace fkc

using namespace fkc;

extern "C" {

FKC_CAPI_EXPORT int fkc_abi_version(void) { return 1; }

FKC_CAPI_EXPORT uint64_t fkc_kernel_launches(void) { return g_launches.load(); }

FKC_CAPI_EXPORT const char* fkc_last_error(void) { return g_last_error; }

FKC_CAPI_EXPORT const char* fkc_status_string(int status) {
  switch (status) {
    case FKC_OK: return "FKC_OK";
    case FKC_EINVAL: return "FKC_EINVAL";
    case FKC_ECUDA: return "FKC_ECUDA";
    case FKC_EUNSUPPORTED: return "FKC_EUNSUPPORTED";
    case FKC_ETIMEOUT: return "FKC_ETIMEOUT";
    case FKC_EWORKSPACE: return "FKC_EWORKSPACE";
    default: return "FKC_E?";
  }
}

FKC_CAPI_EXPORT int fkc_device_supported(void) {
  const DeviceInfo* di = nullptr;
  if (current_device_info(&di) != FKC_OK) return 0;
  return di->cc_major == 10 ? 1 : 0;
}

FKC_CAPI_EXPORT int fkc_device_status(void) {
  clear_error();
  FKC_CUDA_TRY(cudaDeviceSynchronize());
  int v = 0;
  FKC_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_fkc_device_error, sizeof(int)));
  if (v != 0) {
    const int zero = 0;
    FKC_CUDA_TRY(cudaMemcpyToSymbol(g_fkc_device_error, &zero, sizeof(int)));
    return set_error(FKC_ETIMEOUT, "a device pipeline wait expired (site code %d)", v);
  }
  return FKC_OK;
}

FKC_CAPI_EXPORT size_t fkc_assign_workspace_size(int64_t B, int64_t N, int64_t K, int64_t D,
                                                 int dtype) {
  if (B < 1 || N < 1 || K < 1 || D < 1) return 0;
  return assign_ws_bytes(B, N, K, D, dtype);
}

FKC_CAPI_EXPORT int fkc_assign(const void* x, const void* centroids, const float* x_sq,
                               const float* c_sq, int32_t* ids, int64_t B, int64_t N, int64_t K,
                               int64_t D, int dtype, void* workspace, size_t workspace_bytes,
                               fkc_stream_t stream) {
  clear_error();
  FKC_TRY(check_dims(B, N, K, D, dtype));
  FKC_REQUIRE(x != nullptr && centroids != nullptr && ids != nullptr,
              "x, centroids and cluster_ids must be non-null");
  const cudaStream_t st = as_stream(stream);
  const bool split = split_f32(D, dtype);
  const size_t need = assign_ws_bytes(B, N, K, D, dtype);
  // fp32 callers without room for the split operands keep the CUDA-core kernel
  // (fp32 needed no workspace before the split path existed).
  if (use_tc(x, centroids, D, dtype) &&
      !(split && (workspace == nullptr || workspace_bytes < need))) {
    if (workspace == nullptr || workspace_bytes < need)
      return set_error(FKC_EWORKSPACE, "assign workspace needs %zu bytes (got %zu)", need,
                       workspace_bytes);
    FKC_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255u) == 0,
                "workspace must be 256-byte aligned");
    uint8_t* aext = static_cast<uint8_t*>(workspace);
    uint8_t* cext = aext + align_up(static_cast<size_t>(B * N) * 32, 256);
    FKC_TRY(launch_xnorm_ext(x, aext, B, N, D, dtype, st));
    FKC_TRY(launch_cnorm_ext(centroids, c_sq, cext, nullptr, B, K, D, dtype, st));
    if (split) {
      const int64_t E = split_row_elems(D);
      uint8_t* x3 = cext + align_up(static_cast<size_t>(B * K) * 32, 256);
      uint8_t* c3 = x3 + align_up(static_cast<size_t>(B * N * E) * 2, 256);
      FKC_TRY(launch_split_bf16(x, x3, B * N, D, st));
      FKC_TRY(launch_split_bf16(centroids, c3, B * K, D, st));
      return launch_assign_tc(x3, c3, aext, cext, ids, nullptr, nullptr, B, N, K, E,
                              FKC_DTYPE_BF16, st, static_cast<int>(D));
    }
    return launch_assign_tc(x, centroids, aext, cext, ids, nullptr, nullptr, B, N, K, D, dtype,
                            st);
  }
  return launch_assign_simt(x, centroids, x_sq, c_sq, ids, B, N, K, D, dtype, st);
}

FKC_CAPI_EXPORT int fkc_update_sorted(const void* x_sorted, const int32_t* ids_sorted,
                                      float* sums, int32_t* counts, int64_t B, int64_t N,
                                      int64_t K, int64_t D, int dtype, fkc_stream_t stream) {
  clear_error();
  FKC_TRY(check_dims(B, N, K, D, dtype));
  FKC_REQUIRE(x_sorted && ids_sorted && sums && counts, "null argument");
  return launch_run_accumulate(x_sorted, nullptr, ids_sorted, sums, counts, B, N, K, D, dtype,
                               as_stream(stream));
}

FKC_CAPI_EXPORT int fkc_update_sorted_indexed(const void* x, const int32_t* sorted_idx,
                                              const int32_t* ids_sorted, float* sums,
                                              int32_t* counts, int64_t B, int64_t N, int64_t K,
                                              int64_t D, int dtype, fkc_stream_t stream) {
  clear_error();
  FKC_TRY(check_dims(B, N, K, D, dtype));
  FKC_REQUIRE(x && sorted_idx && ids_sorted && sums && counts, "null argument");
  return launch_run_accumulate(x, sorted_idx, ids_sorted, sums, counts, B, N, K, D, dtype,
                               as_stream(stream));
}

FKC_CAPI_EXPORT size_t fkc_update_workspace_size(int64_t B, int64_t N, int64_t K) {
  if (B < 1 || N < 1 || K < 1) return 0;
  return update_workspace_bytes(B, N, K);
}

FKC_CAPI_EXPORT int fkc_update(const void* x, const int32_t* ids, float* sums, int32_t* counts,
                               int64_t B, int64_t N, int64_t K, int64_t D, int dtype,
                               void* workspace, size_t workspace_bytes, fkc_stream_t stream) {
  clear_error();
  FKC_TRY(check_dims(B, N, K, D, dtype));
  FKC_REQUIRE(x && ids && sums && counts, "null argument");
  const size_t need = update_workspace_bytes(B, N, K);
  if (workspace == nullptr || workspace_bytes < need)
    return set_error(FKC_EWORKSPACE, "update workspace needs %zu bytes (got %zu)", need,
                     workspace_bytes);
  const UpdateWorkspace uw = carve_update_workspace(workspace, B, N, K);
  return update_from_ids(x, ids, sums, counts, false, uw, B, N, K, D, dtype, as_stream(stream));
}

FKC_CAPI_EXPORT int fkc_finalize(const float* sums, const int32_t* counts, const void* old_c,
                                 void* new_c, float* c_sq_out, float* shift_out, int64_t B,
                                 int64_t K, int64_t D, int dtype, fkc_stream_t stream) {
  clear_error();
  FKC_TRY(check_dims(B, 1, K, D, dtype));
  FKC_REQUIRE(sums && counts && old_c && new_c, "null argument");
  return launch_finalize(sums, counts, old_c, new_c, c_sq_out, nullptr, shift_out, B, K, D,
                         dtype, as_stream(stream));
}

FKC_CAPI_EXPORT size_t fkc_lloyd_workspace_size(int64_t B, int64_t N, int64_t K, int64_t D,
                                                int dtype) {
  if (B < 1 || N < 1 || K < 1 || D < 1) return 0;
  return lloyd_ws_bytes(B, N, K, D, dtype);
}

FKC_CAPI_EXPORT int fkc_lloyd_prepare(const void* x, int64_t B, int64_t N, int64_t K, int64_t D,
                                      int dtype, void* workspace, size_t workspace_bytes,
                                      fkc_stream_t stream) {
  clear_error();
  FKC_TRY(check_dims(B, N, K, D, dtype));
  FKC_REQUIRE(x != nullptr, "x must be non-null");
  LloydWs w;
  FKC_TRY(carve_lloyd(workspace, workspace_bytes, B, N, K, D, dtype, &w));
  // The fused update's per-cluster accumulators start (and stay) zero.
  FKC_TRY(launch_zero_fill(w.plan.done, w.plan.zero_bytes, as_stream(stream)));
  if (w.aext != nullptr) FKC_TRY(launch_xnorm_ext(x, w.aext, B, N, D, dtype, as_stream(stream)));
  if (w.x3 != nullptr) FKC_TRY(launch_split_bf16(x, w.x3, B * N, D, as_stream(stream)));
  return FKC_OK;
}

FKC_CAPI_EXPORT int fkc_lloyd_set_centroids(const void* centroids, int64_t B, int64_t N,
                                            int64_t K, int64_t D, int dtype, void* workspace,
                                            size_t workspace_bytes, fkc_stream_t stream) {
  clear_error();
  FKC_TRY(check_dims(B, N, K, D, dtype));
  FKC_REQUIRE(centroids != nullptr, "centroids must be non-null");
  LloydWs w;
  FKC_TRY(carve_lloyd(workspace, workspace_bytes, B, N, K, D, dtype, &w));
  return launch_cnorm_ext(centroids, nullptr, w.cext, w.c_sq, B, K, D, dtype, as_stream(stream));
}

FKC_CAPI_EXPORT int fkc_lloyd_assign(const void* x, const void* centroids, int32_t* ids,
                                     int32_t* counts, int64_t B, int64_t N, int64_t K, int64_t D,
                                     int dtype, void* workspace, size_t workspace_bytes,
                                     fkc_stream_t stream) {
  clear_error();
  FKC_TRY(check_dims(B, N, K, D, dtype));
  FKC_REQUIRE(x && centroids && ids && counts, "null argument");
  LloydWs w;
  FKC_TRY(carve_lloyd(workspace, workspace_bytes, B, N, K, D, dtype, &w));
  const cudaStream_t st = as_stream(stream);
  FKC_TRY(launch_zero_fill(counts, static_cast<size_t>(B * K) * 4, st));
  if (w.aext != nullptr && use_tc(x, centroids, D, dtype)) {
    if (w.x3 != nullptr) {
      // fp32: this iteration's centroids as split bf16 rows (x3: prepare).
      FKC_TRY(launch_split_bf16(centroids, w.c3, B * K, D, st));
      return launch_assign_tc(w.x3, w.c3, w.aext, w.cext, ids, counts, w.splitk, B, N, K,
                              split_row_elems(D), FKC_DTYPE_BF16, st, static_cast<int>(D));
    }
    return launch_assign_tc(x, centroids, w.aext, w.cext, ids, counts, w.splitk, B, N, K, D,
                            dtype, st);
  }
  FKC_TRY(launch_assign_simt(x, centroids, nullptr, w.c_sq, ids, B, N, K, D, dtype, st));
  return launch_histogram(ids, counts, B, N, K, st);
}

FKC_CAPI_EXPORT int fkc_lloyd_update(const void* x, const int32_t* ids, const int32_t* counts,
                                     float* sums, int64_t B, int64_t N, int64_t K, int64_t D,
                                     int dtype, void* workspace, size_t workspace_bytes,
                                     fkc_stream_t stream) {
  clear_error();
  FKC_TRY(check_dims(B, N, K, D, dtype));
  FKC_REQUIRE(x && ids && counts && sums, "null argument");
  LloydWs w;
  FKC_TRY(carve_lloyd(workspace, workspace_bytes, B, N, K, D, dtype, &w));
  if (deterministic_update() && det_update_ok(w.det, x, sums, nullptr, nullptr, N, K, D, dtype))
    return launch_det_update(x, ids, counts, w.upd, w.det, sums, nullptr, nullptr, nullptr,
                             nullptr, nullptr, B, N, K, D, dtype, as_stream(stream));
  return update_from_ids(x, ids, sums, const_cast<int32_t*>(counts), true, w.upd, B, N, K, D,
                         dtype, as_stream(stream));
}

FKC_CAPI_EXPORT int fkc_lloyd_local(const void* x, const void* centroids, int32_t* ids,
                                    float* sums, int32_t* counts, int64_t B, int64_t N,
                                    int64_t K, int64_t D, int dtype, void* workspace,
                                    size_t workspace_bytes, fkc_stream_t stream) {
  FKC_TRY(fkc_lloyd_assign(x, centroids, ids, counts, B, N, K, D, dtype, workspace,
                           workspace_bytes, stream));
  return fkc_lloyd_update(x, ids, counts, sums, B, N, K, D, dtype, workspace, workspace_bytes,
                          stream);
}

FKC_CAPI_EXPORT int fkc_lloyd_finalize(const float* sums, const int32_t* counts,
                                       const void* old_c, void* new_c, float* shift_out,
                                       int64_t B, int64_t N, int64_t K, int64_t D, int dtype,
                                       void* workspace, size_t workspace_bytes,
                                       fkc_stream_t stream) {
  clear_error();
  FKC_TRY(check_dims(B, N, K, D, dtype));
  FKC_REQUIRE(sums && counts && old_c && new_c, "null argument");
  LloydWs w;
  FKC_TRY(carve_lloyd(workspace, workspace_bytes, B, N, K, D, dtype, &w));
  return launch_finalize(sums, counts, old_c, new_c, w.c_sq, w.cext, shift_out, B, K, D, dtype,
                         as_stream(stream));
}

FKC_CAPI_EXPORT int fkc_lloyd_iter(const void* x, const void* old_c, void* new_c, int32_t* ids,
                                   float* sums, int32_t* counts, float* shift_out, int64_t B,
                                   int64_t N, int64_t K, int64_t D, int dtype, void* workspace,
                                   size_t workspace_bytes, fkc_stream_t stream) {
  {
    // Deterministic path: assign -> stable counting sort -> span gather -> join +
    // finalize (every float addition in an order fixed by the labels).
    LloydWs w;
    if (deterministic_update() && old_c != nullptr && new_c != nullptr &&
        carve_lloyd(workspace, workspace_bytes, B, N, K, D, dtype, &w) == FKC_OK &&
        det_update_ok(w.det, x, sums, old_c, new_c, N, K, D, dtype)) {
      FKC_TRY(fkc_lloyd_assign(x, old_c, ids, counts, B, N, K, D, dtype, workspace,
                               workspace_bytes, stream));
      return launch_det_update(x, ids, counts, w.upd, w.det, sums, old_c, new_c, w.c_sq, w.cext,
                               shift_out, B, N, K, D, dtype, as_stream(stream));
    }
    clear_error();
  }
  if (x != nullptr && old_c != nullptr && new_c != nullptr && sums != nullptr &&
      N <= 32 * K && fused_update_ok(x, old_c, new_c, sums, D, dtype)) {
    // Single GPU, small clusters (at most 32 rows on average): the update and
    // the finalize are one pass over the clusters, with no sums zero-fill and
    // no atomics on whole clusters. Measured on B200: c4 (16 rows per cluster)
    // 160-179 -> 136-148 us per iteration; with 64 rows per cluster the
    // position-balanced accumulator + finalize stays faster (c3 0.899 vs 0.921
    // ms, c2 88.5 vs 93.4 us), its spans keep more rows in flight per warp.
    FKC_TRY(fkc_lloyd_assign(x, old_c, ids, counts, B, N, K, D, dtype, workspace,
                             workspace_bytes, stream));
    LloydWs w;
    FKC_TRY(carve_lloyd(workspace, workspace_bytes, B, N, K, D, dtype, &w));
    return launch_update_finalize(x, ids, counts, w.upd, w.plan, old_c, new_c, sums, w.c_sq,
                                  w.cext, shift_out, B, N, K, D, dtype, as_stream(stream));
  }
  // assign -> counting sort + accumulate (the scatter also zeroes the shift)
  // -> finalize
  FKC_TRY(fkc_lloyd_assign(x, old_c, ids, counts, B, N, K, D, dtype, workspace, workspace_bytes,
                           stream));
  FKC_REQUIRE(old_c && new_c && sums, "null argument");
  LloydWs w;
  FKC_TRY(carve_lloyd(workspace, workspace_bytes, B, N, K, D, dtype, &w));
  const cudaStream_t st = as_stream(stream);
  FKC_TRY(update_from_ids(x, ids, sums, counts, true, w.upd, B, N, K, D, dtype, st, shift_out));
  return launch_finalize(sums, counts, old_c, new_c, w.c_sq, w.cext, shift_out, B, K, D, dtype,
                         st, /*shift_zeroed=*/shift_out != nullptr);
}

FKC_CAPI_EXPORT int fkc_lloyd_finalize_multimem(
    const float* mc_sums, const int32_t* mc_counts, const void* centroids, void* mc_centroids,
    void* mc_workspace, unsigned int* mc_shift, float* shift_clear, int64_t row_begin,
    int64_t row_end, int64_t B, int64_t K, int64_t D, int dtype, fkc_stream_t stream) {
  clear_error();
  FKC_TRY(check_dims(B, 1, K, D, dtype));
  FKC_REQUIRE(mc_sums && mc_counts && centroids && mc_centroids && mc_workspace,
              "null argument");
  FKC_REQUIRE(row_begin >= 0 && row_begin <= row_end && row_end <= B * K,
              "rows [%lld, %lld) outside [0, B*K=%lld)", static_cast<long long>(row_begin),
              static_cast<long long>(row_end), static_cast<long long>(B * K));
  // The centroid terms sit at offsets that do not depend on N.
  LloydWs w;
  FKC_TRY(carve_lloyd(mc_workspace, lloyd_ws_bytes(B, 1, K, D, dtype), B, 1, K, D, dtype, &w));
  if (row_begin == row_end) {
    if (shift_clear != nullptr)
      FKC_CUDA_TRY(cudaMemsetAsync(shift_clear, 0, sizeof(float), as_stream(stream)));
    return FKC_OK;
  }
  return launch_finalize_multimem(mc_sums, mc_counts, centroids, mc_centroids, w.c_sq, w.cext,
                                  mc_shift, shift_clear, row_begin, row_end, D, dtype,
                                  as_stream(stream));
}

FKC_CAPI_EXPORT int fkc_lloyd_finalize_multimem_synced(
    const float* mc_sums, const int32_t* mc_counts, const void* centroids, void* mc_centroids,
    void* mc_workspace, unsigned int* mc_shift, float* shift_clear, int64_t row_begin,
    int64_t row_end, int64_t B, int64_t K, int64_t D, int dtype, unsigned int* bar,
    unsigned int* mc_bar, uint32_t epoch, int world, fkc_stream_t stream) {
  clear_error();
  FKC_TRY(check_dims(B, 1, K, D, dtype));
  FKC_REQUIRE(mc_sums && mc_counts && centroids && mc_centroids && mc_workspace && bar && mc_bar,
              "null argument");
  FKC_REQUIRE(world >= 1 && epoch >= 1, "world (%d) and epoch (%u) must be >= 1", world, epoch);
  FKC_REQUIRE(row_begin >= 0 && row_begin < row_end && row_end <= B * K,
              "rows [%lld, %lld) must be a non-empty part of [0, B*K=%lld)",
              static_cast<long long>(row_begin), static_cast<long long>(row_end),
              static_cast<long long>(B * K));
  FKC_REQUIRE((reinterpret_cast<uintptr_t>(bar) & 3u) == 0 &&
                  (reinterpret_cast<uintptr_t>(mc_bar) & 3u) == 0,
              "barrier words must be 4-byte aligned");
  LloydWs w;
  FKC_TRY(carve_lloyd(mc_workspace, lloyd_ws_bytes(B, 1, K, D, dtype), B, 1, K, D, dtype, &w));
  return launch_finalize_multimem(mc_sums, mc_counts, centroids, mc_centroids, w.c_sq, w.cext,
                                  mc_shift, shift_clear, row_begin, row_end, D, dtype,
                                  as_stream(stream), bar, mc_bar,
                                  epoch * static_cast<uint32_t>(world));
}

FKC_CAPI_EXPORT int fkc_multimem_step_wait(const unsigned int* bar, uint32_t epoch, int world,
                                           fkc_stream_t stream) {
  clear_error();
  FKC_REQUIRE(bar != nullptr && world >= 1, "bar must be non-null and world >= 1");
  return launch_step_wait(bar, epoch * static_cast<uint32_t>(world), as_stream(stream));
}

FKC_CAPI_EXPORT int fkc_lloyd_run(const void* x, void* centroids, int32_t* ids, float* sums,
                                  int32_t* counts, float* shift, int32_t* n_iters, int max_iters,
                                  float tol, int64_t B, int64_t N, int64_t K, int64_t D,
                                  int dtype, void* workspace, size_t workspace_bytes,
                                  fkc_stream_t stream) {
  clear_error();
  FKC_TRY(check_dims(B, N, K, D, dtype));
  FKC_REQUIRE(x && centroids && ids && sums && counts && shift, "null argument");
  FKC_REQUIRE(max_iters >= 0, "max_iters must be >= 0 (got %d)", max_iters);
  LloydWs w;
  FKC_TRY(carve_lloyd(workspace, workspace_bytes, B, N, K, D, dtype, &w));
  const cudaStream_t st = as_stream(stream);
  // Centroid terms of the initial centroids (later iterations: finalize), and
  // the fused update's accumulators back to zero in case an earlier call on
  // this workspace stopped part-way.
  FKC_TRY(launch_cnorm_ext(centroids, nullptr, w.cext, w.c_sq, B, K, D, dtype, st));
  FKC_TRY(launch_zero_fill(w.plan.done, w.plan.zero_bytes, st));
  if (max_iters == 0) {
    if (n_iters != nullptr) FKC_CUDA_TRY(cudaMemsetAsync(n_iters, 0, sizeof(int32_t), st));
    return FKC_OK;
  }
  int dev = 0;
  FKC_CUDA_TRY(cudaGetDevice(&dev));
  LloydGraphKey key;
  std::memset(&key, 0, sizeof(key));
  key.device = dev;
  key.dtype = dtype;
  key.x = x;
  key.centroids = centroids;
  key.ids = ids;
  key.sums = sums;
  key.counts = counts;
  key.shift = shift;
  key.workspace = workspace;
  key.B = B;
  key.N = N;
  key.K = K;
  key.D = D;
  // One in-place iteration: finalize reads each old centroid element before
  // writing the new one, and the next assign reads the updated centroids.
  const LoopBody body = [&](cudaStream_t cs) -> int {
    return fkc_lloyd_iter(x, centroids, centroids, ids, sums, counts, shift, B, N, K, D, dtype,
                          workspace, workspace_bytes, reinterpret_cast<fkc_stream_t>(cs));
  };
  return run_lloyd_graph(key, body, w.ctl, shift, max_iters, tol, n_iters, st);
}

}  // extern "C"
