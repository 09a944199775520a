// Host-side internals shared by the translation units of libfkc_b200.so:
// status/error reporting, per-device properties, TMA descriptor encoding and
// the launcher entry points the C-ABI dispatches to.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <functional>
#include <cstdio>
#include <string>

#include "fkc_capi.h"  // include/ is on the include path

namespace fkc {

// Records a formatted message for fkc_last_error() and returns `status`.
int set_error(int status, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
void clear_error();

#define FKC_REQUIRE(cond, ...)                                                  \
  do {                                                                          \
    if (!(cond)) return ::fkc::set_error(FKC_EINVAL, __VA_ARGS__);              \
  } while (0)

#define FKC_CUDA_TRY(expr)                                                      \
  do {                                                                          \
    cudaError_t fkc_e_ = (expr);                                                \
    if (fkc_e_ != cudaSuccess)                                                  \
      return ::fkc::set_error(FKC_ECUDA, "%s failed: %s (%s:%d)", #expr,        \
                              cudaGetErrorString(fkc_e_), __FILE__, __LINE__); \
  } while (0)

#define FKC_TRY(expr)                                                           \
  do {                                                                          \
    int fkc_s_ = (expr);                                                        \
    if (fkc_s_ != FKC_OK) return fkc_s_;                                        \
  } while (0)

struct DeviceInfo {
  int device = -1;
  int sm_count = 0;
  int cc_major = 0;
  int cc_minor = 0;
  size_t smem_optin = 0;
};

// Cached per device (queried once; the reference re-queried on every call).
int current_device_info(const DeviceInfo** out);

// 3-D tiled tensor map {dim0 (contiguous), dim1, dim2} for a row-major array.
int encode_tmap_3d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base,
                   uint64_t dim0, uint64_t dim1, uint64_t dim2, uint64_t stride1_bytes,
                   uint64_t stride2_bytes, uint32_t box0, uint32_t box1,
                   CUtensorMapSwizzle swizzle);

inline size_t dtype_size(int dtype) { return dtype == FKC_DTYPE_F32 ? 4 : 2; }
inline bool dtype_valid(int dtype) {
  return dtype == FKC_DTYPE_F16 || dtype == FKC_DTYPE_BF16 || dtype == FKC_DTYPE_F32;
}
inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Device-resident error word written by kernels whose bounded waits expired.
int* device_error_word();

// Counts kernels launched by this library (reported by fkc_kernel_launches()).
void count_launches(int n);

// ----------------------------------------------------------------------------
// Launchers (each validates what is specific to it and launches on `stream`).
// ----------------------------------------------------------------------------

// True when the tcgen05 assignment kernel handles this shape/dtype on the
// current device.
// split_rows: D is the width of split fp32 rows (launch_split_bf16), which
// may exceed the 16-bit limit (x is then streamed through the stages).
bool assign_tc_supported(int64_t D, int dtype, bool split_rows = false);
// The host-only part of fkc_assign's route choice (no CUDA call): false when
// the call certainly takes the CUDA-core kernel, which needs no workspace
// (shape/dtype outside the tensor-core path, FKC_ASSIGN_FORCE_SAFE=1, or x /
// centroids not 16-byte aligned).
bool assign_may_use_tc_host(const void* x, const void* c, int64_t D, int dtype);

// Row-norm extension rows for the tcgen05 path: aext[b,n,:] = {h1,h2,h3,1,1,1,0...}
// with h1+h2+h3 = -0.5*||x[b,n]||^2 split over three bf16 values.
int launch_xnorm_ext(const void* x, void* aext, int64_t B, int64_t N, int64_t D, int dtype,
                     cudaStream_t stream);
// Centroid terms: extension rows cext[b,k,:] = {1,1,1,h1,h2,h3,0...} with
// h = -0.5*c_sq (cext nullable) and/or c_sq_out[b,k] (nullable). c_sq is taken
// from `c_sq` when non-null, otherwise computed from the centroids.
// fp32 rows (rows x D) -> bf16 rows (rows x 2 Dp, Dp = D rounded up to 64):
// [hi | 0 | lo | 0] with hi = bf16(v), lo = bf16(v - hi). The tensor-core
// assignment accumulates hi.hi + hi.lo + lo.hi (three passes), the fp32 dot
// product to ~2^-16 |x||c|.
int64_t split_row_elems(int64_t D);  // 2 * Dp
int launch_split_bf16(const void* src, void* dst, int64_t rows, int64_t D, cudaStream_t stream);
int launch_cnorm_ext(const void* centroids, const float* c_sq, void* cext, float* c_sq_out,
                     int64_t B, int64_t K, int64_t D, int dtype, cudaStream_t stream);

// splitk_ws (nullable, assign_splitk_bytes()): lets the kernel balance an
// uneven last wave by sharing tiles between CTAs (merged by a fixup kernel).
// split_d > 0: x and centroids are split fp32 rows (launch_split_bf16) of
// D = split_row_elems(split_d) bf16 elements.
int launch_assign_tc(const void* x, const void* centroids, const void* aext, const void* cext,
                     int32_t* ids, int32_t* counts, void* splitk_ws, int64_t B, int64_t N,
                     int64_t K, int64_t D, int dtype, cudaStream_t stream, int split_d = 0);
size_t assign_splitk_bytes();

int launch_assign_simt(const void* x, const void* centroids, const float* x_sq,
                       const float* c_sq, int32_t* ids, int64_t B, int64_t N, int64_t K,
                       int64_t D, int dtype, cudaStream_t stream);

// Update: counting sort of labels + permutation-driven gather-accumulate.
struct UpdateWorkspace {
  int32_t* offsets;     // (B, K) exclusive prefix of counts
  int32_t* cursor;      // (B, K) scatter cursors
  int32_t* perm;        // (B, N) row index in cluster order
  int32_t* ids_sorted;  // (B, N) label in cluster order; follows perm directly (the
                        // deterministic update stores (row, label) pairs over both)
  // Optional: zero_count floats at zero_f32 (16-byte aligned) are zeroed by the
  // scatter kernel after its dependency wait (saves a separate fill launch).
  float* zero_f32 = nullptr;
  int64_t zero_count = 0;
  float* zero_scalar = nullptr;  // one float zeroed likewise (the shift of the step)
};
size_t update_workspace_bytes(int64_t B, int64_t N, int64_t K);
UpdateWorkspace carve_update_workspace(void* ws, int64_t B, int64_t N, int64_t K);

// counts += histogram of the labels of ids that lie in [0,K).
int launch_histogram(const int32_t* ids, int32_t* counts, int64_t B, int64_t N, int64_t K,
                     cudaStream_t stream);
// offsets = exclusive scan of counts (which must be the histogram of ids), then
// perm/ids_sorted. all_valid: every label lies in [0,K), so every sorted
// position is written; otherwise unwritten positions read as label -1.
int launch_counting_sort(const int32_t* ids, const int32_t* counts, const UpdateWorkspace& w,
                         int64_t B, int64_t N, int64_t K, bool all_valid, cudaStream_t stream);
// sums[b, ids_sorted[i], :] += x[b, perm ? perm[i] : i, :] over sorted runs.
// counts (nullable) += run lengths. sums/counts must be initialised by the caller.
int launch_run_accumulate(const void* x, const int32_t* perm, const int32_t* ids_sorted,
                          float* sums, int32_t* counts, int64_t B, int64_t N, int64_t K,
                          int64_t D, int dtype, cudaStream_t stream);

// Fused update + finalize of the single-GPU Lloyd step (update.cu): clusters
// of more than 64 rows are cut into units that add into a per-cluster row of
// acc; the last unit of the cluster finishes it. done and acc are zero between
// passes (zero_bytes from done on are zeroed when the workspace is prepared).
struct UpdatePlan {
  int2* extras;          // (B, cap) (cluster b*K+k, chunk) of the split clusters' units
  int32_t* extra_count;  // (B) entries used in each row of extras
  int32_t* done;         // (B, K) finished units of each split cluster
  float* acc;            // (B, K, D) sums of split clusters being accumulated
  int cap;
  size_t zero_bytes;     // done .. end of acc
};
size_t update_plan_bytes(int64_t B, int64_t N, int64_t K, int64_t D);
UpdatePlan carve_update_plan(void* ws, int64_t B, int64_t N, int64_t K, int64_t D);
// Rows of whole 16-byte vectors (at most 32 per row) and 16-byte aligned buffers.
bool fused_update_ok(const void* x, const void* old_c, const void* new_c, const float* sums,
                     int64_t D, int dtype);
// counts: the histogram of ids (labels all in [0,K)). Writes sums, new_c,
// c_sq/cext (nullable) of new_c and shift (nullable) = max ||new - old||.
int launch_update_finalize(const void* x, const int32_t* ids, const int32_t* counts,
                           const UpdateWorkspace& w, const UpdatePlan& plan, const void* old_c,
                           void* new_c, float* sums, float* c_sq, void* cext, float* shift,
                           int64_t B, int64_t N, int64_t K, int64_t D, int dtype,
                           cudaStream_t stream);

// Deterministic update of the Lloyd step (update_det.cu): stable counting sort
// (per-chunk ranks, chunk bases, scatter), span gather and a fixed-order join of
// the clusters split between spans, the finalize fused into the last kernel.
// Labels must lie in [0, K); K <= 65536; rows of 64..512 bytes, 16-byte aligned.
struct DetWorkspace {
  uint16_t* rank = nullptr;  // (B, N) stable rank of each row inside its chunk
  int32_t* hist = nullptr;   // (B, C, K) chunk histograms, then chunk slot bases
  float* part = nullptr;     // (spans, 2, D) partial sums of clusters cut by span ends
};
// 0 when the shape is outside the deterministic path.
size_t det_update_bytes(int64_t B, int64_t N, int64_t K, int64_t D, int dtype);
DetWorkspace carve_det(void* ws, int64_t B, int64_t N, int64_t K, int64_t D, int dtype);
bool det_update_ok(const DetWorkspace& dw, const void* x, const float* sums, const void* old_c,
                   const void* new_c, int64_t N, int64_t K, int64_t D, int dtype);
// counts: the histogram of ids. Writes offsets/perm/ids_sorted (uw), every row of
// sums and, when old_c is non-null, new_c (may alias old_c), c_sq / cext
// (nullable) of new_c and shift (nullable, zeroed here first).
int launch_det_update(const void* x, const int32_t* ids, const int32_t* counts,
                      const UpdateWorkspace& uw, const DetWorkspace& dw, float* sums,
                      const void* old_c, void* new_c, float* c_sq, void* cext, float* shift,
                      int64_t B, int64_t N, int64_t K, int64_t D, int dtype,
                      cudaStream_t stream);

// Whole-loop CUDA graph (lloyd_graph.cu).
struct LoopCtl {
  int32_t iter;       // iterations completed in the current launch
  int32_t max_iters;
  float tol;          // stop when the shift falls below tol (tol > 0)
  int32_t n_iters;    // iterations run (read after the launch)
};
// Identifies the buffers and shape a cached graph was captured for. Built
// with memset(0) so that padding compares equal.
struct LloydGraphKey {
  int device;
  int dtype;
  const void* x;
  void* centroids;
  int32_t* ids;
  float* sums;
  int32_t* counts;
  float* shift;
  void* workspace;
  int64_t B, N, K, D;
};
using LoopBody = std::function<int(cudaStream_t)>;
// Launches (building and caching on first use) WHILE { body; control } with
// at most max_iters iterations; writes the iterations run to n_iters_out
// (device, nullable). ctl: device control block; shift: the body's shift.
int run_lloyd_graph(const LloydGraphKey& key, const LoopBody& body, LoopCtl* ctl,
                    const float* shift, int max_iters, float tol, int32_t* n_iters_out,
                    cudaStream_t stream);
// True (and the launches recorded for the graph) while this thread captures.
bool count_captured_launch(int n);
uint64_t capture_launch_count();

// Rows [row0, row1) of the multi-GPU finalize over NVLink multicast (mc_*:
// multicast addresses of symmetric buffers; old_c: this rank's copy).
// bar (nullable): this rank's copy of the step's barrier words, mc_bar their
// multicast address, target = epoch * world (see finalize.cu).
int launch_finalize_multimem(const float* mc_sums, const int32_t* mc_counts, const void* old_c,
                             void* mc_new_c, float* mc_c_sq, void* mc_cext,
                             unsigned int* mc_shift, float* shift_clear, int64_t row0,
                             int64_t row1, int64_t D, int dtype, cudaStream_t stream,
                             unsigned int* bar = nullptr, unsigned int* mc_bar = nullptr,
                             unsigned target = 0);
// Bounded wait until bar[1] (ranks whose synced finalize completed) reaches target.
int launch_step_wait(const unsigned int* bar, unsigned target, cudaStream_t stream);

// shift_zeroed: *shift_out is already 0 (the scatter of this step zeroed it).
int launch_finalize(const float* sums, const int32_t* counts, const void* old_c, void* new_c,
                    float* c_sq_out, void* cext_out, float* shift_out, int64_t B, int64_t K,
                    int64_t D, int dtype, cudaStream_t stream, bool shift_zeroed = false);

}  // namespace fkc
