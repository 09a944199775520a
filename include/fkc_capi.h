/*
 * fkc_capi.h - C-ABI of libfkc_b200.so, the B200 (sm_100a) implementation of
 * the batched Euclidean K-Means Lloyd iteration of flash-kmeans-cuda.
 *
 * Plain pointers and sizes only: no torch or C++ types cross this boundary.
 * Every entry point
 *   - validates its arguments on the host and returns FKC_OK (0) or a
 *     negative FKC_E* status; fkc_last_error() then returns a message for the
 *     calling thread (the counterpart of the reference's TORCH_CHECK text);
 *   - launches asynchronously on `stream` (a cudaStream_t; NULL = legacy
 *     default stream) on the CURRENT CUDA device, and never synchronises;
 *   - takes device pointers; dense row-major layouts as documented per call.
 *
 * Element types: FKC_DTYPE_F16 / FKC_DTYPE_BF16 / FKC_DTYPE_F32 select the
 * type of x and of the centroids. Sums are always fp32, labels and counts
 * int32, as in the reference.
 *
 * Reference interfaces replaced (paths inside OpsiClear/flash-kmeans-cuda):
 *   flash_kmeans_cuda/csrc/bindings.cpp:43-102  (_C.euclid_assign, _C.centroid_update_sorted,
 *                                                _C.centroid_update_sorted_indexed,
 *                                                _C.centroid_finalize)
 *   flash_kmeans_cuda/csrc/api.cpp:47-113       (fkc:: libtorch API)
 *   flash_kmeans_cuda/csrc/assign/assign.h:32-44, csrc/update/update.h:28-63 (launchers)
 *   flash_kmeans_cuda/ops.py:58-112, kmeans.py:73-105 (sort/route and iteration glue)
 */
#ifndef FKC_CAPI_H_
#define FKC_CAPI_H_

#include <stddef.h>
#include <stdint.h>

#if defined(_WIN32)
#define FKC_CAPI_EXPORT __declspec(dllexport)
#else
#define FKC_CAPI_EXPORT __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Same type as cudaStream_t; declared here so the header needs no CUDA include. */
typedef struct CUstream_st* fkc_stream_t;

enum {
  FKC_OK = 0,
  FKC_EINVAL = -1,        /* bad argument: shape, dtype, null or misaligned pointer */
  FKC_ECUDA = -2,         /* CUDA runtime/driver call failed (launch, attribute, tensor map) */
  FKC_EUNSUPPORTED = -3,  /* no CUDA device / device is not sm_100 */
  FKC_ETIMEOUT = -4,      /* a bounded device-side pipeline wait expired (see fkc_device_status) */
  FKC_EWORKSPACE = -5     /* workspace missing or smaller than *_workspace_size() */
};

enum { FKC_DTYPE_F16 = 0, FKC_DTYPE_BF16 = 1, FKC_DTYPE_F32 = 2 };

/* ABI revision of this header (bumped on incompatible change). */
FKC_CAPI_EXPORT int fkc_abi_version(void);

/* Message describing the last failing call on this thread ("" if none). */
FKC_CAPI_EXPORT const char* fkc_last_error(void);

/* Name of a status code. */
FKC_CAPI_EXPORT const char* fkc_status_string(int status);

/* 1 when the current device runs the tcgen05 kernels (sm_100), else 0. */
FKC_CAPI_EXPORT int fkc_device_supported(void);

/* Number of CUDA kernels this library has launched in this process. */
FKC_CAPI_EXPORT uint64_t fkc_kernel_launches(void);

/* Synchronises the current device and returns FKC_OK, or FKC_ETIMEOUT if a
 * kernel of this library recorded an expired pipeline wait since the last
 * call (the record is cleared). Use in tests and health checks. */
FKC_CAPI_EXPORT int fkc_device_status(void);

/* Test of the device-side failure path, without a fault: launches a one-warp
 * kernel whose bounded mbarrier wait (the wait the assignment pipeline uses)
 * can never complete. After timeout_us (1 .. 10^7) it gives up, records site
 * code 199 in the device error word and returns, so the next
 * fkc_device_status() returns FKC_ETIMEOUT and the context stays usable.
 * No counterpart in the reference. */
FKC_CAPI_EXPORT int fkc_selftest_wait_timeout(uint32_t timeout_us, fkc_stream_t stream);

/* ------------------------------------------------------------------------
 * Assignment
 *   ids[b,n] = argmin_k ||x[b,n,:] - c[b,k,:]||^2, ties -> lowest k.
 *   x (B,N,D), centroids (B,K,D) of `dtype`; ids (B,N) int32.
 *   c_sq (B,K) fp32 = ||c||^2 or NULL (computed). x_sq (B,N) fp32 or NULL:
 *   read only by the fp32 / odd-D fallback, which clamps distances at 0 as
 *   the reference's safe kernel does; the tensor-core path ignores it (as the
 *   reference's raw-distance mma path does).
 *   fp16/bf16 with D % 16 == 0 and D <= 512 run the tcgen05 kernel; so does
 *   fp32 with D % 16 == 0 and D <= 384 (x and c as split bf16 rows [hi | lo]
 *   of 2 Dp elements, Dp = D rounded up to 64; the kernel accumulates hi.hi +
 *   hi.lo + lo.hi, ~2^-16 relative), when the workspace holds those rows
 *   (fkc_assign_workspace_size counts them); fp32 with a smaller or no
 *   workspace keeps the CUDA-core kernel.
 * Replaces: _C.euclid_assign (csrc/bindings.cpp:43-71),
 *           fkc::euclid_assign_out (csrc/api.cpp:58-72),
 *           launch_assign_sm80 / launch_assign_safe (csrc/assign/assign.h:32-44).
 * ---------------------------------------------------------------------- */
FKC_CAPI_EXPORT size_t fkc_assign_workspace_size(int64_t B, int64_t N, int64_t K, int64_t D,
                                                 int dtype);
FKC_CAPI_EXPORT int fkc_assign(const void* x, const void* centroids, const float* x_sq,
                               const float* c_sq, int32_t* ids, int64_t B, int64_t N, int64_t K,
                               int64_t D, int dtype, void* workspace, size_t workspace_bytes,
                               fkc_stream_t stream);

/* ------------------------------------------------------------------------
 * Assignment without a workspace and without device allocation. No
 * counterpart in the reference (which allocates through torch); added for
 * callers that cannot allocate device memory: FFI bindings of the 5-argument
 * euclid_assign signature that only receive device pointers, hosts whose
 * device memory a pooling allocator has reserved, and latency-critical
 * pipelines that cannot take cudaFree's device-wide synchronisation.
 *   Same arguments, results and errors as fkc_assign minus the workspace.
 *   Scratch: a static device array of FKC_ASSIGN_NOALLOC_SCRATCH_BYTES per
 *   device (32 MiB), needed on the tensor-core path only. A tensor-core call
 *   needing more than that, i.e. fkc_assign_workspace_size() > the limit
 *   (about B*N + B*K > 1,048,000 rows), returns FKC_EWORKSPACE with a message
 *   and launches nothing. Calls that take the CUDA-core kernel (fp32 beyond
 *   the scratch, odd D, FKC_ASSIGN_FORCE_SAFE=1, x or centroids not 16-byte
 *   aligned) need no scratch and have no limit.
 *   Every call looks up the scratch address on the current device (a host-side
 *   query; the address stays right across a device reset). The first call on
 *   a device also loads this library's device code there (a set-up step): make
 *   that first call before any stream capture.
 *   All calls on a device share the scratch: calls that overlap on the GPU
 *   (unordered streams, concurrent host threads) race. Order them.
 *   Allocates nothing: no cudaMalloc, cudaFree or allocating library call.
 * ---------------------------------------------------------------------- */
#define FKC_ASSIGN_NOALLOC_SCRATCH_BYTES (32u * 1024u * 1024u)
FKC_CAPI_EXPORT int fkc_assign_noalloc(const void* x, const void* centroids, const float* x_sq,
                                       const float* c_sq, int32_t* ids, int64_t B, int64_t N,
                                       int64_t K, int64_t D, int dtype, fkc_stream_t stream);

/* ------------------------------------------------------------------------
 * Sorted-run accumulators with the reference _C semantics: they ADD into
 * caller-initialised sums (B,K,D) fp32 and counts (B,K) int32.
 *   ids_sorted (B,N): labels sorted ascending along N.
 *   fkc_update_sorted:          rows read from x_sorted (B,N,D).
 *   fkc_update_sorted_indexed:  rows read from x[b, sorted_idx[b,i], :].
 * Labels outside [0,K) are skipped (reference: update_sorted.cu:94).
 * Replaces: _C.centroid_update_sorted (csrc/bindings.cpp:73-80),
 *           _C.centroid_update_sorted_indexed (csrc/bindings.cpp:82-90),
 *           csrc/update/update.h:28-48.
 * ---------------------------------------------------------------------- */
FKC_CAPI_EXPORT int fkc_update_sorted(const void* x_sorted, const int32_t* ids_sorted,
                                      float* sums, int32_t* counts, int64_t B, int64_t N,
                                      int64_t K, int64_t D, int dtype, fkc_stream_t stream);
FKC_CAPI_EXPORT int fkc_update_sorted_indexed(const void* x, const int32_t* sorted_idx,
                                              const int32_t* ids_sorted, float* sums,
                                              int32_t* counts, int64_t B, int64_t N, int64_t K,
                                              int64_t D, int dtype, fkc_stream_t stream);

/* ------------------------------------------------------------------------
 * Centroid update from UNSORTED labels: counting sort of ids (histogram,
 * scan, scatter of a permutation) then a permutation-driven gather-accumulate.
 * Writes sums (B,K,D) fp32 and counts (B,K) int32 completely (no pre-zeroing).
 * Labels must lie in [0,K).
 * Replaces: ops.centroid_update_sorted (flash_kmeans_cuda/ops.py:58-112),
 *           i.e. torch.sort + zero_ + _C.centroid_update_sorted[_indexed].
 * ---------------------------------------------------------------------- */
FKC_CAPI_EXPORT size_t fkc_update_workspace_size(int64_t B, int64_t N, int64_t K);
FKC_CAPI_EXPORT int fkc_update(const void* x, const int32_t* ids, float* sums, int32_t* counts,
                               int64_t B, int64_t N, int64_t K, int64_t D, int dtype,
                               void* workspace, size_t workspace_bytes, fkc_stream_t stream);

/* ------------------------------------------------------------------------
 * Finalize: new[b,k,:] = counts[b,k] > 0 ? dtype(sums[b,k,:] / counts[b,k])
 *                                        : old[b,k,:]
 * Optional outputs (NULL to skip):
 *   c_sq_out (B,K) fp32: ||new[b,k]||^2 of the dtype-rounded centroids
 *                        (reference computes it next iteration, kmeans.py:94);
 *   shift_out (1) fp32:  max_{b,k} ||new - old||_2 (kmeans.py:102-104).
 * new_c may alias old_c (in-place update; each element is read before it is
 * written by the same thread).
 * Replaces: _C.centroid_finalize (csrc/bindings.cpp:92-102),
 *           fkc::centroid_finalize_out (csrc/api.cpp:105-113).
 * ---------------------------------------------------------------------- */
FKC_CAPI_EXPORT int fkc_finalize(const float* sums, const int32_t* counts, const void* old_c,
                                 void* new_c, float* c_sq_out, float* shift_out, int64_t B,
                                 int64_t K, int64_t D, int dtype, fkc_stream_t stream);

/* ------------------------------------------------------------------------
 * Lloyd iteration (kmeans.py:73-105 as device-resident steps). One workspace
 * of fkc_lloyd_workspace_size() bytes carries state between the calls:
 *   fkc_lloyd_prepare   once per x: per-row terms of the assignment; also
 *                       zeroes the fused update's accumulators (call it
 *                       again after a failed fkc_lloyd_iter).
 *   fkc_lloyd_assign    labels ids (B,N) and per-cluster counts (B,K) (the
 *                       histogram is fused into the assignment kernel);
 *   fkc_lloyd_update    sums (B,K,D) fp32 from x, ids and those counts;
 *   fkc_lloyd_local     assign + update of this rank's x.
 *                       Multi-GPU callers all-reduce sums/counts here.
 *   fkc_lloyd_finalize  new centroids (+ shift_out if non-NULL) from the
 *                       (reduced) sums/counts; also prepares the next
 *                       iteration's centroid terms inside the workspace.
 *   fkc_lloyd_iter      local + finalize. On one GPU (rows of whole 16-byte
 *                       vectors, 16-byte aligned buffers) the update and the
 *                       finalize run as one pass over the clusters; sums and
 *                       counts are written all the same.
 * The centroids passed to fkc_lloyd_local must be those last produced by
 * fkc_lloyd_finalize with the same workspace, or fkc_lloyd_set_centroids
 * must be called first (initial centroids).
 * Reproducibility: with FKC_DETERMINISTIC=1 in the environment (read once),
 * fkc_lloyd_update and fkc_lloyd_iter sum every cluster in an order fixed by
 * the labels (labels in [0,K), K <= 65536, rows of 64..512 bytes, 16-byte
 * aligned buffers), so repeated runs on one device give bit-identical sums
 * and centroids; by default the sums accumulate with atomics (faster; equal
 * up to fp32 rounding).
 * ---------------------------------------------------------------------- */
FKC_CAPI_EXPORT size_t fkc_lloyd_workspace_size(int64_t B, int64_t N, int64_t K, int64_t D,
                                                int dtype);
FKC_CAPI_EXPORT int fkc_lloyd_prepare(const void* x, int64_t B, int64_t N, int64_t K, int64_t D,
                                      int dtype, void* workspace, size_t workspace_bytes,
                                      fkc_stream_t stream);
FKC_CAPI_EXPORT int fkc_lloyd_set_centroids(const void* centroids, int64_t B, int64_t N,
                                            int64_t K, int64_t D, int dtype, void* workspace,
                                            size_t workspace_bytes, fkc_stream_t stream);
FKC_CAPI_EXPORT int fkc_lloyd_assign(const void* x, const void* centroids, int32_t* ids,
                                     int32_t* counts, int64_t B, int64_t N, int64_t K, int64_t D,
                                     int dtype, void* workspace, size_t workspace_bytes,
                                     fkc_stream_t stream);
FKC_CAPI_EXPORT int fkc_lloyd_update(const void* x, const int32_t* ids, const int32_t* counts,
                                     float* sums, int64_t B, int64_t N, int64_t K, int64_t D,
                                     int dtype, void* workspace, size_t workspace_bytes,
                                     fkc_stream_t stream);
FKC_CAPI_EXPORT int fkc_lloyd_local(const void* x, const void* centroids, int32_t* ids,
                                    float* sums, int32_t* counts, int64_t B, int64_t N,
                                    int64_t K, int64_t D, int dtype, void* workspace,
                                    size_t workspace_bytes, fkc_stream_t stream);
FKC_CAPI_EXPORT int fkc_lloyd_finalize(const float* sums, const int32_t* counts,
                                       const void* old_c, void* new_c, float* shift_out,
                                       int64_t B, int64_t N, int64_t K, int64_t D, int dtype,
                                       void* workspace, size_t workspace_bytes,
                                       fkc_stream_t stream);
FKC_CAPI_EXPORT int fkc_lloyd_iter(const void* x, const void* old_c, void* new_c, int32_t* ids,
                                   float* sums, int32_t* counts, float* shift_out, int64_t B,
                                   int64_t N, int64_t K, int64_t D, int dtype, void* workspace,
                                   size_t workspace_bytes, fkc_stream_t stream);

/* ------------------------------------------------------------------------
 * Multi-GPU finalize fused with the all-reduce, over NVLink multicast
 * (NVSwitch in-switch reduction). Each rank keeps its per-cluster sums
 * (B,K,D) fp32 and counts (B,K) int32 from fkc_lloyd_local in symmetric
 * memory (same layout on every rank, mapped to one multicast object), and the
 * centroids and Lloyd workspace likewise. After a barrier that follows every
 * rank's fkc_lloyd_local, each rank calls this for its own slice
 * [row_begin, row_end) of the B*K centroid rows: it reads the SUM over all
 * ranks with multimem.ld_reduce from mc_sums / mc_counts (multicast
 * addresses), computes the new rows from `centroids` (this rank's copy, old
 * values), and writes them, their ||c||^2 and norm-slice rows into every
 * rank's centroids and workspace through mc_centroids / mc_workspace
 * (in place). mc_shift (nullable, multicast u32): max-reduced with the
 * shift of the slice, as the bits of a non-negative float; shift_clear
 * (nullable, this rank's copy of a float): set to 0 (a parity double buffer
 * for the next iteration's shift). A second barrier must follow before any
 * rank reads the centroids or reuses the sums. D % 4 == 0.
 * Replaces: the NCCL all-reduce of sums/counts + replicated centroid_finalize
 * of a data-parallel Lloyd step (kmeans.py:73-105 with sharded x).
 * ---------------------------------------------------------------------- */
FKC_CAPI_EXPORT int fkc_lloyd_finalize_multimem(
    const float* mc_sums, const int32_t* mc_counts, const void* centroids, void* mc_centroids,
    void* mc_workspace, unsigned int* mc_shift, float* shift_clear, int64_t row_begin,
    int64_t row_end, int64_t B, int64_t K, int64_t D, int dtype, fkc_stream_t stream);

/* ------------------------------------------------------------------------
 * fkc_lloyd_finalize_multimem with the step's two cross-GPU barriers folded
 * into device code (no reference counterpart; the reference is single-GPU).
 *   bar: this rank's copy of 3 uint32 words in the symmetric buffer (zero
 *   before the first step), mc_bar: their multicast address; epoch: 1 for the
 *   first step, +1 for each later one; world: ranks. Every rank must call it
 *   once per step with the same epoch and a non-empty row range.
 *   The kernel adds this rank's arrival to every rank's bar[0], waits until all
 *   ranks have arrived (their local sums and counts are final), finalizes its
 *   rows, and its last CTA adds this rank's completion to every rank's bar[1].
 *   fkc_multimem_step_wait(bar, epoch, world) then waits, on the stream, until
 *   every rank's finalize of step `epoch` has completed: call it before the
 *   next local step (which overwrites the sums the ranks read and reads the
 *   centroids they write).
 *   Waits are bounded (4 s): on expiry the kernel records FKC_ETIMEOUT for
 *   fkc_device_status() and returns instead of hanging.
 * ---------------------------------------------------------------------- */
FKC_CAPI_EXPORT int fkc_lloyd_finalize_multimem_synced(
    const float* mc_sums, const int32_t* mc_counts, const void* centroids, void* mc_centroids,
    void* mc_workspace, unsigned int* mc_shift, float* shift_clear, int64_t row_begin,
    int64_t row_end, int64_t B, int64_t K, int64_t D, int dtype, unsigned int* bar,
    unsigned int* mc_bar, uint32_t epoch, int world, fkc_stream_t stream);
FKC_CAPI_EXPORT int fkc_multimem_step_wait(const unsigned int* bar, uint32_t epoch, int world,
                                           fkc_stream_t stream);

/* ------------------------------------------------------------------------
 * The whole Lloyd loop (batch_kmeans_Euclid without init, kmeans.py:162-195)
 * as ONE CUDA graph launch: a device-side WHILE loop over in-place iterations
 * (assign -> update -> finalize) that stops after max_iters iterations or,
 * when tol > 0, after the first iteration whose shift is below tol. No host
 * synchronisation inside the loop.
 *   centroids (B,K,D): initial centroids in, final centroids out (in place).
 *   ids: labels of the last assignment (against the centroids entering the
 *   last iteration); sums/counts: of the last iteration; shift (1) fp32
 *   device: shift of the last iteration; n_iters (1) int32 device, nullable:
 *   iterations run. Call fkc_lloyd_prepare(x) first (workspace of
 *   fkc_lloyd_workspace_size).
 * The first call for a set of buffers and shape captures and instantiates the
 * graph (host cost about a millisecond); later calls with the same pointers
 * replay it. Do not call it while the stream is being captured.
 * Replaces: the Python loop of batch_kmeans_Euclid (kmeans.py:162-195).
 * ---------------------------------------------------------------------- */
FKC_CAPI_EXPORT int fkc_lloyd_run(const void* x, void* centroids, int32_t* ids, float* sums,
                                  int32_t* counts, float* shift, int32_t* n_iters, int max_iters,
                                  float tol, int64_t B, int64_t N, int64_t K, int64_t D,
                                  int dtype, void* workspace, size_t workspace_bytes,
                                  fkc_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* FKC_CAPI_H_ */
