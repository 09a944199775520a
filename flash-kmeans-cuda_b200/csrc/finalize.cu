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

#include <type_traits>

#include "fkc_common.cuh"
#include "fkc_internal.h"
#include "fkc_launch.cuh"
#include "fkc_ptx.cuh"

namespace fkc {
namespace {

template <typename T>
__global__ void __launch_bounds__(256) finalize_kernel(
    const float* __restrict__ sums, const int32_t* __restrict__ counts,
    const T* __restrict__ old_c, T* __restrict__ new_c, float* __restrict__ c_sq_out,
    uint8_t* __restrict__ cext_out, float* __restrict__ shift_out, int64_t rows, int D) {
  pdl_wait();
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

// Vector variant for D % 4 == 0 and aligned rows: L lanes per centroid row
// (32/L rows per warp), each lane 4 consecutive features per step (16-byte
// sums loads, 8- or 16-byte centroid loads/stores); one shift atomic per warp.
template <typename T, int L>
__global__ void __launch_bounds__(256) finalize_vec_kernel(
    const float* __restrict__ sums, const int32_t* __restrict__ counts,
    const T* __restrict__ old_c, T* __restrict__ new_c, float* __restrict__ c_sq_out,
    uint8_t* __restrict__ cext_out, float* __restrict__ shift_out, int64_t rows, int D) {
  pdl_wait();
  constexpr int G = 32 / L;  // rows per warp
  using V = typename std::conditional<sizeof(T) == 2, uint2, uint4>::type;  // 4 elements
  const int lane = threadIdx.x & 31;
  const int g = lane / L, i = lane % L;
  const int64_t warps_total = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t r0 = (static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5)) * G;
       r0 < rows; r0 += warps_total * G) {
    const int64_t r = r0 + g;
    const bool on = r < rows;
    float sq = 0.f, sh = 0.f;
    if (on) {
      const int32_t cnt = counts[r];
      const float fc = static_cast<float>(cnt);
      for (int d = 4 * i; d < D; d += 4 * L) {
        const float4 sv = *reinterpret_cast<const float4*>(sums + r * D + d);
        const V ov = *reinterpret_cast<const V*>(old_c + r * D + d);
        const T* o = reinterpret_cast<const T*>(&ov);
        const float s4[4] = {sv.x, sv.y, sv.z, sv.w};
        V nvv;
        T* nv = reinterpret_cast<T*>(&nvv);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          nv[e] = cnt > 0 ? from_f32<T>(__fdiv_rn(s4[e], fc)) : o[e];
          const float nf = to_f32<T>(nv[e]);
          const float df = nf - to_f32<T>(o[e]);
          sq = fmaf(nf, nf, sq);
          sh = fmaf(df, df, sh);
        }
        *reinterpret_cast<V*>(new_c + r * D + d) = nvv;
      }
    }
#pragma unroll
    for (int off = L / 2; off >= 1; off >>= 1) {
      sq += __shfl_xor_sync(0xFFFFFFFFu, sq, off);
      sh += __shfl_xor_sync(0xFFFFFFFFu, sh, off);
    }
    if (on && i == 0) {
      if (c_sq_out != nullptr) c_sq_out[r] = sq;
      if (cext_out != nullptr) write_norm_ext(cext_out + r * kNormExtBytes, -0.5f * sq, false);
    }
    if (shift_out != nullptr) {
      float m = on ? sqrtf(sh) : 0.f;
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, off));
      if (lane == 0) atomicMax(reinterpret_cast<unsigned int*>(shift_out), __float_as_uint(m));
    }
  }
}

// ---------------------------------------------------------------------------
// Multi-GPU finalize over NVLink multicast. Every rank holds its own per-cluster
// sums/counts in a symmetric buffer; a rank finalizes only the centroid rows
// [row0, row1) of the flattened (B*K) rows: it reads the SUM over all ranks
// with multimem.ld_reduce (the NVSwitch adds the copies), and writes each new
// row, its ||c||^2 and its norm-slice row to every rank with multimem.st. The
// shift is max-reduced with multimem.red.max on the bits of a non-negative
// float. So the all-reduce of sums/counts and the replicated finalize become
// one kernel whose NVLink traffic per rank is one slice of the sums in and the
// new centroids out.
// ---------------------------------------------------------------------------

__device__ __forceinline__ float4 mc_ld_reduce_v4(const float* mc) {
  float4 r;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "l"(mc)
               : "memory");
  return r;
}

__device__ __forceinline__ uint32_t mc_ld_reduce_u32(const int32_t* mc) {
  uint32_t r;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.u32 %0, [%1];"
               : "=r"(r)
               : "l"(mc)
               : "memory");
  return r;
}

__device__ __forceinline__ void mc_st_v2(void* mc, uint32_t a, uint32_t b) {
  asm volatile("multimem.st.relaxed.sys.global.v2.f32 [%0], {%1, %2};" ::"l"(mc),
               "f"(__uint_as_float(a)), "f"(__uint_as_float(b))
               : "memory");
}

__device__ __forceinline__ void mc_st_v4(void* mc, uint32_t a, uint32_t b, uint32_t c,
                                         uint32_t d) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc),
               "f"(__uint_as_float(a)), "f"(__uint_as_float(b)), "f"(__uint_as_float(c)),
               "f"(__uint_as_float(d))
               : "memory");
}

__device__ __forceinline__ void mc_st_f32(void* mc, float v) {
  asm volatile("multimem.st.relaxed.sys.global.f32 [%0], %1;" ::"l"(mc), "f"(v) : "memory");
}

__device__ __forceinline__ void mc_red_max_u32(void* mc, uint32_t v) {
  asm volatile("multimem.red.relaxed.sys.global.max.u32 [%0], %1;" ::"l"(mc), "r"(v) : "memory");
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(T a, T b) {
  static_assert(sizeof(T) == 2, "16-bit element");
  uint16_t ua, ub;
  memcpy(&ua, &a, 2);
  memcpy(&ub, &b, 2);
  return static_cast<uint32_t>(ua) | (static_cast<uint32_t>(ub) << 16);
}

__device__ __forceinline__ void mc_red_add_release_u32(unsigned int* mc, uint32_t v) {
  asm volatile("multimem.red.release.sys.global.add.u32 [%0], %1;" ::"l"(mc), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned int* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Cross-GPU step barrier words (this rank's copies; the multicast address adds
// to every rank's copy): [0] ranks arrived at the finalize of the step,
// [1] ranks whose finalize of the step has completed, [2] finished CTAs of
// this rank's finalize launch (local).
enum : int { kBarArrive = 0, kBarDone = 1, kBarCtas = 2 };
constexpr uint64_t kStepBarrierNs = 4000000000ull;
enum : int { kErrStepBarrier = 141 };

// Bounded wait until *word - target >= 0 (wrapping epoch counters); records
// kErrStepBarrier in the device error word and returns false on timeout.
__device__ bool wait_counter(const unsigned int* word, unsigned target, int* err) {
  const uint64_t t0 = ptx::globaltimer_ns();
  while (static_cast<int>(ld_acquire_sys(word) - target) < 0) {
    if (ptx::globaltimer_ns() - t0 > kStepBarrierNs) {
      if (err != nullptr) atomicCAS(err, 0, kErrStepBarrier);
      return false;
    }
    __nanosleep(64);
  }
  return true;
}

// D % 4 == 0: lane l owns elements [4l + 128i, 4l + 128i + 4) of the row.
// With bar != nullptr the step's cross-GPU barriers are folded in: thread 0 of
// CTA 0 adds this rank's arrival to every rank's bar[0] (multicast, release),
// every CTA waits until bar[0] reaches epoch * world (all ranks' local sums and
// counts are final), and the last CTA of the launch adds this rank's
// completion to every rank's bar[1] after its multicast stores.
template <typename T>
__global__ void __launch_bounds__(256) finalize_multimem_kernel(
    const float* __restrict__ mc_sums, const int32_t* __restrict__ mc_counts,
    const T* __restrict__ old_c, T* mc_new_c, float* mc_c_sq, uint8_t* mc_cext,
    unsigned int* mc_shift, float* shift_clear, int64_t row0, int64_t row1, int D,
    unsigned int* bar, unsigned int* mc_bar, unsigned target, int* err) {
  pdl_wait();
  const int lane = threadIdx.x & 31;
  __shared__ int go;
  if (bar != nullptr) {
    if (threadIdx.x == 0) {
      if (blockIdx.x == 0) {
        asm volatile("fence.acq_rel.sys;" ::: "memory");
        mc_red_add_release_u32(mc_bar + kBarArrive, 1u);
      }
      go = wait_counter(bar + kBarArrive, target, err) ? 1 : 0;
    }
    __syncthreads();
  } else if (threadIdx.x == 0) {
    go = 1;
  }
  if (bar == nullptr) __syncthreads();
  if (shift_clear != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *shift_clear = 0.f;
  const int64_t warps_total = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t r = row0 + static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) +
                   (threadIdx.x >> 5);
       go != 0 && r < row1; r += warps_total) {
    // the sums reduction does not depend on the count: issue both before waiting
    float4 sv0 = make_float4(0.f, 0.f, 0.f, 0.f);
    if (4 * lane < D) sv0 = mc_ld_reduce_v4(mc_sums + r * D + 4 * lane);
    int32_t cnt = 0;
    if (lane == 0) cnt = static_cast<int32_t>(mc_ld_reduce_u32(mc_counts + r));
    cnt = __shfl_sync(0xFFFFFFFFu, cnt, 0);
    const float fc = static_cast<float>(cnt);
    float sq = 0.f, sh = 0.f;
    for (int d = 4 * lane; d < D; d += 128) {
      const float4 sv = d == 4 * lane ? sv0 : mc_ld_reduce_v4(mc_sums + r * D + d);
      const float s4[4] = {sv.x, sv.y, sv.z, sv.w};
      T nv[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const T ov = old_c[r * D + d + e];
        nv[e] = cnt > 0 ? from_f32<T>(__fdiv_rn(s4[e], fc)) : ov;
        const float nf = to_f32<T>(nv[e]);
        const float df = nf - to_f32<T>(ov);
        sq = fmaf(nf, nf, sq);
        sh = fmaf(df, df, sh);
      }
      if constexpr (sizeof(T) == 4) {
        mc_st_v4(mc_new_c + r * D + d, __float_as_uint(to_f32<T>(nv[0])),
                 __float_as_uint(to_f32<T>(nv[1])), __float_as_uint(to_f32<T>(nv[2])),
                 __float_as_uint(to_f32<T>(nv[3])));
      } else {
        mc_st_v2(mc_new_c + r * D + d, pack2<T>(nv[0], nv[1]), pack2<T>(nv[2], nv[3]));
      }
    }
    sq = warp_sum(sq);
    sh = warp_sum(sh);
    if (lane == 0) {
      if (mc_c_sq != nullptr) mc_st_f32(mc_c_sq + r, sq);
      if (mc_cext != nullptr) {
        alignas(16) uint8_t row[kNormExtBytes];
        write_norm_ext(row, -0.5f * sq, false);
        const uint32_t* w = reinterpret_cast<const uint32_t*>(row);
        mc_st_v4(mc_cext + r * kNormExtBytes, w[0], w[1], w[2], w[3]);
        mc_st_v4(mc_cext + r * kNormExtBytes + 16, w[4], w[5], w[6], w[7]);
      }
      if (mc_shift != nullptr) mc_red_max_u32(mc_shift, __float_as_uint(sqrtf(sh)));
    }
  }
  // The multicast stores and reductions are ordered before whatever follows
  // this kernel on the stream (the cross-GPU barrier's release).
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  if (bar != nullptr) {
    __syncthreads();
    if (threadIdx.x == 0) {
      // the last CTA out signals this rank's completion to every rank
      if (atomicAdd(bar + kBarCtas, 1u) == gridDim.x - 1) {
        bar[kBarCtas] = 0u;
        asm volatile("fence.acq_rel.sys;" ::: "memory");
        mc_red_add_release_u32(mc_bar + kBarDone, 1u);
      }
    }
  }
}

// Waits (bounded) until every rank's finalize of the previous step has
// completed (bar[1] reaches target): before the next local step writes the
// sums the other ranks read and reads the centroids they write.
__global__ void step_wait_kernel(const unsigned int* bar, unsigned target, int* err) {
  pdl_wait();
  if (threadIdx.x == 0) wait_counter(bar + kBarDone, target, err);
}

__global__ void __launch_bounds__(256) zero_fill_kernel(uint32_t* __restrict__ p, int64_t words,
                                                         bool vec) {
  pdl_wait();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (vec) {
    uint4* q = reinterpret_cast<uint4*>(p);
    for (; i < words / 4; i += stride) q[i] = make_uint4(0u, 0u, 0u, 0u);
  } else {
    for (; i < words; i += stride) p[i] = 0u;
  }
}

}  // namespace

int launch_zero_fill(void* ptr, size_t bytes, cudaStream_t stream) {
  FKC_REQUIRE(bytes % 4 == 0 && (reinterpret_cast<uintptr_t>(ptr) & 3u) == 0,
              "zero_fill: 4-byte aligned ranges only");
  const int64_t words = static_cast<int64_t>(bytes / 4);
  if (words == 0) return FKC_OK;
  const bool vec = (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0 && words % 4 == 0;
  const DeviceInfo* di = nullptr;
  FKC_TRY(current_device_info(&di));
  int64_t grid = ((vec ? words / 4 : words) + 255) / 256;
  const int64_t cap = static_cast<int64_t>(di->sm_count) * 8;
  if (grid > cap) grid = cap;
  if (grid < 1) grid = 1;
  return launch_pdl(zero_fill_kernel, dim3(static_cast<unsigned>(grid)), dim3(256), 0, stream,
                    static_cast<uint32_t*>(ptr), words, vec);
}

int launch_step_wait(const unsigned int* bar, unsigned target, cudaStream_t stream) {
  return launch_pdl(step_wait_kernel, dim3(1), dim3(32), 0, stream, bar, target,
                    device_error_word());
}

int launch_finalize_multimem(const float* mc_sums, const int32_t* mc_counts, const void* old_c,
                             void* mc_new_c, float* mc_c_sq, void* mc_cext,
                             unsigned int* mc_shift, float* shift_clear, int64_t row0,
                             int64_t row1, int64_t D, int dtype, cudaStream_t stream,
                             unsigned int* bar, unsigned int* mc_bar, unsigned target) {
  FKC_REQUIRE(D % 4 == 0, "finalize_multimem: D must be a multiple of 4 (got %lld)",
              static_cast<long long>(D));
  const int64_t rows = row1 - row0;
  const DeviceInfo* di = nullptr;
  FKC_TRY(current_device_info(&di));
  int64_t grid = (rows + 7) / 8;
  // With the arrival barrier in the kernel every CTA waits for all ranks' CTA
  // 0: keep the grid within one resident wave (4 CTAs of 256 threads and at
  // most 48 registers per thread fit an SM), so CTA 0 is always running.
  const int64_t cap = static_cast<int64_t>(di->sm_count) * (bar != nullptr ? 4 : 16);
  if (grid > cap) grid = cap;
  if (grid < 1) grid = 1;
  uint8_t* ce = static_cast<uint8_t*>(mc_cext);
  const int d = static_cast<int>(D);
  const dim3 g(static_cast<unsigned>(grid)), blk(256);
  int* err = bar != nullptr ? device_error_word() : nullptr;
  switch (dtype) {
    case FKC_DTYPE_F16:
      return launch_pdl(finalize_multimem_kernel<__half>, g, blk, 0, stream, mc_sums, mc_counts,
                        static_cast<const __half*>(old_c), static_cast<__half*>(mc_new_c),
                        mc_c_sq, ce, mc_shift, shift_clear, row0, row1, d, bar, mc_bar, target,
                        err);
    case FKC_DTYPE_BF16:
      return launch_pdl(finalize_multimem_kernel<__nv_bfloat16>, g, blk, 0, stream, mc_sums,
                        mc_counts, static_cast<const __nv_bfloat16*>(old_c),
                        static_cast<__nv_bfloat16*>(mc_new_c), mc_c_sq, ce, mc_shift,
                        shift_clear, row0, row1, d, bar, mc_bar, target, err);
    case FKC_DTYPE_F32:
      return launch_pdl(finalize_multimem_kernel<float>, g, blk, 0, stream, mc_sums, mc_counts,
                        static_cast<const float*>(old_c), static_cast<float*>(mc_new_c),
                        mc_c_sq, ce, mc_shift, shift_clear, row0, row1, d, bar, mc_bar, target,
                        err);
    default:
      return set_error(FKC_EINVAL, "finalize_multimem: bad dtype %d", dtype);
  }
}

int launch_finalize(const float* sums, const int32_t* counts, const void* old_c, void* new_c,
                    float* c_sq_out, void* cext_out, float* shift_out, int64_t B, int64_t K,
                    int64_t D, int dtype, cudaStream_t stream, bool shift_zeroed) {
  const int64_t rows = B * K;
  if (shift_out != nullptr && !shift_zeroed)
    FKC_TRY(launch_zero_fill(shift_out, sizeof(float), stream));
  const DeviceInfo* di = nullptr;
  FKC_TRY(current_device_info(&di));
  int64_t grid = (rows + 7) / 8;
  const int64_t cap = static_cast<int64_t>(di->sm_count) * 16;
  if (grid > cap) grid = cap;
  if (grid < 1) grid = 1;
  uint8_t* ce = static_cast<uint8_t*>(cext_out);
  const int d = static_cast<int>(D);
  const dim3 g(static_cast<unsigned>(grid)), blk(256);
  const size_t es = dtype == FKC_DTYPE_F32 ? 4 : 2;
  const bool vec = D % 4 == 0 && (reinterpret_cast<uintptr_t>(sums) & 15u) == 0 &&
                   (reinterpret_cast<uintptr_t>(old_c) & (4 * es - 1)) == 0 &&
                   (reinterpret_cast<uintptr_t>(new_c) & (4 * es - 1)) == 0;
  if (vec) {
    const int L = D <= 32 ? 8 : (D <= 64 ? 16 : 32);  // lanes per row
    const int64_t warps = (rows * L + 31) / 32;
    int64_t gv = (warps + 7) / 8;
    if (gv > cap) gv = cap;
    const dim3 gg(static_cast<unsigned>(gv < 1 ? 1 : gv));
    auto go = [&](auto tag, auto lanes) -> int {
      using T = decltype(tag);
      return launch_pdl(finalize_vec_kernel<T, decltype(lanes)::value>, gg, blk, 0, stream, sums,
                        counts, static_cast<const T*>(old_c), static_cast<T*>(new_c), c_sq_out,
                        ce, shift_out, rows, d);
    };
    using L8 = std::integral_constant<int, 8>;
    using L16 = std::integral_constant<int, 16>;
    using L32 = std::integral_constant<int, 32>;
    switch (dtype) {
      case FKC_DTYPE_F16:
        return L == 8 ? go(__half{}, L8{}) : L == 16 ? go(__half{}, L16{}) : go(__half{}, L32{});
      case FKC_DTYPE_BF16:
        return L == 8    ? go(__nv_bfloat16{}, L8{})
               : L == 16 ? go(__nv_bfloat16{}, L16{})
                         : go(__nv_bfloat16{}, L32{});
      case FKC_DTYPE_F32:
        return L == 8 ? go(float{}, L8{}) : L == 16 ? go(float{}, L16{}) : go(float{}, L32{});
      default:
        return set_error(FKC_EINVAL, "finalize: bad dtype %d", dtype);
    }
  }
  switch (dtype) {
    case FKC_DTYPE_F16:
      return launch_pdl(finalize_kernel<__half>, g, blk, 0, stream, sums, counts,
                        static_cast<const __half*>(old_c), static_cast<__half*>(new_c), c_sq_out,
                        ce, shift_out, rows, d);
    case FKC_DTYPE_BF16:
      return launch_pdl(finalize_kernel<__nv_bfloat16>, g, blk, 0, stream, sums, counts,
                        static_cast<const __nv_bfloat16*>(old_c),
                        static_cast<__nv_bfloat16*>(new_c), c_sq_out, ce, shift_out, rows, d);
    case FKC_DTYPE_F32:
      return launch_pdl(finalize_kernel<float>, g, blk, 0, stream, sums, counts,
                        static_cast<const float*>(old_c), static_cast<float*>(new_c), c_sq_out,
                        ce, shift_out, rows, d);
    default:
      return set_error(FKC_EINVAL, "finalize: bad dtype %d", dtype);
  }
}

}  // namespace fkc
