// Centroid update: per-cluster fp32 sums and int32 counts.
//
// The reference sorts labels with torch.sort and then runs a sorted-run
// accumulator whose run boundaries are found serially by thread 0 and whose
// flushes are one fp32 atomicAdd per feature
// (flash_kmeans_cuda/ops.py:89-111, csrc/update/update_sorted.cu:39-186).
// Here:
//   * the permutation comes from a counting sort on labels in [0, K):
//     histogram (warp-aggregated atomics; fused into the assignment kernel on
//     the Lloyd path) -> exclusive scan per batch row -> scatter of row indices
//     (warp-aggregated cursors);
//   * the accumulator walks sorted positions with one warp per range of 64
//     positions: run boundaries come from a warp ballot, rows are gathered with
//     16-byte vector loads (a D=128 fp16 row is 16 lanes x 16 B), partial sums
//     live in registers and each run piece is flushed with 16-byte vector
//     atomics (red.global.add.v4.f32). No sorted copy of x is written.
// The same accumulator serves the reference's _C.centroid_update_sorted and
// _C.centroid_update_sorted_indexed entry points (perm == nullptr for the
// former).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "fkc_common.cuh"
#include "fkc_internal.h"

namespace fkc {
namespace {

constexpr int kRange = 64;  // sorted positions per warp in the accumulator

__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t m;
  asm volatile("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

__global__ void histogram_kernel(const int32_t* __restrict__ ids, int32_t* __restrict__ counts,
                                 int64_t total, int64_t N, int K) {
  const int lane = threadIdx.x & 31;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * blockDim.x + (threadIdx.x & ~31);
       base < total; base += stride) {
    const int64_t i = base + lane;
    bool v = false;
    long long key = -1;
    if (i < total) {
      const int id = ids[i];
      if (id >= 0 && id < K) {
        v = true;
        key = (i / N) * K + id;
      }
    }
    const uint32_t act = __ballot_sync(0xFFFFFFFFu, v);
    if (v) {
      const uint32_t peers = __match_any_sync(act, key);
      if (lane == __ffs(peers) - 1) atomicAdd(counts + key, __popc(peers));
    }
  }
}

// Exclusive scan of counts[b, 0..K) into offsets and cursor; one CTA per b.
__global__ void __launch_bounds__(1024) scan_kernel(const int32_t* __restrict__ counts,
                                                    int32_t* __restrict__ offsets,
                                                    int32_t* __restrict__ cursor, int K) {
  __shared__ int warp_tot[32];
  const int b = blockIdx.x;
  const int t = threadIdx.x;
  const int lane = t & 31, w = t >> 5;
  const int32_t* cnt = counts + static_cast<size_t>(b) * K;
  const int per = (K + blockDim.x - 1) / blockDim.x;
  const int beg = min(K, t * per), end = min(K, beg + per);
  int local = 0;
  for (int i = beg; i < end; ++i) local += cnt[i];
  // inclusive warp scan
  int v = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int u = __shfl_up_sync(0xFFFFFFFFu, v, o);
    if (lane >= o) v += u;
  }
  if (lane == 31) warp_tot[w] = v;
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    int s = lane < nw ? warp_tot[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xFFFFFFFFu, s, o);
      if (lane >= o) s += u;
    }
    if (lane < nw) warp_tot[lane] = s;  // inclusive over warps
  }
  __syncthreads();
  int run = v - local + (w > 0 ? warp_tot[w - 1] : 0);
  int32_t* off = offsets + static_cast<size_t>(b) * K;
  int32_t* cur = cursor + static_cast<size_t>(b) * K;
  for (int i = beg; i < end; ++i) {
    off[i] = run;
    cur[i] = run;
    run += cnt[i];
  }
}

// perm[b, pos] = n and ids_sorted[b, pos] = id, pos = offsets[b,id] + rank.
// Rank within a cluster follows atomic order (not n order).
__global__ void scatter_kernel(const int32_t* __restrict__ ids, int32_t* __restrict__ cursor,
                               int32_t* __restrict__ perm, int32_t* __restrict__ ids_sorted,
                               int64_t total, int64_t N, int K) {
  const int lane = threadIdx.x & 31;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * blockDim.x + (threadIdx.x & ~31);
       base < total; base += stride) {
    const int64_t i = base + lane;
    bool v = false;
    long long key = -1;
    int id = 0;
    int64_t b = 0;
    if (i < total) {
      id = ids[i];
      b = i / N;
      if (id >= 0 && id < K) {
        v = true;
        key = b * K + id;
      }
    }
    const uint32_t act = __ballot_sync(0xFFFFFFFFu, v);
    if (v) {
      const uint32_t peers = __match_any_sync(act, key);
      const int leader = __ffs(peers) - 1;
      int pos0 = 0;
      if (lane == leader) pos0 = atomicAdd(cursor + key, __popc(peers));
      pos0 = __shfl_sync(peers, pos0, leader);
      const int pos = pos0 + __popc(peers & lanemask_lt());
      const int64_t dst = b * N + pos;
      perm[dst] = static_cast<int32_t>(i - b * N);
      ids_sorted[dst] = id;
    }
  }
}

__device__ __forceinline__ void red_add_v4(float* addr, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b),
               "f"(c), "f"(d)
               : "memory");
}

// Finds the end of the run of `id` starting at `pos` inside [pos, lim).
__device__ __forceinline__ int run_end_of(const int32_t* __restrict__ ids_b, int pos, int lim,
                                          int id, int lane) {
  for (int c = pos; c < lim; c += 32) {
    const int q = c + lane;
    const bool diff = (q < lim) && (ids_b[q] != id);
    const uint32_t m = __ballot_sync(0xFFFFFFFFu, diff);
    if (m) return c + __ffs(m) - 1;
  }
  return lim;
}

// Vector path: a row is L = D*sizeof(T)/16 sixteen-byte vectors (L <= 32);
// lane l handles vector (l % L) of rows (l / L) + i*RPS, RPS = 32 / L.
template <typename T>
__global__ void __launch_bounds__(256) run_accumulate_vec_kernel(
    const T* __restrict__ x, const int32_t* __restrict__ perm,
    const int32_t* __restrict__ ids_sorted, float* __restrict__ sums,
    int32_t* __restrict__ counts, int N, int K, int D, int L, int ranges_per_batch,
    int64_t total_ranges) {
  constexpr int kVec = 16 / sizeof(T);  // elements per 16-byte vector
  const int lane = threadIdx.x & 31;
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (gw >= total_ranges) return;
  const int b = static_cast<int>(gw / ranges_per_batch);
  const int r = static_cast<int>(gw - static_cast<int64_t>(b) * ranges_per_batch);
  const int p0 = r * kRange;
  const int p1 = min(p0 + kRange, N);
  const int32_t* ids_b = ids_sorted + static_cast<size_t>(b) * N;
  const int32_t* perm_b = perm ? perm + static_cast<size_t>(b) * N : nullptr;
  const T* xb = x + static_cast<size_t>(b) * N * D;
  const int RPS = 32 / L;
  const int v = lane % L;
  const int sub = lane / L;
  const bool on = sub < RPS;
  const bool pow2 = (L & (L - 1)) == 0;

  int pos = p0;
  while (pos < p1) {
    const int id = ids_b[pos];
    const int end = run_end_of(ids_b, pos, p1, id, lane);
    if (id >= 0 && id < K) {
      float acc[kVec];
#pragma unroll
      for (int e = 0; e < kVec; ++e) acc[e] = 0.f;
      if (on) {
        int row = pos + sub;
        // Four rows in flight per lane.
        for (; row + 3 * RPS < end; row += 4 * RPS) {
          uint4 u[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int q = row + i * RPS;
            const int src = perm_b ? perm_b[q] : q;
            u[i] = reinterpret_cast<const uint4*>(xb + static_cast<size_t>(src) * D)[v];
          }
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const T* e = reinterpret_cast<const T*>(&u[i]);
#pragma unroll
            for (int k = 0; k < kVec; ++k) acc[k] += to_f32<T>(e[k]);
          }
        }
        for (; row < end; row += RPS) {
          const int src = perm_b ? perm_b[row] : row;
          const uint4 u = reinterpret_cast<const uint4*>(xb + static_cast<size_t>(src) * D)[v];
          const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
          for (int k = 0; k < kVec; ++k) acc[k] += to_f32<T>(e[k]);
        }
      }
      // Reduce the RPS partial sums of each vector slot into lanes sub == 0.
      if (pow2) {
        for (int o = L; o < 32; o <<= 1) {
#pragma unroll
          for (int k = 0; k < kVec; ++k) acc[k] += __shfl_xor_sync(0xFFFFFFFFu, acc[k], o);
        }
      } else {
        for (int s = 1; s < RPS; ++s) {
#pragma unroll
          for (int k = 0; k < kVec; ++k) {
            const float o = __shfl_sync(0xFFFFFFFFu, acc[k], (v + s * L) & 31);
            if (sub == 0) acc[k] += o;
          }
        }
      }
      if (sub == 0) {
        float* dst = sums + (static_cast<size_t>(b) * K + id) * D + v * kVec;
#pragma unroll
        for (int k = 0; k < kVec; k += 4) red_add_v4(dst + k, acc[k], acc[k + 1], acc[k + 2], acc[k + 3]);
      }
      if (counts != nullptr && lane == 0)
        atomicAdd(counts + static_cast<size_t>(b) * K + id, end - pos);
    }
    pos = end;
  }
}

// Scalar path for any D: lanes stride over features, 128 columns per pass.
template <typename T>
__global__ void __launch_bounds__(256) run_accumulate_scalar_kernel(
    const T* __restrict__ x, const int32_t* __restrict__ perm,
    const int32_t* __restrict__ ids_sorted, float* __restrict__ sums,
    int32_t* __restrict__ counts, int N, int K, int D, int ranges_per_batch,
    int64_t total_ranges) {
  const int lane = threadIdx.x & 31;
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (gw >= total_ranges) return;
  const int b = static_cast<int>(gw / ranges_per_batch);
  const int r = static_cast<int>(gw - static_cast<int64_t>(b) * ranges_per_batch);
  const int p0 = r * kRange;
  const int p1 = min(p0 + kRange, N);
  const int32_t* ids_b = ids_sorted + static_cast<size_t>(b) * N;
  const int32_t* perm_b = perm ? perm + static_cast<size_t>(b) * N : nullptr;
  const T* xb = x + static_cast<size_t>(b) * N * D;
  int pos = p0;
  while (pos < p1) {
    const int id = ids_b[pos];
    const int end = run_end_of(ids_b, pos, p1, id, lane);
    if (id >= 0 && id < K) {
      float* dst = sums + (static_cast<size_t>(b) * K + id) * D;
      for (int d0 = 0; d0 < D; d0 += 128) {
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        for (int row = pos; row < end; ++row) {
          const T* src = xb + static_cast<size_t>(perm_b ? perm_b[row] : row) * D;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int d = d0 + lane + 32 * i;
            if (d < D) acc[i] += to_f32<T>(src[d]);
          }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int d = d0 + lane + 32 * i;
          if (d < D) atomicAdd(dst + d, acc[i]);
        }
      }
      if (counts != nullptr && lane == 0)
        atomicAdd(counts + static_cast<size_t>(b) * K + id, end - pos);
    }
    pos = end;
  }
}

int sm_count_or_default() {
  const DeviceInfo* di = nullptr;
  if (current_device_info(&di) == FKC_OK) return di->sm_count;
  return 148;
}

int grid_for(int64_t items, int per_block) {
  int64_t g = (items + per_block - 1) / per_block;
  const int64_t cap = static_cast<int64_t>(sm_count_or_default()) * 8;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return static_cast<int>(g);
}

template <typename T>
int run_accumulate_typed(const void* x, const int32_t* perm, const int32_t* ids_sorted,
                         float* sums, int32_t* counts, int64_t B, int64_t N, int64_t K,
                         int64_t D, cudaStream_t stream) {
  const int64_t ranges_per_batch = (N + kRange - 1) / kRange;
  const int64_t total = ranges_per_batch * B;
  const int64_t blocks = (total + 7) / 8;  // 8 warps per block
  FKC_REQUIRE(blocks < (1ll << 31), "update: too many rows");
  const size_t row_bytes = static_cast<size_t>(D) * sizeof(T);
  const bool vec_ok = row_bytes % 16 == 0 && row_bytes <= 512 &&
                      reinterpret_cast<uintptr_t>(x) % 16 == 0 &&
                      reinterpret_cast<uintptr_t>(sums) % 16 == 0 && (D % 4 == 0);
  if (vec_ok) {
    const int L = static_cast<int>(row_bytes / 16);
    run_accumulate_vec_kernel<T><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
        static_cast<const T*>(x), perm, ids_sorted, sums, counts, static_cast<int>(N),
        static_cast<int>(K), static_cast<int>(D), L, static_cast<int>(ranges_per_batch), total);
  } else {
    run_accumulate_scalar_kernel<T><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
        static_cast<const T*>(x), perm, ids_sorted, sums, counts, static_cast<int>(N),
        static_cast<int>(K), static_cast<int>(D), static_cast<int>(ranges_per_batch), total);
  }
  FKC_CUDA_TRY(cudaGetLastError());
  count_launches(1);
  return FKC_OK;
}

}  // namespace

size_t update_workspace_bytes(int64_t B, int64_t N, int64_t K) {
  const size_t bk = align_up(static_cast<size_t>(B * K) * 4, 256);
  const size_t bn = align_up(static_cast<size_t>(B * N) * 4, 256);
  return 2 * bk + 2 * bn;
}

UpdateWorkspace carve_update_workspace(void* ws, int64_t B, int64_t N, int64_t K) {
  const size_t bk = align_up(static_cast<size_t>(B * K) * 4, 256);
  const size_t bn = align_up(static_cast<size_t>(B * N) * 4, 256);
  uint8_t* p = static_cast<uint8_t*>(ws);
  UpdateWorkspace w;
  w.offsets = reinterpret_cast<int32_t*>(p);
  w.cursor = reinterpret_cast<int32_t*>(p + bk);
  w.perm = reinterpret_cast<int32_t*>(p + 2 * bk);
  w.ids_sorted = reinterpret_cast<int32_t*>(p + 2 * bk + bn);
  return w;
}

int launch_histogram(const int32_t* ids, int32_t* counts, int64_t B, int64_t N, int64_t K,
                     cudaStream_t stream) {
  const int64_t total = B * N;
  histogram_kernel<<<grid_for(total, 256), 256, 0, stream>>>(ids, counts, total, N,
                                                             static_cast<int>(K));
  FKC_CUDA_TRY(cudaGetLastError());
  count_launches(1);
  return FKC_OK;
}

int launch_counting_sort(const int32_t* ids, const int32_t* counts, const UpdateWorkspace& w,
                         int64_t B, int64_t N, int64_t K, cudaStream_t stream) {
  FKC_REQUIRE(B <= 2147483647ll, "update: B too large");
  scan_kernel<<<static_cast<unsigned>(B), 1024, 0, stream>>>(counts, w.offsets, w.cursor,
                                                             static_cast<int>(K));
  FKC_CUDA_TRY(cudaGetLastError());
  count_launches(1);
  // Positions not filled by the scatter (labels outside [0,K)) read as -1 and
  // are skipped by the accumulator.
  FKC_CUDA_TRY(cudaMemsetAsync(w.ids_sorted, 0xFF, static_cast<size_t>(B * N) * 4, stream));
  const int64_t total = B * N;
  scatter_kernel<<<grid_for(total, 256), 256, 0, stream>>>(ids, w.cursor, w.perm, w.ids_sorted,
                                                           total, N, static_cast<int>(K));
  FKC_CUDA_TRY(cudaGetLastError());
  count_launches(1);
  return FKC_OK;
}

int launch_run_accumulate(const void* x, const int32_t* perm, const int32_t* ids_sorted,
                          float* sums, int32_t* counts, int64_t B, int64_t N, int64_t K,
                          int64_t D, int dtype, cudaStream_t stream) {
  switch (dtype) {
    case FKC_DTYPE_F16:
      return run_accumulate_typed<__half>(x, perm, ids_sorted, sums, counts, B, N, K, D, stream);
    case FKC_DTYPE_BF16:
      return run_accumulate_typed<__nv_bfloat16>(x, perm, ids_sorted, sums, counts, B, N, K, D,
                                                 stream);
    case FKC_DTYPE_F32:
      return run_accumulate_typed<float>(x, perm, ids_sorted, sums, counts, B, N, K, D, stream);
    default:
      return set_error(FKC_EINVAL, "update: bad dtype %d", dtype);
  }
}

}  // namespace fkc
