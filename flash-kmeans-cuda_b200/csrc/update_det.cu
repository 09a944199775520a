// Deterministic centroid update of the Lloyd step, in two launches: a stable
// counting sort of the labels, then a span gather that sums every cluster in
// sorted order and finishes it (the finalize fused in).
//
// The reference sorts labels with torch.sort and accumulates sorted runs with
// one fp32 atomicAdd per run and feature (flash_kmeans_cuda/ops.py:89-111,
// csrc/update/update_sorted.cu:118-186); the order of those atomics, and so the
// last bits of its sums, change from run to run. Here every float addition
// happens in an order fixed by the labels and the launch geometry, so two runs
// on the same device give bit-identical sums and centroids.
//
//   sort (det_sort_kernel, one cooperative launch, three phases separated by
//        grid barriers whose waits are bounded):
//     rank     rows in chunks of R; inside a chunk each warp walks its slice of
//              rows in order and counts labels in its own shared-memory row of
//              16-bit counters (match_any ranks a 32-row step), so every row
//              gets its stable rank inside the chunk; the chunk's histogram
//              goes to hist[b][c][:].
//     base     offsets[b][k] = exclusive scan of the counts (the assignment
//              kernel's histogram) and, in place, hist[b][c][k] = offsets[b][k]
//              + the counts of label k in the earlier chunks.
//     scatter  sorted[b][hist[b][c][label] + rank] = {row, label}: a stable
//              counting sort with no returning atomics.
//   gather (det_gather_kernel): CTA spans of Pc sorted positions, cut into one
//        span per group of L lanes (lane i holds 16-byte vector i of a row);
//        each group walks its span with P row loads in flight and sums runs in
//        registers in position order. A run that touches neither end of its
//        group span is a whole cluster and is finished on the spot. Runs at
//        the group-span ends meet in shared memory, where warp 0 joins them in
//        group order: a cluster inside the CTA span is finished there; one that
//        reaches across the CTA span's ends leaves a partial in one of the
//        span's two slots, and the last CTA to leave one (a per-cluster
//        counter) adds the cluster's slots in span order and finishes it.
//        Empty clusters are finished too (sums 0, the old centroid kept).
//        "Finished": the sums row; with the finalize also sum / count in IEEE
//        fp32 rounded to the compute dtype, ||new||^2 and its norm slice for the
//        next assignment, and the shift max ||new - old||.
//
// No zero fill of the sums is needed: every row is written exactly once. The
// path takes labels in [0, K) (the assignment's), K <= 65536, rows of 64 to
// 512 bytes in 16-byte aligned buffers.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <atomic>
#include <type_traits>

#include "fkc_common.cuh"
#include "fkc_internal.h"
#include "fkc_launch.cuh"
#include "fkc_ptx.cuh"

namespace fkc {
namespace {

constexpr int kDetMaxK = 65536;
constexpr int kGatherWarps = 8;
constexpr int kGatherThreads = 32 * kGatherWarps;
// CTA spans of the gather: at most kDetMaxSpans per call (plus one per batch
// element), at least kDetMinSpan positions each; this bounds the partial slots.
constexpr int64_t kDetMaxSpans = 4096;
constexpr int kDetMinSpan = 128;
// About kRankChunks chunks per call, at least 64 rows per warp, at most 32768
// rows per chunk (ranks, warp prefixes and chunk totals all fit 16 bits).
constexpr int64_t kRankChunks = 128;
constexpr int64_t kRankMaxRows = 32768;
constexpr int kRankBatch = 16;  // 32-row steps whose labels are loaded together
// Grid barriers of the sort kernel give up after this long (the co-resident
// grid of a cooperative launch reaches them in microseconds).
constexpr uint64_t kSortBarrierNs = 2000000000ull;
enum : int { kErrSortBarrier = 131 };
// Control words of the sort kernel (zeroed when the workspace is prepared; the
// last CTA of every launch sets them back to zero): barrier arrivals, exits,
// abort flag.
enum : int { kCtlArrive = 0, kCtlExit = 1, kCtlAbort = 2 };
constexpr size_t kDetCtlBytes = 256;

__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t m;
  asm volatile("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Chunk geometry of the stable counting sort (host side).
struct DetGeom {
  int W;   // warps (counter rows) per chunk: W * K uint16 counters <= 128 KB
  int RW;  // rows per warp (a multiple of 32)
  int R;   // rows per chunk = W * RW <= 32768
  int C;   // chunks per batch element
};

DetGeom det_geom(int64_t B, int64_t N, int64_t K) {
  DetGeom g;
  g.W = K <= 4096 ? 16 : static_cast<int>(65536 / K);
  if (g.W < 1) g.W = 1;
  const int64_t per_batch = std::max<int64_t>(1, (kRankChunks + B - 1) / B);
  int64_t rw = (N + per_batch * g.W - 1) / (per_batch * g.W);
  rw = std::max<int64_t>(64, (rw + 31) / 32 * 32);
  g.RW = static_cast<int>(std::min<int64_t>(rw, kRankMaxRows / g.W / 32 * 32));
  g.R = g.W * g.RW;
  g.C = static_cast<int>((N + g.R - 1) / g.R);
  return g;
}

int64_t det_max_spans(int64_t B) { return kDetMaxSpans + B; }

// ---------------------------------------------------------------------------
// sort
struct SortArgs {
  const int32_t* ids;
  const int32_t* counts;
  int32_t* hist;     // (B, C, K) chunk histograms, then chunk slot bases
  uint16_t* rank;    // (B, N) stable rank of each row inside its chunk
  int32_t* offsets;  // (B, K)
  int2* sorted;      // (B, N) {row, label} in cluster order
  unsigned* ctl;     // kCtl* words
  int* err;          // device error word (a barrier wait that gave up)
  float* zero_one;   // nullable: zeroed (the shift the gather max-reduces into)
  int B, N, K, RW, R, C, KS, slices_per_batch;
};

// All CTAs of the co-resident grid arrive before any leaves; false when the
// wait gave up (error recorded) or another CTA gave up before.
__device__ bool grid_barrier(const SortArgs& a, unsigned target) {
  __shared__ int ok_s;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(a.ctl + kCtlArrive, 1u);
    int ok = 1;
    const uint64_t t0 = ptx::globaltimer_ns();
    while (ld_acquire_gpu(a.ctl + kCtlArrive) < target) {
      if (ld_acquire_gpu(a.ctl + kCtlAbort) != 0u) {
        ok = 0;
        break;
      }
      if (ptx::globaltimer_ns() - t0 > kSortBarrierNs) {
        atomicExch(a.ctl + kCtlAbort, 1u);
        if (a.err != nullptr) atomicCAS(a.err, 0, kErrSortBarrier);
        ok = 0;
        break;
      }
      __nanosleep(100);
    }
    __threadfence();
    ok_s = ok;
  }
  __syncthreads();
  return ok_s != 0;
}

__device__ void sort_rank_chunk(const SortArgs& a, uint16_t* cnt, int q) {
  const int W = static_cast<int>(blockDim.x >> 5);
  const int warp = static_cast<int>(threadIdx.x >> 5), lane = threadIdx.x & 31;
  const int K = a.K, N = a.N, RW = a.RW, C = a.C;
  const int b = q / C, c = q - b * C;
  {
    uint4* c128 = reinterpret_cast<uint4*>(cnt);
    const int n128 = (W * K * 2 + 15) / 16;
    for (int i = threadIdx.x; i < n128; i += blockDim.x) c128[i] = make_uint4(0u, 0u, 0u, 0u);
  }
  __syncthreads();
  const int64_t rb = static_cast<int64_t>(b) * N;
  const int r0 = c * a.R + warp * RW;
  const int r1 = min(r0 + RW, N);
  uint16_t* my = cnt + warp * K;
  const uint32_t lt = lanemask_lt();
  for (int base = r0; base < r1; base += 32 * kRankBatch) {
    int lab[kRankBatch];
#pragma unroll
    for (int u = 0; u < kRankBatch; ++u) {
      const int row = base + u * 32 + lane;
      const int l = row < r1 ? a.ids[rb + row] : -1;
      lab[u] = (l >= 0 && l < K) ? l : -1;  // labels come from the assignment: in [0, K)
    }
#pragma unroll
    for (int u = 0; u < kRankBatch; ++u) {
      const uint32_t peers = __match_any_sync(0xFFFFFFFFu, lab[u]);
      const int leader = __ffs(peers) - 1;
      int old = 0;
      if (lane == leader && lab[u] >= 0) {
        old = my[lab[u]];
        my[lab[u]] = static_cast<uint16_t>(old + __popc(peers));
      }
      old = __shfl_sync(0xFFFFFFFFu, old, leader);
      if (lab[u] >= 0)
        a.rank[rb + base + u * 32 + lane] = static_cast<uint16_t>(old + __popc(peers & lt));
    }
  }
  __syncthreads();
  // counters -> exclusive prefix over the warps (per label); chunk histogram.
  // With K % 8 == 0 a thread takes 8 labels at once: 16-byte rows of packed
  // 16-bit counters, added as 32-bit pairs (no prefix reaches 2^16: R <= 32768).
  int32_t* h = a.hist + (static_cast<int64_t>(b) * C + c) * K;
  if ((K & 7) == 0) {
    const int K8 = K / 8;
    uint4* c8 = reinterpret_cast<uint4*>(cnt);
    for (int k8 = threadIdx.x; k8 < K8; k8 += blockDim.x) {
      uint4 run = make_uint4(0u, 0u, 0u, 0u);
      for (int w = 0; w < W; ++w) {
        const uint4 v = c8[w * K8 + k8];
        c8[w * K8 + k8] = run;
        run.x += v.x;
        run.y += v.y;
        run.z += v.z;
        run.w += v.w;
      }
      reinterpret_cast<int4*>(h)[2 * k8] =
          make_int4(static_cast<int>(run.x & 0xFFFFu), static_cast<int>(run.x >> 16),
                    static_cast<int>(run.y & 0xFFFFu), static_cast<int>(run.y >> 16));
      reinterpret_cast<int4*>(h)[2 * k8 + 1] =
          make_int4(static_cast<int>(run.z & 0xFFFFu), static_cast<int>(run.z >> 16),
                    static_cast<int>(run.w & 0xFFFFu), static_cast<int>(run.w >> 16));
    }
  } else {
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
      int run = 0;
      for (int w = 0; w < W; ++w) {
        const int v = cnt[w * K + k];
        cnt[w * K + k] = static_cast<uint16_t>(run);
        run += v;
      }
      h[k] = run;
    }
  }
  __syncthreads();
  for (int base = r0; base < r1; base += 32 * kRankBatch) {
    int lab[kRankBatch];
    uint16_t rk[kRankBatch];
#pragma unroll
    for (int u = 0; u < kRankBatch; ++u) {
      const int row = base + u * 32 + lane;
      lab[u] = row < r1 ? a.ids[rb + row] : -1;
      rk[u] = row < r1 ? a.rank[rb + row] : 0;
    }
#pragma unroll
    for (int u = 0; u < kRankBatch; ++u)
      if (lab[u] >= 0 && lab[u] < K)
        a.rank[rb + base + u * 32 + lane] = static_cast<uint16_t>(rk[u] + my[lab[u]]);
  }
  __syncthreads();  // the counters are reused by the next chunk
}

// KS slices of 32 labels of batch row b starting at kbeg; the warps split the chunks.
__device__ void sort_base_slice(const SortArgs& a, int b, int kbeg, int (*part)[32], int* red) {
  const int W = static_cast<int>(blockDim.x >> 5);
  const int warp = static_cast<int>(threadIdx.x >> 5), lane = threadIdx.x & 31;
  const int K = a.K, C = a.C;
  const int32_t* cb = a.counts + static_cast<int64_t>(b) * K;
  int32_t* hb = a.hist + static_cast<int64_t>(b) * C * K;
  // sum of the counts before kbeg (a multiple of 32)
  int s = 0;
  if ((reinterpret_cast<uintptr_t>(cb) & 15u) == 0) {
    const int4* c4 = reinterpret_cast<const int4*>(cb);
    const int n4 = kbeg / 4;
    const int T = static_cast<int>(blockDim.x);
    int i = threadIdx.x;
    for (; i + 3 * T < n4; i += 4 * T) {
      int4 q[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) q[u] = c4[i + u * T];
#pragma unroll
      for (int u = 0; u < 4; ++u) s += q[u].x + q[u].y + q[u].z + q[u].w;
    }
    for (; i < n4; i += T) {
      const int4 q = c4[i];
      s += q.x + q.y + q.z + q.w;
    }
  } else {
    for (int i = threadIdx.x; i < kbeg; i += blockDim.x) s += cb[i];
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
  if (lane == 0) red[warp] = s;
  __syncthreads();
  int carry = 0;
  for (int w = 0; w < W; ++w) carry += red[w];
  const int cpg = (C + W - 1) / W;
  const int c0 = min(C, warp * cpg), c1 = min(C, c0 + cpg);
  for (int sl = 0; sl < a.KS; ++sl) {
    if (kbeg + sl * 32 >= K) break;  // uniform over the CTA
    const int k = kbeg + sl * 32 + lane;
    int tot = 0;
    if (k < K)
      for (int c = c0; c < c1; ++c) tot += hb[static_cast<int64_t>(c) * K + k];
    part[warp][lane] = tot;
    const int ck = k < K ? cb[k] : 0;
    int inc = ck;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xFFFFFFFFu, inc, o);
      if (lane >= o) inc += u;
    }
    const int slice_total = __shfl_sync(0xFFFFFFFFu, inc, 31);
    const int off = carry + inc - ck;
    __syncthreads();
    int run = off;
    for (int w = 0; w < warp; ++w) run += part[w][lane];
    if (warp == 0 && k < K) a.offsets[static_cast<int64_t>(b) * K + k] = off;
    if (k < K)
      for (int c = c0; c < c1; ++c) {
        int32_t* p = hb + static_cast<int64_t>(c) * K + k;
        const int v = *p;
        *p = run;
        run += v;
      }
    carry += slice_total;
    __syncthreads();  // part[] is rewritten by the next slice
  }
}

// One cooperative launch (every CTA co-resident): rank all chunks -> barrier ->
// bases -> barrier -> scatter. blockDim.x = 32 * W, dynamic shared memory W * K
// 16-bit counters.
__global__ void __launch_bounds__(512) det_sort_kernel(const SortArgs a) {
  extern __shared__ uint16_t cnt[];  // [W][K]
  __shared__ int part[16][32];
  __shared__ int red[16];
  const unsigned G = gridDim.x;
  if (a.zero_one != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *a.zero_one = 0.f;
  for (int q = blockIdx.x; q < a.B * a.C; q += G) sort_rank_chunk(a, cnt, q);
  bool ok = grid_barrier(a, G);
  if (ok) {
    for (int s = blockIdx.x; s < a.B * a.slices_per_batch; s += G) {
      const int b = s / a.slices_per_batch;
      sort_base_slice(a, b, (s - b * a.slices_per_batch) * 32 * a.KS, part, red);
      __syncthreads();  // red[] is rewritten by the next slice
    }
    ok = grid_barrier(a, 2 * G);
  }
  if (ok) {
    const int64_t total = static_cast<int64_t>(a.B) * a.N;
    const int64_t stride = static_cast<int64_t>(G) * blockDim.x;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += stride) {
      const int b = static_cast<int>(static_cast<uint32_t>(i) / static_cast<uint32_t>(a.N));
      const int n = static_cast<int>(i - static_cast<int64_t>(b) * a.N);
      const int lab = a.ids[i];
      if (lab < 0 || lab >= a.K) continue;
      const int pos = a.hist[(static_cast<int64_t>(b) * a.C + n / a.R) * a.K + lab] + a.rank[i];
      if (pos < 0 || pos >= a.N) continue;  // counts inconsistent with the labels: drop
      a.sorted[static_cast<int64_t>(b) * a.N + pos] = make_int2(n, lab);
    }
  }
  // The last CTA out sets the control words back to zero for the next launch
  // (every CTA has left both barriers by then).
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(a.ctl + kCtlExit, 1u) == G - 1) {
      a.ctl[kCtlArrive] = 0u;
      a.ctl[kCtlExit] = 0u;
      a.ctl[kCtlAbort] = 0u;
      __threadfence();
    }
  }
}

// ---------------------------------------------------------------------------
// gather
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

template <typename T>
__device__ __forceinline__ void add_vec(float (&acc)[16 / sizeof(T)], const uint4& u) {
  if constexpr (sizeof(T) == 4) {
    acc[0] += __uint_as_float(u.x);
    acc[1] += __uint_as_float(u.y);
    acc[2] += __uint_as_float(u.z);
    acc[3] += __uint_as_float(u.w);
  } else {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float2 f;
      if constexpr (std::is_same<T, __half>::value)
        f = __half22float2(*reinterpret_cast<const __half2*>(&w[k]));
      else
        f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[k]));
      acc[2 * k] += f.x;
      acc[2 * k + 1] += f.y;
    }
  }
}

__device__ __forceinline__ void add4(float4& a, const float4& v) {
  a.x += v.x;
  a.y += v.y;
  a.z += v.z;
  a.w += v.w;
}

template <typename T>
struct GatherArgs {
  const T* x;
  const int2* sorted;
  const int32_t* counts;
  const int32_t* offsets;
  float* sums;
  float* part;    // (spans, 2, D) partial sums at CTA-span ends
  int32_t* done;  // (B, K) slots arrived per split cluster (zero between launches)
  const T* old_c;  // FINAL: old centroids (may alias new_c)
  T* new_c;
  float* c_sq;     // nullable
  uint8_t* cext;   // nullable
  float* shift;    // nullable (zeroed by the sort kernel)
  int B, N, K, Pc, ncta;
  int64_t spans;
};

// Finishes elements [e0, e0 + 4) of cluster row kg: the sums entry and, with
// FINAL, the new centroid (sum / count rounded to T; the old value when the
// cluster is empty) and this part's ||new||^2 and ||new - old||^2.
template <typename T, int D, bool FINAL>
__device__ __forceinline__ void finish4(const GatherArgs<T>& a, int64_t kg, int e0, const float4& v,
                                        int cnt, float& sq, float& sh) {
  *reinterpret_cast<float4*>(a.sums + kg * D + e0) = v;
  if constexpr (FINAL) {
    using V = typename std::conditional<sizeof(T) == 2, uint2, uint4>::type;  // 4 elements
    const V ov = *reinterpret_cast<const V*>(a.old_c + kg * D + e0);
    const T* o = reinterpret_cast<const T*>(&ov);
    V nvv;
    T* nv = reinterpret_cast<T*>(&nvv);
    const float s4[4] = {v.x, v.y, v.z, v.w};
    const float fc = static_cast<float>(cnt);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      nv[e] = cnt > 0 ? from_f32<T>(__fdiv_rn(s4[e], fc)) : o[e];
      const float nf = to_f32<T>(nv[e]);
      const float df = nf - to_f32<T>(o[e]);
      sq = fmaf(nf, nf, sq);
      sh = fmaf(df, df, sh);
    }
    *reinterpret_cast<V*>(a.new_c + kg * D + e0) = nvv;
  }
}

template <typename T>
__device__ __forceinline__ void finish_norms(const GatherArgs<T>& a, int64_t kg, float sq, float sh,
                                             float& shift_max) {
  if (a.c_sq != nullptr) a.c_sq[kg] = sq;
  if (a.cext != nullptr) write_norm_ext(a.cext + kg * kNormExtBytes, -0.5f * sq, false);
  shift_max = fmaxf(shift_max, sqrtf(sh));
}

template <typename T, int L, int P, bool FINAL>
__global__ void __launch_bounds__(kGatherThreads, 4) det_gather_kernel(const GatherArgs<T> a) {
  constexpr int kVec = 16 / sizeof(T);
  constexpr int G = 32 / L;
  constexpr int NG = kGatherWarps * G;  // group spans per CTA span
  constexpr int D = L * kVec;
  constexpr int kCols = D / 4;                       // float4 columns of a row
  constexpr int CPL = kCols > 32 ? kCols / 32 : 1;   // columns per lane of warp 0 in the join
  static_assert(32 % L == 0 && L % P == 0 && L >= 4, "group layout");
  static_assert(kCols <= 32 || kCols % 32 == 0, "join columns");
  __shared__ int2 ends[NG];  // (label of the run at the group-span start, at the end or -1)
  __shared__ __align__(16) float first_acc[NG][D];
  __shared__ __align__(16) float last_acc[NG][D];
  __shared__ float block_max[kGatherWarps];
  const int lane = threadIdx.x & 31, warp = static_cast<int>(threadIdx.x >> 5);
  const int g = lane / L, i = lane % L;
  const uint32_t gmask = L == 32 ? 0xFFFFFFFFu : (((1u << L) - 1u) << (g * L));
  const int j = warp * G + g;  // group index in the CTA
  const int Sg = a.Pc / NG;    // Pc is a multiple of NG
  const int K = a.K, N = a.N;
  const int64_t BK = static_cast<int64_t>(a.B) * K;
  float shift_max = 0.f;
  pdl_wait();

  // A whole cluster summed by this group (lane i holds elements i*kVec ..).
  auto finish_group = [&](int64_t kg, const float (&acc)[kVec], int cnt) {
    float sq = 0.f, sh = 0.f;
#pragma unroll
    for (int v = 0; v < kVec; v += 4)
      finish4<T, D, FINAL>(a, kg, i * kVec + v, make_float4(acc[v], acc[v + 1], acc[v + 2], acc[v + 3]),
                           cnt, sq, sh);
    if constexpr (FINAL) {
#pragma unroll
      for (int o = L / 2; o >= 1; o >>= 1) {
        sq += __shfl_xor_sync(gmask, sq, o);
        sh += __shfl_xor_sync(gmask, sh, o);
      }
      if (i == 0) finish_norms(a, kg, sq, sh, shift_max);
    }
  };
  // A cluster held by warp 0 in the join (lane: float4 columns lane + 32 u).
  auto finish_warp = [&](int64_t kg, const float4 (&acc)[CPL], int cnt) {
    float sq = 0.f, sh = 0.f;
#pragma unroll
    for (int u = 0; u < CPL; ++u) {
      const int t = lane + 32 * u;
      if (t < kCols) finish4<T, D, FINAL>(a, kg, 4 * t, acc[u], cnt, sq, sh);
    }
    if constexpr (FINAL) {
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) {
        sq += __shfl_xor_sync(0xFFFFFFFFu, sq, o);
        sh += __shfl_xor_sync(0xFFFFFFFFu, sh, o);
      }
      if (lane == 0) finish_norms(a, kg, sq, sh, shift_max);
    }
  };

  // Empty clusters: no sorted position belongs to them.
  for (int64_t u0 = (static_cast<int64_t>(blockIdx.x) * kGatherWarps + warp) * G; u0 < BK;
       u0 += static_cast<int64_t>(gridDim.x) * kGatherWarps * G) {
    const int64_t kg = u0 + g;
    if (kg < BK && a.counts[kg] == 0) {  // uniform over the group
      float z[kVec];
#pragma unroll
      for (int v = 0; v < kVec; ++v) z[v] = 0.f;
      finish_group(kg, z, 0);
    }
  }

  for (int64_t cs = blockIdx.x; cs < a.spans; cs += gridDim.x) {
    const int b = static_cast<int>(cs / a.ncta);
    const int S0 = static_cast<int>(cs - static_cast<int64_t>(b) * a.ncta) * a.Pc;
    const int S1 = min(S0 + a.Pc, N);
    const int p0 = min(S0 + j * Sg, S1);
    const int p1 = min(p0 + Sg, S1);
    const int64_t rb = static_cast<int64_t>(b) * N;
    const T* xb = a.x + rb * D + i * kVec;
    // meta of positions m .. m + L - 1 (lane i: position m + i)
    auto load_meta = [&](int m, int& lab, int& src) {
      const int q = m + i;
      const int2 e = q < p1 ? __ldg(a.sorted + rb + q) : make_int2(0, -1);
      // labels outside [0, K) or rows outside [0, N) never occur on this path; such an
      // entry would read nothing
      const bool ok = e.y >= 0 && e.y < K && e.x >= 0 && e.x < N;
      lab = ok ? e.y : -1;
      src = ok ? e.x : 0;
    };
    auto at = [&](int v, int jj) { return __shfl_sync(gmask, v, g * L + jj); };
    int labA, srcA, labB, srcB;
    load_meta(p0, labA, srcA);
    load_meta(p0 + L, labB, srcB);
    uint4 buf[P];
#pragma unroll
    for (int q = 0; q < P; ++q) {
      const int l = at(labA, q), s = at(srcA, q);
      if (l >= 0) buf[q] = ld_stream_v4(xb + static_cast<size_t>(s) * D);
    }
    float acc[kVec];
#pragma unroll
    for (int v = 0; v < kVec; ++v) acc[v] = 0.f;
    int cur = -1, run_start = p0, first_lab = -1, last_lab = -1;
    // Hands a finished run over: a whole cluster -> its sums row (finished
    // after the walk); the run at the span start -> shared memory (first), the
    // run at the span end -> (last).
    auto flush = [&](bool at_end) {
      if (cur < 0) return;
      const bool at_start = run_start == p0;
      float* dst = (!at_start && !at_end)
                       ? a.sums + (static_cast<int64_t>(b) * K + cur) * D + i * kVec
                       : (at_start ? &first_acc[j][i * kVec] : &last_acc[j][i * kVec]);
#pragma unroll
      for (int v = 0; v < kVec; v += 4)
        *reinterpret_cast<float4*>(dst + v) = make_float4(acc[v], acc[v + 1], acc[v + 2], acc[v + 3]);
    };
    for (int m = p0; m < p1; m += L) {
#pragma unroll
      for (int jj = 0; jj < L; ++jj) {
        const int q = m + jj;
        if (q < p1) {
          const int l = at(labA, jj);
          if (l != cur) {
            flush(false);
            if (run_start == p0 && cur >= 0 && first_lab < 0) first_lab = cur;
#pragma unroll
            for (int v = 0; v < kVec; ++v) acc[v] = 0.f;
            cur = l;
            run_start = q;
          }
          if (l >= 0) add_vec<T>(acc, buf[jj % P]);
          const int jn = jj + P;  // the position whose row load goes out now
          const int ln = jn < L ? at(labA, jn % L) : at(labB, jn - L);
          const int sn = jn < L ? at(srcA, jn % L) : at(srcB, jn - L);
          if (ln >= 0) buf[jj % P] = ld_stream_v4(xb + static_cast<size_t>(sn) * D);
        }
      }
      labA = labB;
      srcA = srcB;
      load_meta(m + 2 * L, labB, srcB);
    }
    if (cur >= 0) {  // the run reaching the span end
      if (run_start == p0)
        first_lab = cur;  // one run covers the whole span
      else
        last_lab = cur;
      flush(true);
    }
    if (i == 0) ends[j] = make_int2(first_lab, last_lab);
    if constexpr (FINAL) {
      // Finish the clusters that lie inside this group span: the runs that
      // start after p0, except the last one (their sums rows, stored above by
      // these lanes, are read back).
      int pend = -1;
      for (int m = p0; m < p1; m += L) {
        const int q = m + i;
        const int lab = q < p1 ? __ldg(a.sorted + rb + q).y : -1;
        const int prv = (q > p0 && q < p1) ? __ldg(a.sorted + rb + q - 1).y : -1;
        uint32_t starts = __ballot_sync(gmask, q > p0 && q < p1 && lab != prv);
        starts = L == 32 ? starts : (starts >> (g * L)) & ((1u << L) - 1u);
        while (starts != 0u) {
          const int jj = __ffs(starts) - 1;
          starts &= starts - 1u;
          if (pend >= 0) {
            const int64_t kg = static_cast<int64_t>(b) * K + pend;
            float v8[kVec];
            const float* srow = a.sums + kg * D + i * kVec;
#pragma unroll
            for (int v = 0; v < kVec; v += 4) {
              const float4 f = *reinterpret_cast<const float4*>(srow + v);
              v8[v] = f.x;
              v8[v + 1] = f.y;
              v8[v + 2] = f.z;
              v8[v + 3] = f.w;
            }
            finish_group(kg, v8, a.counts[kg]);
          }
          pend = __shfl_sync(gmask, lab, g * L + jj);
        }
      }
    }
    __syncthreads();
    // CTA join of the group-span ends, in group order (warp 0).
    if (warp == 0) {
      const int lab_before = S0 > 0 ? a.sorted[rb + S0 - 1].y : -1;
      const int lab_after = S1 < N ? a.sorted[rb + S1].y : -1;
      int c_lab = -1;
      bool c_start = false;  // the carried run began at the CTA span start
      float4 c_acc[CPL];
#pragma unroll
      for (int u = 0; u < CPL; ++u) c_acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      auto emit = [&](bool at_cta_end) {
        if (c_lab < 0) return;
        const bool before = c_start && lab_before == c_lab;
        const bool after = at_cta_end && lab_after == c_lab;
        const int64_t kg = static_cast<int64_t>(b) * K + c_lab;
        if (!before && !after) {  // the whole cluster lies in this CTA span
          finish_warp(kg, c_acc, FINAL ? a.counts[kg] : 0);
          return;
        }
        float4* slot = reinterpret_cast<float4*>(a.part + (cs * 2 + (before ? 0 : 1)) * D);
#pragma unroll
        for (int u = 0; u < CPL; ++u) {
          const int t = lane + 32 * u;
          if (t < kCols) slot[t] = c_acc[u];
        }
        __threadfence();
        __syncwarp();
        int last = 0, cnt = 0, ca = 0, cb = 0;
        if (lane == 0) {
          cnt = a.counts[kg];
          // counts consistent with the labels keep the segment inside [0, N)
          const int cs0 = min(max(a.offsets[kg], 0), N - 1);
          ca = cs0 / a.Pc;
          cb = (min(cs0 + cnt, N) - 1) / a.Pc;
          last = atomicAdd(a.done + kg, 1) == cb - ca ? 1 : 0;
        }
        last = __shfl_sync(0xFFFFFFFFu, last, 0);
        if (!last) return;
        // the last span in: add the cluster's slots in span order and finish it
        cnt = __shfl_sync(0xFFFFFFFFu, cnt, 0);
        ca = __shfl_sync(0xFFFFFFFFu, ca, 0);
        cb = __shfl_sync(0xFFFFFFFFu, cb, 0);
        __threadfence();
        const int64_t sb = static_cast<int64_t>(b) * a.ncta;
        float4 sum[CPL];
#pragma unroll
        for (int u = 0; u < CPL; ++u) {
          const int t = lane + 32 * u;
          sum[u] = t < kCols ? __ldcg(reinterpret_cast<const float4*>(a.part + ((sb + ca) * 2 + 1) * D) + t)
                             : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        for (int c = ca + 1; c <= cb; c += 4) {
          float4 f[4][CPL];
#pragma unroll
          for (int w = 0; w < 4; ++w)
#pragma unroll
            for (int u = 0; u < CPL; ++u) {
              const int t = lane + 32 * u;
              f[w][u] = (c + w <= cb && t < kCols)
                            ? __ldcg(reinterpret_cast<const float4*>(a.part + ((sb + c + w) * 2) * D) + t)
                            : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
          for (int w = 0; w < 4; ++w)
            if (c + w <= cb)
#pragma unroll
              for (int u = 0; u < CPL; ++u) add4(sum[u], f[w][u]);
        }
        finish_warp(kg, sum, cnt);
        if (lane == 0) a.done[kg] = 0;
      };
      for (int jj = 0; jj < NG; ++jj) {
        const int2 e = ends[jj];
        if (e.x < 0) continue;  // empty group span (past the end of the positions)
        if (e.x == c_lab) {
#pragma unroll
          for (int u = 0; u < CPL; ++u) {
            const int t = lane + 32 * u;
            if (t < kCols) add4(c_acc[u], reinterpret_cast<const float4*>(first_acc[jj])[t]);
          }
        } else {
          emit(false);
          c_lab = e.x;
          c_start = jj == 0;
#pragma unroll
          for (int u = 0; u < CPL; ++u) {
            const int t = lane + 32 * u;
            c_acc[u] = t < kCols ? reinterpret_cast<const float4*>(first_acc[jj])[t]
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
          }
        }
        if (e.y >= 0) {  // the first run ended inside this group span
          emit(false);
          c_lab = e.y;
          c_start = false;
#pragma unroll
          for (int u = 0; u < CPL; ++u) {
            const int t = lane + 32 * u;
            c_acc[u] = t < kCols ? reinterpret_cast<const float4*>(last_acc[jj])[t]
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
          }
        }
      }
      emit(true);
    }
    __syncthreads();  // ends[] and the run ends are rewritten by the next span
  }
  if (FINAL && a.shift != nullptr) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1)
      shift_max = fmaxf(shift_max, __shfl_xor_sync(0xFFFFFFFFu, shift_max, o));
    if (lane == 0) block_max[warp] = shift_max;
    __syncthreads();
    if (threadIdx.x == 0) {
      float m = 0.f;
#pragma unroll
      for (int w = 0; w < kGatherWarps; ++w) m = fmaxf(m, block_max[w]);
      atomicMax(reinterpret_cast<unsigned int*>(a.shift), __float_as_uint(m));
    }
  }
}

int det_sm_count() {
  const DeviceInfo* di = nullptr;
  if (current_device_info(&di) == FKC_OK) return di->sm_count;
  return 148;
}

int64_t row_lanes(int64_t D, int dtype) { return D * static_cast<int64_t>(dtype_size(dtype)) / 16; }

bool det_shape_ok(int64_t N, int64_t K, int64_t D, int dtype) {
  if (K < 1 || K > kDetMaxK || N < 1) return false;
  if ((D * static_cast<int64_t>(dtype_size(dtype))) % 16 != 0) return false;
  const int64_t L = row_lanes(D, dtype);
  return L == 4 || L == 8 || L == 16 || L == 32;
}

// CTA-span length of the gather: about one span per resident CTA (at least
// kDetMinSpan positions, at most kDetMaxSpans spans), a multiple of the group
// count NG so every group span has the same length.
int det_span_len(int64_t B, int64_t N, int NG, int resident) {
  const int64_t target = std::max<int64_t>(1, std::min<int64_t>(resident, kDetMaxSpans));
  int64_t pc = std::max<int64_t>(kDetMinSpan, (B * N + target - 1) / target);
  pc = std::max<int64_t>(pc, (B * N + kDetMaxSpans - 1) / kDetMaxSpans);
  pc = (pc + NG - 1) / NG * NG;
  // fewer spans than resident CTAs where the rounding per batch row adds some
  while (B * ((N + pc - 1) / pc) > std::max<int64_t>(target, B) && pc < N) pc += NG;
  return static_cast<int>(std::min<int64_t>(pc, (N + NG - 1) / NG * NG));
}

// Resident CTAs of a kernel (persistent grids).
template <typename Kern>
int det_resident(Kern kern, int threads, size_t smem) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem) != cudaSuccess ||
      per_sm < 1) {
    cudaGetLastError();
    per_sm = 1;
  }
  return per_sm * det_sm_count();
}

template <typename T, int L, bool FINAL>
int launch_gather(const GatherArgs<T>& proto, int64_t B, int64_t N, cudaStream_t stream) {
  constexpr int P = L >= 8 ? 8 : L;
  constexpr int NG = kGatherWarps * (32 / L);
  auto kern = det_gather_kernel<T, L, P, FINAL>;
  static std::atomic<int> res_cache{0};  // same value on every device of one model
  int res = res_cache.load(std::memory_order_relaxed);
  if (res == 0) {
    res = det_resident(kern, kGatherThreads, 0);
    res_cache.store(res, std::memory_order_relaxed);
  }
  GatherArgs<T> a = proto;
  a.Pc = det_span_len(B, N, NG, res);
  a.ncta = static_cast<int>((N + a.Pc - 1) / a.Pc);
  a.spans = B * a.ncta;
  FKC_REQUIRE(a.spans <= det_max_spans(B), "update: %lld spans exceed the partial slots",
              static_cast<long long>(a.spans));
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(a.spans, res));
  return launch_pdl(kern, dim3(grid), dim3(kGatherThreads), 0, stream, a);
}

template <typename T>
int launch_gather_dtype(const GatherArgs<T>& a, int64_t B, int64_t N, int64_t D, bool final_,
                        cudaStream_t stream) {
  switch (static_cast<int>(D * sizeof(T) / 16)) {
#define FKC_DET(L_)                                                                    \
  case L_:                                                                             \
    return final_ ? launch_gather<T, L_, true>(a, B, N, stream)                        \
                  : launch_gather<T, L_, false>(a, B, N, stream);
    FKC_DET(4)
    FKC_DET(8)
    FKC_DET(16)
    FKC_DET(32)
#undef FKC_DET
    default:
      return set_error(FKC_EINVAL, "update: unsupported row size (D=%lld)",
                       static_cast<long long>(D));
  }
}

template <typename T>
int launch_det_gather(const void* x, const int32_t* counts, const UpdateWorkspace& uw,
                      const DetWorkspace& dw, int32_t* done, float* sums, const void* old_c,
                      void* new_c, float* c_sq, void* cext, float* shift, int64_t B, int64_t N,
                      int64_t K, int64_t D, cudaStream_t stream) {
  GatherArgs<T> a{};
  a.x = static_cast<const T*>(x);
  a.sorted = reinterpret_cast<const int2*>(uw.perm);
  a.counts = counts;
  a.offsets = uw.offsets;
  a.sums = sums;
  a.part = dw.part;
  a.done = done;
  a.old_c = static_cast<const T*>(old_c);
  a.new_c = static_cast<T*>(new_c);
  a.c_sq = c_sq;
  a.cext = static_cast<uint8_t*>(cext);
  a.shift = shift;
  a.B = static_cast<int>(B);
  a.N = static_cast<int>(N);
  a.K = static_cast<int>(K);
  return launch_gather_dtype<T>(a, B, N, D, old_c != nullptr, stream);
}

}  // namespace

size_t det_update_bytes(int64_t B, int64_t N, int64_t K, int64_t D, int dtype) {
  if (!det_shape_ok(N, K, D, dtype)) return 0;
  const DetGeom g = det_geom(B, N, K);
  return kDetCtlBytes + align_up(static_cast<size_t>(B * N) * 2, 256) +
         align_up(static_cast<size_t>(B) * g.C * K * 4, 256) +
         align_up(static_cast<size_t>(det_max_spans(B)) * 2 * D * 4, 256);
}

DetWorkspace carve_det(void* ws, int64_t B, int64_t N, int64_t K, int64_t D, int dtype) {
  DetWorkspace w{};
  if (!det_shape_ok(N, K, D, dtype)) return w;
  const DetGeom g = det_geom(B, N, K);
  uint8_t* p = static_cast<uint8_t*>(ws);
  w.ctl = reinterpret_cast<unsigned*>(p);
  p += kDetCtlBytes;
  w.rank = reinterpret_cast<uint16_t*>(p);
  p += align_up(static_cast<size_t>(B * N) * 2, 256);
  w.hist = reinterpret_cast<int32_t*>(p);
  p += align_up(static_cast<size_t>(B) * g.C * K * 4, 256);
  w.part = reinterpret_cast<float*>(p);
  return w;
}

size_t det_ctl_bytes() { return kDetCtlBytes; }

bool det_update_ok(const DetWorkspace& dw, const void* x, const float* sums, const void* old_c,
                   const void* new_c, int64_t B, int64_t N, int64_t K, int64_t D, int dtype) {
  if (dw.rank == nullptr || !det_shape_ok(N, K, D, dtype)) return false;
  if (B * N > 2147483647ll || B * K > 2147483647ll) return false;
  auto al = [](const void* p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  return x != nullptr && sums != nullptr && al(x) && al(sums) && al(old_c) && al(new_c);
}

int launch_det_update(const void* x, const int32_t* ids, const int32_t* counts,
                      const UpdateWorkspace& uw, const DetWorkspace& dw, int32_t* done,
                      float* sums, const void* old_c, void* new_c, float* c_sq, void* cext,
                      float* shift, int64_t B, int64_t N, int64_t K, int64_t D, int dtype,
                      cudaStream_t stream) {
  FKC_REQUIRE(B * N <= 2147483647ll && B * K <= 2147483647ll, "update: sizes out of range");
  const DetGeom g = det_geom(B, N, K);
  FKC_REQUIRE(g.R <= kRankMaxRows && g.RW >= 32, "update: chunk of %d rows", g.R);
  // ---- sort: one cooperative launch
  SortArgs sa{};
  sa.ids = ids;
  sa.counts = counts;
  sa.hist = dw.hist;
  sa.rank = dw.rank;
  sa.offsets = uw.offsets;
  sa.sorted = reinterpret_cast<int2*>(uw.perm);
  sa.ctl = dw.ctl;
  sa.err = device_error_word();
  sa.zero_one = (old_c != nullptr) ? shift : nullptr;
  sa.B = static_cast<int>(B);
  sa.N = static_cast<int>(N);
  sa.K = static_cast<int>(K);
  sa.RW = g.RW;
  sa.R = g.R;
  sa.C = g.C;
  const int64_t slices = (K + 31) / 32;
  sa.KS = static_cast<int>(std::max<int64_t>(1, (slices + 255) / 256));
  sa.slices_per_batch = static_cast<int>((slices + sa.KS - 1) / sa.KS);
  const int threads = 32 * g.W;
  const size_t smem = align_up(static_cast<size_t>(g.W) * K * 2, 16);
  FKC_CUDA_TRY(cudaFuncSetAttribute(det_sort_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(std::max<size_t>(smem, 1))));
  int per_sm = 0;
  FKC_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, det_sort_kernel, threads, smem));
  FKC_REQUIRE(per_sm >= 1, "update: the sort kernel does not fit an SM (K=%lld)",
              static_cast<long long>(K));
  const int64_t work = std::max<int64_t>(B * g.C, B * sa.slices_per_batch);
  const int grid = static_cast<int>(std::min<int64_t>(static_cast<int64_t>(per_sm) * det_sm_count(),
                                                      std::max<int64_t>(work, 1)));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(static_cast<unsigned>(threads));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA co-resident: the grid barriers end
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  FKC_CUDA_TRY(cudaLaunchKernelEx(&cfg, det_sort_kernel, sa));
  count_launches(1);
  // ---- gather (+ join of split clusters, empty clusters, finalize)
  switch (dtype) {
    case FKC_DTYPE_F16:
      return launch_det_gather<__half>(x, counts, uw, dw, done, sums, old_c, new_c, c_sq, cext,
                                       shift, B, N, K, D, stream);
    case FKC_DTYPE_BF16:
      return launch_det_gather<__nv_bfloat16>(x, counts, uw, dw, done, sums, old_c, new_c, c_sq,
                                              cext, shift, B, N, K, D, stream);
    case FKC_DTYPE_F32:
      return launch_det_gather<float>(x, counts, uw, dw, done, sums, old_c, new_c, c_sq, cext,
                                      shift, B, N, K, D, stream);
    default:
      return set_error(FKC_EINVAL, "update: bad dtype %d", dtype);
  }
}

}  // namespace fkc
