// Deterministic centroid update of the Lloyd step: a stable counting sort of
// the labels, a span gather that sums every cluster in sorted order, and a
// fixed-order combine of the clusters that cross span boundaries, with the
// finalize fused into it.
//
// The reference sorts labels with torch.sort and accumulates sorted runs with
// one fp32 atomicAdd per run and feature (flash_kmeans_cuda/ops.py:89-111,
// csrc/update/update_sorted.cu:118-186); the order of those atomics, and so the
// last bits of its sums, change from run to run. Here every float addition
// happens in an order fixed by the labels and the launch geometry, so two runs
// on the same device give bit-identical sums and centroids:
//
//   rank     (det_rank_kernel)    rows in chunks of R; inside a chunk each warp
//            walks its slice of rows in order and counts labels in its own
//            shared-memory row of counters (match_any gives ranks inside a
//            32-row step), so every row gets its stable rank inside the chunk;
//            the chunk's histogram goes to hist[b][c][:].
//   base     (det_base_kernel)    base[b][c][k] = offsets[b][k] + sum over the
//            earlier chunks of hist[b][c'][k] (in place), offsets = exclusive
//            scan of the counts (which the assignment kernel produced).
//   scatter  (det_scatter_kernel) sorted[base + rank] = {row, label}: a stable
//            counting sort with no returning atomics, one 8-byte store per row.
//   gather   (det_gather_kernel)  CTA spans of Pc sorted positions, cut into one
//            span per group of L lanes (lane i holds 16-byte vector i of a row);
//            each group walks its span with P row loads in flight and sums runs
//            in registers in position order. A run that does not touch either
//            end of its group span is a whole cluster: its sums row is stored.
//            The runs at the span ends go to shared memory and the CTA joins
//            them across its groups in order; a run that reaches across the
//            CTA span's ends leaves a partial in one of the span's two slots.
//   fixup    (det_fixup_kernel)   one group per cluster: a cluster split over
//            CTA spans a..b is slot1[a] + slot0[a+1] + ... + slot0[b] (in that
//            order); an empty cluster gets a zero row. With FINAL it also
//            finishes every cluster: sum / count in IEEE fp32 rounded to the
//            compute dtype (the old centroid when empty), ||new||^2 and its norm
//            slice for the next assignment, and the shift max ||new - old||.
//
// No zero fill of the sums is needed: every row is written exactly once. The
// path takes labels in [0, K) (the assignment's), K <= 65536, rows of 64 to
// 512 bytes in 16-byte aligned buffers.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <atomic>

#include "fkc_common.cuh"
#include "fkc_internal.h"
#include "fkc_launch.cuh"

namespace fkc {
namespace {

constexpr int kDetMaxK = 65536;
constexpr int kGatherWarps = 8;
constexpr int kGatherThreads = 32 * kGatherWarps;
// CTA spans: at most kDetMaxSpans per call (plus one per batch element), at
// least kDetMinSpan positions each; this bounds the partial slots.
constexpr int64_t kDetMaxSpans = 4096;
constexpr int kDetMinSpan = 128;

__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t m;
  asm volatile("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// Chunk geometry of the stable counting sort (same on host and device).
struct DetGeom {
  int W;   // warps (counter rows) per chunk CTA: W * K uint16 counters <= 128 KB
  int RW;  // rows per warp (a multiple of 32)
  int R;   // rows per chunk = W * RW <= 32768: ranks, prefixes and totals fit 16 bits
  int C;   // chunks per batch element
};

// About kRankChunks chunk CTAs per call (one wave on 148 SMs), each at least
// 64 rows per warp; at most 32768 rows per chunk, so that ranks, warp prefixes
// and chunk totals all fit 16 bits.
constexpr int64_t kRankChunks = 128;
constexpr int64_t kRankMaxRows = 32768;

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
// rank: stable ranks inside a chunk + the chunk's histogram. A warp's rows are
// taken in batches of kRankBatch 32-row steps whose labels are loaded together
// (one memory round trip per batch), then counted step by step in order.
constexpr int kRankBatch = 16;

__global__ void __launch_bounds__(512) det_rank_kernel(const int32_t* __restrict__ ids, int N,
                                                       int K, int RW, int C,
                                                       int32_t* __restrict__ hist,
                                                       uint16_t* __restrict__ rank,
                                                       float* zero_one) {
  extern __shared__ uint16_t cnt[];  // [W][K]
  const int W = static_cast<int>(blockDim.x >> 5);
  const int warp = static_cast<int>(threadIdx.x >> 5), lane = threadIdx.x & 31;
  const int b = blockIdx.x / C, c = blockIdx.x - b * C;
  {
    // zero the counters (independent of the previous kernel)
    uint4* c128 = reinterpret_cast<uint4*>(cnt);
    const int n128 = (W * K * 2 + 15) / 16;
    for (int i = threadIdx.x; i < n128; i += blockDim.x) c128[i] = make_uint4(0u, 0u, 0u, 0u);
  }
  __syncthreads();
  pdl_wait();
  if (zero_one != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *zero_one = 0.f;
  const int64_t rb = static_cast<int64_t>(b) * N;
  const int r0 = c * (W * RW) + warp * RW;
  const int r1 = min(r0 + RW, N);
  uint16_t* my = cnt + warp * K;
  const uint32_t lt = lanemask_lt();
  for (int base = r0; base < r1; base += 32 * kRankBatch) {
    int lab[kRankBatch];
#pragma unroll
    for (int u = 0; u < kRankBatch; ++u) {
      const int row = base + u * 32 + lane;
      const int l = row < r1 ? ids[rb + row] : -1;
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
        rank[rb + base + u * 32 + lane] = static_cast<uint16_t>(old + __popc(peers & lt));
    }
  }
  __syncthreads();
  // counters -> exclusive prefix over the warps (per label); chunk histogram.
  // With K % 8 == 0 a thread takes 8 labels at once: 16-byte rows of packed
  // 16-bit counters, added as 32-bit pairs (a prefix is below R <= 65536, so no
  // carry crosses a half).
  int32_t* h = hist + (static_cast<int64_t>(b) * C + c) * K;
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
      const uint32_t q[4] = {run.x, run.y, run.z, run.w};
      int4 lo, hi;
      lo.x = static_cast<int>(q[0] & 0xFFFFu); lo.y = static_cast<int>(q[0] >> 16);
      lo.z = static_cast<int>(q[1] & 0xFFFFu); lo.w = static_cast<int>(q[1] >> 16);
      hi.x = static_cast<int>(q[2] & 0xFFFFu); hi.y = static_cast<int>(q[2] >> 16);
      hi.z = static_cast<int>(q[3] & 0xFFFFu); hi.w = static_cast<int>(q[3] >> 16);
      reinterpret_cast<int4*>(h)[2 * k8] = lo;
      reinterpret_cast<int4*>(h)[2 * k8 + 1] = hi;
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
      lab[u] = row < r1 ? ids[rb + row] : -1;
      rk[u] = row < r1 ? rank[rb + row] : 0;
    }
#pragma unroll
    for (int u = 0; u < kRankBatch; ++u)
      if (lab[u] >= 0 && lab[u] < K)
        rank[rb + base + u * 32 + lane] = static_cast<uint16_t>(rk[u] + my[lab[u]]);
  }
}

// ---------------------------------------------------------------------------
// base: offsets (exclusive scan of counts) and per-chunk slot bases, in place.
// A CTA handles KS slices of 32 labels of one batch element; its 8 warps
// split the chunks.
__global__ void __launch_bounds__(256) det_base_kernel(const int32_t* __restrict__ counts,
                                                       int32_t* __restrict__ hist,
                                                       int32_t* __restrict__ offsets, int K,
                                                       int C, int KS, int ctas_per_batch) {
  __shared__ int part[8][32];
  __shared__ int red[8];
  pdl_wait();
  const int b = blockIdx.x / ctas_per_batch;
  const int kbeg = (blockIdx.x - b * ctas_per_batch) * (32 * KS);
  const int lane = threadIdx.x & 31, grp = threadIdx.x >> 5;
  const int32_t* cb = counts + static_cast<int64_t>(b) * K;
  int32_t* hb = hist + static_cast<int64_t>(b) * C * K;
  // sum of the counts before this CTA's labels (kbeg is a multiple of 32: whole
  // 16-byte vectors when the row of counts is 16-byte aligned)
  int s = 0;
  if ((reinterpret_cast<uintptr_t>(cb) & 15u) == 0) {
    const int4* c4 = reinterpret_cast<const int4*>(cb);
    const int n4 = kbeg / 4;
    int i = threadIdx.x;
    for (; i + 3 * 256 < n4; i += 4 * 256) {
      int4 q[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) q[u] = c4[i + u * 256];
#pragma unroll
      for (int u = 0; u < 4; ++u) s += q[u].x + q[u].y + q[u].z + q[u].w;
    }
    for (; i < n4; i += 256) {
      const int4 q = c4[i];
      s += q.x + q.y + q.z + q.w;
    }
  } else {
    for (int i = threadIdx.x; i < kbeg; i += 256) s += cb[i];
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
  if (lane == 0) red[grp] = s;
  __syncthreads();
  int carry = 0;
#pragma unroll
  for (int w = 0; w < 8; ++w) carry += red[w];
  const int cpg = (C + 7) / 8;
  const int c0 = grp * cpg, c1 = min(C, c0 + cpg);
  for (int sl = 0; sl < KS; ++sl) {
    const int k = kbeg + sl * 32 + lane;
    if (kbeg + sl * 32 >= K) break;  // uniform over the CTA
    int tot = 0;
    if (k < K)
      for (int c = c0; c < c1; ++c) tot += hb[static_cast<int64_t>(c) * K + k];
    part[grp][lane] = tot;
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
    for (int w = 0; w < grp; ++w) run += part[w][lane];
    if (grp == 0 && k < K) offsets[static_cast<int64_t>(b) * K + k] = off;
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

// ---------------------------------------------------------------------------
// scatter: sorted[base[b][chunk][label] + rank] = {row, label} (stable counting sort).
__global__ void __launch_bounds__(256) det_scatter_kernel(
    const int32_t* __restrict__ ids, const uint16_t* __restrict__ rank,
    const int32_t* __restrict__ base, int2* __restrict__ sorted, int N, int K, int R, int C,
    int64_t total) {
  pdl_wait();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += stride) {
    const int b = static_cast<int>(i / N);
    const int n = static_cast<int>(i - static_cast<int64_t>(b) * N);
    const int lab = ids[i];
    if (lab < 0 || lab >= K) continue;
    const int pos = base[(static_cast<int64_t>(b) * C + n / R) * K + lab] + rank[i];
    if (pos < 0 || pos >= N) continue;  // counts inconsistent with the labels: drop, never overrun
    sorted[static_cast<int64_t>(b) * N + pos] = make_int2(n, lab);
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

template <int N>
__device__ __forceinline__ void store_row(float* dst, const float (&acc)[N]) {
#pragma unroll
  for (int v = 0; v < N; v += 4)
    *reinterpret_cast<float4*>(dst + v) = make_float4(acc[v], acc[v + 1], acc[v + 2], acc[v + 3]);
}

// Group-span summary kept in shared memory for the CTA join.
struct SpanEnds {
  int first_lab;  // label of the run at the start of the group span (-1: none)
  int last_lab;   // label of the run at the end (-1: none, or the same run as first)
};

template <typename T, int L, int P>
__global__ void __launch_bounds__(kGatherThreads, 4) det_gather_kernel(
    const T* __restrict__ x, const int2* __restrict__ sorted, float* __restrict__ sums,
    float* __restrict__ part, int N, int K, int Pc, int ncta_per_batch, int64_t total_spans) {
  constexpr int kVec = 16 / sizeof(T);
  constexpr int G = 32 / L;
  constexpr int NG = kGatherWarps * G;  // group spans per CTA span
  constexpr int D = L * kVec;
  static_assert(32 % L == 0 && L % P == 0 && L >= 4, "group layout");
  __shared__ SpanEnds ends[NG];
  __shared__ __align__(16) float first_acc[NG][D];
  __shared__ __align__(16) float last_acc[NG][D];
  const int lane = threadIdx.x & 31;
  const int g = lane / L, i = lane % L;
  const uint32_t gmask = L == 32 ? 0xFFFFFFFFu : (((1u << L) - 1u) << (g * L));
  const int j = static_cast<int>(threadIdx.x >> 5) * G + g;  // group index in the CTA
  const int Sg = Pc / NG;                                    // Pc is a multiple of NG
  pdl_wait();
  for (int64_t cs = blockIdx.x; cs < total_spans; cs += gridDim.x) {
    const int b = static_cast<int>(cs / ncta_per_batch);
    const int S0 = static_cast<int>(cs - static_cast<int64_t>(b) * ncta_per_batch) * Pc;
    const int S1 = min(S0 + Pc, N);
    const int p0 = min(S0 + j * Sg, S1);
    const int p1 = min(p0 + Sg, S1);
    const int64_t rb = static_cast<int64_t>(b) * N;
    const T* xb = x + rb * D + i * kVec;
    // meta of positions m .. m + L - 1 (lane i: position m + i)
    auto load_meta = [&](int m, int& lab, int& src) {
      const int q = m + i;
      const int2 e = q < p1 ? __ldg(sorted + rb + q) : make_int2(0, -1);
      // labels outside [0, K) or rows outside [0, N) never occur on this path; such
      // an entry would read nothing
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
    int cur = -1, run_start = p0;
    // Hands a finished run over: whole cluster -> sums row; run at the span
    // start -> shared memory (first), run at the span end -> shared memory (last).
    auto flush = [&](bool at_end) {
      if (cur < 0) return;
      const bool at_start = run_start == p0;
      if (!at_start && !at_end) {
        store_row(sums + (static_cast<int64_t>(b) * K + cur) * D + i * kVec, acc);
      } else if (at_start) {
        store_row(&first_acc[j][i * kVec], acc);
      } else {
        store_row(&last_acc[j][i * kVec], acc);
      }
    };
    int first_lab = -1, last_lab = -1;
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
          if (ln >= 0 && q + P < p1) buf[jj % P] = ld_stream_v4(xb + static_cast<size_t>(sn) * D);
        }
      }
      labA = labB;
      srcA = srcB;
      load_meta(m + 2 * L, labB, srcB);
    }
    // the last run of the span
    if (cur >= 0) {
      if (run_start == p0) {
        first_lab = cur;  // one run covers the whole span
        flush(true);      // at_start: goes to first
      } else {
        if (first_lab < 0) first_lab = -1;
        last_lab = cur;
        flush(true);
      }
    }
    if (i == 0 && g * L + i == lane) {
      ends[j].first_lab = first_lab;
      ends[j].last_lab = last_lab;
    }
    __syncthreads();
    // CTA join of the group-span ends, in group order: thread t owns float4
    // column t of a row.
    constexpr int kCols = D / 4;
    if (static_cast<int>(threadIdx.x) < kCols) {
      const int t = threadIdx.x;
      const int lab_before = S0 > 0 ? sorted[rb + S0 - 1].y : -1;
      const int lab_after = S1 < N ? sorted[rb + S1].y : -1;
      int c_lab = -1;
      bool c_start = false;  // the carried run began at the CTA span start
      float4 c_acc = make_float4(0.f, 0.f, 0.f, 0.f);
      auto emit = [&](bool at_cta_end) {
        if (c_lab < 0) return;
        const bool before = c_start && lab_before == c_lab;
        const bool after = at_cta_end && lab_after == c_lab;
        float* dst;
        if (!before && !after)
          dst = sums + (static_cast<int64_t>(b) * K + c_lab) * D;
        else
          dst = part + (cs * 2 + (before ? 0 : 1)) * D;
        reinterpret_cast<float4*>(dst)[t] = c_acc;
      };
      auto add4 = [](float4& a, const float4& v) {
        a.x += v.x;
        a.y += v.y;
        a.z += v.z;
        a.w += v.w;
      };
      for (int jj = 0; jj < NG; ++jj) {
        const int fl = ends[jj].first_lab;
        if (fl < 0) continue;  // empty group span (past the end of the positions)
        const float4 fa = reinterpret_cast<const float4*>(first_acc[jj])[t];
        if (fl == c_lab) {
          add4(c_acc, fa);
        } else {
          emit(false);
          c_lab = fl;
          c_acc = fa;
          c_start = jj == 0;
        }
        const int ll = ends[jj].last_lab;
        if (ll >= 0) {  // the first run ended inside this group span
          emit(false);
          c_lab = ll;
          c_acc = reinterpret_cast<const float4*>(last_acc[jj])[t];
          c_start = false;
        }
      }
      emit(true);
    }
    __syncthreads();  // ends[] and the slots are reused by the next span
  }
}

// ---------------------------------------------------------------------------
// fixup (+ finalize)
template <typename T, int L, bool FINAL>
__global__ void __launch_bounds__(256) det_fixup_kernel(
    const float* __restrict__ part, const int32_t* __restrict__ counts,
    const int32_t* __restrict__ offsets, float* __restrict__ sums, const T* old_c, T* new_c,
    float* __restrict__ c_sq_out, uint8_t* __restrict__ cext_out, float* __restrict__ shift_out,
    int N, int K, int Pc, int ncta_per_batch, int64_t BK) {
  constexpr int kVec = 16 / sizeof(T);
  constexpr int G = 32 / L;
  constexpr int D = L * kVec;
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int g = lane / L, i = lane % L;
  const uint32_t gmask = L == 32 ? 0xFFFFFFFFu : (((1u << L) - 1u) << (g * L));
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  float shift_max = 0.f;
  for (int64_t u0 = (static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5)) * G;
       u0 < BK; u0 += warps * G) {
    const int64_t kg = u0 + g;
    if (kg >= BK) continue;  // whole groups only: the shuffles below stay inside the group
    const int cnt = counts[kg];
    uint4 ov = make_uint4(0u, 0u, 0u, 0u);
    if constexpr (FINAL) ov = *reinterpret_cast<const uint4*>(old_c + kg * D + i * kVec);
    float acc[kVec];
#pragma unroll
    for (int v = 0; v < kVec; ++v) acc[v] = 0.f;
    float* srow = sums + kg * D + i * kVec;
    bool write = true;
    if (cnt > 0) {
      // (counts consistent with the labels keep cs + cnt <= N; clamped so that a
      // caller's inconsistent counts can never index past the partial slots)
      const int cs = min(max(offsets[kg], 0), N - 1);
      const int ca = cs / Pc, cb = (min(cs + cnt, N) - 1) / Pc;
      if (ca == cb) {
        write = false;  // whole cluster inside one CTA span: the gather stored it
        if (!FINAL) continue;
#pragma unroll
        for (int v = 0; v < kVec; v += 4) {
          const float4 f = *reinterpret_cast<const float4*>(srow + v);
          acc[v] = f.x;
          acc[v + 1] = f.y;
          acc[v + 2] = f.z;
          acc[v + 3] = f.w;
        }
      } else {
        const int64_t sb = (kg / K) * ncta_per_batch;
        const float* p = part + ((sb + ca) * 2 + 1) * D + i * kVec;
#pragma unroll
        for (int v = 0; v < kVec; v += 4) {
          const float4 f = *reinterpret_cast<const float4*>(p + v);
          acc[v] = f.x;
          acc[v + 1] = f.y;
          acc[v + 2] = f.z;
          acc[v + 3] = f.w;
        }
        // slot 0 of spans ca+1 .. cb, added in span order (loads 4 ahead)
        for (int c = ca + 1; c <= cb; c += 4) {
          float4 f[4][kVec / 4];
#pragma unroll
          for (int u = 0; u < 4; ++u)
            if (c + u <= cb) {
              const float* q = part + ((sb + c + u) * 2) * D + i * kVec;
#pragma unroll
              for (int v = 0; v < kVec / 4; ++v) f[u][v] = *reinterpret_cast<const float4*>(q + 4 * v);
            }
#pragma unroll
          for (int u = 0; u < 4; ++u)
            if (c + u <= cb) {
#pragma unroll
              for (int v = 0; v < kVec / 4; ++v) {
                acc[4 * v] += f[u][v].x;
                acc[4 * v + 1] += f[u][v].y;
                acc[4 * v + 2] += f[u][v].z;
                acc[4 * v + 3] += f[u][v].w;
              }
            }
        }
      }
    }
    if (write) store_row(srow, acc);
    if constexpr (FINAL) {
      const int64_t row = kg * D + i * kVec;
      const T* o = reinterpret_cast<const T*>(&ov);
      uint4 nvv;
      T* nv = reinterpret_cast<T*>(&nvv);
      const float fc = static_cast<float>(cnt);
      float sq = 0.f, sh = 0.f;
#pragma unroll
      for (int v = 0; v < kVec; ++v) {
        nv[v] = cnt > 0 ? from_f32<T>(__fdiv_rn(acc[v], fc)) : o[v];
        const float nf = to_f32<T>(nv[v]);
        const float df = nf - to_f32<T>(o[v]);
        sq = fmaf(nf, nf, sq);
        sh = fmaf(df, df, sh);
      }
      *reinterpret_cast<uint4*>(new_c + row) = nvv;
#pragma unroll
      for (int o2 = L / 2; o2 >= 1; o2 >>= 1) {
        sq += __shfl_xor_sync(gmask, sq, o2);
        sh += __shfl_xor_sync(gmask, sh, o2);
      }
      if (i == 0) {
        if (c_sq_out != nullptr) c_sq_out[kg] = sq;
        if (cext_out != nullptr)
          write_norm_ext(cext_out + kg * kNormExtBytes, -0.5f * sq, false);
        shift_max = fmaxf(shift_max, sqrtf(sh));
      }
    }
  }
  if (FINAL && shift_out != nullptr) {
    __shared__ float block_max[8];
#pragma unroll
    for (int o2 = 16; o2 >= 1; o2 >>= 1)
      shift_max = fmaxf(shift_max, __shfl_xor_sync(0xFFFFFFFFu, shift_max, o2));
    if (lane == 0) block_max[threadIdx.x >> 5] = shift_max;
    __syncthreads();
    if (threadIdx.x == 0) {
      float m = 0.f;
      for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) m = fmaxf(m, block_max[w]);
      atomicMax(reinterpret_cast<unsigned int*>(shift_out), __float_as_uint(m));
    }
  }
}

// The sorted {row, label} pairs occupy the update workspace's perm and ids_sorted
// arrays (adjacent, 256-byte aligned, each B*N int32 rounded up to 256 bytes).
int2* det_sorted(const UpdateWorkspace& uw) { return reinterpret_cast<int2*>(uw.perm); }

int det_sm_count() {
  const DeviceInfo* di = nullptr;
  if (current_device_info(&di) == FKC_OK) return di->sm_count;
  return 148;
}

// Resident CTAs of a kernel (persistent grids).
template <typename Kern>
int det_resident(Kern kern, int threads) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, 0) != cudaSuccess ||
      per_sm < 1) {
    cudaGetLastError();
    per_sm = 1;
  }
  return per_sm * det_sm_count();
}

int64_t row_lanes(int64_t D, int dtype) { return D * static_cast<int64_t>(dtype_size(dtype)) / 16; }

bool det_shape_ok(int64_t N, int64_t K, int64_t D, int dtype) {
  if (K < 1 || K > kDetMaxK || N < 1) return false;
  if ((D * static_cast<int64_t>(dtype_size(dtype))) % 16 != 0) return false;
  const int64_t L = row_lanes(D, dtype);
  return L == 4 || L == 8 || L == 16 || L == 32;
}

// CTA-span length: spans of the gather cover about one per resident CTA (at
// least kDetMinSpan positions, at most kDetMaxSpans spans), a multiple of the
// group count NG so every group span has the same length.
int det_span_len(int64_t B, int64_t N, int NG, int resident) {
  const int64_t target = std::max<int64_t>(1, std::min<int64_t>(resident, kDetMaxSpans));
  int64_t pc = std::max<int64_t>(kDetMinSpan, (B * N + target - 1) / target);
  pc = std::max<int64_t>(pc, (B * N + kDetMaxSpans - 1) / kDetMaxSpans);
  pc = (pc + NG - 1) / NG * NG;
  // fewer spans than resident CTAs where batch rounding adds some
  while (B * ((N + pc - 1) / pc) > std::max<int64_t>(target, B) && pc < N) pc += NG;
  return static_cast<int>(std::min<int64_t>(pc, (N + NG - 1) / NG * NG));
}

template <typename T, int L>
int launch_det_typed(const void* x, const int32_t* counts, const UpdateWorkspace& uw,
                     const DetWorkspace& dw, float* sums, const void* old_c, void* new_c,
                     float* c_sq, void* cext, float* shift, int64_t B, int64_t N, int64_t K,
                     cudaStream_t stream) {
  constexpr int P = L >= 8 ? 8 : L;
  constexpr int G = 32 / L;
  constexpr int NG = kGatherWarps * G;
  auto gk = det_gather_kernel<T, L, P>;
  static std::atomic<int> res_cache{0};  // same value on every device of one model
  int res = res_cache.load(std::memory_order_relaxed);
  if (res == 0) {
    res = det_resident(gk, kGatherThreads);
    res_cache.store(res, std::memory_order_relaxed);
  }
  const int pc = det_span_len(B, N, NG, res);
  const int64_t ncta = (N + pc - 1) / pc;
  const int64_t spans = B * ncta;
  FKC_REQUIRE(spans <= det_max_spans(B), "update: %lld spans exceed the partial slots",
              static_cast<long long>(spans));
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(spans, res));
  FKC_TRY(launch_pdl(gk, dim3(grid), dim3(kGatherThreads), 0, stream, static_cast<const T*>(x),
                     static_cast<const int2*>(det_sorted(uw)), sums, dw.part,
                     static_cast<int>(N), static_cast<int>(K), pc, static_cast<int>(ncta), spans));
  const int64_t BK = B * K;
  const int64_t blocks = std::min<int64_t>((BK + 8 * G - 1) / (8 * G), det_sm_count() * 8ll);
  if (old_c != nullptr) {
    return launch_pdl(det_fixup_kernel<T, L, true>, dim3(static_cast<unsigned>(blocks)), dim3(256),
                      0, stream, static_cast<const float*>(dw.part), counts,
                      static_cast<const int32_t*>(uw.offsets), sums, static_cast<const T*>(old_c),
                      static_cast<T*>(new_c), c_sq, static_cast<uint8_t*>(cext), shift,
                      static_cast<int>(N), static_cast<int>(K), pc, static_cast<int>(ncta), BK);
  }
  return launch_pdl(det_fixup_kernel<T, L, false>, dim3(static_cast<unsigned>(blocks)), dim3(256),
                    0, stream, static_cast<const float*>(dw.part), counts,
                    static_cast<const int32_t*>(uw.offsets), sums, static_cast<const T*>(nullptr),
                    static_cast<T*>(nullptr), static_cast<float*>(nullptr),
                    static_cast<uint8_t*>(nullptr), static_cast<float*>(nullptr),
                    static_cast<int>(N), static_cast<int>(K), pc, static_cast<int>(ncta), BK);
}

template <typename T>
int launch_det_dtype(const void* x, const int32_t* counts, const UpdateWorkspace& uw,
                     const DetWorkspace& dw, float* sums, const void* old_c, void* new_c,
                     float* c_sq, void* cext, float* shift, int64_t B, int64_t N, int64_t K,
                     int64_t D, cudaStream_t stream) {
  switch (static_cast<int>(D * sizeof(T) / 16)) {
#define FKC_DET(L_)                                                                       \
  case L_:                                                                                \
    return launch_det_typed<T, L_>(x, counts, uw, dw, sums, old_c, new_c, c_sq, cext, shift, \
                                   B, N, K, stream);
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

}  // namespace

size_t det_update_bytes(int64_t B, int64_t N, int64_t K, int64_t D, int dtype) {
  if (!det_shape_ok(N, K, D, dtype)) return 0;
  const DetGeom g = det_geom(B, N, K);
  return align_up(static_cast<size_t>(B * N) * 2, 256) +
         align_up(static_cast<size_t>(B) * g.C * K * 4, 256) +
         align_up(static_cast<size_t>(det_max_spans(B)) * 2 * D * 4, 256);
}

DetWorkspace carve_det(void* ws, int64_t B, int64_t N, int64_t K, int64_t D, int dtype) {
  DetWorkspace w{};
  if (!det_shape_ok(N, K, D, dtype)) return w;
  const DetGeom g = det_geom(B, N, K);
  uint8_t* p = static_cast<uint8_t*>(ws);
  w.rank = reinterpret_cast<uint16_t*>(p);
  p += align_up(static_cast<size_t>(B * N) * 2, 256);
  w.hist = reinterpret_cast<int32_t*>(p);
  p += align_up(static_cast<size_t>(B) * g.C * K * 4, 256);
  w.part = reinterpret_cast<float*>(p);
  return w;
}

bool det_update_ok(const DetWorkspace& dw, const void* x, const float* sums, const void* old_c,
                   const void* new_c, int64_t N, int64_t K, int64_t D, int dtype) {
  if (dw.rank == nullptr || !det_shape_ok(N, K, D, dtype)) return false;
  auto al = [](const void* p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  return x != nullptr && sums != nullptr && al(x) && al(sums) && al(old_c) && al(new_c);
}

int launch_det_update(const void* x, const int32_t* ids, const int32_t* counts,
                      const UpdateWorkspace& uw, const DetWorkspace& dw, float* sums,
                      const void* old_c, void* new_c, float* c_sq, void* cext, float* shift,
                      int64_t B, int64_t N, int64_t K, int64_t D, int dtype,
                      cudaStream_t stream) {
  FKC_REQUIRE(B * N <= 2147483647ll && B * K <= 2147483647ll, "update: sizes out of range");
  const DetGeom g = det_geom(B, N, K);
  FKC_REQUIRE(g.R <= kRankMaxRows && g.RW >= 32, "update: chunk of %d rows", g.R);
  // rank + chunk histograms
  const size_t smem = align_up(static_cast<size_t>(g.W) * K * 2, 16);
  if (smem > 48 * 1024)
    FKC_CUDA_TRY(cudaFuncSetAttribute(det_rank_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(smem)));
  FKC_TRY(launch_pdl(det_rank_kernel, dim3(static_cast<unsigned>(B * g.C)), dim3(32 * g.W), smem,
                     stream, ids, static_cast<int>(N), static_cast<int>(K), g.RW, g.C, dw.hist,
                     dw.rank, (old_c != nullptr) ? shift : static_cast<float*>(nullptr)));
  // chunk bases + offsets: a CTA takes KS slices of 32 labels (at most 256 CTAs per batch row)
  const int64_t slices = (K + 31) / 32;
  const int KS = static_cast<int>(std::max<int64_t>(1, (slices + 255) / 256));
  const int ctas_b = static_cast<int>((slices + KS - 1) / KS);
  FKC_TRY(launch_pdl(det_base_kernel, dim3(static_cast<unsigned>(B * ctas_b)), dim3(256), 0, stream,
                     counts, dw.hist, uw.offsets, static_cast<int>(K), g.C, KS, ctas_b));
  const int64_t total = B * N;
  const int64_t sblocks = std::min<int64_t>((total + 255) / 256, det_sm_count() * 16ll);
  FKC_TRY(launch_pdl(det_scatter_kernel, dim3(static_cast<unsigned>(sblocks)), dim3(256), 0, stream,
                     ids, static_cast<const uint16_t*>(dw.rank),
                     static_cast<const int32_t*>(dw.hist), det_sorted(uw), static_cast<int>(N),
                     static_cast<int>(K), g.R, g.C, total));
  switch (dtype) {
    case FKC_DTYPE_F16:
      return launch_det_dtype<__half>(x, counts, uw, dw, sums, old_c, new_c, c_sq, cext, shift, B,
                                      N, K, D, stream);
    case FKC_DTYPE_BF16:
      return launch_det_dtype<__nv_bfloat16>(x, counts, uw, dw, sums, old_c, new_c, c_sq, cext,
                                             shift, B, N, K, D, stream);
    case FKC_DTYPE_F32:
      return launch_det_dtype<float>(x, counts, uw, dw, sums, old_c, new_c, c_sq, cext, shift, B,
                                     N, K, D, stream);
    default:
      return set_error(FKC_EINVAL, "update: bad dtype %d", dtype);
  }
}

}  // namespace fkc
