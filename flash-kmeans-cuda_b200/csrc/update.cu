// Centroid update: per-cluster fp32 sums and int32 counts.
//
// The reference sorts labels with torch.sort and then runs a sorted-run
// accumulator whose run boundaries are found serially by thread 0 and whose
// flushes are one fp32 atomicAdd per feature
// (flash_kmeans_cuda/ops.py:89-111, csrc/update/update_sorted.cu:39-186).
// Here:
//   * the permutation comes from a counting sort on labels in [0, K):
//     histogram (warp-aggregated atomics; fused into the assignment kernel on
//     the Lloyd path) -> exclusive scan per batch row -> scatter. The scatter
//     ranks rows inside a chunk of 512-4096 rows with shared-memory atomics and
//     claims each cluster's slots with one global atomic per (chunk, cluster),
//     so a heavily populated cluster costs one global atomic per chunk, not per
//     row;
//   * the accumulator gives each warp 64 sorted positions and splits them into
//     32/L contiguous row streams, L = lanes per row (a D=128 fp16 row is 16
//     lanes x 16 B). Each stream keeps P rows in flight (16-byte cp.async copies
//     into a per-warp shared-memory ring), accumulates in registers and flushes
//     every run with 16-byte vector atomics (red.global.add.v4.f32). No sorted
//     copy of x is written.
//   * the scatter kernel also zeroes the sums the accumulator adds into;
//   * with at most 32 rows per cluster on average, a single-GPU Lloyd step
//     replaces accumulate + finalize by one pass over the clusters
//     (gather_finalize_kernel): whole clusters are summed in row order and
//     finished with plain stores; clusters of more than 64 rows are cut into
//     pieces (laid out by the scan) that add into a per-cluster row, and the
//     last piece finishes the cluster.
// The same accumulator serves the reference's _C.centroid_update_sorted and
// _C.centroid_update_sorted_indexed entry points (perm == nullptr for the
// former).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <atomic>
#include <type_traits>

#include "fkc_common.cuh"
#include "fkc_internal.h"
#include "fkc_launch.cuh"

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
  pdl_wait();
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

// Exclusive scan of counts[b, 0..K) into offsets[b, 0..K) and cursor[b, 0..K);
// one CTA of kScanThreads per b, V consecutive counts per thread per tile
// (V = 4 with 16-byte loads and stores when K % 4 == 0). With PLAN it also
// lays out the units of the fused update (clusters of more than kUnitRows
// rows: ceil(count / kUnitRows) units each, listed in extras[b, 0..cap) in
// cluster order).
constexpr int kScanThreads = 1024;
constexpr int kUnitRows = 64;  // rows of x summed by one unit of the fused update

// Exclusive scan over the CTA (every thread gets the CTA total too). Ends with
// a barrier, so warp_tot can be reused at once.
__device__ __forceinline__ int block_excl_scan(int v, int* warp_tot, int& total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int u = __shfl_up_sync(0xFFFFFFFFu, inc, o);
    if (lane >= o) inc += u;
  }
  if (lane == 31) warp_tot[w] = inc;
  __syncthreads();
  if (w == 0) {
    int t = warp_tot[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xFFFFFFFFu, t, o);
      if (lane >= o) t += u;
    }
    warp_tot[lane] = t;  // inclusive over warps
  }
  __syncthreads();
  const int excl = inc - v + (w > 0 ? warp_tot[w - 1] : 0);
  total = warp_tot[kScanThreads / 32 - 1];
  __syncthreads();
  return excl;
}

template <int V, bool PLAN>
__global__ void __launch_bounds__(kScanThreads) scan_kernel(
    const int32_t* __restrict__ counts, int32_t* __restrict__ offsets,
    int32_t* __restrict__ cursor, int K, int2* __restrict__ extras,
    int32_t* __restrict__ extra_count, int cap) {
  pdl_wait();
  static_assert(kScanThreads == 1024, "block_excl_scan assumes 32 warps");
  __shared__ int warp_tot[kScanThreads / 32];
  const int t = threadIdx.x;
  const size_t kb = static_cast<size_t>(blockIdx.x) * K;
  const int32_t* cnt = counts + kb;
  int32_t* off = offsets + kb;
  int32_t* cur = cursor + kb;
  int carry = 0, xcarry = 0;
  for (int t0 = 0; t0 < K; t0 += kScanThreads * V) {
    const int i0 = t0 + t * V;
    int c[V];
    if constexpr (V == 4) {
      if (i0 < K) {
        const int4 q = *reinterpret_cast<const int4*>(cnt + i0);
        c[0] = q.x; c[1] = q.y; c[2] = q.z; c[3] = q.w;
      } else {
        c[0] = c[1] = c[2] = c[3] = 0;
      }
    } else {
#pragma unroll
      for (int e = 0; e < V; ++e) c[e] = (i0 + e < K) ? cnt[i0 + e] : 0;
    }
    int local = 0;
#pragma unroll
    for (int e = 0; e < V; ++e) local += c[e];
    int total = 0;
    int run = carry + block_excl_scan(local, warp_tot, total);
    carry += total;
    int o[V];
#pragma unroll
    for (int e = 0; e < V; ++e) {
      o[e] = run;
      run += c[e];
    }
    if constexpr (V == 4) {
      if (i0 < K) {
        *reinterpret_cast<int4*>(off + i0) = make_int4(o[0], o[1], o[2], o[3]);
        *reinterpret_cast<int4*>(cur + i0) = make_int4(o[0], o[1], o[2], o[3]);
      }
    } else {
#pragma unroll
      for (int e = 0; e < V; ++e)
        if (i0 + e < K) off[i0 + e] = cur[i0 + e] = o[e];
    }
    if constexpr (PLAN) {
      int ux[V], lx = 0;
#pragma unroll
      for (int e = 0; e < V; ++e) {
        ux[e] = c[e] > kUnitRows ? (c[e] + kUnitRows - 1) / kUnitRows : 0;
        lx += ux[e];
      }
      int xtotal = 0;
      int xrun = xcarry + block_excl_scan(lx, warp_tot, xtotal);
      xcarry += xtotal;
#pragma unroll
      for (int e = 0; e < V; ++e) {
        if (ux[e] == 0) continue;
        const int kg = static_cast<int>(kb) + i0 + e;
        int2* dst = extras + static_cast<size_t>(blockIdx.x) * cap + xrun;
        for (int j = 0; j < ux[e]; ++j) dst[j] = make_int2(kg, j);
        xrun += ux[e];
      }
    }
  }
  if (PLAN && t == 0) extra_count[blockIdx.x] = xcarry;
}

// Grid-stride zero fill of n floats at p (16-byte aligned), folded into the
// scatter kernels after their dependency wait.
__device__ __forceinline__ void zero_floats(float* p, int64_t n) {
  if (p == nullptr) return;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  float4* p4 = reinterpret_cast<float4*>(p);
  for (int64_t i = t0; i < n / 4; i += stride) p4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int64_t i = (n / 4) * 4 + t0; i < n; i += stride) p[i] = 0.f;
}

// Chunked scatter (K <= kLocalMaxK): the CTA ranks its rows per cluster with
// shared-memory atomics, claims slots [base, base + local count) of each
// cluster it holds with one global atomic on cursor, then writes
// perm[b, base + local rank] = n and ids_sorted likewise. Within a cluster the
// order follows the atomics (chunks in claim order, rows in rank order).
constexpr int kSortThreads = 512;
constexpr int kLocalMaxK = 16384;  // 64 KB of shared-memory counters

template <int RPT>
__global__ void __launch_bounds__(kSortThreads) scatter_chunk_kernel(
    const int32_t* __restrict__ ids, int32_t* __restrict__ cursor, int32_t* __restrict__ perm,
    int32_t* __restrict__ ids_sorted, int N, int K, int chunks_per_batch, float* zero_p,
    int64_t zero_n, float* zero_one) {
  pdl_wait();
  zero_floats(zero_p, zero_n);
  if (zero_one != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *zero_one = 0.f;
  extern __shared__ int cnt[];  // K counters, then reused for the K slot bases
  const int t = threadIdx.x;
  const int b = blockIdx.x / chunks_per_batch;
  const int r0 = (blockIdx.x - b * chunks_per_batch) * (kSortThreads * RPT);
  const size_t rb = static_cast<size_t>(b) * N;
  for (int k = t; k < K; k += kSortThreads) cnt[k] = 0;
  __syncthreads();
  int id[RPT], lr[RPT];
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const int n = r0 + i * kSortThreads + t;
    id[i] = n < N ? ids[rb + n] : -1;
    if (id[i] >= K) id[i] = -1;
    lr[i] = id[i] >= 0 ? atomicAdd(&cnt[id[i]], 1) : 0;
  }
  __syncthreads();
  int32_t* cur = cursor + static_cast<size_t>(b) * K;
  for (int k0 = 0; k0 < K; k0 += kSortThreads * 8) {
    int c[8], base[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int k = k0 + j * kSortThreads + t;
      c[j] = k < K ? cnt[k] : 0;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j)
      base[j] = c[j] > 0 ? atomicAdd(cur + k0 + j * kSortThreads + t, c[j]) : 0;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (c[j] > 0) cnt[k0 + j * kSortThreads + t] = base[j];
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    if (id[i] < 0) continue;
    const int pos = cnt[id[i]] + lr[i];
    if (pos >= N) continue;  // counts inconsistent with ids: drop rather than overrun
    perm[rb + pos] = r0 + i * kSortThreads + t;
    if (ids_sorted != nullptr) ids_sorted[rb + pos] = id[i];
  }
}

// Scatter for any K: warp-aggregated atomics on the cursors.
__global__ void scatter_atomic_kernel(const int32_t* __restrict__ ids,
                                      int32_t* __restrict__ cursor, int32_t* __restrict__ perm,
                                      int32_t* __restrict__ ids_sorted, int64_t total, int64_t N,
                                      int K, float* zero_p, int64_t zero_n, float* zero_one) {
  pdl_wait();
  zero_floats(zero_p, zero_n);
  if (zero_one != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *zero_one = 0.f;
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
      if (pos < N) {  // counts inconsistent with ids: drop rather than overrun
        const int64_t dst = b * N + pos;
        perm[dst] = static_cast<int32_t>(i - b * N);
        if (ids_sorted != nullptr) ids_sorted[dst] = id;
      }
    }
  }
}

__device__ __forceinline__ void red_add_v4(float* addr, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b),
               "f"(c), "f"(d)
               : "memory");
}

// 16-byte load that does not allocate in L1 (each x row is read once here).
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

// Gather-accumulate over sorted positions. Each warp owns a span of
// consecutive positions of one batch row (a multiple of 64, about equal spans
// for all resident warps) and walks it in segments of 64 positions. A segment
// is split into 32/L row streams of R = 2L consecutive positions; lane i of
// stream g handles 16-byte vector i of the stream's current row. The labels and
// source rows of a segment sit in two registers per lane (position
// g*R + h*L + i in register h of lane g*L + i), so each step needs one shuffle
// per value; the next segment's are loaded while the current one is walked.
// Every stream keeps P rows in flight, across segment boundaries, in shared
// memory: each lane copies its 16-byte vector of a row with cp.async into a
// per-warp ring of P slots (one copy group per step, empty when the position
// has no row) and reads it back once the oldest group has landed; a lane reads
// only what it copied itself, so no barrier is needed. Rows of one label are
// summed in registers (a stream's positions are sorted, so its runs are
// contiguous even across segments) and flushed with vector atomics when the
// label changes. Labels outside [0,K), including the -1 of unwritten
// positions, load nothing and are never flushed.
// Measured at c3 (D = 128 fp16, P = 16, 2 CTAs per SM): the update phase 52 us
// against 57.6 us with P = 8 rows in flight held in registers (106 registers,
// 2 CTAs per SM; capped at 80 registers for 3 CTAs per SM that version was no
// faster); a row-read probe reaches 30.7 us for the same 134 MB of random
// 256-byte rows at 4 CTAs per SM without the run bookkeeping.
template <typename T, int L, int P>
__global__ void __launch_bounds__(256) gather_accumulate_kernel(
    const T* __restrict__ x, const int32_t* __restrict__ perm,
    const int32_t* __restrict__ ids_sorted, float* __restrict__ sums,
    int32_t* __restrict__ counts, int N, int K, int spans_per_batch, int span_len,
    int64_t total_spans) {
  pdl_wait();
  extern __shared__ uint4 gather_ring[];  // (warps, P, 32) 16-byte slots
  constexpr int kVec = 16 / sizeof(T);
  constexpr int R = 2 * L;
  static_assert(32 % L == 0 && R % P == 0, "stream layout");
  const int lane = threadIdx.x & 31;
  const int g = lane / L;
  const int i = lane % L;
  const int D = L * kVec;
  uint4* my_ring = gather_ring + (threadIdx.x >> 5) * (P * 32) + lane;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t sp = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
       sp < total_spans; sp += warps) {
    const int b = static_cast<int>(sp / spans_per_batch);
    const int sp0 = static_cast<int>(sp - static_cast<int64_t>(b) * spans_per_batch) * span_len;
    const int sp1 = min(sp0 + span_len, N);
    if (sp0 >= sp1) continue;
    const int nseg = (sp1 - sp0 + kRange - 1) / kRange;
    const size_t rb = static_cast<size_t>(b) * N;
    const T* xb = x + rb * D;
    auto load_meta = [&](int base, int (&lab)[2], int (&src)[2]) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int q = base + g * R + h * L + i;
        int l = q < sp1 ? ids_sorted[rb + q] : -1;
        if (l >= K) l = -1;
        int sr = l >= 0 ? (perm ? perm[rb + q] : q) : 0;
        if (sr < 0 || sr >= N) {
          l = -1;
          sr = 0;
        }
        lab[h] = l;
        src[h] = sr;
      }
    };
    auto meta_at = [&](const int (&a)[2], int j) {
      return __shfl_sync(0xFFFFFFFFu, a[j / L], g * L + (j % L));
    };
    // One copy group per step (empty when the position has no row).
    auto load_row = [&](int slot, int src, bool on) {
      if (on) {
        const uint32_t dst = static_cast<uint32_t>(__cvta_generic_to_shared(my_ring + slot * 32));
        const T* srcp = xb + static_cast<size_t>(src) * D + i * kVec;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(srcp)
                     : "memory");
      }
      asm volatile("cp.async.commit_group;" ::: "memory");
    };
    int lab[2], src[2], labn[2], srcn[2];
    load_meta(sp0, lab, src);
    int ring[P];
#pragma unroll
    for (int j = 0; j < P; ++j) {
      ring[j] = meta_at(lab, j);
      const int sr = meta_at(src, j);
      load_row(j, sr, ring[j] >= 0);
    }
    float acc[kVec];
#pragma unroll
    for (int e = 0; e < kVec; ++e) acc[e] = 0.f;
    int cur = -1, len = 0;
    auto flush = [&]() {
      if (cur >= 0) {
        float* dst = sums + (static_cast<size_t>(b) * K + cur) * D + i * kVec;
#pragma unroll
        for (int e = 0; e < kVec; e += 4)
          red_add_v4(dst + e, acc[e], acc[e + 1], acc[e + 2], acc[e + 3]);
        if (counts != nullptr && i == 0)
          atomicAdd(counts + static_cast<size_t>(b) * K + cur, len);
      }
    };
    for (int seg = 0; seg < nseg; ++seg) {
      if (seg + 1 < nseg) {
        load_meta(sp0 + (seg + 1) * kRange, labn, srcn);
      } else {
        labn[0] = labn[1] = -1;
        srcn[0] = srcn[1] = 0;
      }
#pragma unroll
      for (int j = 0; j < R; ++j) {
        const int l = ring[j % P];
        const int jn = j + P;
        const int ln = jn < R ? meta_at(lab, jn) : meta_at(labn, jn - R);
        const int sn = jn < R ? meta_at(src, jn) : meta_at(srcn, jn - R);
        if (l != cur) {
          flush();
#pragma unroll
          for (int e = 0; e < kVec; ++e) acc[e] = 0.f;
          cur = l;
          len = 0;
        }
        // the oldest of the P groups in flight (this step's row) has landed
        asm volatile("cp.async.wait_group %0;" ::"n"(P - 1) : "memory");
        if (l >= 0) {
          add_vec<T>(acc, my_ring[(j % P) * 32]);
          ++len;
        }
        ring[j % P] = ln;
        load_row(j % P, sn, ln >= 0);
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        lab[h] = labn[h];
        src[h] = srcn[h];
      }
    }
    flush();
    asm volatile("cp.async.wait_all;" ::: "memory");  // no copy outlives the span's ring use
  }
}

// Fused update + finalize (single-GPU Lloyd step). Work units: unit b*K+k is
// cluster k of batch row b when it has at most kUnitRows rows; larger clusters
// are cut into units of kUnitRows rows listed in extras (scan_kernel<.., true>).
// A group of L lanes (lane i: 16-byte vector i of a row) takes a unit, reads
// its rows through perm with P loads in flight (the next P row indices are
// fetched while the rows arrive) and sums them in registers in row order.
// A whole cluster is finished at once: sums row (plain stores), new centroid
// = sums / count rounded to T (the old one when empty), ||new||^2, its norm
// slice and ||new - old|| for the shift, so no sums zero-fill, no atomics on
// sums and no separate finalize pass are needed. A unit of a split cluster
// adds its partial sum into the cluster's row of `acc` (16-byte vector
// atomics); the last one to finish (done counter) reads the row, finishes the
// cluster and sets the row and the counter back to zero, so both stay zero
// between passes (they are zeroed once, when the workspace is prepared).
// new_c may alias old_c: each lane reads its old elements before writing.
template <typename T, int L, int P>
__global__ void __launch_bounds__(256) gather_finalize_kernel(
    const T* __restrict__ x, const int32_t* __restrict__ perm,
    const int32_t* __restrict__ offsets, const int32_t* __restrict__ counts,
    const int2* __restrict__ extras, const int32_t* __restrict__ extra_count,
    int32_t* __restrict__ done, float* __restrict__ acc_rows, const T* old_c, T* new_c,
    float* __restrict__ sums, float* __restrict__ c_sq_out, uint8_t* __restrict__ cext_out,
    float* __restrict__ shift_out, int N, int K, int B, int cap) {
  pdl_wait();
  constexpr int kVec = 16 / sizeof(T);
  constexpr int G = 32 / L;
  static_assert(32 % L == 0, "groups tile the warp");
  const int lane = threadIdx.x & 31;
  const int g = lane / L;
  const int i = lane % L;
  const uint32_t gmask = L == 32 ? 0xFFFFFFFFu : (((1u << L) - 1u) << (g * L));
  const int D = L * kVec;
  const int64_t BK = static_cast<int64_t>(B) * K;
  const int64_t U = BK + static_cast<int64_t>(B) * cap;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  float shift_max = 0.f;
  for (int64_t u0 = (static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5)) * G;
       u0 < U; u0 += warps * G) {
    const int64_t u = u0 + g;
    int kg = -1, cnt = 0, r0 = 0, r1 = 0, nunits = 1;
    int64_t e = -1;
    if (u < BK) {
      cnt = counts[u];
      if (cnt <= kUnitRows) {
        kg = static_cast<int>(u);
        r0 = offsets[u];
        r1 = r0 + cnt;
      }
    } else if (u < U) {
      const int64_t q = u - BK;
      const int b = static_cast<int>(q / cap);
      if (q - static_cast<int64_t>(b) * cap < extra_count[b]) {
        const int2 en = extras[q];
        kg = en.x;
        e = q;
        cnt = counts[kg];
        nunits = (cnt + kUnitRows - 1) / kUnitRows;
        r0 = offsets[kg] + en.y * kUnitRows;
        r1 = min(r0 + kUnitRows, offsets[kg] + cnt);
      }
    }
    float acc[kVec];
#pragma unroll
    for (int v = 0; v < kVec; ++v) acc[v] = 0.f;
    if (kg >= 0) {
      const int b = kg / K;
      const int32_t* pb = perm + static_cast<size_t>(b) * N;
      const T* xb = x + static_cast<size_t>(b) * N * D + i * kVec;
      int pr[P];
#pragma unroll
      for (int p = 0; p < P; ++p) pr[p] = r0 + p < r1 ? pb[r0 + p] : 0;
      for (int r = r0; r < r1; r += P) {
        uint4 v[P];
#pragma unroll
        for (int p = 0; p < P; ++p)
          if (r + p < r1) v[p] = ld_stream_v4(xb + static_cast<size_t>(pr[p]) * D);
#pragma unroll
        for (int p = 0; p < P; ++p) pr[p] = r + P + p < r1 ? pb[r + P + p] : 0;
#pragma unroll
        for (int p = 0; p < P; ++p)
          if (r + p < r1) add_vec<T>(acc, v[p]);
      }
      if (e >= 0) {
        // A unit of a split cluster: add the partial, count it, and let the
        // last unit of the cluster finish it.
        float* arow = acc_rows + static_cast<size_t>(kg) * D + i * kVec;
#pragma unroll
        for (int v = 0; v < kVec; v += 4) red_add_v4(arow + v, acc[v], acc[v + 1], acc[v + 2], acc[v + 3]);
        __threadfence();
        __syncwarp(gmask);
        int prev = 0;
        if (i == 0) prev = atomicAdd(done + kg, 1);
        prev = __shfl_sync(gmask, prev, g * L);
        if (prev != nunits - 1) {
          kg = -1;
        } else {
          __threadfence();
#pragma unroll
          for (int v = 0; v < kVec; v += 4) {
            const float4 f = __ldcg(reinterpret_cast<const float4*>(arow + v));
            acc[v] = f.x;
            acc[v + 1] = f.y;
            acc[v + 2] = f.z;
            acc[v + 3] = f.w;
            *reinterpret_cast<float4*>(arow + v) = make_float4(0.f, 0.f, 0.f, 0.f);
          }
          if (i == 0) done[kg] = 0;
        }
      }
    }
    if (kg >= 0) {
      const size_t row = static_cast<size_t>(kg) * D + i * kVec;
      float* srow = sums + row;
#pragma unroll
      for (int v = 0; v < kVec; v += 4)
        *reinterpret_cast<float4*>(srow + v) = make_float4(acc[v], acc[v + 1], acc[v + 2], acc[v + 3]);
      const uint4 ov = *reinterpret_cast<const uint4*>(old_c + row);
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
          write_norm_ext(cext_out + static_cast<size_t>(kg) * kNormExtBytes, -0.5f * sq, false);
        shift_max = fmaxf(shift_max, sqrtf(sh));
      }
    }
  }
  if (shift_out != nullptr) {
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
  pdl_wait();
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
        for (int k = 0; k < kVec; k += 4)
          red_add_v4(dst + k, acc[k], acc[k + 1], acc[k + 2], acc[k + 3]);
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
  pdl_wait();
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

// Resident blocks of `kern` on this device (block size 256), for persistent grids.
template <typename K>
int resident_blocks(K kern, size_t smem = 0) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 256, smem) != cudaSuccess ||
      per_sm < 1) {
    cudaGetLastError();
    per_sm = 1;
  }
  return per_sm * sm_count_or_default();
}

template <typename T, int L>
int launch_gather(const T* x, const int32_t* perm, const int32_t* ids_sorted, float* sums,
                  int32_t* counts, int64_t B, int64_t N, int64_t K, cudaStream_t stream) {
  constexpr int R = 2 * L;
  constexpr int P = R < 16 ? R : 16;  // rows in flight per stream
  auto kern = gather_accumulate_kernel<T, L, P>;
  constexpr int kSmem = 8 * P * 32 * 16;  // 8 warps x P slots x 32 lanes x 16 bytes
  // The shared-memory opt-in is a property of the kernel in each device's
  // context: set it once per device ordinal (every call beyond ordinal 63).
  static std::atomic<uint64_t> smem_set{0};
  int dev = 0;
  FKC_CUDA_TRY(cudaGetDevice(&dev));
  const uint64_t bit = dev < 64 ? (uint64_t{1} << dev) : 0;
  if (bit == 0 || (smem_set.load(std::memory_order_relaxed) & bit) == 0) {
    FKC_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
    smem_set.fetch_or(bit, std::memory_order_relaxed);
  }
  // Resident blocks (the same on every device of one model). Host threads
  // driving several GPUs may race on the first call: atomic, same value.
  static std::atomic<int> cap_cache{0};
  int cap = cap_cache.load(std::memory_order_relaxed);
  if (cap == 0) {
    cap = resident_blocks(kern, kSmem);
    cap_cache.store(cap, std::memory_order_relaxed);
  }
  // About one span per resident warp (spans a multiple of 32 positions), so
  // every SM gets the same number of positions.
  const int64_t warps = static_cast<int64_t>(cap) * 8;
  int64_t spans_per_batch = std::max<int64_t>(1, (warps + B - 1) / B);
  int64_t span_len = (N + spans_per_batch - 1) / spans_per_batch;
  span_len = (span_len + 31) / 32 * 32;
  spans_per_batch = (N + span_len - 1) / span_len;
  const int64_t total = spans_per_batch * B;
  const int64_t blocks = std::min<int64_t>((total + 7) / 8, cap);
  return launch_pdl(kern, dim3(static_cast<unsigned>(blocks)), dim3(256), kSmem, stream, x, perm,
                    ids_sorted, sums, counts, static_cast<int>(N), static_cast<int>(K),
                    static_cast<int>(spans_per_batch), static_cast<int>(span_len), total);
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
  const T* xt = static_cast<const T*>(x);
  if (vec_ok) {
    const int L = static_cast<int>(row_bytes / 16);
    switch (L) {
      case 1: return launch_gather<T, 1>(xt, perm, ids_sorted, sums, counts, B, N, K, stream);
      case 2: return launch_gather<T, 2>(xt, perm, ids_sorted, sums, counts, B, N, K, stream);
      case 4: return launch_gather<T, 4>(xt, perm, ids_sorted, sums, counts, B, N, K, stream);
      case 8: return launch_gather<T, 8>(xt, perm, ids_sorted, sums, counts, B, N, K, stream);
      case 16: return launch_gather<T, 16>(xt, perm, ids_sorted, sums, counts, B, N, K, stream);
      case 32: return launch_gather<T, 32>(xt, perm, ids_sorted, sums, counts, B, N, K, stream);
      default:
        break;
    }
    return launch_pdl(run_accumulate_vec_kernel<T>, dim3(static_cast<unsigned>(blocks)), dim3(256),
                      0, stream, xt, perm, ids_sorted, sums, counts, static_cast<int>(N),
                      static_cast<int>(K), static_cast<int>(D), L,
                      static_cast<int>(ranges_per_batch), total);
  }
  return launch_pdl(run_accumulate_scalar_kernel<T>, dim3(static_cast<unsigned>(blocks)),
                    dim3(256), 0, stream, xt, perm, ids_sorted, sums, counts, static_cast<int>(N),
                    static_cast<int>(K), static_cast<int>(D), static_cast<int>(ranges_per_batch),
                    total);
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
  return launch_pdl(histogram_kernel, dim3(grid_for(total, 256)), dim3(256), 0, stream, ids,
                    counts, total, N, static_cast<int>(K));
}

namespace {

template <int RPT>
int launch_scatter_chunk(const int32_t* ids, const UpdateWorkspace& w, int64_t B, int64_t N,
                         int64_t K, cudaStream_t stream) {
  auto kern = scatter_chunk_kernel<RPT>;
  const int smem = static_cast<int>(K) * 4;
  if (smem > 48 * 1024)
    FKC_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  const int64_t chunks = (N + kSortThreads * RPT - 1) / (kSortThreads * RPT);
  FKC_REQUIRE(chunks * B < (1ll << 31), "update: too many row chunks");
  return launch_pdl(kern, dim3(static_cast<unsigned>(chunks * B)), dim3(kSortThreads),
                    static_cast<size_t>(smem), stream, ids, w.cursor, w.perm, w.ids_sorted,
                    static_cast<int>(N), static_cast<int>(K), static_cast<int>(chunks),
                    w.zero_f32, w.zero_count, w.zero_scalar);
}

}  // namespace

namespace {

// perm (and ids_sorted, when non-null) from the cursors of the scan.
int launch_scatter(const int32_t* ids, const UpdateWorkspace& w, int64_t B, int64_t N, int64_t K,
                   cudaStream_t stream) {
  if (K <= kLocalMaxK) {
    // Rows per chunk: the largest of 4096/2048/1024/512 that still gives about
    // two chunks per SM.
    const int64_t rows = B * N;
    const int64_t want = 2ll * sm_count_or_default();
    if (rows >= want * kSortThreads * 8) return launch_scatter_chunk<8>(ids, w, B, N, K, stream);
    if (rows >= want * kSortThreads * 4) return launch_scatter_chunk<4>(ids, w, B, N, K, stream);
    if (rows >= want * kSortThreads * 2) return launch_scatter_chunk<2>(ids, w, B, N, K, stream);
    return launch_scatter_chunk<1>(ids, w, B, N, K, stream);
  }
  const int64_t total = B * N;
  return launch_pdl(scatter_atomic_kernel, dim3(grid_for(total, 256)), dim3(256), 0, stream, ids,
                    w.cursor, w.perm, w.ids_sorted, total, N, static_cast<int>(K), w.zero_f32,
                    w.zero_count, w.zero_scalar);
}

}  // namespace

int launch_counting_sort(const int32_t* ids, const int32_t* counts, const UpdateWorkspace& w,
                         int64_t B, int64_t N, int64_t K, bool all_valid, cudaStream_t stream) {
  FKC_REQUIRE(B <= 2147483647ll && N <= 2147483647ll && K <= 2147483647ll,
              "update: sizes out of range");
  if (K % 4 == 0)
    FKC_TRY(launch_pdl(scan_kernel<4, false>, dim3(static_cast<unsigned>(B)), dim3(kScanThreads),
                       0, stream, counts, w.offsets, w.cursor, static_cast<int>(K), nullptr,
                       nullptr, 0));
  else
    FKC_TRY(launch_pdl(scan_kernel<1, false>, dim3(static_cast<unsigned>(B)), dim3(kScanThreads),
                       0, stream, counts, w.offsets, w.cursor, static_cast<int>(K), nullptr,
                       nullptr, 0));
  // With labels outside [0,K) some sorted positions stay unwritten: they must
  // read as label -1, which the accumulator skips.
  if (!all_valid)
    FKC_CUDA_TRY(cudaMemsetAsync(w.ids_sorted, 0xFF, static_cast<size_t>(B * N) * 4, stream));
  return launch_scatter(ids, w, B, N, K, stream);
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

namespace {

int64_t plan_cap(int64_t N) {
  // Units of split clusters in one batch row: sum of ceil(c / kUnitRows) over
  // clusters with c > kUnitRows <= N / kUnitRows + (number of such clusters)
  // <= 2 N / kUnitRows.
  return 2 * ((N + kUnitRows - 1) / kUnitRows);
}

template <typename T, int L>
int launch_gather_finalize(const T* x, const UpdateWorkspace& w, const UpdatePlan& plan,
                           const int32_t* counts, const T* old_c, T* new_c, float* sums,
                           float* c_sq, void* cext, float* shift, int64_t B, int64_t N,
                           int64_t K, cudaStream_t stream) {
  constexpr int P = L >= 16 ? 16 : 8;  // row loads in flight per group
  auto kern = gather_finalize_kernel<T, L, P>;
  // Resident blocks (the same on every device of one model). Host threads
  // driving several GPUs may race on the first call: atomic, same value.
  static std::atomic<int> cap_cache{0};
  int cap = cap_cache.load(std::memory_order_relaxed);
  if (cap == 0) {
    cap = resident_blocks(kern);
    cap_cache.store(cap, std::memory_order_relaxed);
  }
  constexpr int G = 32 / L;
  const int64_t units = B * K + B * static_cast<int64_t>(plan.cap);
  const int64_t blocks = std::min<int64_t>((units + 8 * G - 1) / (8 * G), cap);
  return launch_pdl(kern, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, stream, x, w.perm,
                    w.offsets, counts, plan.extras, plan.extra_count, plan.done, plan.acc,
                    old_c, new_c, sums, c_sq, static_cast<uint8_t*>(cext), shift,
                    static_cast<int>(N), static_cast<int>(K), static_cast<int>(B), plan.cap);
}

template <typename T>
int update_finalize_typed(const void* x, const UpdateWorkspace& w, const UpdatePlan& plan,
                          const int32_t* counts, const void* old_c, void* new_c, float* sums,
                          float* c_sq, void* cext, float* shift, int64_t B, int64_t N, int64_t K,
                          int64_t D, cudaStream_t stream) {
  const T* xt = static_cast<const T*>(x);
  const T* oc = static_cast<const T*>(old_c);
  T* nc = static_cast<T*>(new_c);
  switch (static_cast<int>(D * sizeof(T) / 16)) {
#define FKC_GF(L_)                                                                           \
  case L_:                                                                                   \
    return launch_gather_finalize<T, L_>(xt, w, plan, counts, oc, nc, sums, c_sq, cext, shift, \
                                         B, N, K, stream);
    FKC_GF(1)
    FKC_GF(2)
    FKC_GF(4)
    FKC_GF(8)
    FKC_GF(16)
    FKC_GF(32)
#undef FKC_GF
    default:
      return set_error(FKC_EINVAL, "fused update: unsupported row size (D=%lld)",
                       static_cast<long long>(D));
  }
}

}  // namespace

size_t update_plan_bytes(int64_t B, int64_t N, int64_t K, int64_t D) {
  const int64_t cap = plan_cap(N);
  return align_up(static_cast<size_t>(B * cap) * 8, 256) + align_up(static_cast<size_t>(B) * 4, 256) +
         align_up(static_cast<size_t>(B * K) * 4, 256) +
         align_up(static_cast<size_t>(B * K * D) * 4, 256);
}

UpdatePlan carve_update_plan(void* ws, int64_t B, int64_t N, int64_t K, int64_t D) {
  const int64_t cap = plan_cap(N);
  uint8_t* p = static_cast<uint8_t*>(ws);
  UpdatePlan u;
  u.extras = reinterpret_cast<int2*>(p);
  p += align_up(static_cast<size_t>(B * cap) * 8, 256);
  u.extra_count = reinterpret_cast<int32_t*>(p);
  p += align_up(static_cast<size_t>(B) * 4, 256);
  u.done = reinterpret_cast<int32_t*>(p);
  p += align_up(static_cast<size_t>(B * K) * 4, 256);
  u.acc = reinterpret_cast<float*>(p);
  u.cap = static_cast<int>(cap);
  u.zero_bytes = static_cast<size_t>(p - reinterpret_cast<uint8_t*>(u.done)) +
                 static_cast<size_t>(B * K * D) * 4;
  return u;
}

bool fused_update_ok(const void* x, const void* old_c, const void* new_c, const float* sums,
                     int64_t D, int dtype) {
  const int64_t es = dtype == FKC_DTYPE_F32 ? 4 : 2;
  const int64_t row = D * es;
  if (row % 16 != 0 || row > 512) return false;
  const int64_t L = row / 16;
  if (32 % L != 0) return false;
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  return al(x) && al(old_c) && al(new_c) && al(sums);
}

int launch_update_finalize(const void* x, const int32_t* ids, const int32_t* counts,
                           const UpdateWorkspace& w, const UpdatePlan& plan, const void* old_c,
                           void* new_c, float* sums, float* c_sq, void* cext, float* shift,
                           int64_t B, int64_t N, int64_t K, int64_t D, int dtype,
                           cudaStream_t stream) {
  FKC_REQUIRE(B <= 2147483647ll && N <= 2147483647ll && K <= 2147483647ll &&
                  B * K <= 2147483647ll,
              "update: sizes out of range");
  if (K % 4 == 0)
    FKC_TRY(launch_pdl(scan_kernel<4, true>, dim3(static_cast<unsigned>(B)), dim3(kScanThreads),
                       0, stream, counts, w.offsets, w.cursor, static_cast<int>(K), plan.extras,
                       plan.extra_count, plan.cap));
  else
    FKC_TRY(launch_pdl(scan_kernel<1, true>, dim3(static_cast<unsigned>(B)), dim3(kScanThreads),
                       0, stream, counts, w.offsets, w.cursor, static_cast<int>(K), plan.extras,
                       plan.extra_count, plan.cap));
  UpdateWorkspace ws = w;
  ws.ids_sorted = nullptr;  // the fused pass walks clusters through offsets
  FKC_TRY(launch_scatter(ids, ws, B, N, K, stream));
  if (shift != nullptr) FKC_TRY(launch_zero_fill(shift, sizeof(float), stream));
  switch (dtype) {
    case FKC_DTYPE_F16:
      return update_finalize_typed<__half>(x, w, plan, counts, old_c, new_c, sums, c_sq, cext,
                                           shift, B, N, K, D, stream);
    case FKC_DTYPE_BF16:
      return update_finalize_typed<__nv_bfloat16>(x, w, plan, counts, old_c, new_c, sums, c_sq,
                                                  cext, shift, B, N, K, D, stream);
    case FKC_DTYPE_F32:
      return update_finalize_typed<float>(x, w, plan, counts, old_c, new_c, sums, c_sq, cext,
                                          shift, B, N, K, D, stream);
    default:
      return set_error(FKC_EINVAL, "update: bad dtype %d", dtype);
  }
}

}  // namespace fkc
