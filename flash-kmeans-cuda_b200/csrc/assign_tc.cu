// Fused Euclidean assignment for sm_100a: TMA + tcgen05.mma (fp32 accumulator
// in TMEM) + a register argmin epilogue. The (B, N, K) distance matrix is
// never written to memory.
//
// Semantics follow the reference: ids[b,n] = argmin_k ||x[b,n]-c[b,k]||^2 with
// ties going to the lowest k (flash_kmeans_cuda/csrc/assign/assign_common.cuh:20-28,
// csrc/assign/assign_sm80.cu:594-611). Unlike the reference mma.sync path, which
// accumulates x.c in fp16 (csrc/common/ptx.cuh:151-170), the dot products here
// accumulate in fp32.
//
// Scoring. The MMA computes, per (row, centroid),
//     acc = x.c - 0.5*||x||^2 - 0.5*||c||^2 - delta = -0.5 * ||x - c||^2 - delta
// The norm terms enter through one extra K=8 slice of tf32 operands (one
// kind::tf32 MMA, half the cycles of a K=16 fp16 step):
//     A_ext[row] = {h1(x), h2(x), h3(x), 1, 1, 1, -delta(x), 0}
//     B_ext[k]   = {1, 1, 1, h1(c), h2(c), h3(c), 1, 0}
// where h1+h2+h3 is a three-term tf32 split (33 significant bits) of
// -0.5*||.||^2 and delta = 2^-12 ||x||^2 (+ 2^-100) is a row-constant bias
// (fkc_common.cuh, norm_ext.cu). So TMEM holds -dist/2 - delta directly: no per-column c_sq
// load and no FMA in the epilogue, and the score is strictly negative whenever
// c_sq is the centroids' own norm (the fp32 accumulation rounds at ~2^-22 ||x||^2).
//
// Argmax on packed keys. The epilogue replaces the 5 low mantissa bits of each
// score with its column index j inside a 32-column group (one LOP3) and takes
// a float max with 3-input max.f32 (about half an issue slot per score). For
// negative scores a larger j makes the key more negative, so exact ties within
// a group resolve to the lowest j; groups and chunks are merged in ascending k
// with a strict comparison of the truncated keys, so exact ties across groups
// resolve to the lowest k as well (the reference's rule). The truncation only
// affects candidates within 2^-18 relative score of each other. Scores of any
// sign order correctly (a caller's c_sq may make them positive); only exact
// ties between positive scores would go to the higher j.
//
// Kernel structure (persistent, one CTA per SM, 64 + 32*kEpiWarps threads):
//   warp 0      TMA producer: x sub-tiles (+ row-norm slice) once per tile,
//               centroid chunks (+ norm slice) through an ST-deep ring.
//   warp 1      TMEM owner and MMA issuer (one thread): for each (chunk,
//               sub-tile) item, D/16 fp16/bf16 MMAs + 1 bf16 norm MMA into
//               one of two TMEM accumulator slots.
//   warps 2..   epilogue, kEpiWarps/4 warpgroups: one TMEM lane (= one x row)
//               per thread, one column slice of each item per warpgroup;
//               tcgen05.ld 32 columns at a time, packed-key max, running best
//               per row; the slices merge once per tile.
// Two accumulator slots ping-pong so the epilogue of one item overlaps the
// MMAs of the next.
//
// CTA pairs (CG = 2). Launched as clusters of two CTAs on one TPC: each CTA
// owns MT x 128 rows of a tile and loads HALF of every 256-centroid chunk; the
// even CTA issues tcgen05.mma.cta_group::2 with M = 256 (128 rows from each
// CTA's shared memory) and N = 256 (128 centroids from each), and every CTA's
// TMEM receives its own 128 rows x 256 columns. Per SM this halves the shared-
// memory operand traffic of the MMA and the L2 reads of centroid chunks. TMA
// completions of both CTAs land on the even CTA's full barriers; MMA
// completions are fanned out to both CTAs' barriers by one commit with a CTA
// mask; the odd CTA's epilogue releases accumulator slots with a relaxed remote
// arrive on the even CTA's barrier. Opt-in (FKC_ASSIGN_CTA_GROUP=2): it measured
// no faster than single CTAs (cta_group_choice).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <atomic>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <utility>

#include "fkc_common.cuh"
#include "fkc_internal.h"
#include "fkc_launch.cuh"
#include "fkc_ptx.cuh"

namespace fkc {
namespace {

using namespace fkc::ptx;

constexpr int kRowsPerSub = 128;  // UMMA M per CTA (one TMEM lane per row)
constexpr int kKBlockElems = 64;  // elements of one 128-byte swizzle row (16-bit types)
constexpr int kKBlockBytes = 128;
constexpr int kExtBytes = kNormExtBytes;  // 8 tf32 of the norm slice
// Epilogue warps: two per TMEM lane quarter (= per SM sub-partition). Measured
// on B200 at c3 (assign ms, single CTA): 8 warps 0.894, 16 warps 0.950 (more
// issue overhead per score); without any epilogue the single-CTA MMA/TMA
// pipeline takes 0.784.
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;  // warp 0 TMA, warp 1 MMA, epilogue
constexpr int kEpiWarpBegin = 2;
constexpr int kParts = kEpiWarps / 4;          // column slices of an item
constexpr int kSmemLimit = 232448;             // 227 KB opt-in per block on sm_100
constexpr int kMaxTcD = 512;  // 256 < D <= 384 on CTA pairs, wider rows streamed
// Split fp32 rows ([hi | lo], 2 Dp bf16 elements) up to fp32 D = 384.
constexpr int kMaxSplitRowElems = 768;
// Split mode partials: 2 slots per CTA x rows of a tile x (f32 score, i32 index).
constexpr int kSplitMaxCtas = 256;
constexpr int kSplitMaxRows = 256;
constexpr size_t kSplitPartialBytes = size_t{2} * kSplitMaxCtas * kSplitMaxRows * 8;

template <int DB, int MT, int NC, int ST, int CG, int XSM>
struct Cfg {
  static constexpr int kNB = NC / CG;  // centroid rows of a chunk held by one CTA
  // XSM != 0: x is streamed with the centroid chunks instead of held as a
  // resident row tile. Every stage holds one 64-element column block j of the
  // item's x rows and centroids (XSM = 2, split fp32 rows: both halves, x_hi,
  // x_lo, c_hi, c_lo), and the row tile keeps only the norm slice. Rows wider
  // than 512 elements (fp32 D > 256) fit no other way.
  static constexpr bool kXStream = XSM != 0;
  static constexpr int kHalves = XSM == 2 ? 2 : 1;
  static constexpr int kXBlockBytes = kRowsPerSub * kKBlockBytes;
  static constexpr int kXSubBytes = kXStream ? 0 : DB * kXBlockBytes;
  static constexpr int kCBlockBytes = kNB * kKBlockBytes;
  static constexpr int kCStageBytes =
      kXStream ? kHalves * (kXBlockBytes + kCBlockBytes) : DB * kCBlockBytes;
  static constexpr int kAextSubBytes = kRowsPerSub * kExtBytes;
  static constexpr int kCextStageBytes = kNB * kExtBytes;
  // Accumulator slots: all 512 TMEM columns, NC columns each (2 or 4 slots).
  static constexpr int kSlots = 512 / NC;
  // Shared memory of the whole layout with xs row-tile buffers.
  static constexpr int layout_bytes(int xs) {
    return xs * MT * (kXSubBytes + kAextSubBytes) + ST * (kCStageBytes + kCextStageBytes) +
           (2 * xs * MT + 2 * ST + 2 * kSlots + 1 + 2 * kParts) * 8 + 16 +
           kParts * MT * kRowsPerSub * 8 + 1024;
  }
  // Row-tile (x) buffers: two where they fit, so the next tile's x is loaded
  // while the MMA still reads the current one (at D <= 64 a tile is only a few
  // chunks long and a single buffer exposes the x load at every tile start).
  static constexpr int kXS = layout_bytes(2) <= kSmemLimit ? 2 : 1;
  static constexpr int kOffX = 0;
  static constexpr int kOffC = kOffX + kXS * MT * kXSubBytes;
  static constexpr int kOffAext = kOffC + ST * kCStageBytes;
  static constexpr int kOffCext = kOffAext + kXS * MT * kAextSubBytes;
  static constexpr int kOffBar = kOffCext + ST * kCextStageBytes;
  // Epilogue ownership: with two sub-tiles per tile, each half of the epilogue
  // warps can own one sub-tile (all NC columns of its items); otherwise the
  // halves split the columns of every item and exchange per-row bests. Owning
  // holds a 256-column slot while the first 128 columns are reduced (only 128
  // fit in registers), which stalls the MMA when an item's MMA is long: on
  // B200 it is faster for D <= 64 (c4 assign 123 -> 100 us) and slower at
  // D = 128 (c3 0.853 -> 0.902 ms), so it is used for short items only.
  static constexpr bool kOwn = MT == kParts && (DB == 1 || NC == 128);
  // x_full[XM] x_empty[XM] c_full[ST] c_empty[ST] acc_full[kSlots]
  // acc_empty[kSlots] drain merge_full[kParts] merge_empty[kParts], XM = kXS * MT
  static constexpr int kXM = kXS * MT;
  static constexpr int kNumBars = 2 * kXM + 2 * ST + 2 * kSlots + 1 + 2 * kParts;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  // per-row bests exchanged between column slices: (sender, sub) x 128 x (f32, i32)
  static constexpr int kOffMerge = kOffMisc + 16;
  static constexpr int kSmemBytes =
      kOffMerge + kParts * MT * kRowsPerSub * 8 + 1024;  // + alignment slack
  // bytes landing on a full barrier per phase (both CTAs for CG = 2)
  static constexpr uint32_t kXTxBytes = CG * (kXSubBytes + kAextSubBytes);
  static constexpr uint32_t kCTxBytes = CG * (kCStageBytes + kCextStageBytes);
  static constexpr uint32_t kTmemCols = kSlots * NC;
  static_assert(kSmemBytes <= kSmemLimit, "shared memory budget exceeded");
  static_assert(kSmemBytes == layout_bytes(kXS), "layout size");
  static_assert(NC % 32 == 0 && NC >= 32 && NC <= 256, "UMMA N");
  static_assert(kNB % 16 == 0, "TMA box rows / UMMA N granularity");
  static_assert(NC == 64 || NC == 128 || NC == 256, "accumulator slots tile the 512 TMEM columns");
  static_assert(NC >= 128 || CG == 2, "64-centroid chunks only on CTA pairs (UMMA M = 256)");
  static_assert(kTmemCols == 512, "TMEM allocation must be a power of two");
  static_assert(kParts >= 2, "the merge handshake expects at least two column slices");
  static_assert(!kXStream || (CG == 1 && MT == 1 && DB % kHalves == 0),
                "streamed x: single CTAs, one sub-tile, [hi | lo] rows of whole blocks");
  static_assert(DB <= 8 || kXStream, "rows wider than 512 elements need streamed x");

  // x buffer xi = (tile buffer) * MT + sub-tile
  __device__ static uint32_t x_full(uint32_t base, int xi) { return base + kOffBar + 8 * xi; }
  __device__ static uint32_t x_empty(uint32_t base, int xi) {
    return base + kOffBar + 8 * (kXM + xi);
  }
  __device__ static uint32_t c_full(uint32_t base, int st) {
    return base + kOffBar + 8 * (2 * kXM + st);
  }
  __device__ static uint32_t c_empty(uint32_t base, int st) {
    return base + kOffBar + 8 * (2 * kXM + ST + st);
  }
  __device__ static uint32_t acc_full(uint32_t base, int a) {
    return base + kOffBar + 8 * (2 * kXM + 2 * ST + a);
  }
  __device__ static uint32_t acc_empty(uint32_t base, int a) {
    return base + kOffBar + 8 * (2 * kXM + 2 * ST + kSlots + a);
  }
  __device__ static uint32_t drain(uint32_t base) {
    return base + kOffBar + 8 * (2 * kXM + 2 * ST + 2 * kSlots);
  }
  // Bests sent by slice p are ready / have been consumed.
  __device__ static uint32_t merge_full(uint32_t base, int p) {
    return base + kOffBar + 8 * (2 * kXM + 2 * ST + 2 * kSlots + 1 + p);
  }
  __device__ static uint32_t merge_empty(uint32_t base, int p) {
    return base + kOffBar + 8 * (2 * kXM + 2 * ST + 2 * kSlots + 1 + kParts + p);
  }
};

// Error codes recorded in the device error word (which wait expired).
enum : int {
  kErrProducerC = 101,
  kErrProducerX = 102,
  kErrMmaC = 111,
  kErrMmaX = 112,
  kErrMmaAcc = 113,
  kErrEpilogue = 121,
};

__device__ __forceinline__ void raise_abort(volatile int* abort_flag, int* err, int code) {
  *abort_flag = 1;
  atomicCAS(err, 0, code);
}

// Bounded wait by lane 0, result broadcast to the warp (the other lanes park in
// the shuffle instead of spinning).
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, const volatile int* abort,
                                          int lane, uint64_t deadline_ns = kWaitDeadlineNs) {
  int ok = 1;
  if (lane == 0) ok = mbar_wait(bar, parity, abort, deadline_ns) ? 1 : 0;
  return __shfl_sync(0xFFFFFFFFu, ok, 0) != 0;
}

// tcgen05.wait::ld that also "rewrites" the destination registers, so no use
// of them can be scheduled before the wait.
__device__ __forceinline__ void tmem_wait_ld_regs(uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.wait::ld.sync.aligned;"
      : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
        "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]),
        "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]),
        "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]),
        "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
      :
      : "memory");
}

// Packed key of column j: the score's bits with the 5 low mantissa bits
// replaced by j, (bits & ~31) | j, one LOP3 with j as an immediate.
template <int J>
__device__ __forceinline__ float pack_key(uint32_t bits, uint32_t mask) {
  uint32_t k;
  asm("lop3.b32 %0, %1, %2, %3, 0xEC;" : "=r"(k) : "r"(bits), "n"(J), "r"(mask));
  return __uint_as_float(k);
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ float fmax2(float a, float b) {
  float d;
  asm("max.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}

template <int... J>
__device__ __forceinline__ void pack_group(const uint32_t (&r)[32], float (&v)[32],
                                           uint32_t mask, std::integer_sequence<int, J...>) {
  ((v[J] = pack_key<J>(r[J], mask)), ...);
}

// Max over 32 packed keys: 15 three-input + 2 two-input max.f32 (17 issue
// slots; measured on B200, 3-input max runs at half the 2-input rate, so the
// win is issue slots, not ALU cycles). Scores are negative (-dist/2 - delta),
// so among keys of equal truncated score the one with the lowest j is the
// largest: ties resolve to the lowest column.
template <bool MASKED>
__device__ __forceinline__ float group_max(const uint32_t (&r)[32], uint32_t mask, int nvalid) {
  float v[32];
  pack_group(r, v, mask, std::make_integer_sequence<int, 32>{});
  if (MASKED) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = (j < nvalid) ? v[j] : -INFINITY;
  }
  float m1[11];
#pragma unroll
  for (int i = 0; i < 10; ++i) m1[i] = fmax3(v[3 * i], v[3 * i + 1], v[3 * i + 2]);
  m1[10] = fmax2(v[30], v[31]);
  float m2[4];
#pragma unroll
  for (int i = 0; i < 3; ++i) m2[i] = fmax3(m1[3 * i], m1[3 * i + 1], m1[3 * i + 2]);
  m2[3] = fmax2(m1[9], m1[10]);
  return fmax2(fmax3(m2[0], m2[1], m2[2]), m2[3]);
}

// Folds a group's winner into the running best (predicated, no branch).
// Groups arrive in ascending column order and only a strictly larger
// truncated score replaces the best, so exact ties keep the lowest column.
__device__ __forceinline__ void merge_best(float m, int col0, float& best_val, int& best_idx) {
  const uint32_t mb = __float_as_uint(m);
  const float mt = __uint_as_float(mb & 0xFFFFFFE0u);
  const int cand = col0 + static_cast<int>(mb & 31u);
  asm("{\n\t.reg .pred p;\n\t"
      "setp.gt.f32 p, %2, %0;\n\t"
      "selp.f32 %0, %2, %0, p;\n\t"
      "selp.b32 %1, %3, %1, p;\n\t}"
      : "+f"(best_val), "+r"(best_idx)
      : "f"(mt), "r"(cand));
}

// Copies this thread's NCH accumulator columns (one TMEM lane) into registers:
// all loads are issued back to back and waited for once, so the TMEM slot can be
// handed back to the MMA before any of the reduction work.
template <int NCH>
__device__ __forceinline__ void epilogue_load(uint32_t taddr, uint32_t (&r)[NCH / 32][32]) {
#pragma unroll
  for (int g = 0; g < NCH / 32; ++g) tmem_ld_32x32b_x32(taddr + g * 32, r[g]);
#pragma unroll
  for (int g = 0; g < NCH / 32; ++g) tmem_wait_ld_regs(r[g]);
}

// Folds NCH columns (already in registers) into the running best.
template <int NCH, bool MASKED>
__device__ __forceinline__ void epilogue_reduce(const uint32_t (&r)[NCH / 32][32], int valid,
                                                int col0, float& best_val, int& best_idx) {
  const uint32_t mask = 0xFFFFFFE0u;
#pragma unroll
  for (int g = 0; g < NCH / 32; ++g)
    merge_best(group_max<MASKED>(r[g], mask, valid - g * 32), col0 + g * 32, best_val, best_idx);
}

template <int CG>
__device__ __forceinline__ void tma_load(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                         int c0, int c1, int c2) {
  if constexpr (CG == 2)
    tma_load_3d_cg2(dst, map, bar, c0, c1, c2);
  else
    tma_load_3d(dst, map, bar, c0, c1, c2);
}

template <int CG>
__device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                    uint32_t acc) {
  if constexpr (CG == 2)
    umma_f16_cg2(d, a, b, idesc, acc);
  else
    umma_f16(d, a, b, idesc, acc);
}

// The norm slice: one K = 8 tf32 MMA (half the cycles of a K = 16 f16 step).
template <int CG>
__device__ __forceinline__ void mma_norm(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc) {
  if constexpr (CG == 2)
    umma_tf32_cg2(d, a, b, idesc, 1u);
  else
    umma_tf32(d, a, b, idesc, 1u);
}

// MMA completion -> barrier `bar` of this CTA, and of the peer CTA for CG = 2.
template <int CG>
__device__ __forceinline__ void mma_done(uint32_t bar) {
  if constexpr (CG == 2)
    umma_commit_cg2_pair(bar, 0x3);
  else
    umma_commit(bar);
}

// Label of one x row (a warp writes 32 consecutive rows) and its histogram
// count: lanes with the same label add once, with the number of such lanes.
__device__ __forceinline__ void write_label(int32_t* __restrict__ ids, int32_t* __restrict__ counts,
                                            int b, int N, int K, int row, int idx, int lane) {
  const bool valid_row = row < N;
  if (valid_row) ids[static_cast<size_t>(b) * N + row] = idx;
  if (counts != nullptr) {
    const uint32_t active = __ballot_sync(0xFFFFFFFFu, valid_row);
    if (valid_row) {
      const uint32_t peers = __match_any_sync(active, idx);
      if (lane == __ffs(peers) - 1)
        atomicAdd(counts + static_cast<size_t>(b) * K + idx, __popc(peers));
    }
  }
}

// Work of one CTA as segments (tile, chunks [ch0, ch1)). Whole-tile mode:
// tiles unit, unit + units, ... with all chunks. Split mode (the grid is
// balanced to the unit: total_tiles x nchunks (tile, chunk) units are cut into
// `units` contiguous equal ranges, so a tile at a range boundary is shared by
// two or more CTAs; each writes its partial per-row best to `partials` and
// splitk_fixup_kernel merges them).
struct SegIter {
  bool split;
  int nchunks, total_tiles, units;
  int64_t u, u_end;
  int tile_next;

  __device__ SegIter(bool split_, int nchunks_, int total_tiles_, int unit, int units_)
      : split(split_), nchunks(nchunks_), total_tiles(total_tiles_), units(units_), u(0),
        u_end(0), tile_next(unit) {
    if (split) {
      const int64_t U = static_cast<int64_t>(total_tiles) * nchunks;
      u = static_cast<int64_t>(unit) * U / units;
      u_end = static_cast<int64_t>(unit + 1) * U / units;
    }
  }

  __device__ bool next(int& tile, int& ch0, int& ch1) {
    if (split) {
      if (u >= u_end) return false;
      tile = static_cast<int>(u / nchunks);
      ch0 = static_cast<int>(u - static_cast<int64_t>(tile) * nchunks);
      const int64_t left = u_end - u;
      ch1 = left < nchunks - ch0 ? ch0 + static_cast<int>(left) : nchunks;
      u += ch1 - ch0;
      return true;
    }
    if (tile_next >= total_tiles) return false;
    tile = tile_next;
    ch0 = 0;
    ch1 = nchunks;
    tile_next += units;
    return true;
  }
};

template <int DB, int MT, int NC, int ST, bool BF16, int CG, bool SPLIT, int XSM>
__global__ void __launch_bounds__(kThreads, 1)
    assign_tc_kernel(const __grid_constant__ CUtensorMap tm_x,
                     const __grid_constant__ CUtensorMap tm_aext,
                     const __grid_constant__ CUtensorMap tm_c,
                     const __grid_constant__ CUtensorMap tm_cext, int32_t* __restrict__ ids,
                     int32_t* __restrict__ counts, int N, int K, int ksteps,
                     int tiles_per_batch, int total_tiles, float* __restrict__ partial_val,
                     int* __restrict__ partial_idx, int* __restrict__ err) {
  using C = Cfg<DB, MT, NC, ST, CG, XSM>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sb = smem_u32(smem);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kOffMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Position in the CTA pair (0 for CG = 1); the even CTA issues the MMAs.
  const uint32_t rank = (CG == 2) ? cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  // Full barriers and the accumulator-release barriers live in the even CTA.
  const uint32_t sb_lead = (CG == 2) ? mapa_shared(sb, 0) : sb;
  // Tiles are processed by CTA pairs (CG = 2) or single CTAs.
  const int unit = blockIdx.x / CG;
  const int units = gridDim.x / CG;
  const int rows_per_tile = CG * MT * kRowsPerSub;

  if (threadIdx.x == 0) {
    for (int xi = 0; xi < C::kXM; ++xi) {
      mbar_init(C::x_full(sb, xi), 1);
      mbar_init(C::x_empty(sb, xi), 1);
    }
    for (int st = 0; st < ST; ++st) {
      mbar_init(C::c_full(sb, st), 1);
      mbar_init(C::c_empty(sb, st), 1);
    }
    for (int a = 0; a < C::kSlots; ++a) {
      mbar_init(C::acc_full(sb, a), 1);
      // one arrival per epilogue warp that reads the slot (of both CTAs of a pair)
      mbar_init(C::acc_empty(sb, a), CG * (C::kOwn ? 4 : kEpiWarps));
    }
    mbar_init(C::drain(sb), 1);
    for (int p = 0; p < kParts; ++p) {
      mbar_init(C::merge_full(sb, p), 4);   // the four warps of the sending slice
      mbar_init(C::merge_empty(sb, p), 4);  // the four warps of the receiving slice
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_aext);
    tma_prefetch_desc(&tm_c);
    tma_prefetch_desc(&tm_cext);
  }
  if (warp == 1) {
    if constexpr (CG == 2) {
      tmem_alloc_cg2(smem_u32(tmem_holder), C::kTmemCols);
      tmem_relinquish_cg2();
    } else {
      tmem_alloc(smem_u32(tmem_holder), C::kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (CG == 2)
    cluster_sync();  // both CTAs' barriers initialised before any remote signal
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  // Everything above is independent of the previous kernel on the stream
  // (centroids, norm rows and counts come from it).
  pdl_wait();
  const int nchunks = (K + NC - 1) / NC;
  const bool split = partial_val != nullptr;  // split mode (CG = 1 only)

  // The producer runs its loop with all 32 lanes on warp-uniform values (lane 0
  // waits and issues the TMA loads); the MMA issuer is a single lane. (A warp-
  // wide MMA loop was measured slower on B200: c3 assign 0.94 ms vs 0.90 ms.)
  if (warp == 0) {
    // ---------------------------------------------------------------- TMA
    uint32_t c_it = 0, x_it = 0;
    int c_last_ph[ST];
    int x_last_ph[C::kXM];
#pragma unroll
    for (int st = 0; st < ST; ++st) c_last_ph[st] = -1;
#pragma unroll
    for (int xi = 0; xi < C::kXM; ++xi) x_last_ph[xi] = -1;
    bool ok = true;
    SegIter seg(split, nchunks, total_tiles, unit, units);
    int tile, ch0, ch1;
    while (ok && seg.next(tile, ch0, ch1)) {
      const int b = tile / tiles_per_batch;
      const int row0 = (tile - b * tiles_per_batch) * rows_per_tile +
                       static_cast<int>(rank) * MT * kRowsPerSub;
      for (int ch = ch0; ok && ch < ch1; ++ch) {
        if constexpr (C::kXStream) {
          // The tile's norm slice first: the MMA waits for it before the item's
          // first stage, and the stages below would fill the ring before it.
          if (ch == ch0) {
            const int xi = static_cast<int>(x_it % C::kXS);
            const uint32_t xph = (x_it / C::kXS) & 1u;
            if (!warp_wait(C::x_empty(sb, xi), xph ^ 1u, abort_flag, lane)) {
              if (lane == 0) raise_abort(abort_flag, err, kErrProducerX);
              ok = false;
              break;
            }
            if (lane == 0) {
              mbar_arrive_expect_tx(C::x_full(sb, xi), C::kXTxBytes);
              tma_load<CG>(sb + C::kOffAext + xi * C::kAextSubBytes, &tm_aext, C::x_full(sb, xi),
                           0, row0, b);
            }
            __syncwarp();
            x_last_ph[xi] = static_cast<int>(xph);
          }
          constexpr int PB = DB / C::kHalves;  // column blocks of one half
          const int crow = ch * NC;
          for (int j = 0; ok && j < PB; ++j) {
            const int st = static_cast<int>(c_it % ST);
            const uint32_t ph = (c_it / ST) & 1u;
            if (!warp_wait(C::c_empty(sb, st), ph ^ 1u, abort_flag, lane)) {
              if (lane == 0) raise_abort(abort_flag, err, kErrProducerC);
              ok = false;
              break;
            }
            if (lane == 0) {
              const uint32_t full = C::c_full(sb, st);
              const uint32_t stage = sb + C::kOffC + st * C::kCStageBytes;
              const uint32_t cblk = stage + C::kHalves * C::kXBlockBytes;
              mbar_arrive_expect_tx(full, C::kCTxBytes);
              tma_load<CG>(stage, &tm_x, full, j * kKBlockElems, row0, b);
              tma_load<CG>(cblk, &tm_c, full, j * kKBlockElems, crow, b);
              if constexpr (C::kHalves == 2) {
                tma_load<CG>(stage + C::kXBlockBytes, &tm_x, full, (j + PB) * kKBlockElems,
                             row0, b);
                tma_load<CG>(cblk + C::kCBlockBytes, &tm_c, full, (j + PB) * kKBlockElems, crow,
                             b);
              }
              tma_load<CG>(sb + C::kOffCext + st * C::kCextStageBytes, &tm_cext, full, 0, crow,
                           b);
            }
            __syncwarp();
            c_last_ph[st] = static_cast<int>(ph);
            ++c_it;
          }
          continue;
        }
        const int st = static_cast<int>(c_it % ST);
        const uint32_t ph = (c_it / ST) & 1u;
        if (!warp_wait(C::c_empty(sb, st), ph ^ 1u, abort_flag, lane)) {
          if (lane == 0) raise_abort(abort_flag, err, kErrProducerC);
          ok = false;
          break;
        }
        if (lane == 0) {
          if (leader) mbar_arrive_expect_tx(C::c_full(sb, st), C::kCTxBytes);
          const uint32_t full = C::c_full(sb_lead, st);
          const int crow = ch * NC + static_cast<int>(rank) * C::kNB;
#pragma unroll
          for (int kb = 0; kb < DB; ++kb)
            tma_load<CG>(sb + C::kOffC + (st * DB + kb) * C::kCBlockBytes, &tm_c, full,
                         kb * kKBlockElems, crow, b);
          tma_load<CG>(sb + C::kOffCext + st * C::kCextStageBytes, &tm_cext, full, 0, crow, b);
        }
        __syncwarp();
        c_last_ph[st] = static_cast<int>(ph);
        ++c_it;
        if (ch == ch0) {
          const int xb = static_cast<int>(x_it % C::kXS);
          const uint32_t xph = (x_it / C::kXS) & 1u;
#pragma unroll
          for (int s = 0; s < MT; ++s) {
            const int xi = xb * MT + s;
            if (!warp_wait(C::x_empty(sb, xi), xph ^ 1u, abort_flag, lane)) {
              if (lane == 0) raise_abort(abort_flag, err, kErrProducerX);
              ok = false;
              break;
            }
            if (lane == 0) {
              if (leader) mbar_arrive_expect_tx(C::x_full(sb, xi), C::kXTxBytes);
              const uint32_t xfull = C::x_full(sb_lead, xi);
#pragma unroll
              for (int kb = 0; kb < DB; ++kb)
                tma_load<CG>(sb + C::kOffX + (xi * DB + kb) * (kRowsPerSub * kKBlockBytes), &tm_x,
                             xfull, kb * kKBlockElems, row0 + s * kRowsPerSub, b);
              tma_load<CG>(sb + C::kOffAext + xi * C::kAextSubBytes, &tm_aext, xfull, 0,
                           row0 + s * kRowsPerSub, b);
            }
            __syncwarp();
            x_last_ph[xi] = static_cast<int>(xph);
          }
        }
      }
      ++x_it;
    }
    if (!ok && leader && lane == 0) {
      // Let every load already issued land before the CTA can exit (the
      // completions of both CTAs are counted on the even CTA's barriers).
#pragma unroll
      for (int st = 0; st < ST; ++st)
        if (c_last_ph[st] >= 0)
          mbar_wait(C::c_full(sb, st), static_cast<uint32_t>(c_last_ph[st]), abort_flag,
                    100000000ull);
#pragma unroll
      for (int xi = 0; xi < C::kXM; ++xi)
        if (x_last_ph[xi] >= 0)
          mbar_wait(C::x_full(sb, xi), static_cast<uint32_t>(x_last_ph[xi]), abort_flag,
                    100000000ull);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0 && leader) {
      const uint32_t idesc = umma_idesc_f16(BF16 ? 1u : 0u, CG * kRowsPerSub, NC);
      const uint32_t idesc_ext = umma_idesc_tf32(CG * kRowsPerSub, NC);
      constexpr uint32_t kHi128 = umma_desc_hi(1024, kLayoutSwizzle128B);
      constexpr uint32_t kHi32 = umma_desc_hi(256, kLayoutSwizzle32B);
      uint32_t c_it = 0, x_it = 0, item = 0;
      bool ok = true;
      SegIter seg(split, nchunks, total_tiles, unit, units);
      int tile, ch0, ch1;
      while (ok && seg.next(tile, ch0, ch1)) {
        for (int ch = ch0; ok && ch < ch1; ++ch) {
          if constexpr (C::kXStream) {
            // One item per chunk (one sub-tile): for each column block j the
            // stage's x.c K steps (split rows: x_hi.c_hi, x_hi.c_lo and
            // x_lo.c_hi), then the norm step with the last stage's centroid norm
            // slice.
            constexpr int PB = DB / C::kHalves;
            const int xi = static_cast<int>(x_it % C::kXS);
            if (ch == ch0 && !mbar_wait(C::x_full(sb, xi), (x_it / C::kXS) & 1u, abort_flag)) {
              raise_abort(abort_flag, err, kErrMmaX);
              ok = false;
              break;
            }
            const uint32_t slot = item % C::kSlots;
            if (!mbar_wait(C::acc_empty(sb, slot), ((item / C::kSlots) & 1u) ^ 1u, abort_flag)) {
              raise_abort(abort_flag, err, kErrMmaAcc);
              ok = false;
              break;
            }
            const uint32_t d_tmem = tmem_base + slot * NC;
            for (int j = 0; ok && j < PB; ++j) {
              const int st = static_cast<int>(c_it % ST);
              const uint32_t ph = (c_it / ST) & 1u;
              if (!mbar_wait(C::c_full(sb, st), ph, abort_flag)) {
                raise_abort(abort_flag, err, kErrMmaC);
                ok = false;
                break;
              }
              tc_fence_after();
              const uint32_t stage = sb + C::kOffC + st * C::kCStageBytes;
              const uint32_t a_hi = umma_desc_lo(stage);
              const uint32_t a_lo = umma_desc_lo(stage + C::kXBlockBytes);
              const uint32_t b_hi = umma_desc_lo(stage + C::kHalves * C::kXBlockBytes);
              const uint32_t b_lo =
                  umma_desc_lo(stage + C::kHalves * C::kXBlockBytes + C::kCBlockBytes);
#pragma unroll
              for (int ks = 0; ks < 4; ++ks) {
                if (j * 4 + ks < ksteps) {
                  uint32_t accf = (j > 0 || ks > 0) ? 1u : 0u;
                  asm volatile("" : "+r"(accf));
                  const uint32_t o = ks * 2;  // 32 bytes per K step, in 16-byte units
                  mma<CG>(d_tmem, umma_desc(a_hi + o, kHi128), umma_desc(b_hi + o, kHi128), idesc,
                          accf);
                  if constexpr (C::kHalves == 2) {
                    mma<CG>(d_tmem, umma_desc(a_hi + o, kHi128), umma_desc(b_lo + o, kHi128),
                            idesc, 1u);
                    mma<CG>(d_tmem, umma_desc(a_lo + o, kHi128), umma_desc(b_hi + o, kHi128),
                            idesc, 1u);
                  }
                }
              }
              if (j == PB - 1)
                mma_norm<CG>(
                    d_tmem,
                    umma_desc(umma_desc_lo(sb + C::kOffAext + xi * C::kAextSubBytes), kHi32),
                    umma_desc(umma_desc_lo(sb + C::kOffCext + st * C::kCextStageBytes), kHi32),
                    idesc_ext);
              mma_done<CG>(C::c_empty(sb, st));
              ++c_it;
            }
            if (!ok) break;
            mma_done<CG>(C::acc_full(sb, slot));
            if (ch == ch1 - 1) mma_done<CG>(C::x_empty(sb, xi));
            ++item;
            continue;
          }
          const int st = static_cast<int>(c_it % ST);
          const uint32_t ph = (c_it / ST) & 1u;
          if (!mbar_wait(C::c_full(sb, st), ph, abort_flag)) {
            raise_abort(abort_flag, err, kErrMmaC);
            ok = false;
            break;
          }
          const uint32_t c_stage = sb + C::kOffC + st * C::kCStageBytes;
#pragma unroll
          for (int s = 0; s < MT; ++s) {
            const int xi = static_cast<int>(x_it % C::kXS) * MT + s;
            if (ch == ch0 && !mbar_wait(C::x_full(sb, xi), (x_it / C::kXS) & 1u, abort_flag)) {
              raise_abort(abort_flag, err, kErrMmaX);
              ok = false;
              break;
            }
            const uint32_t slot = item % C::kSlots;
            if (!mbar_wait(C::acc_empty(sb, slot), ((item / C::kSlots) & 1u) ^ 1u, abort_flag)) {
              raise_abort(abort_flag, err, kErrMmaAcc);
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + slot * NC;
            // Few instructions per MMA: this lane shares its SM sub-partition
            // with two epilogue warps, and every issue slot it needs is one
            // they compete for (measured: the MMA stream slows by the
            // epilogue work of this sub-partition alone).
            const uint32_t a_lo = umma_desc_lo(sb + C::kOffX + xi * C::kXSubBytes);
            const uint32_t b_lo = umma_desc_lo(c_stage);
            // SPLIT (fp32 inputs): rows hold [hi | lo] bf16 halves of PB blocks
            // each; the three passes accumulate hi.hi, hi.lo and lo.hi into the
            // same accumulator (A's lo half in pass 2, B's lo half in pass 1).
            constexpr int kPasses = SPLIT ? 3 : 1;
            constexpr int PB = SPLIT ? DB / 2 : DB;  // 64-element blocks per pass
            static_assert(!SPLIT || DB % 2 == 0, "split rows: two halves of whole blocks");
#pragma unroll
            for (int pass = 0; pass < kPasses; ++pass) {
              const int ao = (SPLIT && pass == 2) ? PB : 0;
              const int bo = (SPLIT && pass == 1) ? PB : 0;
#pragma unroll
              for (int ks = 0; ks < PB * 4; ++ks) {
                if (ks < ksteps) {
                  // K step of 16 elements = 32 bytes = 2 start units; a 64-element
                  // swizzle block is block_bytes / 16 units further.
                  constexpr uint32_t kStepA = (kRowsPerSub * kKBlockBytes) >> 4;
                  constexpr uint32_t kStepB = C::kCBlockBytes >> 4;
                  const uint32_t da = ((ks >> 2) + ao) * kStepA + (ks & 3) * 2;
                  const uint32_t db = ((ks >> 2) + bo) * kStepB + (ks & 3) * 2;
                  // Opaque to the compiler: the first step's "overwrite" flag stays
                  // a runtime predicate.
                  uint32_t accf = (pass > 0 || ks > 0) ? 1u : 0u;
                  asm volatile("" : "+r"(accf));
                  mma<CG>(d_tmem, umma_desc(a_lo + da, kHi128), umma_desc(b_lo + db, kHi128),
                          idesc, accf);
                }
              }
            }
            mma_norm<CG>(d_tmem,
                         umma_desc(umma_desc_lo(sb + C::kOffAext + xi * C::kAextSubBytes), kHi32),
                         umma_desc(umma_desc_lo(sb + C::kOffCext + st * C::kCextStageBytes), kHi32),
                         idesc_ext);
            mma_done<CG>(C::acc_full(sb, slot));
            if (ch == ch1 - 1) mma_done<CG>(C::x_empty(sb, xi));
            ++item;
          }
          mma_done<CG>(C::c_empty(sb, st));
          ++c_it;
        }
        ++x_it;
      }
      // Every MMA issued above has completed once this commit arrives.
      if constexpr (CG == 2)
        umma_commit_cg2_pair(C::drain(sb), 0x1);
      else
        umma_commit(C::drain(sb));
      mbar_wait(C::drain(sb), 0u, abort_flag, ok ? kWaitDeadlineNs : 100000000ull);
    }
  } else if constexpr (C::kOwn) {
    // ------------------------------------------- epilogue, sub-tile owners
    // Warps of half p read all NC columns of the items of sub-tile p (one x
    // row per thread, TMEM lane quarter = warp % 4) and keep that row's best
    // over the whole sweep, so no per-tile merge is needed. The two warps on
    // each SM sub-partition belong to different halves and so work on items
    // one MMA apart instead of in lockstep.
    constexpr int kBatch = 128;  // columns held in registers at once
    static_assert(NC % kBatch == 0, "whole register batches per item");
    const int part = (warp - kEpiWarpBegin) >> 2;  // = the sub-tile owned
    const int q = warp & 3;
    const int row_in_sub = q * 32 + lane;
    const uint32_t lane_addr = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
    uint32_t item = 0;
    bool ok = true;
    SegIter seg(split, nchunks, total_tiles, unit, units);
    int tile, ch0, ch1;
    for (bool first_seg = true; ok && seg.next(tile, ch0, ch1); first_seg = false) {
      const int b = tile / tiles_per_batch;
      const int row0 = (tile - b * tiles_per_batch) * rows_per_tile +
                       static_cast<int>(rank) * MT * kRowsPerSub;
      float best_val = -INFINITY;
      int best_idx = 0;
      for (int ch = ch0; ok && ch < ch1; ++ch) {
#pragma unroll
        for (int s = 0; s < MT; ++s, ++item) {
          if (s != part) continue;
          const uint32_t slot = item % C::kSlots;
          int got = 1;
          if (lane == 0) got = mbar_wait(C::acc_full(sb, slot), (item / C::kSlots) & 1u, abort_flag);
          got = __shfl_sync(0xFFFFFFFFu, got, 0);
          if (!got) {
            if (lane == 0) raise_abort(abort_flag, err, kErrEpilogue);
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int h = 0; h < NC / kBatch; ++h) {
            const int col0 = ch * NC + h * kBatch;
            const int valid = min(kBatch, K - col0);  // may be <= 0 in the last chunk
            uint32_t r[kBatch / 32][32];
            if (valid > 0) epilogue_load<kBatch>(lane_addr + slot * NC + h * kBatch, r);
            if (h == NC / kBatch - 1) {
              // The last columns are in registers: release the slot to the MMA.
              tc_fence_before();
              __syncwarp();
              if (lane == 0) {
                if (CG == 1 || leader)
                  mbar_arrive(C::acc_empty(sb, slot));
                else
                  mbar_arrive_cluster_relaxed(C::acc_empty(sb_lead, slot));
              }
            }
            if (valid >= kBatch)
              epilogue_reduce<kBatch, false>(r, valid, col0, best_val, best_idx);
            else if (valid > 0)
              epilogue_reduce<kBatch, true>(r, valid, col0, best_val, best_idx);
          }
        }
      }
      if (!ok) break;
      if (ch0 != 0 || ch1 != nchunks) {
        // Part of a tile shared with other CTAs (split mode).
        const int pslot = 2 * unit + (first_seg ? 0 : 1);
        const size_t at =
            static_cast<size_t>(pslot) * rows_per_tile + part * kRowsPerSub + row_in_sub;
        partial_val[at] = best_val;
        partial_idx[at] = best_idx;
        continue;
      }
      write_label(ids, counts, b, N, K, row0 + part * kRowsPerSub + row_in_sub, best_idx, lane);
    }
  } else {
    // ----------------------------------------------------------- epilogue
    // Two column slices: slice p reads columns [p*NCH, (p+1)*NCH) of every item
    // for all 128 TMEM lanes (one x row per thread). Sub-tile s is finished
    // (labels, histogram) by slice s % 2, which takes the other slice's per-row
    // best for it through shared memory. A finished tile waits in registers and
    // is merged and written once the first item of the next tile has been
    // released to the MMA and reduced: neither slice waits for the
    // other at a tile boundary, and with two sub-tiles both share the work.
    // (The merge runs after that item's reduction, when its 128 score
    // registers are free.)
    static_assert(kParts == 2, "one peer slice");
    constexpr int NCH = NC / kParts;
    static_assert(NCH % 32 == 0, "each epilogue slice reads whole 32-column groups");
    const int part = (warp - kEpiWarpBegin) >> 2;
    const int peer = part ^ 1;
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row_in_sub = q * 32 + lane;
    const uint32_t lane_addr =
        tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(part * NCH);
    float* merge_val = reinterpret_cast<float*>(smem + C::kOffMerge);
    int* merge_idx =
        reinterpret_cast<int*>(smem + C::kOffMerge + kParts * MT * kRowsPerSub * 4);
    const bool owns = part < MT;             // finishes sub-tile `part`
    const bool sends = MT > 1 || part == 1;  // sends its bests of the other sub-tile(s)
    // The finished tile waiting for the peer's bests (pend_tile < 0: none).
    int pend_tile = -1, pend_pslot = -1, pend_idx = 0;
    float pend_val = -INFINITY;
    uint32_t tcount = 0;
    // Merges the peer's bests into the pending tile's sub-tile `part` and
    // writes its labels (or split-mode partials). Called once the tile counter
    // has moved past the pending tile.
    auto finish = [&]() -> bool {
      int got = 1;
      if (lane == 0) got = mbar_wait(C::merge_full(sb, peer), (tcount & 1u) ^ 1u, abort_flag);
      got = __shfl_sync(0xFFFFFFFFu, got, 0);
      if (!got) {
        if (lane == 0) raise_abort(abort_flag, err, kErrEpilogue);
        return false;
      }
      const int at_m = (peer * MT + part) * kRowsPerSub + row_in_sub;
      const float v1 = merge_val[at_m];
      const int i1 = merge_idx[at_m];
      __syncwarp();
      if (lane == 0) mbar_arrive(C::merge_empty(sb, peer));
      if (v1 > pend_val || (v1 == pend_val && i1 < pend_idx)) {
        pend_val = v1;
        pend_idx = i1;
      }
      if (pend_pslot >= 0) {
        const size_t at = static_cast<size_t>(pend_pslot) * rows_per_tile + part * kRowsPerSub +
                          row_in_sub;
        partial_val[at] = pend_val;
        partial_idx[at] = pend_idx;
      } else {
        const int pb = pend_tile / tiles_per_batch;
        const int prow = (pend_tile - pb * tiles_per_batch) * rows_per_tile +
                         static_cast<int>(rank) * MT * kRowsPerSub + part * kRowsPerSub +
                         row_in_sub;
        write_label(ids, counts, pb, N, K, prow, pend_idx, lane);
      }
      pend_tile = -1;
      return true;
    };
    uint32_t item = 0;
    bool ok = true;
    SegIter seg(split, nchunks, total_tiles, unit, units);
    int tile, ch0, ch1;
    for (bool first_seg = true; ok && seg.next(tile, ch0, ch1); first_seg = false, ++tcount) {
      float best_val[MT];
      int best_idx[MT];
#pragma unroll
      for (int s = 0; s < MT; ++s) {
        best_val[s] = -INFINITY;
        best_idx[s] = 0;
      }
      for (int ch = ch0; ok && ch < ch1; ++ch) {
        const int col0 = ch * NC + part * NCH;
        const int valid = min(NCH, K - col0);  // may be <= 0 in the last chunk
#pragma unroll
        for (int s = 0; s < MT; ++s) {
          const uint32_t slot = item % C::kSlots;
          int got = 1;
          if (lane == 0) got = mbar_wait(C::acc_full(sb, slot), (item / C::kSlots) & 1u, abort_flag);
          got = __shfl_sync(0xFFFFFFFFu, got, 0);
          if (!got) {
            if (lane == 0) raise_abort(abort_flag, err, kErrEpilogue);
            ok = false;
            break;
          }
          tc_fence_after();
          uint32_t r[NCH / 32][32];
          if (valid > 0) epilogue_load<NCH>(lane_addr + slot * NC, r);
          // The slot's columns are in registers: release it to the MMA now.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            // Only "TMEM read done" is signalled (tcgen05.wait::ld above): the
            // even CTA arrives locally, the odd one remotely with relaxed
            // semantics (measured: a release arrive at cluster scope made the
            // pair kernel 20% slower).
            if (CG == 1 || leader)
              mbar_arrive(C::acc_empty(sb, slot));
            else
              mbar_arrive_cluster_relaxed(C::acc_empty(sb_lead, slot));
          }
          if (valid >= NCH)
            epilogue_reduce<NCH, false>(r, valid, col0, best_val[s], best_idx[s]);
          else if (valid > 0)
            epilogue_reduce<NCH, true>(r, valid, col0, best_val[s], best_idx[s]);
          ++item;
          if (pend_tile >= 0 && !finish()) {
            ok = false;
            break;
          }
        }
      }
      if (!ok) break;
      const uint32_t mph = tcount & 1u;
      if (sends) {
        int got = 1;
        if (lane == 0) got = mbar_wait(C::merge_empty(sb, part), mph ^ 1u, abort_flag);
        got = __shfl_sync(0xFFFFFFFFu, got, 0);
        if (!got) {
          if (lane == 0) raise_abort(abort_flag, err, kErrEpilogue);
          ok = false;
          break;
        }
#pragma unroll
        for (int s = 0; s < MT; ++s) {
          if (s == part) continue;
          merge_val[(part * MT + s) * kRowsPerSub + row_in_sub] = best_val[s];
          merge_idx[(part * MT + s) * kRowsPerSub + row_in_sub] = best_idx[s];
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(C::merge_full(sb, part));
      }
      if (owns) {
        pend_tile = tile;
        pend_val = part == 0 ? best_val[0] : best_val[MT - 1];
        pend_idx = part == 0 ? best_idx[0] : best_idx[MT - 1];
        // A tile shared with other CTAs (split mode) leaves its per-row best in
        // the partials slot of this CTA's first or last segment.
        pend_pslot = (ch0 != 0 || ch1 != nchunks) ? 2 * unit + (first_seg ? 0 : 1) : -1;
      }
    }
    if (ok && pend_tile >= 0) finish();
  }
  // No remote signal may target a CTA that has exited: the pair leaves together.
  if constexpr (CG == 2)
    cluster_sync();
  else
    __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    if constexpr (CG == 2)
      tmem_dealloc_cg2(tmem_base, C::kTmemCols);
    else
      tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

// First unit of CTA c in split mode, and the CTA whose range holds unit u.
__device__ __forceinline__ int64_t split_u0(int c, int64_t U, int G) {
  return static_cast<int64_t>(c) * U / G;
}
__device__ __forceinline__ int split_cta_of(int64_t u, int64_t U, int G) {
  int c = static_cast<int>(u * G / U);
  while (c + 1 < G && split_u0(c + 1, U, G) <= u) ++c;
  while (c > 0 && split_u0(c, U, G) > u) --c;
  return c;
}

// Merges the partial per-row bests of every tile that split mode shared
// between CTAs and writes its labels (and histogram). One CTA per range
// boundary c (between CTA c-1 and c); the first boundary inside a tile
// handles it. Contributors come in ascending column order; ties keep the
// lower column (the merge compares (truncated score, index) like the kernel).
__global__ void __launch_bounds__(256) splitk_fixup_kernel(
    const float* __restrict__ partial_val, const int* __restrict__ partial_idx,
    int32_t* __restrict__ ids, int32_t* __restrict__ counts, int N, int K, int nchunks,
    int total_tiles, int tiles_per_batch, int rows_per_tile, int G) {
  pdl_wait();
  const int c = blockIdx.x + 1;
  const int64_t U = static_cast<int64_t>(total_tiles) * nchunks;
  const int64_t u0 = split_u0(c, U, G);
  if (u0 % nchunks == 0) return;  // the boundary falls between tiles
  const int t = static_cast<int>(u0 / nchunks);
  const int64_t t_begin = static_cast<int64_t>(t) * nchunks;
  if (split_u0(c - 1, U, G) > t_begin) return;  // an earlier boundary is inside t too
  const int c_first = split_cta_of(t_begin, U, G);
  const int c_last = split_cta_of(t_begin + nchunks - 1, U, G);
  const int b = t / tiles_per_batch;
  const int row0 = (t - b * tiles_per_batch) * rows_per_tile;
  const int lane = threadIdx.x & 31;
  for (int base = 0; base < rows_per_tile; base += blockDim.x) {
    const int r = base + static_cast<int>(threadIdx.x);
    const bool in_tile = r < rows_per_tile;
    float best = -INFINITY;
    int idx = 0;
    if (in_tile) {
      for (int cc = c_first; cc <= c_last; ++cc) {
        const int slot = 2 * cc + (split_u0(cc, U, G) >= t_begin ? 0 : 1);
        const float v = partial_val[static_cast<size_t>(slot) * rows_per_tile + r];
        const int i = partial_idx[static_cast<size_t>(slot) * rows_per_tile + r];
        if (v > best || (v == best && i < idx)) {
          best = v;
          idx = i;
        }
      }
    }
    const int row = row0 + r;
    const bool valid_row = in_tile && row < N;
    if (valid_row) ids[static_cast<size_t>(b) * N + row] = idx;
    if (counts != nullptr) {
      const uint32_t active = __ballot_sync(0xFFFFFFFFu, valid_row);
      if (valid_row) {
        const uint32_t peers = __match_any_sync(active, idx);
        if (lane == __ffs(peers) - 1)
          atomicAdd(counts + static_cast<size_t>(b) * K + idx, __popc(peers));
      }
    }
  }
}

// FKC_ASSIGN_CTA_GROUP=2 selects the CTA-pair kernel; default: single CTAs,
// which measured as fast or faster on B200 (assign ms, CG=1 vs CG=2: c3 0.831
// vs 0.827, c2 0.068 vs 0.072, c4 0.117 vs 0.130). The pair kernel halves the
// L2 reads of centroid chunks per SM, but both are bound by the MMA stream and
// the epilogue warps that share its SM sub-partition, and the pair adds a
// cross-CTA handshake to every accumulator slot.
int cta_group_choice() {
  static const int v = [] {
    const char* s = std::getenv("FKC_ASSIGN_CTA_GROUP");
    return (s != nullptr && std::strcmp(s, "2") == 0) ? 2 : 1;
  }();
  return v;
}

// D: elements per stored row (split fp32: 2 * Dp, the [hi | lo] halves);
// ksteps: K steps of 16 elements per pass (D / 16, or the fp32 row's D / 16).
template <int DB, int MT, int NC, int ST, bool BF16, int CG, bool SPLIT, int XSM>
int launch_tc_impl(const void* x, const void* centroids, const void* aext, const void* cext,
                   int32_t* ids, int32_t* counts, void* splitk_ws, int64_t B, int64_t N,
                   int64_t K, int64_t D, int ksteps, cudaStream_t stream) {
  using C = Cfg<DB, MT, NC, ST, CG, XSM>;
  auto kern = assign_tc_kernel<DB, MT, NC, ST, BF16, CG, SPLIT, XSM>;
  const DeviceInfo* di = nullptr;
  FKC_TRY(current_device_info(&di));
  FKC_CUDA_TRY(
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes));

  const CUtensorMapDataType tdt =
      BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  alignas(64) CUtensorMap tm_x, tm_aext, tm_c, tm_cext;
  const uint64_t es = 2;
  FKC_TRY(encode_tmap_3d(&tm_x, tdt, x, D, N, B, D * es, N * D * es, kKBlockElems, kRowsPerSub,
                         CU_TENSOR_MAP_SWIZZLE_128B));
  FKC_TRY(encode_tmap_3d(&tm_aext, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, aext, 8, N, B, kExtBytes,
                         N * kExtBytes, 8, kRowsPerSub, CU_TENSOR_MAP_SWIZZLE_32B));
  FKC_TRY(encode_tmap_3d(&tm_c, tdt, centroids, D, K, B, D * es, K * D * es, kKBlockElems,
                         C::kNB, CU_TENSOR_MAP_SWIZZLE_128B));
  FKC_TRY(encode_tmap_3d(&tm_cext, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, cext, 8, K, B, kExtBytes,
                         K * kExtBytes, 8, C::kNB, CU_TENSOR_MAP_SWIZZLE_32B));

  const int64_t rows_per_tile = static_cast<int64_t>(CG) * MT * kRowsPerSub;
  const int64_t tiles_per_batch = (N + rows_per_tile - 1) / rows_per_tile;
  const int64_t total_tiles = tiles_per_batch * B;
  FKC_REQUIRE(total_tiles < (1ll << 31), "assign: too many row tiles (%lld)",
              static_cast<long long>(total_tiles));

  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  if constexpr (CG == 1) {  // programmatic dependent launch (see fkc_launch.cuh)
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  int units = di->sm_count;
  if constexpr (CG == 2) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    // Number of CTA pairs the device can hold at once (a persistent grid must
    // not exceed it: pairs beyond it would wait for a second wave).
    static std::atomic<int> pairs_cached[64] = {};  // per device; racing threads store the same
    int pairs = pairs_cached[di->device & 63].load(std::memory_order_relaxed);
    if (pairs == 0) {
      cfg.gridDim = dim3(2 * (di->sm_count / 2), 1, 1);
      int clusters = 0;
      FKC_CUDA_TRY(cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg));
      pairs = clusters > 0 ? clusters : -1;
      pairs_cached[di->device & 63].store(pairs, std::memory_order_relaxed);
    }
    FKC_REQUIRE(pairs > 0, "assign: this device cannot co-schedule 2-CTA clusters");
    units = pairs;
  }
  int64_t n_units = std::min<int64_t>(total_tiles, units);
  // Split mode when whole tiles leave the last wave short (c3 on 8 GPUs: 256
  // tiles on 148 SMs, 86% of the grid busy): the (tile, chunk) units are cut
  // into one equal range per SM and shared tiles are merged by the fixup.
  const int64_t nchunks = (K + NC - 1) / NC;
  float* pval = nullptr;
  int* pidx = nullptr;
  if (CG == 1 && splitk_ws != nullptr && nchunks >= 2 && total_tiles % units != 0 &&
      total_tiles * nchunks >= units && units <= kSplitMaxCtas &&
      MT * kRowsPerSub <= kSplitMaxRows) {
    const int64_t waves = (total_tiles + units - 1) / units;
    const double busy = static_cast<double>(total_tiles) / static_cast<double>(waves * units);
    if (busy < 0.97) {
      n_units = units;
      pval = static_cast<float*>(splitk_ws);
      pidx = reinterpret_cast<int*>(static_cast<uint8_t*>(splitk_ws) + kSplitPartialBytes / 2);
    }
  }
  cfg.gridDim = dim3(static_cast<unsigned>(CG * n_units), 1, 1);
  FKC_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, tm_x, tm_aext, tm_c, tm_cext, ids, counts,
                                  static_cast<int>(N), static_cast<int>(K), ksteps,
                                  static_cast<int>(tiles_per_batch),
                                  static_cast<int>(total_tiles), pval, pidx,
                                  device_error_word()));
  count_launches(1);
  if (pval != nullptr && n_units > 1) {
    FKC_TRY(launch_pdl(splitk_fixup_kernel, dim3(static_cast<unsigned>(n_units - 1)), dim3(256),
                       0, stream, static_cast<const float*>(pval),
                       static_cast<const int*>(pidx), ids, counts, static_cast<int>(N),
                       static_cast<int>(K), static_cast<int>(nchunks),
                       static_cast<int>(total_tiles), static_cast<int>(tiles_per_batch),
                       static_cast<int>(rows_per_tile), static_cast<int>(n_units)));
  }
  return FKC_OK;
}

template <bool BF16, int CG>
int launch_tc_dispatch(const void* x, const void* centroids, const void* aext, const void* cext,
                       int32_t* ids, int32_t* counts, void* splitk_ws, int64_t B, int64_t N,
                       int64_t K, int64_t D, int split_d, cudaStream_t stream) {
  // (DB, MT, NC, ST) per D so that x sub-tiles + ST centroid stages fit in 227 KB.
#define FKC_TC(DB_, MT_, NC_, ST_, CG_)                                                    \
  launch_tc_impl<DB_, MT_, NC_, ST_, BF16, CG_, false, 0>(                                 \
      x, centroids, aext, cext, ids, counts, (CG_) == 1 ? splitk_ws : nullptr, B, N, K, D, \
      static_cast<int>(D / 16), stream)
#define FKC_TC_SPLIT(DB_, MT_, NC_, ST_, CG_, XST_)                                        \
  launch_tc_impl<DB_, MT_, NC_, ST_, true, CG_, true, (XST_) ? 2 : 0>(                     \
      x, centroids, aext, cext, ids, counts, (CG_) == 1 ? splitk_ws : nullptr, B, N, K, D, \
      split_d / 16, stream)
  if constexpr (BF16 && CG == 1) {
    if (split_d > 0) {
      // fp32 rows as [hi | lo] bf16 halves of Dp = D / 2 elements (a multiple of
      // 64): the configurations of a bf16 row of D = 2 Dp elements, each item
      // running three passes of split_d / 16 K steps.
      if (D <= 128) return FKC_TC_SPLIT(2, 2, 256, 2, 1, false);
      if (D <= 256) return FKC_TC_SPLIT(4, 1, 128, 2, 1, false);
      if (D <= 384) return FKC_TC_SPLIT(6, 1, 128, 2, 2, false);
      // Rows wider than 384 elements (fp32 D > 192): x streamed with the
      // centroid stages (Cfg::kXStream), three 68 KB stages of one column block
      // each. Measured at N=131072, K=2048: fp32 D=256 0.41 ms against 0.62 ms
      // for CTA pairs holding [hi | lo] row tiles with 64-centroid chunks; at
      // D=128 and D=192 the resident row tile is as fast or faster (0.235 /
      // 0.324 ms against 0.235 / 0.328 streamed).
      if (D <= 512) return FKC_TC_SPLIT(8, 1, 128, 3, 1, true);
      return D <= 640 ? FKC_TC_SPLIT(10, 1, 128, 3, 1, true)
                      : FKC_TC_SPLIT(12, 1, 128, 3, 1, true);
    }
  }
  if (D > 384) {
    if constexpr (CG == 1) {
      // 384 < D <= 512: x streamed with 256-centroid chunks (three 56 KB stages
      // of one 64-element column block of x and of the chunk each).
      return D <= 448
                 ? launch_tc_impl<7, 1, 256, 3, BF16, 1, false, 1>(
                       x, centroids, aext, cext, ids, counts, splitk_ws, B, N, K, D,
                       static_cast<int>(D / 16), stream)
                 : launch_tc_impl<8, 1, 256, 3, BF16, 1, false, 1>(
                       x, centroids, aext, cext, ids, counts, splitk_ws, B, N, K, D,
                       static_cast<int>(D / 16), stream);
    }
    // CTA pairs (opted in): 64-centroid chunks, each CTA holding 32 centroid
    // rows per stage (x 128 KB + 2 x 32 KB per CTA); an item is M = 256 x
    // N = 64 x K = D, long enough that the MMA stream dominates.
    return FKC_TC(8, 1, 64, 2, 2);
  }
  if (D > 256) {
    // A single CTA cannot hold a 128-row x sub-tile plus two stages of a
    // 128-centroid chunk in 227 KB. A CTA pair splits every chunk: each CTA
    // keeps 64 of its rows (x 96 KB + 2 x 48 KB at D = 384), and the M = 256,
    // N = 128 MMAs read the same shared-memory bytes per SM as the single-CTA
    // M = 128, N = 256 ones.
    return D <= 320 ? FKC_TC(5, 1, 128, 2, 2) : FKC_TC(6, 1, 128, 2, 2);
  }
  if constexpr (CG == 2) {
    if (D <= 64) return FKC_TC(1, 2, 256, 8, 2);
    if (D <= 128) return FKC_TC(2, 2, 256, 4, 2);
    if (D <= 192) return FKC_TC(3, 2, 256, 2, 2);
    return FKC_TC(4, 1, 256, 2, 2);
  } else {
    if (D <= 64) return FKC_TC(1, 2, 256, 3, 1);  // two x tile buffers fit
    if (D <= 128) return FKC_TC(2, 2, 256, 2, 1);
    if (D <= 192) return FKC_TC(3, 2, 128, 2, 1);
    return FKC_TC(4, 1, 128, 2, 1);
  }
#undef FKC_TC
#undef FKC_TC_SPLIT
}

}  // namespace

size_t assign_splitk_bytes() { return kSplitPartialBytes; }

bool assign_tc_supported(int64_t D, int dtype, bool split_rows) {
  if (dtype != FKC_DTYPE_F16 && dtype != FKC_DTYPE_BF16) return false;
  if (D < 16 || D % 16 != 0) return false;
  if (D > (split_rows ? kMaxSplitRowElems : kMaxTcD)) return false;
  const DeviceInfo* di = nullptr;
  if (current_device_info(&di) != FKC_OK) return false;
  return di->cc_major == 10 && di->smem_optin >= static_cast<size_t>(kSmemLimit);
}

int launch_assign_tc(const void* x, const void* centroids, const void* aext, const void* cext,
                     int32_t* ids, int32_t* counts, void* splitk_ws, int64_t B, int64_t N,
                     int64_t K, int64_t D, int dtype, cudaStream_t stream, int split_d) {
  FKC_REQUIRE(assign_tc_supported(D, dtype, split_d > 0),
              "assign_tc: unsupported D=%lld / dtype=%d", static_cast<long long>(D), dtype);
  FKC_REQUIRE(split_d == 0 || (dtype == FKC_DTYPE_BF16 && D % 128 == 0 && split_d % 16 == 0 &&
                               split_d > 0 && split_d <= D / 2),
              "assign_tc: bad split rows (D=%lld, split_d=%d)", static_cast<long long>(D),
              split_d);
  const bool bf16 = dtype == FKC_DTYPE_BF16;
  // The opt-in pair choice applies to 16-bit inputs; split fp32 rows take the
  // configuration of their width (launch_tc_dispatch).
  const bool pairs = cta_group_choice() == 2 && split_d == 0;
  if (bf16)
    return pairs ? launch_tc_dispatch<true, 2>(x, centroids, aext, cext, ids, counts, splitk_ws,
                                               B, N, K, D, 0, stream)
                 : launch_tc_dispatch<true, 1>(x, centroids, aext, cext, ids, counts, splitk_ws,
                                               B, N, K, D, split_d, stream);
  return pairs ? launch_tc_dispatch<false, 2>(x, centroids, aext, cext, ids, counts, splitk_ws, B,
                                              N, K, D, 0, stream)
               : launch_tc_dispatch<false, 1>(x, centroids, aext, cext, ids, counts, splitk_ws, B,
                                              N, K, D, 0, stream);
}

}  // namespace fkc
