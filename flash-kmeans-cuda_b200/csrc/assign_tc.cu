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
// The norm terms enter through one extra K=16 slice of bf16 operands:
//     A_ext[row] = {h1(x), h2(x), h3(x), 1, 1, 1, -delta(x), 0...}
//     B_ext[k]   = {1, 1, 1, h1(c), h2(c), h3(c), 1, 0...}
// where h1+h2+h3 is a three-term bf16 split (24 significant bits) of
// -0.5*||.||^2 and delta = 2^-12 ||x||^2 (+ 2^-100) is a row-constant bias.
// So TMEM holds -dist/2 - delta directly: no per-column c_sq load and no FMA
// in the epilogue, and the score is strictly negative whenever c_sq is the
// centroids' own norm (rounding of the fp32 accumulation is ~2^-22 ||x||^2).
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
// Kernel structure (one persistent CTA per SM, 64 + 32*kEpiWarps threads):
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
// MMAs of the next; two warps per scheduler hide the ALU latencies.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cmath>
#include <utility>

#include "fkc_common.cuh"
#include "fkc_internal.h"
#include "fkc_ptx.cuh"

namespace fkc {
namespace {

using namespace fkc::ptx;

constexpr int kRowsPerSub = 128;  // UMMA M (one TMEM lane per row)
constexpr int kKBlockElems = 64;  // elements of one 128-byte swizzle row (16-bit types)
constexpr int kKBlockBytes = 128;
constexpr int kExtBytes = 32;     // 16 bf16 of the norm slice
// Epilogue warps: two per TMEM lane quarter (= per SM sub-partition). Measured
// on B200 at c3 (assign ms): 8 warps 0.894, 16 warps 0.950 (more issue
// overhead per score); without any epilogue the MMA/TMA pipeline takes 0.784.
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;  // warp 0 TMA, warp 1 MMA, epilogue
constexpr int kEpiWarpBegin = 2;
constexpr int kSmemLimit = 232448;  // 227 KB opt-in per block on sm_100

template <int DB, int MT, int NC, int ST>
struct Cfg {
  static constexpr int kXSubBytes = DB * kRowsPerSub * kKBlockBytes;
  static constexpr int kCBlockBytes = NC * kKBlockBytes;
  static constexpr int kCStageBytes = DB * kCBlockBytes;
  static constexpr int kAextSubBytes = kRowsPerSub * kExtBytes;
  static constexpr int kCextStageBytes = NC * kExtBytes;
  static constexpr int kOffX = 0;
  static constexpr int kOffC = kOffX + MT * kXSubBytes;
  static constexpr int kOffAext = kOffC + ST * kCStageBytes;
  static constexpr int kOffCext = kOffAext + MT * kAextSubBytes;
  static constexpr int kOffBar = kOffCext + ST * kCextStageBytes;
  // x_full[MT] x_empty[MT] c_full[ST] c_empty[ST] acc_full[2] acc_empty[2] drain
  // merge_full merge_empty
  static constexpr int kNumBars = 2 * MT + 2 * ST + 7;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  // best per row of column parts 1..3: 3 x MT*128 x (f32, i32)
  static constexpr int kOffMerge = kOffMisc + 16;
  static constexpr int kSmemBytes = kOffMerge + 3 * MT * kRowsPerSub * 8 + 1024;  // + align slack
  static constexpr uint32_t kXTxBytes = kXSubBytes + kAextSubBytes;
  static constexpr uint32_t kCTxBytes = kCStageBytes + kCextStageBytes;
  static constexpr uint32_t kTmemCols = 2 * NC;
  static_assert(kSmemBytes <= kSmemLimit, "shared memory budget exceeded");
  static_assert(NC % 32 == 0 && NC >= 32 && NC <= 256, "UMMA N");
  static_assert(kTmemCols == 256 || kTmemCols == 512, "TMEM allocation must be a power of two");

  __device__ static uint32_t x_full(uint32_t base, int s) { return base + kOffBar + 8 * s; }
  __device__ static uint32_t x_empty(uint32_t base, int s) { return base + kOffBar + 8 * (MT + s); }
  __device__ static uint32_t c_full(uint32_t base, int st) {
    return base + kOffBar + 8 * (2 * MT + st);
  }
  __device__ static uint32_t c_empty(uint32_t base, int st) {
    return base + kOffBar + 8 * (2 * MT + ST + st);
  }
  __device__ static uint32_t acc_full(uint32_t base, int a) {
    return base + kOffBar + 8 * (2 * MT + 2 * ST + a);
  }
  __device__ static uint32_t acc_empty(uint32_t base, int a) {
    return base + kOffBar + 8 * (2 * MT + 2 * ST + 2 + a);
  }
  __device__ static uint32_t drain(uint32_t base) {
    return base + kOffBar + 8 * (2 * MT + 2 * ST + 4);
  }
  __device__ static uint32_t merge_full(uint32_t base) {
    return base + kOffBar + 8 * (2 * MT + 2 * ST + 5);
  }
  __device__ static uint32_t merge_empty(uint32_t base) {
    return base + kOffBar + 8 * (2 * MT + 2 * ST + 6);
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

// Reads NCH accumulator columns of this thread's TMEM lane and folds them into
// the running best. Loads of group g+1 are in flight while group g is reduced.
template <int NCH, bool MASKED>
__device__ __forceinline__ void epilogue_item(uint32_t taddr, int valid, int col0,
                                              float& best_val, int& best_idx) {
  constexpr int G = NCH / 32;
  const uint32_t mask = 0xFFFFFFE0u;
  uint32_t ra[32], rb[32];
  tmem_ld_32x32b_x32(taddr, ra);
  tmem_wait_ld_regs(ra);
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if ((g & 1) == 0) {
      if (g + 1 < G) tmem_ld_32x32b_x32(taddr + (g + 1) * 32, rb);
      merge_best(group_max<MASKED>(ra, mask, valid - g * 32), col0 + g * 32, best_val, best_idx);
      if (g + 1 < G) tmem_wait_ld_regs(rb);
    } else {
      if (g + 1 < G) tmem_ld_32x32b_x32(taddr + (g + 1) * 32, ra);
      merge_best(group_max<MASKED>(rb, mask, valid - g * 32), col0 + g * 32, best_val, best_idx);
      if (g + 1 < G) tmem_wait_ld_regs(ra);
    }
  }
}

template <int DB, int MT, int NC, int ST, bool BF16>
__global__ void __launch_bounds__(kThreads, 1)
    assign_tc_kernel(const __grid_constant__ CUtensorMap tm_x,
                     const __grid_constant__ CUtensorMap tm_aext,
                     const __grid_constant__ CUtensorMap tm_c,
                     const __grid_constant__ CUtensorMap tm_cext, int32_t* __restrict__ ids,
                     int32_t* __restrict__ counts, int N, int K, int ksteps,
                     int tiles_per_batch, int total_tiles, int* __restrict__ err) {
  using C = Cfg<DB, MT, NC, ST>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sb = smem_u32(smem);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kOffMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < MT; ++s) {
      mbar_init(C::x_full(sb, s), 1);
      mbar_init(C::x_empty(sb, s), 1);
    }
    for (int st = 0; st < ST; ++st) {
      mbar_init(C::c_full(sb, st), 1);
      mbar_init(C::c_empty(sb, st), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(C::acc_full(sb, a), 1);
      mbar_init(C::acc_empty(sb, a), kEpiWarps);  // one arrival per epilogue warp
    }
    mbar_init(C::drain(sb), 1);
    mbar_init(C::merge_full(sb), kEpiWarps - 4);  // the warps of column parts 1..3
    mbar_init(C::merge_empty(sb), 4);             // the four warps of part 0
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
    tmem_alloc(smem_u32(tmem_holder), C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const int nchunks = (K + NC - 1) / NC;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA
    if (lane == 0) {
      uint32_t c_it = 0, x_it = 0;
      int c_last_ph[ST];
      int x_last_ph[MT];
#pragma unroll
      for (int st = 0; st < ST; ++st) c_last_ph[st] = -1;
#pragma unroll
      for (int s = 0; s < MT; ++s) x_last_ph[s] = -1;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < total_tiles; tile += gridDim.x) {
        const int b = tile / tiles_per_batch;
        const int row0 = (tile - b * tiles_per_batch) * (MT * kRowsPerSub);
        for (int ch = 0; ok && ch < nchunks; ++ch) {
          const int st = static_cast<int>(c_it % ST);
          const uint32_t ph = (c_it / ST) & 1u;
          if (!mbar_wait(C::c_empty(sb, st), ph ^ 1u, abort_flag)) {
            raise_abort(abort_flag, err, kErrProducerC);
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(C::c_full(sb, st), C::kCTxBytes);
#pragma unroll
          for (int kb = 0; kb < DB; ++kb)
            tma_load_3d(sb + C::kOffC + (st * DB + kb) * C::kCBlockBytes, &tm_c,
                        C::c_full(sb, st), kb * kKBlockElems, ch * NC, b);
          tma_load_3d(sb + C::kOffCext + st * C::kCextStageBytes, &tm_cext, C::c_full(sb, st),
                      0, ch * NC, b);
          c_last_ph[st] = static_cast<int>(ph);
          ++c_it;
          if (ch == 0) {
#pragma unroll
            for (int s = 0; s < MT; ++s) {
              if (!mbar_wait(C::x_empty(sb, s), (x_it & 1u) ^ 1u, abort_flag)) {
                raise_abort(abort_flag, err, kErrProducerX);
                ok = false;
                break;
              }
              mbar_arrive_expect_tx(C::x_full(sb, s), C::kXTxBytes);
#pragma unroll
              for (int kb = 0; kb < DB; ++kb)
                tma_load_3d(sb + C::kOffX + (s * DB + kb) * (kRowsPerSub * kKBlockBytes), &tm_x,
                            C::x_full(sb, s), kb * kKBlockElems, row0 + s * kRowsPerSub, b);
              tma_load_3d(sb + C::kOffAext + s * C::kAextSubBytes, &tm_aext, C::x_full(sb, s), 0,
                          row0 + s * kRowsPerSub, b);
              x_last_ph[s] = static_cast<int>(x_it & 1u);
            }
          }
        }
        ++x_it;
      }
      if (!ok) {
        // Let every load already issued land before the CTA can exit.
#pragma unroll
        for (int st = 0; st < ST; ++st)
          if (c_last_ph[st] >= 0)
            mbar_wait(C::c_full(sb, st), static_cast<uint32_t>(c_last_ph[st]), abort_flag,
                      100000000ull);
#pragma unroll
        for (int s = 0; s < MT; ++s)
          if (x_last_ph[s] >= 0)
            mbar_wait(C::x_full(sb, s), static_cast<uint32_t>(x_last_ph[s]), abort_flag,
                      100000000ull);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_f16(BF16 ? 1u : 0u, kRowsPerSub, NC);
      const uint32_t idesc_ext = umma_idesc_f16(1u, kRowsPerSub, NC);
      uint32_t c_it = 0, x_it = 0, item = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < total_tiles; tile += gridDim.x) {
        for (int ch = 0; ok && ch < nchunks; ++ch) {
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
            if (ch == 0 && !mbar_wait(C::x_full(sb, s), x_it & 1u, abort_flag)) {
              raise_abort(abort_flag, err, kErrMmaX);
              ok = false;
              break;
            }
            const uint32_t slot = item & 1u;
            if (!mbar_wait(C::acc_empty(sb, slot), ((item >> 1) & 1u) ^ 1u, abort_flag)) {
              raise_abort(abort_flag, err, kErrMmaAcc);
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + slot * NC;
            const uint32_t x_sub = sb + C::kOffX + s * C::kXSubBytes;
            for (int ks = 0; ks < ksteps; ++ks) {
              const uint32_t koff = (ks >> 2), kin = (ks & 3) * 32;
              const uint64_t a_desc = umma_smem_desc(
                  x_sub + koff * (kRowsPerSub * kKBlockBytes) + kin, 1024, kLayoutSwizzle128B);
              const uint64_t b_desc =
                  umma_smem_desc(c_stage + koff * C::kCBlockBytes + kin, 1024, kLayoutSwizzle128B);
              umma_f16(d_tmem, a_desc, b_desc, idesc, ks > 0 ? 1u : 0u);
            }
            const uint64_t ae = umma_smem_desc(sb + C::kOffAext + s * C::kAextSubBytes, 256,
                                               kLayoutSwizzle32B);
            const uint64_t be = umma_smem_desc(sb + C::kOffCext + st * C::kCextStageBytes, 256,
                                               kLayoutSwizzle32B);
            umma_f16(d_tmem, ae, be, idesc_ext, 1u);
            umma_commit(C::acc_full(sb, slot));
            if (ch == nchunks - 1) umma_commit(C::x_empty(sb, s));
            ++item;
          }
          umma_commit(C::c_empty(sb, st));
          ++c_it;
        }
        ++x_it;
      }
      // Every MMA issued above has completed once this commit arrives.
      umma_commit(C::drain(sb));
      mbar_wait(C::drain(sb), 0u, abort_flag, ok ? kWaitDeadlineNs : 100000000ull);
    }
  } else {
    // ----------------------------------------------------------- epilogue
    // kParts warpgroups: part p reads columns [p*NCP, (p+1)*NCP) of every item
    // for all 128 TMEM lanes (one x row per thread). At the end of a tile parts
    // 1.. hand their per-row best to part 0 through shared memory (bounded
    // mbarrier handshake) and part 0 writes the labels.
    constexpr int kParts = kEpiWarps / 4;
    constexpr int NCH = NC / kParts;
    static_assert(NCH % 32 == 0, "each epilogue part reads whole 32-column groups");
    const int epi = warp - kEpiWarpBegin;
    const int part = epi >> 2;
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row_in_sub = q * 32 + lane;
    const uint32_t lane_addr =
        tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(part * NCH);
    float* merge_val = reinterpret_cast<float*>(smem + C::kOffMerge);
    int* merge_idx =
        reinterpret_cast<int*>(smem + C::kOffMerge + (kParts - 1) * MT * kRowsPerSub * 4);
    uint32_t item = 0, tcount = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < total_tiles; tile += gridDim.x, ++tcount) {
      const int b = tile / tiles_per_batch;
      const int row0 = (tile - b * tiles_per_batch) * (MT * kRowsPerSub);
      float best_val[MT];
      int best_idx[MT];
#pragma unroll
      for (int s = 0; s < MT; ++s) {
        best_val[s] = -INFINITY;
        best_idx[s] = 0;
      }
      for (int ch = 0; ok && ch < nchunks; ++ch) {
        const int col0 = ch * NC + part * NCH;
        const int valid = min(NCH, K - col0);  // may be <= 0 in the last chunk
#pragma unroll
        for (int s = 0; s < MT; ++s) {
          const uint32_t slot = item & 1u;
          int got = 1;
          if (lane == 0) got = mbar_wait(C::acc_full(sb, slot), (item >> 1) & 1u, abort_flag);
          got = __shfl_sync(0xFFFFFFFFu, got, 0);
          if (!got) {
            if (lane == 0) raise_abort(abort_flag, err, kErrEpilogue);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t taddr = lane_addr + slot * NC;
          if (valid >= NCH)
            epilogue_item<NCH, false>(taddr, valid, col0, best_val[s], best_idx[s]);
          else if (valid > 0)
            epilogue_item<NCH, true>(taddr, valid, col0, best_val[s], best_idx[s]);
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(C::acc_empty(sb, slot));
          ++item;
        }
      }
      if (!ok) break;
      const uint32_t mph = tcount & 1u;
      if (part > 0) {
        int got = 1;
        if (lane == 0) got = mbar_wait(C::merge_empty(sb), mph ^ 1u, abort_flag);
        got = __shfl_sync(0xFFFFFFFFu, got, 0);
        if (!got) {
          if (lane == 0) raise_abort(abort_flag, err, kErrEpilogue);
          break;
        }
#pragma unroll
        for (int s = 0; s < MT; ++s) {
          const int slot_m = ((part - 1) * MT + s) * kRowsPerSub + row_in_sub;
          merge_val[slot_m] = best_val[s];
          merge_idx[slot_m] = best_idx[s];
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(C::merge_full(sb));
        continue;
      }
      int got = 1;
      if (lane == 0) got = mbar_wait(C::merge_full(sb), mph, abort_flag);
      got = __shfl_sync(0xFFFFFFFFu, got, 0);
      if (!got) {
        if (lane == 0) raise_abort(abort_flag, err, kErrEpilogue);
        break;
      }
#pragma unroll
      for (int s = 0; s < MT; ++s) {
#pragma unroll
        for (int p = 1; p < kParts; ++p) {
          const int slot_m = ((p - 1) * MT + s) * kRowsPerSub + row_in_sub;
          const float v1 = merge_val[slot_m];
          const int i1 = merge_idx[slot_m];
          if (v1 > best_val[s] || (v1 == best_val[s] && i1 < best_idx[s])) {
            best_val[s] = v1;
            best_idx[s] = i1;
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(C::merge_empty(sb));
#pragma unroll
      for (int s = 0; s < MT; ++s) {
        const int row = row0 + s * kRowsPerSub + row_in_sub;
        const bool valid_row = row < N;
        if (valid_row) ids[static_cast<size_t>(b) * N + row] = best_idx[s];
        if (counts != nullptr) {
          const uint32_t active = __ballot_sync(0xFFFFFFFFu, valid_row);
          if (valid_row) {
            const uint32_t peers = __match_any_sync(active, best_idx[s]);
            if (lane == __ffs(peers) - 1)
              atomicAdd(counts + static_cast<size_t>(b) * K + best_idx[s], __popc(peers));
          }
        }
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

// Sum of squares of one row, one warp. 16-byte vector loads when the row
// length allows it, scalar loads otherwise.
template <typename T>
__device__ __forceinline__ float warp_row_sumsq(const T* row, int D, int lane) {
  constexpr int kVec = 16 / sizeof(T);
  float acc = 0.f;
  if ((D * sizeof(T)) % 16 == 0) {
    for (int v = lane; v * kVec < D; v += 32) {
      const uint4 u = reinterpret_cast<const uint4*>(row)[v];
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int i = 0; i < kVec; ++i) {
        const float f = to_f32<T>(e[i]);
        acc = fmaf(f, f, acc);
      }
    }
  } else {
    for (int d = lane; d < D; d += 32) {
      const float f = to_f32<T>(row[d]);
      acc = fmaf(f, f, acc);
    }
  }
  return warp_sum(acc);
}

template <typename T>
__global__ void xnorm_ext_kernel(const T* __restrict__ x, uint8_t* __restrict__ aext,
                                 int64_t rows, int D) {
  const int lane = threadIdx.x & 31;
  const int64_t warps_total = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
       r < rows; r += warps_total) {
    const float s = warp_row_sumsq<T>(x + r * D, D, lane);
    if (lane == 0) write_norm_ext(aext + r * kExtBytes, -0.5f * s, true);
  }
}

// Centroid terms: the norm-extension row (cext, nullable) and ||c||^2 (c_sq_out,
// nullable). The squared norm is taken from c_sq when given (the caller's
// value, as the reference's raw-distance path does), else computed from c.
template <typename T>
__global__ void cnorm_ext_kernel(const T* __restrict__ c, const float* __restrict__ c_sq,
                                 uint8_t* __restrict__ cext, float* __restrict__ c_sq_out,
                                 int64_t rows, int D) {
  const int lane = threadIdx.x & 31;
  const int64_t warps_total = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
       r < rows; r += warps_total) {
    const float s = (c_sq != nullptr) ? c_sq[r] : warp_row_sumsq<T>(c + r * D, D, lane);
    if (lane == 0) {
      if (cext != nullptr) write_norm_ext(cext + r * kExtBytes, -0.5f * s, false);
      if (c_sq_out != nullptr) c_sq_out[r] = s;
    }
  }
}

int grid_for_rows(int64_t rows, int warps_per_block) {
  const DeviceInfo* di = nullptr;
  int sms = 148;
  if (current_device_info(&di) == FKC_OK) sms = di->sm_count;
  int64_t blocks = (rows + warps_per_block - 1) / warps_per_block;
  const int64_t cap = static_cast<int64_t>(sms) * 16;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return static_cast<int>(blocks);
}

template <int DB, int MT, int NC, int ST, bool BF16>
int launch_tc_impl(const void* x, const void* centroids, const void* aext, const void* cext,
                   int32_t* ids, int32_t* counts, int64_t B, int64_t N, int64_t K, int64_t D,
                   cudaStream_t stream) {
  using C = Cfg<DB, MT, NC, ST>;
  auto kern = assign_tc_kernel<DB, MT, NC, ST, BF16>;
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
  FKC_TRY(encode_tmap_3d(&tm_aext, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, aext, 16, N, B, kExtBytes,
                         N * kExtBytes, 16, kRowsPerSub, CU_TENSOR_MAP_SWIZZLE_32B));
  FKC_TRY(encode_tmap_3d(&tm_c, tdt, centroids, D, K, B, D * es, K * D * es, kKBlockElems, NC,
                         CU_TENSOR_MAP_SWIZZLE_128B));
  FKC_TRY(encode_tmap_3d(&tm_cext, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, cext, 16, K, B, kExtBytes,
                         K * kExtBytes, 16, NC, CU_TENSOR_MAP_SWIZZLE_32B));

  const int64_t rows_per_tile = static_cast<int64_t>(MT) * kRowsPerSub;
  const int64_t tiles_per_batch = (N + rows_per_tile - 1) / rows_per_tile;
  const int64_t total_tiles = tiles_per_batch * B;
  FKC_REQUIRE(total_tiles < (1ll << 31), "assign: too many row tiles (%lld)",
              static_cast<long long>(total_tiles));
  const int grid = static_cast<int>(std::min<int64_t>(total_tiles, di->sm_count));
  kern<<<grid, kThreads, C::kSmemBytes, stream>>>(
      tm_x, tm_aext, tm_c, tm_cext, ids, counts, static_cast<int>(N), static_cast<int>(K),
      static_cast<int>(D / 16), static_cast<int>(tiles_per_batch), static_cast<int>(total_tiles),
      device_error_word());
  FKC_CUDA_TRY(cudaGetLastError());
  count_launches(1);
  return FKC_OK;
}

template <bool BF16>
int launch_tc_dispatch(const void* x, const void* centroids, const void* aext, const void* cext,
                       int32_t* ids, int32_t* counts, int64_t B, int64_t N, int64_t K, int64_t D,
                       cudaStream_t stream) {
  if (D <= 64)
    return launch_tc_impl<1, 2, 256, 4, BF16>(x, centroids, aext, cext, ids, counts, B, N, K, D,
                                              stream);
  if (D <= 128)
    return launch_tc_impl<2, 2, 256, 2, BF16>(x, centroids, aext, cext, ids, counts, B, N, K, D,
                                              stream);
  if (D <= 192)
    return launch_tc_impl<3, 2, 128, 2, BF16>(x, centroids, aext, cext, ids, counts, B, N, K, D,
                                              stream);
  return launch_tc_impl<4, 1, 128, 2, BF16>(x, centroids, aext, cext, ids, counts, B, N, K, D,
                                            stream);
}

}  // namespace

bool assign_tc_supported(int64_t D, int dtype) {
  if (dtype != FKC_DTYPE_F16 && dtype != FKC_DTYPE_BF16) return false;
  if (D < 16 || D > 256 || D % 16 != 0) return false;
  const DeviceInfo* di = nullptr;
  if (current_device_info(&di) != FKC_OK) return false;
  return di->cc_major == 10 && di->smem_optin >= static_cast<size_t>(kSmemLimit);
}

int launch_xnorm_ext(const void* x, void* aext, int64_t B, int64_t N, int64_t D, int dtype,
                     cudaStream_t stream) {
  const int64_t rows = B * N;
  const int grid = grid_for_rows(rows, 8);
  if (dtype == FKC_DTYPE_BF16)
    xnorm_ext_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(x), static_cast<uint8_t*>(aext), rows,
        static_cast<int>(D));
  else
    xnorm_ext_kernel<__half><<<grid, 256, 0, stream>>>(
        static_cast<const __half*>(x), static_cast<uint8_t*>(aext), rows, static_cast<int>(D));
  FKC_CUDA_TRY(cudaGetLastError());
  count_launches(1);
  return FKC_OK;
}

int launch_cnorm_ext(const void* centroids, const float* c_sq, void* cext, float* c_sq_out,
                     int64_t B, int64_t K, int64_t D, int dtype, cudaStream_t stream) {
  const int64_t rows = B * K;
  const int grid = grid_for_rows(rows, 8);
  uint8_t* ce = static_cast<uint8_t*>(cext);
  const int d = static_cast<int>(D);
  switch (dtype) {
    case FKC_DTYPE_BF16:
      cnorm_ext_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(
          static_cast<const __nv_bfloat16*>(centroids), c_sq, ce, c_sq_out, rows, d);
      break;
    case FKC_DTYPE_F16:
      cnorm_ext_kernel<__half><<<grid, 256, 0, stream>>>(static_cast<const __half*>(centroids),
                                                         c_sq, ce, c_sq_out, rows, d);
      break;
    case FKC_DTYPE_F32:
      cnorm_ext_kernel<float><<<grid, 256, 0, stream>>>(static_cast<const float*>(centroids),
                                                        c_sq, ce, c_sq_out, rows, d);
      break;
    default:
      return set_error(FKC_EINVAL, "bad dtype %d", dtype);
  }
  FKC_CUDA_TRY(cudaGetLastError());
  count_launches(1);
  return FKC_OK;
}

int launch_assign_tc(const void* x, const void* centroids, const void* aext, const void* cext,
                     int32_t* ids, int32_t* counts, int64_t B, int64_t N, int64_t K, int64_t D,
                     int dtype, cudaStream_t stream) {
  FKC_REQUIRE(assign_tc_supported(D, dtype), "assign_tc: unsupported D=%lld / dtype=%d",
              static_cast<long long>(D), dtype);
  if (dtype == FKC_DTYPE_BF16)
    return launch_tc_dispatch<true>(x, centroids, aext, cext, ids, counts, B, N, K, D, stream);
  return launch_tc_dispatch<false>(x, centroids, aext, cext, ids, counts, B, N, K, D, stream);
}

}  // namespace fkc
