// Weight-streaming projection for decode batches on B200:
//
//   y[m, n] = sum_k x[m, k] w[n, k]      (nn.Linear without bias: y = x w^T)
//
// for a few tokens (m <= 64) against a large weight, optionally for several groups at once
// (per-head weights, such as W_UV in tmla_o_unabsorb).  The layer's projections (wq_a + wkv_a
// as one GEMM, wq_b, wo: src/triton_mla/model.py:104-108 and 124 of the reference) read
// 374 MB of weights per step for 16 tokens per GPU, so the work is a stream of the weight
// through the tensor cores at HBM speed.  The weight of a group is stored [n][k] (nn.Linear)
// or [k][n] (an einsum operand); the MMA reads either layout from shared memory.
//
// Layout of the work.  The weight is cut into tiles of 128 rows (outputs, the MMA's M) by
// kStepK = 128 columns (a "k-step": two 64-column TMA boxes with 128-byte swizzled rows, so
// every weight row is read in 256 contiguous bytes).  The units (group, tile, k-step), in that
// order, are split into `grid` contiguous ranges of equal length, one per CTA (one CTA per SM,
// persistent).  A CTA's range covers the end of one tile, whole tiles and the start of
// another; each piece is a "segment".  With tile_aligned the ranges hold whole tiles.
//
// Per CTA (192 threads):
//   warp 0   TMA producer: per k-step, the weight boxes (evict-first) and the boxes of x
//            (tokens x 64 columns, evict-last: every tile re-reads them) into a ring of
//            `stages` stages.  The weight boxes of the first TMLA_LIN_EARLY stages are
//            requested before griddepcontrol.wait: under a programmatic launch they overlap
//            the preceding kernel, which must not write the weight.
//   warp 1   MMA issuer: tcgen05.mma kind::f16, M = 128 (weight rows), N = tokens rounded
//            up to 16, from shared memory (weight K-major or MN-major, x K-major), into one
//            of two TMEM accumulators (double-buffered across segments).
//   warps 2-5  epilogue: one thread per weight row (TMEM lane).  A tile covered by one
//            segment is written to y directly.  Otherwise each segment writes its fp32
//            partial into its slot of the workspace and counts itself on the tile's
//            counter; the last one sums the slots in slot order (so the result does not
//            depend on timing), writes y and resets the counter to zero.
//
// Every wait is bounded (2 s): on expiry the kernel sets TMLA_STATUS_TIMEOUT, stops,
// drains the copies and MMAs it issued, frees TMEM and returns.  No CTA waits on
// another CTA.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <type_traits>

#include "tmla_common.cuh"
#include "tmla_ptx.cuh"

namespace tmla {
namespace sm100 {
PFN_cuTensorMapEncodeTiled_v12000 encode_fn();
}

namespace linear {

using namespace ptx;

constexpr int kTileN = 128;                  // weight rows per tile (MMA M)
#ifndef TMLA_LIN_KBOXES
#define TMLA_LIN_KBOXES 2
#endif
#ifndef TMLA_LIN_PROMO
#define TMLA_LIN_PROMO 2
#endif
// Stages whose weight boxes are requested before griddepcontrol.wait.  In the layer step all
// of them (5) delayed the kernel before (its loads queue behind the prefetch) and none lost
// the overlap: 2 measured best (167.9 against 168.7 and 170.8 us for the step).
#ifndef TMLA_LIN_EARLY
#define TMLA_LIN_EARLY 2
#endif
#ifndef TMLA_LIN_EVICT_FIRST
#define TMLA_LIN_EVICT_FIRST 1
#endif
constexpr int kBoxK = 64;                    // columns per TMA box (128 bytes of 16-bit values)
constexpr int kKBoxes = TMLA_LIN_KBOXES;     // boxes per k-step: 128 * kKBoxes contiguous bytes per weight row
constexpr int kStepK = kBoxK * kKBoxes;      // columns per k-step
constexpr int kWBoxBytes = kTileN * kBoxK * 2;  // one 128 x 64 weight box
constexpr int kWStageBytes = kWBoxBytes * kKBoxes;
constexpr int kMaxStages = 16;
constexpr int kThreads = 192;
constexpr int kEpiThreads = 128;
constexpr int kAccCols = 64;                 // TMEM columns per accumulator buffer
constexpr int kTmemCols = 2 * kAccCols;
constexpr int kMaxTokens = 64;
#ifndef TMLA_LIN_RING_KB
#define TMLA_LIN_RING_KB 192
#endif
constexpr uint32_t kSmemBudget = TMLA_LIN_RING_KB * 1024;  // stage ring
constexpr uint64_t kWaitNs = 2000000000ull;

// Barrier area after the ring: full[kMaxStages], empty[kMaxStages], acc_full[2],
// acc_empty[2], mma_done, then the TMEM address, the abort flag, the "last" flag and
// two "accumulator ready" flags.
constexpr int kBarFull = 0, kBarEmpty = kMaxStages, kBarAccFull = 2 * kMaxStages, kBarAccEmpty = kBarAccFull + 2,
              kBarMmaDone = kBarAccEmpty + 2, kNumBars = kBarMmaDone + 1;
constexpr uint32_t kBarAreaBytes = 8 * kNumBars + 32;

struct Plan {
  int tokens_mma;   // MMA N
  int stages, stage_bytes;
  int n_tiles, k_steps;   // per group
  int tiles;              // groups * n_tiles
  long long units;
  int grid;
  int max_parts;    // most segments any tile is cut into
  size_t counter_bytes, partial_bytes;
  size_t smem_bytes;
};

// First unit of CTA c, and the CTA whose range holds unit u.
__host__ __device__ __forceinline__ long long unit_begin(long long c, long long units, int grid) {
  return c * units / grid;
}
__host__ __device__ __forceinline__ int unit_owner(long long u, long long units, int grid) {
  return (int)(((u + 1) * grid - 1) / units);
}

struct Args {
  int m, n, k;
  int w_kn;          // weight stored [k][n] per group (else [n][k])
  int tile_aligned;  // CTA ranges hold whole tiles (no workspace needed)
  int stages, stage_bytes, x_box_bytes;  // x_box_bytes: tokens x 64 columns
  int n_tiles, k_steps;  // tiles per group, k-steps per tile
  long long units;
  int grid, max_parts;
  void* y;
  long long y_stride, y_group_stride;
  int* counters;     // [groups * n_tiles], zero between launches
  float* partials;   // [groups * n_tiles][max_parts][tokens_mma][128]
  int* status;
  unsigned long long wait_ns;  // limit of each wait
  int stall;         // test only: CTA 0 never loads its first stage
};

// A wait that gives up after `limit_ns` or as soon as another role of the CTA gave up.
struct Waiter {
  volatile int* abort_flag;
  int* status;
  uint64_t limit_ns;
  __device__ __forceinline__ bool wait(uint32_t bar, uint32_t parity) const {
    uint64_t t0 = 0;
    for (uint32_t i = 0;; ++i) {
      if (mbar_try_wait(bar, parity)) return true;
      if ((i & 63) == 63) {
        if (*abort_flag) return false;
        const uint64_t now = globaltimer();
        if (t0 == 0) {
          t0 = now;
        } else if (now - t0 > limit_ns) {
          *abort_flag = 1;
          if (status) atomicOr(status, TMLA_STATUS_TIMEOUT);
          return false;
        }
      }
    }
  }
};

// Bounded wait for drains on the way out (no abort shortcut).
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity, uint64_t limit_ns) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity) && globaltimer() - t0 < limit_ns) {
  }
}

// Tile counters count the finished pieces of a cut tile in their low 16 bits and the
// pieces that gave up (a timed-out wait) in the high bits.  The piece that completes the
// count resets the counter to zero, and writes y only when no piece gave up.
constexpr int kPoisoned = 1 << 16;

// The weight boxes of unit (tile = group * n_tiles + t, k-step ks): per 64 columns j, 128
// rows x 64 columns at dst + j * kWBoxBytes, K-major ([n][k] storage: one box) or MN-major
// ([k][n]: two boxes of 64 n x 64 k, kWBoxBytes / 2 apart).
__device__ __forceinline__ void load_w(uint32_t dst, const CUtensorMap* tm, uint32_t bar, const Args& a, int tile,
                                       int ks, uint64_t pol) {
  const int g = tile / a.n_tiles, t = tile - g * a.n_tiles;
#pragma unroll
  for (int j = 0; j < kKBoxes; ++j) {
    const int k0 = ks * kStepK + j * kBoxK;
    const uint32_t d = dst + (uint32_t)(j * kWBoxBytes);
    if (a.w_kn) {
      tma_load_3d(d, tm, bar, t * kTileN, k0, g, pol);
      tma_load_3d(d + kWBoxBytes / 2, tm, bar, t * kTileN + 64, k0, g, pol);
    } else {
      tma_load_3d(d, tm, bar, k0, t * kTileN, g, pol);
    }
  }
}
__device__ __forceinline__ void load_x(uint32_t dst, const CUtensorMap* tm, uint32_t bar, const Args& a, int tile,
                                       int ks, uint64_t pol) {
#pragma unroll
  for (int j = 0; j < kKBoxes; ++j)
    tma_load_3d(dst + (uint32_t)(j * a.x_box_bytes), tm, bar, ks * kStepK + j * kBoxK, 0, tile / a.n_tiles, pol);
}

// 32 lanes x 16 consecutive 32-bit columns: thread i of the warp gets lane (base lane + i).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

template <typename T>
__device__ __forceinline__ T from_float(float v);
template <>
__device__ __forceinline__ __nv_bfloat16 from_float<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ __half from_float<__half>(float v) {
  return __float2half_rn(v);
}

// Segment i of this CTA: tile t and k-steps [ka, kb) of it.  Returns false past the end.
struct Segments {
  long long u, u1;
  int k_steps;
  __device__ __forceinline__ bool next(int& t, int& ka, int& kb) {
    if (u >= u1) return false;
    t = (int)(u / k_steps);
    const long long tile_end = (long long)(t + 1) * k_steps;
    const long long e = tile_end < u1 ? tile_end : u1;
    ka = (int)(u - (long long)t * k_steps);
    kb = (int)(e - (long long)t * k_steps);
    u = e;
    return true;
  }
};

template <typename T, int kTok>
__global__ void __launch_bounds__(kThreads, 1)
    linear_m16_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                      const Args a) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t bars = base + (uint32_t)(a.stages * a.stage_bytes);
  auto bar = [&](int i) { return bars + 8u * (uint32_t)i; };
  uint8_t* bar_gen = smem_raw + (bars - raw);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_gen + 8 * kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bar_gen + 8 * kNumBars + 4);
  volatile int* last_flag = reinterpret_cast<volatile int*>(bar_gen + 8 * kNumBars + 8);
  volatile int* seg_ok = reinterpret_cast<volatile int*>(bar_gen + 8 * kNumBars + 16);  // [2]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(bar(kBarFull + s), 1);
      mbar_init(bar(kBarEmpty + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar(kBarAccFull + b), 1);
      mbar_init(bar(kBarAccEmpty + b), kEpiThreads);
    }
    mbar_init(bar(kBarMmaDone), 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tm_w);
    prefetch_tmap(&tm_x);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const Waiter waiter{abort_flag, a.status, a.wait_ns};
  // Test only: CTA 0's first stage is never loaded, so the waits for it run out.
  const long long stalled = (a.stall && blockIdx.x == 0) ? 0 : -1;
  // Tile-aligned ranges (no tile is cut, so no partial sums), or equal unit ranges.
  const long long tiles = a.units / a.k_steps;
  const long long u0 = a.tile_aligned ? a.k_steps * unit_begin(blockIdx.x, tiles, a.grid)
                                      : unit_begin(blockIdx.x, a.units, a.grid);
  const long long u1 = a.tile_aligned ? a.k_steps * unit_begin(blockIdx.x + 1, tiles, a.grid)
                                      : unit_begin(blockIdx.x + 1, a.units, a.grid);

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_w = TMLA_LIN_EVICT_FIRST ? policy_evict_first() : policy_evict_normal();
      const uint64_t pol_x = policy_evict_last();
      const uint32_t tx = (uint32_t)(kKBoxes * (kWBoxBytes + a.x_box_bytes));
      const long long n_units = u1 - u0;
      // Weight boxes of the first `early` stages before the predecessor completes, then x
      // (and the weight boxes of the other first stages).
      const int pre = (int)(n_units < a.stages ? n_units : a.stages);
      const int early = pre < TMLA_LIN_EARLY ? pre : TMLA_LIN_EARLY;
      for (int i = 0; i < early; ++i) {
        if (i == stalled) continue;
        const long long u = u0 + i;
        const int tile = (int)(u / a.k_steps), ks = (int)(u - (long long)tile * a.k_steps);
        const uint32_t st = base + (uint32_t)(i * a.stage_bytes);
        mbar_arrive_expect_tx(bar(kBarFull + i), tx);
        load_w(st, &tm_w, bar(kBarFull + i), a, tile, ks, pol_w);
      }
      griddep_wait();
      griddep_launch_dependents();
      for (int i = 0; i < pre; ++i) {
        if (i == stalled) continue;
        const long long u = u0 + i;
        const int tile = (int)(u / a.k_steps), ks = (int)(u - (long long)tile * a.k_steps);
        const uint32_t st = base + (uint32_t)(i * a.stage_bytes);
        if (i >= early) {
          mbar_arrive_expect_tx(bar(kBarFull + i), tx);
          load_w(st, &tm_w, bar(kBarFull + i), a, tile, ks, pol_w);
        }
        load_x(st + kWStageBytes, &tm_x, bar(kBarFull + i), a, tile, ks, pol_x);
      }
      long long issued = pre;
      bool ok = true;
      for (long long i = pre; i < n_units && ok; ++i) {
        const int s = (int)(i % a.stages);
        const uint32_t round = (uint32_t)(i / a.stages);
        ok = waiter.wait(bar(kBarEmpty + s), (round - 1) & 1);
        if (!ok) break;
        const long long u = u0 + i;
        const int tile = (int)(u / a.k_steps), ks = (int)(u - (long long)tile * a.k_steps);
        const uint32_t st = base + (uint32_t)(s * a.stage_bytes);
        mbar_arrive_expect_tx(bar(kBarFull + s), tx);
        load_w(st, &tm_w, bar(kBarFull + s), a, tile, ks, pol_w);
        load_x(st + kWStageBytes, &tm_x, bar(kBarFull + s), a, tile, ks, pol_x);
        issued = i + 1;
      }
      if (!ok) {
        // Let the copies already in flight land before the CTA can exit.
        const long long first = issued > a.stages ? issued - a.stages : 0;
        for (long long i = first; i < issued; ++i)
          if (i != stalled) drain_wait(bar(kBarFull + (int)(i % a.stages)), (uint32_t)(i / a.stages) & 1, a.wait_ns);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t fmt = std::is_same<T, __half>::value ? 0u : 1u;
      // Bit 15: A (the weight) MN-major.
      const uint32_t idesc = idesc_f16(fmt, 128, kTok, 0) | (a.w_kn ? (1u << 15) : 0u);
      Segments seg{u0, u1, a.k_steps};
      int t, ka, kb;
      long long i = 0;  // unit counter (ring position)
      int acc_iter = 0;
      bool ok = true, issued_any = false;
      while (ok && seg.next(t, ka, kb)) {
        const int buf = acc_iter & 1;
        const int use = acc_iter >> 1;
        if (use > 0) ok = waiter.wait(bar(kBarAccEmpty + buf), (uint32_t)(use - 1) & 1);
        if (!ok) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(buf * kAccCols);
        for (int k = ka; k < kb; ++k, ++i) {
          const int s = (int)(i % a.stages);
          ok = waiter.wait(bar(kBarFull + s), (uint32_t)(i / a.stages) & 1);
          if (!ok) break;
          tc_fence_after();
          const uint32_t st = base + (uint32_t)(s * a.stage_bytes);
#pragma unroll
          for (int kk = 0; kk < kStepK / 16; ++kk) {
            // Box kk / 4 of the stage.  K-major: 16 columns are 32 bytes along the swizzled row.
            // MN-major: 16 k-rows of 128 bytes; the two 64-row halves of M are kWBoxBytes / 2 apart.
            const uint32_t wb = st + (uint32_t)((kk >> 2) * kWBoxBytes), kr = (uint32_t)(kk & 3);
            const uint64_t adesc = a.w_kn ? smem_desc(wb + kr * 16 * 128, kWBoxBytes / 2, 1024, kSwizzle128B)
                                          : smem_desc(wb + kr * 32, 16, 1024, kSwizzle128B);
            const uint32_t xb = st + (uint32_t)(kWStageBytes + (kk >> 2) * a.x_box_bytes);
            const uint64_t bdesc = smem_desc(xb + kr * 32, 16, 1024, kSwizzle128B);
            mma_ss(d, adesc, bdesc, idesc, (k > ka || kk > 0) ? 1u : 0u);
          }
          issued_any = true;
          mma_commit(bar(kBarEmpty + s));
        }
        if (!ok) break;
        mma_commit(bar(kBarAccFull + buf));
        ++acc_iter;
      }
      if (!ok && issued_any) {
        mma_commit(bar(kBarMmaDone));
        drain_wait(bar(kBarMmaDone), 0, a.wait_ns);
      }
    }
  } else {
    // Epilogue: thread `row` owns weight row (TMEM lane) row of each tile.
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    griddep_wait();
    T* y = static_cast<T*>(a.y);
    Segments seg{u0, u1, a.k_steps};
    int t, ka, kb;
    int acc_iter = 0;
    bool gave_up = false;
    while (seg.next(t, ka, kb)) {
      const int buf = acc_iter & 1;
      // One thread waits and the verdict is shared, so that all 128 threads leave
      // together on a timeout (the named barriers below count all of them).  Two flag
      // slots: slot (i & 1) is rewritten only after every thread passed barrier i + 1.
      if (row == 0) seg_ok[buf] = waiter.wait(bar(kBarAccFull + buf), (uint32_t)(acc_iter >> 1) & 1) ? 1 : 0;
      named_sync(1, kEpiThreads);
      if (!seg_ok[buf]) {
        gave_up = true;
        break;
      }
      tc_fence_after();
      float v[kTok];
#pragma unroll
      for (int c = 0; c < kTok / 16; ++c) {
        uint32_t r[16];
        tmem_ld16(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(buf * kAccCols + c * 16), r);
        tc_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; ++j) v[c * 16 + j] = __uint_as_float(r[j]);
      }
      tc_fence_before();
      mbar_arrive(bar(kBarAccEmpty + buf));
      ++acc_iter;

      const int g = t / a.n_tiles;
      const int n = (t - g * a.n_tiles) * kTileN + row;
      T* yg = y + (long long)g * a.y_group_stride;
      const long long tile_u0 = (long long)t * a.k_steps;
      const int first = a.tile_aligned ? 0 : unit_owner(tile_u0, a.units, a.grid);
      const int parts = a.tile_aligned ? 1 : unit_owner(tile_u0 + a.k_steps - 1, a.units, a.grid) - first + 1;
      if (parts == 1) {
        if (n < a.n) {
#pragma unroll
          for (int m = 0; m < kTok; ++m)
            if (m < a.m) yg[(long long)m * a.y_stride + n] = from_float<T>(v[m]);
        }
        continue;
      }
      const int slot = (int)blockIdx.x - first;
      float* mine = a.partials + ((size_t)t * a.max_parts + slot) * (size_t)(kTok * kTileN);
#pragma unroll
      for (int m = 0; m < kTok; ++m) mine[m * kTileN + row] = v[m];
      __threadfence();
      named_sync(1, kEpiThreads);
      if (row == 0) {
        const int total = atomicAdd(a.counters + t, 1) + 1;
        const bool last = (total & (kPoisoned - 1)) == parts;
        if (last && total >= kPoisoned) a.counters[t] = 0;  // a piece gave up: y stays unwritten
        *last_flag = (last && total < kPoisoned) ? 1 : 0;
      }
      named_sync(1, kEpiThreads);
      // Read before the next segment's barrier, after which the flag may be rewritten.
      if (!*last_flag) continue;
      __threadfence();
      float acc[kTok];
#pragma unroll
      for (int m = 0; m < kTok; ++m) acc[m] = 0.f;
      const float* tile_parts = a.partials + (size_t)t * a.max_parts * (size_t)(kTok * kTileN) + row;
      // kLoad slots' loads in flight at once; the sum still runs in slot order.
      constexpr int kLoad = kTok >= 64 ? 1 : 64 / kTok;
      for (int q0 = 0; q0 < parts; q0 += kLoad) {
        float part[kLoad][kTok];
#pragma unroll
        for (int j = 0; j < kLoad; ++j) {
          const int q = q0 + j < parts ? q0 + j : parts - 1;
#pragma unroll
          for (int m = 0; m < kTok; ++m) part[j][m] = __ldcg(tile_parts + (size_t)q * (kTok * kTileN) + m * kTileN);
        }
#pragma unroll
        for (int j = 0; j < kLoad; ++j) {
          if (q0 + j < parts) {
#pragma unroll
            for (int m = 0; m < kTok; ++m) acc[m] += part[j][m];
          }
        }
      }
      if (n < a.n) {
#pragma unroll
        for (int m = 0; m < kTok; ++m)
          if (m < a.m) yg[(long long)m * a.y_stride + n] = from_float<T>(acc[m]);
      }
      if (row == 0) a.counters[t] = 0;
    }
    // After a timed-out wait the rest of this CTA's pieces of cut tiles (the one whose wait
    // gave up included) are counted as given up, so that every counter ends at zero.
    if (gave_up && row == 0) {
      do {
        const long long tile_u0 = (long long)t * a.k_steps;
        const int parts = a.tile_aligned ? 1 : unit_owner(tile_u0 + a.k_steps - 1, a.units, a.grid) -
                                                  unit_owner(tile_u0, a.units, a.grid) + 1;
        if (parts > 1) {
          const int total = atomicAdd(a.counters + t, 1 + kPoisoned) + 1 + kPoisoned;
          if ((total & (kPoisoned - 1)) == parts) a.counters[t] = 0;
        }
      } while (seg.next(t, ka, kb));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------- host side

bool make_plan(int m, int n, int k, int groups, int num_sms, bool tile_aligned, Plan& pl) {
  if (m < 1 || m > kMaxTokens || n < 1 || k < 1 || groups < 1 || num_sms < 1) return false;
  pl.tokens_mma = m <= 16 ? 16 : (m <= 32 ? 32 : 64);
  pl.stage_bytes = kKBoxes * (kWBoxBytes + pl.tokens_mma * kBoxK * 2);  // multiple of 1024
  pl.stages = (int)(kSmemBudget / (uint32_t)pl.stage_bytes);
  if (pl.stages > kMaxStages) pl.stages = kMaxStages;
  pl.n_tiles = (n + kTileN - 1) / kTileN;
  pl.k_steps = (k + kStepK - 1) / kStepK;
  if ((long long)pl.n_tiles * groups > TMLA_LINEAR_MAX_TILES) return false;
  pl.tiles = pl.n_tiles * groups;
  pl.units = (long long)pl.tiles * pl.k_steps;
  const long long spread = tile_aligned ? pl.tiles : pl.units;
  pl.grid = (int)(spread < num_sms ? spread : num_sms);
  pl.max_parts = 1;
  for (int t = 0; t < (tile_aligned ? 0 : pl.tiles); ++t) {
    const long long u = (long long)t * pl.k_steps;
    const int parts = unit_owner(u + pl.k_steps - 1, pl.units, pl.grid) - unit_owner(u, pl.units, pl.grid) + 1;
    if (parts > pl.max_parts) pl.max_parts = parts;
  }
  // A fixed counter area, so that the partials of one shape never overlap the counters of
  // another shape that reuses the workspace.
  pl.counter_bytes = tile_aligned ? 0 : TMLA_LINEAR_MAX_TILES * 4;
  pl.partial_bytes =
      pl.max_parts > 1 ? (size_t)pl.tiles * pl.max_parts * pl.tokens_mma * kTileN * sizeof(float) : 0;
  pl.smem_bytes = 1024 + (size_t)pl.stages * pl.stage_bytes + kBarAreaBytes;
  return true;
}

int sm_count(int num_sms) {
  if (num_sms > 0) return num_sms;
  int dev = 0, v = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return -1;
  return v;
}

// A 3-D map {inner, outer, groups} with 128-byte swizzled boxes {box_inner, box_outer, 1}.
int encode3d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
             uint64_t groups, uint64_t row_bytes, uint64_t group_bytes, uint32_t box_inner, uint32_t box_outer) {
  auto fn = sm100::encode_fn();
  if (!fn) return TMLA_ERR_CUDA;
  cuuint64_t dims[3] = {inner, outer, groups};
  cuuint64_t strides[2] = {row_bytes, group_bytes};
  cuuint32_t box[3] = {box_inner, box_outer, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B,
                  TMLA_LIN_PROMO == 2   ? CU_TENSOR_MAP_L2_PROMOTION_L2_256B
                  : TMLA_LIN_PROMO == 1 ? CU_TENSOR_MAP_L2_PROMOTION_L2_128B
                                        : CU_TENSOR_MAP_L2_PROMOTION_NONE,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : TMLA_ERR_MISALIGNED;
}

template <typename T, int kTok>
cudaError_t launch(const CUtensorMap& tw, const CUtensorMap& tx, const Args& a, size_t smem, bool pdl,
                   cudaStream_t stream) {
  cudaError_t e =
      cudaFuncSetAttribute(linear_m16_kernel<T, kTok>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3(a.grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, linear_m16_kernel<T, kTok>, tw, tx, a);
}

}  // namespace linear
}  // namespace tmla

extern "C" {

int64_t tmla_linear_workspace_bytes(int32_t m, int32_t n, int32_t k, int32_t groups, int32_t num_sms) {
  tmla::linear::Plan pl;
  const int sms = tmla::linear::sm_count(num_sms);  // <= 0: the current device's SM count
  if (sms < 1) return -tmla::record_cuda_error(cudaGetLastError());
  if (!tmla::linear::make_plan(m, n, k, groups, sms, false, pl)) return -TMLA_ERR_INVALID_ARG;
  return (int64_t)(pl.counter_bytes + pl.partial_bytes);
}

int tmla_linear(const TmlaLinearParams* p, void* stream) {
  if (!p) return TMLA_ERR_INVALID_ARG;
  return tmla::linear_launch(*p, false, static_cast<cudaStream_t>(stream));
}

}  // extern "C"

namespace tmla {

int linear_launch(const TmlaLinearParams& pr, bool tile_aligned, cudaStream_t s) {
  using namespace tmla::linear;
  const TmlaLinearParams* p = &pr;
  if (!p->x || !p->w || !p->y) return TMLA_ERR_INVALID_ARG;
  if (p->dtype != TMLA_DTYPE_BF16 && p->dtype != TMLA_DTYPE_FP16) return TMLA_ERR_UNSUPPORTED;
  if (p->m < 1 || p->m > kMaxTokens || p->n < 1 || p->k < 1 || p->groups < 1) return TMLA_ERR_INVALID_ARG;
  if (p->w_layout != TMLA_W_NK && p->w_layout != TMLA_W_KN) return TMLA_ERR_INVALID_ARG;
  const bool kn = p->w_layout == TMLA_W_KN;
  if (p->x_stride < p->k || p->y_stride < p->n || p->w_stride < (kn ? p->n : p->k)) return TMLA_ERR_INVALID_ARG;
  if (p->groups > 1 && (p->x_group_stride < 0 || p->w_group_stride < 0 || p->y_group_stride < 0))
    return TMLA_ERR_INVALID_ARG;
  if (((uintptr_t)p->x | (uintptr_t)p->w) % 16 || p->x_stride % 8 || p->w_stride % 8 ||
      (p->groups > 1 && (p->x_group_stride % 8 || p->w_group_stride % 8)))
    return TMLA_ERR_MISALIGNED;
  const int sms = sm_count(p->num_sms);
  if (sms < 1) return record_cuda_error(cudaGetLastError());
  Plan pl;
  if (!make_plan(p->m, p->n, p->k, p->groups, sms, tile_aligned, pl)) return TMLA_ERR_INVALID_ARG;
  if (!tile_aligned && (!p->workspace || p->workspace_bytes < (int64_t)(pl.counter_bytes + pl.partial_bytes) ||
                        (uintptr_t)p->workspace % 16))
    return TMLA_ERR_WORKSPACE;
  const CUtensorMapDataType dt =
      p->dtype == TMLA_DTYPE_FP16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  // One group: the group stride of the maps is unused but must be a valid stride.
  const uint64_t w_rows = kn ? (uint64_t)p->k : (uint64_t)p->n;
  const uint64_t w_gs = p->groups > 1 ? (uint64_t)p->w_group_stride * 2 : (uint64_t)p->w_stride * 2 * w_rows;
  const uint64_t x_gs = p->groups > 1 ? (uint64_t)p->x_group_stride * 2 : (uint64_t)p->x_stride * 2 * p->m;
  CUtensorMap tw, tx;
  int rc = kn ? encode3d(&tw, dt, p->w, (uint64_t)p->n, (uint64_t)p->k, (uint64_t)p->groups,
                         (uint64_t)p->w_stride * 2, w_gs, 64, kBoxK)
              : encode3d(&tw, dt, p->w, (uint64_t)p->k, (uint64_t)p->n, (uint64_t)p->groups,
                         (uint64_t)p->w_stride * 2, w_gs, kBoxK, kTileN);
  if (!rc)
    rc = encode3d(&tx, dt, p->x, (uint64_t)p->k, (uint64_t)p->m, (uint64_t)p->groups, (uint64_t)p->x_stride * 2,
                  x_gs, kBoxK, (uint32_t)pl.tokens_mma);
  if (rc) return rc;
  Args a;
  a.m = p->m;
  a.n = p->n;
  a.k = p->k;
  a.w_kn = kn ? 1 : 0;
  a.tile_aligned = tile_aligned ? 1 : 0;
  a.stages = pl.stages;
  a.stage_bytes = pl.stage_bytes;
  a.x_box_bytes = pl.tokens_mma * kBoxK * 2;
  a.n_tiles = pl.n_tiles;
  a.k_steps = pl.k_steps;
  a.units = pl.units;
  a.grid = pl.grid;
  a.max_parts = pl.max_parts;
  a.y = p->y;
  a.y_stride = p->y_stride;
  a.y_group_stride = p->groups > 1 ? p->y_group_stride : 0;
  a.counters = tile_aligned ? nullptr : static_cast<int*>(p->workspace);
  a.partials = tile_aligned ? nullptr : reinterpret_cast<float*>(static_cast<char*>(p->workspace) + pl.counter_bytes);
  a.status = p->status;
  a.wait_ns = p->wait_ns > 0 ? (unsigned long long)p->wait_ns : kWaitNs;
  a.stall = (p->flags & TMLA_LINEAR_FLAG_TEST_STALL) ? 1 : 0;
  const bool pdl = (p->flags & TMLA_LAYER_FLAG_PDL) != 0;
  cudaError_t e;
  const bool half = p->dtype == TMLA_DTYPE_FP16;
  switch (pl.tokens_mma) {
    case 16:
      e = half ? launch<__half, 16>(tw, tx, a, pl.smem_bytes, pdl, s)
               : launch<__nv_bfloat16, 16>(tw, tx, a, pl.smem_bytes, pdl, s);
      break;
    case 32:
      e = half ? launch<__half, 32>(tw, tx, a, pl.smem_bytes, pdl, s)
               : launch<__nv_bfloat16, 32>(tw, tx, a, pl.smem_bytes, pdl, s);
      break;
    default:
      e = half ? launch<__half, 64>(tw, tx, a, pl.smem_bytes, pdl, s)
               : launch<__nv_bfloat16, 64>(tw, tx, a, pl.smem_bytes, pdl, s);
      break;
  }
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? TMLA_OK : record_cuda_error(e);
}

}  // namespace tmla
