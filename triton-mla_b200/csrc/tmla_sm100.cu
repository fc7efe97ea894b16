// Split-KV MLA decode for B200: TMA -> shared-memory ring -> tcgen05 tensor
// cores with accumulators in TMEM, warp-specialised, one 2-CTA cluster per
// (request, 128-head tile, split).
//
// Replaces the reference's `_mla_decode_stage1` (src/triton_mla/kernel.py:43-138)
// for its DeepSeek shape (d_qk 576 = 512 latent + 64 RoPE, d_v 512, bf16/fp16):
// same partial outputs (normalised O and base-2 LSE per split, merged by
// tmla_combine.cu), or the final output directly when there is one split.
//
// Work split inside the cluster.  A 128-head query against 576-d cache rows
// needs O = 128 x 512 fp32 (all 512 TMEM columns of one SM) plus room for the
// scores, so the two CTAs of a cluster split the latent dimension:
//   CTA r holds latent dims [256r, 256r+256) and RoPE dims [512+32r, 544+32r)
//   of Q and of every 64-token cache tile (4-stage TMA ring), and accumulates
//   O[:, 256r:256r+256] for all 128 heads in TMEM.
//   * QK: each CTA computes a partial S = Q_r . K_r^T (128 heads x 64 tokens,
//     fp32) into one of two TMEM score buffers.
//   * Softmax rows are split too: CTA r owns heads [64r, 64r+64).  Each CTA
//     sends the partial score rows of the heads it does not own to the peer
//     (16 KB per tile over distributed shared memory); the owner adds them to
//     its own partial, runs the online softmax and sends the 16-bit P rows
//     (8 KB) and the rescale factor back, so both CTAs hold the same P for all
//     128 heads in one of two TMEM P buffers.
//   * PV: each CTA accumulates O_r += P . V_r with V_r the latent half of the
//     tile it already holds: the cache is read from HBM once and no MMA is
//     duplicated.
// Score and P buffers are double-buffered and QK and PV are issued by
// different warps, so QK of tile j+1 and the score swap of tile j+1 run while
// tile j is in the softmax.
//
// TMEM (512 columns): O half 256 | Q latent dims [0,128) of the half 64 |
// S0 64 | S1 64 | P0 32 | P1 32.  Q latent dims [128,256) of the half and the
// RoPE half sit in shared memory (A operand of the remaining K steps).
//
// Warp roles (352 threads).  warp 0: TMA producer (block table -> page
// coordinates); warp 1: TMEM allocation and QK issue; warp 10: PV issue;
// warps 2-9 are two groups of four (warp w reaches TMEM lanes
// 32*(w%4)..+31, lane == head):
//   own heads, both groups   softmax, 32 of the 64 score columns each
//   peer's heads, group X    score sender: ship the partial rows to the owner
//   peer's heads, group Y    P receiver: write the owner's P into TMEM, rescale O
// O is rescaled lazily: only when a row maximum grows by more than 2^8.
//
// Every wait is bounded (2 s per wait, %globaltimer); on expiry the CTA sets
// TMLA_STATUS_TIMEOUT, all roles leave their loops, in-flight copies and MMAs
// are drained (again bounded), TMEM is freed and the kernel returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "tmla_common.cuh"
#include "tmla_ptx.cuh"

namespace tmla {
namespace sm100 {

using namespace ptx;

constexpr int kTile = 64;                 // tokens per pipeline stage
constexpr int kStages = 4;                // cache-tile ring depth
constexpr int kThreads = 352;
constexpr int kHalfLatent = 256;          // latent columns per CTA
constexpr int kHalfRope = 32;             // RoPE columns per CTA
constexpr uint32_t kBoxBytes = kTile * 128;                 // one 64-token x 64-dim swizzled box
constexpr uint32_t kRopeBytes = kTile * kHalfRope * 2;      // 64 tokens x 32 dims
constexpr uint32_t kStageBytes = 4 * kBoxBytes + kRopeBytes;  // 36864
constexpr uint32_t kRowBytes = (kHalfLatent + kHalfRope) * 2;  // cache bytes per token per CTA (576)
constexpr uint32_t kQBoxBytes = 128 * 128;                  // 128 heads x 64 dims, swizzled
constexpr uint32_t kQRopeBytes = 128 * kHalfRope * 2;       // 8192
constexpr uint32_t kSinBytes = 64 * kTile * 4;              // 16384: peer's partial S for my 64 heads
constexpr uint32_t kPinBytes = 64 * kTile * 2;              // 8192: owner's P for the peer's 64 heads
constexpr uint32_t kAlphaBytes = 64 * 4;                    // rescale factors that come with P
constexpr uint32_t kFinBytes = 64 * 8;                      // final (l, m) of the peer's heads
constexpr uint32_t kMaxBufBytes = 2048;  // row-max swap [tile parity][own quarter][half][lane], then row sums

constexpr uint32_t kOffStages = 0;
constexpr uint32_t kOffQLat = kOffStages + kStages * kStageBytes;
constexpr uint32_t kOffQRope = kOffQLat + 2 * kQBoxBytes;
constexpr uint32_t kOffSin = kOffQRope + kQRopeBytes;
constexpr uint32_t kOffPin = kOffSin + kSinBytes;
constexpr uint32_t kOffAlpha = kOffPin + kPinBytes;
constexpr uint32_t kOffFin = kOffAlpha + kAlphaBytes;
constexpr uint32_t kOffMax = kOffFin + kFinBytes;
constexpr uint32_t kOffBar = kOffMax + kMaxBufBytes;
constexpr uint32_t kNumBars = 2 * kStages + 18;
constexpr uint32_t kOffMisc = kOffBar + ((kNumBars * 8 + 63) / 64) * 64;
constexpr uint32_t kSmemBytes = kOffMisc + 64 + 1024;  // + alignment slack

constexpr uint32_t kColO = 0;
constexpr uint32_t kColQ = 256;
constexpr uint32_t kColS = 320;   // + 64 * buffer
constexpr uint32_t kColP = 448;   // + 32 * buffer

constexpr int kWarpProducer = 0;
constexpr int kWarpQK = 1;
constexpr int kWarpPV = 10;

constexpr uint64_t kWaitNs = 2000000000ull;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: P stays <= 2^8 between rescales

// Barrier indices.
enum : uint32_t {
  kBarKvFull = 0,
  kBarKvEmpty = kStages,
  kBarQFull = 2 * kStages,
  kBarSFull0,
  kBarSFull1,
  kBarSEmpty0,
  kBarSEmpty1,
  kBarPFull0,
  kBarPFull1,
  kBarPvDone0,
  kBarPvDone1,
  kBarSinFull,     // peer's partial score rows landed in my Sin buffer
  kBarSoutEmpty,   // peer has consumed what my score senders last sent
  kBarPinFull,     // owner's P rows (+ rescale factors) landed in my Pin buffer
  kBarPoutEmpty,   // peer has consumed the P rows my softmax warps last sent
  kBarFinFull,     // owner's final (l, m) of the peer's heads landed
  kBarDrainQK,
  kBarDrainPV,
  kBarHalf0,       // the two softmax warps of own quarter 0 / 1 swap row maxima (and sums)
  kBarHalf1,
};

struct Shared {
  uint32_t base;  // 1024-aligned shared address of the layout above
  __device__ uint32_t bar(uint32_t i) const { return base + kOffBar + 8 * i; }
  __device__ uint32_t stage(uint32_t s) const { return base + kOffStages + s * kStageBytes; }
};

// A wait that gives up after kWaitNs or as soon as another role gave up.
struct Waiter {
  volatile int* abort_flag;
  int* status;
  __device__ __forceinline__ bool wait(uint32_t bar, uint32_t parity, bool cluster_scope = false) const {
    uint64_t t0 = 0;
    for (uint32_t i = 0;; ++i) {
      bool ok = cluster_scope ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity);
      if (ok) return true;
      if ((i & 63) == 63) {
        if (*abort_flag) return false;
        uint64_t now = globaltimer();
        if (t0 == 0) {
          t0 = now;
        } else if (now - t0 > kWaitNs) {
          *abort_flag = 1;
          if (status) atomicOr(status, TMLA_STATUS_TIMEOUT);
          return false;
        }
      }
    }
  }
};

// Bounded wait for drains on the way out (no abort shortcut).
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity) && globaltimer() - t0 < kWaitNs) {
  }
}

struct KernelArgs {
  TmlaDecodeParams p;
  int rows_per_load;   // g: token rows per TMA box (64 for dense / page % 64 == 0)
  float scale_log2;    // softmax_scale * log2(e)
};

__device__ __forceinline__ uint32_t pack2(float a, float b, bool fp16) {
  if (fp16) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// O[row, c0:c0+32*n] *= alpha for this warp's lanes, in place in TMEM.
__device__ __forceinline__ void rescale_o(uint32_t t_row, int c0, int nchunks, float alpha) {
#pragma unroll 1
  for (int c = 0; c < nchunks; ++c) {
    uint32_t o[32];
    tmem_ld32(t_row + kColO + c0 + 32 * c, o);
    tc_wait_ld();
#pragma unroll
    for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
    tmem_st32(t_row + kColO + c0 + 32 * c, o);
  }
  tc_wait_st();
}

// Tokens past the end of the split may hold anything (even NaN); P is 0 there
// but 0 * NaN is NaN, so their V rows are zeroed before PV reads the stage.
// Called by the 128 softmax threads (thread index t in [0, 128)).
__device__ __forceinline__ void zero_tail_rows(unsigned char* stage, int nvalid, int t) {
  const int nrows = kTile - nvalid;
  for (int i = t; i < nrows * 4 * 8; i += 128) {
    const int r = nvalid + i / 32, box = (i / 8) & 3, chunk = i & 7;
    *reinterpret_cast<uint4*>(stage + box * kBoxBytes + r * 128 + chunk * 16) = make_uint4(0, 0, 0, 0);
  }
  fence_proxy_async_smem();
}

// Write columns [c0, c0 + 32*nchunks) of this CTA's output half for one head row.
template <typename T>
__device__ __forceinline__ void write_rows(const TmlaDecodeParams& p, uint32_t t_row, bool have_o, int b, int h,
                                           int split, uint32_t rank, float inv, int c0, int nchunks) {
  constexpr bool kFp16 = std::is_same<T, __half>::value;
  const bool final_out = (p.num_splits == 1) && !(p.flags & TMLA_FLAG_PARTIAL_ONLY);
  const int H = p.num_heads;
#pragma unroll 1
  for (int c = 0; c < nchunks; ++c) {
    uint32_t o[32];
    if (have_o) {
      tmem_ld32(t_row + kColO + c0 + 32 * c, o);
      tc_wait_ld();
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) o[i] = 0u;
    }
    if (h < H) {
      const int col = kHalfLatent * rank + c0 + 32 * c;
      if (final_out) {
        T* dst = static_cast<T*>(p.out) + (int64_t)b * p.out_stride_b + (int64_t)h * p.out_stride_h + col;
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          uint4 w;
          w.x = pack2(__uint_as_float(o[8 * v + 0]) * inv, __uint_as_float(o[8 * v + 1]) * inv, kFp16);
          w.y = pack2(__uint_as_float(o[8 * v + 2]) * inv, __uint_as_float(o[8 * v + 3]) * inv, kFp16);
          w.z = pack2(__uint_as_float(o[8 * v + 4]) * inv, __uint_as_float(o[8 * v + 5]) * inv, kFp16);
          w.w = pack2(__uint_as_float(o[8 * v + 6]) * inv, __uint_as_float(o[8 * v + 7]) * inv, kFp16);
          *reinterpret_cast<uint4*>(dst + 8 * v) = w;
        }
      } else {
        float* dst = p.ws_o + (((int64_t)b * H + h) * p.num_splits + split) * 512 + col;
#pragma unroll
        for (int v = 0; v < 8; ++v)
          *reinterpret_cast<float4*>(dst + 4 * v) =
              make_float4(__uint_as_float(o[4 * v]) * inv, __uint_as_float(o[4 * v + 1]) * inv,
                          __uint_as_float(o[4 * v + 2]) * inv, __uint_as_float(o[4 * v + 3]) * inv);
      }
    }
  }
}

template <typename T>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    mla_sm100_split_kernel(const __grid_constant__ CUtensorMap tm_kv_lat, const __grid_constant__ CUtensorMap tm_kv_rope,
                           const __grid_constant__ CUtensorMap tm_q_lat, const __grid_constant__ CUtensorMap tm_q_rope,
                           const __grid_constant__ KernelArgs args) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const TmlaDecodeParams& p = args.p;
  constexpr bool kFp16 = std::is_same<T, __half>::value;

  Shared sh;
  sh.base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  unsigned char* smem_gen = smem_raw + (sh.base - smem_u32(smem_raw));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem_gen + kOffMisc);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem_gen + kOffMisc + 8);
  const uint32_t tmem_slot_addr = sh.base + kOffMisc + 8;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const uint32_t peer = rank ^ 1u;
  const int head_tile = blockIdx.x >> 1;
  const int h0 = head_tile * 128;
  const int split = blockIdx.y, b = blockIdx.z;
  const int H = p.num_heads;
  Waiter waiter{abort_flag, p.status};

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    mbar_init(sh.bar(kBarQFull), 1 + 4);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(sh.bar(kBarKvFull + s), 1);
      mbar_init(sh.bar(kBarKvEmpty + s), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(sh.bar(kBarSFull0 + i), 1);
      mbar_init(sh.bar(kBarSEmpty0 + i), 6);
      mbar_init(sh.bar(kBarPFull0 + i), 6);
      mbar_init(sh.bar(kBarPvDone0 + i), 1);
    }
    mbar_init(sh.bar(kBarSinFull), 1);
    mbar_init(sh.bar(kBarSoutEmpty), 4);
    mbar_init(sh.bar(kBarPinFull), 1);
    mbar_init(sh.bar(kBarPoutEmpty), 2);
    mbar_init(sh.bar(kBarFinFull), 1);
    mbar_init(sh.bar(kBarDrainQK), 1);
    mbar_init(sh.bar(kBarDrainPV), 1);
    mbar_init(sh.bar(kBarHalf0), 2);
    mbar_init(sh.bar(kBarHalf1), 2);
    fence_mbar_init();
  }
  if (warp == kWarpQK) {
    tmem_alloc(tmem_slot_addr, 512);
    tmem_relinquish();
  }
  if (warp == kWarpProducer && lane == 0) {
    prefetch_tmap(&tm_kv_lat);
    prefetch_tmap(&tm_kv_rope);
    prefetch_tmap(&tm_q_lat);
    prefetch_tmap(&tm_q_rope);
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the peer's barriers are initialised before any remote arrive / st.async
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Token range of this split (whole 64-token tiles; see split_range).
  int len = p.seqlens[b];
  const int cap = p.block_table ? p.bt_width * p.page_size : p.page_size;
  if (len < 0 || len > cap) {
    if (p.status && threadIdx.x == 0) atomicOr(p.status, TMLA_STATUS_BAD_PAGE);
    len = len < 0 ? 0 : cap;
  }
  int start, end;
  split_range(len, p.num_splits, split, start, end);
  const int ntiles = end > start ? (end - start + kTile - 1) / kTile : 0;

  if (warp == kWarpProducer) {
    // ------------------------------------------------------------ TMA producer
    const int g = args.rows_per_load;
    const int nsub = kTile / g;
    const uint64_t pol_stream = policy_evict_first();
    if (lane == 0) {
      const uint64_t pol_q = policy_evict_last();
      mbar_arrive_expect_tx(sh.bar(kBarQFull), 2 * kQBoxBytes + kQRopeBytes);
      for (int k = 0; k < 2; ++k)
        tma_load_3d(sh.base + kOffQLat + k * kQBoxBytes, &tm_q_lat, sh.bar(kBarQFull),
                    kHalfLatent * rank + 128 + 64 * k, h0, b, pol_q);
      tma_load_3d(sh.base + kOffQRope, &tm_q_rope, sh.bar(kBarQFull), 512 + kHalfRope * rank, h0, b, pol_q);
    }
    // Page id of sub-box `sb` of tile `j` (-1: past the end of the request).
    auto page_of = [&](int j, int sb) -> int {
      const int t = start + j * kTile + sb * g;
      if (sb >= nsub || t >= end) return -1;
      if (!p.block_table) return b;
      int pg = __ldg(p.block_table + (int64_t)b * p.bt_stride + t / p.page_size);
      if (pg < 0 || (int64_t)pg >= p.num_pages) {
        if (p.status) atomicOr(p.status, TMLA_STATUS_BAD_PAGE);
        pg = 0;
      }
      return pg;
    };
    int pg_next = ntiles > 0 ? page_of(0, lane) : -1;
    int issued = 0;
    for (int j = 0; j < ntiles; ++j) {
      const int pg = pg_next;
      pg_next = (j + 1 < ntiles) ? page_of(j + 1, lane) : -1;
      const int s = j % kStages;
      bool ok = true;
      if (lane == 0 && j >= kStages) ok = waiter.wait(sh.bar(kBarKvEmpty + s), ((j / kStages) - 1) & 1);
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) break;
      const int t0 = start + j * kTile;
      const int live = min(nsub, (end - t0 + g - 1) / g);
      if (lane == 0) mbar_arrive_expect_tx(sh.bar(kBarKvFull + s), (uint32_t)(live * g) * kRowBytes);
      __syncwarp();
      if (pg >= 0) {
        const int t = t0 + lane * g;
        const int slot = p.block_table ? t % p.page_size : t;
        const uint32_t dst = sh.stage(s);
        const uint32_t bar = sh.bar(kBarKvFull + s);
#pragma unroll
        for (int kb = 0; kb < 4; ++kb)
          tma_load_3d(dst + kb * kBoxBytes + lane * g * 128, &tm_kv_lat, bar, kHalfLatent * rank + 64 * kb, slot, pg,
                      pol_stream);
        tma_load_3d(dst + 4 * kBoxBytes + lane * g * (kHalfRope * 2), &tm_kv_rope, bar, 512 + kHalfRope * rank, slot,
                    pg, pol_stream);
      }
      issued = j + 1;
    }
    // Drain: every issued load (the last ring stages and Q) has landed before the CTA may exit.
    if (lane == 0) {
      for (int j = max(0, issued - kStages); j <= issued; ++j) {
        if (j < issued)
          drain_wait(sh.bar(kBarKvFull + j % kStages), (j / kStages) & 1);
        else
          drain_wait(sh.bar(kBarQFull), 0);
      }
    }
  } else if (warp == kWarpQK) {
    // ------------------------------------------------------------ QK issuer: S[j&1] = Q_r . K_r(j)^T
    if (lane == 0) {
      const uint32_t fmt = kFp16 ? 0u : 1u;
      const uint32_t idesc = idesc_f16(fmt, 128, kTile, 0);
      const uint32_t q_lat = sh.base + kOffQLat, q_rope = sh.base + kOffQRope;
      bool ok = ntiles == 0 || waiter.wait(sh.bar(kBarQFull), 0);
      for (int j = 0; ok && j < ntiles; ++j) {
        const int s = j % kStages, sb = j & 1;
        if (!waiter.wait(sh.bar(kBarKvFull + s), (j / kStages) & 1)) break;
        // Score buffer sb was last read for tile j-2.
        if (j >= 2 && !waiter.wait(sh.bar(kBarSEmpty0 + sb), ((j - 2) >> 1) & 1)) break;
        tc_fence_after();
        const uint32_t st = sh.stage(s);
        const uint32_t d = tmem + kColS + 64 * sb;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          const uint64_t bdesc = smem_desc(st + (k >> 2) * kBoxBytes + (k & 3) * 32, 16, 1024, kSwizzle128B);
          if (k < 8) {
            mma_ts(d, tmem + kColQ + k * 8, bdesc, idesc, k > 0 ? 1u : 0u);
          } else {
            const uint64_t adesc = smem_desc(q_lat + ((k - 8) >> 2) * kQBoxBytes + (k & 3) * 32, 16, 1024,
                                             kSwizzle128B);
            mma_ss(d, adesc, bdesc, idesc, 1u);
          }
        }
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const uint64_t adesc = smem_desc(q_rope + k * 32, 16, 512, kSwizzle64B);
          const uint64_t bdesc = smem_desc(st + 4 * kBoxBytes + k * 32, 16, 512, kSwizzle64B);
          mma_ss(d, adesc, bdesc, idesc, 1u);
        }
        mma_commit(sh.bar(kBarSFull0 + sb));
      }
      mma_commit(sh.bar(kBarDrainQK));
      drain_wait(sh.bar(kBarDrainQK), 0);
    }
    __syncwarp();
  } else if (warp == kWarpPV) {
    // ------------------------------------------------------------ PV issuer: O_r += P(j) . V_r(j)
    if (lane == 0) {
      const uint32_t fmt = kFp16 ? 0u : 1u;
      const uint32_t idesc = idesc_f16(fmt, 128, kHalfLatent, 1);
      for (int j = 0; j < ntiles; ++j) {
        const int pb = j & 1;
        if (!waiter.wait(sh.bar(kBarPFull0 + pb), (j >> 1) & 1)) break;
        tc_fence_after();
        const uint32_t st = sh.stage(j % kStages);
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk) {
          // B = V: 16 tokens x 256 latent dims, MN-major 128B-swizzled, 64-dim boxes 8 KB apart.
          const uint64_t bdesc = smem_desc(st + kk * 16 * 128, kBoxBytes, 1024, kSwizzle128B);
          mma_ts(tmem + kColO, tmem + kColP + 32 * pb + kk * 8, bdesc, idesc, (j > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(sh.bar(kBarKvEmpty + j % kStages));
        mma_commit(sh.bar(kBarPvDone0 + pb));
      }
      mma_commit(sh.bar(kBarDrainPV));
      drain_wait(sh.bar(kBarDrainPV), 0);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ head-row warps (TMEM lane == head)
    const int quarter = warp & 3;
    const int grp = (warp - 2) >> 2;  // 0: warps 2-5, 1: warps 6-9
    const bool own = (uint32_t)(quarter >> 1) == rank;
    const int row = quarter * 32 + lane;
    const int idx = row & 63;  // index among the owner's 64 heads
    const int h = h0 + row;
    const uint32_t t_row = tmem + ((uint32_t)(quarter * 32) << 16);
    const int last = ntiles - 1;

    if (grp == 0) {
      // Q latent dims [0, 128) of this CTA's half -> TMEM (bf16 pairs; rows past H are zero).
      const T* qrow = static_cast<const T*>(p.q) + (int64_t)b * p.q_stride_b + (int64_t)h * p.q_stride_h +
                      kHalfLatent * rank;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t w[32];
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          uint4 x = make_uint4(0, 0, 0, 0);
          if (h < H) x = __ldg(reinterpret_cast<const uint4*>(qrow + 64 * c + 8 * v));
          w[4 * v] = x.x;
          w[4 * v + 1] = x.y;
          w[4 * v + 2] = x.z;
          w[4 * v + 3] = x.w;
        }
        tmem_st32(t_row + kColQ + 32 * c, w);
      }
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(sh.bar(kBarQFull));
    }

    if (own) {
      // ---------------------------------------------------------- softmax, columns [32 grp, 32 grp + 32)
      const int qi = quarter & 1;
      const int t128 = qi * 64 + grp * 32 + lane;  // 0..127 over the four softmax warps
      const float4* sin = reinterpret_cast<const float4*>(smem_gen + kOffSin);
      float* maxbuf = reinterpret_cast<float*>(smem_gen + kOffMax);
      const uint32_t pin_remote = map_to_rank(sh.base + kOffPin, peer);
      const uint32_t alpha_remote = map_to_rank(sh.base + kOffAlpha, peer);
      const uint32_t fin_remote = map_to_rank(sh.base + kOffFin, peer);
      const uint32_t pinfull_remote = map_to_rank(sh.bar(kBarPinFull), peer);
      const uint32_t finfull_remote = map_to_rank(sh.bar(kBarFinFull), peer);
      const uint32_t soutempty_remote = map_to_rank(sh.bar(kBarSoutEmpty), peer);
      const bool arm = qi == 0 && grp == 0 && lane == 0;
      float m_used = -INFINITY, l = 0.f;
      bool ok = true;
      for (int j = 0; j < ntiles; ++j) {
        const int sb = j & 1;
        if (arm) mbar_arrive_expect_tx(sh.bar(kBarSinFull), kSinBytes);
        if (!waiter.wait(sh.bar(kBarSFull0 + sb), (j >> 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float s[32];
        {
          uint32_t r[32];
          tmem_ld32(t_row + kColS + 64 * sb + 32 * grp, r);
          tc_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) s[i] = __uint_as_float(r[i]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(sh.bar(kBarSEmpty0 + sb));
        if (!waiter.wait(sh.bar(kBarSinFull), j & 1, true)) {
          ok = false;
          break;
        }
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const float4 v = sin[(8 * grp + c) * 64 + idx];
          s[4 * c] += v.x;
          s[4 * c + 1] += v.y;
          s[4 * c + 2] += v.z;
          s[4 * c + 3] += v.w;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster_relaxed(soutempty_remote);

        // Online softmax (base 2) with lazy rescaling; the row max is shared by the two halves.
        const int nvalid = min(kTile, end - (start + j * kTile)) - 32 * grp;
        float mx = -INFINITY;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          s[i] = (i < nvalid) ? s[i] * args.scale_log2 : -INFINITY;
          mx = fmaxf(mx, s[i]);
        }
        maxbuf[((sb * 2 + qi) * 2 + grp) * 32 + lane] = mx;
        __syncwarp();
        if (lane == 0) mbar_arrive(sh.bar(kBarHalf0 + qi));
        if (!waiter.wait(sh.bar(kBarHalf0 + qi), j & 1)) {
          ok = false;
          break;
        }
        mx = fmaxf(mx, maxbuf[((sb * 2 + qi) * 2 + (grp ^ 1)) * 32 + lane]);
        float alpha = 1.f;
        const bool need = mx > m_used + kRescaleThreshold;
        if (need) {
          alpha = ex2(m_used - mx);  // 0 on the first tile (m_used = -inf)
          m_used = mx;
        }
        uint32_t pk[16];
        float sum = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float a = ex2(s[2 * i] - m_used), c2 = ex2(s[2 * i + 1] - m_used);
          sum += a + c2;
          pk[i] = pack2(a, c2, kFp16);
        }
        l = l * alpha + sum;  // this half's share of the row sum
        // Ship P (and the rescale factor) to the peer's copy of these heads' rows.
        if (j >= 1 && !waiter.wait(sh.bar(kBarPoutEmpty), (j - 1) & 1, true)) {
          ok = false;
          break;
        }
#pragma unroll
        for (int c = 0; c < 4; ++c)
          st_async_u4(pin_remote + (uint32_t)((4 * grp + c) * 64 + idx) * 16u,
                      make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]), pinfull_remote);
        if (grp == 0) st_async_f1(alpha_remote + (uint32_t)idx * 4u, alpha, pinfull_remote);
        if (j > 0 && __any_sync(0xffffffffu, need)) {
          if (!waiter.wait(sh.bar(kBarPvDone0 + ((j - 1) & 1)), ((j - 1) >> 1) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          rescale_o(t_row, 128 * grp, 4, alpha);
        }
        // P buffer sb was last read by PV(j-2).
        if (j >= 2 && !waiter.wait(sh.bar(kBarPvDone0 + sb), ((j - 2) >> 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        tmem_st16(t_row + kColP + 32 * sb + 16 * grp, pk);
        tc_wait_st();
        if (nvalid + 32 * grp < kTile)
          zero_tail_rows(smem_gen + kOffStages + (j % kStages) * kStageBytes, nvalid + 32 * grp, t128);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(sh.bar(kBarPFull0 + sb));
      }
      // Row sum = both halves' shares; the peer normalises its half of these rows with it.
      maxbuf[256 + (qi * 2 + grp) * 32 + lane] = l;
      __syncwarp();
      if (lane == 0) mbar_arrive(sh.bar(kBarHalf0 + qi));
      if (waiter.wait(sh.bar(kBarHalf0 + qi), ntiles & 1))
        l += maxbuf[256 + (qi * 2 + (grp ^ 1)) * 32 + lane];
      else
        ok = false;
      if (grp == 0) st_async_f2(fin_remote + (uint32_t)idx * 8u, l, m_used, finfull_remote);
      bool have_o = ok && ntiles > 0;
      if (have_o) {
        have_o = waiter.wait(sh.bar(kBarPvDone0 + (last & 1)), (last >> 1) & 1);
        tc_fence_after();
      }
      write_rows<T>(p, t_row, have_o, b, h, split, rank, l > 0.f ? 1.f / l : 0.f, 128 * grp, 4);
      if (h < H && grp == 0) {
        const float lse2 = l > 0.f ? m_used + log2f(l) : -INFINITY;
        const bool final_out = (p.num_splits == 1) && !(p.flags & TMLA_FLAG_PARTIAL_ONLY);
        if (final_out) {
          if (p.lse) p.lse[(int64_t)b * p.lse_stride_b + h] = l > 0.f ? lse2 * kLn2 : -INFINITY;
        } else {
          p.ws_lse[((int64_t)b * H + h) * p.num_splits + split] = lse2;
        }
      }
    } else if (grp == 0) {
      // ---------------------------------------------------------- score sender for the peer's 64 heads
      const uint32_t sin_remote = map_to_rank(sh.base + kOffSin, peer);
      const uint32_t sinfull_remote = map_to_rank(sh.bar(kBarSinFull), peer);
      const float2* fin = reinterpret_cast<const float2*>(smem_gen + kOffFin);
      bool ok = true;
      for (int j = 0; j < ntiles; ++j) {
        const int sb = j & 1;
        if (!waiter.wait(sh.bar(kBarSFull0 + sb), (j >> 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t r0[32], r1[32];
        tmem_ld32(t_row + kColS + 64 * sb, r0);
        tmem_ld32(t_row + kColS + 64 * sb + 32, r1);
        tc_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(sh.bar(kBarSEmpty0 + sb));
        if (j >= 1 && !waiter.wait(sh.bar(kBarSoutEmpty), (j - 1) & 1, true)) {
          ok = false;
          break;
        }
#pragma unroll
        for (int c = 0; c < 8; ++c)
          st_async_u4(sin_remote + (uint32_t)(c * 64 + idx) * 16u,
                      make_uint4(r0[4 * c], r0[4 * c + 1], r0[4 * c + 2], r0[4 * c + 3]), sinfull_remote);
#pragma unroll
        for (int c = 0; c < 8; ++c)
          st_async_u4(sin_remote + (uint32_t)((8 + c) * 64 + idx) * 16u,
                      make_uint4(r1[4 * c], r1[4 * c + 1], r1[4 * c + 2], r1[4 * c + 3]), sinfull_remote);
      }
      // Epilogue share: output columns [0, 128) of these rows, normalised with the owner's row sum.
      float l = 0.f;
      bool have_o = ok && ntiles > 0;
      if (waiter.wait(sh.bar(kBarFinFull), 0, true))
        l = fin[idx].x;
      else
        have_o = false;
      if (have_o) {
        have_o = waiter.wait(sh.bar(kBarPvDone0 + (last & 1)), (last >> 1) & 1);
        tc_fence_after();
      }
      write_rows<T>(p, t_row, have_o, b, h, split, rank, l > 0.f ? 1.f / l : 0.f, 0, 4);
    } else {
      // ---------------------------------------------------------- P receiver for the peer's 64 heads
      const uint4* pin = reinterpret_cast<const uint4*>(smem_gen + kOffPin);
      const float* alpha_in = reinterpret_cast<const float*>(smem_gen + kOffAlpha);
      const float2* fin = reinterpret_cast<const float2*>(smem_gen + kOffFin);
      const uint32_t poutempty_remote = map_to_rank(sh.bar(kBarPoutEmpty), peer);
      const bool arm = (quarter & 1) == 0 && lane == 0;
      if (arm) mbar_arrive_expect_tx(sh.bar(kBarFinFull), kFinBytes);
      bool ok = true;
      for (int j = 0; j < ntiles; ++j) {
        const int pb = j & 1;
        if (arm) mbar_arrive_expect_tx(sh.bar(kBarPinFull), kPinBytes + kAlphaBytes);
        if (!waiter.wait(sh.bar(kBarPinFull), j & 1, true)) {
          ok = false;
          break;
        }
        const float alpha = alpha_in[idx];
        uint32_t pk[32];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 v = pin[c * 64 + idx];
          pk[4 * c] = v.x;
          pk[4 * c + 1] = v.y;
          pk[4 * c + 2] = v.z;
          pk[4 * c + 3] = v.w;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster_relaxed(poutempty_remote);
        const bool need = j > 0 && alpha != 1.f;
        if (__any_sync(0xffffffffu, need)) {
          if (!waiter.wait(sh.bar(kBarPvDone0 + ((j - 1) & 1)), ((j - 1) >> 1) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          rescale_o(t_row, 0, 8, need ? alpha : 1.f);
        }
        if (j >= 2 && !waiter.wait(sh.bar(kBarPvDone0 + pb), ((j - 2) >> 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        tmem_st32(t_row + kColP + 32 * pb, pk);
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(sh.bar(kBarPFull0 + pb));
      }
      // Epilogue share: output columns [128, 256) of these rows.
      float l = 0.f;
      bool have_o = ok && ntiles > 0;
      if (waiter.wait(sh.bar(kBarFinFull), 0, true))
        l = fin[idx].x;
      else
        have_o = false;
      if (have_o) {
        have_o = waiter.wait(sh.bar(kBarPvDone0 + (last & 1)), (last >> 1) & 1);
        tc_fence_after();
      }
      write_rows<T>(p, t_row, have_o, b, h, split, rank, l > 0.f ? 1.f / l : 0.f, 128, 4);
    }
  }

  // Teardown: both CTAs are done with each other's shared memory before either exits.
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == kWarpQK) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------- host side

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

static int encode3d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                    uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t box0, uint32_t box1,
                    CUtensorMapSwizzle swz) {
  auto fn = encode_fn();
  if (!fn) return TMLA_ERR_CUDA;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  cuuint32_t box[3] = {box0, box1, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : TMLA_ERR_MISALIGNED;
}

static int pow2_rows(int page) {
  int g = 64;
  while (g > 1 && page % g) g >>= 1;
  return g;
}

}  // namespace sm100

int sm100_supported(const TmlaDecodeParams& p) {
  if (p.d_qk != 576 || p.d_v != 512) return 0;
  if (p.dtype != TMLA_DTYPE_BF16 && p.dtype != TMLA_DTYPE_FP16) return 0;
  if (p.batch > 65535 || p.num_splits > 65535) return 0;
  if (((uintptr_t)p.q | (uintptr_t)p.kv) % 16) return 0;
  if (p.q_stride_b % 8 || p.q_stride_h % 8 || p.kv_stride_page % 8 || p.kv_stride_tok % 8) return 0;
  if ((uintptr_t)p.out % 16 || p.out_stride_b % 8 || p.out_stride_h % 8) return 0;
  if (p.block_table && sm100::pow2_rows(p.page_size) < 8) return 0;
  return 1;
}

int launch_sm100(const TmlaDecodeParams& p, cudaStream_t stream) {
  using namespace sm100;
  if (!sm100_supported(p)) return TMLA_ERR_UNSUPPORTED;
  const CUtensorMapDataType dt =
      p.dtype == TMLA_DTYPE_FP16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const int g = p.block_table ? pow2_rows(p.page_size) : kTile;
  const uint64_t pages = p.block_table ? (uint64_t)p.num_pages : (uint64_t)p.batch;
  CUtensorMap tm_lat, tm_rope, tm_q, tm_qlat;
  int rc = encode3d(&tm_lat, dt, p.kv, 576, (uint64_t)p.page_size, pages, (uint64_t)p.kv_stride_tok * 2,
                    (uint64_t)p.kv_stride_page * 2, 64, (uint32_t)g, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc)
    rc = encode3d(&tm_rope, dt, p.kv, 576, (uint64_t)p.page_size, pages, (uint64_t)p.kv_stride_tok * 2,
                  (uint64_t)p.kv_stride_page * 2, kHalfRope, (uint32_t)g, CU_TENSOR_MAP_SWIZZLE_64B);
  if (!rc)
    rc = encode3d(&tm_q, dt, p.q, 576, (uint64_t)p.num_heads, (uint64_t)p.batch, (uint64_t)p.q_stride_h * 2,
                  (uint64_t)p.q_stride_b * 2, kHalfRope, 128, CU_TENSOR_MAP_SWIZZLE_64B);
  if (!rc)
    rc = encode3d(&tm_qlat, dt, p.q, 576, (uint64_t)p.num_heads, (uint64_t)p.batch, (uint64_t)p.q_stride_h * 2,
                  (uint64_t)p.q_stride_b * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  KernelArgs a;
  a.p = p;
  a.rows_per_load = g;
  a.scale_log2 = p.softmax_scale * kLog2e;
  const dim3 grid(2 * ((p.num_heads + 127) / 128), p.num_splits, p.batch);
  cudaError_t e;
  if (p.dtype == TMLA_DTYPE_FP16) {
    e = cudaFuncSetAttribute(mla_sm100_split_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e == cudaSuccess)
      mla_sm100_split_kernel<__half><<<grid, kThreads, kSmemBytes, stream>>>(tm_lat, tm_rope, tm_qlat, tm_q, a);
  } else {
    e = cudaFuncSetAttribute(mla_sm100_split_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kSmemBytes);
    if (e == cudaSuccess)
      mla_sm100_split_kernel<__nv_bfloat16><<<grid, kThreads, kSmemBytes, stream>>>(tm_lat, tm_rope, tm_qlat, tm_q, a);
  }
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? 0 : -(int)e;
}

}  // namespace tmla
