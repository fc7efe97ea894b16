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
//   CTA r owns latent dims [256r, 256r+256) and RoPE dims [512+32r, 544+32r).
//   * QK: each CTA multiplies its 288-d half of Q (latent part resident in TMEM,
//     RoPE part in shared memory) by its 288-d half of every 64-token cache tile,
//     giving a partial S (128 heads x 64 tokens, fp32, TMEM).
//   * The partial S rows are swapped through distributed shared memory
//     (st.async with mbarrier completion); both CTAs add them (the same two
//     fp32 numbers, so both get identical S), run the same online softmax and
//     write the same P (16-bit, TMEM).
//   * PV: each CTA accumulates its 256 output columns, O_r += P . V_r, with V_r
//     the latent half of the very tile it already holds: the cache is read from
//     HBM once, and no MMA is duplicated.
//
// Warp roles (192 threads): warp 0 issues TMA loads of the cache tiles (block
// table -> page coordinates), warp 1 allocates TMEM and issues tcgen05.mma,
// warps 2-5 (one warpgroup; thread i owns TMEM lane / head i) load Q into
// TMEM, swap scores, run the softmax, rescale O lazily (only when a row
// maximum grows by more than 2^8) and write the result.
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
constexpr int kStages = 5;                // cache-tile ring depth
constexpr int kThreads = 192;
constexpr int kHalfLatent = 256;          // latent columns per CTA
constexpr int kHalfRope = 32;             // RoPE columns per CTA
constexpr uint32_t kBoxBytes = kTile * 128;                 // one 64-token x 64-dim swizzled box
constexpr uint32_t kRopeBytes = kTile * kHalfRope * 2;      // 64 tokens x 32 dims
constexpr uint32_t kStageBytes = 4 * kBoxBytes + kRopeBytes;  // 36864
constexpr uint32_t kRowBytes = (kHalfLatent + kHalfRope) * 2;  // cache bytes per token per CTA (576)
constexpr uint32_t kQRopeBytes = 128 * kHalfRope * 2;       // 8192
constexpr uint32_t kXBytes = 128 * kTile * 4;               // 32768: partial-S exchange buffer

constexpr uint32_t kOffStages = 0;
constexpr uint32_t kOffQRope = kOffStages + kStages * kStageBytes;
constexpr uint32_t kOffX = kOffQRope + kQRopeBytes;
constexpr uint32_t kOffBar = kOffX + kXBytes;
constexpr uint32_t kNumBars = 2 * kStages + 10;
constexpr uint32_t kOffMisc = kOffBar + kNumBars * 8;
constexpr uint32_t kSmemBytes = kOffMisc + 64 + 1024;  // + alignment slack

// TMEM columns (512 allocated): O half, Q latent half (bf16 pairs), S, P x2.
constexpr uint32_t kColO = 0;
constexpr uint32_t kColQ = 256;
constexpr uint32_t kColS = 384;
constexpr uint32_t kColP0 = 448;
constexpr uint32_t kColP1 = 480;

constexpr uint64_t kWaitNs = 2000000000ull;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: P stays <= 2^8 between rescales

// Barrier indices.
enum : uint32_t {
  kBarKvFull = 0,
  kBarKvEmpty = kStages,
  kBarQFull = 2 * kStages,
  kBarSFull,
  kBarSEmpty,
  kBarPFull0,
  kBarPFull1,
  kBarPvDone0,
  kBarPvDone1,
  kBarXFull,
  kBarXEmpty,
  kBarDrain,
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

template <typename T>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    mla_sm100_split_kernel(const __grid_constant__ CUtensorMap tm_kv_lat, const __grid_constant__ CUtensorMap tm_kv_rope,
                           const __grid_constant__ CUtensorMap tm_q_rope, const __grid_constant__ KernelArgs args) {
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
    mbar_init(sh.bar(kBarSFull), 1);
    mbar_init(sh.bar(kBarSEmpty), 4);
    mbar_init(sh.bar(kBarPFull0), 4);
    mbar_init(sh.bar(kBarPFull1), 4);
    mbar_init(sh.bar(kBarPvDone0), 1);
    mbar_init(sh.bar(kBarPvDone1), 1);
    mbar_init(sh.bar(kBarXFull), 1);
    mbar_init(sh.bar(kBarXEmpty), 4);
    mbar_init(sh.bar(kBarDrain), 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot_addr, 512);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_kv_lat);
    prefetch_tmap(&tm_kv_rope);
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

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    const int g = args.rows_per_load;
    const int nsub = kTile / g;
    const uint64_t pol_stream = policy_evict_first();
    if (lane == 0) {
      mbar_arrive_expect_tx(sh.bar(kBarQFull), kQRopeBytes);
      tma_load_3d(sh.base + kOffQRope, &tm_q_rope, sh.bar(kBarQFull), 512 + kHalfRope * rank, h0, b,
                  policy_evict_last());
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
    // Drain: every issued load (the last ring stages and Q's RoPE half) has landed before the CTA may exit.
    if (lane == 0) {
      for (int j = max(0, issued - kStages); j <= issued; ++j) {
        const uint32_t bar = j < issued ? sh.bar(kBarKvFull + j % kStages) : sh.bar(kBarQFull);
        const uint32_t parity = j < issued ? (j / kStages) & 1 : 0;
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(bar, parity) && globaltimer() - t0 < kWaitNs) {
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t fmt = kFp16 ? 0u : 1u;
      const uint32_t idesc_qk = idesc_f16(fmt, 128, kTile, 0);
      const uint32_t idesc_pv = idesc_f16(fmt, 128, kHalfLatent, 1);
      const uint32_t q_rope = sh.base + kOffQRope;
      bool ok = ntiles == 0 || waiter.wait(sh.bar(kBarQFull), 0);
      if (ok) tc_fence_after();
      auto issue_pv = [&](int i) -> bool {
        const int pb = i & 1;
        if (!waiter.wait(sh.bar(kBarPFull0 + pb), (i >> 1) & 1)) return false;
        tc_fence_after();
        const uint32_t st = sh.stage(i % kStages);
        const uint32_t pcol = pb ? kColP1 : kColP0;
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk) {
          // B = V: 16 tokens x 256 latent dims, MN-major 128B-swizzled, 64-dim boxes 8 KB apart.
          const uint64_t bdesc = smem_desc(st + kk * 16 * 128, kBoxBytes, 1024, kSwizzle128B);
          mma_ts(tmem + kColO, tmem + pcol + kk * 8, bdesc, idesc_pv, (i > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(sh.bar(kBarKvEmpty + i % kStages));
        mma_commit(sh.bar(kBarPvDone0 + pb));
        return true;
      };
      for (int j = 0; ok && j < ntiles; ++j) {
        const int s = j % kStages;
        if (!waiter.wait(sh.bar(kBarKvFull + s), (j / kStages) & 1)) break;
        if (j >= 1 && !waiter.wait(sh.bar(kBarSEmpty), (j - 1) & 1)) break;
        tc_fence_after();
        const uint32_t st = sh.stage(s);
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          const uint64_t bdesc = smem_desc(st + (k >> 2) * kBoxBytes + (k & 3) * 32, 16, 1024, kSwizzle128B);
          mma_ts(tmem + kColS, tmem + kColQ + k * 8, bdesc, idesc_qk, k > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const uint64_t adesc = smem_desc(q_rope + k * 32, 16, 512, kSwizzle64B);
          const uint64_t bdesc = smem_desc(st + 4 * kBoxBytes + k * 32, 16, 512, kSwizzle64B);
          mma_ss(tmem + kColS, adesc, bdesc, idesc_qk, 1u);
        }
        mma_commit(sh.bar(kBarSFull));
        if (j >= 1 && !issue_pv(j - 1)) {
          ok = false;
          break;
        }
        if (j == ntiles - 1 && !issue_pv(j)) ok = false;
      }
      // Drain: every issued MMA has completed before TMEM is read or freed.
      mma_commit(sh.bar(kBarDrain));
      uint64_t t0 = globaltimer();
      while (!mbar_try_wait(sh.bar(kBarDrain), 0) && globaltimer() - t0 < kWaitNs) {
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax warpgroup
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int h = h0 + row;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t t_row = tmem + lane_off;

    // Q latent half -> TMEM (bf16 pairs; rows past H are zero).
    {
      const T* qrow = static_cast<const T*>(p.q) + (int64_t)b * p.q_stride_b + (int64_t)h * p.q_stride_h +
                      kHalfLatent * rank;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
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

    const uint32_t x_local = sh.base + kOffX;
    const uint32_t x_remote = map_to_rank(x_local, peer);
    const uint32_t xfull_remote = map_to_rank(sh.bar(kBarXFull), peer);
    const uint32_t xempty_remote = map_to_rank(sh.bar(kBarXEmpty), peer);
    const float4* xbuf = reinterpret_cast<const float4*>(smem_gen + kOffX);

    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    int j = 0;
    for (; j < ntiles; ++j) {
      if (!waiter.wait(sh.bar(kBarSFull), j & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[64];
      {
        uint32_t r0[32], r1[32];
        tmem_ld32(t_row + kColS, r0);
        tmem_ld32(t_row + kColS + 32, r1);
        tc_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          s[i] = __uint_as_float(r0[i]);
          s[32 + i] = __uint_as_float(r1[i]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(sh.bar(kBarSEmpty));

      // Swap partial scores with the peer CTA.
      if (j >= 1 && !waiter.wait(sh.bar(kBarXEmpty), (j - 1) & 1, true)) {
        ok = false;
        break;
      }
      if (warp == 2 && lane == 0) mbar_arrive_expect_tx(sh.bar(kBarXFull), kXBytes);
#pragma unroll
      for (int c = 0; c < 16; ++c)
        st_async_v4(x_remote + (uint32_t)(c * 128 + row) * 16u,
                    make_float4(s[4 * c], s[4 * c + 1], s[4 * c + 2], s[4 * c + 3]), xfull_remote);
      if (!waiter.wait(sh.bar(kBarXFull), j & 1, true)) {
        ok = false;
        break;
      }
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const float4 v = xbuf[c * 128 + row];
        s[4 * c] += v.x;
        s[4 * c + 1] += v.y;
        s[4 * c + 2] += v.z;
        s[4 * c + 3] += v.w;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(xempty_remote);

      // Online softmax (base 2) with lazy rescaling of O.
      const int t0 = start + j * kTile;
      const int nvalid = min(kTile, end - t0);
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        s[i] = (i < nvalid) ? s[i] * args.scale_log2 : -INFINITY;
        mx = fmaxf(mx, s[i]);
      }
      float alpha = 1.f;
      const bool need = mx > m_used + kRescaleThreshold;
      if (need) {
        alpha = exp2f(m_used - mx);  // 0 on the first tile (m_used = -inf)
        m_used = mx;
      }
      if (j > 0 && __any_sync(0xffffffffu, need)) {
        const int pj = j - 1;
        if (!waiter.wait(sh.bar(kBarPvDone0 + (pj & 1)), (pj >> 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < 8; ++c) {
          uint32_t o[32];
          tmem_ld32(t_row + kColO + 32 * c, o);
          tc_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(t_row + kColO + 32 * c, o);
        }
        tc_wait_st();
      }
      l *= alpha;
      uint32_t pk[32];
      float sum = 0.f;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float a = exp2f(s[2 * i] - m_used), c2 = exp2f(s[2 * i + 1] - m_used);
        sum += a + c2;
        pk[i] = pack2(a, c2, kFp16);
      }
      l += sum;
      // P buffer (j & 1) was last read by PV(j - 2).
      if (j >= 2 && !waiter.wait(sh.bar(kBarPvDone0 + (j & 1)), ((j - 2) >> 1) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      tmem_st32(t_row + ((j & 1) ? kColP1 : kColP0), pk);
      tc_wait_st();
      if (nvalid < kTile) {
        // Tokens past the end may hold anything (even NaN); P is 0 there but 0 * NaN is NaN,
        // so their V rows are zeroed before PV reads the stage.
        unsigned char* st = smem_gen + kOffStages + (j % kStages) * kStageBytes;
        const int nrows = kTile - nvalid;
        for (int i = row; i < nrows * 4 * 8; i += 128) {
          const int r = nvalid + i / 32, box = (i / 8) & 3, chunk = i & 7;
          *reinterpret_cast<uint4*>(st + box * kBoxBytes + r * 128 + chunk * 16) = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async_smem();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(sh.bar((j & 1) ? kBarPFull1 : kBarPFull0));
    }

    // Epilogue.
    if (ok && ntiles > 0) {
      const int lj = ntiles - 1;
      ok = waiter.wait(sh.bar(kBarPvDone0 + (lj & 1)), (lj >> 1) & 1);
      tc_fence_after();
    }
    const bool final_out = (p.num_splits == 1) && !(p.flags & TMLA_FLAG_PARTIAL_ONLY);
    const float inv = l > 0.f ? 1.f / l : 0.f;
    const float lse2 = l > 0.f ? m_used + log2f(l) : -INFINITY;
    const bool have_o = ok && ntiles > 0;
#pragma unroll 1
    for (int c = 0; c < 8; ++c) {
      uint32_t o[32];
      if (have_o) {
        tmem_ld32(t_row + kColO + 32 * c, o);
        tc_wait_ld();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = 0u;
      }
      if (h < H) {
        const int col = kHalfLatent * rank + 32 * c;
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
    if (h < H && rank == 0) {
      if (final_out) {
        if (p.lse) p.lse[(int64_t)b * p.lse_stride_b + h] = l > 0.f ? lse2 * kLn2 : -INFINITY;
      } else {
        p.ws_lse[((int64_t)b * H + h) * p.num_splits + split] = lse2;
      }
    }
  }

  // Teardown: both CTAs are done with each other's shared memory before either exits.
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) {
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
  CUtensorMap tm_lat, tm_rope, tm_q;
  int rc = encode3d(&tm_lat, dt, p.kv, 576, (uint64_t)p.page_size, pages, (uint64_t)p.kv_stride_tok * 2,
                    (uint64_t)p.kv_stride_page * 2, 64, (uint32_t)g, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc)
    rc = encode3d(&tm_rope, dt, p.kv, 576, (uint64_t)p.page_size, pages, (uint64_t)p.kv_stride_tok * 2,
                  (uint64_t)p.kv_stride_page * 2, kHalfRope, (uint32_t)g, CU_TENSOR_MAP_SWIZZLE_64B);
  if (!rc)
    rc = encode3d(&tm_q, dt, p.q, 576, (uint64_t)p.num_heads, (uint64_t)p.batch, (uint64_t)p.q_stride_h * 2,
                  (uint64_t)p.q_stride_b * 2, kHalfRope, 128, CU_TENSOR_MAP_SWIZZLE_64B);
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
      mla_sm100_split_kernel<__half><<<grid, kThreads, kSmemBytes, stream>>>(tm_lat, tm_rope, tm_q, a);
  } else {
    e = cudaFuncSetAttribute(mla_sm100_split_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kSmemBytes);
    if (e == cudaSuccess)
      mla_sm100_split_kernel<__nv_bfloat16><<<grid, kThreads, kSmemBytes, stream>>>(tm_lat, tm_rope, tm_q, a);
  }
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? 0 : -(int)e;
}

}  // namespace tmla
