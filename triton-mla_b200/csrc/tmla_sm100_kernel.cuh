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
//   of Q and of every 64-token cache tile, and accumulates O[:, 256r:256r+256]
//   for all 128 heads in TMEM.
//   * QK: each CTA computes a partial S = Q_r . K_r^T (128 heads x 64 tokens,
//     fp32) into one of two TMEM score buffers.
//   * Softmax rows are split too.  Within each 32-lane TMEM quarter q the
//     sixteen lanes 32q + 16r + [0,16) are the heads CTA r owns.  Each CTA
//     sends the partial score rows of the heads it does not own to the peer
//     (16 KB per tile over distributed shared memory, double-buffered); the
//     owner adds them to its own partial and runs the online softmax.
//   * P lives in shared memory, in the 128B-swizzled K-major layout the PV MMA
//     reads as its A operand: the owner writes its 16 rows per quarter into its
//     own P buffer and copies the same 2 KB (contiguous) into the peer's buffer
//     with one bulk copy, together with the rows' rescale factors.
//   * PV: each CTA accumulates O_r += P . V_r with V_r the latent part of the
//     tile it already holds: the cache is read from HBM once and no MMA is
//     duplicated.  Both CTAs' PV commits are counted on a barrier in each CTA,
//     so a P buffer is rewritten only after both CTAs have read it.
// Cache tiles flow through two rings: the latent part (V as well as K) is held
// until PV (4 stages), the RoPE part only until QK (4 slots).  Score and P
// buffers are double-buffered and QK and PV are issued by different warps, so
// QK of tile j+1 and the score swap of tile j+1 run while tile j is in the
// softmax.
//
// TMEM (512 columns): O half 256 | Q latent half 128 | S0 64 | S1 64.  The Q
// RoPE half sits in shared memory (A operand of the last two K steps).
//
// Warp roles (512 threads).  warp 0: TMA producer (block table -> page
// coordinates); warp 1: TMEM allocation and QK issue; warp 2: PV issue;
// warp 3: forwards "score buffer read" signals to the peer.
// Warps 4-15 work on TMEM lane quarter w % 4 (the only lanes a warp can reach),
// one warp of each role per quarter:
//   warps 4-7    softmax warpgroup A: tiles 0, 2, 4, ...
//   warps 8-11   softmax warpgroup B: tiles 1, 3, 5, ...
//   warps 12-15  score senders: ship the peer-owned partial rows to the owner
// A softmax warpgroup takes its 16 owned rows per quarter (4 threads per row,
// 16-lane TMEM access shapes), writes P to both CTAs' P buffers, rescales O for
// those rows, then waits for the peer's P rows of the same tile and rescales O
// for them when the peer asks.  The running maximum of tile j-1 reaches the
// warpgroup of tile j through shared memory (one barrier per quarter); each
// warpgroup keeps partial row sums relative to the maximum of its own last tile
// and the two are combined at the end.  O is rescaled lazily: only when a row
// maximum grows by more than 2^8.
//
// Prologue: the producer's barriers are initialised by its own lane 0, so the
// first tile (page ids read speculatively at entry) and Q's RoPE half are
// requested before the CTA-wide and cluster-wide syncs.  Epilogue: warpgroups A
// and B stage O (scaled by 1/l) into 128B-swizzled tiles in the idle cache ring
// and one thread writes them with TMA tensor stores (split partials in fp32 or 16-bit,
// or the final 16-bit output; rows past H lie outside the tensor map and are skipped).
//
// Every wait is bounded (2 s per wait, %globaltimer); on expiry the CTA sets
// TMLA_STATUS_TIMEOUT, all roles leave their loops, in-flight copies and MMAs
// are drained (again bounded), TMEM is freed and the kernel returns.
//
// This body is compiled twice (tmla_sm100.cu): into namespace sm100 for caches of 16-bit
// rows and, with TMLA_SM100_FP8 = 1, into namespace sm100_fp8 for FP8 rows; the layout
// constants below differ between the two.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp8.h>

#include <cstring>

#include "tmla_common.cuh"
#include "tmla_ptx.cuh"

#ifndef TMLA_SM100_NS
#error "define TMLA_SM100_NS and TMLA_SM100_FP8 before including this file"
#endif

namespace tmla {

#ifndef TMLA_SM100_ARGS_DEFINED
#define TMLA_SM100_ARGS_DEFINED
// Launch arguments of both variants.
struct Sm100Args {
  TmlaDecodeParams p;
  int rows_per_load;   // g: token rows per TMA box (64 for dense / page % 64 == 0)
  float scale_log2;    // softmax_scale * log2(e)
  // Per-request split plan (tmla_decode_units) or NULL: entry z = {request, split,
  // splits of that request, partial slot (-1: the request has one split)}.
  const int4* units;
  uint64_t wait_ns;    // limit of each wait
  int stall;           // test only: the first cluster's rank-0 CTA never loads its first tile
};
#endif

namespace TMLA_SM100_NS {


using namespace ptx;

// FP8 rows: the producer's TMA loads land in their own slots (e4m3 latent values, scales,
// RoPE) and a fifth warpgroup dequantises each tile into the ring as fp16, the type of every
// latent product (Q's latent half is converted once, P is written as fp16).  A ring stage
// is then held from its dequantisation, not from its TMA issue, to the end of PV (the landing
// slots absorb the TMA latency), and shared memory pays for the landing slots with one ring
// stage; the RoPE slots are held across the dequantisation too.
constexpr bool kFp8 = TMLA_SM100_FP8 != 0;
constexpr int kTile = 64;                 // tokens per pipeline stage
constexpr int kStages = kFp8 ? 3 : 4;     // latent cache-tile ring depth (held until PV)
constexpr int kRopeSlots = kFp8 ? 3 : 4;  // RoPE cache-tile ring depth (held until QK)
constexpr int kLandSlots = 2;             // FP8 landing slots (FP8 rows only)
constexpr int kSinBufs = 2;              // score-exchange buffers (1 or 2)
constexpr int kPBufs = 2;                // P buffers, the A operand of PV (1 or 2)
static_assert(kSinBufs == 1 || kSinBufs == 2, "score-exchange buffers");
static_assert(kPBufs == 1 || kPBufs == 2, "P buffers");
constexpr int kThreads = kFp8 ? 640 : 512;  // FP8: + warps 16-19, the dequantising warpgroup
constexpr int kHalfLatent = 256;          // latent columns per CTA
constexpr int kHalfRope = 32;             // RoPE columns per CTA
constexpr uint32_t kBoxBytes = kTile * 128;                 // one 64-token x 64-dim swizzled box
constexpr uint32_t kRopeBytes = kTile * kHalfRope * 2;      // 64 tokens x 32 dims
constexpr uint32_t kStageBytes = 4 * kBoxBytes;               // 32768: latent boxes of one tile
constexpr uint32_t kRowBytes = (kHalfLatent + kHalfRope) * 2;  // cache bytes per token per CTA (576)
constexpr uint32_t kQBoxBytes = 128 * 128;                  // 128 heads x 64 dims, swizzled
constexpr uint32_t kQRopeBytes = 128 * kHalfRope * 2;       // 8192
constexpr uint32_t kQLatBytes = 4 * kQBoxBytes;             // this CTA's 256 latent dims of 128 heads
constexpr int kQStage = kStages - 2;  // Q's latent half lands in the last two ring stages
constexpr uint32_t kSinBytes = 64 * kTile * 4;              // 16384: peer's partial S for my 64 heads
constexpr uint32_t kPBufBytes = 128 * kTile * 2;            // 16384: P of all 128 rows, SW128 K-major
constexpr uint32_t kPPeerBytes = 64 * kTile * 2;            // 8192: the rows of P that come from the peer
constexpr uint32_t kAlphaBytes = 64 * 4;                    // rescale factors that come with P
constexpr uint32_t kFinBytes = 64 * 8;                      // final (l, m) of the peer's heads
constexpr uint32_t kStatBytes = 128 * 8;  // final (l, m) of all 128 rows for the epilogue
// An FP8 landing slot: this CTA's 256 e4m3 latent values of 64 tokens as two 128B-swizzled
// boxes of 128 values (8 KB each; token r, 16-byte chunk c at r * 128 + (c ^ (r & 7)) * 16),
// then the tokens' 16-byte scale quadruples.
constexpr uint32_t kLandLatBytes = kTile * kHalfLatent;
constexpr uint32_t kLandBoxBytes = kTile * 128;
constexpr uint32_t kLandBytes = kLandLatBytes + kTile * 16;
constexpr uint32_t kFp8Row = 656;         // bytes per token of an FP8 row
constexpr int kFp8RopeElem = 264;         // its RoPE half starts at byte 528: bf16 element 264

constexpr uint32_t kOffStages = 0;
constexpr uint32_t kOffRope = kOffStages + kStages * kStageBytes;
constexpr uint32_t kOffPBuf = kOffRope + kRopeSlots * kRopeBytes;  // P buffers: A operand of PV (1024-aligned)
constexpr uint32_t kOffLand = kOffPBuf + kPBufs * kPBufBytes;     // FP8 landing slots (1024-aligned)
constexpr uint32_t kOffQRope = kOffLand + (kFp8 ? kLandSlots * kLandBytes : 0);
constexpr uint32_t kOffSin = kOffQRope + kQRopeBytes;
constexpr uint32_t kOffAlpha = kOffSin + kSinBufs * kSinBytes;  // alpha is double-buffered
constexpr uint32_t kOffMx = kOffAlpha + 2 * kAlphaBytes;      // running maxima handed between the warpgroups
constexpr uint32_t kOffWst = kOffMx + 2 * 64 * 4;              // each warpgroup's final (l, m) of the owned rows
constexpr uint32_t kOffBar = kOffWst + 2 * 64 * 8;
// The epilogue's row statistics and the peer's final (l, m) reuse the RoPE ring:
// both are written only after the last QK of the CTA has completed.
constexpr uint32_t kOffFin = kOffRope;
constexpr uint32_t kOffStat = kOffRope + kFinBytes;
static_assert(kFinBytes + kStatBytes <= kRopeSlots * kRopeBytes, "epilogue scratch must fit in the RoPE ring");
static_assert(kOffPBuf % 1024 == 0 && kOffSin % 1024 == 0,
              "P buffers and epilogue tiles must be 1024-byte aligned for the 128-byte swizzle");
// Epilogue tiles (8 of 16 KB for fp32 partials, 4 for 16-bit ones) reuse the cache-tile
// ring and, past its end, the score-exchange buffers.
static_assert(kStages * kStageBytes + kSinBufs * kSinBytes >= 8 * 128 * 128, "no room for the epilogue tiles");
constexpr uint32_t kNumBars = 2 * kStages + kRopeSlots + 40;
constexpr uint32_t kOffMisc = kOffBar + ((kNumBars * 8 + 63) / 64) * 64;
constexpr uint32_t kSmemBytes = kOffMisc + 64 + 1024;  // + alignment slack
static_assert(kSmemBytes <= 232448, "shared memory layout exceeds the 227 KB per-CTA limit");
static_assert(16 + 4 * kStages + 8 + 4 * kLandSlots <= 64,
              "the misc area holds the abort flag, the TMEM address and the masks");

constexpr uint32_t kColO = 0;
constexpr uint32_t kColQ = 256;   // Q latent dims [0, 256) of the half: 128 columns
constexpr uint32_t kColS = 384;   // + 64 * buffer

constexpr int kWarpProducer = 0;
constexpr int kWarpQK = 1;
constexpr int kWarpPV = 2;
constexpr int kWarpRelay = 3;

constexpr uint64_t kWaitNs = 2000000000ull;   // default limit of each wait
constexpr uint64_t kInFlightNs = 100000ull;   // how long a pair that gave up keeps its shared memory
constexpr float kRescaleThreshold = 8.0f;  // log2 units: P stays <= 2^8 between rescales

// Barrier indices.
enum : uint32_t {
  kBarKvFull = 0,
  kBarKvEmpty = kStages,
  kBarRopeEmpty = 2 * kStages,      // QK of the tile in this RoPE slot has completed
  kBarQFull = 2 * kStages + kRopeSlots,
  kBarSFull0,
  kBarSFull1,
  kBarSEmpty0,
  kBarSEmpty1,
  kBarPFull0,
  kBarPFull1,
  kBarPvDone0,
  kBarPvDone1,
  kBarSinFull0,    // peer's partial score rows landed in my Sin buffer 0 / 1
  kBarSinFull1,
  kBarSoutEmpty0,  // peer has consumed what my score senders sent into its Sin buffer 0 / 1
  kBarSoutEmpty1,
  kBarPinFull0,    // the peer's P rows (+ rescale factors) landed in my P buffer 0 / 1
  kBarPinFull1,
  kBarPairPvDone0, // PV of the tile in P buffer 0 / 1 has completed in both CTAs (count 2)
  kBarPairPvDone1,
  kBarFinFull,     // owner's final (l, m) of the peer's heads landed
  kBarDrainQK,
  kBarDrainPV,
  kBarStats,       // every row's final (l, m) is in shared memory for the epilogue
  kBarSinRead0,    // my softmax warps have read Sin buffer 0 / 1 (forwarded to the peer's SoutEmpty)
  kBarSinRead1,
  kBarMaxA0,       // softmax warpgroup A (even tiles) published its running maximum, per quarter
  kBarMaxB0 = kBarMaxA0 + 4,  // warpgroup B (odd tiles), per quarter
  kBarWgStats = kBarMaxB0 + 4,  // both warpgroups' final (l, m) are in shared memory
  kBarEpi,         // the epilogue tiles are staged (8 warps)
  kBarQCopied,     // Q's latent half has been copied from its two ring stages into TMEM
  kBarQConv,       // FP8 rows: Q's latent half is fp16 in its ring stages (4 dequantising warps)
  kBarLandFull0,   // FP8 rows: the loads of landing slot 0 / 1 have landed
  kBarLandEmpty0 = kBarLandFull0 + kLandSlots,  // FP8 rows: landing slot 0 / 1 was dequantised (4 warps)
  kBarCount = kBarLandEmpty0 + kLandSlots,
};

static_assert(kBarCount <= kNumBars, "barrier area too small");

struct Shared {
  uint32_t base;  // 1024-aligned shared address of the layout above
  __device__ uint32_t bar(uint32_t i) const { return base + kOffBar + 8 * i; }
  __device__ uint32_t stage(uint32_t s) const { return base + kOffStages + s * kStageBytes; }
  __device__ uint32_t rope(uint32_t r) const { return base + kOffRope + r * kRopeBytes; }
  __device__ uint32_t land(uint32_t l) const { return base + kOffLand + l * kLandBytes; }
};

// A wait that gives up after `limit` ns or as soon as another role of this CTA or of the
// peer gave up; on giving up it raises the abort flag of both CTAs of the pair.
struct Waiter {
  volatile int* abort_flag;
  int* status;
  uint64_t limit;
  uint32_t peer_abort;  // the peer's abort flag (shared::cluster address)
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
        } else if (now - t0 > limit) {
          *abort_flag = 1;
          asm volatile("st.relaxed.cluster.shared::cluster.u32 [%0], %1;" ::"r"(peer_abort), "r"(1) : "memory");
          if (status) atomicOr(status, TMLA_STATUS_TIMEOUT);
          return false;
        }
      }
    }
  }
};

// Bounded wait for drains on the way out (no abort shortcut).
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity, uint64_t limit) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity) && globaltimer() - t0 < limit) {
  }
}

using KernelArgs = ::tmla::Sm100Args;

__device__ __forceinline__ uint32_t pack2(float a, float b, bool fp16) {
  if (fp16) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// FP8 rows: sixteen e4m3 values (one 16-byte word, value i in byte i) times `scale` as
// sixteen fp16 values in two 16-byte words (values 0-7, 8-15).  e4m3 -> fp16 is exact (one
// conversion per pair); the product is formed in fp32 and rounded to fp16 once.  (Forming it
// with fp16 FMAs and a scale split into two fp16 parts needs a third of the conversions but
// measured 6% slower on the whole kernel.)
__device__ __forceinline__ void dequant16(uint4 v, float scale, uint4& lo, uint4& hi) {
  const uint32_t in[4] = {v.x, v.y, v.z, v.w};
  uint32_t out[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const __half2 x = __half2(__nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(in[i] >> (16 * h)), __NV_E4M3));
      const float2 f = __half22float2(x);
      out[2 * i + h] = pack2(f.x * scale, f.y * scale, true);
    }
  }
  lo = make_uint4(out[0], out[1], out[2], out[3]);
  hi = make_uint4(out[4], out[5], out[6], out[7]);
}

// Eight bf16 values -> fp16 (in place); sets `range` when one is too large for fp16.
__device__ __forceinline__ void bf16x8_to_fp16(uint4& v, bool& range) {
  uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&w[i]);
    const float2 f = __bfloat1622float2(b);
    range |= fabsf(f.x) >= 65520.f || fabsf(f.y) >= 65520.f;
    w[i] = pack2(f.x, f.y, true);
  }
  v = make_uint4(w[0], w[1], w[2], w[3]);
}

// `a` plus a term that is always 0 but is computed from `v` (min(~v, v) < 2^31)
// by instructions the compiler cannot fold away.  A shared-memory operation at
// the returned address cannot issue before the loads that produced `v` have
// returned their data: the register scoreboard holds it until then.
__device__ __forceinline__ uint32_t after_loads(uint32_t a, uint32_t v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .b32 n;\n\tnot.b32 n, %1;\n\tmin.u32 n, n, %1;\n\tshr.u32 n, n, 31;\n\tadd.u32 %0, %2, n;\n\t}"
      : "=r"(r)
      : "r"(v), "r"(a));
  return r;
}

// O[r, :] *= alpha_r for the 16 TMEM lanes at `lanes` (256 fp32 columns, in place):
// thread t scales lane t/4 by alpha_a and lane t/4 + 8 by alpha_b.
__device__ __forceinline__ void rescale_rows16(uint32_t lanes, float alpha_a, float alpha_b) {
#pragma unroll 1
  for (int c = 0; c < 4; ++c) {
    uint32_t o[32];
    tmem_ld16x256_x8(lanes + kColO + 64 * c, o);
    tc_wait_ld();
#pragma unroll
    for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * ((i & 2) ? alpha_b : alpha_a));
    tmem_st16x256_x8(lanes + kColO + 64 * c, o);
  }
  tc_wait_st();
}

// Masked tokens (past the end of the split, or in a sub-box whose page id was outside
// the pool and was not loaded) may hold anything in shared memory, even NaN; P is 0 there
// but 0 * NaN is NaN, so their V rows are zeroed before PV reads the stage.  Row r is
// masked when r >= nvalid or bit r >> g_log2 of `bad` is set.  Called by the 128 softmax
// threads (thread index t in [0, 128)).
__device__ __forceinline__ void zero_masked_rows(unsigned char* stage, int nvalid, uint32_t bad, int g_log2, int t) {
  for (int i = t; i < kTile * 4 * 8; i += 128) {
    const int r = i / 32, box = (i / 8) & 3, chunk = i & 7;
    if (r >= nvalid || ((bad >> (r >> g_log2)) & 1u))
      *reinterpret_cast<uint4*>(stage + box * kBoxBytes + r * 128 + chunk * 16) = make_uint4(0, 0, 0, 0);
  }
  fence_proxy_async_smem();
}

// Epilogue tiles: 128 rows x 128 bytes, 128B-swizzled (16-byte chunk k of row r at
// (k ^ (r & 7)) * 16), one per TMA store box: 32 fp32 columns of the split partial, or
// 64 16-bit columns of the final output.  They reuse the cache-tile ring, which is idle
// once the last PV has completed.
constexpr uint32_t kOutBoxBytes = 128 * 128;
// Shared-memory offset of epilogue tile c: the cache-tile ring (idle once the last PV has
// completed), then the score-exchange buffers (read for the last time before the last P).
__host__ __device__ constexpr uint32_t out_box_off(int c) {
  return c < 2 * kStages ? kOffStages + (uint32_t)c * kOutBoxBytes
                         : kOffSin + (uint32_t)(c - 2 * kStages) * kOutBoxBytes;
}

// Stage columns [32 c0, 32 (c0 + nchunks)) of this CTA's output half of row r (scaled by
// inv; zeros when there is no output) into the epilogue tiles (`tiles`: the layout's base).
template <typename T>
__device__ __forceinline__ void stage_rows(unsigned char* tiles, uint32_t t_row, bool have_o, int r, float inv,
                                           int c0, int nchunks, bool final_out) {
  constexpr bool kFp16 = std::is_same<T, __half>::value;
#pragma unroll 1
  for (int c = c0; c < c0 + nchunks; ++c) {
    uint32_t o[32];
    if (have_o) {
      tmem_ld32(t_row + kColO + 32 * c, o);
      tc_wait_ld();
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) o[i] = 0u;
    }
    if (final_out) {
      unsigned char* row = tiles + out_box_off(c >> 1) + r * 128;
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        uint4 w;
        w.x = pack2(__uint_as_float(o[8 * v + 0]) * inv, __uint_as_float(o[8 * v + 1]) * inv, kFp16);
        w.y = pack2(__uint_as_float(o[8 * v + 2]) * inv, __uint_as_float(o[8 * v + 3]) * inv, kFp16);
        w.z = pack2(__uint_as_float(o[8 * v + 4]) * inv, __uint_as_float(o[8 * v + 5]) * inv, kFp16);
        w.w = pack2(__uint_as_float(o[8 * v + 6]) * inv, __uint_as_float(o[8 * v + 7]) * inv, kFp16);
        const int k = (c & 1) * 4 + v;
        *reinterpret_cast<uint4*>(row + ((k ^ (r & 7)) << 4)) = w;
      }
    } else {
      unsigned char* row = tiles + out_box_off(c) + r * 128;
#pragma unroll
      for (int v = 0; v < 8; ++v)
        *reinterpret_cast<float4*>(row + ((v ^ (r & 7)) << 4)) =
            make_float4(__uint_as_float(o[4 * v]) * inv, __uint_as_float(o[4 * v + 1]) * inv,
                        __uint_as_float(o[4 * v + 2]) * inv, __uint_as_float(o[4 * v + 3]) * inv);
    }
  }
}

// kPart16: split partials in the q dtype (tmla_decode's own merge reads them), else fp32.
template <typename T, bool kPart16>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    mla_sm100_split_kernel(const __grid_constant__ CUtensorMap tm_kv_lat, const __grid_constant__ CUtensorMap tm_kv_rope,
                           const __grid_constant__ CUtensorMap tm_kv_scale,
                           const __grid_constant__ CUtensorMap tm_out, const __grid_constant__ CUtensorMap tm_part,
                           const __grid_constant__ CUtensorMap tm_q_rope,
                           const __grid_constant__ CUtensorMap tm_q_lat,
                           const __grid_constant__ KernelArgs args) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const TmlaDecodeParams& p = args.p;
  constexpr bool kFp16 = std::is_same<T, __half>::value;
  // Type of the latent products (Q's latent half, K, V and P): the q dtype, or fp16 for FP8 rows.
  constexpr bool kLatFp16 = kFp16 || kFp8;

  Shared sh;
  sh.base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  unsigned char* smem_gen = smem_raw + (sh.base - smem_u32(smem_raw));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem_gen + kOffMisc);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem_gen + kOffMisc + 8);
  // Per ring stage: the sub-boxes of its tile whose page id was outside the pool; per score
  // buffer: the same mask for the tile whose scores it holds.
  volatile uint32_t* bad_mask = reinterpret_cast<volatile uint32_t*>(smem_gen + kOffMisc + 16);
  volatile uint32_t* tile_mask = reinterpret_cast<volatile uint32_t*>(smem_gen + kOffMisc + 16 + 4 * kStages);
  // FP8 rows: the masked sub-boxes of the tile in each landing slot.
  volatile uint32_t* land_mask = reinterpret_cast<volatile uint32_t*>(smem_gen + kOffMisc + 24 + 4 * kStages);
  const uint32_t tmem_slot_addr = sh.base + kOffMisc + 8;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const uint32_t peer = rank ^ 1u;
  const int head_tile = blockIdx.x >> 1;
  const int h0 = head_tile * 128;
  // Launched as a programmatic dependent: every global read (the plan, lengths, table, q,
  // cache) and write comes after the preceding kernel has completed.
  griddep_wait();
  // Which split of which request: the grid's (y, z) for uniform splits, or a plan entry.
  int split = blockIdx.y, b = blockIdx.z, nsplit = p.num_splits, slot = -1;
  if (args.units) {
    const int4 un = __ldg(args.units + blockIdx.z);
    // A padding entry of a fixed-capacity plan (tmla_plan_units_device): both CTAs of the
    // cluster read the same entry and leave before touching any barrier or the peer.
    if (un.x < 0) return;
    b = un.x, split = un.y, nsplit = un.z, slot = un.w;
  }
  // One split writes the final output (and natural-log LSE); several write partials.
  const bool final_out = args.units ? nsplit == 1 : (p.num_splits == 1 && !(p.flags & TMLA_FLAG_PARTIAL_ONLY));
  const int H = p.num_heads;
  const Waiter waiter{abort_flag, p.status, args.wait_ns, map_to_rank(sh.base + kOffMisc, peer)};
  // Test only (TMLA_FLAG_TEST_STALL): this CTA never loads tile 0, so the waits for it run out.
  const bool stalled = args.stall && rank == 0 && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0;

  // The request length, the block-table entries of the split and this CTA's Q rows are
  // requested before the set-up below, so that their latency overlaps it.
  const int len_req = __ldg(p.seqlens + b);
  const int cap = p.block_table ? p.bt_width * p.page_size : p.page_size;
  // Several query tokens per request: this head tile's token attends causally, to the
  // request's first len - (q_len - 1 - token) rows (a length out of range is flagged below).
  int len_in = len_req;
  if (p.q_len > 1 && len_req >= 0 && len_req <= cap)
    len_in = max(0, len_req - (p.q_len - 1 - h0 / (H / p.q_len)));
  const int g = args.rows_per_load;  // token rows per TMA box
  const int nsub = kTile / g;
  const int g_log2 = __ffs(g) - 1;
  // The producer reads the page ids of its first tile as if the request filled its table:
  // the first tile of a split then does not wait for the length and the table one after
  // the other (when the guess is wrong they are read again once the length is known).
  int spec_start = 0, pg_spec = 0;
  if (warp == kWarpProducer) {
    int spec_end;
    split_range(cap, nsplit, split, spec_start, spec_end);
    const int t = spec_start + lane * g;
    if (lane < nsub && t < spec_end) pg_spec = p.block_table ? __ldg(p.block_table + (int64_t)b * p.bt_stride + t / p.page_size) : b;
  }
  if (warp == kWarpProducer && p.block_table) {
    // 32 lines of the block-table row around where this split starts when the request
    // fills the table (a split of a shorter request starts earlier in the row).
    const int cap_tiles = (p.bt_width * p.page_size + kTile - 1) / kTile;
    const int per = (cap_tiles + p.num_splits - 1) / p.num_splits;
    const int64_t first = (int64_t)split * per * kTile / p.page_size;  // entry index
    const int64_t line = max((int64_t)0, first / 32 - 8) + lane;
    if (line * 32 < p.bt_width) prefetch_l2(p.block_table + (int64_t)b * p.bt_stride + line * 32);
  }
  if (threadIdx.x == 0) {
    *abort_flag = 0;
    *reinterpret_cast<volatile int*>(smem_gen + kOffMisc + 4) = 0;
    mbar_init(sh.bar(kBarQFull), 1);
    mbar_init(sh.bar(kBarQCopied), 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(sh.bar(kBarKvFull + s), kFp8 ? 4 : 1);  // TMA bytes, or the four dequantising warps
      mbar_init(sh.bar(kBarKvEmpty + s), 1);
    }
    if (kFp8) {
      mbar_init(sh.bar(kBarQConv), 4);
      for (int l = 0; l < kLandSlots; ++l) {
        mbar_init(sh.bar(kBarLandFull0 + l), 1);
        mbar_init(sh.bar(kBarLandEmpty0 + l), 4);
      }
    }
    for (int r = 0; r < kRopeSlots; ++r) mbar_init(sh.bar(kBarRopeEmpty + r), 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(sh.bar(kBarSFull0 + i), 2);  // the QK commit + the QK thread (tile mask published)
      mbar_init(sh.bar(kBarSEmpty0 + i), 8);
      mbar_init(sh.bar(kBarPFull0 + i), 4);
      mbar_init(sh.bar(kBarPvDone0 + i), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(sh.bar(kBarSinFull0 + i), 1);
      mbar_init(sh.bar(kBarSoutEmpty0 + i), 1);
      mbar_init(sh.bar(kBarSinRead0 + i), 4);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(sh.bar(kBarPinFull0 + i), 1);
      mbar_init(sh.bar(kBarPairPvDone0 + i), 2);
    }
    mbar_init(sh.bar(kBarFinFull), 1);
    mbar_init(sh.bar(kBarDrainQK), 1);
    mbar_init(sh.bar(kBarDrainPV), 1);
    mbar_init(sh.bar(kBarStats), 8);
    mbar_init(sh.bar(kBarWgStats), 8);
    mbar_init(sh.bar(kBarEpi), 8);
    for (int q = 0; q < 4; ++q) {
      mbar_init(sh.bar(kBarMaxA0 + q), 1);
      mbar_init(sh.bar(kBarMaxB0 + q), 1);
    }
    fence_mbar_init();
  }
  if (warp == kWarpQK) {
    tmem_alloc(tmem_slot_addr, 512);
    tmem_relinquish();
  }
  if (warp == kWarpProducer && lane == 0) {
    prefetch_tmap(&tm_kv_lat);
    prefetch_tmap(&tm_kv_rope);
    if (kFp8) prefetch_tmap(&tm_kv_scale);
    prefetch_tmap(&tm_q_rope);
    prefetch_tmap(&tm_q_lat);
  }

  // Token range of this split (whole 64-token tiles; see split_range).
  int len = len_in;
  if (len < 0 || len > cap) {
    if (p.status && threadIdx.x == 0) atomicOr(p.status, TMLA_STATUS_BAD_PAGE);
    len = len < 0 ? 0 : cap;
  }
  int start, end;
  split_range(len, nsplit, split, start, end);
  const int ntiles = end > start ? (end - start + kTile - 1) / kTile : 0;

  // ------------------------------------------------------------ TMA producer, part 1
  // The producer's barriers were initialised by its own lane 0 above, so Q's RoPE half
  // and the first cache tile are requested before the CTA-wide and cluster-wide syncs.
  const uint64_t pol_stream = policy_evict_first();
  // Raw page id of sub-box `sb` of tile `j` (0 when the sub-box is past the end of
  // the split); read ahead of use, checked against the pool when used.
  const int64_t npages = p.block_table ? p.num_pages : (int64_t)p.batch;
  auto page_of = [&](int j, int sb) -> int {
    const int t = start + j * kTile + sb * g;
    if (sb >= nsub || t >= end || j >= ntiles) return 0;
    if (!p.block_table) return b;
    return __ldg(p.block_table + (int64_t)b * p.bt_stride + t / p.page_size);
  };
  // Loads of tile j (ring stage j % kStages, RoPE slot j % kRopeSlots) once both are free.
  // Lane l loads sub-box l.  A page id outside the pool is reported and its sub-box is not
  // loaded: the stage's mask word records it, and the softmax masks those tokens (score
  // -inf, V rows zeroed), as the CUDA-core kernel does.
  auto issue_tile = [&](int j, int pg) {
    const int s = j % kStages, rs = j % kRopeSlots;
    const int t = start + j * kTile + lane * g;
    const bool live = lane < nsub && t < end;
    const bool bad = live && (pg < 0 || (int64_t)pg >= npages);
    const uint32_t loads = __ballot_sync(0xffffffffu, live && !bad);
    const uint32_t bads = __ballot_sync(0xffffffffu, bad);
    if (bads && lane == 0 && p.status) atomicOr(p.status, TMLA_STATUS_BAD_PAGE);
    if constexpr (kFp8) {
      // FP8 rows: the e4m3 latent values and the scales into landing slot j % kLandSlots, the
      // bf16 RoPE half into its slot; the dequantising warps take them from there.
      const int ls = j % kLandSlots;
      if (lane == 0) {
        land_mask[ls] = bads;
        mbar_arrive_expect_tx(sh.bar(kBarLandFull0 + ls),
                              (uint32_t)(__popc(loads) * g) * (uint32_t)(kHalfLatent + 16 + kHalfRope * 2));
      }
      __syncwarp();
      if (live && !bad) {
        const int slot = p.block_table ? t % p.page_size : t;
        const uint32_t dst = sh.land(ls), bar = sh.bar(kBarLandFull0 + ls);
#pragma unroll
        for (int hb = 0; hb < 2; ++hb)
          tma_load_3d(dst + hb * kLandBoxBytes + lane * g * 128, &tm_kv_lat, bar, kHalfLatent * rank + 128 * hb, slot,
                      pg, pol_stream);
        tma_load_3d(dst + kLandLatBytes + lane * g * 16, &tm_kv_scale, bar, 512, slot, pg, pol_stream);
        tma_load_3d(sh.rope(rs) + lane * g * (kHalfRope * 2), &tm_kv_rope, bar, kFp8RopeElem + kHalfRope * rank, slot,
                    pg, pol_stream);
      }
      return;
    }
    if (lane == 0) {
      bad_mask[s] = bads;
      mbar_arrive_expect_tx(sh.bar(kBarKvFull + s), (uint32_t)(__popc(loads) * g) * kRowBytes);
    }
    __syncwarp();
    if (live && !bad) {
      const int slot = p.block_table ? t % p.page_size : t;
      const uint32_t dst = sh.stage(s);
      const uint32_t bar = sh.bar(kBarKvFull + s);
#pragma unroll
      for (int kb = 0; kb < 4; ++kb)
        tma_load_3d(dst + kb * kBoxBytes + lane * g * 128, &tm_kv_lat, bar, kHalfLatent * rank + 64 * kb, slot, pg,
                    pol_stream);
      tma_load_3d(sh.rope(rs) + lane * g * (kHalfRope * 2), &tm_kv_rope, bar, 512 + kHalfRope * rank, slot, pg,
                  pol_stream);
    }
  };
  int pg_next = -1;
  if (warp == kWarpProducer) {
    __syncwarp();
    if (lane == 0) {
      // Q: the RoPE half into its own buffer, this CTA's 256 latent dims (four 64-dim boxes of
      // 128 heads) into the last two ring stages, which the QK warp copies into TMEM before its first MMA
      // (rows past H are zero-filled).
      mbar_arrive_expect_tx(sh.bar(kBarQFull), kQRopeBytes + kQLatBytes);
      tma_load_3d(sh.base + kOffQRope, &tm_q_rope, sh.bar(kBarQFull), 512 + kHalfRope * rank, h0, b,
                  policy_evict_last());
#pragma unroll
      for (int c = 0; c < 4; ++c)
        tma_load_3d(sh.stage(kQStage) + c * kQBoxBytes, &tm_q_lat, sh.bar(kBarQFull), kHalfLatent * rank + 64 * c, h0, b,
                    policy_evict_last());
    }
    if (ntiles > 0) {
      if (!stalled) issue_tile(0, start == spec_start ? pg_spec : page_of(0, lane));
      pg_next = page_of(1, lane);
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the peer's barriers are initialised before any remote arrive / st.async
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kWarpProducer) {
    // ------------------------------------------------------------ TMA producer, part 2
    int issued = ntiles > 0 ? 1 : 0;
    for (int j = 1; j < ntiles; ++j) {
      const int pg = pg_next;
      pg_next = page_of(j + 1, lane);
      const int s = j % kStages, rs = j % kRopeSlots;
      bool ok = true;
      if (kFp8) {
        // The landing slot was dequantised for tile j - kLandSlots (the ring is the
        // dequantising warps' concern).
        if (lane == 0 && j >= kLandSlots)
          ok = waiter.wait(sh.bar(kBarLandEmpty0 + j % kLandSlots), ((j / kLandSlots) - 1) & 1);
      } else {
        if (lane == 0 && j >= kStages) ok = waiter.wait(sh.bar(kBarKvEmpty + s), ((j / kStages) - 1) & 1);
        // Stages 2 and 3 first held Q's latent half, until the QK warp copied it into TMEM.
        if (lane == 0 && ok && j == kQStage) ok = waiter.wait(sh.bar(kBarQCopied), 0);
      }
      if (lane == 0 && ok && j >= kRopeSlots) ok = waiter.wait(sh.bar(kBarRopeEmpty + rs), ((j / kRopeSlots) - 1) & 1);
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) break;
      issue_tile(j, pg);
      issued = j + 1;
    }
    // Drain: every issued load (the last ring stages or landing slots, and Q) has landed
    // before the CTA may exit.
    if (lane == 0) {
      const int depth = kFp8 ? kLandSlots : kStages;
      for (int j = max(0, issued - depth); j <= issued; ++j) {
        if (j < issued) {
          if (!(stalled && j == 0))
            drain_wait(kFp8 ? sh.bar(kBarLandFull0 + j % kLandSlots) : sh.bar(kBarKvFull + j % kStages),
                       (j / depth) & 1, args.wait_ns);
        } else {
          drain_wait(sh.bar(kBarQFull), 0, args.wait_ns);
        }
      }
    }
  } else if (warp == kWarpQK) {
    // ------------------------------------------------------------ QK issuer: S[j&1] = Q_r . K_r(j)^T
    if (lane == 0) {
      // Latent steps in the latent product type; the RoPE steps in the q dtype (FP8 rows
      // hold bf16 RoPE values, converted to fp16 for fp16 queries before QK).
      const uint32_t idesc = idesc_f16(kLatFp16 ? 0u : 1u, 128, kTile, 0);
      const uint32_t idesc_rope = idesc_f16(kFp16 ? 0u : 1u, 128, kTile, 0);
      const uint32_t q_rope = sh.base + kOffQRope;
      bool ok = ntiles == 0 || waiter.wait(sh.bar(kBarQFull), 0);
      // FP8 rows: Q's latent half is converted to fp16 in place first.
      if (kFp8) ok = ok && (ntiles == 0 || waiter.wait(sh.bar(kBarQConv), 0));
      if (ok && ntiles > 0) {
        // Q's latent half: smem (its two ring stages, 128B-swizzled 64-dim boxes) -> TMEM columns
        // kColQ + 8k for the 16-dim step k, ahead of (and in order with) the first QK.
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 16; ++k)
          tmem_cp_128x256b(tmem + kColQ + 8 * k,
                           smem_desc(sh.stage(kQStage) + (k >> 2) * kQBoxBytes + (k & 3) * 32, 16, 1024, kSwizzle128B));
        mma_commit(sh.bar(kBarQCopied));
      }
      for (int j = 0; ok && j < ntiles; ++j) {
        const int s = j % kStages, sb = j & 1;
        if (!waiter.wait(sh.bar(kBarKvFull + s), (j / kStages) & 1)) break;
        // Score buffer sb was last read for tile j-2.
        if (j >= 2 && !waiter.wait(sh.bar(kBarSEmpty0 + sb), ((j - 2) >> 1) & 1)) break;
        tc_fence_after();
        const uint32_t st = sh.stage(s), rp = sh.rope(j % kRopeSlots);
        const uint32_t d = tmem + kColS + 64 * sb;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          const uint64_t bdesc = smem_desc(st + (k >> 2) * kBoxBytes + (k & 3) * 32, 16, 1024, kSwizzle128B);
          mma_ts(d, tmem + kColQ + k * 8, bdesc, idesc, k > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const uint64_t adesc = smem_desc(q_rope + k * 32, 16, 512, kSwizzle64B);
          const uint64_t bdesc = smem_desc(rp + k * 32, 16, 512, kSwizzle64B);
          mma_ss(d, adesc, bdesc, idesc_rope, 1u);
        }
        mma_commit(sh.bar(kBarSFull0 + sb));
        mma_commit(sh.bar(kBarRopeEmpty + j % kRopeSlots));
        // The tile's masked sub-boxes travel with its scores: the softmax reads them after
        // SFull, whose phase completes with this thread's arrival as well as the commit.
        tile_mask[sb] = bad_mask[s];
        mbar_arrive(sh.bar(kBarSFull0 + sb));
      }
      mma_commit(sh.bar(kBarDrainQK));
      drain_wait(sh.bar(kBarDrainQK), 0, args.wait_ns);
    }
    __syncwarp();
  } else if (warp == kWarpPV) {
    // ------------------------------------------------------------ PV issuer: O_r += P(j) . V_r(j)
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(kLatFp16 ? 0u : 1u, 128, kHalfLatent, 1);
      const uint32_t pairdone_remote = map_to_rank(sh.bar(kBarPairPvDone0), peer);  // + 8 * buffer
      for (int j = 0; j < ntiles; ++j) {
        const int pb = j & 1;
        if (!waiter.wait(sh.bar(kBarPFull0 + pb), (j >> 1) & 1)) break;
        tc_fence_after();
        const uint32_t st = sh.stage(j % kStages), pbuf = sh.base + kOffPBuf + (j % kPBufs) * kPBufBytes;
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk) {
          // A = P: 128 rows x 16 tokens, K-major 128B-swizzled (same layout as a Q box).
          // B = V: 16 tokens x 256 latent dims, MN-major 128B-swizzled, 64-dim boxes 8 KB apart.
          const uint64_t adesc = smem_desc(pbuf + kk * 32, 16, 1024, kSwizzle128B);
          const uint64_t bdesc = smem_desc(st + kk * 16 * 128, kBoxBytes, 1024, kSwizzle128B);
          mma_ss(tmem + kColO, adesc, bdesc, idesc, (j > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(sh.bar(kBarKvEmpty + j % kStages));
        mma_commit(sh.bar(kBarPvDone0 + pb));
        // Both CTAs count this PV on their pair barrier: P buffer pb is free once both have run.
        mma_commit(sh.bar(kBarPairPvDone0 + pb));
        mma_commit_cluster(pairdone_remote + 8u * pb);
      }
      mma_commit(sh.bar(kBarDrainPV));
      drain_wait(sh.bar(kBarDrainPV), 0, args.wait_ns);
      // The peer's commits on this CTA's pair barriers have all landed once their last
      // phases completed; only then may this CTA exit.  (After a timeout the teardown below
      // waits for them instead: the peer may not have issued those PVs.)
      if (!*abort_flag)
        for (int j = max(0, ntiles - 2); j < ntiles; ++j)
          drain_wait(sh.bar(kBarPairPvDone0 + (j & 1)), (j >> 1) & 1, args.wait_ns);
    }
    __syncwarp();
  } else if (warp == kWarpRelay) {
    // ------------------------------------------------------------ buffer-empty relay to the peer
    // The readers arrive on the local barriers only once their loads of Sin have
    // returned data (see after_loads), so when this thread sees a phase complete
    // the peer may overwrite that buffer.
    if (lane == 0) {
      // It also arms each Sin buffer's barrier for the bytes of its next tile, in tile
      // order: a buffer's next phase is armed only after its last one was consumed.
      const uint32_t soutempty_remote = map_to_rank(sh.bar(kBarSoutEmpty0), peer);  // + 8 * buffer
      for (int j = 0; j < ntiles && j < kSinBufs; ++j) mbar_arrive_expect_tx(sh.bar(kBarSinFull0 + j), kSinBytes);
      for (int j = 0; j < ntiles; ++j) {
        const int ib = j % kSinBufs;
        if (!waiter.wait(sh.bar(kBarSinRead0 + ib), (j / kSinBufs) & 1)) break;
        if (j + kSinBufs < ntiles) mbar_arrive_expect_tx(sh.bar(kBarSinFull0 + ib), kSinBytes);
        mbar_arrive_cluster_relaxed(soutempty_remote + 8u * ib);
      }
    }
    __syncwarp();
  } else if (kFp8 && warp >= 16) {
    // ------------------------------------------------------------ FP8 rows: dequantising warpgroup
    // Thread t takes the 16-value chunk k = t / 8 of this CTA's 256 latent values (scale group
    // 2 rank + k / 8) for tokens r = t % 8 + 8u, u = 0..7.  The eight threads of each quarter-warp
    // phase of a 16-byte access hold eight tokens with r & 7 = 0..7, so their reads of the
    // swizzled landing boxes and their writes into the 128B-swizzled ring boxes QK and PV read
    // (token r, 16-byte chunk c at r * 128 + (c ^ (r & 7)) * 16) fall in eight different bank
    // groups.  Masked tokens (past the split or in a sub-box that was not loaded) are written
    // as zeros.
    const int t = threadIdx.x - 512;
    const int rl = t & 7, k = t >> 3;
    const int grp = 2 * (int)rank + (k >> 3);
    const uint32_t src_off = (uint32_t)(k >> 3) * kLandBoxBytes + (uint32_t)rl * 128u + (uint32_t)(((k & 7) ^ rl) << 4);
    const int c0 = 2 * (k & 3);
    const uint32_t dst_off0 = (uint32_t)(k >> 2) * kBoxBytes + (uint32_t)rl * 128u + (uint32_t)((c0 ^ rl) << 4);
    const uint32_t dst_off1 = (uint32_t)(k >> 2) * kBoxBytes + (uint32_t)rl * 128u + (uint32_t)(((c0 + 1) ^ rl) << 4);
    bool range = false, ok = true;
    // Every lane waits (each reads what the barrier guards); a warp leaves together.
    auto wait_warp = [&](uint32_t bar, uint32_t parity) {
      return __all_sync(0xffffffffu, waiter.wait(bar, parity) ? 1 : 0) != 0;
    };
    // Q's latent half (its two ring stages), bf16 -> fp16, before the QK warp copies it into TMEM.
    if (ntiles > 0) {
      ok = wait_warp(sh.bar(kBarQFull), 0);
      if (ok && !kFp16) {
        uint4* qs = reinterpret_cast<uint4*>(smem_gen + kOffStages + kQStage * kStageBytes);
#pragma unroll 4
        for (int i = t; i < (int)(kQLatBytes / 16); i += 128) {
          uint4 v = qs[i];
          bf16x8_to_fp16(v, range);
          qs[i] = v;
        }
      }
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(sh.bar(kBarQConv));
    for (int j = 0; ok && j < ntiles; ++j) {
      const int s = j % kStages, ls = j % kLandSlots;
      if (!wait_warp(sh.bar(kBarLandFull0 + ls), (j / kLandSlots) & 1)) break;
      // Ring stage s was last read by PV(j - kStages); the last two stages first held Q's latent half.
      if (j >= kStages && !wait_warp(sh.bar(kBarKvEmpty + s), ((j / kStages) - 1) & 1)) break;
      if (j == kQStage && !wait_warp(sh.bar(kBarQCopied), 0)) break;
      const uint32_t bm = land_mask[ls];
      const int nvalid = min(kTile, end - (start + j * kTile));
      const unsigned char* src = smem_gen + kOffLand + ls * kLandBytes;
      unsigned char* dst = smem_gen + kOffStages + s * kStageBytes;
#pragma unroll 2
      for (int u = 0; u < 8; ++u) {
        const int r = rl + 8 * u;
        uint4 lo = make_uint4(0, 0, 0, 0), hi = lo;
        if (r < nvalid && !((bm >> (r >> g_log2)) & 1u)) {
          const uint4 v = *reinterpret_cast<const uint4*>(src + src_off + u * 1024);
          const float sc = *reinterpret_cast<const float*>(src + kLandLatBytes + r * 16 + grp * 4);
          // A scale that can take an e4m3 value (at most 448) past the fp16 range.
          range |= !(fabsf(sc) * 448.f < 65520.f);
          dequant16(v, sc, lo, hi);
        }
        *reinterpret_cast<uint4*>(dst + dst_off0 + u * 1024) = lo;
        *reinterpret_cast<uint4*>(dst + dst_off1 + u * 1024) = hi;
      }
      if (kFp16) {
        // fp16 queries: the tile's bf16 RoPE values -> fp16 in place (the RoPE QK steps are fp16).
        uint4* rp = reinterpret_cast<uint4*>(smem_gen + kOffRope + (j % kRopeSlots) * kRopeBytes);
        for (int i = t; i < (int)(kRopeBytes / 16); i += 128) {
          uint4 v = rp[i];
          bf16x8_to_fp16(v, range);
          rp[i] = v;
        }
      }
      if (t == 0) bad_mask[s] = bm;
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(sh.bar(kBarKvFull + s));
        mbar_arrive(sh.bar(kBarLandEmpty0 + ls));
      }
    }
    if (range && p.status) atomicOr(p.status, TMLA_STATUS_RANGE);
  } else if (warp >= 4) {
    // ------------------------------------------------------------ head-row warps
    // Warp w (4..15) works on TMEM lane quarter q = w % 4.  Within a quarter,
    // lanes 32q + 16r + [0,16) are the heads this CTA owns, the other sixteen the
    // peer's.  With the 16-lane shapes thread t holds head rows t/4 and t/4 + 8 of
    // a 16-lane group (4 threads per row).
    const int quarter = warp & 3;
    const int role = warp >> 2;  // 1, 2: softmax warpgroups A (even tiles) and B (odd tiles); 3: score sender
    const int L = lane >> 2, t4 = lane & 3;
    const uint32_t q_lanes = (uint32_t)(quarter * 32) << 16;
    const uint32_t own_lanes = (uint32_t)(quarter * 32 + 16 * (int)rank) << 16;
    const uint32_t peer_lanes = (uint32_t)(quarter * 32 + 16 * (int)peer) << 16;
    const int last = ntiles - 1;
    float* lstat = reinterpret_cast<float*>(smem_gen + kOffStat);  // [128 rows] (l, m)

    if (role <= 2) {
      const int wg = role - 1;  // this warpgroup runs the tiles j with j % 2 == wg
      // ---------------------------------------------------------- softmax of my 16 rows of this quarter
      // Tiles alternate between the two warpgroups.  The running maximum of tile j-1
      // comes from the other warpgroup through shared memory (one barrier per quarter);
      // each warpgroup keeps partial row sums relative to the maximum of its own last tile.
      // After its own rows, the warpgroup also takes the peer's P rows of the tile
      // (copied straight into this CTA's P buffer) and rescales O for them when asked.
      const float4* sin = reinterpret_cast<const float4*>(smem_gen + kOffSin);
      const float2* alpha_in = reinterpret_cast<const float2*>(smem_gen + kOffAlpha);
      float* m_mine = reinterpret_cast<float*>(smem_gen + kOffMx) + 64 * wg;
      const float* m_other = reinterpret_cast<const float*>(smem_gen + kOffMx) + 64 * (wg ^ 1);
      const uint32_t alpha_remote = map_to_rank(sh.base + kOffAlpha, peer);
      const uint32_t pinfull_remote = map_to_rank(sh.bar(kBarPinFull0), peer);  // + 8 * buffer
      const uint32_t max_out = sh.bar((wg ? kBarMaxB0 : kBarMaxA0) + quarter);
      const uint32_t max_in = sh.bar((wg ? kBarMaxA0 : kBarMaxB0) + quarter);
      const bool arm = quarter == 0 && lane == 0;
      const int t128 = quarter * 32 + lane;
      const int orow = quarter * 16 + L;  // index of row L among this CTA's 64 owned rows (row L + 8: orow + 8)
      if (wg == 1 && arm) mbar_arrive_expect_tx(sh.bar(kBarFinFull), kFinBytes);
      float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;  // rows L and L + 8 (partial sums)
      bool ok = true;
      for (int j = wg; j < ntiles; j += 2) {
        const int sb = wg;  // S, alpha and barrier set of this tile (j % 2)
        const int ib = j % kSinBufs, pbi = j % kPBufs;  // its Sin buffer and P buffer
        const uint32_t ph = (uint32_t)(j >> 1) & 1u;
        if (arm) mbar_arrive_expect_tx(sh.bar(kBarPinFull0 + sb), kPPeerBytes + kAlphaBytes);
        if (!waiter.wait(sh.bar(kBarSFull0 + sb), ph)) {
          ok = false;
          break;
        }
        const uint32_t bm = tile_mask[sb];  // the tile's masked sub-boxes (published with SFull)
        tc_fence_after();
        float s[32];
        {
          uint32_t r[32];
          tmem_ld16x256_x8(tmem + own_lanes + kColS + 64 * sb, r);
          tc_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) s[i] = __uint_as_float(r[i]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(sh.bar(kBarSEmpty0 + sb));
        // The running maximum after tile j-1, published by the other warpgroup once it has
        // read Sin(j-1).  With one Sin buffer it is taken first: until Sin(j-1) was read,
        // the buffer's barrier may still be in tile j-1's phase, whose parity differs from
        // tile j's, and a parity wait would pass at once.
        float mp_a = -INFINITY, mp_b = -INFINITY;
        auto take_running_max = [&]() -> bool {
          if (!waiter.wait(max_in, (uint32_t)((j - 1) >> 1) & 1u)) return false;
          mp_a = m_other[orow];
          mp_b = m_other[orow + 8];
          return true;
        };
        if (kSinBufs == 1 && j > 0 && !take_running_max()) {
          ok = false;
          break;
        }
        if (!waiter.wait(sh.bar(kBarSinFull0 + ib), (uint32_t)(j / kSinBufs) & 1u, true)) {
          ok = false;
          break;
        }
        uint32_t dep = 0;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const float4 v = sin[ib * (kSinBytes / 16) + (quarter * 8 + c) * 32 + lane];
          dep ^= __float_as_uint(v.x) ^ __float_as_uint(v.y) ^ __float_as_uint(v.z) ^ __float_as_uint(v.w);
          s[4 * c] += v.x;
          s[4 * c + 1] += v.y;
          s[4 * c + 2] += v.z;
          s[4 * c + 3] += v.w;
        }
        // Sin has been read: a local arrive that warp 3 forwards to the peer, which may then
        // overwrite Sin.  The arrive's address depends on every loaded word, so it cannot
        // issue while a load of this warp is still in flight (a warp's loads complete for
        // all lanes at once).
        if (lane == 0) mbar_arrive(after_loads(sh.bar(kBarSinRead0 + ib), dep));

        // Online softmax (base 2) with lazy rescaling; a row's 64 scores sit in 4 threads.
        // The scale is folded into the exponent's FMA, so the row maximum of the scaled
        // scores is the largest raw score times the scale for a positive scale and the
        // smallest for a negative one.  Only a tile with masked tokens (the last one of the
        // split, or one with a page id outside the pool) needs masking.
        const float sc = args.scale_log2;
        const bool neg = sc < 0.f;
        const int nvalid = min(kTile, end - (start + j * kTile));

        const bool partial = nvalid < kTile || bm != 0u;
        // Fast path for the common tile (all 64 tokens valid, positive scale); the general
        // path masks tokens and takes the minimum for a negative scale.
        const bool general = partial || neg;
        float mx_a = -INFINITY, mx_b = -INFINITY;
        if (!general) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            if (i & 2)
              mx_b = fmaxf(mx_b, s[i]);
            else
              mx_a = fmaxf(mx_a, s[i]);
          }
          mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
          mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
          mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2)) * sc;
          mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2)) * sc;
        } else {
          if (partial) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int col = 8 * (i >> 2) + 2 * t4 + (i & 1);
              if (col >= nvalid || ((bm >> (col >> g_log2)) & 1u)) s[i] = neg ? INFINITY : -INFINITY;
            }
          }
          if (!neg) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              if (i & 2)
                mx_b = fmaxf(mx_b, s[i]);
              else
                mx_a = fmaxf(mx_a, s[i]);
            }
            mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
            mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
            mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
            mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
          } else {
            mx_a = mx_b = INFINITY;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              if (i & 2)
                mx_b = fminf(mx_b, s[i]);
              else
                mx_a = fminf(mx_a, s[i]);
            }
            mx_a = fminf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
            mx_b = fminf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
            mx_a = fminf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
            mx_b = fminf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
          }
          // A row whose tokens are all masked in this tile has no maximum here (and a zero
          // scale must not turn the infinite mask value into NaN).
          mx_a = isinf(mx_a) ? -INFINITY : mx_a * sc;
          mx_b = isinf(mx_b) ? -INFINITY : mx_b * sc;
        }
        if (kSinBufs == 2 && j > 0 && !take_running_max()) {
          ok = false;
          break;
        }
        float mn_a = mp_a, mn_b = mp_b, al_a = 1.f, al_b = 1.f;
        const bool need_a = mx_a > mp_a + kRescaleThreshold, need_b = mx_b > mp_b + kRescaleThreshold;
        if (need_a) {
          al_a = ex2(mp_a - mx_a);  // 0 on the first tile (m = -inf)
          mn_a = mx_a;
        }
        if (need_b) {
          al_b = ex2(mp_b - mx_b);
          mn_b = mx_b;
        }
        if (t4 == 0) {
          m_mine[orow] = mn_a;
          m_mine[orow + 8] = mn_b;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(max_out);
        // This warpgroup's partial sums were relative to the maximum of its previous tile.
        l_a = m_a == -INFINITY ? 0.f : l_a * ex2(m_a - mn_a);
        l_b = m_b == -INFINITY ? 0.f : l_b * ex2(m_b - mn_b);
        m_a = mn_a;
        m_b = mn_b;
        uint32_t pw[16];
        float sum_a = 0.f, sum_b = 0.f;
        if (!partial) {
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const float p0 = ex2(fmaf(s[4 * k], sc, -mn_a)), p1 = ex2(fmaf(s[4 * k + 1], sc, -mn_a));
            const float p2 = ex2(fmaf(s[4 * k + 2], sc, -mn_b)), p3 = ex2(fmaf(s[4 * k + 3], sc, -mn_b));
            sum_a += p0 + p1;
            sum_b += p2 + p3;
            pw[2 * k] = pack2(p0, p1, kLatFp16);
            pw[2 * k + 1] = pack2(p2, p3, kLatFp16);
          }
        } else {
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            float p0 = ex2(fmaf(s[4 * k], sc, -mn_a)), p1 = ex2(fmaf(s[4 * k + 1], sc, -mn_a));
            float p2 = ex2(fmaf(s[4 * k + 2], sc, -mn_b)), p3 = ex2(fmaf(s[4 * k + 3], sc, -mn_b));
            // Masked tokens weigh exactly 0, also when the row has no maximum yet.
            const int c0 = 8 * k + 2 * t4;
            const bool v0 = c0 < nvalid && !((bm >> (c0 >> g_log2)) & 1u);
            const bool v1 = c0 + 1 < nvalid && !((bm >> ((c0 + 1) >> g_log2)) & 1u);
            p0 = v0 ? p0 : 0.f;
            p2 = v0 ? p2 : 0.f;
            p1 = v1 ? p1 : 0.f;
            p3 = v1 ? p3 : 0.f;
            sum_a += p0 + p1;
            sum_b += p2 + p3;
            pw[2 * k] = pack2(p0, p1, kLatFp16);
            pw[2 * k + 1] = pack2(p2, p3, kLatFp16);
          }
        }
        l_a += sum_a;
        l_b += sum_b;
        // P buffer pbi (in both CTAs) was last read by PV(j - kPBufs).
        if (j >= kPBufs && !waiter.wait(sh.bar(kBarPairPvDone0 + ((j - kPBufs) & 1)), (uint32_t)((j - kPBufs) >> 1) & 1u)) {
          ok = false;
          break;
        }
        {
          // Own rows of P into this CTA's buffer, in the 128B-swizzled K-major layout PV
          // reads (row r: 128 bytes at r * 128, 16-byte chunk c at (c ^ (r & 7)) * 16): word
          // t4 of chunk k holds this thread's tokens 8k + 2 t4 and 8k + 2 t4 + 1.
          unsigned char* pbuf = smem_gen + kOffPBuf + pbi * kPBufBytes;
          const int ra = quarter * 32 + 16 * (int)rank + L, rb = ra + 8;
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            *reinterpret_cast<uint32_t*>(pbuf + ra * 128 + ((k ^ (ra & 7)) << 4) + 4 * t4) = pw[2 * k];
            *reinterpret_cast<uint32_t*>(pbuf + rb * 128 + ((k ^ (rb & 7)) << 4) + 4 * t4) = pw[2 * k + 1];
          }
          fence_proxy_async_smem();
          __syncwarp();
          // The same 16 rows (2 KB, contiguous) into the peer's buffer, with the rescale factors.
          if (lane == 0) {
            const uint32_t off = kOffPBuf + pbi * kPBufBytes + (uint32_t)(quarter * 32 + 16 * (int)rank) * 128u;
            bulk_copy_to_cta(map_to_rank(sh.base + off, peer), sh.base + off, 2048u, pinfull_remote + 8u * sb);
          }
          if (t4 == 0)
            st_async_f2(alpha_remote + (uint32_t)sb * kAlphaBytes + (uint32_t)(quarter * 8 + L) * 8u, al_a, al_b,
                        pinfull_remote + 8u * sb);
        }
        if (j > 0 && __any_sync(0xffffffffu, need_a || need_b)) {
          if (!waiter.wait(sh.bar(kBarPvDone0 + ((j - 1) & 1)), (uint32_t)((j - 1) >> 1) & 1u)) {
            ok = false;
            break;
          }
          tc_fence_after();
          rescale_rows16(tmem + own_lanes, al_a, al_b);
        }
        // (FP8 rows: the dequantising warps wrote zeros there already.)
        if (!kFp8 && partial)
          zero_masked_rows(smem_gen + kOffStages + (j % kStages) * kStageBytes, nvalid, bm, g_log2, t128);
        // The peer's rows of P(j) and their rescale factors.
        if (!waiter.wait(sh.bar(kBarPinFull0 + sb), ph, true)) {
          ok = false;
          break;
        }
        const float2 al = alpha_in[sb * 32 + quarter * 8 + L];
        if (__any_sync(0xffffffffu, j > 0 && (al.x != 1.f || al.y != 1.f))) {
          if (!waiter.wait(sh.bar(kBarPvDone0 + ((j - 1) & 1)), (uint32_t)((j - 1) >> 1) & 1u)) {
            ok = false;
            break;
          }
          tc_fence_after();
          rescale_rows16(tmem + peer_lanes, al.x, al.y);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(sh.bar(kBarPFull0 + sb));
      }
      // Row sums: add the four threads' shares; both warpgroups' (l, m) meet in shared memory.
      l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
      l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
      l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
      l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);
      float2* wst = reinterpret_cast<float2*>(smem_gen + kOffWst);  // [2 warpgroups][64 owned rows]
      if (t4 == 0) {
        wst[64 * wg + orow] = make_float2(l_a, m_a);
        wst[64 * wg + orow + 8] = make_float2(l_b, m_b);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(sh.bar(kBarWgStats));
      const bool stats_ok = waiter.wait(sh.bar(kBarWgStats), 0);
      if (wg == 0) {
        // Owned rows: the final maximum is the larger of the two warpgroups' last ones
        // (maxima only grow); (l, m) go to the peer for its half of these rows' output.
        if (lane < 16 && stats_ok) {
          const int o = quarter * 16 + lane;
          const float2 A = wst[o], Bw = wst[64 + o];
          const float mf = fmaxf(A.y, Bw.y);
          // A warpgroup whose maximum never left -inf has a zero sum, or NaN (a NaN scale),
          // which must reach the LSE.
          float l = 0.f;
          l += A.y != -INFINITY ? A.x * ex2(A.y - mf) : (A.x != A.x ? A.x : 0.f);
          l += Bw.y != -INFINITY ? Bw.x * ex2(Bw.y - mf) : (Bw.x != Bw.x ? Bw.x : 0.f);
          const int row = quarter * 32 + 16 * (int)rank + lane;
          st_async_f2(map_to_rank(sh.base + kOffFin, peer) + (uint32_t)o * 8u, l, mf,
                      map_to_rank(sh.bar(kBarFinFull), peer));
          lstat[2 * row] = l;
          const int hh = h0 + row;
          if (hh < H) {
            // An empty row gives -inf; a NaN sum (a NaN scale or input) stays NaN.
            const float lse2 = l <= 0.f ? -INFINITY : mf + log2f(l);
            if (final_out) {
              if (p.lse) p.lse[(int64_t)b * p.lse_stride_b + hh] = lse2 * kLn2;
            } else if (args.units) {
              p.ws_lse[(int64_t)slot * H + hh] = lse2;
            } else {
              p.ws_lse[((int64_t)b * H + hh) * p.num_splits + split] = lse2;
            }
          }
        }
      } else {
        // The peer's final row sums of its rows, for this CTA's half of their output.
        const float2* fin = reinterpret_cast<const float2*>(smem_gen + kOffFin);
        if (waiter.wait(sh.bar(kBarFinFull), 0, true) && lane < 16) {
          const float2 f = fin[quarter * 16 + lane];
          lstat[2 * (quarter * 32 + 16 * (int)peer + lane)] = f.x;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(sh.bar(kBarStats));
      // Epilogue share: output columns [128 wg, 128 wg + 128) of all 32 rows of this quarter.
      bool have_o = ok && stats_ok && ntiles > 0;
      have_o = waiter.wait(sh.bar(kBarStats), 0) && have_o;
      if (have_o) {
        have_o = waiter.wait(sh.bar(kBarPvDone0 + (last & 1)), (last >> 1) & 1);
        tc_fence_after();
      }
      // The tiles below reuse the ring, where Q's latent half landed first (a split with no
      // tokens never waited for it).
      drain_wait(sh.bar(kBarQFull), 0, args.wait_ns);
      if (kFp8) drain_wait(sh.bar(kBarQConv), 0, args.wait_ns);
      const float l = lstat[2 * (quarter * 32 + lane)];
      // 16-bit tiles for the final output and for 16-bit partials, fp32 tiles otherwise.
      stage_rows<T>(smem_gen, tmem + q_lanes, have_o, quarter * 32 + lane, l > 0.f ? 1.f / l : 0.f,
                    4 * wg, 4, final_out || kPart16);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(sh.bar(kBarEpi));
      if (wg == 0 && quarter == 0 && lane == 0) {
        // One thread stores the staged half-tile; rows past H fall outside the tensor map
        // and are not written.
        if (waiter.wait(sh.bar(kBarEpi), 0)) {
          if (final_out) {
#pragma unroll 1
            for (int c = 0; c < 4; ++c)
              tma_store_3d(&tm_out, sh.base + out_box_off(c), kHalfLatent * (int)rank + 64 * c, h0, b);
          } else if (kPart16) {
            // 16-bit partials: four boxes of 64 columns, like the final output.
#pragma unroll 1
            for (int c = 0; c < 4; ++c) {
              if (args.units)
                tma_store_3d(&tm_part, sh.base + out_box_off(c), kHalfLatent * (int)rank + 64 * c, h0, slot);
              else
                tma_store_4d(&tm_part, sh.base + out_box_off(c), kHalfLatent * (int)rank + 64 * c, split, h0, b);
            }
          } else if (args.units) {
#pragma unroll 1
            for (int c = 0; c < 8; ++c)
              tma_store_3d(&tm_part, sh.base + out_box_off(c), kHalfLatent * (int)rank + 32 * c, h0,
                           slot);
          } else {
#pragma unroll 1
            for (int c = 0; c < 8; ++c)
              tma_store_4d(&tm_part, sh.base + out_box_off(c), kHalfLatent * (int)rank + 32 * c, split,
                           h0, b);
          }
          bulk_commit_group();
          bulk_wait_group0();
        }
      }
    } else {
      // ---------------------------------------------------------- score sender for the peer's 16 rows
      const uint32_t sin_remote = map_to_rank(sh.base + kOffSin, peer);
      const uint32_t sinfull_remote = map_to_rank(sh.bar(kBarSinFull0), peer);  // + 8 * buffer
      for (int j = 0; j < ntiles; ++j) {
        const int sb = j & 1;
        if (!waiter.wait(sh.bar(kBarSFull0 + sb), (j >> 1) & 1)) break;
        tc_fence_after();
        uint32_t r[32];
        tmem_ld16x256_x8(tmem + peer_lanes + kColS + 64 * sb, r);
        tc_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(sh.bar(kBarSEmpty0 + sb));
        // Into the peer's score buffer it last read for tile j - kSinBufs.
        const int ib = j % kSinBufs;
        if (j >= kSinBufs && !waiter.wait(sh.bar(kBarSoutEmpty0 + ib), ((j - kSinBufs) / kSinBufs) & 1, true)) break;
#pragma unroll
        for (int c = 0; c < 8; ++c)
          st_async_u4(sin_remote + (uint32_t)ib * kSinBytes + (uint32_t)((quarter * 8 + c) * 32 + lane) * 16u,
                      make_uint4(r[4 * c], r[4 * c + 1], r[4 * c + 2], r[4 * c + 3]), sinfull_remote + 8u * ib);
      }
    }
  }

  // The split merge, when it follows in the stream, may be scheduled once every CTA got here.
  griddep_launch_dependents();
  // Teardown: both CTAs are done with each other's shared memory before either exits.
  // Each CTA tells the peer whether it gave up (a plain remote store, which the cluster
  // barrier orders).  The barrier orders such stores, not the asynchronous transfers the peer
  // issued into this CTA before reaching it (st.async score rows and rescale factors, bulk
  // copies of P rows, MMA-commit arrivals on the pair barriers).  On the normal path this CTA
  // waited for every one of them; after a timed-out wait it did not, so both CTAs then hold
  // their shared memory a while longer (kInFlightNs, far above a transfer's latency) before
  // leaving: a CTA that exits under a landing transfer loses the context.
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0)
    asm volatile("st.relaxed.cluster.shared::cluster.u32 [%0], %1;" ::"r"(map_to_rank(sh.base + kOffMisc + 4, peer)),
                 "r"(*abort_flag ? 1 : 0)
                 : "memory");
  cluster_sync();
  if (threadIdx.x == 0 && (*abort_flag || *reinterpret_cast<volatile int*>(smem_gen + kOffMisc + 4))) {
    const uint64_t t0 = globaltimer();
    while (globaltimer() - t0 < kInFlightNs) {
    }
  }
  if (warp == kWarpQK) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace TMLA_SM100_NS
}  // namespace tmla
