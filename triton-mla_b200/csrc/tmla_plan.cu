// Per-request split plan computed on the GPU from the lengths in device memory.
//
// The host planner (tmla_plan_units) needs the lengths on the host, and the unit count it
// returns becomes the split kernel's grid.  This planner reads the lengths where the decode
// reads them, in the same stream, and writes a table of a fixed capacity: entries past the
// plan's units are {-1, 0, 0, -1}, whose clusters exit at once.  So the plan kernel, the
// split kernel and the merge can be captured in a CUDA graph once and replayed while the
// lengths change.  The reference has no counterpart: its `num_splits=None` reads
// max(cache_seqlens) on the host (src/triton_mla/kernel.py:264-266) and splits every
// request alike.
//
// The choice follows the host planner: candidate targets are the longest request cut into
// k = 1 .. 64 equal parts; a request of t tiles gets ceil(t / target) splits, each unit costs
// its tiles + 8 tiles of fixed cost (+ 2 of merge when the request is split).  The host
// planner simulates the longest-first schedule for each candidate; here each candidate's
// schedule length is estimated from bounds instead:
//   * the longest unit;
//   * the total cost over the machines (the clusters that run at once);
//   * waves: among the j * machines + 1 longest units, one machine runs at least j + 1, so
//     the schedule is at least (j + 1) x the (j * machines + 1)-th longest unit.
// For the last bound, the requests are bucketed by tile count (8 buckets per octave, each
// standing at its lower edge) and the units' costs by 8 buckets per octave; the unit and
// slot counts, the longest unit and the total cost are exact.  The smallest
// estimate wins (ties: fewer units); candidates with more units or partial slots than the
// table holds are skipped, and k = 1 (one unit per request, no slots) always fits.
// Units are written longest first (bucketed by their tile count, 128 buckets), which is the
// order the hardware starts clusters in.
//
// One launch of a cluster of 8 CTAs: every CTA reads the lengths; CTA c evaluates candidates
// 8c .. 8c + 7 (4 warps each); CTA 0 gathers the 64 estimates from the others' shared memory,
// picks one and writes the plan.
#include <algorithm>

#include "tmla_common.cuh"
#include "tmla_ptx.cuh"

namespace tmla {
namespace {

using namespace ptx;

constexpr int kPlanCtas = 8;        // one cluster
constexpr int kPlanThreads = 1024;
constexpr int kPlanCand = 64;      // candidate targets, and the most splits of one request
constexpr int kCandPerCta = kPlanCand / kPlanCtas;
constexpr int kWarpsPerCand = kPlanThreads / 32 / kCandPerCta;  // 4
constexpr int kCostBuckets = 128;  // unit costs, 8 buckets per octave (costs below 2^16); 4 per lane
constexpr int kOrderBuckets = 128;  // unit tile counts relative to the target, longest first
constexpr int kPlanFixed = 8;      // per-unit fixed cost in tiles (the host planner's constant)
constexpr int kPlanMerge = 2;      // per-unit merge cost of a split request, in tiles
constexpr int kTilesInSmem = 8192;  // requests whose tile counts sit in shared memory (32 KB,
                                    // with the static arrays under the 48 KB that need no opt-in)

__device__ __forceinline__ int tiles_of(int len) { return len > 0 ? (len + 63) / 64 : 0; }

__device__ __forceinline__ int splits_for(int tiles, int target) {
  return min(kPlanCand, max(1, (tiles + target - 1) / target));
}

// ceil(a / b) for a >= 0, b >= 1, given rb ~ 1 / b: a float estimate of the quotient, then
// exact integer correction (the candidate loop runs this for every request and candidate,
// and the integer divide is many instructions).
__device__ __forceinline__ int ceil_div_rcp(int a, int b, float rb) {
  int q = (int)((float)a * rb);
  int r = a - q * b;
  while (r < 0) {
    --q;
    r += b;
  }
  while (r >= b) {
    ++q;
    r -= b;
  }
  return q + (r > 0 ? 1 : 0);
}

// Splits and unit cost of a request of t tiles for a candidate target (rcp_target ~ 1 / target).
__device__ __forceinline__ void unit_shape(int t, int target, float rcp_target, int& ns, int& cost) {
  ns = min(kPlanCand, max(1, ceil_div_rcp(t, target, rcp_target)));
  cost = ceil_div_rcp(t, ns, __frcp_rn((float)ns)) + kPlanFixed + (ns > 1 ? kPlanMerge : 0);
}

__device__ __forceinline__ int cost_bucket(int cost) {
  return min(kCostBuckets - 1, max(0, (int)(8.f * log2f((float)max(cost, 1)))));
}

__device__ __forceinline__ float bucket_floor(int q) { return exp2f((float)q * 0.125f); }

// Tile counts in 8 buckets per octave: bucket 0 holds empty requests, bucket q >= 1 the
// counts in [2^((q-1)/8), 2^(q/8)); its lower edge stands for every request in it.
__device__ __forceinline__ int tile_bucket(int t) {
  return t <= 0 ? 0 : min(kCostBuckets - 1, 1 + (int)(8.f * log2f((float)t)));
}
__device__ __forceinline__ int tile_bucket_floor(int q) {
  return q == 0 ? 0 : (int)ceilf(exp2f((float)(q - 1) * 0.125f));
}

__device__ __forceinline__ unsigned long long warp_sum64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ int ld_cluster_s32(uint32_t addr) {
  int v;
  asm volatile("ld.shared::cluster.s32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}

__global__ void __cluster_dims__(kPlanCtas, 1, 1) __launch_bounds__(kPlanThreads)
    plan_units_kernel(const int32_t* __restrict__ seqlens, int batch, int machines, int capacity, int slot_capacity,
                      int4* __restrict__ units, int32_t* __restrict__ req_first) {
  __shared__ int s_hist[kCandPerCta][kCostBuckets];  // per local candidate: units per cost bucket
  __shared__ int s_tile_hist[kCostBuckets];           // requests per tile-count bucket
  __shared__ unsigned long long s_pcost[kCandPerCta];
  __shared__ int s_pn[kCandPerCta], s_psl[kCandPerCta], s_plg[kCandPerCta];
  __shared__ int s_units[kPlanCand];
  __shared__ float s_est[kPlanCand];
  __shared__ int s_scan[kPlanThreads];
  __shared__ int s_order[kOrderBuckets];
  __shared__ int s_max_tiles, s_target, s_units_used;
  extern __shared__ int s_tiles[];  // tile counts of the first kTilesInSmem requests
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int crank = (int)cluster_ctarank();

  for (int i = tid; i < kCandPerCta * kCostBuckets; i += kPlanThreads) (&s_hist[0][0])[i] = 0;
  if (tid < kCostBuckets) s_tile_hist[tid] = 0;
  if (tid < kOrderBuckets) s_order[tid] = 0;
  if (tid < kCandPerCta) {
    s_pcost[tid] = 0;
    s_pn[tid] = 0;
    s_psl[tid] = 0;
    s_plg[tid] = 0;
  }
  if (tid == 0) s_max_tiles = 0;
  __syncthreads();

  // Every CTA: tile counts, the longest request, and requests per tile-count bucket.  Each
  // thread owns a contiguous run of requests, so slots are numbered in request order.
  const int chunk = (batch + kPlanThreads - 1) / kPlanThreads;
  const int b0 = min(batch, tid * chunk), b1 = min(batch, b0 + chunk);
  int mx = 0;
  for (int i = 0; i < chunk; ++i) {  // the same trip count in every lane
    const int b = b0 + i;
    const bool live = b < b1;
    const int t = live ? tiles_of(seqlens[b]) : 0;
    if (live && b < kTilesInSmem) s_tiles[b] = t;
    mx = max(mx, t);
    // Requests of a warp often share a bucket (uniform batches): one atomic then.
    const int q = live ? tile_bucket(t) : -1;
    const int q0 = __shfl_sync(0xffffffffu, q, 0);
    const unsigned live_mask = __ballot_sync(0xffffffffu, live);
    if (__all_sync(0xffffffffu, !live || q == q0)) {
      if (lane == 0 && live_mask) atomicAdd(&s_tile_hist[q0], __popc(live_mask));
    } else if (live) {
      atomicAdd(&s_tile_hist[q], 1);
    }
  }
  mx = __reduce_max_sync(0xffffffffu, mx);
  if (lane == 0) atomicMax(&s_max_tiles, mx);
  __syncthreads();
  const int max_tiles = s_max_tiles;
  auto tiles_at = [&](int b) { return b < kTilesInSmem ? s_tiles[b] : tiles_of(seqlens[b]); };

  // Candidates: CTA c takes k = 8c + 1 .. 8c + 8, four warps per candidate splitting the
  // requests; a target equal to the previous k's is skipped.
  {
    const int lc = warp / kWarpsPerCand, sub = warp % kWarpsPerCand;
    const int k = crank * kCandPerCta + lc + 1, target = max(1, (max_tiles + k - 1) / k);
    const bool repeat = k > 1 && target == max(1, (max_tiles + k - 2) / (k - 1));
    if (!repeat) {
      const float rcp_target = __frcp_rn((float)target);
      unsigned long long cost = 0;
      int n = 0, sl = 0, lg = 0;
      for (int b = sub * 32 + lane; b < batch; b += 32 * kWarpsPerCand) {
        int ns, c;
        unit_shape(tiles_at(b), target, rcp_target, ns, c);
        cost += (unsigned long long)ns * (unsigned long long)c;
        n += ns;
        sl += ns > 1 ? ns : 0;
        lg = max(lg, c);
      }
      cost = warp_sum64(cost);
      n = (int)__reduce_add_sync(0xffffffffu, (unsigned)n);
      sl = (int)__reduce_add_sync(0xffffffffu, (unsigned)sl);
      lg = __reduce_max_sync(0xffffffffu, lg);
      if (lane == 0) {
        atomicAdd(&s_pcost[lc], cost);
        atomicAdd(&s_pn[lc], n);
        atomicAdd(&s_psl[lc], sl);
        atomicMax(&s_plg[lc], lg);
      }
      if (sub == 0) {
        // The unit-cost histogram of the wave bound from the tile-count buckets, each
        // standing at its lower edge (lane l maps buckets 4l .. 4l + 3).
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int qt = 4 * lane + i, m = s_tile_hist[qt];
          if (m > 0) {
            int ns, c;
            unit_shape(tile_bucket_floor(qt), target, rcp_target, ns, c);
            atomicAdd(&s_hist[lc][cost_bucket(c)], m * ns);
          }
        }
      }
    }
    __syncthreads();
    if (sub == 0) {
      float est = INFINITY;
      const int n = s_pn[lc];
      if (!repeat && n <= capacity && s_psl[lc] <= slot_capacity) {
        // Wave bound for every bucket q at once: with C_q units in buckets >= q and
        // C_q >= j * machines + 1, the (j * machines + 1)-th longest unit is >= floor(q).
        // Lane l holds buckets 4l .. 4l + 3; C_q needs the counts of the higher lanes.
        int cq[4], local = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          cq[i] = s_hist[lc][4 * lane + i];
          local += cq[i];
        }
        int above = local;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int v = __shfl_down_sync(0xffffffffu, above, o);
          if (lane + o < 32) above += v;
        }
        int C = above - local;
        float bound = 0.f;
#pragma unroll
        for (int i = 3; i >= 0; --i) {
          C += cq[i];
          if (C >= machines + 1) bound = fmaxf(bound, (float)((C - 1) / machines + 1) * bucket_floor(4 * lane + i));
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) bound = fmaxf(bound, __shfl_xor_sync(0xffffffffu, bound, o));
        est = fmaxf(fmaxf((float)s_plg[lc], (float)s_pcost[lc] / (float)machines), bound);
      }
      if (lane == 0) {
        s_est[lc] = est;  // this CTA's candidates sit in entries 0 .. 7
        s_units[lc] = repeat ? 0 : n;
      }
    }
  }
  cluster_sync();
  if (crank == 0 && tid < kPlanCand) {
    const int src = tid / kCandPerCta, i = tid % kCandPerCta;
    const float e = ld_cluster_f32(map_to_rank(smem_u32(&s_est[i]), (uint32_t)src));
    const int n = ld_cluster_s32(map_to_rank(smem_u32(&s_units[i]), (uint32_t)src));
    __syncwarp();
    s_est[tid] = e;  // candidate tid of the whole cluster (the loads above are done: the
    s_units[tid] = n;  // entries 0 .. 7 they read are overwritten only after the warp sync)
  }
  // The other CTAs' shared memory stays alive until CTA 0 has read it; then they leave.
  cluster_sync();
  if (crank != 0) return;
  if (tid == 0) {
    int best = 0;  // k = 1 fits whenever capacity >= batch
    for (int k = 1; k < kPlanCand; ++k) {
      const float e = s_est[k], eb = s_est[best];
      if (e < eb * (1.f - 1e-6f) || (e <= eb * (1.f + 1e-6f) && s_units[k] < s_units[best])) best = k;
    }
    s_target = max(1, (max_tiles + best) / (best + 1));
    s_units_used = s_units[best];
  }
  __syncthreads();
  const int target = s_target;

  // Partial slots: an exclusive scan, in request order, of the splits of split requests.
  int mine_slots = 0;
  for (int b = b0; b < b1; ++b) {
    const int ns = splits_for(tiles_at(b), target);
    mine_slots += ns > 1 ? ns : 0;
  }
  s_scan[tid] = mine_slots;
  __syncthreads();
  for (int off = 1; off < kPlanThreads; off <<= 1) {
    const int v = tid >= off ? s_scan[tid - off] : 0;
    __syncthreads();
    s_scan[tid] += v;
    __syncthreads();
  }
  int slot = s_scan[tid] - mine_slots;

  // Longest-first order: count the units per tile-count bucket, then place them.
  auto order_bucket = [&](int unit_tiles) {
    return (int)(((long long)(target - min(unit_tiles, target)) * (kOrderBuckets - 1)) / target);
  };
  for (int b = b0; b < b1; ++b) {
    const int t = tiles_at(b);
    const int ns = splits_for(t, target), per = (t + ns - 1) / ns;
    for (int s = 0; s < ns; ++s) atomicAdd(&s_order[order_bucket(min(t, (s + 1) * per) - min(t, s * per))], 1);
  }
  __syncthreads();
  if (tid == 0) {
    int acc = 0;
    for (int q = 0; q < kOrderBuckets; ++q) {
      const int c = s_order[q];
      s_order[q] = acc;
      acc += c;
    }
  }
  __syncthreads();
  for (int b = b0; b < b1; ++b) {
    const int t = tiles_at(b);
    const int ns = splits_for(t, target), per = (t + ns - 1) / ns;
    req_first[b] = slot;
    for (int s = 0; s < ns; ++s) {
      const int pos = atomicAdd(&s_order[order_bucket(min(t, (s + 1) * per) - min(t, s * per))], 1);
      units[pos] = make_int4(b, s, ns, ns > 1 ? slot + s : -1);
    }
    slot += ns > 1 ? ns : 0;
  }
  if (tid == kPlanThreads - 1) req_first[batch] = s_scan[kPlanThreads - 1];
  for (int u = s_units_used + tid; u < capacity; u += kPlanThreads) units[u] = make_int4(-1, 0, 0, -1);
}

}  // namespace
}  // namespace tmla

extern "C" {

int tmla_plan_units_device(const int32_t* seqlens, int32_t batch, int32_t num_heads, int32_t num_sms,
                           int32_t capacity, int32_t slot_capacity, int32_t* units, int32_t* req_first, void* stream) {
  if (batch < 0 || num_heads <= 0 || capacity < batch || capacity > 65535 || slot_capacity < 0 || !req_first ||
      (batch > 0 && !seqlens) || (capacity > 0 && !units))
    return TMLA_ERR_INVALID_ARG;
  if (num_sms <= 0) num_sms = 148;
  const int head_tiles = (num_heads + 127) / 128;
  const int machines = std::max(1, num_sms / 2 / head_tiles);
  const size_t smem = sizeof(int) * (size_t)std::min<int>(batch, tmla::kTilesInSmem);
  tmla::plan_units_kernel<<<tmla::kPlanCtas, tmla::kPlanThreads, smem, static_cast<cudaStream_t>(stream)>>>(
      seqlens, batch, machines, capacity, slot_capacity, reinterpret_cast<int4*>(units), req_first);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? TMLA_OK : TMLA_ERR_CUDA;
}

}  // extern "C"
