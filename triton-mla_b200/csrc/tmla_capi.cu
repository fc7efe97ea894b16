// C ABI of the library (declared in include/triton_mla_b200.h): argument
// validation, kernel selection, split heuristic and the launches.
//
// The checks mirror the assertions of the reference wrapper `mla_decode`
// (src/triton_mla/kernel.py:235-262): 3-D q, cache width == d_qk, unit
// innermost strides, power-of-two head_dim_v and RoPE width, equal dtypes,
// dense cache batch == q batch.  Anything that breaks them returns
// TMLA_ERR_INVALID_ARG (the Python wrapper raises AssertionError before it
// gets here, as the reference does).
#include <math.h>
#include <stdio.h>

#include <algorithm>
#include <functional>
#include <queue>
#include <vector>

#include "tmla_common.cuh"

namespace tmla {
int launch_generic(const TmlaDecodeParams& p, cudaStream_t stream);
int launch_combine(const void* ws_o, const float* ws_lse, void* out, int64_t osb, int64_t osh, float* lse,
                   int64_t lsb, int B, int H, int S, int DV, int dtype, bool part16, cudaStream_t stream);
int sm100_supported(const TmlaDecodeParams& p);
int launch_sm100(const TmlaDecodeParams& p, cudaStream_t stream, const int32_t* units = nullptr,
                 int32_t num_units = 0, int32_t num_slots = 0, bool part16 = false);
int launch_combine_slots(const void* ws_o, const float* ws_lse, const int32_t* req_first, void* out, int64_t osb,
                         int64_t osh, float* lse, int64_t lsb, int B, int H, int DV, int dtype, bool part16,
                         cudaStream_t stream);
}  // namespace tmla

namespace {
thread_local char g_cuda_error[256] = "";
}  // namespace

int tmla::record_cuda_error(cudaError_t e) {
  snprintf(g_cuda_error, sizeof(g_cuda_error), "%s: %s", cudaGetErrorName(e), cudaGetErrorString(e));
  return TMLA_ERR_CUDA;
}

namespace {

int cuda_fail(int neg_code) { return tmla::record_cuda_error((cudaError_t)(-neg_code)); }

// Launch helpers return 0, a positive TMLA_ERR_* code or minus a cudaError_t.
int finish(int rc) { return rc < 0 ? cuda_fail(rc) : rc; }

bool is_pow2(int v) { return v > 0 && (v & (v - 1)) == 0; }

int validate(const TmlaDecodeParams* p) {
  if (!p) return TMLA_ERR_INVALID_ARG;
  if (p->batch < 0 || p->num_heads <= 0 || p->num_splits <= 0) return TMLA_ERR_INVALID_ARG;
  // The kernels' grids index requests and splits in grid dimensions of at most 65535 blocks.
  if (p->batch > TMLA_MAX_BATCH || p->num_splits > TMLA_MAX_BATCH) return TMLA_ERR_UNSUPPORTED;
  if (p->d_v <= 0 || p->d_qk <= p->d_v) return TMLA_ERR_INVALID_ARG;
  if (!is_pow2(p->d_v) || !is_pow2(p->d_qk - p->d_v)) return TMLA_ERR_INVALID_ARG;
  if (p->dtype != TMLA_DTYPE_BF16 && p->dtype != TMLA_DTYPE_FP16 && p->dtype != TMLA_DTYPE_FP32)
    return TMLA_ERR_INVALID_ARG;
  if (p->page_size <= 0) return TMLA_ERR_INVALID_ARG;
  if (p->q_len < 0 || (p->q_len > 1 && p->num_heads % p->q_len)) return TMLA_ERR_INVALID_ARG;
  if (p->kv_format != TMLA_KV_SAME && p->kv_format != TMLA_KV_FP8_E4M3) return TMLA_ERR_INVALID_ARG;
  if (p->kv_format == TMLA_KV_FP8_E4M3 && (p->d_qk != 576 || p->d_v != 512 || p->dtype == TMLA_DTYPE_FP32))
    return TMLA_ERR_INVALID_ARG;
  if (p->batch == 0) return TMLA_OK;
  if (!p->q || !p->kv || !p->seqlens || !p->out) return TMLA_ERR_INVALID_ARG;
  if (p->block_table) {
    if (p->bt_width <= 0 || p->num_pages <= 0) return TMLA_ERR_INVALID_ARG;
  } else if (p->num_pages != p->batch) {
    return TMLA_ERR_INVALID_ARG;  // dense cache: one row of pages per request (kernel.py:258)
  }
  if ((p->num_splits > 1 || (p->flags & TMLA_FLAG_PARTIAL_ONLY)) && (!p->ws_o || !p->ws_lse))
    return TMLA_ERR_WORKSPACE;
  return TMLA_OK;
}

int select_kernel(const TmlaDecodeParams& p) {
  if (p.kernel == TMLA_KERNEL_GENERIC) return TMLA_KERNEL_GENERIC;
  if (p.kernel == TMLA_KERNEL_SM100) return tmla::sm100_supported(p) ? TMLA_KERNEL_SM100 : -TMLA_ERR_UNSUPPORTED;
  return tmla::sm100_supported(p) ? TMLA_KERNEL_SM100 : TMLA_KERNEL_GENERIC;
}

// part16: the tcgen05 kernel writes its split partials in the q dtype (16-bit) instead of fp32.
int run_partial(const TmlaDecodeParams& p, cudaStream_t stream, bool part16 = false) {
  const int k = select_kernel(p);
  if (k < 0) return -k;
  if (k == TMLA_KERNEL_SM100) return finish(tmla::launch_sm100(p, stream, nullptr, 0, 0, part16));
  return finish(tmla::launch_generic(p, stream));
}

}  // namespace

extern "C" {

int tmla_abi_version(void) { return TMLA_ABI_VERSION; }

size_t tmla_params_bytes(void) { return sizeof(TmlaDecodeParams); }

const char* tmla_error_string(int code) {
  switch (code) {
    case TMLA_OK: return "ok";
    case TMLA_ERR_INVALID_ARG: return "invalid argument (shape, stride, dtype or size rule broken)";
    case TMLA_ERR_UNSUPPORTED: return "configuration not supported by this build";
    case TMLA_ERR_MISALIGNED: return "pointer or stride is not 16-byte aligned as TMA requires";
    case TMLA_ERR_CUDA: return "CUDA call failed";
    case TMLA_ERR_WORKSPACE: return "split workspace missing or too small";
    default: return "unknown error";
  }
}

const char* tmla_last_cuda_error(void) { return g_cuda_error; }

size_t tmla_workspace_bytes(int32_t batch, int32_t num_heads, int32_t num_splits, int32_t d_v) {
  if (num_splits <= 1 || batch <= 0 || num_heads <= 0 || d_v <= 0) return 0;
  const size_t rows = (size_t)batch * num_heads * num_splits;
  const size_t o = rows * d_v * sizeof(float);
  const size_t l = rows * sizeof(float);
  return ((o + 255) & ~(size_t)255) + ((l + 255) & ~(size_t)255);
}

// B200 split rule.  One unit of work is a 2-CTA cluster (the tcgen05 kernel's
// 128-head tile of one request's split); 148 SMs run 74 such units per wave.
// The estimate, in units of "one cluster streaming one cache row", is
//   waves(s) * (rows per split + fixed cost per unit) + s * merge cost per split
// (below).  The smallest split count within 2% of the best estimate wins.
int32_t tmla_num_splits(int32_t batch, int32_t num_heads, int32_t max_seqlen, int32_t num_sms) {
  if (batch <= 0 || num_heads <= 0 || max_seqlen <= 0) return 1;
  if (num_sms <= 0) num_sms = 148;
  const int clusters = num_sms / 2 > 0 ? num_sms / 2 : 1;
  const long units = (long)batch * ((num_heads + 127) / 128);
  const int tiles = (max_seqlen + 63) / 64;
  const int max_s = tiles < 64 ? tiles : 64;
  const double fixed_rows = 256.0;
  // The merge, in cache rows streamed by one cluster, per split: the 16-bit partials the split
  // writes (2 bytes per output element; the merge reads them back from L2 while the split
  // kernel drains) spread over all clusters, plus 8 rows of merge latency.  Fitted to B200
  // call times of uniform batches (1-256 requests of 1024-16384 tokens, every split count).
  const double merge_rows_per_split = (double)batch * num_heads * 512.0 * 2.0 / (clusters * 1152.0) + 8.0;
  double cost[65];
  double best = INFINITY;
  for (int s = 1; s <= max_s; ++s) {
    const long waves = (units * s + clusters - 1) / clusters;
    const double rows = (double)((tiles + s - 1) / s) * 64.0;
    cost[s] = (double)waves * (rows + fixed_rows) + (s > 1 ? merge_rows_per_split * s : 0.0);
    if (cost[s] < best) best = cost[s];
  }
  for (int s = 1; s <= max_s; ++s)
    if (cost[s] <= best * 1.02) return s;
  return 1;
}

int tmla_select_kernel(const TmlaDecodeParams* p) {
  int rc = validate(p);
  if (rc) return -rc;
  return select_kernel(*p);
}

int tmla_decode_partial(const TmlaDecodeParams* p, void* stream) {
  int rc = validate(p);
  if (rc) return rc;
  if (p->batch == 0) return TMLA_OK;
  if (!p->ws_o || !p->ws_lse) return TMLA_ERR_WORKSPACE;
  // Stage 1 alone always produces partials, also for a single split.
  TmlaDecodeParams q = *p;
  q.flags |= TMLA_FLAG_PARTIAL_ONLY;
  return run_partial(q, static_cast<cudaStream_t>(stream));
}

int tmla_combine(const float* ws_o, const float* ws_lse, void* out, int64_t out_stride_b, int64_t out_stride_h,
                 float* lse, int64_t lse_stride_b, int32_t batch, int32_t num_heads, int32_t num_splits, int32_t d_v,
                 int32_t dtype, void* stream) {
  if (batch < 0 || num_heads <= 0 || num_splits <= 0 || d_v <= 0) return TMLA_ERR_INVALID_ARG;
  if (batch == 0) return TMLA_OK;
  if (!ws_o || !ws_lse || !out) return TMLA_ERR_INVALID_ARG;
  return finish(tmla::launch_combine(ws_o, ws_lse, out, out_stride_b, out_stride_h, lse, lse_stride_b, batch,
                                     num_heads, num_splits, d_v, dtype, false, static_cast<cudaStream_t>(stream)));
}

int tmla_decode(const TmlaDecodeParams* p, void* stream) {
  if (!p) return TMLA_ERR_INVALID_ARG;
  // A whole decode: the stage-1-only flag does not apply (with one split it would ask for a
  // workspace the call does not need).
  TmlaDecodeParams q = *p;
  q.flags &= ~TMLA_FLAG_PARTIAL_ONLY;
  int rc = validate(&q);
  if (rc) return rc;
  if (q.batch == 0) return TMLA_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Between its two stages this call owns the workspace, so the tcgen05 kernel hands the merge
  // its partials in the q dtype (half the bytes to store and read back); the generic kernel's
  // are fp32, and tmla_decode_partial / tmla_combine keep the documented fp32 layout.
  const bool part16 = q.num_splits > 1 && select_kernel(q) == TMLA_KERNEL_SM100;
  rc = run_partial(q, s, part16);
  if (rc) return rc;
  if (q.num_splits == 1) return TMLA_OK;
  return finish(tmla::launch_combine(q.ws_o, q.ws_lse, q.out, q.out_stride_b, q.out_stride_h, q.lse, q.lse_stride_b,
                                     q.batch, q.num_heads, q.num_splits, q.d_v, q.dtype, part16, s));
}

// ---------------------------------------------------------------- per-request split plan
// Costs in units of "one 2-CTA cluster streaming one 64-token tile": a work unit costs its
// tiles plus a fixed start-up / epilogue cost, plus the write and read-back of its fp32
// partial when its request is split.
namespace {
constexpr double kUnitFixedTiles = 8.0;
constexpr double kUnitMergeTiles = 2.0;
constexpr int kMaxSplitsPerRequest = 64;

double lpt_makespan(std::vector<double>& costs, int machines) {
  std::sort(costs.begin(), costs.end(), std::greater<double>());
  std::priority_queue<double, std::vector<double>, std::greater<double>> load;
  for (int i = 0; i < machines; ++i) load.push(0.0);
  double span = 0.0;
  for (double c : costs) {
    double l = load.top() + c;
    load.pop();
    load.push(l);
    span = std::max(span, l);
  }
  return span;
}
}  // namespace

int32_t tmla_plan_units(const int32_t* seqlens, int32_t batch, int32_t num_heads, int32_t num_sms, int32_t max_units,
                        int32_t* units, int32_t* req_first) {
  if (!seqlens || batch < 0 || num_heads <= 0 || max_units < 0 || !req_first || (batch > 0 && !units))
    return -TMLA_ERR_INVALID_ARG;
  req_first[0] = 0;
  if (batch == 0) return 0;
  if (num_sms <= 0) num_sms = 148;
  const int head_tiles = (num_heads + 127) / 128;
  const int machines = std::max(1, num_sms / 2 / head_tiles);  // units running at once
  std::vector<int> tiles(batch);
  int max_tiles = 0;
  for (int b = 0; b < batch; ++b) {
    tiles[b] = seqlens[b] > 0 ? (seqlens[b] + 63) / 64 : 0;
    max_tiles = std::max(max_tiles, tiles[b]);
  }
  // Candidate targets: the longest request cut into k equal parts, k = 1 .. 64.
  int best_target = std::max(1, max_tiles);
  double best_span = INFINITY;
  long best_units = 0;
  std::vector<double> costs;
  for (int k = 1; k <= kMaxSplitsPerRequest; ++k) {
    const int target = std::max(1, (max_tiles + k - 1) / k);
    if (k > 1 && target == (max_tiles + k - 2) / (k - 1)) continue;  // same target as k - 1
    costs.clear();
    long n = 0;
    for (int b = 0; b < batch; ++b) {
      const int ns = std::min(kMaxSplitsPerRequest, std::max(1, (tiles[b] + target - 1) / target));
      const int per = (tiles[b] + ns - 1) / ns;
      for (int s = 0; s < ns; ++s) costs.push_back(per + kUnitFixedTiles + (ns > 1 ? kUnitMergeTiles : 0.0));
      n += ns;
    }
    if (n > max_units) continue;
    const double span = lpt_makespan(costs, machines);
    if (span < best_span * (1.0 - 1e-9) || (span <= best_span * (1.0 + 1e-9) && n < best_units)) {
      best_span = span;
      best_target = target;
      best_units = n;
    }
  }
  if (best_units == 0) return -TMLA_ERR_INVALID_ARG;  // max_units too small for one unit per request
  // Emit the plan: slots per request in request order, units longest first.
  struct Unit {
    int b, split, ns, slot, per;
  };
  std::vector<Unit> plan;
  plan.reserve(best_units);
  int slot = 0;
  for (int b = 0; b < batch; ++b) {
    const int ns = std::min(kMaxSplitsPerRequest, std::max(1, (tiles[b] + best_target - 1) / best_target));
    const int per = (tiles[b] + ns - 1) / ns;
    for (int s = 0; s < ns; ++s) {
      const int first_tile = std::min(tiles[b], s * per);
      const int mine = std::min(tiles[b], first_tile + per) - first_tile;
      plan.push_back({b, s, ns, ns > 1 ? slot + s : -1, mine});
    }
    if (ns > 1) slot += ns;
    req_first[b + 1] = slot;
  }
  std::stable_sort(plan.begin(), plan.end(), [](const Unit& a, const Unit& c) { return a.per > c.per; });
  for (size_t u = 0; u < plan.size(); ++u) {
    units[4 * u] = plan[u].b;
    units[4 * u + 1] = plan[u].split;
    units[4 * u + 2] = plan[u].ns;
    units[4 * u + 3] = plan[u].slot;
  }
  return (int32_t)plan.size();
}

size_t tmla_units_workspace_bytes(int32_t num_slots, int32_t num_heads, int32_t d_v) {
  if (num_slots <= 0 || num_heads <= 0 || d_v <= 0) return 0;
  const size_t o = (((size_t)num_slots * num_heads * d_v * sizeof(float)) + 255) & ~(size_t)255;
  const size_t l = (((size_t)num_slots * num_heads * sizeof(float)) + 255) & ~(size_t)255;
  return o + l;
}

int tmla_decode_units(const TmlaDecodeParams* p, const int32_t* units, const int32_t* req_first, int32_t num_units,
                      int32_t num_slots, void* stream) {
  if (!p) return TMLA_ERR_INVALID_ARG;
  TmlaDecodeParams q = *p;
  q.num_splits = 1;
  q.flags &= ~TMLA_FLAG_PARTIAL_ONLY;
  int rc = validate(&q);
  if (rc) return rc;
  if (q.batch == 0) return TMLA_OK;
  if (!units || !req_first || num_units < q.batch || num_units > 65535 || num_slots < 0) return TMLA_ERR_INVALID_ARG;
  if (num_slots > 0 && (!q.ws_o || !q.ws_lse)) return TMLA_ERR_WORKSPACE;
  if (q.kernel == TMLA_KERNEL_GENERIC || !tmla::sm100_supported(q)) return TMLA_ERR_UNSUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The slots' partials are in the q dtype (the workspace is this call's own, as in tmla_decode).
  rc = finish(tmla::launch_sm100(q, s, units, num_units, num_slots, true));
  if (rc || num_slots == 0) return rc;
  return finish(tmla::launch_combine_slots(q.ws_o, q.ws_lse, req_first, q.out, q.out_stride_b, q.out_stride_h, q.lse,
                                           q.lse_stride_b, q.batch, q.num_heads, q.d_v, q.dtype, true, s));
}

}  // extern "C"

