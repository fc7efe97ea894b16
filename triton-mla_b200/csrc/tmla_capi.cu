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

#include "tmla_common.cuh"

namespace tmla {
int launch_generic(const TmlaDecodeParams& p, cudaStream_t stream);
int launch_combine(const float* ws_o, const float* ws_lse, void* out, int64_t osb, int64_t osh, float* lse,
                   int64_t lsb, int B, int H, int S, int DV, int dtype, cudaStream_t stream);
int sm100_supported(const TmlaDecodeParams& p);
int launch_sm100(const TmlaDecodeParams& p, cudaStream_t stream);
}  // namespace tmla

namespace {

thread_local char g_cuda_error[256] = "";

int cuda_fail(int neg_code) {
  cudaError_t e = (cudaError_t)(-neg_code);
  snprintf(g_cuda_error, sizeof(g_cuda_error), "%s: %s", cudaGetErrorName(e), cudaGetErrorString(e));
  return TMLA_ERR_CUDA;
}

// Launch helpers return 0, a positive TMLA_ERR_* code or minus a cudaError_t.
int finish(int rc) { return rc < 0 ? cuda_fail(rc) : rc; }

bool is_pow2(int v) { return v > 0 && (v & (v - 1)) == 0; }

int validate(const TmlaDecodeParams* p) {
  if (!p) return TMLA_ERR_INVALID_ARG;
  if (p->batch < 0 || p->num_heads <= 0 || p->num_splits <= 0) return TMLA_ERR_INVALID_ARG;
  if (p->d_v <= 0 || p->d_qk <= p->d_v) return TMLA_ERR_INVALID_ARG;
  if (!is_pow2(p->d_v) || !is_pow2(p->d_qk - p->d_v)) return TMLA_ERR_INVALID_ARG;
  if (p->dtype != TMLA_DTYPE_BF16 && p->dtype != TMLA_DTYPE_FP16 && p->dtype != TMLA_DTYPE_FP32)
    return TMLA_ERR_INVALID_ARG;
  if (p->page_size <= 0) return TMLA_ERR_INVALID_ARG;
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

int run_partial(const TmlaDecodeParams& p, cudaStream_t stream) {
  const int k = select_kernel(p);
  if (k < 0) return -k;
  if (k == TMLA_KERNEL_SM100) return finish(tmla::launch_sm100(p, stream));
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
//   waves(s) * (rows per split + fixed cost per unit) + merge traffic(s)
// where the merge traffic (fp32 partials written then read back, 2 x 4 bytes
// x 512 columns per head and split) is spread over all clusters.  The
// smallest split count within 2% of the best estimate wins.
int32_t tmla_num_splits(int32_t batch, int32_t num_heads, int32_t max_seqlen, int32_t num_sms) {
  if (batch <= 0 || num_heads <= 0 || max_seqlen <= 0) return 1;
  if (num_sms <= 0) num_sms = 148;
  const int clusters = num_sms / 2 > 0 ? num_sms / 2 : 1;
  const long units = (long)batch * ((num_heads + 127) / 128);
  const int tiles = (max_seqlen + 63) / 64;
  const int max_s = tiles < 64 ? tiles : 64;
  const double fixed_rows = 256.0;
  const double merge_rows_per_split = (double)batch * num_heads * 512.0 * 8.0 / (clusters * 1152.0);
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
                                     num_heads, num_splits, d_v, dtype, static_cast<cudaStream_t>(stream)));
}

int tmla_decode(const TmlaDecodeParams* p, void* stream) {
  int rc = validate(p);
  if (rc) return rc;
  if (p->batch == 0) return TMLA_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  TmlaDecodeParams q = *p;
  q.flags &= ~TMLA_FLAG_PARTIAL_ONLY;
  rc = run_partial(q, s);
  if (rc) return rc;
  if (p->num_splits == 1) return TMLA_OK;
  return tmla_combine(p->ws_o, p->ws_lse, p->out, p->out_stride_b, p->out_stride_h, p->lse, p->lse_stride_b,
                      p->batch, p->num_heads, p->num_splits, p->d_v, p->dtype, stream);
}

}  // extern "C"
