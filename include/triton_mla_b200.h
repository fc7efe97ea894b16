/*
 * triton_mla_b200.h — C ABI of the B200 (sm_100a) MLA single-token decode library.
 *
 * This is the drop-in boundary for the hot path of luvadlamudi/triton-mla.
 * The reference exposes the path as the Python function
 * `triton_mla.mla_decode` (src/triton_mla/kernel.py:204-323), which launches
 * two Triton kernels: `_mla_decode_stage1` (kernel.py:43-138, split-KV partial
 * attention) and `_mla_decode_stage2` (kernel.py:141-181, log-sum-exp merge),
 * after picking a split count with `get_num_splits` (kernel.py:190-201).
 * Each entry point below replaces one of those pieces; the Python package
 * `triton_mla` (triton-mla_b200/triton_mla/) binds them with ctypes.
 *
 * Conventions
 *  - Plain pointers and sizes only.  All tensor pointers are DEVICE pointers of
 *    the current CUDA device; strides are in ELEMENTS; the innermost dimension
 *    of q, kv_cache and out is contiguous (stride 1), as the reference asserts
 *    (kernel.py:241).
 *  - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *  - Every function returns 0 on success or a TMLA_ERR_* code; nothing is
 *    allocated or freed by the library except where noted (it never calls
 *    cudaMalloc).  Launches are asynchronous; device-side faults of the
 *    input (a block-table entry outside [0, num_pages), a bounded wait that
 *    timed out) are reported through the optional `status` word, never by
 *    trapping.
 */
#ifndef TRITON_MLA_B200_H
#define TRITON_MLA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TMLA_ABI_VERSION 4

/* Return codes. */
#define TMLA_OK 0
#define TMLA_ERR_INVALID_ARG 1     /* shape / stride / dtype rule broken (reference: AssertionError) */
#define TMLA_ERR_UNSUPPORTED 2     /* a configuration this build does not implement */
#define TMLA_ERR_MISALIGNED 3      /* a pointer or stride breaks the 16-byte TMA rule */
#define TMLA_ERR_CUDA 4            /* a CUDA runtime/driver call failed; see tmla_last_cuda_error() */
#define TMLA_ERR_WORKSPACE 5       /* workspace missing or too small */

/* Largest batch and split count of one decode call (a grid dimension's limit). */
#define TMLA_MAX_BATCH 65535

/* Bits of the device status word (OR-ed by kernels). */
#define TMLA_STATUS_BAD_PAGE 0x1   /* a block-table entry was outside [0, num_pages); its tokens were masked */
#define TMLA_STATUS_TIMEOUT 0x2    /* a bounded pipeline wait gave up; the result is invalid */
#define TMLA_STATUS_RANGE 0x4      /* FP8 rows on the tcgen05 kernel, whose latent products are fp16: a query
                                      value, a RoPE value or a row scale (times 448, the largest e4m3
                                      value) was beyond the fp16 range; those rows may hold inf / NaN
                                      (TMLA_KERNEL_GENERIC computes such rows in fp32) */

/* Element types of q / kv_cache / out. */
#define TMLA_DTYPE_BF16 0
#define TMLA_DTYPE_FP16 1
#define TMLA_DTYPE_FP32 2          /* generic kernel only */

/* Kernel selection for tmla_decode / tmla_decode_partial. */
#define TMLA_KERNEL_AUTO 0         /* tcgen05 kernel when the shape allows it, else the generic kernel */
#define TMLA_KERNEL_GENERIC 1      /* CUDA-core split-KV kernel: any power-of-two head_dim_v / rope dim */
#define TMLA_KERNEL_SM100 2        /* TMA + tcgen05 + TMEM kernel: d_qk 576, d_v 512, 16-bit q, 16-bit or FP8 rows */

/* Flags. */
#define TMLA_FLAG_PARTIAL_ONLY 0x1  /* write ws_o / ws_lse even when num_splits == 1 (stage-1 semantics) */
/* Tests of the timeout path only (tcgen05 kernel): the first cluster's first CTA never loads its
   first cache tile, so its waits run out after wait_ns; the call sets TMLA_STATUS_TIMEOUT and
   returns normally, with the rows of that cluster invalid. */
#define TMLA_FLAG_TEST_STALL 0x100

/* Cache row formats (TmlaDecodeParams.kv_format).
   TMLA_KV_SAME: d_qk values of the q dtype per token.
   TMLA_KV_FP8_E4M3: 656 bytes per token (d_qk 576, d_v 512): 512 float8 e4m3 latent values,
   4 fp32 scales (scale i multiplies latent values 128 i .. 128 i + 127), then the 64 RoPE
   values in bf16.  The kv strides count bytes.  q and out are bf16 or fp16.  The tcgen05
   kernel (16-byte aligned rows and strides) dequantises each tile in shared memory and forms
   the latent products in fp16 (value = e4m3 x scale rounded to fp16 once, relative error
   <= 2^-11; queries converted to fp16), flagging TMLA_STATUS_RANGE for values beyond fp16;
   the CUDA-core kernel computes in fp32.  The reference has no FP8 cache; the layout is the
   public 656-byte FP8 MLA cache row of FlashMLA (DeepSeek-V3.2). */
#define TMLA_KV_SAME 0
#define TMLA_KV_FP8_E4M3 1

typedef struct TmlaDecodeParams {
  /* q [batch, num_heads, d_qk]: absorbed nope query (first d_v dims) then the RoPE query.
     With q_len > 1 (several new tokens per request, e.g. multi-token prediction) the
     num_heads rows are q_len groups of num_heads / q_len heads, one group per token, and
     row group i attends causally: to the first seqlens[b] - (q_len - 1 - i) cache rows. */
  const void* q;
  int64_t q_stride_b, q_stride_h;

  /* kv_cache: paged [num_pages, page_size, d_qk] when block_table != NULL,
     otherwise dense [batch, page_size (= capacity), d_qk] with num_pages = batch. */
  const void* kv;
  int64_t kv_stride_page, kv_stride_tok;
  int64_t num_pages;
  int32_t page_size;

  const int32_t* seqlens;          /* [batch] valid tokens per request */
  const int32_t* block_table;      /* [batch, bt_width] page ids, or NULL for dense */
  int64_t bt_stride;               /* row stride of block_table */
  int32_t bt_width;                /* pages per row (entries beyond are never read) */

  void* out;                       /* [batch, num_heads, d_v] in the q dtype */
  int64_t out_stride_b, out_stride_h;
  float* lse;                      /* [batch, num_heads] fp32 natural-log LSE, or NULL */
  int64_t lse_stride_b;

  /* Split workspace (only read when num_splits > 1):
     ws_o [batch, num_heads, num_splits, d_v] fp32 partial outputs (normalised),
     ws_lse [batch, num_heads, num_splits] fp32 base-2 partial LSE.
     This is the layout tmla_decode_partial writes and tmla_combine reads.  Within one
     tmla_decode (or tmla_decode_units) call the workspace is the call's own: on the tcgen05
     kernel the partials there are in the q dtype (16-bit, the first half of ws_o's bytes),
     which halves what the split kernel stores and the merge reads back. */
  float* ws_o;
  float* ws_lse;

  int32_t* status;                 /* optional device status word (TMLA_STATUS_* bits), or NULL */

  /* batch and num_splits are at most TMLA_MAX_BATCH: larger values give TMLA_ERR_UNSUPPORTED
     (decode such a batch as several calls).  The reference's Triton grid has no such limit. */
  int32_t batch, num_heads, d_qk, d_v, num_splits;
  int32_t dtype;                   /* TMLA_DTYPE_* */
  int32_t kernel;                  /* TMLA_KERNEL_* */
  int32_t flags;                   /* TMLA_FLAG_* bits */
  float softmax_scale;
  int32_t q_len;                   /* query tokens per request (0 or 1: one); divides num_heads */
  int32_t kv_format;               /* TMLA_KV_*: the cache row format */
  /* Limit of each pipeline wait of the tcgen05 kernel in nanoseconds (<= 0: 2 s).  A wait that
     runs out sets TMLA_STATUS_TIMEOUT; the kernel stops, lets its copies and MMAs finish and
     returns, and the device stays usable. */
  int64_t wait_ns;
} TmlaDecodeParams;

/* Whole decode: partial attention over num_splits KV ranges, then the merge.
   Replaces `mla_decode` (kernel.py:204-323) after its host-side validation.
   TMLA_FLAG_PARTIAL_ONLY is ignored (it is stage-1 semantics, tmla_decode_partial). */
int tmla_decode(const TmlaDecodeParams* p, void* stream);

/* Whole decode without any allocation.  No counterpart in the reference: it is
   for callers that cannot allocate device memory (an FFI host without a device
   allocator of its own, or a serving loop that must not call cudaMalloc, which
   can synchronise the device).  Same as tmla_decode except that p->ws_o and
   p->ws_lse are ignored: the split partials go to a fixed array of
   TMLA_NOALLOC_SCRATCH_BYTES of device memory that the library holds on every
   GPU that loads it, until exit.  A call needing more workspace than that
   (tmla_workspace_bytes) returns TMLA_ERR_WORKSPACE; num_splits == 1 needs none.
   The first call on a device looks up the array's device address (make it
   before any stream capture); the address is cached for the life of the process,
   so after a cudaDeviceReset this entry point must not be called again.
   TMLA_FLAG_PARTIAL_ONLY is ignored, as in tmla_decode.  All calls share the array: calls that can
   overlap on the GPU (different streams or host threads) race on it; calls on
   one stream are safe.  Allocates nothing (no cudaMalloc / cudaFree). */
#define TMLA_NOALLOC_SCRATCH_BYTES (32u << 20)
int tmla_decode_noalloc(const TmlaDecodeParams* p, void* stream);

/* Per-request split plan for ragged batches.  No counterpart in the reference, whose split
   count is one number for the whole batch (kernel.py:190-201, 264-266).  From the request
   lengths (host memory) it picks how many splits each request gets, so that the tcgen05
   kernel's 2-CTA clusters, scheduled longest unit first, finish together: it simulates
   longest-first scheduling of each candidate plan on num_sms / 2 clusters and keeps the
   shortest.  Output, for up to max_units work units (batch * 64 always suffices):
     units[4u .. 4u+3] = {request, split, splits of that request, partial slot or -1},
     longest unit first; a request with one split has slot -1 and writes its output itself;
     req_first[b] = first partial slot of request b, req_first[batch] = slots in all.
   Returns the number of units, or -TMLA_ERR_INVALID_ARG.  Host-only: touches no GPU. */
int32_t tmla_plan_units(const int32_t* seqlens, int32_t batch, int32_t num_heads, int32_t num_sms,
                        int32_t max_units, int32_t* units, int32_t* req_first);

/* Workspace of a plan with num_slots partial slots: room for ws_o = [num_slots, num_heads, d_v]
   fp32 at its start (tmla_decode_units keeps its partials there in the q dtype), and
   ws_lse = [num_slots, num_heads] fp32 at the next 256-byte boundary. */
size_t tmla_units_workspace_bytes(int32_t num_slots, int32_t num_heads, int32_t d_v);

/* Whole decode following a plan from tmla_plan_units (units and req_first copied to device
   memory; p->num_splits is ignored): one cluster per unit and head tile, then the merge of
   the split requests.  tcgen05 kernel only (TMLA_ERR_UNSUPPORTED for other shapes).  No
   counterpart in the reference (see tmla_plan_units). */
int tmla_decode_units(const TmlaDecodeParams* p, const int32_t* units, const int32_t* req_first,
                      int32_t num_units, int32_t num_slots, void* stream);

/* Per-request split plan computed on the GPU, in `stream`, from the lengths in device memory
   (no host sync; a plan kernel, tmla_decode_units and its merge can be captured in one CUDA
   graph and replayed as the lengths change).  Writes `capacity` units (device int4
   [capacity]) and req_first (device int32 [batch + 1]) in the layout of tmla_plan_units;
   entries past the plan's own units are {-1, 0, 0, -1}, and their clusters exit at once.
   The plan uses at most `slot_capacity` partial slots.  Pass num_units = capacity and
   num_slots = slot_capacity to tmla_decode_units (workspace: tmla_units_workspace_bytes of
   slot_capacity).  Requires batch <= capacity <= 65535.  The reference has no counterpart:
   its num_splits=None reads max(cache_seqlens) on the host (kernel.py:264-266). */
int tmla_plan_units_device(const int32_t* seqlens, int32_t batch, int32_t num_heads, int32_t num_sms,
                           int32_t capacity, int32_t slot_capacity, int32_t* units, int32_t* req_first,
                           void* stream);

/* Stage 1 only: writes ws_o / ws_lse for every (request, head, split).
   Replaces the `_mla_decode_stage1` launch (kernel.py:276-302). */
int tmla_decode_partial(const TmlaDecodeParams* p, void* stream);

/* Stage 2 only: merges ws_o / ws_lse into out (q dtype) and lse (natural log).
   Replaces the `_mla_decode_stage2` launch (kernel.py:303-320). */
int tmla_combine(const float* ws_o, const float* ws_lse, void* out, int64_t out_stride_b,
                 int64_t out_stride_h, float* lse, int64_t lse_stride_b, int32_t batch,
                 int32_t num_heads, int32_t num_splits, int32_t d_v, int32_t dtype, void* stream);

/* Split count for a batch.  Replaces `get_num_splits` (kernel.py:190-201) with
   a B200 rule keyed on batch, heads, longest request and SM count. */
int32_t tmla_num_splits(int32_t batch, int32_t num_heads, int32_t max_seqlen, int32_t num_sms);

/* Bytes of split workspace tmla_decode needs (0 when num_splits == 1). */
size_t tmla_workspace_bytes(int32_t batch, int32_t num_heads, int32_t num_splits, int32_t d_v);

/* Which kernel TMLA_KERNEL_AUTO would choose for these parameters (TMLA_KERNEL_*),
   or a negative TMLA_ERR_* code if the parameters are invalid. */
int tmla_select_kernel(const TmlaDecodeParams* p);

/* Human-readable text of a return code; the CUDA error string of the last
   TMLA_ERR_CUDA on this thread; and the library's ABI version. */
const char* tmla_error_string(int code);
const char* tmla_last_cuda_error(void);
int tmla_abi_version(void);

/* sizeof(TmlaDecodeParams) as compiled, so an FFI binding can check its mirror of the struct. */
size_t tmla_params_bytes(void);

/* ---------------------------------------------------------------- MLA layer step, fused
   The small operations of one MLA layer decode step around the decode itself, one
   launch each (the reference runs them as PyTorch ops in MLA.forward,
   src/triton_mla/model.py:74-94 and 111-123).  dtype is TMLA_DTYPE_*; all tensors
   of one call share it.  w_kv_b is wkv_b.weight, [heads * (d_nope + d_v), rank]
   row-major: head h's W_UK is rows [h (d_nope + d_v), + d_nope), its W_UV the next
   d_v rows.  RoPE is the reference's half-split form at the given positions. */

/* q_out[b, h, :] = [ q_in[b, h, :d_nope] . W_UK[h]  |  rope(q_in[b, h, d_nope:], positions[b]) ]:
   the decode query from wq_b's output (model.py:111-113 with the q_pe RoPE of model.py:78).
   Needs rank even and w_kv_b 8-byte aligned (else TMLA_ERR_MISALIGNED); d_nope <= 512. */
/* Layer-op flag: launch as a programmatic dependent of the preceding kernel in the stream
   (its launch and the op's weight-tile loads overlap that kernel's end; every input other
   than the weights is read only after that kernel has completed).  Do not set it when the
   preceding kernel writes w_kv_b / norm_weight. */
#define TMLA_LAYER_FLAG_PDL 1

typedef struct TmlaQPrepParams {
  const void* q_in;                /* [batch, heads, d_nope + d_rope] */
  int64_t q_in_stride_b, q_in_stride_h;
  const void* w_kv_b;
  const int32_t* positions;        /* [batch]: the new token's position (cache length before the append) */
  void* q_out;                     /* [batch, heads, rank + d_rope] */
  int64_t q_out_stride_b, q_out_stride_h;
  int32_t batch, num_heads, d_nope, d_rope, d_v, rank;
  int32_t dtype;
  float rope_theta;
  int32_t flags;                   /* TMLA_LAYER_FLAG_* */
} TmlaQPrepParams;
int tmla_q_absorb_rope(const TmlaQPrepParams* p, void* stream);

/* The new token's cache row [ rmsnorm(kv_in[b, :rank]) * norm_weight | rope(kv_in[b, rank:]) ]
   written at position positions[b] of request b (paged through block_table, or dense
   [batch, page_size, rank + d_rope] when block_table is NULL), and seqlens_out[b] =
   positions[b] + 1 when seqlens_out is not NULL (model.py:74-94, 116-117).  A position
   past the cache or a page id outside the pool sets TMLA_STATUS_BAD_PAGE and drops the row.
   With q_in set, the same launch also writes q_out[b, :q_rank] = rmsnorm(q_in[b, :q_rank]) *
   q_norm_weight (q_norm of the query path, model.py:75): both down-projections of x come out
   of one GEMM, and its two halves are normalised here. */
typedef struct TmlaKvAppendParams {
  const void* kv_in;               /* [batch, rank + d_rope]: wkv_a's output */
  int64_t kv_in_stride_b;
  const void* norm_weight;         /* [rank] */
  const int32_t* positions;        /* [batch] */
  int32_t* seqlens_out;            /* [batch] or NULL */
  void* kv_cache;                  /* pages [num_pages, page_size, rank + d_rope] */
  int64_t kv_stride_page, kv_stride_tok, num_pages;
  int32_t page_size;
  const int32_t* block_table;      /* [batch, bt_width] or NULL */
  int64_t bt_stride;
  int32_t bt_width;
  int32_t* status;                 /* optional device status word */
  int32_t batch, rank, d_rope;
  int32_t dtype;
  float eps, rope_theta;
  int32_t flags;                   /* TMLA_LAYER_FLAG_* */
  const void* q_in;                /* [batch, q_rank] (row stride q_in_stride_b) or NULL */
  int64_t q_in_stride_b;
  const void* q_norm_weight;       /* [q_rank] */
  void* q_out;                     /* [batch, q_rank] (row stride q_out_stride_b) */
  int64_t q_out_stride_b;
  int32_t q_rank;
  float q_eps;
} TmlaKvAppendParams;
int tmla_kv_norm_rope_append(const TmlaKvAppendParams* p, void* stream);

/* out[b, h * d_v + d] = sum_c o[b, h, c] W_UV[h][d][c]: the decode output projected back per
   head, the input of wo (model.py:123).  Needs rank a multiple of 16 (<= 2048) and w_kv_b
   16-byte aligned (else TMLA_ERR_MISALIGNED).  Up to 64 requests of a 16-bit dtype with
   16-byte aligned o rows run on the projection kernel of tmla_linear (one group per head,
   tile-aligned, no workspace); others on a mma.sync / CUDA-core kernel. */
typedef struct TmlaOUnabsorbParams {
  const void* o;                   /* [batch, heads, rank]: mla_decode's output */
  int64_t o_stride_b, o_stride_h;
  const void* w_kv_b;
  void* out;                       /* [batch, heads * d_v] */
  int64_t out_stride_b;
  int32_t batch, num_heads, d_nope, d_v, rank;
  int32_t dtype;
  int32_t flags;                   /* TMLA_LAYER_FLAG_* */
} TmlaOUnabsorbParams;
int tmla_o_unabsorb(const TmlaOUnabsorbParams* p, void* stream);

/* L2 prefetch (no counterpart in the reference): brings count chunks of chunk_bytes at
   base + i * stride_bytes into L2, as bulk prefetches issued by ctas one-warp CTAs, and returns
   without waiting for them.  The layer step runs it on a side stream during the decode, which
   leaves HBM bandwidth and SMs idle, for the weights the products after the decode read (W_UV
   and the first part of wo).  base, chunk_bytes and stride_bytes must be multiples of 16
   (else TMLA_ERR_MISALIGNED); it reads nothing into the caller's memory and writes nothing. */
int tmla_l2_prefetch(const void* base, int64_t chunk_bytes, int64_t stride_bytes, int32_t count, int32_t ctas,
                     void* stream);

/* y[i, j] = sum_c x[i, c] w[j, c] for m <= 64 rows of x: a bias-free nn.Linear of a decode
   batch (replaces the cuBLAS GEMMs behind the reference layer's wq_a, wkv_a, wq_b and wo,
   model.py:104-108,124), streaming w once through tcgen05 MMAs on every SM.  With groups > 1
   the same product is taken for each group g over x + g * x_group_stride,
   w + g * w_group_stride and y + g * y_group_stride (per-head weights: the absorption
   einsums of model.py:111-113,123).  w is stored [n][k] (TMLA_W_NK, nn.Linear) or [k][n]
   (TMLA_W_KN) with rows w_stride apart.  Needs 16-bit x / w / y of one dtype; x and w
   16-byte aligned with row and group strides a multiple of 8 elements (else
   TMLA_ERR_MISALIGNED).  groups * ceil(n / 128) <= TMLA_LINEAR_MAX_TILES.  The workspace
   (tmla_linear_workspace_bytes, 16-byte aligned) starts with TMLA_LINEAR_MAX_TILES int32 tile
   counters, which must be zero before its first use; every call leaves them at zero again,
   also a call whose waits timed out (the partial sums after them need no initial value).
   Calls that may run at the same time (different streams) need separate workspaces.  With
   TMLA_LAYER_FLAG_PDL the weight loads may overlap the preceding kernel, which must not
   write w.  Every pipeline wait of the kernel gives up after wait_ns nanoseconds (<= 0: 2 s):
   the call then sets TMLA_STATUS_TIMEOUT in *status, leaves the output tiles of the CTAs that
   gave up unwritten, and returns normally (the device stays usable).
   TMLA_LINEAR_FLAG_TEST_STALL exists for tests of that path only: the first CTA never loads
   its first stage, so its waits run out after wait_ns. */
#define TMLA_W_NK 0
#define TMLA_W_KN 1
#define TMLA_LINEAR_MAX_TILES 65536
#define TMLA_LINEAR_FLAG_TEST_STALL 0x100
typedef struct TmlaLinearParams {
  const void* x;                   /* [m, k] per group */
  int64_t x_stride;
  const void* w;                   /* [n, k] or [k, n] per group */
  int64_t w_stride;
  void* y;                         /* [m, n] per group */
  int64_t y_stride;
  int32_t m, n, k;
  int32_t dtype;                   /* TMLA_DTYPE_BF16 or TMLA_DTYPE_FP16 */
  void* workspace;
  int64_t workspace_bytes;
  int32_t num_sms;                 /* CTAs to spread the weight over (<= 0: the device's SM count) */
  int32_t flags;                   /* TMLA_LAYER_FLAG_* */
  int32_t* status;                 /* optional device status word (TMLA_STATUS_TIMEOUT) */
  int32_t groups;                  /* >= 1 */
  int32_t w_layout;                /* TMLA_W_NK or TMLA_W_KN */
  int64_t x_group_stride, w_group_stride, y_group_stride;  /* elements; used when groups > 1 */
  int64_t wait_ns;                 /* limit of each pipeline wait (<= 0: 2 s) */
} TmlaLinearParams;
int tmla_linear(const TmlaLinearParams* p, void* stream);
/* Workspace bytes tmla_linear needs for this shape and SM count, or -TMLA_ERR_INVALID_ARG.
   Host-only. */
int64_t tmla_linear_workspace_bytes(int32_t m, int32_t n, int32_t k, int32_t groups, int32_t num_sms);

#ifdef __cplusplus
}
#endif

#endif /* TRITON_MLA_B200_H */
