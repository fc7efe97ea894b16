// tcgen05 split-KV MLA decode for B200: the two kernel variants and their host launch.
// The kernel itself (its design, warp roles and waits) is in tmla_sm100_kernel.cuh.
//
// Replaces the reference's `_mla_decode_stage1` (src/triton_mla/kernel.py:43-138) for its
// DeepSeek shape (d_qk 576 = 512 latent + 64 RoPE, d_v 512, bf16/fp16 queries).

// Caches of 16-bit rows (the q dtype).
#define TMLA_SM100_NS sm100
#define TMLA_SM100_FP8 0
#include "tmla_sm100_kernel.cuh"
#undef TMLA_SM100_NS
#undef TMLA_SM100_FP8

// Caches of 656-byte FP8 rows (TMLA_KV_FP8_E4M3), dequantised in shared memory.
#define TMLA_SM100_NS sm100_fp8
#define TMLA_SM100_FP8 1
#include "tmla_sm100_kernel.cuh"
#undef TMLA_SM100_NS
#undef TMLA_SM100_FP8

namespace tmla {
namespace sm100 {

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

// The split partials ws_o [batch, heads, splits, 512] as a 4-D map with boxes of 128 bytes of
// columns (32 fp32 or 64 16-bit) x 1 split x 128 heads x 1 request.  part_dt: the element type
// (fp32, or the q dtype when tmla_decode hands the partials to its own merge).
static int encode_partials(CUtensorMap* map, void* ws_o, int batch, int heads, int splits, CUtensorMapDataType part_dt) {
  auto fn = encode_fn();
  if (!fn) return TMLA_ERR_CUDA;
  const cuuint64_t e = part_dt == CU_TENSOR_MAP_DATA_TYPE_FLOAT32 ? 4 : 2;
  cuuint64_t dims[4] = {512, (cuuint64_t)splits, (cuuint64_t)heads, (cuuint64_t)batch};
  cuuint64_t strides[3] = {512 * e, (cuuint64_t)splits * 512 * e, (cuuint64_t)heads * splits * 512 * e};
  cuuint32_t box[4] = {(cuuint32_t)(128 / e), 1, 128, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, part_dt, 4, ws_o, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : TMLA_ERR_MISALIGNED;
}

// The partials of a per-request split plan, ws_o [slots, heads, 512], as a 3-D map with boxes of
// 128 bytes of columns x 128 heads x 1 slot (element type as for encode_partials).
static int encode_slot_partials(CUtensorMap* map, void* ws_o, int slots, int heads, CUtensorMapDataType part_dt) {
  auto fn = encode_fn();
  if (!fn) return TMLA_ERR_CUDA;
  const cuuint64_t e = part_dt == CU_TENSOR_MAP_DATA_TYPE_FLOAT32 ? 4 : 2;
  cuuint64_t dims[3] = {512, (cuuint64_t)heads, (cuuint64_t)slots};
  cuuint64_t strides[2] = {512 * e, (cuuint64_t)heads * 512 * e};
  cuuint32_t box[3] = {(cuuint32_t)(128 / e), 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, part_dt, 3, ws_o, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : TMLA_ERR_MISALIGNED;
}

// Token rows per TMA box: the largest power of two <= kTile dividing the page size.
static int pow2_rows(int page) {
  int g = 64;
  while (g > 1 && page % g) g >>= 1;
  return g;
}

}  // namespace sm100

int sm100_supported(const TmlaDecodeParams& p) {
  if (p.d_qk != 576 || p.d_v != 512) return 0;
  if (p.kv_format != TMLA_KV_SAME && p.kv_format != TMLA_KV_FP8_E4M3) return 0;
  if (p.dtype != TMLA_DTYPE_BF16 && p.dtype != TMLA_DTYPE_FP16) return 0;
  if (p.batch > 65535 || p.num_splits > 65535) return 0;
  if (((uintptr_t)p.q | (uintptr_t)p.kv) % 16) return 0;
  if (p.q_stride_b % 8 || p.q_stride_h % 8) return 0;
  // Row strides in elements of the cache: 16-bit values, or bytes of FP8 rows (TMA: 16-byte multiples).
  const int64_t sm = p.kv_format == TMLA_KV_FP8_E4M3 ? 16 : 8;
  if (p.kv_stride_page % sm || p.kv_stride_tok % sm) return 0;
  if ((uintptr_t)p.out % 16 || p.out_stride_b % 8 || p.out_stride_h % 8) return 0;
  if (p.block_table && sm100::pow2_rows(p.page_size) < 8) return 0;
  if (p.q_len > 1 && (p.num_heads / p.q_len) % 128) return 0;  // a head tile within one query token
  return 1;
}

int launch_sm100(const TmlaDecodeParams& p, cudaStream_t stream, const int32_t* units, int32_t num_units,
                 int32_t num_slots, bool part16) {
  using namespace sm100;
  if (!sm100_supported(p)) return TMLA_ERR_UNSUPPORTED;
  const CUtensorMapDataType dt =
      p.dtype == TMLA_DTYPE_FP16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const bool fp8 = p.kv_format == TMLA_KV_FP8_E4M3;
  const int g = p.block_table ? pow2_rows(p.page_size) : kTile;
  const uint64_t pages = p.block_table ? (uint64_t)p.num_pages : (uint64_t)p.batch;
  CUtensorMap tm_lat, tm_rope, tm_scale, tm_q, tm_qlat, tm_out, tm_part;
  memset(&tm_scale, 0, sizeof(tm_scale));
  memset(&tm_out, 0, sizeof(tm_out));
  memset(&tm_part, 0, sizeof(tm_part));
  int rc;
  if (fp8) {
    // FP8 rows (656 bytes): the e4m3 latent values as 128-byte swizzled boxes (two per CTA half),
    // the scale quadruple (bytes 512-527), and the RoPE half as bf16 elements 264-327.
    const uint64_t st = (uint64_t)p.kv_stride_tok, sp = (uint64_t)p.kv_stride_page;
    rc = encode3d(&tm_lat, CU_TENSOR_MAP_DATA_TYPE_UINT8, p.kv, sm100_fp8::kFp8Row, (uint64_t)p.page_size, pages, st,
                  sp, 128, (uint32_t)g, CU_TENSOR_MAP_SWIZZLE_128B);
    if (!rc)
      rc = encode3d(&tm_scale, CU_TENSOR_MAP_DATA_TYPE_UINT8, p.kv, sm100_fp8::kFp8Row, (uint64_t)p.page_size, pages,
                    st, sp, 16, (uint32_t)g, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (!rc)
      rc = encode3d(&tm_rope, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, p.kv, sm100_fp8::kFp8Row / 2, (uint64_t)p.page_size,
                    pages, st, sp, kHalfRope, (uint32_t)g, CU_TENSOR_MAP_SWIZZLE_64B);
  } else {
    rc = encode3d(&tm_lat, dt, p.kv, 576, (uint64_t)p.page_size, pages, (uint64_t)p.kv_stride_tok * 2,
                  (uint64_t)p.kv_stride_page * 2, 64, (uint32_t)g, CU_TENSOR_MAP_SWIZZLE_128B);
    if (!rc)
      rc = encode3d(&tm_rope, dt, p.kv, 576, (uint64_t)p.page_size, pages, (uint64_t)p.kv_stride_tok * 2,
                    (uint64_t)p.kv_stride_page * 2, kHalfRope, (uint32_t)g, CU_TENSOR_MAP_SWIZZLE_64B);
  }
  if (!rc)
    rc = encode3d(&tm_q, dt, p.q, 576, (uint64_t)p.num_heads, (uint64_t)p.batch, (uint64_t)p.q_stride_h * 2,
                  (uint64_t)p.q_stride_b * 2, kHalfRope, 128, CU_TENSOR_MAP_SWIZZLE_64B);
  if (!rc)
    rc = encode3d(&tm_qlat, dt, p.q, 576, (uint64_t)p.num_heads, (uint64_t)p.batch, (uint64_t)p.q_stride_h * 2,
                  (uint64_t)p.q_stride_b * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B);
  // The final 16-bit output (one split) and the partials (several; fp32, or 16-bit with
  // part16) as tensor maps; a plan of per-request splits can need both in one launch.
  const bool any_final = units ? num_slots < num_units : (p.num_splits == 1 && !(p.flags & TMLA_FLAG_PARTIAL_ONLY));
  const bool any_part = units ? num_slots > 0 : !any_final;
  if (!rc && any_final)
    rc = encode3d(&tm_out, dt, p.out, 512, (uint64_t)p.num_heads, (uint64_t)p.batch, (uint64_t)p.out_stride_h * 2,
                  (uint64_t)p.out_stride_b * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc && any_part) {
    const CUtensorMapDataType part_dt = part16 ? dt : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    rc = units ? encode_slot_partials(&tm_part, p.ws_o, num_slots, p.num_heads, part_dt)
               : encode_partials(&tm_part, p.ws_o, p.batch, p.num_heads, p.num_splits, part_dt);
  }
  if (rc) return rc;
  KernelArgs a;
  a.p = p;
  a.rows_per_load = g;
  a.scale_log2 = p.softmax_scale * kLog2e;
  a.units = reinterpret_cast<const int4*>(units);
  a.wait_ns = p.wait_ns > 0 ? (uint64_t)p.wait_ns : kWaitNs;
  a.stall = (p.flags & TMLA_FLAG_TEST_STALL) ? 1 : 0;
  const dim3 grid(2 * ((p.num_heads + 127) / 128), units ? 1 : p.num_splits, units ? num_units : p.batch);
  // A programmatic dependent of the preceding kernel in the stream: the CTAs may be placed
  // while that kernel finishes, and every read of an input follows griddep_wait().
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = grid;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  auto launch = [&](auto kernel, uint32_t threads, uint32_t smem) {
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err == cudaSuccess)
      err = cudaLaunchKernelEx(&cfg, kernel, tm_lat, tm_rope, tm_scale, tm_out, tm_part, tm_q, tm_qlat, a);
    return err;
  };
  cudaError_t e;
  if (fp8) {
    namespace v = sm100_fp8;
    if (p.dtype == TMLA_DTYPE_FP16)
      e = part16 ? launch(v::mla_sm100_split_kernel<__half, true>, v::kThreads, v::kSmemBytes)
                 : launch(v::mla_sm100_split_kernel<__half, false>, v::kThreads, v::kSmemBytes);
    else
      e = part16 ? launch(v::mla_sm100_split_kernel<__nv_bfloat16, true>, v::kThreads, v::kSmemBytes)
                 : launch(v::mla_sm100_split_kernel<__nv_bfloat16, false>, v::kThreads, v::kSmemBytes);
  } else {
    if (p.dtype == TMLA_DTYPE_FP16)
      e = part16 ? launch(mla_sm100_split_kernel<__half, true>, kThreads, kSmemBytes)
                 : launch(mla_sm100_split_kernel<__half, false>, kThreads, kSmemBytes);
    else
      e = part16 ? launch(mla_sm100_split_kernel<__nv_bfloat16, true>, kThreads, kSmemBytes)
                 : launch(mla_sm100_split_kernel<__nv_bfloat16, false>, kThreads, kSmemBytes);
  }
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? 0 : -(int)e;
}

}  // namespace tmla
