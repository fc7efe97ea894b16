// Shared device helpers of the B200 MLA decode library.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "triton_mla_b200.h"

namespace tmla {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

template <typename T>
struct Elem;
template <>
struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
  static __device__ __forceinline__ float2 pair_to_f(uint32_t v) {
    __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162*>(&v);
    return __bfloat1622float2(h);
  }
};
template <>
struct Elem<__half> {
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
  static __device__ __forceinline__ float2 pair_to_f(uint32_t v) {
    __half2 h = *reinterpret_cast<__half2*>(&v);
    return __half22float2(h);
  }
};

// Resolve the cache row of token `t` of request `b`.  Returns nullptr (and
// flags the status word) when the block-table entry is outside [0, num_pages),
// so a corrupt table masks tokens instead of reading foreign memory.
template <typename T>
__device__ __forceinline__ const T* kv_row(const TmlaDecodeParams& p, int b, int t) {
  const T* base = static_cast<const T*>(p.kv);
  if (p.block_table == nullptr) {
    return base + (int64_t)b * p.kv_stride_page + (int64_t)t * p.kv_stride_tok;
  }
  int slot = t / p.page_size;
  int page = (slot < p.bt_width) ? p.block_table[(int64_t)b * p.bt_stride + slot] : -1;
  if (page < 0 || (int64_t)page >= p.num_pages) {
    if (p.status) atomicOr(p.status, TMLA_STATUS_BAD_PAGE);
    return nullptr;
  }
  return base + (int64_t)page * p.kv_stride_page + (int64_t)(t - slot * p.page_size) * p.kv_stride_tok;
}

// Token range [start, end) of split `s` of a request with `len` tokens.  Splits
// are whole 64-token tiles so that the tcgen05 kernel's tiles never straddle
// two splits; the generic kernel uses the same boundaries.
__device__ __forceinline__ void split_range(int len, int num_splits, int s, int& start, int& end) {
  int tiles = (len + 63) >> 6;
  int per = (tiles + num_splits - 1) / num_splits;
  start = min(s * per * 64, len);
  end = min(start + per * 64, len);
}

// Records the name of a failed CUDA call for tmla_last_cuda_error() (per host thread) and
// returns TMLA_ERR_CUDA: every C entry point reports CUDA failures this way.
int record_cuda_error(cudaError_t e);

// The projection kernel behind tmla_linear, for the library's own callers too: with
// tile_aligned every CTA takes whole 128-row tiles (no partial sums, no workspace).
int linear_launch(const TmlaLinearParams& p, bool tile_aligned, cudaStream_t stream);

}  // namespace tmla
