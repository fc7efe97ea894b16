// Generic split-KV MLA decode kernel (CUDA cores, fp32 accumulation).
//
// Covers every shape the reference's `_mla_decode_stage1` accepts
// (src/triton_mla/kernel.py:43-138): any power-of-two head_dim_v up to 1024 and
// any power-of-two RoPE width, bf16 / fp16 / fp32 caches, paged or dense, any
// page size.  The DeepSeek shape (d_qk 576, d_v 512, 16-bit types) runs on the
// tcgen05 kernel in tmla_sm100.cu instead; this one is its shape-general
// companion and the cross-check used while developing it.
//
// One CTA per (16-head group, split, request).  Per 32-token tile the CTA
// stages the cache rows in shared memory, computes the 16x32 score block with
// one dot product per thread, runs a base-2 online softmax per head and
// accumulates P.V into registers (each thread owns up to 4 latent columns for
// all 16 heads).  Output: the normalised partial and its base-2 LSE per split,
// or, with one split, the final output and natural-log LSE directly.
#include <cuda_fp8.h>

#include <type_traits>

#include "tmla_common.cuh"

namespace tmla {

constexpr int kGenHeads = 16;   // heads per CTA
constexpr int kGenTok = 32;     // tokens per tile
constexpr int kGenThreads = 256;
constexpr int kGenMaxCols = 4;  // latent columns per thread -> d_v <= 1024

template <typename T>
struct Vec;
template <>
struct Vec<__nv_bfloat16> { static constexpr int kPerChunk = 8; };
template <>
struct Vec<__half> { static constexpr int kPerChunk = 8; };
template <>
struct Vec<float> { static constexpr int kPerChunk = 4; };

template <typename T>
__device__ __forceinline__ float ld_f(const T* p) { return Elem<T>::to_f(*p); }
template <>
__device__ __forceinline__ float ld_f<float>(const float* p) { return *p; }

template <typename T>
__device__ __forceinline__ T st_f(float v) { return Elem<T>::from_f(v); }
template <>
__device__ __forceinline__ float st_f<float>(float v) { return v; }

__host__ __device__ inline int gen_row_pad(int d) { return d + 8; }
__host__ __device__ inline int gen_q_pad(int d) { return d + 4; }

size_t generic_smem_bytes(int d_qk, int elt) {
  size_t f = (size_t)kGenHeads * gen_q_pad(d_qk) + kGenHeads * kGenTok + 3 * kGenHeads + kGenTok;
  return f * 4 + (size_t)kGenTok * gen_row_pad(d_qk) * elt + 16;
}

// FP8 cache rows (TMLA_KV_FP8_E4M3, 656 bytes): the row of token t of request b, or nullptr
// (flagged) when its block-table entry is outside the pool.
__device__ __forceinline__ const unsigned char* fp8_row(const TmlaDecodeParams& p, int b, int t) {
  const unsigned char* base = static_cast<const unsigned char*>(p.kv);
  if (p.block_table == nullptr) return base + (int64_t)b * p.kv_stride_page + (int64_t)t * p.kv_stride_tok;
  const int slot = t / p.page_size;
  const int page = (slot < p.bt_width) ? p.block_table[(int64_t)b * p.bt_stride + slot] : -1;
  if (page < 0 || (int64_t)page >= p.num_pages) {
    if (p.status) atomicOr(p.status, TMLA_STATUS_BAD_PAGE);
    return nullptr;
  }
  return base + (int64_t)page * p.kv_stride_page + (int64_t)(t - slot * p.page_size) * p.kv_stride_tok;
}

// Eight e4m3 values (one 8-byte word) times `scale`, in fp32.
template <typename T>
__device__ __forceinline__ void fp8x8_to(T* dst, uint2 w, float scale) {
  static_assert(std::is_same<T, float>::value, "FP8 rows are dequantised to fp32");
  const uint32_t words[2] = {w.x, w.y};
#pragma unroll
  for (int i = 0; i < 2; ++i) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(words[i] >> (16 * j)), __NV_E4M3);
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h));
      dst[4 * i + 2 * j] = f.x * scale;
      dst[4 * i + 2 * j + 1] = f.y * scale;
    }
  }
}

template <typename T, bool kFp8Cache>
__global__ void __launch_bounds__(kGenThreads) mla_generic_split_kernel(TmlaDecodeParams p, int vec_ok) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int D = p.d_qk, DV = p.d_v, H = p.num_heads;
  const int Dq = gen_q_pad(D), Dk = gen_row_pad(D);
  float* q_s = reinterpret_cast<float*>(smem_raw);  // [16][Dq], pre-scaled by scale*log2(e)
  float* p_s = q_s + kGenHeads * Dq;                 // [16][32] scores, then probabilities
  float* m_s = p_s + kGenHeads * kGenTok;            // running max (base 2)
  float* l_s = m_s + kGenHeads;                      // running sum
  float* a_s = l_s + kGenHeads;                      // per-tile rescale factor
  int* bad_s = reinterpret_cast<int*>(a_s + kGenHeads);  // [32]: the row's page id is outside the pool
  // FP8 rows are dequantised to fp32 (a 16-bit tile would round the scaled values again).
  using KT = typename std::conditional<kFp8Cache, float, T>::type;
  KT* k_s = reinterpret_cast<KT*>(bad_s + kGenTok);  // [32][Dk]

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int h0 = blockIdx.x * kGenHeads, split = blockIdx.y, b = blockIdx.z;
  const T* q = static_cast<const T*>(p.q);

  int len = p.seqlens[b];
  const int cap = p.block_table ? p.bt_width * p.page_size : p.page_size;
  if (len > cap || len < 0) {
    if (p.status) atomicOr(p.status, TMLA_STATUS_BAD_PAGE);
    len = len < 0 ? 0 : cap;
  }
  int start, end;
  split_range(len, p.num_splits, split, start, end);
  // Several query tokens per request: head row hh belongs to token hh / (H / q_len), which
  // attends to the first len - (q_len - 1 - token) rows.
  const int q_len = p.q_len > 1 ? p.q_len : 1;
  const int h_tok = H / q_len;

  const float qscale = p.softmax_scale * kLog2e;
  for (int i = tid; i < kGenHeads * D; i += kGenThreads) {
    int h = i / D, d = i - h * D;
    float v = 0.f;
    if (h0 + h < H) v = ld_f<T>(q + (int64_t)b * p.q_stride_b + (int64_t)(h0 + h) * p.q_stride_h + d) * qscale;
    q_s[h * Dq + d] = v;
  }
  if (tid < kGenHeads) {
    m_s[tid] = -INFINITY;
    l_s[tid] = 0.f;
  }
  float acc[kGenHeads][kGenMaxCols];
#pragma unroll
  for (int h = 0; h < kGenHeads; ++h)
#pragma unroll
    for (int j = 0; j < kGenMaxCols; ++j) acc[h][j] = 0.f;
  __syncthreads();

  constexpr int VE = Vec<T>::kPerChunk;
  for (int t0 = start; t0 < end; t0 += kGenTok) {
    // Tokens behind a block-table entry outside the pool are masked out of the softmax (their
    // rows below are zeros); the row loads report them in the status word.
    if (tid < kGenTok) {
      const int tok = t0 + tid, slot = tok / p.page_size;
      int bad = 0;
      if (p.block_table && tok < end) {
        const int page = slot < p.bt_width ? p.block_table[(int64_t)b * p.bt_stride + slot] : -1;
        bad = page < 0 || (int64_t)page >= p.num_pages;
      }
      bad_s[tid] = bad;
    }
    // Stage the tile's cache rows (zeros past `end` or behind a bad page id).
    if constexpr (kFp8Cache) {
      // 656-byte rows: 64 words of 8 latent e4m3 values (scaled by the row's 4 fp32 scales)
      // and 8 chunks of 8 bf16 RoPE values per token, dequantised into the tile as T.
      for (int c = tid; c < kGenTok * 72; c += kGenThreads) {
        const int r = c / 72, k = c - r * 72, tok = t0 + r;
        const unsigned char* row = tok < end ? fp8_row(p, b, tok) : nullptr;
        KT* dst = k_s + r * Dk;
        if (k < 64) {
          if (row) {
            const float scale = reinterpret_cast<const float*>(row + 512)[k >> 4];
            fp8x8_to<KT>(dst + 8 * k, *reinterpret_cast<const uint2*>(row + 8 * k), scale);
          } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) dst[8 * k + i] = 0.f;
          }
        } else {
          const int e = 8 * (k - 64);
          const __nv_bfloat16* rope = row ? reinterpret_cast<const __nv_bfloat16*>(row + 528) : nullptr;
#pragma unroll
          for (int i = 0; i < 8; ++i) dst[512 + e + i] = rope ? __bfloat162float(rope[e + i]) : 0.f;
        }
      }
    } else if (vec_ok) {
      const int chunks = D / VE;
      for (int c = tid; c < kGenTok * chunks; c += kGenThreads) {
        int r = c / chunks, e = (c - r * chunks) * VE;
        int tok = t0 + r;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (tok < end) {
          const T* row = kv_row<T>(p, b, tok);
          if (row) v = *reinterpret_cast<const uint4*>(row + e);
        }
        *reinterpret_cast<uint4*>(k_s + r * Dk + e) = v;
      }
    } else {
      for (int c = tid; c < kGenTok * D; c += kGenThreads) {
        int r = c / D, e = c - r * D;
        int tok = t0 + r;
        T v = st_f<T>(0.f);
        if (tok < end) {
          const T* row = kv_row<T>(p, b, tok);
          if (row) v = row[e];
        }
        k_s[r * Dk + e] = v;
      }
    }
    __syncthreads();

    // Scores: thread -> head (tid >> 4), tokens (tid & 15) and (tid & 15) + 16.
    {
      const int h = tid >> 4;
      const int row_end = min(end, len - (q_len - 1 - min(h0 + h, H - 1) / h_tok));
      const float* qr = q_s + h * Dq;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int r = (tid & 15) + half * 16;
        const KT* kr = k_s + r * Dk;
        float s = 0.f;
        for (int d = 0; d < D; ++d) s = fmaf(qr[d], ld_f<KT>(kr + d), s);
        p_s[h * kGenTok + r] = (t0 + r < row_end && !bad_s[r]) ? s : -INFINITY;
      }
    }
    __syncthreads();

    // Online softmax: warp w owns heads 2w and 2w+1, 16 lanes per head, 2 tokens per lane.
    {
      const int h = warp * 2 + (lane >> 4);
      const int r = lane & 15;
      float s0 = p_s[h * kGenTok + r], s1 = p_s[h * kGenTok + r + 16];
      float mx = fmaxf(s0, s1);
      int nan = (s0 != s0) || (s1 != s1);
#pragma unroll
      for (int o = 8; o >= 1; o >>= 1) {
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        nan |= __shfl_xor_sync(0xffffffffu, nan, o);
      }
      if (nan) mx = __int_as_float(0x7fc00000);  // fmaxf drops NaN scores; keep them
      const float m_old = m_s[h];
      // A row of NaN scores (a NaN scale) stays NaN, as in the reference; fmaxf would drop it.
      const float m_new = mx != mx ? mx : fmaxf(m_old, mx);
      const bool none = m_new == -INFINITY;  // every token so far masked for this row
      const float p0 = none ? 0.f : exp2f(s0 - m_new), p1 = none ? 0.f : exp2f(s1 - m_new);
      float sum = p0 + p1;
#pragma unroll
      for (int o = 8; o >= 1; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      p_s[h * kGenTok + r] = p0;
      p_s[h * kGenTok + r + 16] = p1;
      __syncwarp();
      if (r == 0) {
        const float alpha = none ? 1.f : exp2f(m_old - m_new);
        a_s[h] = alpha;
        l_s[h] = l_s[h] * alpha + sum;
        m_s[h] = m_new;
      }
    }
    __syncthreads();

    // acc[h][j] = acc[h][j] * alpha[h] + sum_t p[h][t] * v[t][d_j]
#pragma unroll
    for (int h = 0; h < kGenHeads; ++h) {
      const float a = a_s[h];
#pragma unroll
      for (int j = 0; j < kGenMaxCols; ++j) acc[h][j] *= a;
    }
    for (int t = 0; t < kGenTok; ++t) {
      float v[kGenMaxCols];
#pragma unroll
      for (int j = 0; j < kGenMaxCols; ++j) {
        const int d = tid + j * kGenThreads;
        v[j] = (d < DV) ? ld_f<KT>(k_s + t * Dk + d) : 0.f;
      }
#pragma unroll
      for (int h = 0; h < kGenHeads; ++h) {
        const float pr = p_s[h * kGenTok + t];
#pragma unroll
        for (int j = 0; j < kGenMaxCols; ++j) acc[h][j] = fmaf(pr, v[j], acc[h][j]);
      }
    }
    __syncthreads();
  }

  // Epilogue: normalise; final output for one split, partial + base-2 LSE otherwise.
  const int S = p.num_splits;
  const bool final_out = (S == 1) && !(p.flags & TMLA_FLAG_PARTIAL_ONLY);
#pragma unroll
  for (int h = 0; h < kGenHeads; ++h) {
    const int hh = h0 + h;
    if (hh >= H) break;
    const float l = l_s[h];
    const float inv = l > 0.f ? 1.f / l : 0.f;
    const float lse2 = l <= 0.f ? -INFINITY : m_s[h] + log2f(l);  // NaN stays NaN
    if (final_out) {
      T* o = static_cast<T*>(p.out) + (int64_t)b * p.out_stride_b + (int64_t)hh * p.out_stride_h;
#pragma unroll
      for (int j = 0; j < kGenMaxCols; ++j) {
        const int d = tid + j * kGenThreads;
        if (d < DV) o[d] = st_f<T>(acc[h][j] * inv);
      }
      if (p.lse && tid == 0) p.lse[(int64_t)b * p.lse_stride_b + hh] = lse2 * kLn2;
    } else {
      const int64_t row = ((int64_t)b * H + hh) * S + split;
      float* o = p.ws_o + row * DV;
#pragma unroll
      for (int j = 0; j < kGenMaxCols; ++j) {
        const int d = tid + j * kGenThreads;
        if (d < DV) o[d] = acc[h][j] * inv;
      }
      if (tid == 0) p.ws_lse[row] = lse2;
    }
  }
}

template <typename T>
static int launch_generic_t(const TmlaDecodeParams& p, cudaStream_t stream) {
  const int elt = (int)sizeof(T);
  const size_t smem = generic_smem_bytes(p.d_qk, elt);
  if (smem > 227 * 1024) return TMLA_ERR_UNSUPPORTED;
  cudaError_t e = cudaFuncSetAttribute(mla_generic_split_kernel<T, false>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return -(int)e;
  const int VE = Vec<T>::kPerChunk;
  int vec_ok = (p.d_qk % VE == 0) && (p.kv_stride_tok % VE == 0) && (p.kv_stride_page % VE == 0) &&
               (((uintptr_t)p.kv) % 16 == 0);
  dim3 grid((p.num_heads + kGenHeads - 1) / kGenHeads, p.num_splits, p.batch);
  if constexpr (!std::is_same<T, float>::value) {
    if (p.kv_format == TMLA_KV_FP8_E4M3) {
      // 8- and 16-byte loads from the rows: the base and the strides are 16-byte aligned.
      if (((uintptr_t)p.kv) % 16 || p.kv_stride_tok % 16 || p.kv_stride_page % 16) return TMLA_ERR_MISALIGNED;
      const size_t smem8 = generic_smem_bytes(p.d_qk, (int)sizeof(float));
      e = cudaFuncSetAttribute(mla_generic_split_kernel<T, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)smem8);
      if (e != cudaSuccess) return -(int)e;
      mla_generic_split_kernel<T, true><<<grid, kGenThreads, smem8, stream>>>(p, 0);
      e = cudaGetLastError();
      return e == cudaSuccess ? 0 : -(int)e;
    }
  }
  mla_generic_split_kernel<T, false><<<grid, kGenThreads, smem, stream>>>(p, vec_ok);
  e = cudaGetLastError();
  return e == cudaSuccess ? 0 : -(int)e;
}

// Returns 0, a positive TMLA_ERR_* code, or minus a cudaError_t.
int launch_generic(const TmlaDecodeParams& p, cudaStream_t stream) {
  if (p.d_v > kGenMaxCols * kGenThreads) return TMLA_ERR_UNSUPPORTED;
  switch (p.dtype) {
    case TMLA_DTYPE_BF16: return launch_generic_t<__nv_bfloat16>(p, stream);
    case TMLA_DTYPE_FP16: return launch_generic_t<__half>(p, stream);
    case TMLA_DTYPE_FP32: return launch_generic_t<float>(p, stream);
    default: return TMLA_ERR_INVALID_ARG;
  }
}

}  // namespace tmla
