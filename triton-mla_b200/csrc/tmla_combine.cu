// Split merge: out[b,h,:] = sum_s w_s * o_s / sum_s w_s with w_s = 2^(lse_s - max lse).
//
// Replaces the reference's `_mla_decode_stage2` (src/triton_mla/kernel.py:141-181):
// same arithmetic (base-2 weights against the split maximum, an all-empty row
// gives out 0 and lse -inf, the final LSE is converted to natural log), but
// warps over (request, head, 128-column group) with 16-byte loads of the fp32
// partials (8-byte loads of 16-bit ones), 8 splits in flight, instead of one 4-warp
// program per row with a serial split loop.  For d_v = 512 and at most 4 splits, one warp per row with
// every load of the row in flight (fewer, fuller warps: one wave of CTAs).
#include "tmla_common.cuh"
#include "tmla_ptx.cuh"

namespace tmla {

constexpr int kCombineWarps = 8;

template <typename T>
__device__ __forceinline__ void store4(T* dst, float4 v);
template <>
__device__ __forceinline__ void store4<__nv_bfloat16>(__nv_bfloat16* dst, float4 v) {
  __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
  uint2 u;
  u.x = *reinterpret_cast<uint32_t*>(&a);
  u.y = *reinterpret_cast<uint32_t*>(&b);
  *reinterpret_cast<uint2*>(dst) = u;
}
template <>
__device__ __forceinline__ void store4<__half>(__half* dst, float4 v) {
  __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
  uint2 u;
  u.x = *reinterpret_cast<uint32_t*>(&a);
  u.y = *reinterpret_cast<uint32_t*>(&b);
  *reinterpret_cast<uint2*>(dst) = u;
}
template <>
__device__ __forceinline__ void store4<float>(float* dst, float4 v) {
  *reinterpret_cast<float4*>(dst) = v;
}

template <typename T>
__device__ __forceinline__ T cvt1(float v);
template <>
__device__ __forceinline__ __nv_bfloat16 cvt1<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half cvt1<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ float cvt1<float>(float v) { return v; }

// Partials: fp32 (the documented stage-1 layout), or 16-bit in the query's type (what
// tmla_decode's tcgen05 path writes into its own workspace).  ld4: four consecutive values
// (16- or 8-byte load); ld1: one value.
template <typename P>
__device__ __forceinline__ float4 ld4(const P* p);
template <>
__device__ __forceinline__ float4 ld4<float>(const float* p) {
  return __ldg(reinterpret_cast<const float4*>(p));
}
template <>
__device__ __forceinline__ float4 ld4<__nv_bfloat16>(const __nv_bfloat16* p) {
  const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}
template <>
__device__ __forceinline__ float4 ld4<__half>(const __half* p) {
  const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}
template <typename P>
__device__ __forceinline__ float ld1(const P* p) {
  return static_cast<float>(*p);
}

// Vector path (d_v a multiple of 128, at most 64 splits): one warp per (row, group of
// 128 columns); lane l owns columns 4l..4l+3 of the group.  The split weights sit in
// two registers per lane (splits l and l + 32) and are broadcast by shuffles, and the
// loads of kVecLoads splits are issued before their FMAs, so a row costs S/kVecLoads memory
// round trips instead of S.  Sixteen loads in flight need the registers of 2 blocks per SM,
// eight fit 4: the launch takes 16 when there are more than 8 splits and the grid still fits
// one wave at 2 blocks per SM.
template <typename T, typename P, int kVecLoads>
__global__ void __launch_bounds__(kCombineWarps * 32, kVecLoads > 8 ? 2 : 4)
    mla_combine_vec_kernel(const P* __restrict__ ws_o, const float* __restrict__ ws_lse, T* __restrict__ out,
                           int64_t osb, int64_t osh, float* __restrict__ lse, int64_t lsb, int B, int H, int S,
                           int DV) {
  // Launched as a programmatic dependent of the split kernel: wait for its partials.
  ptx::griddep_wait();
  ptx::griddep_launch_dependents();  // a programmatic successor may be scheduled now
  const int lane = threadIdx.x & 31;
  const int groups = DV / 128;
  const int64_t wid = (int64_t)blockIdx.x * kCombineWarps + (threadIdx.x >> 5);
  if (wid >= (int64_t)B * H * groups) return;
  const int64_t row = wid / groups;
  const int grp = (int)(wid - row * groups);
  const int b = (int)(row / H), h = (int)(row - (int64_t)b * H);
  const float* L = ws_lse + row * S;
  const P* src = ws_o + row * (int64_t)S * DV + grp * 128 + 4 * lane;
  const int64_t sstride = DV;
  // The first kVecLoads splits' partials are requested before the LSEs have come back: the
  // two loads do not depend on each other.
  float4 v[kVecLoads];
#pragma unroll
  for (int u = 0; u < kVecLoads; ++u) v[u] = (u < S) ? ld4<P>(src + u * sstride) : make_float4(0.f, 0.f, 0.f, 0.f);

  const float l0 = lane < S ? L[lane] : -INFINITY, l1 = lane + 32 < S ? L[lane + 32] : -INFINITY;
  float m = fmaxf(l0, l1);
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (m == -INFINITY) m = 0.f;
  const float w0 = exp2f(l0 - m), w1 = exp2f(l1 - m);  // 0 for -inf (empty splits, lanes past S)
  float wsum = w0 + w1;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) wsum += __shfl_xor_sync(0xffffffffu, wsum, o);

  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int s0 = 0; s0 < S; s0 += kVecLoads) {
    float w[kVecLoads];
#pragma unroll
    for (int u = 0; u < kVecLoads; ++u) {
      const int s = s0 + u;
      w[u] = __shfl_sync(0xffffffffu, s < 32 ? w0 : w1, s & 31);
      if (s0 > 0) v[u] = (s < S) ? ld4<P>(src + s * sstride) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < kVecLoads; ++u) {
      acc.x = fmaf(w[u], v[u].x, acc.x);
      acc.y = fmaf(w[u], v[u].y, acc.y);
      acc.z = fmaf(w[u], v[u].z, acc.z);
      acc.w = fmaf(w[u], v[u].w, acc.w);
    }
  }
  const float inv = wsum > 0.f ? 1.f / wsum : 1.f;
  T* dst = out + (int64_t)b * osb + (int64_t)h * osh + grp * 128 + 4 * lane;
  store4<T>(dst, make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv));
  if (lse && grp == 0 && lane == 0) lse[(int64_t)b * lsb + h] = wsum <= 0.f ? -INFINITY : (m + log2f(wsum)) * kLn2;
}

// One warp merges one output row of d_v = 512 (the DeepSeek shape): lane l owns the float4
// columns l, l + 32, l + 64 and l + 96, and two splits are in flight at a time (eight 16-byte
// loads per lane, issued with the LSE loads before the weights are known).  Split s of the row
// is at O + s * split_stride values and its base-2 LSE at L[s * lse_stride].
template <typename T, typename P>
__device__ __forceinline__ void merge_row512(const P* __restrict__ O, int64_t split_stride, const float* __restrict__ L,
                                             int64_t lse_stride, int S, T* dst, float* lse_dst, int lane) {
  const P* src = O + 4 * lane;
  float4 v[2][4];
#pragma unroll
  for (int u = 0; u < 2; ++u)
#pragma unroll
    for (int c = 0; c < 4; ++c)
      v[u][c] = u < S ? ld4<P>(src + u * split_stride + 128 * c) : make_float4(0.f, 0.f, 0.f, 0.f);
  const float l0 = lane < S ? L[lane * lse_stride] : -INFINITY;
  const float l1 = lane + 32 < S ? L[(lane + 32) * lse_stride] : -INFINITY;
  float m = fmaxf(l0, l1);
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (m == -INFINITY) m = 0.f;
  const float w0 = exp2f(l0 - m), w1 = exp2f(l1 - m);  // 0 for -inf (empty splits, lanes past S)
  float wsum = w0 + w1;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) wsum += __shfl_xor_sync(0xffffffffu, wsum, o);
  float4 acc[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) acc[c] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int s0 = 0; s0 < S; s0 += 2) {
    if (s0 > 0) {
#pragma unroll
      for (int u = 0; u < 2; ++u)
#pragma unroll
        for (int c = 0; c < 4; ++c)
          v[u][c] = s0 + u < S ? ld4<P>(src + (s0 + u) * split_stride + 128 * c) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int s = s0 + u;
      const float w = __shfl_sync(0xffffffffu, s < 32 ? w0 : w1, s & 31);  // 0 past S (l = -inf)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        acc[c].x = fmaf(w, v[u][c].x, acc[c].x);
        acc[c].y = fmaf(w, v[u][c].y, acc[c].y);
        acc[c].z = fmaf(w, v[u][c].z, acc[c].z);
        acc[c].w = fmaf(w, v[u][c].w, acc[c].w);
      }
    }
  }
  const float inv = wsum > 0.f ? 1.f / wsum : 1.f;
#pragma unroll
  for (int c = 0; c < 4; ++c)
    store4<T>(dst + 4 * (lane + 32 * c), make_float4(acc[c].x * inv, acc[c].y * inv, acc[c].z * inv, acc[c].w * inv));
  if (lse_dst && lane == 0) *lse_dst = wsum <= 0.f ? -INFINITY : (m + log2f(wsum)) * kLn2;
}

constexpr int kRowWarps = 4;  // rows per CTA of the d_v = 512 merges (8 CTAs, 1024 threads per SM)

// Uniform splits, d_v = 512: ws_o [B, H, S, 512], ws_lse [B, H, S]; one warp per (b, h).
template <typename T, typename P>
__global__ void __launch_bounds__(kRowWarps * 32, 8)
    mla_combine_row512_kernel(const P* __restrict__ ws_o, const float* __restrict__ ws_lse, T* __restrict__ out,
                              int64_t osb, int64_t osh, float* __restrict__ lse, int64_t lsb, int B, int H, int S) {
  ptx::griddep_wait();
  ptx::griddep_launch_dependents();  // a programmatic successor may be scheduled now
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kRowWarps + (threadIdx.x >> 5);
  if (row >= (int64_t)B * H) return;
  const int b = (int)(row / H), h = (int)(row - (int64_t)b * H);
  merge_row512<T, P>(ws_o + row * S * 512, 512, ws_lse + row * S, 1, S, out + (int64_t)b * osb + (int64_t)h * osh,
                  lse ? lse + (int64_t)b * lsb + h : nullptr, lane);
}

// Merge of a per-request split plan (tmla_decode_units): request b's partials sit in slots
// req_first[b] .. req_first[b + 1] - 1 of ws_o [slots, H, DV] / ws_lse [slots, H]; a request
// with no slots (one split) was written by the split kernel and is skipped.  Same layout of
// the work and the same arithmetic as mla_combine_vec_kernel.
template <typename T, typename P>
__global__ void __launch_bounds__(kCombineWarps * 32, 4)
    mla_combine_slots_kernel(const P* __restrict__ ws_o, const float* __restrict__ ws_lse,
                             const int32_t* __restrict__ req_first, T* __restrict__ out, int64_t osb, int64_t osh,
                             float* __restrict__ lse, int64_t lsb, int B, int H, int DV) {
  ptx::griddep_wait();
  ptx::griddep_launch_dependents();  // a programmatic successor may be scheduled now
  const int lane = threadIdx.x & 31;
  const int groups = DV / 128;
  const int64_t wid = (int64_t)blockIdx.x * kCombineWarps + (threadIdx.x >> 5);
  if (wid >= (int64_t)B * H * groups) return;
  const int64_t row = wid / groups;
  const int grp = (int)(wid - row * groups);
  const int b = (int)(row / H), h = (int)(row - (int64_t)b * H);
  const int s0 = req_first[b], S = req_first[b + 1] - s0;
  if (S <= 0) return;
  const P* src = ws_o + ((int64_t)s0 * H + h) * DV + grp * 128 + 4 * lane;
  const int64_t sstride = (int64_t)H * DV;
  float4 v[8];
#pragma unroll
  for (int u = 0; u < 8; ++u) v[u] = (u < S) ? ld4<P>(src + u * sstride) : make_float4(0.f, 0.f, 0.f, 0.f);
  const float* L = ws_lse + (int64_t)s0 * H + h;
  const float l0 = lane < S ? L[(int64_t)lane * H] : -INFINITY;
  const float l1 = lane + 32 < S ? L[(int64_t)(lane + 32) * H] : -INFINITY;
  float m = fmaxf(l0, l1);
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (m == -INFINITY) m = 0.f;
  const float w0 = exp2f(l0 - m), w1 = exp2f(l1 - m);
  float wsum = w0 + w1;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) wsum += __shfl_xor_sync(0xffffffffu, wsum, o);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int q0 = 0; q0 < S; q0 += 8) {
    float w[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int sp = q0 + u;
      w[u] = __shfl_sync(0xffffffffu, sp < 32 ? w0 : w1, sp & 31);
      if (q0 > 0) v[u] = (sp < S) ? ld4<P>(src + sp * sstride) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      acc.x = fmaf(w[u], v[u].x, acc.x);
      acc.y = fmaf(w[u], v[u].y, acc.y);
      acc.z = fmaf(w[u], v[u].z, acc.z);
      acc.w = fmaf(w[u], v[u].w, acc.w);
    }
  }
  const float inv = wsum > 0.f ? 1.f / wsum : 1.f;
  T* dst = out + (int64_t)b * osb + (int64_t)h * osh + grp * 128 + 4 * lane;
  store4<T>(dst, make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv));
  if (lse && grp == 0 && lane == 0) lse[(int64_t)b * lsb + h] = wsum <= 0.f ? -INFINITY : (m + log2f(wsum)) * kLn2;
}

// General path (any d_v, any split count): one warp per row, serial over splits.
template <typename T, typename P>
__global__ void __launch_bounds__(kCombineWarps * 32, 4)
    mla_combine_kernel(const P* __restrict__ ws_o, const float* __restrict__ ws_lse, T* __restrict__ out,
                       int64_t osb, int64_t osh, float* __restrict__ lse, int64_t lsb, int B, int H, int S, int DV) {
  ptx::griddep_wait();
  ptx::griddep_launch_dependents();  // a programmatic successor may be scheduled now
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kCombineWarps + (threadIdx.x >> 5);
  if (row >= (int64_t)B * H) return;
  const int b = (int)(row / H), h = (int)(row - (int64_t)b * H);
  const float* L = ws_lse + row * S;

  float m = -INFINITY;
  for (int s = lane; s < S; s += 32) m = fmaxf(m, L[s]);
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (m == -INFINITY) m = 0.f;

  const P* O = ws_o + row * (int64_t)S * DV;
  T* dst = out + (int64_t)b * osb + (int64_t)h * osh;
  float wsum = 0.f;
  for (int s = 0; s < S; ++s) wsum += exp2f(L[s] - m);
  const float inv = wsum > 0.f ? 1.f / wsum : 1.f;
  for (int d = lane; d < DV; d += 32) {
    float a = 0.f;
    for (int s = 0; s < S; ++s) a = fmaf(exp2f(L[s] - m), ld1<P>(O + (int64_t)s * DV + d), a);
    dst[d] = cvt1<T>(a * inv);
  }
  if (lse && lane == 0) lse[(int64_t)b * lsb + h] = wsum <= 0.f ? -INFINITY : (m + log2f(wsum)) * kLn2;
}

template <typename T, typename P>
static int launch_combine_t(const void* ws_o_v, const float* ws_lse, void* out, int64_t osb, int64_t osh, float* lse,
                            int64_t lsb, int B, int H, int S, int DV, cudaStream_t stream) {
  const int64_t rows = (int64_t)B * H;
  if (rows == 0) return 0;
  const P* ws_o = static_cast<const P*>(ws_o_v);
  const bool vec_ok = (DV % 128 == 0) && (S <= 64) && (osb % 4 == 0) && (osh % 4 == 0) &&
                      (((uintptr_t)out) % (4 * sizeof(T)) == 0) && (((uintptr_t)ws_o) % 16 == 0);
  // Programmatic dependent launch: the merge's launch overlaps the end of the split
  // kernel, and its CTAs wait for the split kernel's writes (griddep_wait) before reading.
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.blockDim = dim3(kCombineWarps * 32);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  T* o = static_cast<T*>(out);
  cudaError_t e;
  // d_v = 512 with few splits: a warp per row, all of a row's loads in flight at once.  With
  // many splits (long requests, few rows) four warps per row over 8 splits at a time do better.
  if (vec_ok && DV == 512 && S <= 4) {
    cfg.blockDim = dim3(kRowWarps * 32);
    cfg.gridDim = dim3((unsigned)((rows + kRowWarps - 1) / kRowWarps));
    e = cudaLaunchKernelEx(&cfg, mla_combine_row512_kernel<T, P>, ws_o, ws_lse, o, osb, osh, lse, lsb, B, H, S);
  } else if (vec_ok) {
    const int64_t warps = rows * (DV / 128);
    const int64_t blocks = (warps + kCombineWarps - 1) / kCombineWarps;
    cfg.gridDim = dim3((unsigned)blocks);
    int dev = 0, sms = 0;
    if (S > 8 && cudaGetDevice(&dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && blocks <= 2 * (int64_t)sms)
      e = cudaLaunchKernelEx(&cfg, mla_combine_vec_kernel<T, P, 16>, ws_o, ws_lse, o, osb, osh, lse, lsb, B, H, S, DV);
    else
      e = cudaLaunchKernelEx(&cfg, mla_combine_vec_kernel<T, P, 8>, ws_o, ws_lse, o, osb, osh, lse, lsb, B, H, S, DV);
  } else {
    cfg.gridDim = dim3((unsigned)((rows + kCombineWarps - 1) / kCombineWarps));
    e = cudaLaunchKernelEx(&cfg, mla_combine_kernel<T, P>, ws_o, ws_lse, o, osb, osh, lse, lsb, B, H, S, DV);
  }
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? 0 : -(int)e;
}

template <typename T, typename P>
static int launch_combine_slots_t(const void* ws_o, const float* ws_lse, const int32_t* req_first, void* out,
                                  int64_t osb, int64_t osh, float* lse, int64_t lsb, int B, int H, int DV,
                                  cudaStream_t stream) {
  const int64_t warps = (int64_t)B * H * (DV / 128);
  if (warps == 0) return 0;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.blockDim = dim3(kCombineWarps * 32);
  cfg.gridDim = dim3((unsigned)((warps + kCombineWarps - 1) / kCombineWarps));
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, mla_combine_slots_kernel<T, P>, static_cast<const P*>(ws_o), ws_lse,
                                     req_first, static_cast<T*>(out), osb, osh, lse, lsb, B, H, DV);
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? 0 : -(int)e;
}

// Merge of a per-request split plan; d_v a multiple of 128, at most 64 splits per request
// (the planner's limit), 16-byte aligned out rows.  part16: the partials are in the output's
// 16-bit type, else fp32.
int launch_combine_slots(const void* ws_o, const float* ws_lse, const int32_t* req_first, void* out, int64_t osb,
                         int64_t osh, float* lse, int64_t lsb, int B, int H, int DV, int dtype, bool part16,
                         cudaStream_t stream) {
  if (DV % 128) return TMLA_ERR_UNSUPPORTED;
  switch (dtype) {
    case TMLA_DTYPE_BF16:
      return part16 ? launch_combine_slots_t<__nv_bfloat16, __nv_bfloat16>(ws_o, ws_lse, req_first, out, osb, osh, lse,
                                                                            lsb, B, H, DV, stream)
                    : launch_combine_slots_t<__nv_bfloat16, float>(ws_o, ws_lse, req_first, out, osb, osh, lse, lsb, B,
                                                                   H, DV, stream);
    case TMLA_DTYPE_FP16:
      return part16 ? launch_combine_slots_t<__half, __half>(ws_o, ws_lse, req_first, out, osb, osh, lse, lsb, B, H, DV,
                                                             stream)
                    : launch_combine_slots_t<__half, float>(ws_o, ws_lse, req_first, out, osb, osh, lse, lsb, B, H, DV,
                                                            stream);
    default:
      return TMLA_ERR_UNSUPPORTED;
  }
}

int launch_combine(const void* ws_o, const float* ws_lse, void* out, int64_t osb, int64_t osh, float* lse,
                   int64_t lsb, int B, int H, int S, int DV, int dtype, bool part16, cudaStream_t stream) {
  switch (dtype) {
    case TMLA_DTYPE_BF16:
      return part16 ? launch_combine_t<__nv_bfloat16, __nv_bfloat16>(ws_o, ws_lse, out, osb, osh, lse, lsb, B, H, S,
                                                                     DV, stream)
                    : launch_combine_t<__nv_bfloat16, float>(ws_o, ws_lse, out, osb, osh, lse, lsb, B, H, S, DV, stream);
    case TMLA_DTYPE_FP16:
      return part16 ? launch_combine_t<__half, __half>(ws_o, ws_lse, out, osb, osh, lse, lsb, B, H, S, DV, stream)
                    : launch_combine_t<__half, float>(ws_o, ws_lse, out, osb, osh, lse, lsb, B, H, S, DV, stream);
    case TMLA_DTYPE_FP32:
      if (part16) return TMLA_ERR_INVALID_ARG;
      return launch_combine_t<float, float>(ws_o, ws_lse, out, osb, osh, lse, lsb, B, H, S, DV, stream);
    default:
      return TMLA_ERR_INVALID_ARG;
  }
}

}  // namespace tmla
