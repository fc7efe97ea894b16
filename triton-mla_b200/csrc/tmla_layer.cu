// The MLA layer's small per-step operations around the decode kernel, fused:
//
//   tmla_q_absorb_rope        q = [q_nope . W_UK | rope(q_pe)]  (the decode query)
//   tmla_kv_norm_rope_append  cache row = [rmsnorm(c_kv) | rope(k_pe)] at the new position
//   tmla_o_unabsorb           o . W_UV per head (the input of the output projection)
//
// They replace, in one launch each, the reference layer's PyTorch glue of one decode
// step (src/triton_mla/model.py:74-94 and 111-123: the RoPE of q_pe and k_pe, kv_norm,
// the cache append, the W_UK / W_UV einsums and the concatenation).  Every operation
// reads its weights once; the arithmetic is fp32 with one rounding to the storage
// type at the end, like the PyTorch ops they replace.
//
// RoPE is the reference's half-split form (model.py:44-50): for i < d_rope / 2,
// angle = pos * theta^(-2i / d_rope), out[i] = a cos - b sin, out[i + d_rope/2] =
// b cos + a sin with a = x[i], b = x[i + d_rope / 2].
#include "tmla_common.cuh"
#include "tmla_ptx.cuh"

namespace tmla {
namespace layer {

// Launched with TMLA_LAYER_FLAG_PDL, a kernel may start while the preceding kernel in the
// stream is finishing: it loads only weights before this point, then waits for that kernel
// (a no-op in an ordinary launch) and lets the next programmatic launch be scheduled.
__device__ __forceinline__ void after_predecessor() {
  ptx::griddep_wait();
  ptx::griddep_launch_dependents();
}

template <typename T>
__device__ __forceinline__ float ld(const T* p) {
  return static_cast<float>(*p);
}
template <>
__device__ __forceinline__ float ld<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}
template <>
__device__ __forceinline__ float ld<__half>(const __half* p) {
  return __half2float(*p);
}
template <typename T>
__device__ __forceinline__ T cvt(float v);
template <>
__device__ __forceinline__ float cvt<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ __nv_bfloat16 cvt<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ __half cvt<__half>(float v) {
  return __float2half_rn(v);
}

// Two consecutive elements (4-byte aligned for 16-bit types, 8-byte for fp32) as floats.
template <typename T>
__device__ __forceinline__ float2 ld2(const T* p);
template <>
__device__ __forceinline__ float2 ld2<float>(const float* p) {
  return *reinterpret_cast<const float2*>(p);
}
template <>
__device__ __forceinline__ float2 ld2<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
}
template <>
__device__ __forceinline__ float2 ld2<__half>(const __half* p) {
  return __half22float2(*reinterpret_cast<const __half2*>(p));
}
// Eight consecutive elements (16-byte aligned) as floats.
__device__ __forceinline__ void unpack2(uint32_t w, const __nv_bfloat16*, float& a, float& b) {
  a = __uint_as_float(w << 16);
  b = __uint_as_float(w & 0xffff0000u);
}
__device__ __forceinline__ void unpack2(uint32_t w, const __half*, float& a, float& b) {
  a = __half2float(__ushort_as_half((unsigned short)(w & 0xffffu)));
  b = __half2float(__ushort_as_half((unsigned short)(w >> 16)));
}
template <typename T>
__device__ __forceinline__ void ld8(const T* p, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  unpack2(u.x, p, v[0], v[1]);
  unpack2(u.y, p, v[2], v[3]);
  unpack2(u.z, p, v[4], v[5]);
  unpack2(u.w, p, v[6], v[7]);
}
template <>
__device__ __forceinline__ void ld8<float>(const float* p, float (&v)[8]) {
  const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
  v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
}

__device__ __forceinline__ void rope_pair(float a, float b, int pos, int i, int d_rope, float theta, float& out_a,
                                          float& out_b) {
  const float inv_freq = powf(theta, -(float)(2 * i) / (float)d_rope);
  const float angle = (float)pos * inv_freq;
  float s, c;
  sincosf(angle, &s, &c);
  out_a = a * c - b * s;
  out_b = b * c + a * s;
}

constexpr int kBChunk = 16;  // requests per pass over a weight slice
constexpr int kCols = 64;     // output columns per CTA (q: absorbed latent columns; o: v rows x 4)

// Copy a rows x vpr grid of 16-byte vectors (row r at src + r * src_stride elements,
// dst + r * dst_stride elements) global -> shared.  Each thread issues up to 8 loads
// before it stores any, so a CTA has its whole tile in flight at once.
template <typename T>
__device__ __forceinline__ void stage_rows16(T* dst, int dst_stride, const T* src, int64_t src_stride, int rows,
                                             int vpr) {
  const int n = rows * vpr;
  for (int base = 0; base < n; base += 8 * blockDim.x) {
    uint4 r[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int i = base + k * blockDim.x + threadIdx.x;
      if (i < n) r[k] = reinterpret_cast<const uint4*>(src + (int64_t)(i / vpr) * src_stride)[i % vpr];
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int i = base + k * blockDim.x + threadIdx.x;
      if (i < n) reinterpret_cast<uint4*>(dst + (i / vpr) * dst_stride)[i % vpr] = r[k];
    }
  }
}

// ---------------------------------------------------------------------------- q: absorb + RoPE
// Grid (heads, ceil(rank / 64)), 128 threads.  The CTA stages W_UK[h][:, c0 : c0 + 64]
// (d_nope rows) and the requests' q_nope rows of the head in shared memory; thread t
// computes column c0 + t % 64 for 8 of the 16 requests of a chunk.
template <typename T>
__global__ void __launch_bounds__(128) q_absorb_rope_kernel(TmlaQPrepParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int h = blockIdx.x, tid = threadIdx.x;
  const int dn = p.d_nope, dr = p.d_rope, R = p.rank;
  const int c0 = blockIdx.y * kCols, ncol = min(kCols, R - c0);
  T* ws = reinterpret_cast<T*>(smem);                                  // [dn][kCols]
  float* qs = reinterpret_cast<float*>(smem + (size_t)dn * kCols * sizeof(T));  // [kBChunk][dn]
  const T* q_in = static_cast<const T*>(p.q_in);
  T* q_out = static_cast<T*>(p.q_out);
  const T* w = static_cast<const T*>(p.w_kv_b) + (int64_t)h * (dn + p.d_v) * R + c0;  // W_UK[h][:, c0:]
  // W tile: row d is ncol contiguous elements at w + d * R.
  if (ncol == kCols && (R * (int)sizeof(T)) % 16 == 0 && (c0 * (int)sizeof(T)) % 16 == 0) {
    stage_rows16(ws, kCols, w, R, dn, kCols * (int)sizeof(T) / 16);
  } else {
    for (int i = tid; i < dn * kCols; i += blockDim.x) {
      const int d = i / kCols, c = i % kCols;
      ws[i] = c < ncol ? w[(int64_t)d * R + c] : cvt<T>(0.f);
    }
  }
  const int col = tid % kCols, bg = tid / kCols;  // requests bg * 8 .. bg * 8 + 7 of the chunk
  constexpr int kEpv = 16 / (int)sizeof(T);  // elements per 16-byte vector
  const bool q_vec = dn % kEpv == 0 && (p.q_in_stride_b * (int)sizeof(T)) % 16 == 0 &&
                     (p.q_in_stride_h * (int)sizeof(T)) % 16 == 0 && (uintptr_t)q_in % 16 == 0;
  after_predecessor();
  for (int b0 = 0; b0 < p.batch; b0 += kBChunk) {
    __syncthreads();
    if (q_vec) {
      // 16-byte loads; all of a thread's loads are issued before the stores.
      const int vpr = dn / kEpv, n = kBChunk * vpr;
      for (int base = 0; base < n; base += 4 * blockDim.x) {
        uint4 r[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int i = base + k * blockDim.x + tid, b = b0 + i / vpr;
          r[k] = (i < n && b < p.batch)
                     ? reinterpret_cast<const uint4*>(q_in + (int64_t)b * p.q_in_stride_b +
                                                      (int64_t)h * p.q_in_stride_h)[i % vpr]
                     : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int i = base + k * blockDim.x + tid;
          if (i < n) {
            float* dst = qs + (i / vpr) * dn + (i % vpr) * kEpv;
            if constexpr (sizeof(T) == 4) {
              dst[0] = __uint_as_float(r[k].x), dst[1] = __uint_as_float(r[k].y);
              dst[2] = __uint_as_float(r[k].z), dst[3] = __uint_as_float(r[k].w);
            } else {
              const T* tp = nullptr;
              unpack2(r[k].x, tp, dst[0], dst[1]);
              unpack2(r[k].y, tp, dst[2], dst[3]);
              unpack2(r[k].z, tp, dst[4], dst[5]);
              unpack2(r[k].w, tp, dst[6], dst[7]);
            }
          }
        }
      }
    } else {
      for (int i = tid; i < kBChunk * dn; i += blockDim.x) {
        const int bb = i / dn, d = i % dn, b = b0 + bb;
        qs[i] = b < p.batch ? ld(q_in + (int64_t)b * p.q_in_stride_b + (int64_t)h * p.q_in_stride_h + d) : 0.f;
      }
    }
    __syncthreads();
    float acc[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[k] = 0.f;
    const float* qrow = qs + bg * 8 * dn;
#pragma unroll 4
    for (int d = 0; d < dn; ++d) {
      const float wv = ld(ws + d * kCols + col);
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[k] = fmaf(qrow[k * dn + d], wv, acc[k]);
    }
    if (col < ncol) {
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int b = b0 + bg * 8 + k;
        if (b < p.batch)
          q_out[(int64_t)b * p.q_out_stride_b + (int64_t)h * p.q_out_stride_h + c0 + col] = cvt<T>(acc[k]);
      }
    }
  }
  {
    // RoPE of q_pe for every request of this head, spread over the head's CTAs (one pair or
    // two per thread, so that no CTA carries a chain of them).
    const int half = dr / 2;
    for (int i = blockIdx.y * blockDim.x + tid; i < p.batch * half; i += gridDim.y * blockDim.x) {
      const int b = i / half, k = i % half;
      const T* src = q_in + (int64_t)b * p.q_in_stride_b + (int64_t)h * p.q_in_stride_h + dn;
      float oa, ob;
      rope_pair(ld(src + k), ld(src + k + half), p.positions[b], k, dr, p.rope_theta, oa, ob);
      T* dst = q_out + (int64_t)b * p.q_out_stride_b + (int64_t)h * p.q_out_stride_h + R;
      dst[k] = cvt<T>(oa);
      dst[k + half] = cvt<T>(ob);
    }
  }
}

// ---------------------------------------------------------------------------- kv: norm + RoPE + append
// One warp per request.
// dst[e] = src[e] * rsqrt(mean(src^2) + eps) * w[e] for e < n, by one warp.  16-bit rows
// with 16-byte alignment and n <= 2048 take 16-byte loads, every lane issuing its loads of the
// row and of the weight at once (at most 8 each); other rows go element by element.
template <typename T>
__device__ __forceinline__ void rms_norm_row(const T* src, const T* w, T* dst, int n, float eps, int lane) {
  constexpr int kMaxVec = 8;
  if constexpr (sizeof(T) == 2) {
    if (n % 8 == 0 && n <= 8 * 32 * kMaxVec && ((uintptr_t)src % 16) == 0 && ((uintptr_t)w % 16) == 0 &&
        ((uintptr_t)dst % 16) == 0) {
      const int nvec = n / 8;
      uint4 xv[kMaxVec], wv[kMaxVec];
#pragma unroll
      for (int i = 0; i < kMaxVec; ++i) {
        const int c = lane + 32 * i;
        if (c < nvec) {
          xv[i] = reinterpret_cast<const uint4*>(src)[c];
          wv[i] = reinterpret_cast<const uint4*>(w)[c];
        }
      }
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < kMaxVec; ++i) {
        if (lane + 32 * i < nvec) {
          const uint32_t xw[4] = {xv[i].x, xv[i].y, xv[i].z, xv[i].w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float a, b;
            unpack2(xw[j], src, a, b);
            ss = fmaf(a, a, fmaf(b, b, ss));
          }
        }
      }
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float rstd = rsqrtf(ss / (float)n + eps);
#pragma unroll
      for (int i = 0; i < kMaxVec; ++i) {
        const int c = lane + 32 * i;
        if (c < nvec) {
          const uint32_t xw[4] = {xv[i].x, xv[i].y, xv[i].z, xv[i].w};
          const uint32_t ww[4] = {wv[i].x, wv[i].y, wv[i].z, wv[i].w};
          uint32_t ow[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float xa, xb, wa, wb;
            unpack2(xw[j], src, xa, xb);
            unpack2(ww[j], src, wa, wb);
            const T pr[2] = {cvt<T>(xa * rstd * wa), cvt<T>(xb * rstd * wb)};
            ow[j] = *reinterpret_cast<const uint32_t*>(pr);
          }
          reinterpret_cast<uint4*>(dst)[c] = make_uint4(ow[0], ow[1], ow[2], ow[3]);
        }
      }
      return;
    }
  }
  float ss = 0.f;
  for (int e = lane; e < n; e += 32) {
    const float x = ld(src + e);
    ss = fmaf(x, x, ss);
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float rstd = rsqrtf(ss / (float)n + eps);
  for (int e = lane; e < n; e += 32) dst[e] = cvt<T>(ld(src + e) * rstd * ld(w + e));
}

// Grid (ceil(batch / 4), 1 or 2), 128 threads, one warp per request.  blockIdx.y = 0: the
// cache row (kv_norm, RoPE of k_pe, append); blockIdx.y = 1: the query path's q_norm.
template <typename T>
__global__ void __launch_bounds__(128) kv_append_kernel(TmlaKvAppendParams p) {
  after_predecessor();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x * 4 + warp;
  if (b >= p.batch) return;
  if (blockIdx.y == 1) {
    rms_norm_row(static_cast<const T*>(p.q_in) + (int64_t)b * p.q_in_stride_b, static_cast<const T*>(p.q_norm_weight),
                 static_cast<T*>(p.q_out) + (int64_t)b * p.q_out_stride_b, p.q_rank, p.q_eps, lane);
    return;
  }
  const int R = p.rank, dr = p.d_rope, half = dr / 2;
  const T* src = static_cast<const T*>(p.kv_in) + (int64_t)b * p.kv_in_stride_b;
  const int pos = p.positions[b];
  if (lane == 0 && p.seqlens_out) p.seqlens_out[b] = pos + 1;
  // Where the row goes; a position past the cache or a page id outside the pool is
  // reported on the status word and the row is dropped.
  const int64_t cap = p.block_table ? (int64_t)p.bt_width * p.page_size : (int64_t)p.page_size;
  int64_t page = b, slot = pos;
  bool ok = pos >= 0 && pos < cap;
  if (ok && p.block_table) {
    page = p.block_table[(int64_t)b * p.bt_stride + pos / p.page_size];
    slot = pos % p.page_size;
    ok = page >= 0 && page < p.num_pages;
  }
  if (!ok) {
    if (lane == 0 && p.status) atomicOr(p.status, TMLA_STATUS_BAD_PAGE);
    return;
  }
  T* dst = static_cast<T*>(p.kv_cache) + page * p.kv_stride_page + slot * p.kv_stride_tok;
  rms_norm_row(src, static_cast<const T*>(p.norm_weight), dst, R, p.eps, lane);
  for (int k = lane; k < half; k += 32) {
    float oa, ob;
    rope_pair(ld(src + R + k), ld(src + R + k + half), pos, k, dr, p.rope_theta, oa, ob);
    dst[R + k] = cvt<T>(oa);
    dst[R + k + half] = cvt<T>(ob);
  }
}

// ---------------------------------------------------------------------------- o: un-absorb
// Grid (heads, ceil(d_v / 16)), 128 threads.  The CTA stages 16 rows of W_UV[h] and the
// requests' o rows of the head in shared memory (row stride rank + 8 elements, so that
// rows fall on different banks); thread t computes 2 of the 16 x 16 outputs (v row, request).
template <typename T>
__global__ void __launch_bounds__(128) o_unabsorb_kernel(TmlaOUnabsorbParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int h = blockIdx.x, tid = threadIdx.x;
  const int R = p.rank, stride = R + 8, dn = p.d_nope, dv = p.d_v;
  const int d0 = blockIdx.y * 16, nd = min(16, dv - d0);
  T* ws = reinterpret_cast<T*>(smem);        // [16][stride]
  T* os = ws + 16 * stride;                  // [kBChunk][stride]
  const T* o = static_cast<const T*>(p.o);
  T* out = static_cast<T*>(p.out);
  const T* w = static_cast<const T*>(p.w_kv_b) + ((int64_t)h * (dn + dv) + dn + d0) * R;  // W_UV[h][d0:]
  const int vpr = R * (int)sizeof(T) / 16;
  stage_rows16(ws, stride, w, R, nd, vpr);
  after_predecessor();
  const bool o_vec = (p.o_stride_b * (int)sizeof(T)) % 16 == 0 && (p.o_stride_h * (int)sizeof(T)) % 16 == 0 &&
                     ((uintptr_t)o % 16) == 0;
  const int dd = tid & 15, bh = tid >> 4;  // v row d0 + dd; requests bh and bh + 8 of the chunk
  for (int b0 = 0; b0 < p.batch; b0 += kBChunk) {
    __syncthreads();
    if (o_vec && b0 + kBChunk <= p.batch) {
      stage_rows16(os, stride, o + (int64_t)b0 * p.o_stride_b + (int64_t)h * p.o_stride_h, p.o_stride_b, kBChunk,
                   vpr);
    } else
    for (int i = tid; i < kBChunk * vpr; i += blockDim.x) {
      const int r = i / vpr, v = i % vpr, b = b0 + r;
      uint4* dst = reinterpret_cast<uint4*>(os + r * stride) + v;
      if (b >= p.batch) {
        *dst = make_uint4(0, 0, 0, 0);
      } else if (o_vec) {
        *dst = reinterpret_cast<const uint4*>(o + (int64_t)b * p.o_stride_b + (int64_t)h * p.o_stride_h)[v];
      } else {
        const int e = 16 / (int)sizeof(T);
        for (int k = 0; k < e; ++k)
          os[r * stride + v * e + k] = o[(int64_t)b * p.o_stride_b + (int64_t)h * p.o_stride_h + v * e + k];
      }
    }
    __syncthreads();
    if (dd < nd) {
      const T* wr = ws + dd * stride;
      const T* oa = os + bh * stride;
      const T* ob = os + (bh + 8) * stride;
      float acc_a = 0.f, acc_b = 0.f;
#pragma unroll 2
      for (int c = 0; c < R; c += 8) {
        float wv[8], xa[8], xb[8];
        ld8(wr + c, wv);
        ld8(oa + c, xa);
        ld8(ob + c, xb);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          acc_a = fmaf(wv[k], xa[k], acc_a);
          acc_b = fmaf(wv[k], xb[k], acc_b);
        }
      }
      const int ba = b0 + bh, bb = b0 + bh + 8;
      if (ba < p.batch) out[(int64_t)ba * p.out_stride_b + (int64_t)h * dv + d0 + dd] = cvt<T>(acc_a);
      if (bb < p.batch) out[(int64_t)bb * p.out_stride_b + (int64_t)h * dv + d0 + dd] = cvt<T>(acc_b);
    }
  }
}

// ---------------------------------------------------------------------------- tensor-core forms (16-bit)
// D[16 x 8] += A[16 x 16] (row-major) * B[16 x 8] (col-major), fp32 accumulation (mma.sync m16n8k16).
// Fragments, with g = lane / 4 and t = lane % 4: a0 = A[g][2t..2t+1], a1 = A[g+8][2t..], a2 =
// A[g][2t+8..], a3 = A[g+8][2t+8..]; b0 = B[2t..2t+1][g], b1 = B[2t+8..2t+9][g]; d0, d1 = D[g][2t],
// D[g][2t+1], d2, d3 = D[g+8][2t], D[g+8][2t+1].  Each pair is one 32-bit register, lower k first.
template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]);
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
template <>
__device__ __forceinline__ void mma16816<__half>(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
template <typename T>
__device__ __forceinline__ uint32_t lds32(const T* p) {
  return *reinterpret_cast<const uint32_t*>(p);
}
template <typename T>
__device__ __forceinline__ uint32_t pack_pair(const T* lo, const T* hi) {
  return (uint32_t)*reinterpret_cast<const unsigned short*>(lo) |
         ((uint32_t)*reinterpret_cast<const unsigned short*>(hi) << 16);
}
template <typename T>
__device__ __forceinline__ void st_pair(T* dst, float a, float b) {
  T v[2] = {cvt<T>(a), cvt<T>(b)};
  *reinterpret_cast<uint32_t*>(dst) = *reinterpret_cast<const uint32_t*>(v);
}

// Rows [b0, b0 + 16) of a [batch, heads, n] input for head h into shared memory (row stride
// `stride` elements), zeros past the batch; 16-byte loads when the layout allows.
template <typename T>
__device__ __forceinline__ void stage_batch_rows(T* dst, int stride, const T* src, int64_t sb, int64_t sh, int h,
                                                 int b0, int batch, int n) {
  const bool vec = (sb * (int)sizeof(T)) % 16 == 0 && (sh * (int)sizeof(T)) % 16 == 0 && (uintptr_t)src % 16 == 0 &&
                   (n * (int)sizeof(T)) % 16 == 0;
  if (vec && b0 + kBChunk <= batch) {
    stage_rows16(dst, stride, src + (int64_t)b0 * sb + (int64_t)h * sh, sb, kBChunk, n * (int)sizeof(T) / 16);
    return;
  }
  for (int i = threadIdx.x; i < kBChunk * n; i += blockDim.x) {
    const int r = i / n, c = i % n, b = b0 + r;
    dst[r * stride + c] = b < batch ? src[(int64_t)b * sb + (int64_t)h * sh + c] : cvt<T>(0.f);
  }
}

// q: grid (heads, rank / 64), 128 threads.  M = 16 requests, N = 64 absorbed columns (warp w:
// columns 16w .. 16w + 15), K = d_nope.  A = q_nope (row-major), B = W_UK tile (row-major in
// shared memory, read as col-major pairs).
template <typename T>
__global__ void __launch_bounds__(128) q_absorb_rope_mma_kernel(TmlaQPrepParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int h = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int dn = p.d_nope, dr = p.d_rope, R = p.rank, c0 = blockIdx.y * kCols;
  constexpr int kWs = kCols + 8;  // W tile row stride
  const int qstride = dn + 8;
  T* ws = reinterpret_cast<T*>(smem);  // [dn][kWs]
  T* qs = ws + dn * kWs;               // [16][dn + 8]
  const T* q_in = static_cast<const T*>(p.q_in);
  T* q_out = static_cast<T*>(p.q_out);
  stage_rows16(ws, kWs, static_cast<const T*>(p.w_kv_b) + (int64_t)h * (dn + p.d_v) * R + c0, R, dn,
               kCols * (int)sizeof(T) / 16);
  after_predecessor();
  for (int b0 = 0; b0 < p.batch; b0 += kBChunk) {
    __syncthreads();
    stage_batch_rows(qs, qstride, q_in, p.q_in_stride_b, p.q_in_stride_h, h, b0, p.batch, dn);
    __syncthreads();
    float acc[2][4] = {};
    for (int k0 = 0; k0 < dn; k0 += 16) {
      uint32_t a[4];
      a[0] = lds32(qs + g * qstride + k0 + 2 * t);
      a[1] = lds32(qs + (g + 8) * qstride + k0 + 2 * t);
      a[2] = lds32(qs + g * qstride + k0 + 2 * t + 8);
      a[3] = lds32(qs + (g + 8) * qstride + k0 + 2 * t + 8);
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const int n = warp * 16 + nt * 8 + g;
        uint32_t bf[2];
        bf[0] = pack_pair(ws + (k0 + 2 * t) * kWs + n, ws + (k0 + 2 * t + 1) * kWs + n);
        bf[1] = pack_pair(ws + (k0 + 2 * t + 8) * kWs + n, ws + (k0 + 2 * t + 9) * kWs + n);
        mma16816<T>(acc[nt], a, bf);
      }
    }
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const int c = c0 + warp * 16 + nt * 8 + 2 * t;
      const int ba = b0 + g, bb = b0 + g + 8;
      if (ba < p.batch)
        st_pair(q_out + (int64_t)ba * p.q_out_stride_b + (int64_t)h * p.q_out_stride_h + c, acc[nt][0], acc[nt][1]);
      if (bb < p.batch)
        st_pair(q_out + (int64_t)bb * p.q_out_stride_b + (int64_t)h * p.q_out_stride_h + c, acc[nt][2], acc[nt][3]);
    }
  }
  {
    // RoPE of q_pe, spread over the head's CTAs like the kernel above.
    const int half = dr / 2;
    for (int i = blockIdx.y * blockDim.x + threadIdx.x; i < p.batch * half; i += gridDim.y * blockDim.x) {
      const int b = i / half, k = i % half;
      const T* src = q_in + (int64_t)b * p.q_in_stride_b + (int64_t)h * p.q_in_stride_h + dn;
      float oa, ob;
      rope_pair(ld(src + k), ld(src + k + half), p.positions[b], k, dr, p.rope_theta, oa, ob);
      T* dst = q_out + (int64_t)b * p.q_out_stride_b + (int64_t)h * p.q_out_stride_h + R;
      dst[k] = cvt<T>(oa);
      dst[k + half] = cvt<T>(ob);
    }
  }
}

// RoPE half of the decode query alone: q_out[b, h, rank + k] for the d_rope values of q_pe
// (the W_UK product goes to the projection kernel).  Grid (heads), 128 threads.
template <typename T>
__global__ void __launch_bounds__(128) q_rope_kernel(TmlaQPrepParams p) {
  after_predecessor();
  const int h = blockIdx.x, half = p.d_rope / 2;
  const T* q_in = static_cast<const T*>(p.q_in);
  T* q_out = static_cast<T*>(p.q_out);
  for (int i = threadIdx.x; i < p.batch * half; i += blockDim.x) {
    const int b = i / half, k = i % half;
    const T* src = q_in + (int64_t)b * p.q_in_stride_b + (int64_t)h * p.q_in_stride_h + p.d_nope;
    float oa, ob;
    rope_pair(ld(src + k), ld(src + k + half), p.positions[b], k, p.d_rope, p.rope_theta, oa, ob);
    T* dst = q_out + (int64_t)b * p.q_out_stride_b + (int64_t)h * p.q_out_stride_h + p.rank;
    dst[k] = cvt<T>(oa);
    dst[k + half] = cvt<T>(ob);
  }
}

// o: grid (heads, d_v / 32), 128 threads.  The CTA computes 32 rows of W_UV[h] (d) x 16
// requests; warp w owns the 16 x 8 tile (d rows 16 (w & 1) .., requests 8 (w >> 1) ..) over
// the whole K = rank, so no partial sums cross warps.  A = W_UV rows (row-major), B = o rows
// (c contiguous, i.e. col-major).  Shared memory (32 + 16 rows of rank + 8 elements, 50 KB
// at rank 512) lets 4 CTAs share an SM, so DeepSeek's 128 x 4 CTAs run in one wave.
template <typename T>
__global__ void __launch_bounds__(128) o_unabsorb_mma_kernel(TmlaOUnabsorbParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int h = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int R = p.rank, stride = R + 8, dn = p.d_nope, dv = p.d_v, d0 = blockIdx.y * 32;
  T* ws = reinterpret_cast<T*>(smem);  // [32][stride]
  T* os = ws + 32 * stride;            // [16][stride]
  const T* o = static_cast<const T*>(p.o);
  T* out = static_cast<T*>(p.out);
  stage_rows16(ws, stride, static_cast<const T*>(p.w_kv_b) + ((int64_t)h * (dn + dv) + dn + d0) * R, R, 32,
               R * (int)sizeof(T) / 16);
  after_predecessor();
  const int mt = warp & 1, nt = warp >> 1;
  const T* wrow = ws + (16 * mt) * stride;
  for (int b0 = 0; b0 < p.batch; b0 += kBChunk) {
    __syncthreads();
    stage_batch_rows(os, stride, o, p.o_stride_b, p.o_stride_h, h, b0, p.batch, R);
    __syncthreads();
    float acc[4] = {};
    const T* orow = os + (nt * 8 + g) * stride;
    for (int k0 = 0; k0 < R; k0 += 16) {
      uint32_t a[4];
      a[0] = lds32(wrow + g * stride + k0 + 2 * t);
      a[1] = lds32(wrow + (g + 8) * stride + k0 + 2 * t);
      a[2] = lds32(wrow + g * stride + k0 + 2 * t + 8);
      a[3] = lds32(wrow + (g + 8) * stride + k0 + 2 * t + 8);
      const uint32_t bf[2] = {lds32(orow + k0 + 2 * t), lds32(orow + k0 + 2 * t + 8)};
      mma16816<T>(acc, a, bf);
    }
    // acc: D[d = g][b = 2t, 2t + 1], D[g + 8][2t, 2t + 1] of the warp's tile.
    const int d = d0 + 16 * mt + g, b = b0 + 8 * nt + 2 * t;
    T* col = out + (int64_t)h * dv;
    if (b < p.batch) {
      col[(int64_t)b * p.out_stride_b + d] = cvt<T>(acc[0]);
      col[(int64_t)b * p.out_stride_b + d + 8] = cvt<T>(acc[2]);
    }
    if (b + 1 < p.batch) {
      col[(int64_t)(b + 1) * p.out_stride_b + d] = cvt<T>(acc[1]);
      col[(int64_t)(b + 1) * p.out_stride_b + d + 8] = cvt<T>(acc[3]);
    }
  }
}

// L2 prefetch of `count` chunks of `chunk` bytes at base + i * stride (no shared memory, no
// completion: a hint that the next kernels' operands should be in L2).  Each lane issues bulk
// prefetches of at most kPrefetchPiece bytes, pieces dealt round-robin over the grid's lanes.
constexpr int64_t kPrefetchPiece = 32 << 10;
__global__ void __launch_bounds__(32) l2_prefetch_kernel(const char* base, int64_t chunk, int64_t stride, int32_t count) {
  const int64_t per_chunk = (chunk + kPrefetchPiece - 1) / kPrefetchPiece;
  const int64_t pieces = per_chunk * count;
  for (int64_t i = (int64_t)blockIdx.x * 32 + threadIdx.x; i < pieces; i += (int64_t)gridDim.x * 32) {
    const int64_t c = i / per_chunk, off = (i - c * per_chunk) * kPrefetchPiece;
    const int64_t bytes = chunk - off < kPrefetchPiece ? chunk - off : kPrefetchPiece;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(base + c * stride + off), "r"((uint32_t)bytes)
                 : "memory");
  }
}

}  // namespace layer
}  // namespace tmla

namespace {

using namespace tmla::layer;

// An ordinary launch, or a programmatic dependent of the preceding kernel in the stream.
template <typename... KArgs, typename... Args>
cudaError_t launch(bool pdl, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                   Args... args) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

int finish_launch() {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? TMLA_OK : tmla::record_cuda_error(e);
}

bool valid_dtype(int dt) { return dt == TMLA_DTYPE_BF16 || dt == TMLA_DTYPE_FP16 || dt == TMLA_DTYPE_FP32; }

}  // namespace

extern "C" {

int tmla_q_absorb_rope(const TmlaQPrepParams* p, void* stream) {
  if (!p || p->batch < 0 || p->num_heads <= 0 || p->d_nope <= 0 || p->d_nope > 512 || p->d_rope < 0 ||
      (p->d_rope & 1) || p->d_v < 0 || p->rank <= 0 || !valid_dtype(p->dtype))
    return TMLA_ERR_INVALID_ARG;
  if (p->batch == 0) return TMLA_OK;
  if (!p->q_in || !p->w_kv_b || !p->q_out || (p->d_rope && !p->positions)) return TMLA_ERR_INVALID_ARG;
  if ((uintptr_t)p->w_kv_b % 16) return TMLA_ERR_MISALIGNED;  // weight tiles are staged with 16-byte loads
  const dim3 grid(p->num_heads, (p->rank + kCols - 1) / kCols), block(128);
  const size_t esz = p->dtype == TMLA_DTYPE_FP32 ? 4 : 2;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool pdl = (p->flags & TMLA_LAYER_FLAG_PDL) != 0;
  cudaError_t e = cudaSuccess;
  if (p->dtype != TMLA_DTYPE_FP32 && p->batch <= 64 && (uintptr_t)p->q_in % 16 == 0 && p->q_in_stride_b % 8 == 0 &&
      p->q_in_stride_h % 8 == 0 && p->rank % 8 == 0) {
    // Up to 64 requests of a 16-bit type: the W_UK product on the weight-streaming tcgen05
    // kernel, one group per head (W_UK[h] is [d_nope][rank], the head's first d_nope rows of
    // w_kv_b: a [k][n] weight), tile-aligned (no partial sums, no workspace).  The RoPE half
    // is a separate small launch before it; the projection kernel is its programmatic
    // dependent (it streams its weight tiles while the RoPE runs, and reads q_in after).
    if (p->d_rope) {
      if (p->dtype == TMLA_DTYPE_BF16)
        e = launch(pdl, q_rope_kernel<__nv_bfloat16>, dim3(p->num_heads), dim3(128), 0, s, *p);
      else
        e = launch(pdl, q_rope_kernel<__half>, dim3(p->num_heads), dim3(128), 0, s, *p);
      if (e != cudaSuccess) return tmla::record_cuda_error(e);
    }
    TmlaLinearParams lp = {};
    lp.x = p->q_in;
    lp.x_stride = p->q_in_stride_b;
    lp.x_group_stride = p->q_in_stride_h;
    lp.w = p->w_kv_b;
    lp.w_stride = p->rank;
    lp.w_group_stride = (int64_t)(p->d_nope + p->d_v) * p->rank;
    lp.w_layout = TMLA_W_KN;
    lp.y = p->q_out;
    lp.y_stride = p->q_out_stride_b;
    lp.y_group_stride = p->q_out_stride_h;
    lp.m = p->batch;
    lp.n = p->rank;
    lp.k = p->d_nope;
    lp.groups = p->num_heads;
    lp.dtype = p->dtype;
    lp.flags = (p->d_rope || pdl) ? TMLA_LAYER_FLAG_PDL : 0;
    return tmla::linear_launch(lp, true, s);
  }
  if (p->dtype != TMLA_DTYPE_FP32 && p->d_nope % 16 == 0 && p->rank % kCols == 0) {
    // 16-bit types, more than 64 requests: the contraction on tensor cores (mma.sync m16n8k16,
    // fp32 accumulation).
    const size_t smem = ((size_t)p->d_nope * (kCols + 8) + (size_t)kBChunk * (p->d_nope + 8)) * esz;
    if (p->dtype == TMLA_DTYPE_BF16) {
      e = cudaFuncSetAttribute(q_absorb_rope_mma_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)smem);
      if (e == cudaSuccess) e = launch(pdl, q_absorb_rope_mma_kernel<__nv_bfloat16>, grid, block, smem, s, *p);
    } else {
      e = cudaFuncSetAttribute(q_absorb_rope_mma_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)smem);
      if (e == cudaSuccess) e = launch(pdl, q_absorb_rope_mma_kernel<__half>, grid, block, smem, s, *p);
    }
    if (e != cudaSuccess) return tmla::record_cuda_error(e);
    return finish_launch();
  }
  const size_t smem = (size_t)p->d_nope * kCols * esz + (size_t)kBChunk * p->d_nope * sizeof(float);
  switch (p->dtype) {
    case TMLA_DTYPE_BF16:
      e = cudaFuncSetAttribute(q_absorb_rope_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)smem);
      if (e == cudaSuccess) e = launch(pdl, q_absorb_rope_kernel<__nv_bfloat16>, grid, block, smem, s, *p);
      break;
    case TMLA_DTYPE_FP16:
      e = cudaFuncSetAttribute(q_absorb_rope_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e == cudaSuccess) e = launch(pdl, q_absorb_rope_kernel<__half>, grid, block, smem, s, *p);
      break;
    default:
      e = cudaFuncSetAttribute(q_absorb_rope_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e == cudaSuccess) e = launch(pdl, q_absorb_rope_kernel<float>, grid, block, smem, s, *p);
  }
  if (e != cudaSuccess) return tmla::record_cuda_error(e);
  return finish_launch();
}

int tmla_kv_norm_rope_append(const TmlaKvAppendParams* p, void* stream) {
  if (!p || p->batch < 0 || p->rank <= 0 || p->d_rope < 0 || (p->d_rope & 1) || p->page_size <= 0 ||
      p->num_pages < 0 || !valid_dtype(p->dtype))
    return TMLA_ERR_INVALID_ARG;
  if (p->batch == 0) return TMLA_OK;
  if (!p->kv_in || !p->norm_weight || !p->positions || !p->kv_cache) return TMLA_ERR_INVALID_ARG;
  if (p->block_table && p->bt_width <= 0) return TMLA_ERR_INVALID_ARG;
  if (p->q_in && (!p->q_norm_weight || !p->q_out || p->q_rank <= 0)) return TMLA_ERR_INVALID_ARG;
  const dim3 grid((p->batch + 3) / 4, p->q_in ? 2 : 1), block(128);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool pdl = (p->flags & TMLA_LAYER_FLAG_PDL) != 0;
  cudaError_t e;
  switch (p->dtype) {
    case TMLA_DTYPE_BF16:
      e = launch(pdl, kv_append_kernel<__nv_bfloat16>, grid, block, 0, s, *p);
      break;
    case TMLA_DTYPE_FP16:
      e = launch(pdl, kv_append_kernel<__half>, grid, block, 0, s, *p);
      break;
    default:
      e = launch(pdl, kv_append_kernel<float>, grid, block, 0, s, *p);
  }
  if (e != cudaSuccess) return tmla::record_cuda_error(e);
  return finish_launch();
}

int tmla_o_unabsorb(const TmlaOUnabsorbParams* p, void* stream) {
  if (!p || p->batch < 0 || p->num_heads <= 0 || p->d_nope < 0 || p->d_v <= 0 || p->rank <= 0 || p->rank > 2048 ||
      !valid_dtype(p->dtype))
    return TMLA_ERR_INVALID_ARG;
  if (p->batch == 0) return TMLA_OK;
  if (!p->o || !p->w_kv_b || !p->out) return TMLA_ERR_INVALID_ARG;
  // Weight rows are staged with 16-byte loads: each row of W_UV must start 16-byte aligned.
  if (p->rank % 16 || (uintptr_t)p->w_kv_b % 16) return TMLA_ERR_MISALIGNED;
  const dim3 grid(p->num_heads, (p->d_v + 15) / 16), block(128);
  const size_t esz = p->dtype == TMLA_DTYPE_FP32 ? 4 : 2;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool pdl = (p->flags & TMLA_LAYER_FLAG_PDL) != 0;
  cudaError_t e = cudaSuccess;
  if (p->dtype != TMLA_DTYPE_FP32 && p->batch <= 64 && (uintptr_t)p->o % 16 == 0 && p->o_stride_b % 8 == 0 &&
      p->o_stride_h % 8 == 0 && ((size_t)p->d_nope * p->rank) % 8 == 0) {
    // Up to 64 requests: the weight-streaming tcgen05 kernel, one group per head (W_UV[h] is
    // [d_v][rank], the rows d_nope .. d_nope + d_v of the head's block of w_kv_b).
    TmlaLinearParams lp = {};
    lp.x = p->o;
    lp.x_stride = p->o_stride_b;
    lp.x_group_stride = p->o_stride_h;
    lp.w = static_cast<const char*>(p->w_kv_b) + (size_t)p->d_nope * p->rank * 2;
    lp.w_stride = p->rank;
    lp.w_group_stride = (int64_t)(p->d_nope + p->d_v) * p->rank;
    lp.w_layout = TMLA_W_NK;
    lp.y = p->out;
    lp.y_stride = p->out_stride_b;
    lp.y_group_stride = p->d_v;
    lp.m = p->batch;
    lp.n = p->d_v;
    lp.k = p->rank;
    lp.groups = p->num_heads;
    lp.dtype = p->dtype;
    lp.flags = p->flags;
    return tmla::linear_launch(lp, true, s);
  }
  if (p->dtype != TMLA_DTYPE_FP32 && p->rank % 64 == 0 && p->d_v % 32 == 0) {
    // 16-bit types: the contraction on tensor cores (mma.sync m16n8k16, fp32 accumulation).
    const dim3 grid_mma(p->num_heads, p->d_v / 32);
    const size_t smem = (size_t)(32 + kBChunk) * (p->rank + 8) * esz;
    if (p->dtype == TMLA_DTYPE_BF16) {
      e = cudaFuncSetAttribute(o_unabsorb_mma_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)smem);
      if (e == cudaSuccess) e = launch(pdl, o_unabsorb_mma_kernel<__nv_bfloat16>, grid_mma, block, smem, s, *p);
    } else {
      e = cudaFuncSetAttribute(o_unabsorb_mma_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e == cudaSuccess) e = launch(pdl, o_unabsorb_mma_kernel<__half>, grid_mma, block, smem, s, *p);
    }
    if (e != cudaSuccess) return tmla::record_cuda_error(e);
    return finish_launch();
  }
  const size_t smem = (size_t)(16 + kBChunk) * (p->rank + 8) * esz;
  switch (p->dtype) {
    case TMLA_DTYPE_BF16:
      e = cudaFuncSetAttribute(o_unabsorb_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e == cudaSuccess) e = launch(pdl, o_unabsorb_kernel<__nv_bfloat16>, grid, block, smem, s, *p);
      break;
    case TMLA_DTYPE_FP16:
      e = cudaFuncSetAttribute(o_unabsorb_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e == cudaSuccess) e = launch(pdl, o_unabsorb_kernel<__half>, grid, block, smem, s, *p);
      break;
    default:
      e = cudaFuncSetAttribute(o_unabsorb_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e == cudaSuccess) e = launch(pdl, o_unabsorb_kernel<float>, grid, block, smem, s, *p);
  }
  if (e != cudaSuccess) return tmla::record_cuda_error(e);
  return finish_launch();
}

int tmla_l2_prefetch(const void* base, int64_t chunk_bytes, int64_t stride_bytes, int32_t count, int32_t ctas,
                     void* stream) {
  if (count == 0) return TMLA_OK;
  if (!base || chunk_bytes <= 0 || count < 0 || ctas < 1 || stride_bytes < chunk_bytes) return TMLA_ERR_INVALID_ARG;
  if ((uintptr_t)base % 16 || chunk_bytes % 16 || stride_bytes % 16) return TMLA_ERR_MISALIGNED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  l2_prefetch_kernel<<<ctas, 32, 0, s>>>(static_cast<const char*>(base), chunk_bytes, stride_bytes, count);
  return finish_launch();
}

}  // extern "C"
