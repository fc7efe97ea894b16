// The decode registered as a PyTorch operator, torch.ops.triton_mla.decode, on top of the C ABI
// (include/triton_mla_b200.h, tmla_decode).
//
// The reference runs its decode as Python code around two Triton launches
// (src/triton_mla/kernel.py:204-323), which torch.compile treats as opaque Python.  Here the
// whole call is one operator with a CUDA kernel and a Meta kernel: torch.compile traces a
// function that calls mla_decode (with an explicit num_splits) into one graph without a
// break, and CUDA-graph capture records the launches.  The Python wrapper (triton_mla.kernel)
// keeps the reference's argument checks and calls this operator.
//
// Schema: decode(q [B, H, D], kv_cache [N, P, D], cache_seqlens int32 [B], block_table int32
// [B, W] or None, out [B, H, Dv] (written), lse fp32 [B, H] (written), num_splits, softmax_scale,
// kernel (TMLA_KERNEL_*), q_len, status int32 [1] or None) -> ().  The split workspace comes from
// the caching allocator on the current stream; the launches go on the current stream.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include "triton_mla_b200.h"

namespace {

int32_t dtype_code(at::ScalarType t) {
  switch (t) {
    case at::kBFloat16: return TMLA_DTYPE_BF16;
    case at::kHalf: return TMLA_DTYPE_FP16;
    case at::kFloat: return TMLA_DTYPE_FP32;
    default: TORCH_CHECK(false, "triton_mla.decode: q must be bfloat16, float16 or float32, got ", t);
  }
  return -1;
}

void decode_cuda(const at::Tensor& q, const at::Tensor& kv, const at::Tensor& lens,
                 const std::optional<at::Tensor>& block_table, const at::Tensor& out, const at::Tensor& lse,
                 int64_t num_splits, double softmax_scale, int64_t kernel, int64_t q_len,
                 const std::optional<at::Tensor>& status) {
  TORCH_CHECK(q.dim() == 3 && kv.dim() == 3, "triton_mla.decode: q [B, H, D] and kv_cache [N, P, D]");
  TORCH_CHECK(q.is_cuda() && kv.is_cuda() && lens.is_cuda() && out.is_cuda() && lse.is_cuda(),
              "triton_mla.decode: CUDA tensors only (there is no CPU implementation)");
  TORCH_CHECK(lens.scalar_type() == at::kInt && lens.dim() == 1 && lens.stride(0) == 1,
              "triton_mla.decode: cache_seqlens must be a contiguous int32 vector");
  TORCH_CHECK(lse.scalar_type() == at::kFloat && out.scalar_type() == q.scalar_type(),
              "triton_mla.decode: out in q's dtype, lse float32");
  const int64_t B = q.size(0), H = q.size(1), D = q.size(2), DV = out.size(2);
  TORCH_CHECK(out.dim() == 3 && out.size(0) == B && out.size(1) == H && out.stride(2) == 1,
              "triton_mla.decode: out must be [B, H, head_dim_v] with unit inner stride");
  TORCH_CHECK(lse.dim() == 2 && lse.size(0) == B && lse.size(1) == H && lse.stride(1) == 1,
              "triton_mla.decode: lse must be [B, H]");
  const bool fp8 = kv.scalar_type() == at::kByte;
  TmlaDecodeParams p = {};
  p.q = q.data_ptr();
  p.q_stride_b = q.stride(0);
  p.q_stride_h = q.stride(1);
  p.kv = kv.data_ptr();
  p.kv_stride_page = kv.stride(0);
  p.kv_stride_tok = kv.stride(1);
  p.page_size = (int32_t)kv.size(1);
  p.seqlens = lens.data_ptr<int32_t>();
  if (block_table.has_value()) {
    const at::Tensor& bt = *block_table;
    TORCH_CHECK(bt.scalar_type() == at::kInt && bt.dim() == 2 && bt.stride(1) == 1 && bt.is_cuda(),
                "triton_mla.decode: block_table must be int32 [B, W] with unit inner stride");
    p.block_table = bt.data_ptr<int32_t>();
    p.bt_stride = bt.stride(0);
    p.bt_width = (int32_t)bt.size(1);
    p.num_pages = kv.size(0);
  } else {
    p.num_pages = B;
  }
  p.out = out.data_ptr();
  p.out_stride_b = out.stride(0);
  p.out_stride_h = out.stride(1);
  p.lse = lse.data_ptr<float>();
  p.lse_stride_b = lse.stride(0);
  p.status = status.has_value() ? status->data_ptr<int32_t>() : nullptr;
  p.batch = (int32_t)B;
  p.num_heads = (int32_t)H;
  p.d_qk = (int32_t)D;
  p.d_v = (int32_t)DV;
  p.num_splits = (int32_t)num_splits;
  p.dtype = dtype_code(q.scalar_type());
  p.kernel = (int32_t)kernel;
  p.softmax_scale = (float)softmax_scale;
  p.q_len = (int32_t)q_len;
  p.kv_format = fp8 ? TMLA_KV_FP8_E4M3 : TMLA_KV_SAME;
  if (B == 0) return;
  const c10::cuda::CUDAGuard guard(q.device());
  const size_t ws_bytes = tmla_workspace_bytes(p.batch, p.num_heads, p.num_splits, p.d_v);
  at::Tensor ws;
  if (ws_bytes) {
    ws = at::empty({(int64_t)ws_bytes}, q.options().dtype(at::kByte));
    const size_t o_bytes = ((size_t)B * H * num_splits * DV * 4 + 255) & ~(size_t)255;
    p.ws_o = reinterpret_cast<float*>(ws.data_ptr());
    p.ws_lse = reinterpret_cast<float*>(static_cast<char*>(ws.data_ptr()) + o_bytes);
  }
  const cudaStream_t stream = c10::cuda::getCurrentCUDAStream(q.device().index()).stream();
  const int rc = tmla_decode(&p, stream);
  TORCH_CHECK(rc == TMLA_OK, "triton_mla.decode: ", tmla_error_string(rc), " ",
              rc == TMLA_ERR_CUDA ? tmla_last_cuda_error() : "");
}

// Shapes only: out and lse are written in place, so there is nothing to return.
void decode_meta(const at::Tensor&, const at::Tensor&, const at::Tensor&, const std::optional<at::Tensor>&,
                 const at::Tensor&, const at::Tensor&, int64_t, double, int64_t, int64_t,
                 const std::optional<at::Tensor>&) {}

}  // namespace

TORCH_LIBRARY(triton_mla, m) {
  m.def(
      "decode(Tensor q, Tensor kv_cache, Tensor cache_seqlens, Tensor? block_table, Tensor(a!) out, "
      "Tensor(b!) lse, int num_splits, float softmax_scale, int kernel, int q_len, Tensor? status) -> ()");
}

TORCH_LIBRARY_IMPL(triton_mla, CUDA, m) { m.impl("decode", &decode_cuda); }

TORCH_LIBRARY_IMPL(triton_mla, Meta, m) { m.impl("decode", &decode_meta); }
