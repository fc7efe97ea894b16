// Decode entry point that allocates nothing.
//
// Who needs it.  `tmla_decode` takes its split workspace from the caller, which
// PyTorch callers get from the caching allocator.  Some callers of this C ABI
// cannot allocate device memory for it.
//  * A plain C / C++ / FFI host that binds the library without PyTorch has no
//    device allocator of its own.
//  * A serving loop may not be allowed to call cudaMalloc on the hot path,
//    because it can synchronise the whole device.
// `tmla_decode_noalloc` serves them: inputs and outputs are still the caller's;
// the split partials go to a fixed array of device memory owned by the library.
//
// Rules (also in include/triton_mla_b200.h):
//  * The array is TMLA_NOALLOC_SCRATCH_BYTES (32 MiB) of device memory on every
//    GPU that loads the library, held until the process exits.  A call whose
//    split workspace (tmla_workspace_bytes) is larger returns TMLA_ERR_WORKSPACE
//    before touching the GPU.  A call with num_splits == 1 uses no scratch.
//  * The array's device address is looked up once per device, by the first call
//    made with that device current (cudaGetSymbolAddress); make that first call
//    before any stream capture.  The address is kept for the life of the process:
//    after a cudaDeviceReset the cached address is stale, so do not call this entry
//    point again in a process that reset its device.
//  * All calls share the one array, so calls that can overlap on the GPU (on
//    different streams or from different host threads) race on it.  Calls on
//    one stream run in order and are safe.
//  * Nothing in the array has to start at zero: a call writes every partial it
//    later reads (empty splits included).
// It allocates nothing: no cudaMalloc, no cudaFree, no allocating library call.
#include <mutex>

#include "tmla_common.cuh"

namespace {

constexpr size_t kScratchBytes = TMLA_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_tmla_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
void* g_scratch_device_ptr[kMaxDevices] = {};
std::mutex g_scratch_mutex;

// Device address of g_tmla_scratch on the current device (the host-side name
// is only a stand-in and must never be passed to a kernel).
int scratch_on_current_device(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return TMLA_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (!g_scratch_device_ptr[dev]) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_tmla_scratch) != cudaSuccess || !ptr) return TMLA_ERR_CUDA;
    g_scratch_device_ptr[dev] = ptr;
  }
  *out = g_scratch_device_ptr[dev];
  return TMLA_OK;
}

}  // namespace

extern "C" int tmla_decode_noalloc(const TmlaDecodeParams* p, void* stream) {
  if (!p) return TMLA_ERR_INVALID_ARG;
  TmlaDecodeParams q = *p;
  q.ws_o = nullptr;
  q.ws_lse = nullptr;
  // A whole decode: as in tmla_decode, the stage-1-only flag does not apply (and with one
  // split it would ask for a workspace this call does not attach).
  q.flags &= ~TMLA_FLAG_PARTIAL_ONLY;
  const size_t need = tmla_workspace_bytes(q.batch, q.num_heads, q.num_splits, q.d_v);
  if (need > kScratchBytes) return TMLA_ERR_WORKSPACE;
  if (need > 0) {
    void* base = nullptr;
    const int rc = scratch_on_current_device(&base);
    if (rc) return rc;
    const size_t rows = (size_t)q.batch * q.num_heads * q.num_splits;
    const size_t o_bytes = (rows * q.d_v * sizeof(float) + 255) & ~(size_t)255;
    q.ws_o = static_cast<float*>(base);
    q.ws_lse = reinterpret_cast<float*>(static_cast<unsigned char*>(base) + o_bytes);
  }
  return tmla_decode(&q, stream);
}
