// Placeholder: the tcgen05 kernel lands here.
#include "tmla_common.cuh"
namespace tmla {
int sm100_supported(const TmlaDecodeParams&) { return 0; }
int launch_sm100(const TmlaDecodeParams&, cudaStream_t) { return TMLA_ERR_UNSUPPORTED; }
}  // namespace tmla
