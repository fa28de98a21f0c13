// Tensor-core decode path (fp16/bf16, window_size % 8 == 0): see the kernel
// notes below.  Until it is enabled every decode runs the portable path.
#include "skv_common.cuh"

namespace skv {

bool decode_mma_supported(const skv_layer_desc*) { return false; }
size_t decode_mma_ws_size(const skv_layer_desc*, int) { return 0; }
int decode_mma(const skv_layer_desc*, int, int, const void*, int64_t, int64_t, void*, int64_t,
               int64_t, float, float*, int, void*, cudaStream_t) {
  return SKV_ERR_UNSUPPORTED;
}

}  // namespace skv
