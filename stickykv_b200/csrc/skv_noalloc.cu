// skv_decode_attention_noalloc: decode attention whose scratch lives in a
// fixed device array owned by this library, for callers that cannot allocate
// device memory (see the declaration in include/stickykv_b200.h).
#include <mutex>

#include "skv_common.cuh"

// Scratch shared by every call on a device.  Each GPU context that loads this
// library reserves SKV_NOALLOC_SCRATCH_BYTES for it until the process exits.
static __device__ __align__(256) unsigned char g_noalloc_scratch[SKV_NOALLOC_SCRATCH_BYTES];

namespace skv {
int decode_precheck(const skv_layer_desc* L, int32_t T, int32_t tier_pages, const void* q, void* out,
                    float* scores, int32_t scores_cap);
}

namespace {

constexpr int kMaxDevices = 64;
// Host code cannot use g_noalloc_scratch as a pointer: its name is a host-side
// stand-in.  The device address is looked up once per device, with that
// device current, and cached here.
void* g_scratch_ptr[kMaxDevices];
cudaError_t g_scratch_err[kMaxDevices];
std::once_flag g_scratch_once[kMaxDevices];

}  // namespace

extern "C" int skv_decode_attention_noalloc(const skv_layer_desc* layer, int32_t seq_len,
                                            int32_t tier_pages, const void* q, int64_t q_stride_b,
                                            int64_t q_stride_h, void* out, int64_t out_stride_b,
                                            int64_t out_stride_h, float scaling, float* window_scores,
                                            int32_t scores_capacity, void* stream) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    skv::set_cuda_error(e);
    return SKV_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) return SKV_ERR_UNSUPPORTED;
  std::call_once(g_scratch_once[dev], [dev] {
    g_scratch_err[dev] = cudaGetSymbolAddress(&g_scratch_ptr[dev], g_noalloc_scratch);
  });
  if (g_scratch_err[dev] != cudaSuccess || g_scratch_ptr[dev] == nullptr) {
    skv::set_cuda_error(g_scratch_err[dev]);
    return SKV_ERR_CUDA;
  }
  // the same argument checks, in the same order, as skv_decode_attention,
  // so both entry points return the same status for the same bad input
  const int rc = skv::decode_precheck(layer, seq_len, tier_pages, q, out, window_scores, scores_capacity);
  if (rc != SKV_OK) return rc;
  const size_t need = skv_decode_workspace_size(layer, seq_len);
  if (need > (size_t)SKV_NOALLOC_SCRATCH_BYTES) return SKV_ERR_CAPACITY;
  // Every scratch byte the decode kernels read is written earlier in the same
  // call, so nothing needs clearing between calls.
  return skv_decode_attention(layer, seq_len, tier_pages, q, q_stride_b, q_stride_h, out,
                              out_stride_b, out_stride_h, scaling, window_scores, scores_capacity,
                              g_scratch_ptr[dev], (size_t)SKV_NOALLOC_SCRATCH_BYTES, stream);
}
