// skv_append: write new post-RoPE K/V tokens into the fp store in place.
// Replaces the per-step torch.cat of CacheState.append
// (modules/windowed_cache/state.py:94-95), which re-copies the whole cache.
#include "skv_common.cuh"

namespace skv {

// One thread per 16-byte chunk of one token's K or V row.
template <typename T>
__global__ void append_kernel(T* __restrict__ k_fp, T* __restrict__ v_fp, const T* __restrict__ k_new,
                              const T* __restrict__ v_new, int64_t sb, int64_t sh, int64_t st, int H,
                              int D, int cap, Geometry geo, int n_new) {
  const int per_row = D * (int)sizeof(T) / 16;  // 16-byte chunks per token row
  const int64_t total = (int64_t)gridDim.y * H * n_new * per_row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < (int64_t)H * n_new * per_row * 2;
       i += (int64_t)gridDim.x * blockDim.x) {
    (void)total;
    int64_t rem = i;
    const int chunk = (int)(rem % per_row); rem /= per_row;
    const int t = (int)(rem % n_new); rem /= n_new;
    const int h = (int)(rem % H); rem /= H;
    const int which = (int)rem;  // 0 = K, 1 = V
    const int b = blockIdx.y;
    const int pos = geo.T + t;
    const int slot = geo.fp_slot(pos);
    const T* src = (which ? v_new : k_new) + b * sb + h * sh + t * st;
    T* dst = (which ? v_fp : k_fp) + (((int64_t)b * H + h) * cap + slot) * D;
    reinterpret_cast<uint4*>(dst)[chunk] = reinterpret_cast<const uint4*>(src)[chunk];
  }
}

template <typename T>
int launch_append(const skv_layer_desc* L, int seq_len, int tier_pages, const void* k_new,
                  const void* v_new, int64_t sb, int64_t sh, int64_t st, int n_new, cudaStream_t stream) {
  Geometry geo{L->num_sink, L->sink_pad, L->window_size, seq_len, tier_pages * kPageTokens};
  const int H = L->num_kv_heads, D = L->head_dim;
  const int64_t work = (int64_t)H * n_new * (D * (int)sizeof(T) / 16) * 2;
  const int threads = 256;
  int blocks = (int)ceil_div64(work, threads);
  if (blocks > 4096) blocks = 4096;
  dim3 grid(blocks, L->batch);
  append_kernel<T><<<grid, threads, 0, stream>>>((T*)L->k_fp, (T*)L->v_fp, (const T*)k_new,
                                                 (const T*)v_new, sb, sh, st, H, D, L->fp_capacity,
                                                 geo, n_new);
  SKV_CHECK_LAUNCH();
  return SKV_OK;
}

int append_dispatch(const skv_layer_desc* L, int seq_len, int tier_pages, const void* k_new,
                    const void* v_new, int64_t sb, int64_t sh, int64_t st, int n_new,
                    cudaStream_t stream) {
  switch (L->kv_dtype) {
    case SKV_F32: return launch_append<float>(L, seq_len, tier_pages, k_new, v_new, sb, sh, st, n_new, stream);
    case SKV_F16: return launch_append<__half>(L, seq_len, tier_pages, k_new, v_new, sb, sh, st, n_new, stream);
    case SKV_BF16: return launch_append<__nv_bfloat16>(L, seq_len, tier_pages, k_new, v_new, sb, sh, st, n_new, stream);
  }
  return SKV_ERR_UNSUPPORTED;
}

}  // namespace skv
