// Prefill attention + causal column mass (window scores of the prompt).
//
// Replaces the prefill branch of the flash score hook
// (modules/windowed_cache/hooks.py:245-290: chunked softmax(q·kᵀ) with a
// causal mask, summed over the query rows, reduced to windows) and, in the
// same pass, produces the prompt's attention output, so the prompt's K is not
// re-read by a second attention kernel.
//
// Portable CUDA-core version (fp32, and head dims without a tensor-core
// kernel; fp16/bf16 at head_dim 64/128 run skv_prefill_mma.cu): pass 1 computes each row's output and
// log-sum-exp with an online softmax (one warp per query row); pass 2 sums
// exp(s_ij - lse_i) over rows i >= j for each key column j (one warp per
// column); pass 3 reduces the column mass to windows in a fixed order.
#include <float.h>

#include "skv_common.cuh"

namespace skv {

constexpr int kMaxDPerLane = 4;  // head_dim <= 128

template <typename T>
__global__ void __launch_bounds__(128) prefill_rows_kernel(PrefillParams p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int i = blockIdx.x * 4 + warp;
  const int h = blockIdx.y, b = blockIdx.z;
  if (i >= p.T) return;
  const int G = p.Hq / p.Hkv, kh = h / G;
  const T* q = (const T*)p.q + (((int64_t)b * p.Hq + h) * p.T + i) * p.D;
  const T* kb = (const T*)p.k + ((int64_t)b * p.Hkv + kh) * p.T * p.D;
  const T* vb = (const T*)p.v + ((int64_t)b * p.Hkv + kh) * p.T * p.D;
  float qr[kMaxDPerLane], acc[kMaxDPerLane];
#pragma unroll
  for (int e = 0; e < kMaxDPerLane; ++e) {
    const int d = lane + 32 * e;
    qr[e] = d < p.D ? ld_f32(q + d) : 0.f;
    acc[e] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  for (int j = 0; j <= i; ++j) {
    float dot = 0.f;
#pragma unroll
    for (int e = 0; e < kMaxDPerLane; ++e) {
      const int d = lane + 32 * e;
      if (d < p.D) dot += qr[e] * ld_f32(kb + (int64_t)j * p.D + d);
    }
    const float sc = warp_sum(dot) * p.scaling;
    const float mn = fmaxf(m, sc);
    const float alpha = expf(m - mn), pr = expf(sc - mn);
    l = l * alpha + pr;
#pragma unroll
    for (int e = 0; e < kMaxDPerLane; ++e) {
      const int d = lane + 32 * e;
      if (d < p.D) acc[e] = acc[e] * alpha + pr * ld_f32(vb + (int64_t)j * p.D + d);
    }
    m = mn;
  }
  T* o = (T*)p.out + (((int64_t)b * p.T + i) * p.Hq + h) * p.D;
#pragma unroll
  for (int e = 0; e < kMaxDPerLane; ++e) {
    const int d = lane + 32 * e;
    if (d < p.D) st_f32(o + d, acc[e] / l);
  }
  if (lane == 0) p.lse[((int64_t)b * p.Hq + h) * p.T + i] = m + logf(l);
}

template <typename T>
__global__ void __launch_bounds__(128) prefill_cols_kernel(PrefillParams p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int j = blockIdx.x * 4 + warp;
  const int h = blockIdx.y, b = blockIdx.z;
  if (j >= p.T) return;
  const int G = p.Hq / p.Hkv, kh = h / G;
  const T* kr = (const T*)p.k + (((int64_t)b * p.Hkv + kh) * p.T + j) * p.D;
  const T* qb = (const T*)p.q + ((int64_t)b * p.Hq + h) * p.T * p.D;
  const float* lse = p.lse + ((int64_t)b * p.Hq + h) * p.T;
  float kv[kMaxDPerLane];
#pragma unroll
  for (int e = 0; e < kMaxDPerLane; ++e) {
    const int d = lane + 32 * e;
    kv[e] = d < p.D ? ld_f32(kr + d) : 0.f;
  }
  float mass = 0.f;
  for (int i = j; i < p.T; ++i) {
    float dot = 0.f;
#pragma unroll
    for (int e = 0; e < kMaxDPerLane; ++e) {
      const int d = lane + 32 * e;
      if (d < p.D) dot += kv[e] * ld_f32(qb + (int64_t)i * p.D + d);
    }
    const float sc = warp_sum(dot) * p.scaling;
    mass += expf(sc - lse[i]);
  }
  if (lane == 0) p.colmass[((int64_t)b * p.Hq + h) * p.T + j] = mass;
}

__global__ void prefill_windows_kernel(PrefillParams p) {
  const int h = blockIdx.y, b = blockIdx.z;
  const int W = p.T > p.s ? (p.T - p.s + p.ws - 1) / p.ws : 0;
  const float* cm = p.colmass + ((int64_t)b * p.Hq + h) * p.T;
  float* dst = p.scores + ((int64_t)b * p.Hq + h) * p.cap;
  for (int w = blockIdx.x * blockDim.x + threadIdx.x; w < W; w += gridDim.x * blockDim.x) {
    const int a = p.s + w * p.ws, e = min(p.T, a + p.ws);
    float sum = 0.f;
    for (int t = a; t < e; ++t) sum += cm[t];
    dst[w] += sum;
  }
}

size_t prefill_ws_size(const skv_layer_desc* L, int T) {
  return 2 * align_up((size_t)L->batch * L->num_q_heads * T * 4, 256);
}

template <typename T>
int launch_prefill(PrefillParams& p, cudaStream_t stream) {
  dim3 grid(ceil_div(p.T, 4), p.Hq, p.B);
  prefill_rows_kernel<T><<<grid, 128, 0, stream>>>(p);
  SKV_CHECK_LAUNCH();
  if (p.scores) {
    prefill_cols_kernel<T><<<grid, 128, 0, stream>>>(p);
    SKV_CHECK_LAUNCH();
    dim3 g2(ceil_div(ceil_div(p.T, p.ws), 128), p.Hq, p.B);
    prefill_windows_kernel<<<g2, 128, 0, stream>>>(p);
    SKV_CHECK_LAUNCH();
  }
  return SKV_OK;
}

bool prefill_mma_supported(const skv_layer_desc* L);
int prefill_mma(const PrefillParams& p, int dtype, bool colmass, cudaStream_t stream);

int prefill_dispatch(const skv_layer_desc* L, int T, const void* q, const void* k, const void* v,
                     void* out, float scaling, float* scores, int scores_cap, void* ws,
                     cudaStream_t stream) {
  PrefillParams p{};
  p.q = q; p.k = k; p.v = v; p.out = out;
  const size_t one = align_up((size_t)L->batch * L->num_q_heads * T * 4, 256);
  p.lse = (float*)ws;
  p.colmass = (float*)((char*)ws + one);
  p.scores = scores;
  p.B = L->batch; p.Hq = L->num_q_heads; p.Hkv = L->num_kv_heads; p.T = T; p.D = L->head_dim;
  p.cap = scores_cap; p.s = L->num_sink; p.ws = L->window_size; p.scaling = scaling;
  if (prefill_mma_supported(L)) {  // tensor cores: output + lse, column mass, then windows
    int rc = prefill_mma(p, L->kv_dtype, scores != nullptr, stream);
    if (rc || !scores) return rc;
    dim3 g2(ceil_div(ceil_div(p.T, p.ws), 128), p.Hq, p.B);
    prefill_windows_kernel<<<g2, 128, 0, stream>>>(p);
    SKV_CHECK_LAUNCH();
    return SKV_OK;
  }
  switch (L->kv_dtype) {
    case SKV_F32: return launch_prefill<float>(p, stream);
    case SKV_F16: return launch_prefill<__half>(p, stream);
    case SKV_BF16: return launch_prefill<__nv_bfloat16>(p, stream);
  }
  return SKV_ERR_UNSUPPORTED;
}

}  // namespace skv
