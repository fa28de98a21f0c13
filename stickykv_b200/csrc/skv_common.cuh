// Shared device/host helpers for the stickykv_b200 kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "../../include/stickykv_b200.h"

namespace skv {

// Raise a kernel's dynamic shared-memory limit on the current device once:
// `done` is the caller's per-kernel bit set of devices already configured
// (devices 32 and up are configured on every call).
template <typename K>
inline void max_smem_once(std::atomic<uint32_t>& done, K kernel, int bytes) {
  int dev = 0;
  cudaGetDevice(&dev);
  const uint32_t bit = dev < 32 ? 1u << dev : 0u;
  if (bit && (done.load(std::memory_order_relaxed) & bit)) return;
  cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  done.fetch_or(bit, std::memory_order_relaxed);
}

constexpr int kPageTokens = 8;   // tokens per int4 page / per MMA half-tile
constexpr int kQGroup = 32;      // channels per int4 scale/zero group

// ---------------------------------------------------------------------------
// element types
// ---------------------------------------------------------------------------
template <typename T> struct Elt;
template <> struct Elt<float> {
  static __device__ __forceinline__ float load(const float* p) { return *p; }
  static __device__ __forceinline__ float to_f32(float x) { return x; }
  static __device__ __forceinline__ float from_f32(float x) { return x; }
};
template <> struct Elt<__half> {
  static __device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from_f32(float x) { return __float2half_rn(x); }
};
template <> struct Elt<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_f32(float x) { return __float2bfloat16_rn(x); }
};

template <typename T>
__device__ __forceinline__ float ld_f32(const T* p) { return Elt<T>::to_f32(*p); }
template <typename T>
__device__ __forceinline__ void st_f32(T* p, float x) { *p = Elt<T>::from_f32(x); }
// Round an fp32 value to T (round to nearest even) and back: the rounding
// torch applies after every elementwise op on a T tensor.
template <typename T>
__device__ __forceinline__ float rnd(float x) { return Elt<T>::to_f32(Elt<T>::from_f32(x)); }

// ---------------------------------------------------------------------------
// RoPE strip + re-apply with the reference's rounding
// (transformers apply_rotary_pos_emb: round(round(k*cos) + round(rot(k)*sin))
// with cos/sin rounded to T), used by the eviction kernel.  (x, y) are the
// channels (i, i+D/2) of one key; c/s the fp32 table entries.
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ void rope_strip_apply(float& x, float& y, float c_old, float s_old,
                                                 float c_new, float s_new) {
  const float co = rnd<T>(c_old), so = rnd<T>(s_old);
  const float cn = rnd<T>(c_new), sn = rnd<T>(s_new);
  // strip: cos, -sin
  float ux = rnd<T>(__fadd_rn(rnd<T>(__fmul_rn(x, co)), rnd<T>(__fmul_rn(-y, -so))));
  float uy = rnd<T>(__fadd_rn(rnd<T>(__fmul_rn(y, co)), rnd<T>(__fmul_rn(x, -so))));
  // re-apply: cos, sin
  x = rnd<T>(__fadd_rn(rnd<T>(__fmul_rn(ux, cn)), rnd<T>(__fmul_rn(-uy, sn))));
  y = rnd<T>(__fadd_rn(rnd<T>(__fmul_rn(uy, cn)), rnd<T>(__fmul_rn(ux, sn))));
}

// Post-RoPE key channel pair at position p -> page-relative frame
// R(r8) R(-p) (fp32, no fused multiply-add so the host oracle reproduces it).
__device__ __forceinline__ void to_page_frame(float& x, float& y, float c, float s, float c8,
                                              float s8) {
  const float xs = __fadd_rn(__fmul_rn(x, c), __fmul_rn(y, s));
  const float ys = __fsub_rn(__fmul_rn(y, c), __fmul_rn(x, s));
  x = __fsub_rn(__fmul_rn(xs, c8), __fmul_rn(ys, s8));
  y = __fadd_rn(__fmul_rn(ys, c8), __fmul_rn(xs, s8));
}

// ---------------------------------------------------------------------------
// int4 page layout (8 tokens of K and V; see skv_pack_pages)
//   K codes  [row r][lane t (4)][word w (D/32)] u32: nibble i   = ch 2t+8(4w+i)
//                                                   nibble i+4 = ch 2t+8(4w+i)+1
//   K scales [row r][group][scale, zero] f16
//   V codes  [pair t (4)][row g (8)][word w] u32:  nibble i   = token 2t,   ch g+8(4w+i)
//                                                   nibble i+4 = token 2t+1, ch g+8(4w+i)
//   V scales [pair t][group][s(2t), s(2t+1), z(2t), z(2t+1)] f16
// ---------------------------------------------------------------------------
__host__ __device__ constexpr int page_bytes(int D) { return 2 * kPageTokens * (D / 2 + (D / kQGroup) * 4); }
__host__ __device__ constexpr int page_k_codes_off(int) { return 0; }
__host__ __device__ constexpr int page_k_scales_off(int D) { return kPageTokens * D / 2; }
__host__ __device__ constexpr int page_v_codes_off(int D) { return kPageTokens * (D / 2 + (D / kQGroup) * 4); }
__host__ __device__ constexpr int page_v_scales_off(int D) { return page_v_codes_off(D) + kPageTokens * D / 2; }

// code of K channel d of page row r
__device__ __forceinline__ int page_k_code(const uint8_t* page, int D, int r, int d) {
  const int t = (d & 7) >> 1, j = d >> 3, w = j >> 2, i = j & 3, hi = d & 1;
  const uint32_t word = reinterpret_cast<const uint32_t*>(page)[(r * 4 + t) * (D / 32) + w];
  return (word >> (4 * (i + 4 * hi))) & 0xF;
}
__device__ __forceinline__ int page_v_code(const uint8_t* page, int D, int r, int d) {
  const int t = r >> 1, hi = r & 1, g = d & 7, j = d >> 3, w = j >> 2, i = j & 3;
  const uint32_t word =
      reinterpret_cast<const uint32_t*>(page + page_v_codes_off(D))[(t * 8 + g) * (D / 32) + w];
  return (word >> (4 * (i + 4 * hi))) & 0xF;
}
__device__ __forceinline__ float2 page_k_sz(const uint8_t* page, int D, int r, int grp) {
  const __half* s = reinterpret_cast<const __half*>(page + page_k_scales_off(D));
  return make_float2(__half2float(s[(r * (D / 32) + grp) * 2]), __half2float(s[(r * (D / 32) + grp) * 2 + 1]));
}
__device__ __forceinline__ float2 page_v_sz(const uint8_t* page, int D, int r, int grp) {
  const __half* s = reinterpret_cast<const __half*>(page + page_v_scales_off(D));
  const int t = r >> 1, hi = r & 1;
  const __half* e = s + ((t * (D / 32) + grp) * 4);
  return make_float2(__half2float(e[hi]), __half2float(e[2 + hi]));
}

// ---------------------------------------------------------------------------
// misc
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// programmatic dependent launch: a primary grid lets its dependent grid start
// early; the dependent waits (in hardware, not by spinning) for the primary's
// completion and memory before it reads what the primary wrote.  In a grid
// launched without the attribute the wait returns at once.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void grid_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;\n" ::); }

__host__ __device__ inline int ceil_div(int a, int b) { return (a + b - 1) / b; }
__host__ __device__ inline int64_t ceil_div64(int64_t a, int64_t b) { return (a + b - 1) / b; }
__host__ __device__ inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// logical layout helpers (identical for every row)
struct Geometry {
  int s;        // num_sink
  int s_pad;    // sinks rounded up to 8
  int ws;       // window size
  int T;        // logical tokens
  int n_tier;   // tier tokens (pages * 8)
  __host__ __device__ int sinks_present() const { return T < s ? T : s; }
  __host__ __device__ int rest_tokens() const { return T > s ? T - s - n_tier : 0; }
  __host__ __device__ int num_windows() const { return T > s ? (T - s + ws - 1) / ws : 0; }
  // fp slot of a logical position in the sink or rest region
  __host__ __device__ int fp_slot(int pos) const { return pos < s ? pos : s_pad + (pos - s - n_tier); }
};

// parameters of the prefill kernels (skv_prefill.cu, skv_prefill_mma.cu)
struct PrefillParams {
  const void* q;  // [B][Hq][T][D]
  const void* k;  // [B][Hkv][T][D]
  const void* v;
  void* out;      // [B][T][Hq][D]
  float* lse;     // [B][Hq][T]
  float* colmass; // [B][Hq][T]
  float* scores;  // [B][Hq][cap] (+=)
  int B, Hq, Hkv, T, D, cap, s, ws;
  float scaling;
};

// parameters of the eviction kernels (skv_evict.cu), filled by skv_capi.cu
struct EvictParams {
  // geometry
  int B, Hq, Hkv, D, s, s_pad, ws, ppw;
  int T_old, n_tier_old_tok, W, E, kprime, local_w, R, T_new, n_tier_new_tok;
  int tier;
  int scores_cap, page_cap, fp_cap_src, fp_cap_dst;
  int dtype;
  // buffers
  const float* scores_src;
  float* scores_dst;
  const int64_t* ids_src;
  int64_t* ids_dst;
  int32_t* retained;   // [B][R] (workspace)
  int32_t* entrant;    // [B][kprime] source window or -1 (workspace)
  uint32_t* keys;      // [B][E] orderable head-mean scores (workspace)
  int32_t* retained_out;
  int64_t next_window_id;
  const int32_t* table_src;
  int32_t* table_dst;
  uint8_t* pages;
  const void* k_src;
  const void* v_src;
  void* k_dst;
  void* v_dst;
  const float* cos;
  const float* sin;
  // this step's token when its append rides in the eviction (else null):
  // [B][Hkv][D] with element strides new_sb, new_sh, logical position T_old - 1
  const void* k_new;
  const void* v_new;
  int64_t new_sb, new_sh;
};

}  // namespace skv

// host-side error helpers (defined in skv_capi.cu)
namespace skv {
void set_cuda_error(cudaError_t e);
}

#define SKV_CHECK_LAUNCH()                                   \
  do {                                                       \
    cudaError_t _e = cudaGetLastError();                     \
    if (_e != cudaSuccess) {                                 \
      skv::set_cuda_error(_e);                               \
      return SKV_ERR_CUDA;                                   \
    }                                                        \
  } while (0)
