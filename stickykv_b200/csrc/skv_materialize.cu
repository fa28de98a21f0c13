// skv_materialize: the retained cache as plain [B][Hkv][T][D] keys and values
// in logical order (the reference's CacheState.key_states / value_states,
// modules/windowed_cache/state.py:20-35, read by its flash score hook,
// modules/windowed_cache/hooks.py:218, and its parity runner).  Sinks and
// the tokens after the tier are copied from the fp store; int4 tier tokens are
// dequantised (code * scale + zero in fp32, as the tier format defines) and
// their keys rotated from the page frame to their current position: a tier
// key stored as R(r8) R(-p) k sits at page start P + r8, so its post-RoPE key
// is R(P) times the stored vector.  Not on the decode path: a compatibility
// read, one thread per (token, channel pair).
#include "skv_common.cuh"

namespace skv {
namespace {

template <typename T, int D>
__global__ void materialize_kernel(skv_layer_desc L, int T_len, int tier_pages, T* k_out, T* v_out) {
  constexpr int half = D / 2;
  const int h = blockIdx.y, b = blockIdx.z;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  const int t = idx / half, i = idx % half;
  if (t >= T_len) return;
  const int s_eff = min(L.num_sink, T_len), n_tier = tier_pages * kPageTokens;
  const int64_t row = ((int64_t)b * L.num_kv_heads + h) * T_len + t;
  T* ko = k_out + row * D;
  T* vo = v_out + row * D;
  if (t >= s_eff && t < L.num_sink + n_tier) {
    const int pg = (t - L.num_sink) / kPageTokens, r = (t - L.num_sink) % kPageTokens;
    const int phys = L.tier_table[(int64_t)b * L.tier_page_capacity + pg];
    const uint8_t* page = L.tier_pages + (((int64_t)b * L.num_kv_heads + h) * L.tier_page_capacity + phys) * page_bytes(D);
    const float2 sx = page_k_sz(page, D, r, i / kQGroup), sy = page_k_sz(page, D, r, (i + half) / kQGroup);
    const float x = __fadd_rn(__fmul_rn((float)page_k_code(page, D, r, i), sx.x), sx.y);
    const float y = __fadd_rn(__fmul_rn((float)page_k_code(page, D, r, i + half), sy.x), sy.y);
    const int P = L.num_sink + pg * kPageTokens;
    const float c = L.rope_cos[(int64_t)P * half + i], sn = L.rope_sin[(int64_t)P * half + i];
    st_f32(ko + i, __fsub_rn(__fmul_rn(x, c), __fmul_rn(y, sn)));
    st_f32(ko + i + half, __fadd_rn(__fmul_rn(y, c), __fmul_rn(x, sn)));
    const float2 vx = page_v_sz(page, D, r, i / kQGroup), vy = page_v_sz(page, D, r, (i + half) / kQGroup);
    st_f32(vo + i, __fadd_rn(__fmul_rn((float)page_v_code(page, D, r, i), vx.x), vx.y));
    st_f32(vo + i + half, __fadd_rn(__fmul_rn((float)page_v_code(page, D, r, i + half), vy.x), vy.y));
    return;
  }
  const Geometry g{L.num_sink, L.sink_pad, L.window_size, T_len, n_tier};
  const int64_t src = (((int64_t)b * L.num_kv_heads + h) * L.fp_capacity + g.fp_slot(t)) * D;
  const T* ks = (const T*)L.k_fp + src;
  const T* vs = (const T*)L.v_fp + src;
  ko[i] = ks[i];
  ko[i + half] = ks[i + half];
  vo[i] = vs[i];
  vo[i + half] = vs[i + half];
}

template <typename T>
int launch_materialize(const skv_layer_desc* L, int T_len, int tier_pages, void* k_out, void* v_out,
                       cudaStream_t stream) {
  constexpr int kThreads = 256;
  const int D = L->head_dim;
  const dim3 grid(ceil_div(T_len * (D / 2), kThreads), L->num_kv_heads, L->batch);
  switch (D) {
    case 16: materialize_kernel<T, 16><<<grid, kThreads, 0, stream>>>(*L, T_len, tier_pages, (T*)k_out, (T*)v_out); break;
    case 32: materialize_kernel<T, 32><<<grid, kThreads, 0, stream>>>(*L, T_len, tier_pages, (T*)k_out, (T*)v_out); break;
    case 64: materialize_kernel<T, 64><<<grid, kThreads, 0, stream>>>(*L, T_len, tier_pages, (T*)k_out, (T*)v_out); break;
    case 128: materialize_kernel<T, 128><<<grid, kThreads, 0, stream>>>(*L, T_len, tier_pages, (T*)k_out, (T*)v_out); break;
    default: return SKV_ERR_UNSUPPORTED;
  }
  SKV_CHECK_LAUNCH();
  return SKV_OK;
}

}  // namespace

int materialize_dispatch(const skv_layer_desc* L, int T_len, int tier_pages, void* k_out, void* v_out,
                         cudaStream_t stream) {
  switch (L->kv_dtype) {
    case SKV_F32: return launch_materialize<float>(L, T_len, tier_pages, k_out, v_out, stream);
    case SKV_F16: return launch_materialize<__half>(L, T_len, tier_pages, k_out, v_out, stream);
    case SKV_BF16: return launch_materialize<__nv_bfloat16>(L, T_len, tier_pages, k_out, v_out, stream);
  }
  return SKV_ERR_UNSUPPORTED;
}

}  // namespace skv
