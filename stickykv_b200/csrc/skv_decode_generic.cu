// Decode attention with per-window attention mass — portable CUDA-core path.
//
// Replaces, for one decode query per row, HF eager attention + the score
// hook (modules/windowed_eager_cache/hooks.py:145-180; flash variant
// modules/windowed_cache/hooks.py:199-290) + scorer.compute_window_scores
// (modules/windowed_cache/scorer.py:17-90) + accumulate (scorer.py:93-109).
//
// This path covers every dtype (fp32 included), head size and window size.
// It materialises the fp32 logits (4 B per token and query head) so that the
// merge can turn them into exact normalised window mass.  The tensor-core
// path (skv_decode_mma.cu) is used instead for fp16/bf16 with window_size 8.
//
// Work split: one CTA per (row, kv head, token range); four warps; a warp
// handles four tokens per iteration with eight lanes per token, each lane
// owning D/16 channel pairs (c, c + D/2) of all G query heads of the group.
#include <float.h>

#include "skv_common.cuh"

namespace skv {

struct DecodeParams {
  const void* k_fp;
  const void* v_fp;
  const uint8_t* pages;
  const int32_t* table;
  const float* cos;
  const float* sin;
  const void* q;
  void* out;
  float* scores;       // [B][Hq][scores_cap] accumulator (may be null)
  float* logits;       // workspace [B][Hq][T_pad]
  float* part;         // workspace [B][Hkv][n_split][G][D+2]
  int64_t q_sb, q_sh, o_sb, o_sh;
  int B, Hkv, cap, page_cap, T_pad, n_split, chunk, scores_cap;
  float scaling;
  Geometry geo;
};

template <typename T, int D, int G>
__global__ void __launch_bounds__(128) decode_generic_kernel(DecodeParams p) {
  constexpr int H8 = D / 16;  // channel pairs per lane
  const int b = blockIdx.z, kh = blockIdx.y, split = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = lane >> 3, sub = lane & 7;
  const Geometry& geo = p.geo;
  const int t0 = split * p.chunk;
  const int t1 = min(geo.T, t0 + p.chunk);
  const int Hq = p.Hkv * G;

  float qx[G][H8], qy[G][H8];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const T* q = (const T*)p.q + b * p.q_sb + (kh * G + g) * p.q_sh;
#pragma unroll
    for (int i = 0; i < H8; ++i) {
      qx[g][i] = ld_f32(q + sub * H8 + i);
      qy[g][i] = ld_f32(q + D / 2 + sub * H8 + i);
    }
  }
  float m[G], l[G], ax[G][H8], ay[G][H8];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int i = 0; i < H8; ++i) ax[g][i] = ay[g][i] = 0.f;
  }
  const T* kbase = (const T*)p.k_fp + ((int64_t)b * p.Hkv + kh) * p.cap * D;
  const T* vbase = (const T*)p.v_fp + ((int64_t)b * p.Hkv + kh) * p.cap * D;
  const int n_tier = geo.n_tier;
  const int pb = page_bytes(D);

  for (int base = t0 + warp * 4; base < t1; base += 16) {
    const int tok = base + grp;
    const bool valid = tok < t1;
    float kx[H8], ky[H8], vx[H8], vy[H8];
    float rqx[G][H8], rqy[G][H8];
    bool tier = valid && tok >= geo.s && tok < geo.s + n_tier;
    if (tier) {
      const int rel = tok - geo.s;
      const int page = rel >> 3, r = rel & 7;
      const int phys = p.table[b * p.page_cap + page];
      const uint8_t* pg = p.pages + (((int64_t)b * p.Hkv + kh) * p.page_cap + phys) * pb;
      const int P = geo.s + page * kPageTokens;
#pragma unroll
      for (int i = 0; i < H8; ++i) {
        const int cx = sub * H8 + i, cy = cx + D / 2;
        const float2 szx = page_k_sz(pg, D, r, cx / kQGroup), szy = page_k_sz(pg, D, r, cy / kQGroup);
        kx[i] = fmaf((float)page_k_code(pg, D, r, cx), szx.x, szx.y);
        ky[i] = fmaf((float)page_k_code(pg, D, r, cy), szy.x, szy.y);
        const float2 vzx = page_v_sz(pg, D, r, cx / kQGroup), vzy = page_v_sz(pg, D, r, cy / kQGroup);
        vx[i] = fmaf((float)page_v_code(pg, D, r, cx), vzx.x, vzx.y);
        vy[i] = fmaf((float)page_v_code(pg, D, r, cy), vzy.x, vzy.y);
        const float c = p.cos[(int64_t)P * (D / 2) + cx], s = p.sin[(int64_t)P * (D / 2) + cx];
#pragma unroll
        for (int g = 0; g < G; ++g) {
          rqx[g][i] = qx[g][i] * c + qy[g][i] * s;
          rqy[g][i] = qy[g][i] * c - qx[g][i] * s;
        }
      }
    } else {
      const int slot = valid ? geo.fp_slot(tok) : 0;
      const T* kr = kbase + (int64_t)slot * D;
      const T* vr = vbase + (int64_t)slot * D;
#pragma unroll
      for (int i = 0; i < H8; ++i) {
        const int cx = sub * H8 + i;
        kx[i] = valid ? ld_f32(kr + cx) : 0.f;
        ky[i] = valid ? ld_f32(kr + cx + D / 2) : 0.f;
        vx[i] = valid ? ld_f32(vr + cx) : 0.f;
        vy[i] = valid ? ld_f32(vr + cx + D / 2) : 0.f;
#pragma unroll
        for (int g = 0; g < G; ++g) {
          rqx[g][i] = qx[g][i];
          rqy[g][i] = qy[g][i];
        }
      }
    }
    float sc[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float d = 0.f;
#pragma unroll
      for (int i = 0; i < H8; ++i) d += rqx[g][i] * kx[i] + rqy[g][i] * ky[i];
      d += __shfl_xor_sync(0xffffffffu, d, 1);
      d += __shfl_xor_sync(0xffffffffu, d, 2);
      d += __shfl_xor_sync(0xffffffffu, d, 4);
      sc[g] = valid ? d * p.scaling : -INFINITY;
      if (valid && sub == g % 8) p.logits[((int64_t)b * Hq + kh * G + g) * p.T_pad + tok] = sc[g];
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float mx = fmaxf(sc[g], __shfl_xor_sync(0xffffffffu, sc[g], 8));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
      const float m_new = fmaxf(m[g], mx);
      if (m_new == -INFINITY) continue;  // warp-uniform: nothing valid yet
      const float alpha = __expf(m[g] - m_new);
      const float pr = valid ? __expf(sc[g] - m_new) : 0.f;
      float ps = pr + __shfl_xor_sync(0xffffffffu, pr, 8);
      ps += __shfl_xor_sync(0xffffffffu, ps, 16);
      l[g] = l[g] * alpha + ps;
      m[g] = m_new;
#pragma unroll
      for (int i = 0; i < H8; ++i) {
        ax[g][i] = ax[g][i] * alpha + pr * vx[i];
        ay[g][i] = ay[g][i] * alpha + pr * vy[i];
      }
    }
  }
  // reduce the four token groups of the warp (same channels, same m)
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int i = 0; i < H8; ++i) {
      ax[g][i] += __shfl_xor_sync(0xffffffffu, ax[g][i], 8);
      ax[g][i] += __shfl_xor_sync(0xffffffffu, ax[g][i], 16);
      ay[g][i] += __shfl_xor_sync(0xffffffffu, ay[g][i], 8);
      ay[g][i] += __shfl_xor_sync(0xffffffffu, ay[g][i], 16);
    }
  // merge the four warps
  __shared__ float sm_m[4][G], sm_l[4][G];
  __shared__ float sm_o[4][G][D];
  if (lane == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) { sm_m[warp][g] = m[g]; sm_l[warp][g] = l[g]; }
  }
  if (grp == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int i = 0; i < H8; ++i) {
        sm_o[warp][g][sub * H8 + i] = ax[g][i];
        sm_o[warp][g][D / 2 + sub * H8 + i] = ay[g][i];
      }
  }
  __syncthreads();
  float* part = p.part + (((int64_t)b * p.Hkv + kh) * p.n_split + split) * G * (D + 2);
  for (int e = threadIdx.x; e < G * (D + 2); e += blockDim.x) {
    const int g = e / (D + 2), c = e % (D + 2);
    float M = -INFINITY;
    for (int w = 0; w < 4; ++w) M = fmaxf(M, sm_m[w][g]);
    float acc = 0.f;
    for (int w = 0; w < 4; ++w) {
      if (sm_m[w][g] == -INFINITY) continue;
      const float f = __expf(sm_m[w][g] - M);
      acc += f * (c == D ? 0.f : (c == D + 1 ? sm_l[w][g] : sm_o[w][g][c]));
    }
    part[e] = (c == D) ? M : acc;
  }
}

// Combine split partials per (row, query head); normalise; add window mass.
template <typename T, int D, int G>
__global__ void __launch_bounds__(256) decode_merge_kernel(DecodeParams p) {
  const int b = blockIdx.y, h = blockIdx.x;
  const int kh = h / G, g = h % G;
  const int Hq = p.Hkv * G;
  __shared__ float s_M, s_L;
  __shared__ float s_f[256];
  const float* part = p.part + ((int64_t)b * p.Hkv + kh) * p.n_split * G * (D + 2);
  if (threadIdx.x == 0) {
    float M = -INFINITY;
    for (int s = 0; s < p.n_split; ++s) M = fmaxf(M, part[(s * G + g) * (D + 2) + D]);
    float L = 0.f;
    for (int s = 0; s < p.n_split; ++s) {
      const float ms = part[(s * G + g) * (D + 2) + D];
      if (ms != -INFINITY) L += __expf(ms - M) * part[(s * G + g) * (D + 2) + D + 1];
    }
    s_M = M;
    s_L = L;
  }
  __syncthreads();
  const float M = s_M, invL = 1.f / s_L;
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < p.n_split; ++s) {
      const float ms = part[(s * G + g) * (D + 2) + D];
      if (ms != -INFINITY) acc += __expf(ms - M) * part[(s * G + g) * (D + 2) + c];
    }
    st_f32((T*)p.out + b * p.o_sb + h * p.o_sh + c, acc * invL);
  }
  (void)s_f;
  if (p.scores == nullptr) return;
  const Geometry& geo = p.geo;
  const int W = geo.num_windows();
  const float* lg = p.logits + ((int64_t)b * Hq + h) * p.T_pad;
  float* acc = p.scores + ((int64_t)b * Hq + h) * p.scores_cap;
  for (int w = threadIdx.x; w < W; w += blockDim.x) {
    const int a = geo.s + w * geo.ws;
    const int e = min(geo.T, a + geo.ws);
    float sum = 0.f;
    for (int t = a; t < e; ++t) sum += __expf(lg[t] - M) * invL;
    acc[w] += sum;
  }
}

template <typename T, int D, int G>
int launch_decode_generic(DecodeParams& p, cudaStream_t stream) {
  dim3 grid(p.n_split, p.Hkv, p.B);
  decode_generic_kernel<T, D, G><<<grid, 128, 0, stream>>>(p);
  SKV_CHECK_LAUNCH();
  dim3 mgrid(p.Hkv * G, p.B);
  decode_merge_kernel<T, D, G><<<mgrid, 256, 0, stream>>>(p);
  SKV_CHECK_LAUNCH();
  return SKV_OK;
}

template <typename T, int D>
int dispatch_g(DecodeParams& p, int G, cudaStream_t s) {
  switch (G) {
    case 1: return launch_decode_generic<T, D, 1>(p, s);
    case 2: return launch_decode_generic<T, D, 2>(p, s);
    case 3: return launch_decode_generic<T, D, 3>(p, s);
    case 4: return launch_decode_generic<T, D, 4>(p, s);
    case 5: return launch_decode_generic<T, D, 5>(p, s);
    case 6: return launch_decode_generic<T, D, 6>(p, s);
    case 7: return launch_decode_generic<T, D, 7>(p, s);
    case 8: return launch_decode_generic<T, D, 8>(p, s);
  }
  return SKV_ERR_UNSUPPORTED;
}

template <typename T>
int dispatch_d(DecodeParams& p, int D, int G, cudaStream_t s) {
  switch (D) {
    case 16: return dispatch_g<T, 16>(p, G, s);
    case 32: return dispatch_g<T, 32>(p, G, s);
    case 64: return dispatch_g<T, 64>(p, G, s);
    case 128: return dispatch_g<T, 128>(p, G, s);
  }
  return SKV_ERR_UNSUPPORTED;
}

// workspace layout shared with the size query
struct GenericWs {
  int n_split, chunk, T_pad;
  size_t logits_bytes, part_bytes, total;
};

GenericWs generic_ws(const skv_layer_desc* L, int T) {
  GenericWs w{};
  const int G = L->num_q_heads / L->num_kv_heads;
  const int units = L->batch * L->num_kv_heads;
  int target = ceil_div(4 * 148, units > 0 ? units : 1);
  int chunk = ceil_div(T > 0 ? T : 1, target);
  chunk = ((chunk + 63) / 64) * 64;
  if (chunk < 64) chunk = 64;
  w.chunk = chunk;
  w.n_split = ceil_div(T > 0 ? T : 1, chunk);
  w.T_pad = (int)align_up((size_t)(T > 0 ? T : 1), 4);
  w.logits_bytes = align_up((size_t)L->batch * L->num_q_heads * w.T_pad * 4, 256);
  w.part_bytes = align_up((size_t)L->batch * L->num_kv_heads * w.n_split * G * (L->head_dim + 2) * 4, 256);
  w.total = w.logits_bytes + w.part_bytes;
  return w;
}

size_t decode_generic_ws_size(const skv_layer_desc* L, int T) { return generic_ws(L, T).total; }

int decode_generic(const skv_layer_desc* L, int T, int tier_pages, const void* q, int64_t q_sb,
                   int64_t q_sh, void* out, int64_t o_sb, int64_t o_sh, float scaling,
                   float* scores, int scores_cap, void* ws, cudaStream_t stream) {
  const GenericWs w = generic_ws(L, T);
  DecodeParams p{};
  p.k_fp = L->k_fp;
  p.v_fp = L->v_fp;
  p.pages = L->tier_pages;
  p.table = L->tier_table;
  p.cos = L->rope_cos;
  p.sin = L->rope_sin;
  p.q = q;
  p.out = out;
  p.scores = scores;
  p.logits = (float*)ws;
  p.part = (float*)((char*)ws + w.logits_bytes);
  p.q_sb = q_sb; p.q_sh = q_sh; p.o_sb = o_sb; p.o_sh = o_sh;
  p.B = L->batch; p.Hkv = L->num_kv_heads; p.cap = L->fp_capacity;
  p.page_cap = L->tier_page_capacity;
  p.T_pad = w.T_pad; p.n_split = w.n_split; p.chunk = w.chunk; p.scores_cap = scores_cap;
  p.scaling = scaling;
  p.geo = Geometry{L->num_sink, L->sink_pad, L->window_size, T, tier_pages * kPageTokens};
  const int G = L->num_q_heads / L->num_kv_heads;
  switch (L->kv_dtype) {
    case SKV_F32: return dispatch_d<float>(p, L->head_dim, G, stream);
    case SKV_F16: return dispatch_d<__half>(p, L->head_dim, G, stream);
    case SKV_BF16: return dispatch_d<__nv_bfloat16>(p, L->head_dim, G, stream);
  }
  return SKV_ERR_UNSUPPORTED;
}

}  // namespace skv
