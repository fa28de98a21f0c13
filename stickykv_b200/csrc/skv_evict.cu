// Eviction: select -> compact -> re-rotate -> quantise, without a host sync.
//
// Replaces the eviction block of WindowedCache.update
// (modules/windowed_cache/cache.py:230-286):
//   EvictionPolicy.compute_retain_window_indices  policy.py:81-146
//   EvictionPolicy.expand_to_token_indices        policy.py:152-209 (the
//       .item() host sync at :202 is gone: every row keeps the same count,
//       computed on the host by skv_evict_plan_compute)
//   CacheState.slice_and_keep                      state.py:125-159
//   CacheState.rerotate_keys                       state.py:165-232
//   window_scores / original_window_ids gather     cache.py:271-283
// and adds the demotion of kept windows into the int4 tier (design.md:130-187).
//
// Kernel 1 (select): one CTA per row.  Head-mean of the window scores, exact
// top-k by a radix select on 64-bit keys (score bits, then inverted window
// index so the lowest index wins ties), chronological compaction, the
// score/id gather and, with the tier, the new page table.
// Kernel 2 (move): fp tokens that stay fp are copied to the destination store
// with their keys stripped at the old and re-applied at the new position,
// op by op in the KV dtype like the reference.
// Kernel 3 (demote): kept fp windows entering the tier are rotated into their
// page frame and quantised to int4 pages, one warp per page.
#include <float.h>

#include "skv_common.cuh"

namespace skv {

// EvictParams is declared in skv_common.cuh


__device__ __forceinline__ uint32_t orderable(float f) {
  f = f + 0.0f;  // -0 -> +0
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Block-wide exclusive scan of one int per thread (blockDim.x <= 1024).
__device__ int block_excl_scan(int v, int* smem, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) smem[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int s = lane < nw ? smem[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    if (lane < nw) smem[lane] = s;
  }
  __syncthreads();
  const int warp_off = warp > 0 ? smem[warp - 1] : 0;
  total = smem[nw - 1];
  __syncthreads();
  return warp_off + x - v;
}

constexpr int kSelectThreads = 512;
// score/id slots initialised past the retained windows at each eviction: a
// decode step adds at most two windows before the next eviction.
constexpr int kTailWindows = 8;

__global__ void __launch_bounds__(kSelectThreads) evict_select_kernel(EvictParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int b = blockIdx.x;
  const int tid = threadIdx.x, nt = blockDim.x;
  uint64_t* keys = reinterpret_cast<uint64_t*>(smem_raw);                 // [E]
  int* hist = reinterpret_cast<int*>(keys + (p.E > 0 ? p.E : 1));           // [256]
  int* scan = hist + 256;                                                   // [32]
  int* ret = scan + 32;                                                     // [R]
  int* free_list = ret + (p.R > 0 ? p.R : 1);                               // [page_cap]
  unsigned char* used = reinterpret_cast<unsigned char*>(free_list + (p.tier ? p.page_cap : 0));
  __shared__ uint64_t s_thr;
  __shared__ int s_krem;

  const int E = p.E, k = p.kprime;
  // 1. head-mean keys over the evictable prefix
  if (k > 0 && k < E) {
    for (int w = tid; w < E; w += nt) {
      float acc = 0.f;
      for (int h = 0; h < p.Hq; ++h) acc = __fadd_rn(acc, p.scores_src[((int64_t)b * p.Hq + h) * p.scores_cap + w]);
      const float mean = __fdiv_rn(acc, (float)p.Hq);
      keys[w] = ((uint64_t)orderable(mean) << 32) | (uint64_t)(0xFFFFFFFFu - (uint32_t)w);
    }
    __syncthreads();
    // 2. radix select of the k-th largest key (keys are unique)
    uint64_t prefix = 0, pmask = 0;
    if (tid == 0) s_krem = k;
    for (int shift = 56; shift >= 0; shift -= 8) {
      for (int i = tid; i < 256; i += nt) hist[i] = 0;
      __syncthreads();
      for (int w = tid; w < E; w += nt) {
        const uint64_t key = keys[w];
        if ((key & pmask) == prefix) atomicAdd(&hist[(key >> shift) & 255], 1);
      }
      __syncthreads();
      if (tid == 0) {
        int krem = s_krem, cum = 0, d = 255;
        for (; d >= 0; --d) {
          if (cum + hist[d] >= krem) break;
          cum += hist[d];
        }
        s_krem = krem - cum;
        s_thr = (uint64_t)d;
      }
      __syncthreads();
      prefix |= s_thr << shift;
      pmask |= (uint64_t)255 << shift;
      __syncthreads();
    }
    if (tid == 0) s_thr = prefix;
    __syncthreads();
  }
  // 3. chronological positions of the kept evictable windows
  const int per = (E + nt - 1) / nt;
  const int w0 = tid * per, w1 = min(E, w0 + per);
  const uint64_t thr = (k > 0 && k < E) ? s_thr : 0;
  auto kept = [&](int w) -> bool {
    if (k == 0) return false;
    if (k >= E) return true;
    return keys[w] >= thr;
  };
  int cnt = 0;
  for (int w = w0; w < w1; ++w) cnt += kept(w) ? 1 : 0;
  int total = 0;
  int pos = block_excl_scan(cnt, scan, total);
  for (int w = w0; w < w1; ++w)
    if (kept(w)) ret[pos++] = w;
  for (int i = tid; i < p.local_w; i += nt) ret[k + i] = E + i;
  __syncthreads();
  // 4. retained list, score and id gather, zero the next windows
  for (int j = tid; j < p.R; j += nt) {
    p.retained[(int64_t)b * p.R + j] = ret[j];
    if (p.retained_out) p.retained_out[(int64_t)b * p.scores_cap + j] = ret[j];
    p.ids_dst[(int64_t)b * p.scores_cap + j] = p.ids_src[(int64_t)b * p.scores_cap + ret[j]];
  }
  // windows that appear before the next eviction start from zero score and
  // take ids from the running counter (cache.py:180-213)
  const int ztail = min(p.scores_cap - p.R, kTailWindows);
  for (int i = tid; i < ztail; i += nt)
    p.ids_dst[(int64_t)b * p.scores_cap + p.R + i] = p.next_window_id + i;
  for (int e = tid; e < p.Hq * (p.R + ztail); e += nt) {
    const int h = e / (p.R + ztail), j = e % (p.R + ztail);
    float* dst = p.scores_dst + ((int64_t)b * p.Hq + h) * p.scores_cap;
    dst[j] = j < p.R ? p.scores_src[((int64_t)b * p.Hq + h) * p.scores_cap + ret[j]] : 0.f;
  }
  if (!p.tier) return;
  // 5. int4 tier page table: kept tier windows keep their pages, entrants get
  //    the lowest free pages in chronological order.
  const int n_tw_old = p.n_tier_old_tok / p.ws;
  for (int i = tid; i < p.page_cap; i += nt) used[i] = 0;
  __syncthreads();
  for (int j = tid; j < k; j += nt) {
    const int w = ret[j];
    if (w < n_tw_old) {
      for (int i = 0; i < p.ppw; ++i) {
        const int pg = p.table_src[(int64_t)b * p.page_cap + w * p.ppw + i];
        used[pg] = 1;
        p.table_dst[(int64_t)b * p.page_cap + j * p.ppw + i] = pg;
      }
      p.entrant[(int64_t)b * k + j] = -1;
    } else {
      p.entrant[(int64_t)b * k + j] = w;
    }
  }
  __syncthreads();
  // free-page ranks (chunked block scan over the pool)
  const int pper = (p.page_cap + nt - 1) / nt;
  const int p0 = tid * pper, p1 = min(p.page_cap, p0 + pper);
  int fcnt = 0;
  for (int i = p0; i < p1; ++i) fcnt += used[i] ? 0 : 1;
  int ftot = 0;
  int fpos = block_excl_scan(fcnt, scan, ftot);
  // entrant ranks
  const int eper = (k + nt - 1) / nt;
  const int e0 = tid * eper, e1 = min(k, e0 + eper);
  int ecnt = 0;
  for (int j = e0; j < e1; ++j) ecnt += (ret[j] >= n_tw_old) ? 1 : 0;
  int etot = 0;
  int epos = block_excl_scan(ecnt, scan, etot);
  for (int i = p0; i < p1; ++i)
    if (!used[i]) free_list[fpos++] = i;
  __syncthreads();
  for (int j = e0; j < e1; ++j) {
    if (ret[j] >= n_tw_old) {
      for (int i = 0; i < p.ppw; ++i)
        p.table_dst[(int64_t)b * p.page_cap + j * p.ppw + i] = free_list[epos * p.ppw + i];
      ++epos;
    }
  }
}

// Copy fp tokens that stay fp into the destination store, keys re-rotated.
template <typename T>
__global__ void evict_move_kernel(EvictParams p, int n_fp_tok) {
  const int b = blockIdx.z, h = blockIdx.y;
  const int half = p.D / 2;
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (idx >= (int64_t)n_fp_tok * half) return;
  const int tau = (int)(idx / half), i = (int)(idx % half);
  const int s_eff = min(p.s, p.T_old);
  int old_pos, new_pos;
  if (tau < s_eff) {
    old_pos = new_pos = tau;
  } else {
    const int f = tau - s_eff;
    const int jf = f / p.ws, r = f % p.ws;
    const int j = p.tier ? p.kprime + jf : jf;
    const int w = p.tier ? p.E + jf : p.retained[(int64_t)b * p.R + j];
    old_pos = p.s + w * p.ws + r;
    new_pos = p.s + j * p.ws + r;
  }
  const Geometry go{p.s, p.s_pad, p.ws, p.T_old, p.n_tier_old_tok};
  const Geometry gn{p.s, p.s_pad, p.ws, p.T_new, p.n_tier_new_tok};
  const int src = go.fp_slot(old_pos), dst = gn.fp_slot(new_pos);
  const int64_t rs = (((int64_t)b * p.Hkv + h) * p.fp_cap_src + src) * p.D;
  const int64_t rd = (((int64_t)b * p.Hkv + h) * p.fp_cap_dst + dst) * p.D;
  const T* ks = (const T*)p.k_src + rs;
  const T* vs = (const T*)p.v_src + rs;
  T* kd = (T*)p.k_dst + rd;
  T* vd = (T*)p.v_dst + rd;
  float x = ld_f32(ks + i), y = ld_f32(ks + i + half);
  rope_strip_apply<T>(x, y, p.cos[(int64_t)old_pos * half + i], p.sin[(int64_t)old_pos * half + i],
                      p.cos[(int64_t)new_pos * half + i], p.sin[(int64_t)new_pos * half + i]);
  st_f32(kd + i, x);
  st_f32(kd + i + half, y);
  vd[i] = vs[i];
  vd[i + half] = vs[i + half];
}

// Quantise one 8-token page (keys rotated to the page frame) and pack it.
// `kin(r, c)` / `vin(r, c)` give token r channel c as fp32; `pos0` is the
// logical position of row 0 (row r sits at pos0 + r; the page starts at a
// multiple of 8 past the sinks).  One warp; smem scratch of 2*8*D codes.
template <typename KF, typename VF>
__device__ void quantize_page_warp(KF kin, VF vin, int D, int pos0, const float* cos, const float* sin,
                                   uint8_t* page, uint8_t* sc) {
  const int lane = threadIdx.x & 31;
  const int half = D / 2, ng = D / kQGroup;
  uint8_t* kc = sc;
  uint8_t* vc = sc + 8 * D;
  __half* kscl = reinterpret_cast<__half*>(page + page_k_scales_off(D));
  __half* vscl = reinterpret_cast<__half*>(page + page_v_scales_off(D));
  for (int task = lane; task < 2 * 8 * ng; task += 32) {
    const int which = task / (8 * ng);  // 0 = K, 1 = V
    const int r = (task / ng) % 8, gq = task % ng;
    float v[kQGroup];
    float mn = FLT_MAX, mx = -FLT_MAX;
    for (int e = 0; e < kQGroup; ++e) {
      const int c = gq * kQGroup + e;
      float val;
      if (which == 0) {
        const int cp = c % half;
        float x = kin(r, cp), y = kin(r, cp + half);
        const int pos = pos0 + r;
        to_page_frame(x, y, cos[(int64_t)pos * half + cp], sin[(int64_t)pos * half + cp],
                      cos[(int64_t)r * half + cp], sin[(int64_t)r * half + cp]);
        val = c < half ? x : y;
      } else {
        val = vin(r, c);
      }
      v[e] = val;
      mn = fminf(mn, val);
      mx = fmaxf(mx, val);
    }
    const __half s16 = __float2half_rn(__fdiv_rn(__fsub_rn(mx, mn), 15.f));
    const __half z16 = __float2half_rn(mn);
    const float s = __half2float(s16), z = __half2float(z16);
    uint8_t* codes = (which ? vc : kc) + r * D + gq * kQGroup;
    for (int e = 0; e < kQGroup; ++e) {
      int q = 0;
      if (s != 0.f) {
        float t = rintf(__fdiv_rn(__fsub_rn(v[e], z), s));
        t = fminf(fmaxf(t, 0.f), 15.f);
        q = (int)t;
      }
      codes[e] = (uint8_t)q;
    }
    if (which == 0) {
      kscl[(r * ng + gq) * 2] = s16;
      kscl[(r * ng + gq) * 2 + 1] = z16;
    } else {
      __half* e4 = vscl + ((r >> 1) * ng + gq) * 4;
      e4[r & 1] = s16;
      e4[2 + (r & 1)] = z16;
    }
  }
  __syncwarp();
  uint32_t* kw = reinterpret_cast<uint32_t*>(page);
  for (int idx = lane; idx < 8 * 4 * ng; idx += 32) {
    const int r = idx / (4 * ng), t = (idx / ng) % 4, w = idx % ng;
    uint32_t word = 0;
    for (int i = 0; i < 4; ++i) {
      const int ch = 2 * t + 8 * (4 * w + i);
      word |= (uint32_t)kc[r * D + ch] << (4 * i);
      word |= (uint32_t)kc[r * D + ch + 1] << (4 * (i + 4));
    }
    kw[idx] = word;
  }
  uint32_t* vw = reinterpret_cast<uint32_t*>(page + page_v_codes_off(D));
  for (int idx = lane; idx < 4 * 8 * ng; idx += 32) {
    const int t = idx / (8 * ng), g = (idx / ng) % 8, w = idx % ng;
    uint32_t word = 0;
    for (int i = 0; i < 4; ++i) {
      const int ch = g + 8 * (4 * w + i);
      word |= (uint32_t)vc[(2 * t) * D + ch] << (4 * i);
      word |= (uint32_t)vc[(2 * t + 1) * D + ch] << (4 * (i + 4));
    }
    vw[idx] = word;
  }
  __syncwarp();
}

constexpr int kDemoteWarps = 4;

template <typename T>
__global__ void __launch_bounds__(32 * kDemoteWarps) evict_demote_kernel(EvictParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int b = blockIdx.z, h = blockIdx.y;
  const int warp = threadIdx.x >> 5;
  const int task = blockIdx.x * kDemoteWarps + warp;  // (j, page i)
  if (task >= p.kprime * p.ppw) return;
  const int j = task / p.ppw, pi = task % p.ppw;
  const int w = p.entrant[(int64_t)b * p.kprime + j];
  if (w < 0) return;
  const int pos0 = p.s + w * p.ws + pi * kPageTokens;
  const Geometry go{p.s, p.s_pad, p.ws, p.T_old, p.n_tier_old_tok};
  const int slot0 = go.fp_slot(pos0);
  const int64_t rb = (((int64_t)b * p.Hkv + h) * p.fp_cap_src + slot0) * p.D;
  const T* ks = (const T*)p.k_src + rb;
  const T* vs = (const T*)p.v_src + rb;
  const int D = p.D;
  const int phys = p.table_dst[(int64_t)b * p.page_cap + j * p.ppw + pi];
  uint8_t* page = p.pages + (((int64_t)b * p.Hkv + h) * p.page_cap + phys) * page_bytes(D);
  quantize_page_warp([&](int r, int c) { return ld_f32(ks + (int64_t)r * D + c); },
                     [&](int r, int c) { return ld_f32(vs + (int64_t)r * D + c); }, D, pos0, p.cos,
                     p.sin, page, smem_raw + warp * 2 * 8 * D);
}

template <typename T>
__global__ void __launch_bounds__(32 * kDemoteWarps) pack_pages_kernel(const T* k, const T* v, int D,
                                                                       int first_pos, int n_pages,
                                                                       const float* cos, const float* sin,
                                                                       uint8_t* out) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int warp = threadIdx.x >> 5;
  const int pg = blockIdx.x * kDemoteWarps + warp;
  if (pg >= n_pages) return;
  const T* ks = k + (int64_t)pg * 8 * D;
  const T* vs = v + (int64_t)pg * 8 * D;
  quantize_page_warp([&](int r, int c) { return ld_f32(ks + (int64_t)r * D + c); },
                     [&](int r, int c) { return ld_f32(vs + (int64_t)r * D + c); }, D,
                     first_pos + pg * 8, cos, sin, out + (int64_t)pg * page_bytes(D),
                     smem_raw + warp * 2 * 8 * D);
}

size_t select_smem_bytes(int E, int R, int page_cap) {
  return (size_t)8 * (E > 0 ? E : 1) + 4 * (256 + 32) + 4 * (size_t)(R > 0 ? R : 1) +
         5 * (size_t)page_cap + 16;
}

template <typename T>
int launch_evict(EvictParams& p, cudaStream_t stream) {
  const size_t smem = select_smem_bytes(p.E, p.R, p.tier ? p.page_cap : 0);
  if (smem > 200 * 1024) return SKV_ERR_CAPACITY;
  cudaFuncSetAttribute(evict_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  evict_select_kernel<<<p.B, kSelectThreads, smem, stream>>>(p);
  SKV_CHECK_LAUNCH();
  const int n_fp_tok = p.T_new - p.n_tier_new_tok;  // sinks + fp windows kept
  if (n_fp_tok > 0) {
    const int64_t work = (int64_t)n_fp_tok * (p.D / 2);
    dim3 grid((unsigned)ceil_div64(work, 256), p.Hkv, p.B);
    evict_move_kernel<T><<<grid, 256, 0, stream>>>(p, n_fp_tok);
    SKV_CHECK_LAUNCH();
  }
  if (p.tier && p.kprime > 0) {
    dim3 grid((unsigned)ceil_div(p.kprime * p.ppw, kDemoteWarps), p.Hkv, p.B);
    evict_demote_kernel<T><<<grid, 32 * kDemoteWarps, kDemoteWarps * 2 * 8 * p.D, stream>>>(p);
    SKV_CHECK_LAUNCH();
  }
  return SKV_OK;
}

int evict_dispatch(EvictParams& p, cudaStream_t stream) {
  switch (p.dtype) {
    case SKV_F32: return launch_evict<float>(p, stream);
    case SKV_F16: return launch_evict<__half>(p, stream);
    case SKV_BF16: return launch_evict<__nv_bfloat16>(p, stream);
  }
  return SKV_ERR_UNSUPPORTED;
}

int pack_pages_dispatch(const skv_layer_desc* L, const void* k, const void* v, int first_pos,
                        int n_pages, uint8_t* out, cudaStream_t stream) {
  const int D = L->head_dim;
  dim3 grid(ceil_div(n_pages, kDemoteWarps));
  const size_t smem = kDemoteWarps * 2 * 8 * D;
  switch (L->kv_dtype) {
    case SKV_F32:
      pack_pages_kernel<float><<<grid, 32 * kDemoteWarps, smem, stream>>>(
          (const float*)k, (const float*)v, D, first_pos, n_pages, L->rope_cos, L->rope_sin, out);
      break;
    case SKV_F16:
      pack_pages_kernel<__half><<<grid, 32 * kDemoteWarps, smem, stream>>>(
          (const __half*)k, (const __half*)v, D, first_pos, n_pages, L->rope_cos, L->rope_sin, out);
      break;
    case SKV_BF16:
      pack_pages_kernel<__nv_bfloat16><<<grid, 32 * kDemoteWarps, smem, stream>>>(
          (const __nv_bfloat16*)k, (const __nv_bfloat16*)v, D, first_pos, n_pages, L->rope_cos,
          L->rope_sin, out);
      break;
    default:
      return SKV_ERR_UNSUPPORTED;
  }
  SKV_CHECK_LAUNCH();
  return SKV_OK;
}

}  // namespace skv
