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
// top-k by a radix select on the orderable score bits (the lowest window
// index wins ties: among keys equal to the threshold the first ones in window
// order are kept), chronological compaction and, with the tier, the new page
// table.
// Kernel 2 (apply): the fp tokens that stay fp are copied to the destination
// store with their keys stripped at the old and re-applied at the new
// position, op by op in the KV dtype like the reference; kept fp windows
// entering the tier are rotated into their page frame and quantised to int4
// pages (a block per page); scores and ids are gathered.
#include <float.h>

#include <type_traits>

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

// The kept candidate windows that enter the int4 tier, by rank: at most
// min(candidates, top-k) per row, the rest -1.  The selects write the list
// into the row's head-mean keys, which they have read by then (and the
// apply's demotion blocks, one per (entrant rank, page), read it).
__host__ __device__ inline int entrant_cap_of(int E, int n_tw_old, int kprime) {
  const int n_cand = E - n_tw_old;
  return n_cand < kprime ? n_cand : kprime;
}
__device__ inline int entrant_cap(const EvictParams& p) { return entrant_cap_of(p.E, p.n_tier_old_tok / p.ws, p.kprime); }
__device__ inline int* entrant_list(const EvictParams& p, int b) {
  return reinterpret_cast<int*>(p.keys) + (int64_t)b * p.E;
}

constexpr int kSelectThreads = 1024;
constexpr int kSelectSmemMax = 200 * 1024;  // dynamic shared memory a select may use
// score/id slots initialised past the retained windows at each eviction: a
// decode step adds at most two windows before the next eviction.
constexpr int kTailWindows = 8;

// Head-mean keys of the evictable windows (policy.py:112 window_scores.mean
// over query heads; heads summed in order h = 0..Hq-1 in fp32, then divided),
// as orderable bits: one thread per (row, window) over the whole GPU, so the
// 32 heads' scores of a row stream in parallel rather than through the one
// CTA that selects for the row.
constexpr int kKeysThreads = 256;
__global__ void __launch_bounds__(kKeysThreads) evict_keys_kernel(EvictParams p) {
  grid_launch_dependents();  // the select kernel stages its page table meanwhile
  const int b = blockIdx.y, w = blockIdx.x * kKeysThreads + threadIdx.x;
  if (w >= p.E) return;
  const float* rowp = p.scores_src + (int64_t)b * p.Hq * p.scores_cap + w;
  float acc = 0.f;
  int h = 0;
  for (; h + 32 <= p.Hq; h += 32) {  // loads issued 32 at a time: one round trip at 32 heads
    float v[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = rowp[(int64_t)(h + i) * p.scores_cap];
#pragma unroll
    for (int i = 0; i < 32; ++i) acc = __fadd_rn(acc, v[i]);
  }
  for (; h + 8 <= p.Hq; h += 8) {
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = rowp[(int64_t)(h + i) * p.scores_cap];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc = __fadd_rn(acc, v[i]);
  }
  for (; h < p.Hq; ++h) acc = __fadd_rn(acc, rowp[(int64_t)h * p.scores_cap]);
  p.keys[(int64_t)b * p.E + w] = orderable(__fdiv_rn(acc, (float)p.Hq));
}

__global__ void __launch_bounds__(kSelectThreads) evict_select_kernel(EvictParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int b = blockIdx.x;
  const int tid = threadIdx.x, nt = blockDim.x;
  grid_launch_dependents();  // the apply kernel's blocks that read the selection wait for it
  uint32_t* keys = reinterpret_cast<uint32_t*>(smem_raw);                   // [E]
  int* hist = reinterpret_cast<int*>(keys + (p.E > 0 ? p.E : 1));           // [256]
  int* scan = hist + 256;                                                   // [32]
  int* ret = scan + 32;                                                     // [R]
  int* free_list = ret + (p.R > 0 ? p.R : 1);                               // [page_cap]
  unsigned char* used = reinterpret_cast<unsigned char*>(free_list + (p.tier ? p.page_cap : 0));
  __shared__ uint32_t s_digit;
  __shared__ int s_krem;

  const int E = p.E, k = p.kprime;
  const bool partial = k > 0 && k < E;
  // 1. head-mean keys over the evictable prefix (orderable float bits)
  uint32_t thr = 0;
  int krem = 0;  // keys equal to thr that are kept, lowest window index first
  grid_dependency_wait();  // the head-mean keys (evict_keys_kernel)
  if (partial) {
    for (int w = tid; w < E; w += nt) keys[w] = p.keys[(int64_t)b * E + w];
    if (tid == 0) s_krem = k;
    // 2. radix select of the k-th largest key, 8 bits per pass
    uint32_t prefix = 0, pmask = 0;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int i = tid; i < 256; i += nt) hist[i] = 0;
      __syncthreads();
      for (int w = tid; w < E; w += nt) {
        const uint32_t key = keys[w];
        if ((key & pmask) == prefix) atomicAdd(&hist[(key >> shift) & 255], 1);
      }
      __syncthreads();
      if (tid < 32) {  // one warp finds the digit holding the krem-th largest key
        const int kr = s_krem;
        int cnt[8], tot = 0;
#pragma unroll
        for (int q = 0; q < 8; ++q) { cnt[q] = hist[255 - (tid * 8 + q)]; tot += cnt[q]; }
        int incl = tot;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int y = __shfl_up_sync(0xffffffffu, incl, o);
          if (tid >= o) incl += y;
        }
        const int excl = incl - tot;
        const unsigned own = __ballot_sync(0xffffffffu, excl < kr && kr <= incl);
        if (tid == __ffs(own) - 1) {
          int c = excl;
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            if (c + cnt[q] >= kr) {
              s_digit = (uint32_t)(255 - (tid * 8 + q));
              s_krem = kr - c;
              break;
            }
            c += cnt[q];
          }
        }
      }
      __syncthreads();
      prefix |= s_digit << shift;
      pmask |= 255u << shift;
    }
    thr = prefix;
    krem = s_krem;
  }
  // 3. chronological positions of the kept evictable windows: keys above the
  //    threshold, and the first krem windows whose key equals it
  const int per = (E + nt - 1) / nt;
  const int w0 = tid * per, w1 = min(E, w0 + per);
  int n_eq = 0;
  if (partial)
    for (int w = w0; w < w1; ++w) n_eq += keys[w] == thr ? 1 : 0;
  int eq_total = 0;
  int eq_rank = block_excl_scan(n_eq, scan, eq_total);
  auto kept = [&](int w, int& rank) -> bool {
    if (k == 0) return false;
    if (k >= E) return true;
    const uint32_t key = keys[w];
    if (key != thr) return key > thr;
    return rank++ < krem;
  };
  int cnt = 0;
  {
    int r = eq_rank;
    for (int w = w0; w < w1; ++w) cnt += kept(w, r) ? 1 : 0;
  }
  int total = 0;
  int pos = block_excl_scan(cnt, scan, total);
  {
    int r = eq_rank;
    for (int w = w0; w < w1; ++w)
      if (kept(w, r)) ret[pos++] = w;
  }
  for (int i = tid; i < p.local_w; i += nt) ret[k + i] = E + i;
  __syncthreads();
  // 4. retained list (the score/id gather runs in the apply kernel)
  for (int j = tid; j < p.R; j += nt) {
    p.retained[(int64_t)b * p.R + j] = ret[j];
    if (p.retained_out) p.retained_out[(int64_t)b * p.scores_cap + j] = ret[j];
  }
  if (!p.tier) return;
  // 5. int4 tier page table: kept tier windows keep their pages, entrants get
  //    the lowest free pages in chronological order.
  const int n_tw_old = p.n_tier_old_tok / p.ws;
  for (int i = tid; i < p.page_cap; i += nt) used[i] = 0;
  __syncthreads();
  const int n_cand = E - n_tw_old;  // kept fp windows can only come from [n_tw_old, E)
  for (int c = tid; c < n_cand; c += nt) p.entrant[(int64_t)b * p.W + c] = -1;
  __syncthreads();
  for (int j = tid; j < k; j += nt) {
    const int w = ret[j];
    if (w < n_tw_old) {
      for (int i = 0; i < p.ppw; ++i) {
        const int pg = p.table_src[(int64_t)b * p.page_cap + w * p.ppw + i];
        used[pg] = 1;
        p.table_dst[(int64_t)b * p.page_cap + j * p.ppw + i] = pg;
      }
    } else {
      p.entrant[(int64_t)b * p.W + (w - n_tw_old)] = j;  // candidate -> new tier slot
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
  // entrants by rank (their candidate index) for the demotion blocks, in
  // the row's keys, which every thread has read into shared memory by now
  int* ent = entrant_list(p, b);
  for (int j = e0; j < e1; ++j) {
    if (ret[j] >= n_tw_old) {
      for (int i = 0; i < p.ppw; ++i)
        p.table_dst[(int64_t)b * p.page_cap + j * p.ppw + i] = free_list[epos * p.ppw + i];
      ent[epos] = ret[j] - n_tw_old;
      ++epos;
    }
  }
  for (int r = etot + tid; r < entrant_cap(p); r += nt) ent[r] = -1;
}

// Select for an eviction that drops only a few evictable windows (in steady
// state exactly one: one window leaves the local region between two
// evictions).  The kept set of the radix path -- the k largest head means,
// the lowest window index first among equal keys -- is the complement of the
// m = E - k smallest keys taken in (key ascending, index descending) order,
// so m block-wide argmin passes find the dropped windows, every kept window's
// chronological slot is its index minus the dropped windows before it, and
// with the int4 tier the few entrants take the lowest free pages, ranked by
// one block scan over the pool.  Used when m <= kDropMax and (with the
// tier) at most 32 candidate windows can enter the tier.
constexpr int kDropMax = 8;
constexpr int kDropThreads = 1024;

__device__ __forceinline__ uint64_t drop_order(uint32_t key, int w) {
  return ((uint64_t)key << 32) | (uint32_t)(0xFFFFFFFFu - (uint32_t)w);  // min: key asc, index desc
}

__global__ void __launch_bounds__(kDropThreads) evict_select_drop_kernel(EvictParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int b = blockIdx.x;
  const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, warp = tid >> 5;
  grid_launch_dependents();  // the apply kernel's blocks that read the selection wait for it
  const int E = p.E, k = p.kprime, m = E - k;
  const int n_tw_old = p.n_tier_old_tok / p.ws, n_cand = E - n_tw_old;
  uint32_t* keys = reinterpret_cast<uint32_t*>(smem_raw);                   // [E]
  int* tbl = reinterpret_cast<int*>(keys + E);                              // [n_tw_old * ppw]
  unsigned char* used = reinterpret_cast<unsigned char*>(tbl + (p.tier ? n_tw_old * p.ppw + 1 : 1));
  __shared__ uint64_t s_best[32];
  __shared__ int s_drop[kDropMax];
  __shared__ int s_ent[32];
  __shared__ int s_free[32 * 4];
  __shared__ int s_scan[32];
  __shared__ int s_need;

  // 1. the row's logical tier page table and cleared page-use flags (before
  //    the head-mean keys arrive), then the keys
  if (p.tier) {
    for (int i = tid; i < p.page_cap; i += nt) used[i] = 0;
    for (int i = tid; i < n_tw_old * p.ppw; i += nt) tbl[i] = p.table_src[(int64_t)b * p.page_cap + i];
    for (int c = tid; c < n_cand; c += nt) p.entrant[(int64_t)b * p.W + c] = -1;
  }
  grid_dependency_wait();  // the head-mean keys (evict_keys_kernel)
  for (int w = tid; w < E; w += nt) keys[w] = p.keys[(int64_t)b * E + w];
  __syncthreads();
  // 2. the m dropped windows, one block-wide argmin each
  for (int it = 0; it < m; ++it) {
    uint64_t best = ~0ull;
    for (int w = tid; w < E; w += nt) {
      bool gone = false;
      for (int d = 0; d < it; ++d) gone |= s_drop[d] == w;
      if (!gone) best = min(best, drop_order(keys[w], w));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) best = min(best, __shfl_xor_sync(0xffffffffu, best, o));
    if (lane == 0) s_best[warp] = best;
    __syncthreads();
    if (warp == 0) {
      uint64_t v = lane < (nt >> 5) ? s_best[lane] : ~0ull;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
      if (lane == 0) s_drop[it] = (int)(0xFFFFFFFFu - (uint32_t)v);
    }
    __syncthreads();
  }
  // 3. chronological slots: a kept window's slot is its index minus the
  //    dropped windows before it; kept tier windows keep their pages,
  //    candidates that stay become entrants
  for (int w = tid; w < E; w += nt) {
    int before = 0;
    bool gone = false;
    for (int d = 0; d < m; ++d) {
      before += s_drop[d] < w;
      gone |= s_drop[d] == w;
    }
    if (gone) continue;
    const int j = w - before;
    p.retained[(int64_t)b * p.R + j] = w;
    if (p.retained_out) p.retained_out[(int64_t)b * p.scores_cap + j] = w;
    if (!p.tier) continue;
    if (w < n_tw_old) {
      for (int i = 0; i < p.ppw; ++i) {
        const int pg = tbl[w * p.ppw + i];
        used[pg] = 1;
        p.table_dst[(int64_t)b * p.page_cap + j * p.ppw + i] = pg;
      }
    } else {
      p.entrant[(int64_t)b * p.W + (w - n_tw_old)] = j;  // candidate -> new tier slot
    }
  }
  for (int i = tid; i < p.local_w; i += nt) {
    p.retained[(int64_t)b * p.R + k + i] = E + i;
    if (p.retained_out) p.retained_out[(int64_t)b * p.scores_cap + k + i] = E + i;
  }
  if (!p.tier) return;
  // 4. entrants (at most 32 candidates) in chronological order take the
  //    lowest free pages, ppw each: warp 0 ranks the entrants while every
  //    thread counts the free pages of its slice of the pool, and one block
  //    scan ranks the free pages
  if (warp == 0) {
    const int w = n_tw_old + lane;
    bool kept = lane < n_cand;
    int j = 0;
    if (kept) {
      int before = 0;
      for (int d = 0; d < m; ++d) {
        before += s_drop[d] < w;
        kept &= s_drop[d] != w;
      }
      j = w - before;
    }
    const unsigned km = __ballot_sync(0xffffffffu, kept);
    const int rank = __popc(km & ((1u << lane) - 1));
    if (kept) {
      s_ent[rank] = j;
      entrant_list(p, b)[rank] = lane;  // candidate n_tw_old + lane: its rank among the entrants
    }
    for (int r = __popc(km) + lane; r < entrant_cap(p); r += 32) entrant_list(p, b)[r] = -1;
    if (lane == 0) s_need = __popc(km) * p.ppw;  // <= 32 * 4
  }
  __syncthreads();  // page-use flags complete
  const int pper = (p.page_cap + nt - 1) / nt;
  const int p0 = min(p.page_cap, tid * pper), p1 = min(p.page_cap, p0 + pper);
  int fcnt = 0;
  for (int i = p0; i < p1; ++i) fcnt += used[i] ? 0 : 1;
  int ftot = 0;
  int r = block_excl_scan(fcnt, s_scan, ftot);  // its barriers also publish s_ent / s_need
  const int need = s_need;
  for (int i = p0; i < p1 && r < need; ++i)
    if (!used[i]) s_free[r++] = i;
  __syncthreads();
  for (int x = tid; x < min(need, ftot); x += nt) {  // the pool always has `need` free pages
    const int rr = x / p.ppw, i = x % p.ppw;
    p.table_dst[(int64_t)b * p.page_cap + s_ent[rr] * p.ppw + i] = s_free[x];
  }
}

// ---------------------------------------------------------------------------
// Kernel 2 (apply): one launch for everything that follows the selection.
// Blocks [0, n_demote) quantise entrant windows into int4 pages, blocks
// [n_demote, +n_gather) gather scores and ids, the rest move the fp tokens
// that stay fp.  The three write disjoint buffers and read only the source
// side and the selection, so they run side by side; the short demotion and
// gather blocks come first in the grid so they overlap the long move.
// ---------------------------------------------------------------------------
constexpr int kApplyThreads = 256;

// Quantise one 8-token page (keys rotated to the page frame) and pack it,
// with the whole block.  `kin(r, c)` / `vin(r, c)` give token r channel c as
// fp32; `pos0` is the logical position of row 0.  The page is staged in
// shared memory as fp32; each (K or V, row, 32-channel group) is quantised
// by kApplyThreads / (16 * D / 32) threads that reduce min/max by shuffles.
// Scratch: 2*8*D floats + 2*8*D code bytes.
template <int D, typename KF, typename VF>
__device__ void quantize_page_block(KF kin, VF vin, int pos0, const float* cos, const float* sin,
                                    uint8_t* page, unsigned char* scratch) {
  constexpr int half = D / 2, ng = D / kQGroup;
  constexpr int kTasks = 2 * 8 * ng;                 // (K|V, row, group)
  constexpr int kTPT = kApplyThreads / kTasks;       // threads per task
  constexpr int kEPT = kQGroup / kTPT;               // elements per thread
  static_assert(kTPT >= 1 && kTPT <= 32 && (32 % kTPT) == 0 && kEPT * kTPT == kQGroup, "task split");
  const int tid = threadIdx.x;
  float* kf = reinterpret_cast<float*>(scratch);
  float* vf = kf + 8 * D;
  uint8_t* kc = reinterpret_cast<uint8_t*>(vf + 8 * D);
  uint8_t* vc = kc + 8 * D;
  for (int idx = tid; idx < 8 * half; idx += kApplyThreads) {
    const int r = idx / half, cp = idx % half;
    float x = kin(r, cp), y = kin(r, cp + half);
    const int64_t pos = pos0 + r;
    to_page_frame(x, y, cos[pos * half + cp], sin[pos * half + cp], cos[(int64_t)r * half + cp],
                  sin[(int64_t)r * half + cp]);
    kf[r * D + cp] = x;
    kf[r * D + cp + half] = y;
  }
  for (int idx = tid; idx < 8 * D; idx += kApplyThreads) vf[idx] = vin(idx / D, idx % D);
  __syncthreads();
  {
    const int task = tid / kTPT, sub = tid % kTPT;
    const int which = task / (8 * ng);  // 0 = K, 1 = V
    const int r = (task / ng) % 8, gq = task % ng;
    const float* src = (which ? vf : kf) + r * D + gq * kQGroup + sub * kEPT;
    float xv[kEPT];
    float mn = FLT_MAX, mx = -FLT_MAX;
#pragma unroll
    for (int e = 0; e < kEPT; ++e) {
      xv[e] = src[e];
      mn = fminf(mn, xv[e]);
      mx = fmaxf(mx, xv[e]);
    }
#pragma unroll
    for (int o = 1; o < kTPT; o <<= 1) {
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    const __half s16 = __float2half_rn(__fdiv_rn(__fsub_rn(mx, mn), 15.f));
    const __half z16 = __float2half_rn(mn);
    const float sc = __half2float(s16), z = __half2float(z16);
    uint8_t* codes = (which ? vc : kc) + r * D + gq * kQGroup + sub * kEPT;
#pragma unroll
    for (int e = 0; e < kEPT; ++e) {
      int q = 0;
      if (sc != 0.f) q = (int)fminf(fmaxf(rintf(__fdiv_rn(__fsub_rn(xv[e], z), sc)), 0.f), 15.f);
      codes[e] = (uint8_t)q;
    }
    if (sub == 0) {
      if (which == 0) {
        __half* kscl = reinterpret_cast<__half*>(page + page_k_scales_off(D));
        kscl[(r * ng + gq) * 2] = s16;
        kscl[(r * ng + gq) * 2 + 1] = z16;
      } else {
        __half* e4 = reinterpret_cast<__half*>(page + page_v_scales_off(D)) + ((r >> 1) * ng + gq) * 4;
        e4[r & 1] = s16;
        e4[2 + (r & 1)] = z16;
      }
    }
  }
  __syncthreads();
  // fragment-order words: K [row][lane t][word], V [pair t][row g][word]
  for (int idx = tid; idx < 2 * 32 * ng; idx += kApplyThreads) {
    uint32_t word = 0;
    if (idx < 32 * ng) {
      const int r = idx / (4 * ng), t = (idx / ng) % 4, w = idx % ng;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int ch = 2 * t + 8 * (4 * w + i);
        word |= (uint32_t)kc[r * D + ch] << (4 * i);
        word |= (uint32_t)kc[r * D + ch + 1] << (4 * (i + 4));
      }
      reinterpret_cast<uint32_t*>(page)[idx] = word;
    } else {
      const int v = idx - 32 * ng;
      const int t = v / (8 * ng), g = (v / ng) % 8, w = v % ng;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int ch = g + 8 * (4 * w + i);
        word |= (uint32_t)vc[(2 * t) * D + ch] << (4 * i);
        word |= (uint32_t)vc[(2 * t + 1) * D + ch] << (4 * (i + 4));
      }
      reinterpret_cast<uint32_t*>(page + page_v_codes_off(D))[v] = word;
    }
  }
}

// shared scratch for quantize_page_block
__host__ __device__ constexpr int quant_scratch_bytes(int D) { return 2 * 8 * D * 4 + 2 * 8 * D; }

// Codes by rounding in the float adder: for ac in [0, 15], ac + 1.5 * 2^23
// lies in [2^23, 2^24), where floats are 1 apart, so the sum is ac rounded
// to the nearest integer, ties to even (rintf), plus 1.5 * 2^23 -- its low
// nibble is the code.  clamp(rint(a), 0, 15) == rint(clamp(a, 0, 15)) since
// rint is monotone and keeps integers (a NaN clamps to 0 either way).
constexpr float kRoundMagic = 12582912.f;
constexpr float kNearHalf = 0.5f - 0x1p-17f;  // quotients farther than this from an integer take the exact path

// One 32-channel group held as 8 values on each of the 4 lanes of a row
// (lanes 4r .. 4r+3): its min/max over those lanes, its fp16 scale and zero
// point and this lane's 8 codes (quantize_page_block's arithmetic), shifted
// into one word: with `pairs` code 2t in nibble t and code 2t+1 in nibble
// t+4 (t < 4), else code j in nibble j.  Lanes of the whole warp call it
// together (its votes are warp-wide).
template <bool pairs>
__device__ __forceinline__ uint32_t quant_group8(const float (&xv)[8], __half& s16, __half& z16) {
  float mn = FLT_MAX, mx = -FLT_MAX;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    mn = fminf(mn, xv[e]);
    mx = fmaxf(mx, xv[e]);
  }
#pragma unroll
  for (int o = 1; o < 4; o <<= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  s16 = __float2half_rn(__fdiv_rn(__fsub_rn(mx, mn), 15.f));
  z16 = __float2half_rn(mn);
  const float sc = __half2float(s16), z = __half2float(z16);
  // code = clamp(rint((x - z) / sc)) with the quotient correctly rounded.
  // (x - z) * (1 / sc), both products correctly rounded, is within 2^-19 of
  // the exact quotient wherever the code is not clamped (|quotient| <= 16),
  // so it rounds to the same integer unless it lies within 2^-17 of a
  // half-integer; those few take the correctly rounded division.  (sc == 0:
  // every code 0.)
  const float inv = sc != 0.f ? __frcp_rn(sc) : 0.f;
  // Fast path: x -> (x - z) * inv (each step rounded) is monotone, so every
  // quotient of the group lies between those of its min and max; when those
  // lie in [-0.5, 15.5) no clamp binds.  A quotient near a half-integer, or
  // a NaN value, sends the warp to the exact path.
  const bool inside = __fmul_rn(__fsub_rn(mn, z), inv) >= -0.5f && __fmul_rn(__fsub_rn(mx, z), inv) < 15.5f;
  uint32_t word = 0;
  bool redo = !inside;
  if (__all_sync(0xffffffffu, inside)) {
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const int e = pairs ? (n & 3) * 2 + (n >> 2) : n;
      const float a = __fmul_rn(__fsub_rn(xv[e], z), inv);
      const float s = __fadd_rn(a, kRoundMagic);
      redo |= !(fabsf(__fsub_rn(a, __fsub_rn(s, kRoundMagic))) <= kNearHalf);
      word = __funnelshift_r(word, __float_as_uint(s), 4);  // the code enters at nibble 7
    }
  }
  if (__any_sync(0xffffffffu, redo)) {  // clamped, the exact quotient near half-integers
    word = 0;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const int e = pairs ? (n & 3) * 2 + (n >> 2) : n;
      const float t = __fsub_rn(xv[e], z);
      const float ac = fminf(fmaxf(__fmul_rn(t, inv), 0.f), 15.f);
      float s = __fadd_rn(ac, kRoundMagic);
      if (fabsf(__fsub_rn(ac, __fsub_rn(s, kRoundMagic))) > kNearHalf)
        s = __fadd_rn(fminf(fmaxf(__fdiv_rn(t, sc), 0.f), 15.f), kRoundMagic);
      word = __funnelshift_r(word, __float_as_uint(s), 4);
    }
  }
  return word;
}

// Butterfly transpose steps between partner lanes (lane ^ dist): the lane
// without the `dist` bit keeps its even blocks and takes the partner's even
// blocks into its odd ones, the other keeps its odd blocks and takes the
// partner's odd blocks into its even ones; blocks of 16, 8 or 4 bits.
__device__ __forceinline__ uint32_t xpose16(uint32_t x, int dist, bool odd) {
  const uint32_t y = __shfl_xor_sync(0xffffffffu, x, dist);
  return __byte_perm(x, y, odd ? 0x3276 : 0x5410);
}
__device__ __forceinline__ uint32_t xpose8(uint32_t x, int dist, bool odd) {
  const uint32_t y = __shfl_xor_sync(0xffffffffu, x, dist);
  return __byte_perm(x, y, odd ? 0x3715 : 0x6240);
}
__device__ __forceinline__ uint32_t xpose4(uint32_t x, int dist, bool odd) {
  const uint32_t y = __shfl_xor_sync(0xffffffffu, x, dist);
  return odd ? (x & 0xF0F0F0F0u) | ((y >> 4) & 0x0F0F0F0Fu) : (x & 0x0F0F0F0Fu) | ((y << 4) & 0xF0F0F0F0u);
}

// Demotion warps take up to kDemoteHeadsMax kv heads of one page slot (the
// index chain and the rotation rows read once for all of them) while that
// still leaves kDemoteFill warps; fewer pages (a steady-state eviction) take
// one head per warp.
constexpr int kDemoteHeadsMax = 8;
constexpr int kDemoteFill = 8192;

// The same quantisation with one warp per page slot and `nh` kv heads (the
// arithmetic of quantize_page_block element for element,
// head_dim 64 or 128): lane t owns row r = t / 4 and, in every 32-channel
// group g, the 8 channels 32g + 8q + j (q = t % 4, j < 8) -- for K the
// rotation pairs (c, c + D/2) of the groups below D/2 -- read with 16-byte
// loads, the next head's while this one is quantised; the rotation rows of
// the tokens' positions are read once for all heads (the page-frame rows
// again per head, from L1).  Each group's min/max is reduced over the row's 4
// lanes, the codes are shifted into one word per group, and butterfly
// transposes over 4 lanes (K) or 8 lanes (V: two rows) turn those into the
// fragment-order words, lane t writing word t * D/32 + g of each part.
// `ks`/`vs` point at the first head's page row 0 (rows D apart, heads
// `head_elems` apart), `page` at its page (heads `head_bytes` apart); `pos0`
// is the logical position of row 0.
template <typename T, int D>
__device__ void quantize_pages_warp(const T* ks, const T* vs, int64_t head_elems, int nh, int pos0,
                                    const float* cos, const float* sin, uint8_t* page, int64_t head_bytes) {
  static_assert(D == 64 || D == 128, "whole 32-channel groups in each half");
  constexpr int half = D / 2, ng = D / kQGroup;
  constexpr int EV = 16 / (int)sizeof(T), NV = 8 / EV;  // elements per 16-byte load, loads per 8
  const int lane = threadIdx.x & 31, r = lane >> 2, q = lane & 3;
  const bool o1 = lane & 1, o2 = lane & 2, o4 = lane & 4;
  union Vec { uint4 u; T e[EV]; };
  const int64_t pos = pos0 + r;
#pragma unroll
  for (int g = 0; g < ng / 2; ++g) {  // K: the lane's rotation pairs in x group g, y group g + ng/2
    const int c0 = 32 * g + 8 * q;
    float cp[8], sp[8];
#pragma unroll
    for (int j = 0; j < 8; j += 4) {
      *reinterpret_cast<float4*>(cp + j) = *reinterpret_cast<const float4*>(cos + pos * half + c0 + j);
      *reinterpret_cast<float4*>(sp + j) = *reinterpret_cast<const float4*>(sin + pos * half + c0 + j);
    }
    const T* src = ks + r * D + c0;
    Vec nx[NV], ny[NV];
#pragma unroll
    for (int l = 0; l < NV; ++l) {
      nx[l].u = *reinterpret_cast<const uint4*>(src + l * EV);
      ny[l].u = *reinterpret_cast<const uint4*>(src + l * EV + half);
    }
#pragma unroll 1
    for (int i = 0; i < nh; ++i) {
      float x[8], y[8];
#pragma unroll
      for (int l = 0; l < NV; ++l) {
#pragma unroll
        for (int e = 0; e < EV; ++e) {
          x[l * EV + e] = Elt<T>::to_f32(nx[l].e[e]);
          y[l * EV + e] = Elt<T>::to_f32(ny[l].e[e]);
        }
      }
      if (i + 1 < nh) {  // the next head's pairs load while this one is quantised
        src += head_elems;
#pragma unroll
        for (int l = 0; l < NV; ++l) {
          nx[l].u = *reinterpret_cast<const uint4*>(src + l * EV);
          ny[l].u = *reinterpret_cast<const uint4*>(src + l * EV + half);
        }
      }
      float c8[8], s8[8];  // the page-frame rows (positions 0..7): read again per head, from L1
#pragma unroll
      for (int j = 0; j < 8; j += 4) {
        *reinterpret_cast<float4*>(c8 + j) = *reinterpret_cast<const float4*>(cos + r * half + c0 + j);
        *reinterpret_cast<float4*>(s8 + j) = *reinterpret_cast<const float4*>(sin + r * half + c0 + j);
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) to_page_frame(x[e], y[e], cp[e], sp[e], c8[e], s8[e]);
      uint8_t* pg = page + i * head_bytes;
      __half2* kscl = reinterpret_cast<__half2*>(pg + page_k_scales_off(D)) + r * ng;
      uint32_t* kw = reinterpret_cast<uint32_t*>(pg) + lane * ng;
      __half s16, z16;
      uint32_t w = quant_group8<true>(x, s16, z16);
      if (q == g) kscl[g] = __halves2half2(s16, z16);
      kw[g] = xpose4(xpose8(w, 2, o2), 1, o1);
      w = quant_group8<true>(y, s16, z16);
      if (q == g + ng / 2) kscl[g + ng / 2] = __halves2half2(s16, z16);
      kw[g + ng / 2] = xpose4(xpose8(w, 2, o2), 1, o1);
    }
  }
  {  // V: the lane's 8 channels of every group
    constexpr bool kPrefetch = ng * NV <= 4;  // the next head's values held as well (16 registers at most)
    const T* src = vs + r * D + 8 * q;
    Vec nv[ng][NV];
    if constexpr (kPrefetch) {
#pragma unroll
      for (int g = 0; g < ng; ++g)
#pragma unroll
        for (int l = 0; l < NV; ++l) nv[g][l].u = *reinterpret_cast<const uint4*>(src + 32 * g + l * EV);
    }
#pragma unroll 1
    for (int i = 0; i < nh; ++i) {
      Vec raw[ng][NV];
#pragma unroll
      for (int g = 0; g < ng; ++g)
#pragma unroll
        for (int l = 0; l < NV; ++l) {
          if constexpr (kPrefetch) {
            raw[g][l] = nv[g][l];
          } else {
            raw[g][l].u = *reinterpret_cast<const uint4*>(src + 32 * g + l * EV);
          }
        }
      if (kPrefetch && i + 1 < nh) {
#pragma unroll
        for (int g = 0; g < ng; ++g)
#pragma unroll
          for (int l = 0; l < NV; ++l)
            nv[g][l].u = *reinterpret_cast<const uint4*>(src + head_elems + 32 * g + l * EV);
      }
      src += head_elems;
      uint8_t* pg = page + i * head_bytes;
      __half* vscl = reinterpret_cast<__half*>(pg + page_v_scales_off(D)) + (r >> 1) * ng * 4;
      uint32_t* vw = reinterpret_cast<uint32_t*>(pg + page_v_codes_off(D)) + lane * ng;
#pragma unroll
      for (int g = 0; g < ng; ++g) {
        float v[8];
#pragma unroll
        for (int l = 0; l < NV; ++l)
#pragma unroll
          for (int e = 0; e < EV; ++e) v[l * EV + e] = Elt<T>::to_f32(raw[g][l].e[e]);
        __half s16, z16;
        const uint32_t w = quant_group8<false>(v, s16, z16);
        if (q == g) {
          vscl[g * 4 + (r & 1)] = s16;
          vscl[g * 4 + 2 + (r & 1)] = z16;
        }
        vw[g] = xpose4(xpose8(xpose16(w, 4, o4), 2, o2), 1, o1);
      }
    }
  }
}

struct ApplyGrid {
  int n_demote, n_gather, n_move, n_move_v;
  int v_runs_per_row; // value-copy runs per row: the sinks and every kept fp window
  int demote_tasks;   // (entrant rank, page) pairs per (row, kv head)
  int ent_cap;        // entrant ranks per row
  int demote_units;   // head_dim >= 64: (row, entrant rank, page, kv-head group) warps; below: pages
  int demote_heads;   // kv heads per demotion warp (head_dim >= 64)
  int gather_chunks;  // kApplyThreads-window chunks per row
  int move_chunks;    // token chunks per row
  int k_hsplit;       // kv-head slices of the key move (more threads when few rows)
  int n_fp_tok;       // fp tokens that stay fp, per row
};

// Demotion: kept fp windows entering the tier are rotated into their page
// frame and quantised (design.md:130-187).
template <typename T, int D>
__device__ void demote_block(const EvictParams& p, const ApplyGrid& a, int bid, unsigned char* smem) {
  int b, h, k, pi, nh = 1;
  if constexpr (D >= 64) {  // a warp per (row, entrant rank, page, kv-head group), head group fastest
    const unsigned n_hg = (unsigned)ceil_div(p.Hkv, a.demote_heads);
    unsigned pid = (unsigned)bid * (kApplyThreads / 32) + (threadIdx.x >> 5);  // demote_units < 2^31
    if (pid >= (unsigned)a.demote_units) return;
    h = (int)(pid % n_hg) * a.demote_heads;
    nh = min(a.demote_heads, p.Hkv - h);
    pid /= n_hg;
    pi = (int)(pid % (unsigned)p.ppw);
    pid /= (unsigned)p.ppw;
    k = (int)(pid % (unsigned)a.ent_cap);
    b = (int)(pid / (unsigned)a.ent_cap);
  } else {  // a block per page
    const int task = bid % a.demote_tasks, bh = bid / a.demote_tasks;
    h = bh % p.Hkv;
    b = bh / p.Hkv;
    k = task / p.ppw;
    pi = task % p.ppw;
  }
  const int n_tw_old = p.n_tier_old_tok / p.ws;
  const int cand = entrant_list(p, b)[k];
  if (cand < 0) return;  // fewer entrants in this row
  const int j = p.entrant[(int64_t)b * p.W + cand];
  const int w = n_tw_old + cand;
  const int pos0 = p.s + w * p.ws + pi * kPageTokens;
  const Geometry go{p.s, p.s_pad, p.ws, p.T_old, p.n_tier_old_tok};
  const int64_t rb = (((int64_t)b * p.Hkv + h) * p.fp_cap_src + go.fp_slot(pos0)) * D;
  const T* ks = (const T*)p.k_src + rb;
  const T* vs = (const T*)p.v_src + rb;
  const int phys = p.table_dst[(int64_t)b * p.page_cap + j * p.ppw + pi];
  uint8_t* page = p.pages + (((int64_t)b * p.Hkv + h) * p.page_cap + phys) * page_bytes(D);
  if constexpr (D >= 64) {
    quantize_pages_warp<T, D>(ks, vs, (int64_t)p.fp_cap_src * D, nh, pos0, p.cos, p.sin, page,
                              (int64_t)p.page_cap * page_bytes(D));
  } else {
    quantize_page_block<D>([&](int r, int c) { return ld_f32(ks + (int64_t)r * D + c); },
                           [&](int r, int c) { return ld_f32(vs + (int64_t)r * D + c); }, pos0, p.cos, p.sin,
                           page, smem);
  }
}

// Score and original-id gather (cache.py:271-283) for one chunk of retained
// windows of one row, all query heads; windows that appear before the next
// eviction start at zero score and take ids from the running counter
// (cache.py:180-213).
__device__ void gather_block(const EvictParams& p, const ApplyGrid& a, int bid) {
  const int b = bid / a.gather_chunks, chunk = bid % a.gather_chunks;
  const int ztail = min(p.scores_cap - p.R, kTailWindows);
  const int j = chunk * kApplyThreads + threadIdx.x;
  if (j >= p.R + ztail) return;
  const int r = j < p.R ? p.retained[(int64_t)b * p.R + j] : -1;
  const float* src = p.scores_src + (int64_t)b * p.Hq * p.scores_cap;
  float* dst = p.scores_dst + (int64_t)b * p.Hq * p.scores_cap;
  const int64_t* ids = p.ids_src + (int64_t)b * p.scores_cap;
  // the next window's original id is one past the newest window's (ids
  // grow by one per new window, cache.py:180-213); reading it here rather
  // than from the host keeps a captured launch valid when replayed.  Every
  // load of the thread (its id, the newest id, 32 heads' scores) is issued
  // before any store, so the gather costs two memory round trips.
  const int64_t newest = p.W > 0 ? ids[p.W - 1] : p.next_window_id - 1;
  const int64_t id = r >= 0 ? ids[r] : 0;
  constexpr int kH = 32;
  for (int h0 = 0; h0 < p.Hq; h0 += kH) {
    float v[kH];
#pragma unroll
    for (int i = 0; i < kH; ++i)
      v[i] = (r >= 0 && h0 + i < p.Hq) ? src[(int64_t)(h0 + i) * p.scores_cap + r] : 0.f;
#pragma unroll
    for (int i = 0; i < kH; ++i)
      if (h0 + i < p.Hq) dst[(int64_t)(h0 + i) * p.scores_cap + j] = v[i];
  }
  p.ids_dst[(int64_t)b * p.scores_cap + j] = r >= 0 ? id : newest + 1 + (j - p.R);
}

// Keys of the fp tokens that stay fp, stripped at the old and re-applied at
// the new position (op by op in the KV dtype).  A thread owns one (token,
// 16-byte vector of the first half of the channels) of one row and walks the
// KV heads, so its cos/sin rows are loaded once; it handles the vector and
// its rotation partner.
template <typename T, int D>
__device__ void move_k_block(const EvictParams& p, const ApplyGrid& a, int bid) {
  constexpr int VE = 16 / sizeof(T);  // elements per 16-byte vector
  constexpr int half = D / 2, nvec = half / VE, tpb = kApplyThreads / nvec;
  const int hs = bid % a.k_hsplit;  // this block's slice of the kv heads
  bid /= a.k_hsplit;
  const int b = bid / a.move_chunks, chunk = bid % a.move_chunks;
  const int h_begin = hs * p.Hkv / a.k_hsplit, h_end = (hs + 1) * p.Hkv / a.k_hsplit;
  const int tau = chunk * tpb + threadIdx.x / nvec, c0 = (threadIdx.x % nvec) * VE;
  if (threadIdx.x >= tpb * nvec || tau >= a.n_fp_tok) return;
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
  const int64_t so_slot = go.fp_slot(old_pos), sd_slot = gn.fp_slot(new_pos);
  const bool fresh = p.k_new && old_pos == p.T_old - 1;  // this step's token: from the caller's buffer
  const float* tco = p.cos + (int64_t)old_pos * half + c0;
  const float* tso = p.sin + (int64_t)old_pos * half + c0;
  const float* tcn = p.cos + (int64_t)new_pos * half + c0;
  const float* tsn = p.sin + (int64_t)new_pos * half + c0;
  if constexpr (sizeof(T) == 2) {
    // fp16/bf16: an fp32 multiply or add of two KV-dtype values followed by a
    // rounding to the KV dtype equals the dtype's own round-to-nearest
    // multiply or add.  The fp32 product is exact; for the sum, fp32 carries
    // at least 2p+2 significand bits of the p-bit dtype, which makes the
    // double rounding innocuous (Figueroa, "When is double rounding
    // innocuous?", SIGNUM 1995).  So the reference's op-by-op rounded strip
    // and re-apply run as packed non-fused multiplies and adds, bit for bit.
    using T2 = typename std::conditional<std::is_same<T, __half>::value, __half2, __nv_bfloat162>::type;
    T2 co[VE / 2], so[VE / 2], cn[VE / 2], sn[VE / 2];
#pragma unroll
    for (int e = 0; e < VE; e += 2) {
      co[e / 2] = T2{Elt<T>::from_f32(tco[e]), Elt<T>::from_f32(tco[e + 1])};
      so[e / 2] = T2{Elt<T>::from_f32(tso[e]), Elt<T>::from_f32(tso[e + 1])};
      cn[e / 2] = T2{Elt<T>::from_f32(tcn[e]), Elt<T>::from_f32(tcn[e + 1])};
      sn[e / 2] = T2{Elt<T>::from_f32(tsn[e]), Elt<T>::from_f32(tsn[e + 1])};
    }
    union V2 { uint4 u; T2 e[VE / 2]; };
    constexpr int HB = 4;  // kv heads whose loads are in flight together
    const int64_t hs_src = fresh ? p.new_sh : (int64_t)p.fp_cap_src * D, hs_dst = (int64_t)p.fp_cap_dst * D;
    const T* ks0 = fresh ? (const T*)p.k_new + (int64_t)b * p.new_sb + c0
                         : (const T*)p.k_src + ((int64_t)b * p.Hkv * p.fp_cap_src + so_slot) * D + c0;
    T* kd0 = (T*)p.k_dst + ((int64_t)b * p.Hkv * p.fp_cap_dst + sd_slot) * D + c0;
#pragma unroll 1
    for (int h0 = h_begin; h0 < h_end; h0 += HB) {
      V2 x[HB], y[HB];
#pragma unroll
      for (int j = 0; j < HB; ++j)
        if (h0 + j < h_end) {
          x[j].u = *reinterpret_cast<const uint4*>(ks0 + (h0 + j) * hs_src);
          y[j].u = *reinterpret_cast<const uint4*>(ks0 + (h0 + j) * hs_src + half);
        }
#pragma unroll
      for (int j = 0; j < HB; ++j) {
        if (h0 + j >= h_end) break;
#pragma unroll
        for (int e = 0; e < VE / 2; ++e) {
          // strip (cos, -sin), then re-apply (cos, sin)
          const T2 ux = __hadd2_rn(__hmul2_rn(x[j].e[e], co[e]), __hmul2_rn(y[j].e[e], so[e]));
          const T2 uy = __hsub2_rn(__hmul2_rn(y[j].e[e], co[e]), __hmul2_rn(x[j].e[e], so[e]));
          x[j].e[e] = __hsub2_rn(__hmul2_rn(ux, cn[e]), __hmul2_rn(uy, sn[e]));
          y[j].e[e] = __hadd2_rn(__hmul2_rn(uy, cn[e]), __hmul2_rn(ux, sn[e]));
        }
        *reinterpret_cast<uint4*>(kd0 + (h0 + j) * hs_dst) = x[j].u;
        *reinterpret_cast<uint4*>(kd0 + (h0 + j) * hs_dst + half) = y[j].u;
      }
    }
  } else {
    float co[VE], so[VE], cn[VE], sn[VE];
#pragma unroll
    for (int e = 0; e < VE; e += 4) {
      *reinterpret_cast<float4*>(co + e) = *reinterpret_cast<const float4*>(tco + e);
      *reinterpret_cast<float4*>(so + e) = *reinterpret_cast<const float4*>(tso + e);
      *reinterpret_cast<float4*>(cn + e) = *reinterpret_cast<const float4*>(tcn + e);
      *reinterpret_cast<float4*>(sn + e) = *reinterpret_cast<const float4*>(tsn + e);
    }
    union Vec { uint4 u; T e[VE]; };
#pragma unroll 1
    for (int h = h_begin; h < h_end; ++h) {
      const T* ks = fresh ? (const T*)p.k_new + (int64_t)b * p.new_sb + (int64_t)h * p.new_sh
                          : (const T*)p.k_src + (((int64_t)b * p.Hkv + h) * p.fp_cap_src + so_slot) * D;
      T* kd = (T*)p.k_dst + (((int64_t)b * p.Hkv + h) * p.fp_cap_dst + sd_slot) * D;
      Vec kx, ky, ox, oy;
      kx.u = *reinterpret_cast<const uint4*>(ks + c0);
      ky.u = *reinterpret_cast<const uint4*>(ks + c0 + half);
#pragma unroll
      for (int e = 0; e < VE; ++e) {
        float x = Elt<T>::to_f32(kx.e[e]), y = Elt<T>::to_f32(ky.e[e]);
        rope_strip_apply<T>(x, y, co[e], so[e], cn[e], sn[e]);
        ox.e[e] = Elt<T>::from_f32(x);
        oy.e[e] = Elt<T>::from_f32(y);
      }
      *reinterpret_cast<uint4*>(kd + c0) = ox.u;
      *reinterpret_cast<uint4*>(kd + c0 + half) = oy.u;
    }
  }
}

// Values of the fp tokens that stay fp: whole windows (and the sink rows) are
// contiguous in both stores, so a block copies kVUnits runs of up to
// window_size rows, 16 bytes per thread, with the run's offsets computed once
// per run.
constexpr int kVUnits = 4;
template <typename T, int D>
__device__ void move_v_block(const EvictParams& p, const ApplyGrid& a, int bid) {
  constexpr int CPR = D * (int)sizeof(T) / 16;  // 16-byte chunks per row
  const int per_unit = kApplyThreads / kVUnits;  // threads per run
  const int unit = bid * kVUnits + threadIdx.x / per_unit;
  const int b = unit / a.v_runs_per_row, run = unit % a.v_runs_per_row;
  if (b >= p.B) return;
  const int s_eff = min(p.s, p.T_old);
  // run 0: the sinks; run 1 + j: kept window j of the fp region (tokens s_eff + 8j ...)
  int tau0, rows;
  if (run == 0) {
    tau0 = 0;
    rows = s_eff;
  } else {
    tau0 = s_eff + (run - 1) * p.ws;
    rows = min(p.ws, a.n_fp_tok - tau0);
  }
  if (rows <= 0) return;
  int old_pos, new_pos;
  if (run == 0) {
    old_pos = new_pos = 0;
  } else {
    const int jf = run - 1;
    const int j = p.tier ? p.kprime + jf : jf;
    const int w = p.tier ? p.E + jf : p.retained[(int64_t)b * p.R + j];
    old_pos = p.s + w * p.ws;
    new_pos = p.s + j * p.ws;
  }
  const Geometry go{p.s, p.s_pad, p.ws, p.T_old, p.n_tier_old_tok};
  const Geometry gn{p.s, p.s_pad, p.ws, p.T_new, p.n_tier_new_tok};
  const int64_t so_slot = go.fp_slot(old_pos), sd_slot = gn.fp_slot(new_pos);
  const int cw = rows * CPR;  // chunks of the run in one head
  const int64_t hs_src = (int64_t)p.fp_cap_src * D, hs_dst = (int64_t)p.fp_cap_dst * D;
  const T* src0 = (const T*)p.v_src + ((int64_t)b * p.Hkv * p.fp_cap_src + so_slot) * D;
  T* dst0 = (T*)p.v_dst + ((int64_t)b * p.Hkv * p.fp_cap_dst + sd_slot) * D;
  for (int c = threadIdx.x % per_unit; c < cw; c += per_unit) {
    // this step's token (when its append rides here) comes from the caller's buffer
    const bool fresh = p.v_new && old_pos + c / CPR == p.T_old - 1;
    const T* sc = fresh ? (const T*)p.v_new + (int64_t)b * p.new_sb : src0;
    const int64_t hsc = fresh ? p.new_sh : hs_src;
    const int cc = fresh ? c % CPR : c;
    // all heads' loads first, then the stores (8 independent 16-byte loads in flight)
    for (int h0 = 0; h0 < p.Hkv; h0 += 8) {
      uint4 v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (h0 + j < p.Hkv) v[j] = reinterpret_cast<const uint4*>(sc + (h0 + j) * hsc)[cc];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (h0 + j < p.Hkv) reinterpret_cast<uint4*>(dst0 + (h0 + j) * hs_dst)[c] = v[j];
    }
  }
}

// Launched as a programmatic dependent of the select kernel.  With the int4
// tier the fp tokens that stay fp are the sinks and the local windows, whose
// new positions follow from the plan's counts alone, so the move blocks (the
// bulk of the bytes) run alongside the selection; blocks that read the
// selection (demotion, gather, and every move in reference mode) wait for it.
// The waiting blocks come first in the grid: they hold a few slots while the
// moves stream and then run beside the rest of them, not as a tail.
template <typename T, int D>
__global__ void __launch_bounds__(kApplyThreads, 3) evict_apply_kernel(EvictParams p, ApplyGrid a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  int bid = blockIdx.x;
  if (bid < a.n_demote + a.n_gather) {
    grid_dependency_wait();
    if constexpr (D % kQGroup == 0) {  // the int4 tier needs whole 32-channel groups
      if (bid < a.n_demote) {
        demote_block<T, D>(p, a, bid, smem_raw);
        return;
      }
    }
    gather_block(p, a, bid - a.n_demote);
    return;
  }
  bid -= a.n_demote + a.n_gather;
  if (!p.tier) grid_dependency_wait();
  if (bid < a.n_move_v) {  // the short value copies first, then the key re-rotation
    move_v_block<T, D>(p, a, bid);
    return;
  }
  move_k_block<T, D>(p, a, bid - a.n_move_v);
}

template <typename T, int D>
__global__ void __launch_bounds__(kApplyThreads) pack_pages_kernel(const T* k, const T* v, int first_pos,
                                                                   const float* cos, const float* sin,
                                                                   uint8_t* out) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int pg = blockIdx.x;
  const T* ks = k + (int64_t)pg * 8 * D;
  const T* vs = v + (int64_t)pg * 8 * D;
  quantize_page_block<D>([&](int r, int c) { return ld_f32(ks + (int64_t)r * D + c); },
                         [&](int r, int c) { return ld_f32(vs + (int64_t)r * D + c); }, first_pos + pg * 8,
                         cos, sin, out + (int64_t)pg * page_bytes(D), smem_raw);
}

size_t select_smem_bytes(int E, int R, int page_cap) {
  return (size_t)4 * (E > 0 ? E : 1) + 4 * (256 + 32) + 4 * (size_t)(R > 0 ? R : 1) +
         5 * (size_t)page_cap + 16;
}

template <typename T, int D>
int launch_apply(EvictParams& p, cudaStream_t stream) {
  ApplyGrid a{};
  const int n_cand = p.E - p.n_tier_old_tok / p.ws;
  // every (row, kv head)'s (entrant rank, page) pairs: a warp per page slot
  // and demote_heads kv heads at head_dim 64 and 128, a block per page below
  a.ent_cap = (D % kQGroup == 0 && p.tier && p.kprime > 0 && n_cand > 0)
                  ? entrant_cap_of(p.E, p.n_tier_old_tok / p.ws, p.kprime)
                  : 0;
  a.demote_tasks = a.ent_cap * p.ppw;
  a.demote_heads = 1;
  if (D >= 64) {
    const int64_t pages = (int64_t)a.demote_tasks * p.Hkv * p.B;
    while (2 * a.demote_heads <= min(p.Hkv, kDemoteHeadsMax) && pages / (2 * a.demote_heads) >= kDemoteFill)
      a.demote_heads *= 2;
  }
  const int64_t demote_units =
      (int64_t)a.demote_tasks * (D >= 64 ? ceil_div(p.Hkv, a.demote_heads) : p.Hkv) * p.B;
  if (demote_units > 0x7FFFFFFF) return SKV_ERR_CAPACITY;
  a.demote_units = (int)demote_units;
  a.n_demote = D >= 64 ? ceil_div(a.demote_units, kApplyThreads / 32) : a.demote_units;
  a.gather_chunks = ceil_div(p.R + min(p.scores_cap - p.R, kTailWindows), kApplyThreads);
  a.n_gather = a.gather_chunks * p.B;
  a.n_fp_tok = p.T_new - p.n_tier_new_tok;  // sinks + fp windows kept
  constexpr int tpb = kApplyThreads / (D / 2 / (16 / (int)sizeof(T)));
  a.move_chunks = a.n_fp_tok > 0 ? ceil_div(a.n_fp_tok, tpb) : 0;
  // few rows: slice the kv heads over blocks so each thread keeps one round of
  // loads in flight instead of walking all heads (4 heads per slice)
  a.k_hsplit = (a.move_chunks * p.B < 2 * 148) ? max(1, p.Hkv / 4) : 1;
  a.n_move = a.move_chunks * p.B * a.k_hsplit;
  {
    const int s_eff = min(p.s, p.T_old);
    const int rest = a.n_fp_tok > s_eff ? a.n_fp_tok - s_eff : 0;
    a.v_runs_per_row = a.n_fp_tok > 0 ? 1 + ceil_div(rest, p.ws) : 0;
    a.n_move_v = ceil_div(a.v_runs_per_row * p.B, kVUnits);
  }
  const int64_t blocks = (int64_t)a.n_demote + a.n_gather + a.n_move + a.n_move_v;
  if (blocks == 0) return SKV_OK;
  if (blocks > 0x7FFFFFFF) return SKV_ERR_CAPACITY;
  const size_t smem = !a.n_demote || D >= 64 ? 0 : quant_scratch_bytes(D);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)blocks);
  cfg.blockDim = dim3(kApplyThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, evict_apply_kernel<T, D>, p, a);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return SKV_ERR_CUDA;
  }
  return SKV_OK;
}

template <typename T>
int launch_evict(EvictParams& p, cudaStream_t stream) {
  const int n_cand = p.E - p.n_tier_old_tok / p.ws;
  const int m = p.E - p.kprime;
  const bool partial = p.kprime > 0 && m > 0;
  const bool drop = partial && m <= kDropMax && (!p.tier || (n_cand <= 32 && p.ppw <= 4));
  const size_t smem = drop ? (size_t)4 * p.E + 4 * ((size_t)(p.n_tier_old_tok / p.ws) * p.ppw + 1) +
                                 (p.tier ? (size_t)p.page_cap : 0) + 16
                           : select_smem_bytes(p.E, p.R, p.tier ? p.page_cap : 0);
  if (smem > (size_t)kSelectSmemMax) return SKV_ERR_CAPACITY;
  if (partial) {  // the selects read the keys only for a partial top-k
    evict_keys_kernel<<<dim3(ceil_div(p.E, kKeysThreads), p.B), kKeysThreads, 0, stream>>>(p);
    SKV_CHECK_LAUNCH();
  }
  auto kernel = drop ? evict_select_drop_kernel : evict_select_kernel;
  static std::atomic<uint32_t> smem_set[2];  // the radix and the few-drops select
  max_smem_once(smem_set[drop ? 1 : 0], kernel, kSelectSmemMax);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(p.B);
  cfg.blockDim = dim3(drop ? kDropThreads : kSelectThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, p);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return SKV_ERR_CUDA;
  }
  switch (p.D) {
    case 16: return launch_apply<T, 16>(p, stream);
    case 32: return launch_apply<T, 32>(p, stream);
    case 64: return launch_apply<T, 64>(p, stream);
    case 128: return launch_apply<T, 128>(p, stream);
  }
  return SKV_ERR_UNSUPPORTED;
}

int evict_dispatch(EvictParams& p, cudaStream_t stream) {
  switch (p.dtype) {
    case SKV_F32: return launch_evict<float>(p, stream);
    case SKV_F16: return launch_evict<__half>(p, stream);
    case SKV_BF16: return launch_evict<__nv_bfloat16>(p, stream);
  }
  return SKV_ERR_UNSUPPORTED;
}

template <typename T>
int launch_pack(const void* k, const void* v, int D, int first_pos, int n_pages, const float* cos,
                const float* sin, uint8_t* out, cudaStream_t stream) {
  const dim3 grid(n_pages);
  const size_t smem = quant_scratch_bytes(D);
  switch (D) {
    case 32: pack_pages_kernel<T, 32><<<grid, kApplyThreads, smem, stream>>>((const T*)k, (const T*)v, first_pos, cos, sin, out); break;
    case 64: pack_pages_kernel<T, 64><<<grid, kApplyThreads, smem, stream>>>((const T*)k, (const T*)v, first_pos, cos, sin, out); break;
    case 128: pack_pages_kernel<T, 128><<<grid, kApplyThreads, smem, stream>>>((const T*)k, (const T*)v, first_pos, cos, sin, out); break;
    default: return SKV_ERR_UNSUPPORTED;
  }
  SKV_CHECK_LAUNCH();
  return SKV_OK;
}

int pack_pages_dispatch(const skv_layer_desc* L, const void* k, const void* v, int first_pos,
                        int n_pages, uint8_t* out, cudaStream_t stream) {
  switch (L->kv_dtype) {
    case SKV_F32: return launch_pack<float>(k, v, L->head_dim, first_pos, n_pages, L->rope_cos, L->rope_sin, out, stream);
    case SKV_F16: return launch_pack<__half>(k, v, L->head_dim, first_pos, n_pages, L->rope_cos, L->rope_sin, out, stream);
    case SKV_BF16: return launch_pack<__nv_bfloat16>(k, v, L->head_dim, first_pos, n_pages, L->rope_cos, L->rope_sin, out, stream);
  }
  return SKV_ERR_UNSUPPORTED;
}

}  // namespace skv
