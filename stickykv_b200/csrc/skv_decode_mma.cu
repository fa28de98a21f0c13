// Tensor-core decode attention with fused window mass (fp16/bf16 KV,
// window_size 8, 4 query heads per KV head, head_dim 64 or 128).
//
// Same contract as the portable path (skv_decode_generic.cu): replaces the
// reference's attention + score hook + scorer for one decode query
// (modules/windowed_eager_cache/hooks.py:145-180, modules/windowed_cache/
// hooks.py:199-290, scorer.py:17-109).
//
// The retained cache of one (row, kv head) is a sequence of 8-token units:
// [sink unit(s) | int4 tier pages | fp units after the tier].  With
// window_size 8 every unit after the sinks is one scoring window.
//
// Work split: one CTA per (row, kv head, unit range); ranges are balanced by
// bytes (an fp unit moves 32*D bytes, an int4 page page_bytes + its cos/sin).
// Each of the 4 warps streams its own 16-token tiles (two units) through a
// private cp.async ring in shared memory, so the main loop has no CTA
// barrier.  Per tile:
//   QK  4 (or 8) mma.m16n8k16: rows = 16 tokens, columns = 4 heads x 2 units;
//       unit A's keys only meet columns 0-3, unit B's columns 4-7, so each
//       column group carries the query of its unit: unrotated for fp units,
//       rotated to the page start R(-P) q for int4 pages (whose keys are
//       stored in their page frame).  int4 codes are dequantised straight
//       into the A fragment registers (one packed FMA per two channels).
//   softmax in the log2 domain, online per warp; the window mass of each
//       unit is the sum of its 8 rows, kept per warp with the running max.
//   PV  4 (or 8) mma: O^T = V^T P, V^T fragments via ldmatrix.trans (fp) or
//       dequantised codes (int4); P converted with movmatrix.trans.
// The CTA merges its warps and writes (max, sum, O) and the window masses
// relative to its max; a merge kernel combines the splits, writes the output
// and adds the normalised window mass to the fp32 score accumulator.
#include <float.h>

#include <type_traits>

#include "skv_common.cuh"

namespace skv {
namespace {

constexpr int kWarps = 4;
constexpr int kThreads = 32 * kWarps;
constexpr int kMaxSplits = 64;
constexpr int kMaxTilesPerWarp = 32;
constexpr int kMaxUnitsPerSplit = 2 * kWarps * kMaxTilesPerWarp;
constexpr float kLog2e = 1.4426950408889634f;

template <int D> struct Cfg {
  static constexpr int kStages = 3;
  static constexpr int kHalfBytes = 32 * D;           // one unit: fp K+V rows, or int4 page + cos/sin
  static constexpr int kPageBytes = page_bytes(D);
  static constexpr int kCPR = D / 8;                  // 16-byte chunks per fp row
  static constexpr int kKB = D / 16;                  // k-blocks (QK) == m-blocks (PV)
  static constexpr int kNW = D / 32;                  // int4 words per (row, lane)
  static constexpr size_t kStageBytes = 2 * kHalfBytes;
  static constexpr size_t kRingBytes = (size_t)kWarps * kStages * kStageBytes;
  static constexpr size_t kMassBytes = (size_t)kWarps * kMaxTilesPerWarp * 12 * 4;
  static constexpr size_t kTableBytes = (size_t)kMaxUnitsPerSplit * 4;
  static constexpr size_t kSmemBytes = kRingBytes + kMassBytes + kTableBytes;
  static_assert(kPageBytes + 4 * D <= kHalfBytes, "int4 unit must fit a half stage");
};

struct MmaParams {
  const void* k_fp;
  const void* v_fp;
  const uint8_t* pages;
  const int32_t* table;
  const float* cos;
  const float* sin;
  const void* q;
  void* out;
  float* scores;   // [B][Hq][scores_cap] accumulator (may be null)
  float* part;     // [B][Hkv][n_split][4][D+2]: O, max (log2 domain), sum
  float* mass;     // [B][Hq][W]: window mass relative to its split's max
  int64_t q_sb, q_sh, o_sb, o_sh;
  int B, Hkv, cap, page_cap, scores_cap, n_split;
  int s, s_eff, s_pad, NS, n_tp, rest, U, W;
  float scale_log2;
  int bnd[kMaxSplits + 1];
};

// ---------------------------------------------------------------------------
// operand-type specifics
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t u32(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ uint32_t u32(__nv_bfloat162 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 h2(uint32_t x) { return *reinterpret_cast<__half2*>(&x); }
__device__ __forceinline__ __nv_bfloat162 b2(uint32_t x) { return *reinterpret_cast<__nv_bfloat162*>(&x); }

template <typename T> struct Op;
template <> struct Op<__half> {
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) { return u32(__floats2half2_rn(lo, hi)); }
  static __device__ __forceinline__ float2 unpack(uint32_t x) { return __half22float2(h2(x)); }
  static __device__ __forceinline__ void mma(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                             uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
  // nibbles i (low half) and i+4 (high half) of w as exact 16-bit values
  static __device__ __forceinline__ uint32_t codes(uint32_t w, int i) {
    const uint32_t x = ((w >> (4 * i)) & 0x000F000Fu) | 0x64006400u;   // 1024 + code
    return u32(__hsub2(h2(x), h2(0x64006400u)));
  }
  // scale/zero stored as fp16 pairs -> operand pairs
  static __device__ __forceinline__ uint32_t from_f16x2(uint32_t x) { return x; }
  static __device__ __forceinline__ uint32_t fma2(uint32_t a, uint32_t b, uint32_t c) {
    return u32(__hfma2(h2(a), h2(b), h2(c)));
  }
};
template <> struct Op<__nv_bfloat16> {
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) { return u32(__floats2bfloat162_rn(lo, hi)); }
  static __device__ __forceinline__ float2 unpack(uint32_t x) { return __bfloat1622float2(b2(x)); }
  static __device__ __forceinline__ void mma(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                             uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
  static __device__ __forceinline__ uint32_t codes(uint32_t w, int i) {
    const uint32_t x = ((w >> (4 * i)) & 0x000F000Fu) | 0x43004300u;   // 128 + code
    return u32(__hsub2(b2(x), b2(0x43004300u)));
  }
  static __device__ __forceinline__ uint32_t from_f16x2(uint32_t x) {
    return u32(__float22bfloat162_rn(__half22float2(h2(x))));
  }
  static __device__ __forceinline__ uint32_t fma2(uint32_t a, uint32_t b, uint32_t c) {
    return u32(__hfma2(b2(a), b2(b), b2(c)));
  }
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }
__device__ __forceinline__ void ldsm_x2(uint32_t& r0, uint32_t& r1, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];\n" : "=r"(r0), "=r"(r1) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t& r0, uint32_t& r1, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];\n"
               : "=r"(r0), "=r"(r1)
               : "r"(addr));
}
__device__ __forceinline__ uint32_t movm_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;\n" : "=r"(y) : "r"(x));
  return y;
}

// kind: 0 none, 1 fp, 2 int4 page
struct Unit {
  int kind, valid, window, src, P;
};

__device__ __forceinline__ Unit unit_info(const MmaParams& p, int u, int u_end, const int* tbl, int tbl0) {
  Unit x{0, 0, -1, 0, 0};
  if (u >= u_end) return x;
  if (u < p.NS) {
    x.kind = 1;
    x.src = 8 * u;
    x.valid = min(8, p.s_eff - 8 * u);
  } else if (u < p.NS + p.n_tp) {
    const int j = u - p.NS;
    x.kind = 2;
    x.src = tbl[j - tbl0];
    x.P = p.s + 8 * j;
    x.valid = 8;
    x.window = j;
  } else {
    const int r = u - p.NS - p.n_tp;
    x.kind = 1;
    x.src = p.s_pad + 8 * r;
    x.valid = min(8, p.rest - 8 * r);
    x.window = p.n_tp + r;
  }
  return x;
}

template <typename T, int D>
__device__ __forceinline__ void issue_unit(const MmaParams& p, const Unit& x, int b, int kh,
                                           unsigned char* half, int lane) {
  using C = Cfg<D>;
  if (x.kind == 1) {
    const T* kr = (const T*)p.k_fp + (((int64_t)b * p.Hkv + kh) * p.cap + x.src) * D;
    const T* vr = (const T*)p.v_fp + (((int64_t)b * p.Hkv + kh) * p.cap + x.src) * D;
    const uint32_t base = smem_u32(half);
#pragma unroll
    for (int idx = lane; idx < 8 * C::kCPR; idx += 32) {
      const int r = idx / C::kCPR, c = idx % C::kCPR;
      const uint32_t off = r * (2 * D) + ((c ^ (r & 7)) * 16);
      cp_async16(base + off, kr + r * D + c * 8);
      cp_async16(base + 16 * D + off, vr + r * D + c * 8);
    }
  } else if (x.kind == 2) {
    const uint8_t* pg = p.pages + (((int64_t)b * p.Hkv + kh) * p.page_cap + x.src) * C::kPageBytes;
    const uint32_t base = smem_u32(half);
    for (int idx = lane; idx < C::kPageBytes / 16; idx += 32) cp_async16(base + idx * 16, pg + idx * 16);
    const float* cs = p.cos + (int64_t)x.P * (D / 2);
    const float* sn = p.sin + (int64_t)x.P * (D / 2);
    for (int idx = lane; idx < D / 8; idx += 32) cp_async16(base + C::kPageBytes + idx * 16, cs + idx * 4);
    for (int idx = lane; idx < D / 8; idx += 32)
      cp_async16(base + C::kPageBytes + 2 * D + idx * 16, sn + idx * 4);
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(kThreads) decode_mma_kernel(const __grid_constant__ MmaParams p) {
  using C = Cfg<D>;
  using O = Op<T>;        // fp units: the KV dtype
  using H = Op<__half>;   // int4 pages: fp16
  constexpr bool kBF = !std::is_same<T, __half>::value;
  constexpr int KB = C::kKB, NW = C::kNW;
  extern __shared__ __align__(128) unsigned char smem[];
  const int split = blockIdx.x, kh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int u0 = p.bnd[split], u1 = p.bnd[split + 1];
  const int n_tiles = (u1 - u0 + 1) >> 1;

  unsigned char* ring = smem + (size_t)warp * C::kStages * C::kStageBytes;
  float* mass_s = reinterpret_cast<float*>(smem + C::kRingBytes) + warp * kMaxTilesPerWarp * 12;
  int* tbl = reinterpret_cast<int*>(smem + C::kRingBytes + C::kMassBytes);

  // page-table slice of this split
  const int j0 = max(0, u0 - p.NS), j1 = min(p.n_tp, max(0, u1 - p.NS));
  for (int j = j0 + threadIdx.x; j < j1; j += kThreads) tbl[j - j0] = p.table[(int64_t)b * p.page_cap + j];
  __syncthreads();

  // query of head (g & 3) in B-fragment order: d = 16kb + 2t + {0,1,8,9}
  const T* qp = (const T*)p.q + b * p.q_sb + (kh * 4 + (g & 3)) * p.q_sh;
  uint32_t qb[KB][2];
  float qf[KB][4];
#pragma unroll
  for (int kb = 0; kb < KB; ++kb) {
    qb[kb][0] = *reinterpret_cast<const uint32_t*>(qp + 16 * kb + 2 * t);
    qb[kb][1] = *reinterpret_cast<const uint32_t*>(qp + 16 * kb + 2 * t + 8);
    const float2 lo = O::unpack(qb[kb][0]), hi = O::unpack(qb[kb][1]);
    qf[kb][0] = lo.x; qf[kb][1] = lo.y; qf[kb][2] = hi.x; qf[kb][3] = hi.y;
  }

  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  float o[KB][4];
#pragma unroll
  for (int mb = 0; mb < KB; ++mb) o[mb][0] = o[mb][1] = o[mb][2] = o[mb][3] = 0.f;

  const int my_tiles = n_tiles > warp ? (n_tiles - warp + kWarps - 1) / kWarps : 0;
  // prologue: fill the ring
#pragma unroll
  for (int i = 0; i < C::kStages - 1; ++i) {
    if (i < my_tiles) {
      const int ua = u0 + 2 * (warp + kWarps * i);
      unsigned char* st = ring + (size_t)i * C::kStageBytes;
      issue_unit<T, D>(p, unit_info(p, ua, u1, tbl, j0), b, kh, st, lane);
      issue_unit<T, D>(p, unit_info(p, ua + 1, u1, tbl, j0), b, kh, st + C::kHalfBytes, lane);
    }
    cp_commit();
  }

  const int hh0 = 2 * (t & 1);  // heads of this thread's score / output columns
  const int my_unit = t >> 1;   // unit of this thread's valid score columns
  for (int i = 0; i < my_tiles; ++i) {
    {  // keep kStages-1 tiles in flight
      const int ni = i + C::kStages - 1;
      if (ni < my_tiles) {
        const int ua = u0 + 2 * (warp + kWarps * ni);
        unsigned char* st = ring + (size_t)(ni % C::kStages) * C::kStageBytes;
        issue_unit<T, D>(p, unit_info(p, ua, u1, tbl, j0), b, kh, st, lane);
        issue_unit<T, D>(p, unit_info(p, ua + 1, u1, tbl, j0), b, kh, st + C::kHalfBytes, lane);
      }
      cp_commit();
    }
    cp_wait<C::kStages - 1>();
    __syncwarp();
    const int ua = u0 + 2 * (warp + kWarps * i);
    const Unit UA = unit_info(p, ua, u1, tbl, j0), UB = unit_info(p, ua + 1, u1, tbl, j0);
    // operand class of each unit's MMAs: 0 = KV dtype (fp units), 1 = fp16
    // (int4 pages, whose fp16 scale/zero make fp16 the exact dequant type);
    // a missing unit follows the other one
    const int clsA = (UA.kind == 2 || (UA.kind == 0 && UB.kind == 2)) ? 1 : 0;
    const int clsB = (UB.kind == 2 || (UB.kind == 0 && UA.kind == 2)) ? 1 : 0;
    unsigned char* st = ring + (size_t)(i % C::kStages) * C::kStageBytes;
    const uint32_t st_s = smem_u32(st);

    // ---- B fragments of the query for this thread's column (unit g>>2) ----
    uint32_t qB[KB][2];
    {
      if (((g >> 2) ? UB.kind : UA.kind) == 2) {
        const float* cs = reinterpret_cast<const float*>(st + (g >> 2) * C::kHalfBytes + C::kPageBytes);
        const float* sn = cs + D / 2;
#pragma unroll
        for (int kb = 0; kb < KB / 2; ++kb) {
          const float2 c0 = *reinterpret_cast<const float2*>(cs + 16 * kb + 2 * t);
          const float2 c1 = *reinterpret_cast<const float2*>(cs + 16 * kb + 2 * t + 8);
          const float2 s0 = *reinterpret_cast<const float2*>(sn + 16 * kb + 2 * t);
          const float2 s1 = *reinterpret_cast<const float2*>(sn + 16 * kb + 2 * t + 8);
          const float cc[4] = {c0.x, c0.y, c1.x, c1.y}, ss[4] = {s0.x, s0.y, s1.x, s1.y};
          float xr[4], yr[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float x = qf[kb][e], y = qf[kb + KB / 2][e];
            xr[e] = fmaf(x, cc[e], y * ss[e]);
            yr[e] = fmaf(y, cc[e], -x * ss[e]);
          }
          qB[kb][0] = H::pack(xr[0], xr[1]);
          qB[kb][1] = H::pack(xr[2], xr[3]);
          qB[kb + KB / 2][0] = H::pack(yr[0], yr[1]);
          qB[kb + KB / 2][1] = H::pack(yr[2], yr[3]);
        }
      } else {
#pragma unroll
        for (int kb = 0; kb < KB; ++kb) { qB[kb][0] = qb[kb][0]; qB[kb][1] = qb[kb][1]; }
      }
    }

    // ---- S = K q (16 tokens x 8 columns) ----
    float sacc[4] = {0.f, 0.f, 0.f, 0.f};
    {
      uint32_t ka[2][KB][2];  // [unit][kb][lo/hi 8 columns]
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t hb = st_s + h * C::kHalfBytes;
        if ((h ? UB.kind : UA.kind) == 2) {
          const unsigned char* pg = st + h * C::kHalfBytes;
          uint32_t w[NW];
#pragma unroll
          for (int e = 0; e < NW; ++e)
            w[e] = reinterpret_cast<const uint32_t*>(pg)[(g * 4 + t) * NW + e];
          uint32_t sz[NW];
#pragma unroll
          for (int e = 0; e < NW; ++e)
            sz[e] = reinterpret_cast<const uint32_t*>(pg + page_k_scales_off(D))[g * NW + e];
#pragma unroll
          for (int kb = 0; kb < KB; ++kb) {
            const uint32_t szw = sz[kb >> 1];
            const uint32_t s2 = __byte_perm(szw, szw, 0x1010);
            const uint32_t z2 = __byte_perm(szw, szw, 0x3232);
            ka[h][kb][0] = H::fma2(H::codes(w[kb >> 1], 2 * (kb & 1)), s2, z2);
            ka[h][kb][1] = H::fma2(H::codes(w[kb >> 1], 2 * (kb & 1) + 1), s2, z2);
          }
        } else {
          const int r = lane & 7, sel = (lane >> 3) & 1;
#pragma unroll
          for (int kb = 0; kb < KB; ++kb)
            ldsm_x2(ka[h][kb][0], ka[h][kb][1], hb + r * (2 * D) + (((2 * kb + sel) ^ r) * 16));
        }
      }
      if (!kBF || clsA == clsB) {
#pragma unroll
        for (int kb = 0; kb < KB; ++kb) {
          if (kBF && clsA == 1)
            H::mma(sacc, ka[0][kb][0], ka[1][kb][0], ka[0][kb][1], ka[1][kb][1], qB[kb][0], qB[kb][1]);
          else
            O::mma(sacc, ka[0][kb][0], ka[1][kb][0], ka[0][kb][1], ka[1][kb][1], qB[kb][0], qB[kb][1]);
        }
      } else {
        // tier boundary in a bf16 cache: one MMA per operand type, the other
        // unit's rows and the other columns' query zeroed
        const bool colF16 = ((g >> 2) ? clsB : clsA) == 1;
#pragma unroll
        for (int kb = 0; kb < KB; ++kb) {
          const uint32_t n0 = clsA == 0 ? 0xFFFFFFFFu : 0u, n1 = clsB == 0 ? 0xFFFFFFFFu : 0u;
          O::mma(sacc, ka[0][kb][0] & n0, ka[1][kb][0] & n1, ka[0][kb][1] & n0, ka[1][kb][1] & n1,
                 colF16 ? 0u : qB[kb][0], colF16 ? 0u : qB[kb][1]);
          H::mma(sacc, ka[0][kb][0] & ~n0, ka[1][kb][0] & ~n1, ka[0][kb][1] & ~n0, ka[1][kb][1] & ~n1,
                 colF16 ? qB[kb][0] : 0u, colF16 ? qB[kb][1] : 0u);
        }
      }
    }

    // ---- online softmax (log2 domain) for this thread's two heads ----
    const bool v = g < (my_unit ? UB.valid : UA.valid);
    float sc[2];
    sc[0] = v ? (my_unit ? sacc[2] : sacc[0]) * p.scale_log2 : -INFINITY;
    sc[1] = v ? (my_unit ? sacc[3] : sacc[1]) * p.scale_log2 : -INFINITY;
    float pr[2], alpha[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float mx = sc[e];
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
      const float mn = fmaxf(m_run[e], mx);
      alpha[e] = (mn == -INFINITY) ? 1.f : exp2f(m_run[e] - mn);
      pr[e] = v ? exp2f(sc[e] - mn) : 0.f;
      l_run[e] = l_run[e] * alpha[e] + pr[e];
      m_run[e] = mn;
    }
#pragma unroll
    for (int mb = 0; mb < KB; ++mb) {
      o[mb][0] *= alpha[0]; o[mb][1] *= alpha[1];
      o[mb][2] *= alpha[0]; o[mb][3] *= alpha[1];
    }
    // window mass of each unit: sum over its 8 rows
    {
      float ms0 = pr[0], ms1 = pr[1];
      ms0 += __shfl_xor_sync(0xffffffffu, ms0, 4);
      ms1 += __shfl_xor_sync(0xffffffffu, ms1, 4);
      ms0 += __shfl_xor_sync(0xffffffffu, ms0, 8);
      ms1 += __shfl_xor_sync(0xffffffffu, ms1, 8);
      ms0 += __shfl_xor_sync(0xffffffffu, ms0, 16);
      ms1 += __shfl_xor_sync(0xffffffffu, ms1, 16);
      if (lane < 4) {
        float* ms = mass_s + i * 12;
        ms[my_unit * 4 + hh0] = ms0;
        ms[my_unit * 4 + hh0 + 1] = ms1;
        if (my_unit == 0) { ms[8 + hh0] = m_run[0]; ms[8 + hh0 + 1] = m_run[1]; }
      }
    }

    // ---- O^T += V^T P ----
    const float xa = my_unit == 0 ? pr[0] : 0.f, xb = my_unit == 0 ? pr[1] : 0.f;
    const float ya = my_unit == 1 ? pr[0] : 0.f, yb = my_unit == 1 ? pr[1] : 0.f;
    const uint32_t px = (kBF && clsA == 1) ? H::pack(xa, xb) : O::pack(xa, xb);
    const uint32_t py = (kBF && clsB == 1) ? H::pack(ya, yb) : O::pack(ya, yb);
    const uint32_t pb0 = movm_t(px), pb1 = movm_t(py);
    {
      uint32_t va[2][KB][2];  // [unit][mb][d rows g / g+8]
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t hb = st_s + h * C::kHalfBytes;
        if ((h ? UB.kind : UA.kind) == 2) {
          const unsigned char* pg = st + h * C::kHalfBytes;
          uint32_t w[NW];
#pragma unroll
          for (int e = 0; e < NW; ++e)
            w[e] = reinterpret_cast<const uint32_t*>(pg + page_v_codes_off(D))[(t * 8 + g) * NW + e];
#pragma unroll
          for (int mb = 0; mb < KB; ++mb) {
            const uint2 sz = reinterpret_cast<const uint2*>(pg + page_v_scales_off(D))[t * NW + (mb >> 1)];
            va[h][mb][0] = H::fma2(H::codes(w[mb >> 1], 2 * (mb & 1)), sz.x, sz.y);
            va[h][mb][1] = H::fma2(H::codes(w[mb >> 1], 2 * (mb & 1) + 1), sz.x, sz.y);
          }
        } else {
          const int r = lane & 7, sel = (lane >> 3) & 1;
          const int nv = h ? UB.valid : UA.valid;
          const uint32_t msk = (2 * t < nv ? 0x0000FFFFu : 0u) | (2 * t + 1 < nv ? 0xFFFF0000u : 0u);
#pragma unroll
          for (int mb = 0; mb < KB; ++mb) {
            ldsm_x2_t(va[h][mb][0], va[h][mb][1], hb + 16 * D + r * (2 * D) + (((2 * mb + sel) ^ r) * 16));
            va[h][mb][0] &= msk;
            va[h][mb][1] &= msk;
          }
        }
      }
      if (!kBF || clsA == clsB) {
#pragma unroll
        for (int mb = 0; mb < KB; ++mb) {
          if (kBF && clsA == 1)
            H::mma(o[mb], va[0][mb][0], va[0][mb][1], va[1][mb][0], va[1][mb][1], pb0, pb1);
          else
            O::mma(o[mb], va[0][mb][0], va[0][mb][1], va[1][mb][0], va[1][mb][1], pb0, pb1);
        }
      } else {
        const uint32_t n0 = clsA == 0 ? 0xFFFFFFFFu : 0u, n1 = clsB == 0 ? 0xFFFFFFFFu : 0u;
#pragma unroll
        for (int mb = 0; mb < KB; ++mb) {
          O::mma(o[mb], va[0][mb][0] & n0, va[0][mb][1] & n0, va[1][mb][0] & n1, va[1][mb][1] & n1,
                 pb0 & n0, pb1 & n1);
          H::mma(o[mb], va[0][mb][0] & ~n0, va[0][mb][1] & ~n0, va[1][mb][0] & ~n1, va[1][mb][1] & ~n1,
                 pb0 & ~n0, pb1 & ~n1);
        }
      }
    }
    __syncwarp();
  }
  cp_wait<0>();

  // ---- warp epilogue: totals per head ----
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    float l = l_run[e];
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    l += __shfl_xor_sync(0xffffffffu, l, 4);
    l += __shfl_xor_sync(0xffffffffu, l, 8);
    l += __shfl_xor_sync(0xffffffffu, l, 16);
    l_run[e] = l;
  }
#pragma unroll
  for (int mb = 0; mb < KB; ++mb)
#pragma unroll
    for (int c = 0; c < 4; ++c) o[mb][c] += __shfl_xor_sync(0xffffffffu, o[mb][c], 2);

  __syncthreads();  // ring and table are free: reuse them for the CTA merge
  float* wm = reinterpret_cast<float*>(smem);       // [kWarps][4]
  float* wl = wm + kWarps * 4;                      // [kWarps][4]
  float* wo = wl + kWarps * 4;                      // [kWarps][4][D]
  if (lane < 2) {
    wm[warp * 4 + 2 * lane] = m_run[0];
    wm[warp * 4 + 2 * lane + 1] = m_run[1];
    wl[warp * 4 + 2 * lane] = l_run[0];
    wl[warp * 4 + 2 * lane + 1] = l_run[1];
  }
  if (t < 2) {
#pragma unroll
    for (int mb = 0; mb < KB; ++mb) {
      wo[(warp * 4 + hh0) * D + 16 * mb + g] = o[mb][0];
      wo[(warp * 4 + hh0 + 1) * D + 16 * mb + g] = o[mb][1];
      wo[(warp * 4 + hh0) * D + 16 * mb + g + 8] = o[mb][2];
      wo[(warp * 4 + hh0 + 1) * D + 16 * mb + g + 8] = o[mb][3];
    }
  }
  __syncthreads();
  __shared__ float s_M[4];
  if (threadIdx.x < 4) {
    float M = -INFINITY;
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, wm[w * 4 + threadIdx.x]);
    s_M[threadIdx.x] = M;
  }
  __syncthreads();
  float* part = p.part + (((int64_t)b * p.Hkv + kh) * p.n_split + split) * 4 * (D + 2);
  for (int e = threadIdx.x; e < 4 * (D + 2); e += kThreads) {
    const int hh = e / (D + 2), c = e % (D + 2);
    const float M = s_M[hh];
    float acc = 0.f;
    if (c == D) {
      acc = M;
    } else {
      for (int w = 0; w < kWarps; ++w) {
        const float mw = wm[w * 4 + hh];
        if (mw == -INFINITY) continue;
        acc += exp2f(mw - M) * (c == D + 1 ? wl[w * 4 + hh] : wo[(w * 4 + hh) * D + c]);
      }
    }
    part[e] = acc;
  }
  // window masses of this warp's units, relative to the CTA max
  const float* msw = reinterpret_cast<const float*>(smem + C::kRingBytes) + warp * kMaxTilesPerWarp * 12;
  for (int e = lane; e < my_tiles * 8; e += 32) {
    const int i = e >> 3, h = (e >> 2) & 1, hh = e & 3;
    const int ua = u0 + 2 * (warp + kWarps * i);
    const int u = ua + h;
    if (u >= u1) continue;
    int window;
    if (u < p.NS) window = -1;
    else window = u - p.NS;  // tier page j -> window j; rest unit r -> n_tp + r
    if (window < 0) continue;
    const float mt = msw[i * 12 + 8 + hh];
    const float val = (mt == -INFINITY) ? 0.f : msw[i * 12 + h * 4 + hh] * exp2f(mt - s_M[hh]);
    p.mass[((int64_t)b * p.Hkv * 4 + kh * 4 + hh) * p.W + window] = val;
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(128) decode_mma_merge_kernel(const __grid_constant__ MmaParams p) {
  const int b = blockIdx.y, h = blockIdx.x;
  const int kh = h >> 2, hh = h & 3;
  const int Hq = p.Hkv * 4;
  __shared__ float s_f[kMaxSplits];
  __shared__ float s_M, s_invL;
  const float* part = p.part + ((int64_t)b * p.Hkv + kh) * p.n_split * 4 * (D + 2);
  if (threadIdx.x == 0) {
    float M = -INFINITY;
    for (int s = 0; s < p.n_split; ++s) M = fmaxf(M, part[(s * 4 + hh) * (D + 2) + D]);
    float L = 0.f;
    for (int s = 0; s < p.n_split; ++s) {
      const float ms = part[(s * 4 + hh) * (D + 2) + D];
      const float f = ms == -INFINITY ? 0.f : exp2f(ms - M);
      s_f[s] = f;
      L += f * part[(s * 4 + hh) * (D + 2) + D + 1];
    }
    s_M = M;
    s_invL = 1.f / L;
  }
  __syncthreads();
  const float invL = s_invL;
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < p.n_split; ++s) acc += s_f[s] * part[(s * 4 + hh) * (D + 2) + c];
    st_f32((T*)p.out + b * p.o_sb + h * p.o_sh + c, acc * invL);
  }
  if (p.scores == nullptr) return;
  const float* ms = p.mass + ((int64_t)b * Hq + h) * p.W;
  float* acc = p.scores + ((int64_t)b * Hq + h) * p.scores_cap;
  for (int w = threadIdx.x; w < p.W; w += blockDim.x) {
    const int u = p.NS + w;
    int lo = 0, hi = p.n_split - 1;  // split s with bnd[s] <= u < bnd[s+1]
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (p.bnd[mid] <= u) lo = mid; else hi = mid - 1;
    }
    acc[w] += ms[w] * s_f[lo] * invL;
  }
}

template <int D>
void plan_splits(MmaParams& p) {
  using C = Cfg<D>;
  const double c_fp = 32.0 * D, c_i4 = (double)(C::kPageBytes + 4 * D);
  const double total = p.NS * c_fp + p.n_tp * c_i4 + (p.U - p.NS - p.n_tp) * c_fp;
  const int units = p.B * p.Hkv;
  const int resident = D == 64 ? 4 : 2;
  int n = ceil_div(2 * 148 * resident, units > 0 ? units : 1);
  n = max(n, ceil_div(p.U, kMaxUnitsPerSplit));
  n = min(n, kMaxSplits);
  n = min(n, max(1, (p.U + 15) / 16));
  auto unit_at = [&](double x) -> int {  // first unit whose cumulative cost reaches x
    const double a = p.NS * c_fp, bcost = a + p.n_tp * c_i4;
    if (x <= a) return (int)(x / c_fp);
    if (x <= bcost) return p.NS + (int)((x - a) / c_i4);
    return p.NS + p.n_tp + (int)((x - bcost) / c_fp);
  };
  p.bnd[0] = 0;
  int k = 1;
  for (int s = 1; s < n; ++s) {
    int u = unit_at(total * s / n) & ~1;
    u = max(u, p.bnd[k - 1] + 2);
    if (u >= p.U) break;
    if (u - p.bnd[k - 1] > kMaxUnitsPerSplit) u = p.bnd[k - 1] + kMaxUnitsPerSplit;
    p.bnd[k++] = u;
  }
  while (p.U - p.bnd[k - 1] > kMaxUnitsPerSplit && k < kMaxSplits) {
    p.bnd[k] = p.bnd[k - 1] + kMaxUnitsPerSplit;
    ++k;
  }
  p.bnd[k] = p.U;
  p.n_split = k;
}

template <typename T, int D>
int launch_mma(MmaParams& p, cudaStream_t stream) {
  using C = Cfg<D>;
  static_assert(C::kSmemBytes <= 227 * 1024, "smem");
  cudaFuncSetAttribute(decode_mma_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::kSmemBytes);
  dim3 grid(p.n_split, p.Hkv, p.B);
  decode_mma_kernel<T, D><<<grid, kThreads, C::kSmemBytes, stream>>>(p);
  SKV_CHECK_LAUNCH();
  decode_mma_merge_kernel<T, D><<<dim3(p.Hkv * 4, p.B), 128, 0, stream>>>(p);
  SKV_CHECK_LAUNCH();
  return SKV_OK;
}

struct MmaWs {
  size_t part, mass, total;
};
MmaWs mma_ws(const skv_layer_desc* L, int T) {
  MmaWs w{};
  const int W = T > L->num_sink ? (T - L->num_sink + L->window_size - 1) / L->window_size : 0;
  w.part = align_up((size_t)L->batch * L->num_kv_heads * kMaxSplits * 4 * (L->head_dim + 2) * 4, 256);
  w.mass = align_up((size_t)L->batch * L->num_q_heads * (W > 0 ? W : 1) * 4, 256);
  w.total = w.part + w.mass;
  return w;
}

}  // namespace

bool decode_mma_supported(const skv_layer_desc* L) {
  return (L->kv_dtype == SKV_F16 || L->kv_dtype == SKV_BF16) && (L->head_dim == 64 || L->head_dim == 128) &&
         L->num_q_heads == 4 * L->num_kv_heads && L->window_size == kPageTokens && L->fp_capacity % 8 == 0;
}

size_t decode_mma_ws_size(const skv_layer_desc* L, int T) { return mma_ws(L, T).total; }

int decode_mma(const skv_layer_desc* L, int T, int tier_pages, const void* q, int64_t q_sb, int64_t q_sh,
               void* out, int64_t o_sb, int64_t o_sh, float scaling, float* scores, int scores_cap, void* ws,
               cudaStream_t stream) {
  if ((q_sb % 2) || (q_sh % 2) || ((uintptr_t)q % 4)) return SKV_ERR_MISALIGNED;  // 32-bit query loads
  MmaParams p{};
  const MmaWs w = mma_ws(L, T);
  p.k_fp = L->k_fp; p.v_fp = L->v_fp; p.pages = L->tier_pages; p.table = L->tier_table;
  p.cos = L->rope_cos; p.sin = L->rope_sin; p.q = q; p.out = out; p.scores = scores;
  p.part = (float*)ws;
  p.mass = (float*)((char*)ws + w.part);
  p.q_sb = q_sb; p.q_sh = q_sh; p.o_sb = o_sb; p.o_sh = o_sh;
  p.B = L->batch; p.Hkv = L->num_kv_heads; p.cap = L->fp_capacity; p.page_cap = L->tier_page_capacity;
  p.scores_cap = scores_cap;
  p.s = L->num_sink; p.s_pad = L->sink_pad; p.n_tp = tier_pages;
  p.s_eff = T < p.s ? T : p.s;
  p.NS = ceil_div(p.s_eff, kPageTokens);
  p.rest = T > p.s ? T - p.s - tier_pages * kPageTokens : 0;
  p.U = p.NS + p.n_tp + ceil_div(p.rest, kPageTokens);
  p.W = T > p.s ? (T - p.s + kPageTokens - 1) / kPageTokens : 0;
  p.scale_log2 = scaling * kLog2e;
  if (p.U == 0) return SKV_ERR_INVALID_ARG;
  switch (L->head_dim) {
    case 64: plan_splits<64>(p); break;
    case 128: plan_splits<128>(p); break;
  }
  if (L->kv_dtype == SKV_F16)
    return L->head_dim == 64 ? launch_mma<__half, 64>(p, stream) : launch_mma<__half, 128>(p, stream);
  return L->head_dim == 64 ? launch_mma<__nv_bfloat16, 64>(p, stream)
                           : launch_mma<__nv_bfloat16, 128>(p, stream);
}

}  // namespace skv
