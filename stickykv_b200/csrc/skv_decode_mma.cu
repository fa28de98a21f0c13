// Tensor-core decode attention with fused window mass (fp16/bf16 KV,
// window_size a multiple of 8, any number of query heads per KV head,
// head_dim 64 or 128).
//
// Same contract as the portable path (skv_decode_generic.cu): replaces the
// reference's attention + score hook + scorer for one decode query
// (modules/windowed_eager_cache/hooks.py:145-180, modules/windowed_cache/
// hooks.py:199-290, scorer.py:17-109).
//
// The retained cache of one (row, kv head) is a sequence of 8-token units:
// [sink unit(s) | int4 tier pages | fp units after the tier].  A scoring
// window is window_size / 8 consecutive units after the sinks (one unit at
// window_size 8): the kernel records the mass of every unit, the merge sums
// a window's units.  A tile is two consecutive units (16 tokens).
//
// Query heads are handled in groups of four MMA columns, ceil(G / 4) groups
// per kv head (each reads the kv head's cache once); the spare columns of a
// short group (GQA 1, 2, 3, 5, 6, 7 ...) carry a zero query and are never
// stored.
//
// Work split: one CTA per (row, head group, unit range); ranges are balanced by
// an estimated per-tile cost.  Each of the 4 warps takes a contiguous run of
// the CTA's tiles (again cost-balanced) and streams it through a private
// cp.async ring in shared memory, so the main loop has no CTA barrier.  A
// warp's run splits into at most five homogeneous segments (sinks, int4
// pages, tier/fp boundary, full fp units, ragged tail) whose bounds are
// computed up front; int4 and full-fp segments run specialised straight-line
// tile bodies with per-lane addresses fixed for the whole kernel.  Per tile:
//   QK  mma.m16n8k16: rows = 16 tokens, columns = 4 heads x 2 units; unit A's
//       keys only meet columns 0-3, unit B's columns 4-7, so each column
//       group carries the query of its unit: unrotated for fp units, rotated
//       to the page start R(-P) q (and pre-scaled into the log2 domain) for
//       int4 pages, whose keys are stored in their page frame.  The rotated
//       query steps R(-16) from one tile to the next (packed f32x2 math).
//       int4 K codes enter the MMA raw, masked into exact fp16 subnormals
//       (per-group accumulators; each token's scale and zero point are
//       applied to its score afterwards, the zero point through the group
//       sums of the query from one more MMA); int4 V codes are expanded by
//       magic-number OR into fp16 and dequantised with one packed FMA per two
//       channels, straight into A fragments.
//   softmax in the log2 domain, online per warp with lazy rescaling; the
//       window mass of each unit is the sum of its 8 rows.
//   PV  mma: O^T = V^T P, V^T fragments via ldmatrix.trans (fp) or
//       dequantised codes (int4); P converted with movmatrix.trans.
// The CTA merges its warps and writes (max, sum, O) and the window masses
// relative to its max; a merge kernel combines the splits, writes the output
// and adds the normalised window mass to the fp32 score accumulator.
#include <float.h>

#include <type_traits>

#include "skv_mma.cuh"

namespace skv {
namespace {

using namespace mma;

constexpr int kWarps = 4;
constexpr int kThreads = 32 * kWarps;
constexpr int kMaxSplits = 64;
constexpr int kMaxTilesPerCta = 128;
constexpr int kMaxUnitsPerSplit = 2 * kMaxTilesPerCta;
constexpr float kLog2e = 1.4426950408889634f;
constexpr int kRotStep = 16;  // positions from one int4 tile of a warp to its next

template <int D> struct Cfg {
  static constexpr int kHalfBytes = 32 * D;           // one fp unit: 8 K rows + 8 V rows
  static constexpr int kTileBytes = 2 * kHalfBytes;   // one fp tile slot
  static constexpr int kPageBytes = page_bytes(D);
  static constexpr int kCPR = D / 8;                  // 16-byte chunks per fp row
  static constexpr int kKB = D / 16;                  // k-blocks (QK) == m-blocks (PV)
  static constexpr int kNW = D / 32;                  // int4 words per (row, lane)
  static constexpr int kFpSlots = 3;
  static constexpr int kWarpRing = kFpSlots * kTileBytes;
  static constexpr int kI4Slots = kWarpRing / (2 * kPageBytes) < 8 ? kWarpRing / (2 * kPageBytes) : 8;
  static constexpr size_t kRingBytes = (size_t)kWarps * kWarpRing;
  static constexpr size_t kMassBytes = (size_t)kMaxTilesPerCta * 12 * 4;
  static constexpr size_t kTableBytes = (size_t)kMaxUnitsPerSplit * 4;
  static constexpr size_t kSmemBytes = kRingBytes + kMassBytes + kTableBytes;
  static_assert(kI4Slots >= 2, "int4 ring");
};

// relative per-tile costs used to balance CTAs and warps
constexpr int kCostGeneric = 5, kCostI4 = 3, kCostFp = 2;

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
  float* part;     // [B][Hv][n_split][4][D+2]: O, max (log2 domain), sum
  float* mass;     // [B][Hv][4][W]: unit mass relative to its split's max
  const void* k_new;  // optional token appended by the last split's blocks
  const void* v_new;
  int64_t q_sb, q_sh, o_sb, o_sh, kn_sb, kn_sh;
  int new_slot;       // fp slot of the appended token
  int B, Hkv, cap, page_cap, scores_cap, n_split;
  // query-head groups: the kernel works on Hv groups of up to 4 query heads,
  // ngrp = ceil(G / 4) per kv head (its K/V read once per group); group j of
  // kv head r holds query heads r*G + 4j ... + min(4, G - 4j) - 1, and the
  // spare columns of a short group carry a zero query and are never stored.
  int Hq, Hv, G, ngrp;
  int s, s_eff, s_pad, NS, n_tp, rest, U, W, rope_rows;
  int upw, Ww;  // 8-token units per window (window_size / 8) and windows; W counts units
  int merge_per;  // windows per merge thread (1 or 2)
  float scale_log2;
  int bnd[kMaxSplits + 1];
};

// ---------------------------------------------------------------------------
// operand-type specifics
// ---------------------------------------------------------------------------
using H = Op<__half>;  // int4 pages are always computed in fp16 (their scale/zero are fp16)

// int4 nibble pairs -> exact fp16 codes.  A word holds nibbles i (bits 4i..)
// in its low half and i+4 in its high half.  Nibbles at bits 0-3 of a half
// become 1024 + code when OR-ed into 0x6400 (1024.0, ulp 1); nibbles at bits
// 4-7 become 64 + code when OR-ed into 0x5400 (64.0, ulp 1/16).  One shift
// by 8 serves nibbles 2 and 3.  The subtraction is exact.
template <int I>
__device__ __forceinline__ uint32_t codes_f16(uint32_t lo, uint32_t hi) {
  const uint32_t w = I < 2 ? lo : hi;
  if constexpr ((I & 1) == 0) {
    const uint32_t x = (w & 0x000F000Fu) | 0x64006400u;
    return u32(__hsub2(h2(x), h2(0x64006400u)));
  } else {
    const uint32_t x = (w & 0x00F000F0u) | 0x54005400u;
    return u32(__hsub2(h2(x), h2(0x54005400u)));
  }
}
__device__ __forceinline__ uint32_t dq(uint32_t c, __half2 s, __half2 z) { return u32(__hfma2(h2(c), s, z)); }

template <int N> struct Words { uint32_t w[N]; };
template <int N>
__device__ __forceinline__ Words<N> lds_words(uint32_t addr) {
  Words<N> r;
  if constexpr (N == 2) {
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];\n" : "=r"(r.w[0]), "=r"(r.w[1]) : "r"(addr));
  } else {
    static_assert(N % 4 == 0, "words");
#pragma unroll
    for (int k = 0; k < N / 4; ++k)
      asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                   : "=r"(r.w[4 * k]), "=r"(r.w[4 * k + 1]), "=r"(r.w[4 * k + 2]), "=r"(r.w[4 * k + 3])
                   : "r"(addr + 16 * k));
  }
  return r;
}
// (d0, d1) = (a0, a1) * (b0, b1) + (c0, c1), one packed fp32 FMA
__device__ __forceinline__ void fma_x2(float& d0, float& d1, float a0, float a1, float b0, float b1, float c0,
                                       float c1) {
  asm("{.reg .b64 ra, rb, rc, rd;\n"
      " mov.b64 ra, {%2,%3};\n mov.b64 rb, {%4,%5};\n mov.b64 rc, {%6,%7};\n"
      " fma.rn.f32x2 rd, ra, rb, rc;\n mov.b64 {%0,%1}, rd;}\n"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}
__device__ __forceinline__ void mul_x2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
  asm("{.reg .b64 ra, rb, rd;\n"
      " mov.b64 ra, {%2,%3};\n mov.b64 rb, {%4,%5};\n"
      " mul.rn.f32x2 rd, ra, rb;\n mov.b64 {%0,%1}, rd;}\n"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}


// floor division by 2 for possibly negative numerators
__device__ __forceinline__ int ceil_half(int x) { return (x + 1) >> 1; }

// Unit kinds: 0 none, 1 fp (KV dtype rows in the fp store), 2 int4 page.
struct Regions {
  int NS, TB, U, u1;  // sinks [0,NS), tier [NS,TB), fp rest [TB,U); split end u1
  __device__ __forceinline__ int kind(int u) const { return u >= u1 ? 0 : ((u >= NS && u < TB) ? 2 : 1); }
};

__device__ __forceinline__ int fp_slot0(const MmaParams& p, const Regions& R, int u) {
  return u < R.NS ? 8 * u : p.s_pad + 8 * (u - R.TB);
}
__device__ __forceinline__ int fp_valid(const MmaParams& p, const Regions& R, int u) {
  return u < R.NS ? min(8, p.s_eff - 8 * u) : min(8, p.rest - 8 * (u - R.TB));
}

// Tile classes of one CTA, in tile order: generic [0,ia) | int4 [ia,ib) |
// generic [ib,fa) | full fp [fa,fb) | generic [fb,n).
struct TileRuns {
  int ia, ib, fa, fb, n;
  __device__ __forceinline__ int cost_before(int i) const {  // cost of tiles [0, i)
    const int c_i4 = max(0, min(i, ib) - ia), c_fp = max(0, min(i, fb) - fa);
    return kCostGeneric * (i - c_i4 - c_fp) + kCostI4 * c_i4 + kCostFp * c_fp;
  }
  // smallest i with cost_before(i) >= target (n if none): the cost grows
  // linearly inside each class segment, so walk the five segments
  __device__ __forceinline__ int at_cost(int target) const {
    if (target <= 0) return 0;
    const int end[5] = {ia, ib, fa, fb, n};
    const int cost[5] = {kCostGeneric, kCostI4, kCostGeneric, kCostFp, kCostGeneric};
    int start = 0, c = 0;
#pragma unroll
    for (int s = 0; s < 5; ++s) {
      const int seg = (end[s] - start) * cost[s];
      if (c + seg >= target) return start + (target - c + cost[s] - 1) / cost[s];
      c += seg;
      start = end[s];
    }
    return n;
  }
};

template <typename T, int D>
__global__ void __launch_bounds__(kThreads, D == 64 ? 4 : 2) decode_mma_kernel(const __grid_constant__ MmaParams p) {
  using C = Cfg<D>;
  using O = Op<T>;        // fp units: the KV dtype
  constexpr bool kBF = !std::is_same<T, __half>::value;
  constexpr int KB = C::kKB, NW = C::kNW, PB = C::kPageBytes, HS = C::kHalfBytes;
  constexpr int FPJ = C::kCPR / 2;                        // cp.async per lane per fp tensor per tile
  constexpr int FP_PER = C::kCPR / 4;                     // swizzle period of those chunks
  constexpr int FP_IT = 8 * C::kCPR / 32;                 // cp.async per lane per fp tensor per unit
  constexpr int PG_CH = PB / 16;                          // 16-byte chunks per page
  constexpr int PG_IT = (PG_CH + 31) / 32;
  constexpr float kThresh = 8.f;                          // lazy rescale margin (log2 domain)
  extern __shared__ __align__(128) unsigned char smem[];
  const int split = blockIdx.x, kh = blockIdx.y, b = blockIdx.z;  // kh: query-head group
  const int kr = kh / p.ngrp;                                      // its kv head
  const int hbase = kr * p.G + 4 * (kh - kr * p.ngrp);             // its first query head
  const int nlive = min(4, p.G - (hbase - kr * p.G));              // its query heads
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int u0 = p.bnd[split], u1 = p.bnd[split + 1];
  const int n_tiles = (u1 - u0 + 1) >> 1;
  const Regions R{p.NS, p.NS + p.n_tp, p.U, u1};

  unsigned char* ring = smem + (size_t)warp * C::kWarpRing;
  const uint32_t ring_s = smem_u32(ring);
  float* mass_s = reinterpret_cast<float*>(smem + C::kRingBytes);  // [tile][12]
  int* tbl = reinterpret_cast<int*>(smem + C::kRingBytes + C::kMassBytes);  // [unit - u0]

  if (p.k_new != nullptr && split == p.n_split - 1) {
    // fused append: the last unit holds the new token; write its key and
    // value rows before any copy of this block reads them (the barrier below
    // orders the stores before the cp.async reads)
    constexpr int VPR = D / 8;  // 16-byte vectors per row
    const int64_t row = (((int64_t)b * p.Hkv + kr) * p.cap + p.new_slot) * D;
    for (int e = threadIdx.x; e < 2 * VPR; e += kThreads) {
      const int which = e / VPR, c = e - which * VPR;
      const T* src = (const T*)(which ? p.v_new : p.k_new) + b * p.kn_sb + kr * p.kn_sh + c * 8;
      T* dst = (T*)(which ? p.v_fp : p.k_fp) + row + c * 8;
      *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
    }
  }
  {  // page table slice, indexed by unit offset within the split
    const int k0 = max(0, R.NS - u0), k1 = min(u1, R.TB) - u0;
    const int32_t* src = p.table + (int64_t)b * p.page_cap + (u0 - R.NS);
    for (int k = k0 + threadIdx.x; k < k1; k += kThreads) tbl[k] = src[k];
  }

  // tile classes and this warp's contiguous, cost-balanced run [tb, te)
  TileRuns tr;
  tr.n = n_tiles;
  tr.ia = min(n_tiles, max(0, ceil_half(R.NS - u0)));
  tr.ib = max(tr.ia, min(n_tiles, max(0, ceil_half(R.TB - 1 - u0))));
  {
    const int uf = min(R.TB + p.rest / 8, u1);  // first unit that is not a full fp unit
    tr.fa = max(tr.ib, min(n_tiles, max(0, ceil_half(R.TB - u0))));
    tr.fb = max(tr.fa, min(n_tiles, max(0, ceil_half(uf - 1 - u0))));
  }
  const int total = tr.cost_before(n_tiles);
  const int tb = warp == 0 ? 0 : tr.at_cost((total * warp + kWarps - 1) / kWarps);
  const int te = warp == kWarps - 1 ? n_tiles : tr.at_cost((total * (warp + 1) + kWarps - 1) / kWarps);
  __syncthreads();

  const int64_t kv_row = ((int64_t)b * p.Hkv + kr) * p.cap * D;
  const int64_t pg_row = ((int64_t)b * p.Hkv + kr) * p.page_cap;
  const T* kfp = (const T*)p.k_fp + kv_row;
  const T* vfp = (const T*)p.v_fp + kv_row;
  const unsigned char* pages_l = p.pages + pg_row * PB + lane * 16;

  // int4 page reads (per-lane offsets within a page)
  const uint32_t kc_off = lane * NW * 4;  // (g*4 + t) words of NW
  const uint32_t ks_off = page_k_scales_off(D) + g * NW * 4;
  const uint32_t vc_off = page_v_codes_off(D) + (t * 8 + g) * NW * 4;
  const uint32_t vs_off = page_v_scales_off(D) + t * NW * 8;

  // query of head (g & 3) in B-fragment order: d = 16kb + 2t + {0,1,8,9}
  const bool q_live = (g & 3) < nlive;  // columns past the group's heads carry a zero query
  const T* qp = (const T*)p.q + b * p.q_sb + (hbase + (q_live ? (g & 3) : 0)) * p.q_sh;
  const uint32_t q_bits = q_live ? 0xFFFFFFFFu : 0u;
  // query rotated to the page start of this thread's column (int4 columns)
  float rq[KB][4];
  int rq_pos = -1;
  const bool can_step = p.rope_rows > kRotStep;
  // rq = scl * R(-P) q; with `raw` the elements e >= 2 (k-rows 8..15 of each
  // k-block, which meet the odd nibbles of the raw int4 codes, 16x larger)
  // carry an extra 1/16 (exact: a power of two)
  // (channel pairs d, d+1 are read as one 8-byte cos/sin and one 4-byte
  // query load each)
  auto seed = [&](int P, float scl, bool raw) {
    union QPair { uint32_t u; T e[2]; };
#pragma unroll
    for (int kb = 0; kb < KB / 2; ++kb)
#pragma unroll
      for (int eh = 0; eh < 2; ++eh) {
        const int d = 16 * kb + 2 * t + 8 * eh;
        const float2 c = *reinterpret_cast<const float2*>(p.cos + (int64_t)P * (D / 2) + d);
        const float2 s = *reinterpret_cast<const float2*>(p.sin + (int64_t)P * (D / 2) + d);
        QPair xq, yq;
        xq.u = q_live ? *reinterpret_cast<const uint32_t*>(qp + d) : 0u;
        yq.u = q_live ? *reinterpret_cast<const uint32_t*>(qp + d + D / 2) : 0u;
        const float f = (raw && eh == 1) ? scl * 0.0625f : scl;
        const float x0 = ld_f32(&xq.e[0]), x1 = ld_f32(&xq.e[1]);
        const float y0 = ld_f32(&yq.e[0]), y1 = ld_f32(&yq.e[1]);
        rq[kb][2 * eh] = fmaf(x0, c.x, y0 * s.x) * f;
        rq[kb][2 * eh + 1] = fmaf(x1, c.y, y1 * s.y) * f;
        rq[kb + KB / 2][2 * eh] = fmaf(y0, c.x, -x0 * s.x) * f;
        rq[kb + KB / 2][2 * eh + 1] = fmaf(y1, c.y, -x1 * s.y) * f;
      }
  };

  auto load_qb = [&](uint32_t (&qb)[KB][2]) {
#pragma unroll
    for (int kb = 0; kb < KB; ++kb) {
      qb[kb][0] = *reinterpret_cast<const uint32_t*>(qp + 16 * kb + 2 * t) & q_bits;
      qb[kb][1] = *reinterpret_cast<const uint32_t*>(qp + 16 * kb + 2 * t + 8) & q_bits;
    }
  };

  float m_run[2] = {-INFINITY, -INFINITY}, m_thr[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  float o[KB][4];
#pragma unroll
  for (int mb = 0; mb < KB; ++mb) o[mb][0] = o[mb][1] = o[mb][2] = o[mb][3] = 0.f;

  const int hh0 = 2 * (t & 1);
  const int my_unit = t >> 1;
  const uint32_t maskA = my_unit ? 0u : 0xFFFFFFFFu;

  // int4 page -> K A-fragments (rows g of the page) and V^T A-fragments
  auto page_k = [&](uint32_t pg, uint32_t (&ka)[KB][2]) {
    const Words<NW> w = lds_words<NW>(pg + kc_off);
    const Words<NW> sz = lds_words<NW>(pg + ks_off);
#pragma unroll
    for (int q = 0; q < NW; ++q) {
      const uint32_t lo = w.w[q], hi = w.w[q] >> 8;
      const __half2 s2 = __low2half2(h2(sz.w[q])), z2 = __high2half2(h2(sz.w[q]));
      ka[2 * q][0] = dq(codes_f16<0>(lo, hi), s2, z2);
      ka[2 * q][1] = dq(codes_f16<1>(lo, hi), s2, z2);
      ka[2 * q + 1][0] = dq(codes_f16<2>(lo, hi), s2, z2);
      ka[2 * q + 1][1] = dq(codes_f16<3>(lo, hi), s2, z2);
    }
  };
  auto page_v = [&](uint32_t pg, uint32_t (&va)[KB][2]) {
    const Words<NW> w = lds_words<NW>(pg + vc_off);
    const Words<2 * NW> sz = lds_words<2 * NW>(pg + vs_off);
#pragma unroll
    for (int q = 0; q < NW; ++q) {
      const uint32_t lo = w.w[q], hi = w.w[q] >> 8;
      const __half2 s2 = h2(sz.w[2 * q]), z2 = h2(sz.w[2 * q + 1]);
      va[2 * q][0] = dq(codes_f16<0>(lo, hi), s2, z2);
      va[2 * q][1] = dq(codes_f16<1>(lo, hi), s2, z2);
      va[2 * q + 1][0] = dq(codes_f16<2>(lo, hi), s2, z2);
      va[2 * q + 1][1] = dq(codes_f16<3>(lo, hi), s2, z2);
    }
  };

  // raw K codes of an int4 page: the nibbles masked in place, each an exact
  // fp16 subnormal c * 2^-24 (even nibbles, A columns 2t..) or c * 2^-20 (odd
  // nibbles, columns 2t+8..; the query rows they meet carry 1/16), one logic
  // op per two codes; the scale and zero point are applied after the MMA.
  // (V codes are dequantised into A fragments: a scale folded into P plus
  // MMAs for the offsets and zero points measured slower.)
  auto page_k_raw = [&](uint32_t pg, uint32_t (&ka)[KB][2]) {
    const Words<NW> w = lds_words<NW>(pg + kc_off);
#pragma unroll
    for (int q = 0; q < NW; ++q) {
      const uint32_t lo = w.w[q], hi = w.w[q] >> 8;
      ka[2 * q][0] = lo & 0x000F000Fu;
      ka[2 * q][1] = lo & 0x00F000F0u;
      ka[2 * q + 1][0] = hi & 0x000F000Fu;
      ka[2 * q + 1][1] = hi & 0x00F000F0u;
    }
  };

  // ---- softmax (log2 domain) with lazy rescale, PV, window mass ----
  // sc0/sc1: this thread's two scores (row g of its unit, heads hh0, hh0+1),
  // -inf where the row holds no token.  kFp16P: P packed as fp16 for both
  // units (int4 tile, or bf16 cache tile whose units are all int4).
  auto softmax_p = [&](float sc0, float sc1, bool guard, float& pr0, float& pr1) {
    if (__any_sync(0xffffffffu, sc0 > m_thr[0] || sc1 > m_thr[1])) {
      float mx0 = sc0, mx1 = sc1;
#pragma unroll
      for (int off = 2; off < 32; off <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
      }
      const float mn0 = fmaxf(m_run[0], mx0), mn1 = fmaxf(m_run[1], mx1);
      const float al0 = mn0 == -INFINITY ? 1.f : ex2(m_run[0] - mn0);
      const float al1 = mn1 == -INFINITY ? 1.f : ex2(m_run[1] - mn1);
      l_run[0] *= al0;
      l_run[1] *= al1;
#pragma unroll
      for (int mb = 0; mb < KB; ++mb) {
        o[mb][0] *= al0; o[mb][1] *= al1;
        o[mb][2] *= al0; o[mb][3] *= al1;
      }
      m_run[0] = mn0;
      m_run[1] = mn1;
      m_thr[0] = mn0 + kThresh;
      m_thr[1] = mn1 + kThresh;
    }
    pr0 = ex2(sc0 - m_run[0]);
    pr1 = ex2(sc1 - m_run[1]);
    if (guard) {  // rows without a token (and nothing seen yet)
      pr0 = sc0 == -INFINITY ? 0.f : pr0;
      pr1 = sc1 == -INFINITY ? 0.f : pr1;
    }
    l_run[0] += pr0;
    l_run[1] += pr1;
  };
  // ---- window mass: sum of the unit's 8 rows per head (exact fp32) ----
  auto store_mass = [&](float pr0, float pr1, int i) {
    // lanes g, g^1 swap one head each, then reduce over the remaining g bits
    float a = (g & 1) ? pr1 : pr0;
    const float other = (g & 1) ? pr0 : pr1;
    a += __shfl_xor_sync(0xffffffffu, other, 4);
    a += __shfl_xor_sync(0xffffffffu, a, 8);
    a += __shfl_xor_sync(0xffffffffu, a, 16);
    if (lane < 8) {  // g in {0,1}: head hh0 + g of unit t>>1
      float* ms = mass_s + i * 12;
      ms[my_unit * 4 + hh0 + g] = a;
      if (lane < 2) *reinterpret_cast<float2*>(ms + 8 + hh0) = make_float2(m_run[0], m_run[1]);
    }
  };
  auto softmax_pv = [&](float sc0, float sc1, bool guard, uint32_t (&va)[2][KB][2], int mode_pv,
                        int clsA, int clsB, int i) {
    float pr0, pr1;
    softmax_p(sc0, sc1, guard, pr0, pr1);
    // ---- O^T += V^T P ----
    if (mode_pv == 1) {  // one operand type for both units
      const uint32_t pk = H::pack(pr0, pr1);
      const uint32_t pb0 = movm_t(pk & maskA), pb1 = movm_t(pk & ~maskA);
#pragma unroll
      for (int mb = 0; mb < KB; ++mb) H::mma(o[mb], va[0][mb][0], va[0][mb][1], va[1][mb][0], va[1][mb][1], pb0, pb1);
    } else if (mode_pv == 2) {
      const uint32_t pk = O::pack(pr0, pr1);
      const uint32_t pb0 = movm_t(pk & maskA), pb1 = movm_t(pk & ~maskA);
#pragma unroll
      for (int mb = 0; mb < KB; ++mb) O::mma(o[mb], va[0][mb][0], va[0][mb][1], va[1][mb][0], va[1][mb][1], pb0, pb1);
    } else {
      // bf16 cache, one int4 unit and one fp unit: one MMA per operand type
      const float xa = my_unit == 0 ? pr0 : 0.f, xb = my_unit == 0 ? pr1 : 0.f;
      const float ya = my_unit == 1 ? pr0 : 0.f, yb = my_unit == 1 ? pr1 : 0.f;
      const uint32_t pb0 = movm_t(clsA == 1 ? H::pack(xa, xb) : O::pack(xa, xb));
      const uint32_t pb1 = movm_t(clsB == 1 ? H::pack(ya, yb) : O::pack(ya, yb));
      const uint32_t n0 = clsA == 0 ? 0xFFFFFFFFu : 0u, n1 = clsB == 0 ? 0xFFFFFFFFu : 0u;
#pragma unroll
      for (int mb = 0; mb < KB; ++mb) {
        O::mma(o[mb], va[0][mb][0] & n0, va[0][mb][1] & n0, va[1][mb][0] & n1, va[1][mb][1] & n1,
               pb0 & n0, pb1 & n1);
        H::mma(o[mb], va[0][mb][0] & ~n0, va[0][mb][1] & ~n0, va[1][mb][0] & ~n1, va[1][mb][1] & ~n1,
               pb0 & ~n0, pb1 & ~n1);
      }
    }
    store_mass(pr0, pr1, i);
  };

  // ======================= int4 tiles (both units pages) =======================
  auto run_int4 = [&](int i0, int i1) {
    constexpr int SL = C::kI4Slots, SB = 2 * PB;
    auto issue = [&](int i, uint32_t dst) {  // chunk 32k + lane of each page
      const int2 pr = *reinterpret_cast<const int2*>(tbl + 2 * i);
      const unsigned char* pa = pages_l + (int64_t)pr.x * PB;
      const unsigned char* pb = pages_l + (int64_t)pr.y * PB;
#pragma unroll
      for (int k = 0; k < PG_IT; ++k)
        if (32 * k + 31 < PG_CH || lane + 32 * k < PG_CH) {
          cp_async16(dst + 512 * k, pa + 512 * k);
          cp_async16(dst + PB + 512 * k, pb + 512 * k);
        }
    };
    const uint32_t dst_l = ring_s + lane * 16;
#pragma unroll
    for (int k = 0; k < SL - 1; ++k) {
      if (i0 + k < i1) issue(i0 + k, dst_l + k * SB);
      cp_commit();
    }
    // R(-16) step for this thread's channels; (c, s, -s)
    float stc[KB / 2][4], sts[KB / 2][4], nst[KB / 2][4];
#pragma unroll
    for (int kb = 0; kb < KB / 2; ++kb)
#pragma unroll
      for (int eh = 0; eh < 2; ++eh) {  // channels d, d+1 as one 8-byte load
        const int d = 16 * kb + 2 * t + 8 * eh;
        const float2 c = can_step ? *reinterpret_cast<const float2*>(p.cos + kRotStep * (D / 2) + d)
                                  : make_float2(1.f, 1.f);
        const float2 sn = can_step ? *reinterpret_cast<const float2*>(p.sin + kRotStep * (D / 2) + d)
                                   : make_float2(0.f, 0.f);
        stc[kb][2 * eh] = c.x;
        stc[kb][2 * eh + 1] = c.y;
        sts[kb][2 * eh] = sn.x;
        sts[kb][2 * eh + 1] = sn.y;
        nst[kb][2 * eh] = -sn.x;
        nst[kb][2 * eh + 1] = -sn.y;
      }
    // query of this thread's column at the first tile
    {
      const int P = p.s + 8 * (u0 + 2 * i0 - R.NS + (g >> 2));
      if (P != rq_pos) seed(P, p.scale_log2, true);
    }
    uint32_t cs = ring_s, is = ring_s + (SL - 1) * SB;
#pragma unroll 2
    for (int i = i0; i < i1; ++i) {
      if (!can_step && i > i0) seed(p.s + 8 * (u0 + 2 * i - R.NS + (g >> 2)), p.scale_log2, true);
      if (i + SL - 1 < i1) issue(i + SL - 1, is + lane * 16);
      cp_commit();
      is = is + SB == ring_s + SL * SB ? ring_s : is + SB;
      uint32_t qB[KB][2];
#pragma unroll
      for (int kb = 0; kb < KB; ++kb) {
        qB[kb][0] = H::pack(rq[kb][0], rq[kb][1]);
        qB[kb][1] = H::pack(rq[kb][2], rq[kb][3]);
      }
      // advance the rotated query to this warp's next tile: R(-(P+16)) q
#pragma unroll
      for (int kb = 0; kb < KB / 2; ++kb)
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          float ys0, ys1, xs0, xs1;
          mul_x2(ys0, ys1, rq[kb + KB / 2][e], rq[kb + KB / 2][e + 1], sts[kb][e], sts[kb][e + 1]);
          mul_x2(xs0, xs1, rq[kb][e], rq[kb][e + 1], nst[kb][e], nst[kb][e + 1]);
          fma_x2(rq[kb][e], rq[kb][e + 1], rq[kb][e], rq[kb][e + 1], stc[kb][e], stc[kb][e + 1], ys0, ys1);
          fma_x2(rq[kb + KB / 2][e], rq[kb + KB / 2][e + 1], rq[kb + KB / 2][e], rq[kb + KB / 2][e + 1],
                 stc[kb][e], stc[kb][e + 1], xs0, xs1);
        }
      cp_wait<SL - 1>();
      __syncwarp();
      uint32_t ka[2][KB][2], va[2][KB][2];
      page_k_raw(cs, ka[0]);
      page_k_raw(cs + PB, ka[1]);
      // per group: acc = 2^-24 sum_d c q (the raw codes), qs = sum_d q (the
      // zero points' factor, from a constant A of ones, 16 on the columns
      // that meet the 1/16-scaled query elements); this thread's two scores
      // (row g of its unit, heads hh0, hh0 + 1) are the sums over groups of
      // s * 2^24 acc + z * qs, s and z of the token's group
      float acc[NW][4], qs[NW][4];
#pragma unroll
      for (int gq = 0; gq < NW; ++gq)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[gq][c] = qs[gq][c] = 0.f;
#pragma unroll
      for (int kb = 0; kb < KB; ++kb) {
        H::mma(acc[kb >> 1], ka[0][kb][0], ka[1][kb][0], ka[0][kb][1], ka[1][kb][1], qB[kb][0], qB[kb][1]);
        H::mma(qs[kb >> 1], 0x3C003C00u, 0x3C003C00u, 0x4C004C00u, 0x4C004C00u, qB[kb][0], qB[kb][1]);
      }
      const Words<NW> ksz = lds_words<NW>(cs + (my_unit ? PB : 0) + ks_off);
      page_v(cs, va[0]);
      page_v(cs + PB, va[1]);
      __syncwarp();
      cs = cs + SB == ring_s + SL * SB ? ring_s : cs + SB;
      float t0 = 0.f, t1 = 0.f, z0 = 0.f, z1 = 0.f;
#pragma unroll
      for (int gq = 0; gq < NW; ++gq) {
        const float2 sz = __half22float2(h2(ksz.w[gq]));
        t0 = fmaf(sz.x, my_unit ? acc[gq][2] : acc[gq][0], t0);
        t1 = fmaf(sz.x, my_unit ? acc[gq][3] : acc[gq][1], t1);
        z0 = fmaf(sz.y, qs[gq][0], z0);
        z1 = fmaf(sz.y, qs[gq][1], z1);
      }
      const float sc0 = fmaf(0x1p24f, t0, z0), sc1 = fmaf(0x1p24f, t1, z1);
      softmax_pv(sc0, sc1, false, va, 1, 1, 1, i);
    }
    rq_pos = can_step ? p.s + 8 * (u0 + 2 * i1 - R.NS + (g >> 2)) : -1;
  };

  // ======================= full fp tiles =======================
  auto run_fp = [&](int i0, int i1) {
    constexpr int SL = C::kFpSlots, SB = C::kTileBytes;
    uint32_t qb[KB][2];
    load_qb(qb);
    // chunk lane + 32j of a tile's 16 rows: rows advance 32/CPR per j, the
    // swizzle repeats every FP_PER chunks, the unit every 8 rows
    uint32_t fp_soff[FP_PER];
#pragma unroll
    for (int q = 0; q < FP_PER; ++q) {
      const int r = lane / C::kCPR + q * (32 / C::kCPR), c = lane % C::kCPR;
      fp_soff[q] = r * (2 * D) + ((c ^ r) * 16);
    }
    // ldmatrix: x4 matrices (unit, 8-channel chunk); offset of k-block kb is
    // base ^ (kb << 5) because the swizzle XORs the chunk index with the row
    const int lr = lane & 7;
    const uint32_t k_base = ((lane >> 3) & 1) * HS + lr * (2 * D) + ((((lane >> 4) ^ lr) & 1) * 16) + ((lr >> 1) << 5);
    const uint32_t v_base = (lane >> 4) * HS + 16 * D + lr * (2 * D) + (((((lane >> 3) & 1) ^ lr) & 1) * 16) + ((lr >> 1) << 5);
    // global source of chunk lane + 32j: rows of unit pair, 512 bytes per j
    const int64_t row0 = (int64_t)(p.s_pad + 8 * (u0 - R.TB)) * D;  // element offset of tile 0
    const unsigned char* kg = reinterpret_cast<const unsigned char*>(kfp + row0) + lane * 16;
    const unsigned char* vg = reinterpret_cast<const unsigned char*>(vfp + row0) + lane * 16;
    auto issue = [&](int i, uint32_t slot) {
      const int64_t off = (int64_t)i * 32 * D;  // 16 rows of D elements, in bytes
#pragma unroll
      for (int j = 0; j < FPJ; ++j) {
        const uint32_t d = slot + fp_soff[j % FP_PER] + (j / FP_PER) * HS;
        cp_async16(d, kg + off + 512 * j);
        cp_async16(d + 16 * D, vg + off + 512 * j);
      }
    };
#pragma unroll
    for (int k = 0; k < SL - 1; ++k) {
      if (i0 + k < i1) issue(i0 + k, ring_s + k * SB);
      cp_commit();
    }
    uint32_t cs = ring_s, is = ring_s + (SL - 1) * SB;
    for (int i = i0; i < i1; ++i) {
      if (i + SL - 1 < i1) issue(i + SL - 1, is);
      cp_commit();
      is = is + SB == ring_s + SL * SB ? ring_s : is + SB;
      cp_wait<SL - 1>();
      __syncwarp();
      uint32_t ka[2][KB][2], va[2][KB][2];
#pragma unroll
      for (int kb = 0; kb < KB; ++kb)
        ldsm_x4(ka[0][kb][0], ka[1][kb][0], ka[0][kb][1], ka[1][kb][1], cs + (k_base ^ (kb << 5)));
      float sacc[4] = {0.f, 0.f, 0.f, 0.f}, s2[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int kb = 0; kb < KB; ++kb)
        O::mma((kb & 1) ? s2 : sacc, ka[0][kb][0], ka[1][kb][0], ka[0][kb][1], ka[1][kb][1], qb[kb][0], qb[kb][1]);
#pragma unroll
      for (int mb = 0; mb < KB; ++mb)
        ldsm_x4_t(va[0][mb][0], va[0][mb][1], va[1][mb][0], va[1][mb][1], cs + (v_base ^ (mb << 5)));
      __syncwarp();
      cs = cs + SB == ring_s + SL * SB ? ring_s : cs + SB;
      const float sc0 = (my_unit ? sacc[2] + s2[2] : sacc[0] + s2[0]) * p.scale_log2;
      const float sc1 = (my_unit ? sacc[3] + s2[3] : sacc[1] + s2[1]) * p.scale_log2;
      softmax_pv(sc0, sc1, false, va, 2, 0, 0, i);
    }
  };

  // ======================= anything else (one tile at a time) =======================
  // sinks, region boundaries, partial or missing units
  auto issue_unit = [&](int u, uint32_t hs) {
    const int kd = R.kind(u);
    if (kd == 1) {
      const int64_t off = (int64_t)fp_slot0(p, R, u) * D;
#pragma unroll
      for (int j = 0; j < FP_IT; ++j) {  // chunk lane + 32j of the unit's 8 rows
        const int idx = lane + 32 * j, r = idx / C::kCPR, c = idx % C::kCPR;
        const uint32_t so = r * (2 * D) + ((c ^ (r & 7)) * 16);
        cp_async16(hs + so, kfp + off + r * D + c * 8);
        cp_async16(hs + 16 * D + so, vfp + off + r * D + c * 8);
      }
    } else if (kd == 2) {
      const unsigned char* pg = pages_l + (int64_t)tbl[u - u0] * PB;
#pragma unroll
      for (int j = 0; j < PG_IT; ++j)
        if (lane + 32 * j < PG_CH) cp_async16(hs + lane * 16 + 512 * j, pg + 512 * j);
    }
  };
  auto run_generic = [&](int i0, int i1) {
    uint32_t qb[KB][2];
    load_qb(qb);
    for (int i = i0; i < i1; ++i) {
      const int ua = u0 + 2 * i;
      issue_unit(ua, ring_s);
      issue_unit(ua + 1, ring_s + HS);
      cp_commit();
      const int kA = R.kind(ua), kB = R.kind(ua + 1);
      const int vA = kA == 2 ? 8 : (kA == 1 ? fp_valid(p, R, ua) : 0);
      const int vB = kB == 2 ? 8 : (kB == 1 ? fp_valid(p, R, ua + 1) : 0);
      // operand class per unit: 1 = fp16 (int4 page, or missing unit next to one)
      const int clsA = (kA == 2 || (kA == 0 && kB == 2)) ? 1 : 0;
      const int clsB = (kB == 2 || (kB == 0 && kA == 2)) ? 1 : 0;
      const bool uniform = !kBF || clsA == clsB;
      const bool use_h = kBF && clsA == 1;
      const int my_kind = (g >> 2) ? kB : kA;
      uint32_t qB[KB][2];
      if (my_kind == 2) {
        seed(p.s + 8 * ((ua + (g >> 2)) - R.NS), 1.f, false);
#pragma unroll
        for (int kb = 0; kb < KB; ++kb) {
          qB[kb][0] = H::pack(rq[kb][0], rq[kb][1]);
          qB[kb][1] = H::pack(rq[kb][2], rq[kb][3]);
        }
      } else {
#pragma unroll
        for (int kb = 0; kb < KB; ++kb) { qB[kb][0] = qb[kb][0]; qB[kb][1] = qb[kb][1]; }
      }
      cp_wait<0>();
      __syncwarp();
      uint32_t ka[2][KB][2], va[2][KB][2];
      auto k_fp_half = [&](int h) {
        const int r = lane & 7, sel = (lane >> 3) & 1;
        const uint32_t hb = ring_s + h * HS;
#pragma unroll
        for (int kb = 0; kb < KB; ++kb)
          ldsm_x2(ka[h][kb][0], ka[h][kb][1], hb + r * (2 * D) + (((2 * kb + sel) ^ r) * 16));
      };
      auto v_fp_half = [&](int h, int nv) {
        const int r = lane & 7, sel = (lane >> 3) & 1;
        const uint32_t msk = (2 * t < nv ? 0x0000FFFFu : 0u) | (2 * t + 1 < nv ? 0xFFFF0000u : 0u);
        const uint32_t hb = ring_s + h * HS;
#pragma unroll
        for (int mb = 0; mb < KB; ++mb) {
          ldsm_x2_t(va[h][mb][0], va[h][mb][1], hb + 16 * D + r * (2 * D) + (((2 * mb + sel) ^ r) * 16));
          va[h][mb][0] &= msk;
          va[h][mb][1] &= msk;
        }
      };
      if (kA == 2) { page_k(ring_s, ka[0]); page_v(ring_s, va[0]); } else { k_fp_half(0); v_fp_half(0, vA); }
      if (kB == 2) { page_k(ring_s + HS, ka[1]); page_v(ring_s + HS, va[1]); } else { k_fp_half(1); v_fp_half(1, vB); }
      float sacc[4] = {0.f, 0.f, 0.f, 0.f};
      if (uniform) {
#pragma unroll
        for (int kb = 0; kb < KB; ++kb) {
          if (use_h || !kBF && clsA == 1)
            H::mma(sacc, ka[0][kb][0], ka[1][kb][0], ka[0][kb][1], ka[1][kb][1], qB[kb][0], qB[kb][1]);
          else
            O::mma(sacc, ka[0][kb][0], ka[1][kb][0], ka[0][kb][1], ka[1][kb][1], qB[kb][0], qB[kb][1]);
        }
      } else {
        // tier boundary in a bf16 cache: one MMA per operand type, the other
        // unit's rows and the other columns' query zeroed
        const bool colF16 = ((g >> 2) ? clsB : clsA) == 1;
        const uint32_t n0 = clsA == 0 ? 0xFFFFFFFFu : 0u, n1 = clsB == 0 ? 0xFFFFFFFFu : 0u;
#pragma unroll
        for (int kb = 0; kb < KB; ++kb) {
          O::mma(sacc, ka[0][kb][0] & n0, ka[1][kb][0] & n1, ka[0][kb][1] & n0, ka[1][kb][1] & n1,
                 colF16 ? 0u : qB[kb][0], colF16 ? 0u : qB[kb][1]);
          H::mma(sacc, ka[0][kb][0] & ~n0, ka[1][kb][0] & ~n1, ka[0][kb][1] & ~n0, ka[1][kb][1] & ~n1,
                 colF16 ? qB[kb][0] : 0u, colF16 ? qB[kb][1] : 0u);
        }
      }
      __syncwarp();
      const bool v = g < (my_unit ? vB : vA);
      const float sc0 = v ? (my_unit ? sacc[2] : sacc[0]) * p.scale_log2 : -INFINITY;
      const float sc1 = v ? (my_unit ? sacc[3] : sacc[1]) * p.scale_log2 : -INFINITY;
      // P operand type: fp16 when the unit is an int4 page (any cache dtype)
      // or the cache is fp16; else bf16.  Uniform tiles use one MMA type.
      const int mode_pv = !uniform ? 0 : ((!kBF || clsA == 1) ? 1 : 2);
      softmax_pv(sc0, sc1, true, va, mode_pv, clsA, clsB, i);
    }
    rq_pos = -1;
  };

  // ---- this warp's run: generic | int4 | generic | fp | generic ----
  {
    const int a = max(tb, min(tr.ia, te)), bi = max(a, min(tr.ib, te));
    const int f = max(bi, min(tr.fa, te)), fe = max(f, min(tr.fb, te));
    if (tb < a) run_generic(tb, a);
    if (a < bi) run_int4(a, bi);
    if (bi < f) run_generic(bi, f);
    if (f < fe) run_fp(f, fe);
    if (fe < te) run_generic(fe, te);
  }
  cp_wait<0>();
  grid_launch_dependents();  // the merge kernel waits for this grid's completion itself

  // ---- warp epilogue: totals per head ----
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    float l = l_run[e];
#pragma unroll
    for (int off = 2; off < 32; off <<= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
    l_run[e] = l;
  }
#pragma unroll
  for (int mb = 0; mb < KB; ++mb)
#pragma unroll
    for (int c = 0; c < 4; ++c) o[mb][c] += __shfl_xor_sync(0xffffffffu, o[mb][c], 2);

  __syncthreads();  // rings are free: reuse them for the CTA merge
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
  float* s_M = wo + kWarps * 4 * D;                 // [4]
  float* s_fw = s_M + 4;                            // [kWarps][4]: exp2(warp max - CTA max)
  if (threadIdx.x < 4) {
    float M = -INFINITY;
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, wm[w * 4 + threadIdx.x]);
    s_M[threadIdx.x] = M;
    for (int w = 0; w < kWarps; ++w) {
      const float mw = wm[w * 4 + threadIdx.x];
      s_fw[w * 4 + threadIdx.x] = mw == -INFINITY ? 0.f : ex2(mw - M);
    }
  }
  __syncthreads();
  // CTA partial per head: O and sum relative to the CTA max, and the max
  for (int e = threadIdx.x; e < 4 * (D + 2); e += kThreads) {
    const int hh = e / (D + 2), c = e % (D + 2);
    float acc = 0.f;
    if (c == D) {
      acc = s_M[hh];
    } else {
#pragma unroll
      for (int w = 0; w < kWarps; ++w)
        acc += s_fw[w * 4 + hh] * (c == D + 1 ? wl[w * 4 + hh] : wo[(w * 4 + hh) * D + c]);
    }
    p.part[(((int64_t)b * p.Hv + kh) * p.n_split + split) * 4 * (D + 2) + e] = acc;
  }
  // window masses of the CTA's units, relative to the CTA max
  float* mrow = p.mass + ((int64_t)b * p.Hv * 4 + kh * 4) * p.W;
  for (int k = threadIdx.x; k < u1 - u0; k += kThreads) {
    const int u = u0 + k;
    if (u < R.NS) continue;
    const float* ms = mass_s + (k >> 1) * 12;
#pragma unroll
    for (int hh = 0; hh < 4; ++hh) {
      const float mt = ms[8 + hh];
      mrow[(int64_t)hh * p.W + (u - R.NS)] = (mt == -INFINITY) ? 0.f : ms[(k & 1) * 4 + hh] * ex2(mt - s_M[hh]);
    }
  }
}

// Combine the splits of one (row, head group) for its query heads.  Every
// block adds the normalised mass of a chunk of kMergeThreads windows (one
// window per thread, all four heads); blocks 0..3 also write the output of
// query head blockIdx.x, with the splits shared between kMergeThreads / D
// threads per channel.  It is launched as a programmatic dependent of the
// decode kernel: its blocks start while the decode's last blocks run, load
// the score accumulator (which the decode does not touch), then wait for
// the decode grid and issue every load of its partials, split statistics and
// masses at once (one memory round trip).
constexpr int kMergeThreads = 256;
constexpr int kMergeWindows = kMergeThreads;  // windows per block
constexpr int kMergeOutBlocks = 4;            // blocks that also write an output head

template <typename T, int D>
__global__ void __launch_bounds__(kMergeThreads) decode_mma_merge_kernel(const __grid_constant__ MmaParams p) {
  constexpr int kHalves = kMergeThreads / D;           // threads per output channel
  constexpr int kSpl = kMaxSplits / kHalves;           // splits per thread
  static_assert(kHalves >= 1 && kHalves * D == kMergeThreads, "merge threads");
  const int chunk = blockIdx.x, kh = blockIdx.y, b = blockIdx.z;  // kh: query-head group
  const int kr = kh / p.ngrp, hbase = kr * p.G + 4 * (kh - kr * p.ngrp);
  const int nlive = min(4, p.G - (hbase - kr * p.G));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ float s_f[4][kMaxSplits];   // split factor / L per head
  __shared__ int s_bnd[kMaxSplits + 1];
  __shared__ float s_o[kMergeThreads];
  float* acc = p.scores ? p.scores + ((int64_t)b * p.Hq + hbase) * p.scores_cap : nullptr;
  const int w0 = chunk * kMergeWindows * p.merge_per + threadIdx.x;
  float av[2][4];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int w = w0 + k * kMergeThreads;
    const bool has = acc != nullptr && k < p.merge_per && w < p.Ww;
#pragma unroll
    for (int hh = 0; hh < 4; ++hh) av[k][hh] = (has && hh < nlive) ? acc[(int64_t)hh * p.scores_cap + w] : 0.f;
  }
  for (int j = threadIdx.x; j <= p.n_split; j += kMergeThreads) s_bnd[j] = p.bnd[j];
  grid_dependency_wait();
  const float* part = p.part + ((int64_t)b * p.Hv + kh) * p.n_split * 4 * (D + 2);
  const float* ms = p.mass + ((int64_t)b * p.Hv * 4 + kh * 4) * p.W;
  // every load of this block, issued before any result is needed
  float mv[2][4];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int w = w0 + k * kMergeThreads;
    const bool has = acc != nullptr && k < p.merge_per && w < p.Ww && p.upw == 1;
#pragma unroll
    for (int hh = 0; hh < 4; ++hh) mv[k][hh] = has ? ms[(int64_t)hh * p.W + w] : 0.f;
  }
  const int oh = chunk;                                          // output head of this block
  const bool out_blk = oh < kMergeOutBlocks && oh < nlive;
  const int c = threadIdx.x % D, half = threadIdx.x / D;
  float ov[kSpl];
#pragma unroll
  for (int k = 0; k < kSpl; ++k) {
    const int sp = half * kSpl + k;
    ov[k] = (out_blk && sp < p.n_split) ? part[(sp * 4 + oh) * (D + 2) + c] : 0.f;
  }
  if (warp < 4) {  // warp hh: the split statistics of head hh
    const int hh = warp;
    float m2[2], l2[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int sp = lane + 32 * k;
      m2[k] = sp < p.n_split ? part[(sp * 4 + hh) * (D + 2) + D] : -INFINITY;
      l2[k] = sp < p.n_split ? part[(sp * 4 + hh) * (D + 2) + D + 1] : 0.f;
    }
    const float M = warp_max(fmaxf(m2[0], m2[1]));
    float f2[2], L = 0.f;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      f2[k] = m2[k] == -INFINITY ? 0.f : exp2f(m2[k] - M);
      L += f2[k] * l2[k];
    }
    const float invL = 1.f / warp_sum(L);
#pragma unroll
    for (int k = 0; k < 2; ++k)
      if (lane + 32 * k < p.n_split) s_f[hh][lane + 32 * k] = f2[k] * invL;
  }
  __syncthreads();
  if (out_blk) {
    float o = 0.f;
#pragma unroll
    for (int k = 0; k < kSpl; ++k) {
      const int sp = half * kSpl + k;
      o += s_f[oh][sp < p.n_split ? sp : 0] * ov[k];
    }
    if (kHalves > 1) {
      s_o[threadIdx.x] = o;
      __syncthreads();
      if (half == 0) {
#pragma unroll
        for (int h = 1; h < kHalves; ++h) o += s_o[threadIdx.x + h * D];
      }
    }
    if (half == 0) st_f32((T*)p.out + b * p.o_sb + (hbase + oh) * p.o_sh + c, o);
  }
  if (acc == nullptr) return;
  auto split_of = [&](int u) {  // last split with bnd <= u
    int lo = 0, hi = p.n_split - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_bnd[mid] <= u) lo = mid; else hi = mid - 1;
    }
    return lo;
  };
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int w = w0 + k * kMergeThreads;
    if (k >= p.merge_per || w >= p.Ww) break;
    if (p.upw == 1) {
      const int lo = split_of(p.NS + w);
#pragma unroll
      for (int hh = 0; hh < 4; ++hh)
        if (hh < nlive) acc[(int64_t)hh * p.scores_cap + w] = av[k][hh] + mv[k][hh] * s_f[hh][lo];
    } else {  // a window of several units, each normalised by its own split
      float sum[4] = {0.f, 0.f, 0.f, 0.f};
      for (int j = 0; j < p.upw && w * p.upw + j < p.W; ++j) {
        const int uo = w * p.upw + j, lo = split_of(p.NS + uo);
#pragma unroll
        for (int hh = 0; hh < 4; ++hh) sum[hh] += ms[(int64_t)hh * p.W + uo] * s_f[hh][lo];
      }
#pragma unroll
      for (int hh = 0; hh < 4; ++hh)
        if (hh < nlive) acc[(int64_t)hh * p.scores_cap + w] = av[k][hh] + sum[hh];
    }
  }
}

// Most splits a cache of U units can get (bounds the partials' workspace):
// at least one full tile per split, at most kMaxUnitsPerSplit units each.
int max_splits(int U) {
  const int n = max(max(1, U / 16), ceil_div(U, kMaxUnitsPerSplit));
  return n < kMaxSplits ? n : kMaxSplits;
}

template <int D>
void plan_splits(MmaParams& p) {
  // Ranges hold equal estimated cost (the per-tile costs of the kernel's
  // tile classes); the split count fills one or two whole waves of resident
  // CTAs.
  const int TB = p.NS + p.n_tp, UF = TB + p.rest / 8;
  auto clampi = [](int x, int lo, int hi) { return x < lo ? lo : (x > hi ? hi : x); };
  // cost of units [0, u), in half-tile units (2x the per-tile cost per pair)
  auto prefix = [&](int u) -> int64_t {
    return (int64_t)kCostGeneric * clampi(u, 0, p.NS) + (int64_t)kCostI4 * clampi(u - p.NS, 0, p.n_tp) +
           (int64_t)kCostFp * clampi(u - TB, 0, UF - TB) + (int64_t)kCostGeneric * max(0, u - UF);
  };
  const int units = p.B * p.Hv;
  const int slots = 148 * (D == 64 ? 4 : 2);
  // one wave of resident CTAs when its ranges fit kMaxUnitsPerSplit (small
  // batches: every CTA's fixed cost paid once), else two waves
  int n = max(1, slots / max(1, units));
  if (ceil_div(p.U, n) > kMaxUnitsPerSplit) n = max(1, (2 * slots) / max(1, units));
  n = max(n, ceil_div(p.U, kMaxUnitsPerSplit));
  n = min(n, kMaxSplits);
  n = min(n, max(1, p.U / 16));
  const int64_t total = prefix(p.U);
  p.bnd[0] = 0;
  int k = 1;
  while (p.bnd[k - 1] < p.U && k <= kMaxSplits) {
    const int64_t target = total * k / n;
    int lo = p.bnd[k - 1] + 1, hi = p.U;  // smallest u with prefix(u) >= target
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (prefix(mid) >= target) hi = mid; else lo = mid + 1;
    }
    int e = (lo + 1) & ~1;
    e = max(e, p.bnd[k - 1] + 2);
    e = min(e, p.bnd[k - 1] + kMaxUnitsPerSplit);
    p.bnd[k] = min(e, p.U);
    ++k;
  }
  p.n_split = k - 1;
  if (p.bnd[p.n_split] != p.U || p.n_split > max_splits(p.U)) {
    // caps left units over: fall back to equal unit counts
    n = max(ceil_div(p.U, kMaxUnitsPerSplit), min(n, kMaxSplits));
    const int per = (ceil_div(p.U, n) + 1) & ~1;
    p.n_split = ceil_div(p.U, per);
    for (int j = 0; j <= p.n_split; ++j) p.bnd[j] = min(p.U, j * per);
  }
}

template <typename T, int D>
int launch_mma(MmaParams& p, cudaStream_t stream) {
  using C = Cfg<D>;
  static_assert(C::kSmemBytes <= 227 * 1024, "smem");
  static std::atomic<uint32_t> smem_set{0};
  max_smem_once(smem_set, decode_mma_kernel<T, D>, (int)C::kSmemBytes);
  decode_mma_kernel<T, D><<<dim3(p.n_split, p.Hv, p.B), kThreads, C::kSmemBytes, stream>>>(p);
  SKV_CHECK_LAUNCH();
  cudaLaunchConfig_t cfg{};
  // two windows per thread when many (row, head group)s fill the GPU anyway
  p.merge_per = p.B * p.Hv >= 64 ? 2 : 1;
  cfg.gridDim = dim3(max(kMergeOutBlocks, p.scores ? ceil_div(p.Ww, kMergeWindows * p.merge_per) : 0), p.Hv, p.B);
  cfg.blockDim = dim3(kMergeThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, decode_mma_merge_kernel<T, D>, p);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return SKV_ERR_CUDA;
  }
  return SKV_OK;
}

struct MmaWs {
  size_t part, mass, total;
};
// query-head groups of up to 4 MMA columns: ceil(G / 4) per kv head
int head_groups(const skv_layer_desc* L) {
  const int G = L->num_q_heads / L->num_kv_heads;
  return L->num_kv_heads * ((G + 3) / 4);
}

MmaWs mma_ws(const skv_layer_desc* L, int T) {
  MmaWs w{};
  const int W = T > L->num_sink ? (T - L->num_sink + kPageTokens - 1) / kPageTokens : 0;  // units
  const int Hv = head_groups(L);
  const int NS = (min(T, L->num_sink) + kPageTokens - 1) / kPageTokens;
  w.part = align_up((size_t)L->batch * Hv * max_splits(W + NS) * 4 * (L->head_dim + 2) * 4, 256);
  w.mass = align_up((size_t)L->batch * Hv * 4 * (W > 0 ? W : 1) * 4, 256);
  w.total = w.part + w.mass;
  return w;
}

}  // namespace

bool decode_mma_supported(const skv_layer_desc* L) {
  const int G = L->num_q_heads / L->num_kv_heads;
  return (L->kv_dtype == SKV_F16 || L->kv_dtype == SKV_BF16) && (L->head_dim == 64 || L->head_dim == 128) &&
         G >= 1 && L->num_q_heads == G * L->num_kv_heads &&
         L->window_size % kPageTokens == 0 && L->fp_capacity % 8 == 0;
}

// Lengths the split plan covers: at least one full tile, at most
// kMaxSplits ranges of kMaxUnitsPerSplit units (the sink unit, a partial
// unit and the 8-token units in between).
bool decode_mma_length_ok(int T) { return T >= 16 && (int64_t)T / kPageTokens + 2 <= (int64_t)kMaxSplits * kMaxUnitsPerSplit; }

size_t decode_mma_ws_size(const skv_layer_desc* L, int T) { return mma_ws(L, T).total; }

int decode_mma(const skv_layer_desc* L, int T, int tier_pages, const void* q, int64_t q_sb, int64_t q_sh,
               void* out, int64_t o_sb, int64_t o_sh, float scaling, float* scores, int scores_cap, void* ws,
               cudaStream_t stream, const void* k_new, const void* v_new, int64_t kn_sb, int64_t kn_sh) {
  if ((q_sb % 2) || (q_sh % 2) || ((uintptr_t)q % 4)) return SKV_ERR_MISALIGNED;  // 32-bit query loads
  MmaParams p{};
  if (k_new != nullptr) {
    p.k_new = k_new;
    p.v_new = v_new;
    p.kn_sb = kn_sb;
    p.kn_sh = kn_sh;
    p.new_slot = Geometry{L->num_sink, L->sink_pad, L->window_size, T, tier_pages * kPageTokens}.fp_slot(T - 1);
  }
  const MmaWs w = mma_ws(L, T);
  p.k_fp = L->k_fp; p.v_fp = L->v_fp; p.pages = L->tier_pages; p.table = L->tier_table;
  p.cos = L->rope_cos; p.sin = L->rope_sin; p.q = q; p.out = out; p.scores = scores;
  p.part = (float*)ws;
  p.mass = (float*)((char*)ws + w.part);
  p.q_sb = q_sb; p.q_sh = q_sh; p.o_sb = o_sb; p.o_sh = o_sh;
  p.B = L->batch; p.Hkv = L->num_kv_heads; p.cap = L->fp_capacity; p.page_cap = L->tier_page_capacity;
  p.Hq = L->num_q_heads;
  p.G = p.Hq / p.Hkv;
  p.ngrp = (p.G + 3) / 4;
  p.Hv = p.Hkv * p.ngrp;
  p.scores_cap = scores_cap;
  p.s = L->num_sink; p.s_pad = L->sink_pad; p.n_tp = tier_pages;
  p.s_eff = T < p.s ? T : p.s;
  p.NS = ceil_div(p.s_eff, kPageTokens);
  p.rest = T > p.s ? T - p.s - tier_pages * kPageTokens : 0;
  p.U = p.NS + p.n_tp + ceil_div(p.rest, kPageTokens);
  p.W = T > p.s ? (T - p.s + kPageTokens - 1) / kPageTokens : 0;
  p.upw = L->window_size / kPageTokens;
  p.Ww = T > p.s ? (T - p.s + L->window_size - 1) / L->window_size : 0;
  p.scale_log2 = scaling * kLog2e;
  p.rope_rows = L->rope_positions;
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
