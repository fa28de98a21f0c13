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
  int s, s_eff, s_pad, NS, n_tp, rest, U, W, rope_rows;
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
__device__ __forceinline__ void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ uint32_t movm_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;\n" : "=r"(y) : "r"(x));
  return y;
}

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

template <typename T, int D>
__global__ void __launch_bounds__(kThreads, D == 64 ? 4 : 2) decode_mma_kernel(const __grid_constant__ MmaParams p) {
  using C = Cfg<D>;
  using O = Op<T>;        // fp units: the KV dtype
  using H = Op<__half>;   // int4 pages: fp16 (their scale/zero are fp16)
  constexpr bool kBF = !std::is_same<T, __half>::value;
  constexpr int KB = C::kKB, NW = C::kNW;
  constexpr int FP_IT = 8 * C::kCPR / 32;                 // cp.async per lane per fp tensor
  constexpr int PG_CH = C::kPageBytes / 16;               // 16-byte chunks per page
  constexpr int PG_IT = (PG_CH + 31) / 32;
  constexpr float kThresh = 8.f;                          // lazy rescale margin (log2 domain)
  extern __shared__ __align__(128) unsigned char smem[];
  const int split = blockIdx.x, kh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int u0 = p.bnd[split], u1 = p.bnd[split + 1];
  const int n_tiles = (u1 - u0 + 1) >> 1;
  const Regions R{p.NS, p.NS + p.n_tp, p.U, u1};

  unsigned char* ring = smem + (size_t)warp * C::kStages * C::kStageBytes;
  float* mass_s = reinterpret_cast<float*>(smem + C::kRingBytes) + warp * kMaxTilesPerWarp * 12;
  int* tbl = reinterpret_cast<int*>(smem + C::kRingBytes + C::kMassBytes);

  const int j0 = max(0, u0 - p.NS), j1 = min(p.n_tp, max(0, u1 - p.NS));
  for (int j = j0 + threadIdx.x; j < j1; j += kThreads) tbl[j - j0] = p.table[(int64_t)b * p.page_cap + j];
  __syncthreads();

  // per-lane copy offsets (constant for the whole kernel)
  uint32_t fp_soff[FP_IT];
  int fp_goff[FP_IT];
#pragma unroll
  for (int j = 0; j < FP_IT; ++j) {
    const int idx = lane + 32 * j, r = idx / C::kCPR, c = idx % C::kCPR;
    fp_soff[j] = r * (2 * D) + ((c ^ (r & 7)) * 16);
    fp_goff[j] = r * D + c * 8;
  }
  const int64_t kv_row = ((int64_t)b * p.Hkv + kh) * p.cap * D;
  const int64_t pg_row = ((int64_t)b * p.Hkv + kh) * p.page_cap;
  const T* kfp = (const T*)p.k_fp + kv_row;
  const T* vfp = (const T*)p.v_fp + kv_row;

  auto issue_unit = [&](int u, unsigned char* half) {
    const int kd = R.kind(u);
    const uint32_t hs = smem_u32(half);
    if (kd == 1) {
      const int64_t off = (int64_t)fp_slot0(p, R, u) * D;
#pragma unroll
      for (int j = 0; j < FP_IT; ++j) {
        cp_async16(hs + fp_soff[j], kfp + off + fp_goff[j]);
        cp_async16(hs + 16 * D + fp_soff[j], vfp + off + fp_goff[j]);
      }
    } else if (kd == 2) {
      const uint8_t* pg = p.pages + (pg_row + tbl[u - p.NS - j0]) * C::kPageBytes;
#pragma unroll
      for (int j = 0; j < PG_IT; ++j) {
        const int idx = lane + 32 * j;
        if (idx < PG_CH) cp_async16(hs + idx * 16, pg + idx * 16);
      }
    }
  };

  // query of head (g & 3) in B-fragment order: d = 16kb + 2t + {0,1,8,9}
  const T* qp = (const T*)p.q + b * p.q_sb + (kh * 4 + (g & 3)) * p.q_sh;
  uint32_t qb[KB][2];
#pragma unroll
  for (int kb = 0; kb < KB; ++kb) {
    qb[kb][0] = *reinterpret_cast<const uint32_t*>(qp + 16 * kb + 2 * t);
    qb[kb][1] = *reinterpret_cast<const uint32_t*>(qp + 16 * kb + 2 * t + 8);
  }
  // query rotated to the page start of this thread's column, advanced by
  // R(-64) from one tile of the warp to its next (8 units = 64 positions on)
  float rq[KB][4];
  int rq_pos = -1;
  float stc[KB / 2][4], sts[KB / 2][4];
  const bool can_step = p.rope_rows > 64;
#pragma unroll
  for (int kb = 0; kb < KB / 2; ++kb)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int d = 16 * kb + 2 * t + (e & 1) + 8 * (e >> 1);
      stc[kb][e] = can_step ? p.cos[64 * (D / 2) + d] : 1.f;
      sts[kb][e] = can_step ? p.sin[64 * (D / 2) + d] : 0.f;
    }

  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  float o[KB][4];
#pragma unroll
  for (int mb = 0; mb < KB; ++mb) o[mb][0] = o[mb][1] = o[mb][2] = o[mb][3] = 0.f;

  const int my_tiles = n_tiles > warp ? (n_tiles - warp + kWarps - 1) / kWarps : 0;

  const int hh0 = 2 * (t & 1);
  const int my_unit = t >> 1;

  // One 16-token tile.  MODE 1: both units int4 pages; MODE 2: both units
  // full fp rows; MODE 0: anything else (sinks, region boundaries, partial
  // or missing units).  The common modes compile to straight-line code.
  auto tile = [&](auto mode_c, auto slots_c, int i, int ua, int kA, int kB, int vA, int vB,
                  const unsigned char* st) {
    constexpr int MODE = decltype(mode_c)::value;
    constexpr int SLOTS = decltype(slots_c)::value;
    constexpr bool I4 = MODE == 1, FP = MODE == 2;
    constexpr int HS = I4 ? C::kPageBytes : C::kHalfBytes;  // bytes between the two units of a slot
    const int clsA = I4 ? 1 : (FP ? 0 : ((kA == 2 || (kA == 0 && kB == 2)) ? 1 : 0));
    const int clsB = I4 ? 1 : (FP ? 0 : ((kB == 2 || (kB == 0 && kA == 2)) ? 1 : 0));
    const bool uniform = I4 || FP || !kBF || clsA == clsB;
    const bool use_h = kBF && clsA == 1;  // uniform tile in fp16 while T is bf16
    const int my_col_kind = I4 ? 2 : (FP ? 1 : ((g >> 2) ? kB : kA));

    // ---- query B fragments for this thread's column ----
    uint32_t qB[KB][2];
    if (my_col_kind == 2) {
      const int P = p.s + 8 * ((ua + (g >> 2)) - p.NS);
      if (P != rq_pos) {  // seed from the table (first tier tile of this warp)
#pragma unroll
        for (int kb = 0; kb < KB / 2; ++kb)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int d = 16 * kb + 2 * t + (e & 1) + 8 * (e >> 1);
            const float c = p.cos[(int64_t)P * (D / 2) + d], s = p.sin[(int64_t)P * (D / 2) + d];
            const float x = ld_f32(qp + d), y = ld_f32(qp + d + D / 2);
            rq[kb][e] = fmaf(x, c, y * s);
            rq[kb + KB / 2][e] = fmaf(y, c, -x * s);
          }
      }
#pragma unroll
      for (int kb = 0; kb < KB; ++kb) {
        qB[kb][0] = H::pack(rq[kb][0], rq[kb][1]);
        qB[kb][1] = H::pack(rq[kb][2], rq[kb][3]);
      }
      if (can_step) {  // advance to this warp's next tile: R(-(P+64)) q = R(-64) R(-P) q
#pragma unroll
        for (int kb = 0; kb < KB / 2; ++kb)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float x = rq[kb][e], y = rq[kb + KB / 2][e];
            rq[kb][e] = fmaf(x, stc[kb][e], y * sts[kb][e]);
            rq[kb + KB / 2][e] = fmaf(y, stc[kb][e], -x * sts[kb][e]);
          }
        rq_pos = P + 64;
      } else {
        rq_pos = -1;
      }
    } else {
#pragma unroll
      for (int kb = 0; kb < KB; ++kb) { qB[kb][0] = qb[kb][0]; qB[kb][1] = qb[kb][1]; }
    }

    cp_wait<SLOTS - 1>();
    __syncwarp();
    const uint32_t st_s = smem_u32(st);

    // ---- S = K q (16 tokens x 8 columns) ----
    float sacc[4] = {0.f, 0.f, 0.f, 0.f};
    {
      uint32_t ka[2][KB][2];  // [unit][kb][columns lo/hi]
      auto k_int4 = [&](int h) {
        const unsigned char* pg = st + h * HS;
        uint32_t w[NW], sz[NW];
#pragma unroll
        for (int e = 0; e < NW; ++e) {
          w[e] = reinterpret_cast<const uint32_t*>(pg)[(g * 4 + t) * NW + e];
          sz[e] = reinterpret_cast<const uint32_t*>(pg + page_k_scales_off(D))[g * NW + e];
        }
#pragma unroll
        for (int kb = 0; kb < KB; ++kb) {
          const uint32_t szw = sz[kb >> 1];
          const uint32_t s2 = __byte_perm(szw, szw, 0x1010), z2 = __byte_perm(szw, szw, 0x3232);
          ka[h][kb][0] = H::fma2(H::codes(w[kb >> 1], 2 * (kb & 1)), s2, z2);
          ka[h][kb][1] = H::fma2(H::codes(w[kb >> 1], 2 * (kb & 1) + 1), s2, z2);
        }
      };
      auto k_fp_half = [&](int h) {
        const int r = lane & 7, sel = (lane >> 3) & 1;
        const uint32_t hb = st_s + h * HS;
#pragma unroll
        for (int kb = 0; kb < KB; ++kb)
          ldsm_x2(ka[h][kb][0], ka[h][kb][1], hb + r * (2 * D) + (((2 * kb + sel) ^ r) * 16));
      };
      if constexpr (FP) {
        const int r = lane & 7, un = (lane >> 3) & 1, hi = lane >> 4;
        const uint32_t rb = st_s + un * HS + r * (2 * D);
#pragma unroll
        for (int kb = 0; kb < KB; ++kb)
          ldsm_x4(ka[0][kb][0], ka[1][kb][0], ka[0][kb][1], ka[1][kb][1], rb + (((2 * kb + hi) ^ r) * 16));
      } else if constexpr (I4) {
        k_int4(0);
        k_int4(1);
      } else {
        if (kA == 2) k_int4(0); else k_fp_half(0);
        if (kB == 2) k_int4(1); else k_fp_half(1);
      }
      if (uniform) {
        float s2[4] = {0.f, 0.f, 0.f, 0.f};  // second chain: halves the MMA dependency depth
#pragma unroll
        for (int kb = 0; kb < KB; ++kb) {
          float(&acc)[4] = (kb & 1) ? s2 : sacc;
          if (I4 || use_h)
            H::mma(acc, ka[0][kb][0], ka[1][kb][0], ka[0][kb][1], ka[1][kb][1], qB[kb][0], qB[kb][1]);
          else
            O::mma(acc, ka[0][kb][0], ka[1][kb][0], ka[0][kb][1], ka[1][kb][1], qB[kb][0], qB[kb][1]);
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) sacc[c] += s2[c];
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
    }

    // ---- V^T fragments (independent of P: built while the QK MMAs run) ----
    uint32_t va[2][KB][2];  // [unit][mb][d rows g / g+8]
      auto v_int4 = [&](int h) {
        const unsigned char* pg = st + h * HS;
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
      };
      auto v_fp_half = [&](int h, int nv) {
        const int r = lane & 7, sel = (lane >> 3) & 1;
        const uint32_t msk = (2 * t < nv ? 0x0000FFFFu : 0u) | (2 * t + 1 < nv ? 0xFFFF0000u : 0u);
        const uint32_t hb = st_s + h * HS;
#pragma unroll
        for (int mb = 0; mb < KB; ++mb) {
          ldsm_x2_t(va[h][mb][0], va[h][mb][1], hb + 16 * D + r * (2 * D) + (((2 * mb + sel) ^ r) * 16));
          va[h][mb][0] &= msk;
          va[h][mb][1] &= msk;
        }
      };
      if constexpr (FP) {
        const int r = lane & 7, sel = (lane >> 3) & 1, un = lane >> 4;
        const uint32_t rb = st_s + un * HS + 16 * D + r * (2 * D);
#pragma unroll
        for (int mb = 0; mb < KB; ++mb)
          ldsm_x4_t(va[0][mb][0], va[0][mb][1], va[1][mb][0], va[1][mb][1], rb + (((2 * mb + sel) ^ r) * 16));
      } else if constexpr (I4) {
        v_int4(0);
        v_int4(1);
      } else {
        if (kA == 2) v_int4(0); else v_fp_half(0, vA);
        if (kB == 2) v_int4(1); else v_fp_half(1, vB);
      }

    // ---- softmax (log2 domain), rescaling only when a score passes the
    //      running max by more than 2^kThresh ----
    const bool v = (I4 || FP) ? true : (g < (my_unit ? vB : vA));
    const float sc0 = v ? (my_unit ? sacc[2] : sacc[0]) * p.scale_log2 : -INFINITY;
    const float sc1 = v ? (my_unit ? sacc[3] : sacc[1]) * p.scale_log2 : -INFINITY;
    if (__any_sync(0xffffffffu, sc0 > m_run[0] + kThresh || sc1 > m_run[1] + kThresh)) {
      float mx0 = sc0, mx1 = sc1;
#pragma unroll
      for (int off = 2; off < 32; off <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
      }
      const float mn0 = fmaxf(m_run[0], mx0), mn1 = fmaxf(m_run[1], mx1);
      const float al0 = mn0 == -INFINITY ? 1.f : exp2f(m_run[0] - mn0);
      const float al1 = mn1 == -INFINITY ? 1.f : exp2f(m_run[1] - mn1);
      l_run[0] *= al0;
      l_run[1] *= al1;
#pragma unroll
      for (int mb = 0; mb < KB; ++mb) {
        o[mb][0] *= al0; o[mb][1] *= al1;
        o[mb][2] *= al0; o[mb][3] *= al1;
      }
      m_run[0] = mn0;
      m_run[1] = mn1;
    }
    const float pr0 = v ? exp2f(sc0 - m_run[0]) : 0.f;
    const float pr1 = v ? exp2f(sc1 - m_run[1]) : 0.f;
    l_run[0] += pr0;
    l_run[1] += pr1;
    // ---- O^T += V^T P ----
    const float xa = my_unit == 0 ? pr0 : 0.f, xb = my_unit == 0 ? pr1 : 0.f;
    const float ya = my_unit == 1 ? pr0 : 0.f, yb = my_unit == 1 ? pr1 : 0.f;
    const uint32_t pb0 = movm_t((I4 || (kBF && clsA == 1)) ? H::pack(xa, xb) : O::pack(xa, xb));
    const uint32_t pb1 = movm_t((I4 || (kBF && clsB == 1)) ? H::pack(ya, yb) : O::pack(ya, yb));
    {
      if (uniform) {
#pragma unroll
        for (int mb = 0; mb < KB; ++mb) {
          if (I4 || use_h)
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
    {  // window mass of each unit: sum over its 8 rows (exact fp32)
      float ms0 = pr0, ms1 = pr1;
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        ms0 += __shfl_xor_sync(0xffffffffu, ms0, off);
        ms1 += __shfl_xor_sync(0xffffffffu, ms1, off);
      }
      if (lane < 4) {
        float* ms = mass_s + i * 12;
        ms[my_unit * 4 + hh0] = ms0;
        ms[my_unit * 4 + hh0 + 1] = ms1;
        if (my_unit == 0) { ms[8 + hh0] = m_run[0]; ms[8 + hh0 + 1] = m_run[1]; }
      }
    }

    __syncwarp();
  };

  // A warp's tiles form a few homogeneous runs (sinks, int4 pages, fp rows,
  // boundaries).  Each run streams through the ring with its own geometry:
  // int4 tiles are small (two pages), so their runs keep many more tiles in
  // flight; the ring drains between runs.
  auto run_segment = [&](auto mode_c, auto slots_c, int i0, int i1) {
    constexpr int MODE = decltype(mode_c)::value;
    constexpr int SLOTS = decltype(slots_c)::value;
    constexpr int HS = MODE == 1 ? C::kPageBytes : C::kHalfBytes;
    constexpr int SLOT_BYTES = 2 * HS;
    static_assert(SLOTS * SLOT_BYTES <= C::kStages * C::kStageBytes, "ring");
#pragma unroll
    for (int k = 0; k < SLOTS - 1; ++k) {
      if (i0 + k < i1) {
        const int ua = u0 + 2 * (warp + kWarps * (i0 + k));
        unsigned char* sl = ring + k * SLOT_BYTES;
        issue_unit(ua, sl);
        issue_unit(ua + 1, sl + HS);
      }
      cp_commit();
    }
    int slot = 0, nslot = SLOTS - 1;
    for (int i = i0; i < i1; ++i) {
      if (i + SLOTS - 1 < i1) {
        const int ua_n = u0 + 2 * (warp + kWarps * (i + SLOTS - 1));
        unsigned char* sl = ring + nslot * SLOT_BYTES;
        issue_unit(ua_n, sl);
        issue_unit(ua_n + 1, sl + HS);
      }
      cp_commit();
      nslot = nslot + 1 == SLOTS ? 0 : nslot + 1;
      const int ua = u0 + 2 * (warp + kWarps * i);
      const int kA = MODE == 1 ? 2 : (MODE == 2 ? 1 : R.kind(ua));
      const int kB = MODE == 1 ? 2 : (MODE == 2 ? 1 : R.kind(ua + 1));
      const int vA = MODE != 0 ? 8 : (kA == 2 ? 8 : (kA == 1 ? fp_valid(p, R, ua) : 0));
      const int vB = MODE != 0 ? 8 : (kB == 2 ? 8 : (kB == 1 ? fp_valid(p, R, ua + 1) : 0));
      tile(mode_c, slots_c, i, ua, kA, kB, vA, vB, ring + slot * SLOT_BYTES);
      slot = slot + 1 == SLOTS ? 0 : slot + 1;
    }
  };
  auto tile_mode = [&](int i) -> int {
    const int ua = u0 + 2 * (warp + kWarps * i);
    const int kA = R.kind(ua), kB = R.kind(ua + 1);
    if (kA == 2 && kB == 2) return 1;
    if (kA == 1 && kB == 1 && fp_valid(p, R, ua) == 8 && fp_valid(p, R, ua + 1) == 8) return 2;
    return 0;
  };
  constexpr int kI4Slots = (int)(C::kStages * C::kStageBytes / (2 * C::kPageBytes)) < 8
                               ? (int)(C::kStages * C::kStageBytes / (2 * C::kPageBytes))
                               : 8;
  for (int i = 0; i < my_tiles;) {
    const int m = tile_mode(i);
    int j = i + 1;
    while (j < my_tiles && tile_mode(j) == m) ++j;
    if (m == 1)
      run_segment(std::integral_constant<int, 1>{}, std::integral_constant<int, kI4Slots>{}, i, j);
    else if (m == 2)
      run_segment(std::integral_constant<int, 2>{}, std::integral_constant<int, C::kStages>{}, i, j);
    else
      run_segment(std::integral_constant<int, 0>{}, std::integral_constant<int, C::kStages>{}, i, j);
    i = j;
  }
  cp_wait<0>();

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
    const int u = u0 + 2 * (warp + kWarps * i) + h;
    if (u >= u1 || u < p.NS) continue;
    const float mt = msw[i * 12 + 8 + hh];
    const float val = (mt == -INFINITY) ? 0.f : msw[i * 12 + h * 4 + hh] * exp2f(mt - s_M[hh]);
    p.mass[((int64_t)b * p.Hkv * 4 + kh * 4 + hh) * p.W + (u - p.NS)] = val;
  }
}

// Combine the splits of one (row, query head): blockIdx.x == 0 writes the
// output, every block adds the normalised mass of its window chunk.
constexpr int kMergeThreads = 128;
constexpr int kMergeWindows = 4 * kMergeThreads;  // windows per block

template <typename T, int D>
__global__ void __launch_bounds__(kMergeThreads) decode_mma_merge_kernel(const __grid_constant__ MmaParams p) {
  const int chunk = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int kh = h >> 2, hh = h & 3;
  const int Hq = p.Hkv * 4;
  __shared__ float s_f[kMaxSplits];
  __shared__ float s_invL;
  const float* part = p.part + ((int64_t)b * p.Hkv + kh) * p.n_split * 4 * (D + 2);
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    float ms[2], ls[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int s = lane + 32 * k;
      ms[k] = s < p.n_split ? part[(s * 4 + hh) * (D + 2) + D] : -INFINITY;
      ls[k] = s < p.n_split ? part[(s * 4 + hh) * (D + 2) + D + 1] : 0.f;
    }
    const float M = warp_max(fmaxf(ms[0], ms[1]));
    float L = 0.f;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const float f = ms[k] == -INFINITY ? 0.f : exp2f(ms[k] - M);
      if (lane + 32 * k < p.n_split) s_f[lane + 32 * k] = f;
      L += f * ls[k];
    }
    L = warp_sum(L);
    if (lane == 0) s_invL = 1.f / L;
  }
  __syncthreads();
  const float invL = s_invL;
  if (chunk == 0) {
    for (int c = threadIdx.x; c < D; c += blockDim.x) {
      float acc = 0.f;
      for (int s = 0; s < p.n_split; ++s) acc += s_f[s] * part[(s * 4 + hh) * (D + 2) + c];
      st_f32((T*)p.out + b * p.o_sb + h * p.o_sh + c, acc * invL);
    }
  }
  if (p.scores == nullptr) return;
  const float* __restrict__ ms = p.mass + ((int64_t)b * Hq + h) * p.W;
  float* __restrict__ acc = p.scores + ((int64_t)b * Hq + h) * p.scores_cap;
  const int w_end = min(p.W, (chunk + 1) * kMergeWindows);
  float mv[4], av[4];
  int ws[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {  // issue all loads first
    ws[k] = chunk * kMergeWindows + threadIdx.x + k * kMergeThreads;
    mv[k] = ws[k] < w_end ? ms[ws[k]] : 0.f;
    av[k] = ws[k] < w_end ? acc[ws[k]] : 0.f;
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    if (ws[k] >= w_end) continue;
    const int u = p.NS + ws[k];
    int sp = 0;
#pragma unroll 1
    for (int step = 32; step > 0; step >>= 1)  // last split with bnd <= u
      if (sp + step < p.n_split && p.bnd[sp + step] <= u) sp += step;
    acc[ws[k]] = av[k] + mv[k] * s_f[sp] * invL;
  }
}

template <int D>
void plan_splits(MmaParams& p) {
  // Every 16-token tile costs about the same time whether it holds fp or int4
  // units (the kernel is bound by per-tile latency, not bytes), so ranges
  // hold equal unit counts; the split count fills whole waves of resident CTAs.
  const int units = p.B * p.Hkv;
  const int slots = 148 * (D == 64 ? 4 : 2);
  int n = max(1, (2 * slots) / max(1, units));
  n = max(n, ceil_div(p.U, kMaxUnitsPerSplit));
  n = min(n, kMaxSplits);
  n = min(n, max(1, p.U / 16));
  int per = ceil_div(p.U, n);
  per = (per + 1) & ~1;
  p.bnd[0] = 0;
  int k = 1;
  while (p.bnd[k - 1] < p.U && k <= kMaxSplits) {
    p.bnd[k] = min(p.U, p.bnd[k - 1] + per);
    ++k;
  }
  p.n_split = k - 1;
}

template <typename T, int D>
int launch_mma(MmaParams& p, cudaStream_t stream) {
  using C = Cfg<D>;
  static_assert(C::kSmemBytes <= 227 * 1024, "smem");
  cudaFuncSetAttribute(decode_mma_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::kSmemBytes);
  dim3 grid(p.n_split, p.Hkv, p.B);
  decode_mma_kernel<T, D><<<grid, kThreads, C::kSmemBytes, stream>>>(p);
  SKV_CHECK_LAUNCH();
  const int chunks = p.scores ? max(1, ceil_div(p.W, kMergeWindows)) : 1;
  decode_mma_merge_kernel<T, D><<<dim3(chunks, p.Hkv * 4, p.B), kMergeThreads, 0, stream>>>(p);
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
