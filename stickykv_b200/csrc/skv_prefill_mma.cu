// Tensor-core prefill: causal attention of the prompt and its column mass
// (fp16/bf16, head_dim 64 or 128, any GQA ratio).
//
// Replaces the prefill branch of the flash score hook
// (modules/windowed_cache/hooks.py:245-290: chunked softmax(q·kᵀ) with a
// causal mask summed over the query rows, reduced to windows) together with
// the prompt's attention, in two passes over 64x64 tiles:
//   1. forward (flash-attention style): each block owns 64 query rows of one
//      head, streams the key/value tiles at or below the diagonal through a
//      cp.async double buffer and keeps an online softmax per row; it writes
//      the output and the row's log-sum-exp (log2 domain).
//   2. column mass: each block owns 64 keys, streams the query tiles at or
//      above the diagonal and sums exp2(s - lse) over the rows of each key
//      column (the same products as pass 1, transposed: S^T = K Q^T).
// Both passes are mma.sync.m16n8k16 with fp32 accumulation; tiles live in
// shared memory with the 16-byte chunk of row r stored at chunk ^ (r & 7),
// which keeps every ldmatrix conflict-free.  The window reduction of the
// column mass is the portable kernel's (skv_prefill.cu).
#include <float.h>

#include "skv_mma.cuh"

namespace skv {
namespace {

using namespace mma;

constexpr int kTile = 64;        // rows (queries or keys) per tile
constexpr int kPThreads = 128;   // 4 warps x 16 rows
constexpr float kLog2eP = 1.4426950408889634f;

template <int D> struct PCfg {
  static constexpr int kRowBytes = 2 * D;
  static constexpr int kTileBytes = kTile * kRowBytes;
  static constexpr int kCPR = D / 8;  // 16-byte chunks per row
  static constexpr int kKB = D / 16;  // k-blocks over head_dim
  static constexpr int kDN = D / 8;   // 8-channel blocks of the output
  static constexpr size_t kFwdSmem = 5 * (size_t)kTileBytes;              // Q, K x2, V x2
  static constexpr size_t kColSmem = 3 * (size_t)kTileBytes + 2 * kTile * 4;  // K, Q x2, lse x2
};

// 64 rows of a [T][D] matrix into a swizzled tile; rows >= T are zero-filled.
template <int D>
__device__ __forceinline__ void load_tile(uint32_t dst, const void* src, int row0, int T) {
  using C = PCfg<D>;
  const unsigned char* base = static_cast<const unsigned char*>(src);
  for (int idx = threadIdx.x; idx < kTile * C::kCPR; idx += kPThreads) {
    const int r = idx / C::kCPR, c = idx % C::kCPR, row = row0 + r;
    const unsigned char* s = base + ((int64_t)min(row, T - 1) * D + c * 8) * 2;
    cp_async16_zfill(dst + r * C::kRowBytes + ((c ^ (r & 7)) * 16), s, row < T ? 16 : 0);
  }
}

// A fragments (m16 x k16, row-major) of rows [r0, r0+16) of a swizzled tile
template <int D>
__device__ __forceinline__ void load_a(uint32_t (&a)[D / 16][4], uint32_t tile, int r0) {
  using C = PCfg<D>;
  const int lane = threadIdx.x & 31, m = lane >> 3;
  const int r = r0 + (m & 1) * 8 + (lane & 7);
#pragma unroll
  for (int kb = 0; kb < C::kKB; ++kb) {
    const int c = 2 * kb + (m >> 1);
    ldsm_x4(a[kb][0], a[kb][1], a[kb][2], a[kb][3], tile + r * C::kRowBytes + ((c ^ (r & 7)) * 16));
  }
}

// acc[nb] += A (16 x D) . B^T for the 64 rows of a swizzled tile used as the
// B operand (B[k = channel][n = tile row]), n-blocks of 8 rows
template <typename T, int D>
__device__ __forceinline__ void mma_rows(float (&acc)[8][4], const uint32_t (&a)[D / 16][4], uint32_t tile) {
  using C = PCfg<D>;
  using O = Op<T>;
  const int lane = threadIdx.x & 31, m = lane >> 3;
#pragma unroll
  for (int kb = 0; kb < C::kKB; ++kb)
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      const int r = (2 * np + (m >> 1)) * 8 + (lane & 7), c = 2 * kb + (m & 1);
      uint32_t b0, b1, b2, b3;
      ldsm_x4(b0, b1, b2, b3, tile + r * C::kRowBytes + ((c ^ (r & 7)) * 16));
      O::mma(acc[2 * np], a[kb][0], a[kb][1], a[kb][2], a[kb][3], b0, b1);
      O::mma(acc[2 * np + 1], a[kb][0], a[kb][1], a[kb][2], a[kb][3], b2, b3);
    }
}

// ---------------------------------------------------------------------------
// pass 1: output and log-sum-exp
// ---------------------------------------------------------------------------
template <typename T, int D>
__global__ void __launch_bounds__(kPThreads) prefill_fwd_kernel(const PrefillParams p) {
  using C = PCfg<D>;
  using O = Op<T>;
  constexpr int KB = C::kKB, DN = C::kDN;
  extern __shared__ __align__(128) unsigned char smem[];
  const int qt = gridDim.x - 1 - blockIdx.x;  // longest rows first
  const int h = blockIdx.y, b = blockIdx.z;
  const int kh = h / (p.Hq / p.Hkv);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int q0 = qt * kTile;
  const T* qg = (const T*)p.q + ((int64_t)b * p.Hq + h) * p.T * D;
  const T* kg = (const T*)p.k + ((int64_t)b * p.Hkv + kh) * p.T * D;
  const T* vg = (const T*)p.v + ((int64_t)b * p.Hkv + kh) * p.T * D;
  const uint32_t sQ = smem_u32(smem), sK = sQ + C::kTileBytes, sV = sK + 2 * C::kTileBytes;
  const float sl2 = p.scaling * kLog2eP;

  load_tile<D>(sQ, qg, q0, p.T);
  load_tile<D>(sK, kg, 0, p.T);
  load_tile<D>(sV, vg, 0, p.T);
  cp_commit();

  uint32_t qa[KB][4];
  float o[DN][4];
#pragma unroll
  for (int dn = 0; dn < DN; ++dn) o[dn][0] = o[dn][1] = o[dn][2] = o[dn][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  const int row_g = q0 + 16 * warp + g;  // query index of accumulator rows g and g+8
  const int n_kt = qt + 1;               // key tiles at or below the diagonal

  for (int kt = 0; kt < n_kt; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < n_kt) {
      load_tile<D>(sK + (buf ^ 1) * C::kTileBytes, kg, (kt + 1) * kTile, p.T);
      load_tile<D>(sV + (buf ^ 1) * C::kTileBytes, vg, (kt + 1) * kTile, p.T);
    }
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    if (kt == 0) load_a<D>(qa, sQ, 16 * warp);

    float s[8][4];
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) s[nb][0] = s[nb][1] = s[nb][2] = s[nb][3] = 0.f;
    mma_rows<T, D>(s, qa, sK + buf * C::kTileBytes);

    // scale into the log2 domain; causal and sequence-end masks
    const int k0 = kt * kTile;
    const bool edge = kt == qt || k0 + kTile > p.T;
#pragma unroll
    for (int nb = 0; nb < 8; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float x = s[nb][e] * sl2;
        if (edge) {
          const int key = k0 + nb * 8 + 2 * t + (e & 1), row = row_g + 8 * (e >> 1);
          if (key > row || key >= p.T) x = -INFINITY;
        }
        s[nb][e] = x;
      }
    // online softmax per row (rows g and g+8 of this warp)
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
      mx[0] = fmaxf(mx[0], fmaxf(s[nb][0], s[nb][1]));
      mx[1] = fmaxf(mx[1], fmaxf(s[nb][2], s[nb][3]));
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
    }
    float alpha[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const float mn = fmaxf(m_run[r], mx[r]);
      alpha[r] = mn == -INFINITY ? 1.f : ex2(m_run[r] - mn);
      m_run[r] = mn;
    }
    float rs[2] = {0.f, 0.f};
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
      s[nb][0] = m_run[0] == -INFINITY ? 0.f : ex2(s[nb][0] - m_run[0]);
      s[nb][1] = m_run[0] == -INFINITY ? 0.f : ex2(s[nb][1] - m_run[0]);
      s[nb][2] = m_run[1] == -INFINITY ? 0.f : ex2(s[nb][2] - m_run[1]);
      s[nb][3] = m_run[1] == -INFINITY ? 0.f : ex2(s[nb][3] - m_run[1]);
      rs[0] += s[nb][0] + s[nb][1];
      rs[1] += s[nb][2] + s[nb][3];
    }
    l_run[0] = l_run[0] * alpha[0] + rs[0];
    l_run[1] = l_run[1] * alpha[1] + rs[1];
#pragma unroll
    for (int dn = 0; dn < DN; ++dn) {
      o[dn][0] *= alpha[0]; o[dn][1] *= alpha[0];
      o[dn][2] *= alpha[1]; o[dn][3] *= alpha[1];
    }
    // O += P V: P's accumulator layout is the A layout of the next MMA
    const uint32_t vt = sV + buf * C::kTileBytes;
    const int m = lane >> 3;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t a0 = O::pack(s[2 * kk][0], s[2 * kk][1]);
      const uint32_t a1 = O::pack(s[2 * kk][2], s[2 * kk][3]);
      const uint32_t a2 = O::pack(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      const uint32_t a3 = O::pack(s[2 * kk + 1][2], s[2 * kk + 1][3]);
      const int r = 16 * kk + (m & 1) * 8 + (lane & 7);
#pragma unroll
      for (int dp = 0; dp < DN / 2; ++dp) {
        const int c = 2 * dp + (m >> 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(b0, b1, b2, b3, vt + r * C::kRowBytes + ((c ^ (r & 7)) * 16));
        O::mma(o[2 * dp], a0, a1, a2, a3, b0, b1);
        O::mma(o[2 * dp + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncthreads();  // the buffer just read is refilled next iteration
  }

  // finalise: totals over the 4 lanes of a row
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 1);
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 2);
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = row_g + 8 * r;
    if (row >= p.T) continue;
    const float inv = 1.f / l_run[r];
    T* orow = (T*)p.out + (((int64_t)b * p.T + row) * p.Hq + h) * D;
#pragma unroll
    for (int dn = 0; dn < DN; ++dn)
      *reinterpret_cast<uint32_t*>(orow + dn * 8 + 2 * t) = O::pack(o[dn][2 * r] * inv, o[dn][2 * r + 1] * inv);
    if (t == 0) p.lse[((int64_t)b * p.Hq + h) * p.T + row] = m_run[r] + __log2f(l_run[r]);
  }
}

// ---------------------------------------------------------------------------
// pass 2: column mass  colmass[j] = sum_{i >= j} exp2(s_ij - lse_i)
// ---------------------------------------------------------------------------
template <typename T, int D>
__global__ void __launch_bounds__(kPThreads) prefill_colmass_kernel(const PrefillParams p) {
  using C = PCfg<D>;
  constexpr int KB = C::kKB;
  extern __shared__ __align__(128) unsigned char smem[];
  const int kt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int kh = h / (p.Hq / p.Hkv);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int k0 = kt * kTile;
  const T* qg = (const T*)p.q + ((int64_t)b * p.Hq + h) * p.T * D;
  const T* kg = (const T*)p.k + ((int64_t)b * p.Hkv + kh) * p.T * D;
  const float* lse = p.lse + ((int64_t)b * p.Hq + h) * p.T;
  const uint32_t sK = smem_u32(smem), sQ = sK + C::kTileBytes;
  float* sL = reinterpret_cast<float*>(smem + 3 * C::kTileBytes);  // [2][64]
  const float sl2 = p.scaling * kLog2eP;
  const int n_qt = (p.T + kTile - 1) / kTile;

  auto load_lse = [&](int buf, int qt) {
    for (int i = threadIdx.x; i < kTile; i += kPThreads) {
      const int row = qt * kTile + i;
      sL[buf * kTile + i] = row < p.T ? lse[row] : INFINITY;  // rows past the end weigh 0
    }
  };
  load_tile<D>(sK, kg, k0, p.T);
  load_tile<D>(sQ, qg, k0, p.T);
  load_lse(0, kt);
  cp_commit();

  uint32_t ka[KB][4];
  float cs[2] = {0.f, 0.f};                // column sums of keys g and g+8 of this warp
  const int key_g = k0 + 16 * warp + g;
  for (int qt = kt; qt < n_qt; ++qt) {
    const int buf = (qt - kt) & 1;
    if (qt + 1 < n_qt) {
      load_tile<D>(sQ + (buf ^ 1) * C::kTileBytes, qg, (qt + 1) * kTile, p.T);
      load_lse(buf ^ 1, qt + 1);
    }
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    if (qt == kt) load_a<D>(ka, sK, 16 * warp);
    float s[8][4];
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) s[nb][0] = s[nb][1] = s[nb][2] = s[nb][3] = 0.f;
    mma_rows<T, D>(s, ka, sQ + buf * C::kTileBytes);
    const bool diag = qt == kt;
    const int qbase = qt * kTile;
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
      const float2 lq = *reinterpret_cast<const float2*>(sL + buf * kTile + nb * 8 + 2 * t);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qi = qbase + nb * 8 + 2 * t + (e & 1), key = key_g + 8 * (e >> 1);
        float x = ex2(s[nb][e] * sl2 - ((e & 1) ? lq.y : lq.x));
        if (diag && qi < key) x = 0.f;
        cs[e >> 1] += x;
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    cs[r] += __shfl_xor_sync(0xffffffffu, cs[r], 1);
    cs[r] += __shfl_xor_sync(0xffffffffu, cs[r], 2);
    const int key = key_g + 8 * r;
    if (t == 0 && key < p.T) p.colmass[((int64_t)b * p.Hq + h) * p.T + key] = cs[r];
  }
}

template <typename T, int D>
int launch(const PrefillParams& p, bool colmass, cudaStream_t stream) {
  using C = PCfg<D>;
  const int tiles = (p.T + kTile - 1) / kTile;
  const dim3 grid(tiles, p.Hq, p.B);
  cudaFuncSetAttribute(prefill_fwd_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::kFwdSmem);
  prefill_fwd_kernel<T, D><<<grid, kPThreads, C::kFwdSmem, stream>>>(p);
  SKV_CHECK_LAUNCH();
  if (colmass) {
    cudaFuncSetAttribute(prefill_colmass_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)C::kColSmem);
    prefill_colmass_kernel<T, D><<<grid, kPThreads, C::kColSmem, stream>>>(p);
    SKV_CHECK_LAUNCH();
  }
  return SKV_OK;
}

}  // namespace

bool prefill_mma_supported(const skv_layer_desc* L) {
  return (L->kv_dtype == SKV_F16 || L->kv_dtype == SKV_BF16) && (L->head_dim == 64 || L->head_dim == 128);
}

// Output, log-sum-exp (log2 domain) and, when colmass, the column mass of
// every prompt position; the caller reduces the column mass to windows.
int prefill_mma(const PrefillParams& p, int dtype, bool colmass, cudaStream_t stream) {
  if (dtype == SKV_F16)
    return p.D == 64 ? launch<__half, 64>(p, colmass, stream) : launch<__half, 128>(p, colmass, stream);
  return p.D == 64 ? launch<__nv_bfloat16, 64>(p, colmass, stream) : launch<__nv_bfloat16, 128>(p, colmass, stream);
}

}  // namespace skv
