// Tensor-core prefill: causal attention of the prompt and its column mass
// (fp16/bf16, head_dim 64 or 128, any GQA ratio).
//
// Replaces the prefill branch of the flash score hook
// (modules/windowed_cache/hooks.py:245-290: chunked softmax(q·kᵀ) with a
// causal mask summed over the query rows, reduced to windows) together with
// the prompt's attention, in two passes:
//   1. forward (flash-attention style, mma.sync.m16n8k16): each block owns 64
//      query rows of one head, streams the 64-key tiles at or below the
//      diagonal through a cp.async double buffer and keeps an online softmax
//      per row; it writes the output and the row's log-sum-exp (log2 domain).
//      Tiles live in shared memory with the 16-byte chunk of row r stored at
//      chunk ^ (r & 7), which keeps every ldmatrix conflict-free.
//   2. column mass (the scoring contraction, tcgen05): each block owns 128
//      keys, streams the 128-query tiles at or above the diagonal and sums
//      exp2(s - lse) over the rows of each key column, S^T = K Q^T computed
//      into tensor memory.
// Both accumulate in fp32.  The window reduction of the column mass is the
// portable kernel's (skv_prefill.cu).
#include <float.h>

#include <type_traits>

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
// pass 2 on the 5th-generation tensor cores (tcgen05): S^T = K Q^T with
// M = 128 keys, N = 128 queries, K = head_dim in 16-element steps, fp32
// accumulators in tensor memory (two 128-column buffers: the MMA of the next
// query tile runs while the warps read and exponentiate the current one).
// Operands are K-major, 128-byte swizzled shared-memory tiles (8-row atoms of
// 1 KiB; head_dim 128 is stored as two 64-channel halves).  One thread issues
// the MMAs and commits them to an mbarrier; every thread owns one key row of
// the accumulator.  Waits are bounded: a wait that runs out poisons the
// block's column mass with NaN instead of hanging.
// ---------------------------------------------------------------------------
namespace tc {

constexpr int kRows = 128;  // keys per block (MMA M) = queries per tile (MMA N)
constexpr int kSpin = 1 << 24;

__device__ __forceinline__ uint64_t desc_sw128(uint32_t addr) {
  uint64_t d = (uint64_t)((addr & 0x3FFFFu) >> 4);  // start address
  d |= (uint64_t)1 << 16;                            // leading byte offset (16 B; unused when swizzled)
  d |= (uint64_t)(1024 >> 4) << 32;                  // stride byte offset: 8-row atoms of 1 KiB
  d |= (uint64_t)1 << 46;                            // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                            // 128-byte swizzle
  return d;
}
__host__ __device__ constexpr uint32_t idesc_f16(bool bf16, int M, int N) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) |  // f32 accumulate, A/B type
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);          // K-major A and B
}
__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n}\n" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(0u));
}
__device__ __forceinline__ void commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar)
               : "memory");
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }
__device__ __forceinline__ void bar_init(uint32_t bar) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(bar));
}
__device__ __forceinline__ bool bar_wait(uint32_t bar, uint32_t parity) {
  for (int it = 0; it < kSpin; ++it) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    if (ok) return true;
  }
  return false;
}
__device__ __forceinline__ void ld32(uint32_t (&r)[32], uint32_t taddr) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }

// 128 rows x D of a [T][D] matrix into K-major 128-byte-swizzled halves of 64
// channels (rows >= T zero-filled).
template <int D>
__device__ __forceinline__ void load_tile128(uint32_t dst, const void* src, int row0, int T) {
  constexpr int CPR = D / 8;                  // 16-byte chunks per row
  constexpr int HALF = kRows * 128;           // bytes of one 64-channel half
  const unsigned char* base = static_cast<const unsigned char*>(src);
  for (int idx = threadIdx.x; idx < kRows * CPR; idx += kPThreads) {
    const int r = idx / CPR, c = idx % CPR, row = row0 + r;
    const int h = c >> 3, cc = c & 7;
    const unsigned char* s = base + ((int64_t)min(row, T - 1) * D + c * 8) * 2;
    cp_async16_zfill(dst + h * HALF + r * 128 + ((cc ^ (r & 7)) * 16), s, row < T ? 16 : 0);
  }
}

template <int D> struct TcCfg {
  static constexpr int kTileBytes = kRows * D * 2;
  // K tile, two query tiles, two lse rows, two mbarriers + TMEM address; sized
  // so at most two blocks share an SM (2 x 256 TMEM columns)
  static constexpr size_t kUsed = 3 * (size_t)kTileBytes + 2 * kRows * 4 + 64 + 1024;  // + alignment slack
  static constexpr size_t kSmem = kUsed > 80 * 1024 ? kUsed : 80 * 1024;
};

}  // namespace tc

template <typename T, int D>
__global__ void __launch_bounds__(kPThreads) prefill_colmass_tc_kernel(const PrefillParams p) {
  using namespace tc;
  using TC = TcCfg<D>;
  constexpr bool kBF = !std::is_same<T, __half>::value;
  constexpr uint32_t kIdesc = idesc_f16(kBF, kRows, kRows);
  constexpr int KSTEPS = D / 16;
  extern __shared__ __align__(128) unsigned char smem_tc[];
  // swizzled operand tiles need 1 KiB alignment (the launch reserves the slack)
  unsigned char* smem = smem_tc + ((1024 - (smem_u32(smem_tc) & 1023)) & 1023);
  const int kt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int kh = h / (p.Hq / p.Hkv);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int k0 = kt * kRows;
  const T* qg = (const T*)p.q + ((int64_t)b * p.Hq + h) * p.T * D;
  const T* kg = (const T*)p.k + ((int64_t)b * p.Hkv + kh) * p.T * D;
  const float* lse = p.lse + ((int64_t)b * p.Hq + h) * p.T;
  const uint32_t sK = smem_u32(smem), sQ = sK + TC::kTileBytes;
  float* sL = reinterpret_cast<float*>(smem + 3 * TC::kTileBytes);       // [2][128]
  const uint32_t bars = smem_u32(smem + 3 * TC::kTileBytes + 2 * kRows * 4);  // 2 mbarriers
  uint32_t* s_taddr = reinterpret_cast<uint32_t*>(smem + 3 * TC::kTileBytes + 2 * kRows * 4 + 16);
  const float sl2 = p.scaling * kLog2eP;
  const int n_qt = (p.T - k0 + kRows - 1) / kRows;  // query tiles at or above the diagonal

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 256;\n" ::"r"(smem_u32(s_taddr)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
  }
  if (threadIdx.x == 0) {
    bar_init(bars);
    bar_init(bars + 8);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  auto load_q = [&](int i) {  // query tile i of this block into buffer i & 1
    const int q0 = k0 + i * kRows, buf = i & 1;
    load_tile128<D>(sQ + buf * TC::kTileBytes, qg, q0, p.T);
    const int row = q0 + threadIdx.x;  // kPThreads == kRows
    sL[buf * kRows + threadIdx.x] = row < p.T ? lse[row] : INFINITY;  // rows past the end weigh 0
  };
  auto issue = [&](int i, uint32_t tmem) {  // S^T tile i into accumulator buffer i & 1
    const uint32_t qb = sQ + (i & 1) * TC::kTileBytes;
#pragma unroll
    for (int k = 0; k < KSTEPS; ++k) {
      const uint32_t off = (k >> 2) * (kRows * 128) + (k & 3) * 32;  // 64-channel half, 32 B per step
      mma_f16(tmem + (i & 1) * kRows, desc_sw128(sK + off), desc_sw128(qb + off), kIdesc, k > 0 ? 1u : 0u);
    }
    commit(bars + 8 * (i & 1));
  };

  load_tile128<D>(sK, kg, k0, p.T);
  load_q(0);
  cp_commit();
  if (n_qt > 1) load_q(1);
  cp_commit();
  cp_wait<1>();
  fence_proxy_async();
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *s_taddr;
  if (threadIdx.x == 0) issue(0, tmem);

  bool lost = false;
  float cs = 0.f;                        // column mass of this thread's key
  const int key = k0 + 32 * warp + lane;  // accumulator row (tensor-memory lane)
  for (int i = 0; i < n_qt; ++i) {
    if (i + 1 < n_qt) {  // the next tile's MMA runs while this one is read
      cp_wait<0>();
      fence_proxy_async();
      fence_before();
      __syncthreads();
      fence_after();
      if (threadIdx.x == 0) issue(i + 1, tmem);
    }
    if (!bar_wait(bars + 8 * (i & 1), (i >> 1) & 1)) lost = true;
    fence_after();
    const int q0 = k0 + i * kRows;
    const float* lt = sL + (i & 1) * kRows;
    const uint32_t tacc = tmem + ((uint32_t)(32 * warp) << 16) + (i & 1) * kRows;
#pragma unroll 1
    for (int c0 = 0; c0 < kRows; c0 += 32) {
      uint32_t r[32];
      ld32(r, tacc + c0);
      ld_wait();
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int q = q0 + c0 + j;
        const float x = ex2(__uint_as_float(r[j]) * sl2 - lt[c0 + j]);
        cs += (i == 0 && q < key) ? 0.f : x;
      }
    }
    // every thread is done with accumulator i & 1 and query buffer i & 1
    fence_before();
    __syncthreads();
    fence_after();
    if (i + 2 < n_qt) {
      load_q(i + 2);
    }
    cp_commit();
  }
  if (key < p.T) p.colmass[((int64_t)b * p.Hq + h) * p.T + key] = lost ? __int_as_float(0x7fc00000) : cs;
  fence_before();
  __syncthreads();
  fence_after();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 256;\n" ::"r"(tmem));
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
    using TC = tc::TcCfg<D>;
    cudaFuncSetAttribute(prefill_colmass_tc_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)TC::kSmem);
    const dim3 g2((p.T + tc::kRows - 1) / tc::kRows, p.Hq, p.B);
    prefill_colmass_tc_kernel<T, D><<<g2, kPThreads, TC::kSmem, stream>>>(p);
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
