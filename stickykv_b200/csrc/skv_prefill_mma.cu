// Tensor-core prefill: causal attention of the prompt and its column mass
// (fp16/bf16, head_dim 64 or 128, any GQA ratio), both on the 5th-generation
// tensor cores (tcgen05, accumulators in tensor memory).
//
// Replaces the prefill branch of the flash score hook
// (modules/windowed_cache/hooks.py:245-290: chunked softmax(q·kᵀ) with a
// causal mask summed over the query rows, reduced to windows) together with
// the prompt's attention, in two passes:
//   1. forward (flash-attention style): each block owns 128 query rows of one
//      head and streams the 128-key tiles at or below the diagonal; S = Q Kᵀ
//      and O += P V are tcgen05 MMAs, the online softmax runs on the CUDA
//      cores between them; it writes the output and the row's log-sum-exp
//      (log2 domain).
//   2. column mass (the scoring contraction): each block owns 128 keys,
//      streams the 128-query tiles at or above the diagonal and sums
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

constexpr float kLog2eP = 1.4426950408889634f;

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
__device__ __forceinline__ void st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
      "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }
__device__ __forceinline__ void st1(uint32_t taddr, uint32_t v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};\n" ::"r"(taddr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld1(uint32_t taddr) {
  uint32_t v;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];\n" : "=r"(v) : "r"(taddr));
  return v;
}
// MN-major 128-byte-swizzled operand: rows of 64 MN elements (128 B), 8-row
// atoms of 1 KiB along K (stride byte offset), 64-element column blocks
// `lbo` bytes apart along MN (leading byte offset)
__device__ __forceinline__ uint64_t desc_sw128_mn(uint32_t addr, uint32_t lbo) {
  uint64_t d = (uint64_t)((addr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// 128 rows x D of a [T][D] matrix into K-major 128-byte-swizzled halves of 64
// channels (rows >= T zero-filled).
template <int D, int NT>
__device__ __forceinline__ void load_tile128(uint32_t dst, const void* src, int row0, int T) {
  constexpr int CPR = D / 8;                  // 16-byte chunks per row
  constexpr int HALF = kRows * 128;           // bytes of one 64-channel half
  const unsigned char* base = static_cast<const unsigned char*>(src);
  for (int idx = threadIdx.x; idx < kRows * CPR; idx += NT) {
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

constexpr int kCThreads = 256;  // scoring: two threads per key row

template <typename T, int D>
__global__ void __launch_bounds__(kCThreads) prefill_colmass_tc_kernel(const PrefillParams p) {
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
  const int quarter = warp & 3, half = warp >> 2;  // key rows 32*quarter.., query columns 64*half..
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
    load_tile128<D, kCThreads>(sQ + buf * TC::kTileBytes, qg, q0, p.T);
    if (threadIdx.x < kRows) {
      const int row = q0 + threadIdx.x;
      sL[buf * kRows + threadIdx.x] = row < p.T ? lse[row] : INFINITY;  // rows past the end weigh 0
    }
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

  load_tile128<D, kCThreads>(sK, kg, k0, p.T);
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
  float cs = 0.f;                                 // this thread's share of its key's column mass
  const int rl = 32 * quarter + lane;
  const int key = k0 + rl;                        // accumulator row (tensor-memory lane)
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
    const int c0 = 64 * half;
    const int qa = k0 + i * kRows + c0;           // first query of this thread's columns
    const float* lt = sL + (i & 1) * kRows + c0;
    const uint32_t tacc = tmem + ((uint32_t)(32 * quarter) << 16) + (i & 1) * kRows + c0;
    uint32_t r[64];
    ld32(*reinterpret_cast<uint32_t(*)[32]>(r), tacc);
    ld32(*reinterpret_cast<uint32_t(*)[32]>(r + 32), tacc + 32);
    ld_wait();
    if (i == 0) {  // diagonal tile: queries before the key do not see it
#pragma unroll
      for (int j = 0; j < 64; ++j) {
        const float x = ex2(fmaf(__uint_as_float(r[j]), sl2, -lt[j]));
        cs += qa + j < key ? 0.f : x;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 64; ++j) cs += ex2(fmaf(__uint_as_float(r[j]), sl2, -lt[j]));
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
  // the two halves of each key's column mass (sL is free now)
  if (half == 1) sL[rl] = cs;
  fence_before();
  __syncthreads();
  fence_after();
  if (half == 0 && key < p.T)
    p.colmass[((int64_t)b * p.Hq + h) * p.T + key] = lost ? __int_as_float(0x7fc00000) : cs + sL[rl];
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 256;\n" ::"r"(tmem));
}

// ---------------------------------------------------------------------------
// pass 1 on tcgen05: each block owns 128 query rows of one head.  Per 128-key
// tile at or below the diagonal:
//   S = Q K^T into tensor memory (M = 128 queries, N = 128 keys, K-major
//     operands);
//   two threads per query row (warps w and w + 4 share a lane quarter and
//     take key columns 0-63 and 64-127) read their half of the row once, after
//     which the next tile's QK MMA is issued; they exchange the half-row
//     maxima, keep an online softmax whose running max
//     moves only when the row max exceeds it by more than 8 (log2 domain; then
//     the row of O is rescaled in tensor memory), and write P (KV dtype) into
//     a K-major swizzled shared tile;
//   one thread issues O += P V into a second accumulator (B = the V tile,
//     MN-major: keys run down its 128-byte rows).
// K tiles are fetched two tiles ahead and V tiles one ahead (cp.async double
// buffers); the MMAs of the next tile run while the threads wait.  Waits are
// bounded: one that runs out poisons the block's output with NaN.
// ---------------------------------------------------------------------------
constexpr int kFThreads = 256;

template <int D> struct FwdTcCfg {
  static constexpr int kTileBytes = tc::kRows * D * 2;         // Q, K or V tile
  static constexpr int kPBytes = tc::kRows * tc::kRows * 2;   // P tile
  // head_dim 64: the two threads of a row exchange their half-row maxima and
  // sums through two free tensor-memory columns (192, 193), which keeps two
  // blocks on an SM; head_dim 128 (one block per SM) uses shared memory
  static constexpr bool kXchTmem = D == 64;
  static constexpr int kXchBytes = kXchTmem ? 0 : 2 * tc::kRows * 4;
  // Q, K x2, V x2, P, exchange, mbarriers + TMEM address (the dynamic shared
  // memory is 1 KiB aligned: declared so, and checked)
  static constexpr size_t kSmem = 5 * (size_t)kTileBytes + kPBytes + kXchBytes + 64;
};

template <typename T, int D>
__global__ void __launch_bounds__(kFThreads, D == 64 ? 2 : 1) prefill_fwd_tc_kernel(const PrefillParams p) {
  using namespace tc;
  using FC = FwdTcCfg<D>;
  using O = Op<T>;
  constexpr bool kBF = !std::is_same<T, __half>::value;
  constexpr uint32_t kIdescS = idesc_f16(kBF, kRows, kRows);
  constexpr uint32_t kIdescO = idesc_f16(kBF, kRows, D) | (1u << 16);  // B (V) MN-major
  constexpr int KS = D / 16;                  // QK steps over head_dim
  constexpr int KP = kRows / 16;              // PV steps over the key tile
  constexpr int HALF = kRows * 128;           // one 64-element column block of a tile
  constexpr uint32_t kOcol = kRows;           // O accumulator columns [128, 128 + D)
  constexpr int OC = D / 2;                   // O columns per thread
  constexpr float kThresh = 8.f;
  extern __shared__ __align__(1024) unsigned char smem_fwd[];
  unsigned char* smem = smem_fwd;
  const int qt = gridDim.x - 1 - blockIdx.x;  // longest rows first
  const int h = blockIdx.y, b = blockIdx.z;
  const int kh = h / (p.Hq / p.Hkv);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int quarter = warp & 3, half = warp >> 2;
  const int rl = 32 * quarter + lane;         // tile row (tensor-memory lane)
  const int q0 = qt * kRows;
  const int row = q0 + rl;                    // this thread's query
  const T* qg = (const T*)p.q + ((int64_t)b * p.Hq + h) * p.T * D;
  const T* kg = (const T*)p.k + ((int64_t)b * p.Hkv + kh) * p.T * D;
  const T* vg = (const T*)p.v + ((int64_t)b * p.Hkv + kh) * p.T * D;
  const uint32_t sQ = smem_u32(smem), sK = sQ + FC::kTileBytes, sV = sK + 2 * FC::kTileBytes;
  const uint32_t sP = sV + 2 * FC::kTileBytes;
  float* xch = reinterpret_cast<float*>(smem + 5 * FC::kTileBytes + FC::kPBytes);  // [2][128] (head_dim 128)
  const uint32_t bars = sP + FC::kPBytes + FC::kXchBytes;  // barS, barPV
  uint32_t* s_taddr = reinterpret_cast<uint32_t*>(smem + 5 * FC::kTileBytes + FC::kPBytes + FC::kXchBytes + 16);
  const float sl2 = p.scaling * kLog2eP;
  const int n_kt = qt + 1;  // key tiles at or below the diagonal

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 256;\n" ::"r"(smem_u32(s_taddr)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
  }
  if (threadIdx.x == 0) {
    bar_init(bars);
    bar_init(bars + 8);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  auto issue_s = [&](int j, uint32_t tmem) {  // S = Q K_j^T
    const uint32_t kb = sK + (j & 1) * FC::kTileBytes;
#pragma unroll
    for (int k = 0; k < KS; ++k) {
      const uint32_t off = (k >> 2) * HALF + (k & 3) * 32;
      mma_f16(tmem, desc_sw128(sQ + off), desc_sw128(kb + off), kIdescS, k > 0 ? 1u : 0u);
    }
    commit(bars);
  };
  auto issue_pv = [&](int j, uint32_t tmem) {  // O += P V_j
    const uint32_t vb = sV + (j & 1) * FC::kTileBytes;
#pragma unroll
    for (int k = 0; k < KP; ++k) {
      const uint32_t offp = (k >> 2) * HALF + (k & 3) * 32;
      mma_f16(tmem + kOcol, desc_sw128(sP + offp), desc_sw128_mn(vb + k * 16 * 128, HALF), kIdescO,
              (j > 0 || k > 0) ? 1u : 0u);
    }
    commit(bars + 8);
  };

  // cp.async groups: {Q, K_0}, {K_1}, {V_0}, then per tile j {K_j+2}, {V_j+1}
  load_tile128<D, kFThreads>(sQ, qg, q0, p.T);
  load_tile128<D, kFThreads>(sK, kg, 0, p.T);
  cp_commit();
  if (n_kt > 1) load_tile128<D, kFThreads>(sK + FC::kTileBytes, kg, kRows, p.T);
  cp_commit();
  load_tile128<D, kFThreads>(sV, vg, 0, p.T);
  cp_commit();
  cp_wait<2>();
  fence_proxy_async();
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *s_taddr;
  const uint32_t trow = tmem + ((uint32_t)(32 * quarter) << 16);  // this warp's lane quarter
  const uint32_t tS = trow + 64 * half, tO = trow + kOcol + OC * half;
  const uint32_t tX = trow + kOcol + D;  // exchange columns (head_dim 64)
  // half-row value exchange: publish before a block barrier, read after it
  auto xch_put = [&](float v) {
    if constexpr (FC::kXchTmem) {
      st1(tX + half, __float_as_uint(v));
      st_wait();
    } else {
      xch[half * kRows + rl] = v;
    }
  };
  auto xch_get = [&]() -> float {
    if constexpr (FC::kXchTmem) {
      const uint32_t v = ld1(tX + (half ^ 1));
      ld_wait();
      return __uint_as_float(v);
    } else {
      return xch[(half ^ 1) * kRows + rl];
    }
  };
  if (threadIdx.x == 0) issue_s(0, tmem);

  bool lost = (smem_u32(smem_fwd) & 1023) != 0;  // swizzled tiles need 1 KiB alignment
  float m_run = -INFINITY, m_thr = -INFINITY, l_run = 0.f;
  for (int j = 0; j < n_kt; ++j) {
    const int k0 = j * kRows + 64 * half;           // first key of this thread's columns
    const bool edge = j == qt || k0 + 64 > p.T;     // causal diagonal or sequence end
    if (!bar_wait(bars, j & 1)) lost = true;        // S_j in tensor memory
    fence_after();
    uint32_t r[64];
    ld32(*reinterpret_cast<uint32_t(*)[32]>(r), tS);
    ld32(*reinterpret_cast<uint32_t(*)[32]>(r + 32), tS + 32);
    if (j + 2 < n_kt) load_tile128<D, kFThreads>(sK + (j & 1) * FC::kTileBytes, kg, (j + 2) * kRows, p.T);
    cp_commit();
    ld_wait();
    // row max of the raw scores (scaling is monotone); keys past the causal
    // diagonal or the prompt become -inf, so they exponentiate to 0 below
    float mx = -INFINITY;
    if (edge) {
      const int lim = min(row + 1, p.T) - k0;  // keys k0 + i with i < lim are valid
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        if (i >= lim) r[i] = __float_as_uint(-INFINITY);
        mx = fmaxf(mx, __uint_as_float(r[i]));
      }
    } else {
#pragma unroll
      for (int i = 0; i < 64; ++i) mx = fmaxf(mx, __uint_as_float(r[i]));
    }
    mx *= sl2;
    xch_put(mx);
    // every thread has read S_j and K_{j+1} is resident: the next QK MMA
    // runs during the rest of this tile
    cp_wait<2>();
    fence_proxy_async();
    fence_before();
    __syncthreads();
    fence_after();
    if (threadIdx.x == 0 && j + 1 < n_kt) issue_s(j + 1, tmem);
    mx = fmaxf(mx, xch_get());
    // PV_{j-1} done: P, V_{j-1} and O are free
    if (j > 0 && !bar_wait(bars + 8, (j - 1) & 1)) lost = true;
    fence_after();
    if (j + 1 < n_kt) load_tile128<D, kFThreads>(sV + ((j + 1) & 1) * FC::kTileBytes, vg, (j + 1) * kRows, p.T);
    cp_commit();
    // lazy rescale: the running max moves only by more than kThresh
    const bool need = mx > m_thr;
    if (__any_sync(0xffffffffu, need)) {
      const float mn = need ? mx : m_run;
      const float alpha = !need ? 1.f : (m_run == -INFINITY ? 0.f : ex2(m_run - mn));
      l_run *= alpha;
      m_run = mn;
      m_thr = mn + kThresh;
      if (j > 0) {  // this thread's half of its O row
#pragma unroll 1
        for (int c0 = 0; c0 < OC; c0 += 32) {
          uint32_t o[32];
          ld32(o, tO + c0);
          ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          st32(tO + c0, o);
        }
        st_wait();
      }
    }
    // P = exp2(s - m) into this thread's half of the swizzled P row, row sum
    float rs = 0.f;
    const int r7 = rl & 7;
#pragma unroll
    for (int c = 0; c < 8; ++c) {  // 16-byte chunks of 8 keys
      uint32_t pk[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float x0 = ex2(fmaf(__uint_as_float(r[8 * c + 2 * e]), sl2, -m_run));
        const float x1 = ex2(fmaf(__uint_as_float(r[8 * c + 2 * e + 1]), sl2, -m_run));
        rs += x0 + x1;
        pk[e] = O::pack(x0, x1);
      }
      const uint32_t dst = sP + half * HALF + rl * 128 + ((c ^ r7) * 16);
      asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};\n" ::"r"(dst), "r"(pk[0]), "r"(pk[1]), "r"(pk[2]),
                   "r"(pk[3])
                   : "memory");
    }
    l_run += rs;
    // V_j resident, P complete
    cp_wait<2>();
    fence_proxy_async();
    fence_before();
    __syncthreads();
    fence_after();
    if (threadIdx.x == 0) issue_pv(j, tmem);
  }
  if (!bar_wait(bars + 8, (n_kt - 1) & 1)) lost = true;
  fence_after();
  xch_put(l_run);
  fence_before();
  __syncthreads();
  fence_after();
  const float l_row = l_run + xch_get();
  // O / l into this thread's half of the output row; log-sum-exp
  const float inv = lost ? __int_as_float(0x7fc00000) : 1.f / l_row;
  T* orow = (T*)p.out + (((int64_t)b * p.T + row) * p.Hq + h) * D + OC * half;
#pragma unroll 1
  for (int c0 = 0; c0 < OC; c0 += 32) {
    uint32_t o[32];
    ld32(o, tO + c0);
    ld_wait();
    if (row < p.T) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 v;
        v.x = O::pack(__uint_as_float(o[8 * q]) * inv, __uint_as_float(o[8 * q + 1]) * inv);
        v.y = O::pack(__uint_as_float(o[8 * q + 2]) * inv, __uint_as_float(o[8 * q + 3]) * inv);
        v.z = O::pack(__uint_as_float(o[8 * q + 4]) * inv, __uint_as_float(o[8 * q + 5]) * inv);
        v.w = O::pack(__uint_as_float(o[8 * q + 6]) * inv, __uint_as_float(o[8 * q + 7]) * inv);
        *reinterpret_cast<uint4*>(orow + c0 + 8 * q) = v;
      }
    }
  }
  if (row < p.T && half == 0)
    p.lse[((int64_t)b * p.Hq + h) * p.T + row] = lost ? __int_as_float(0x7fc00000) : m_run + __log2f(l_row);
  fence_before();
  __syncthreads();
  fence_after();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 256;\n" ::"r"(tmem));
}

template <typename T, int D>
int launch(const PrefillParams& p, bool colmass, cudaStream_t stream) {
  using FC = FwdTcCfg<D>;
  const dim3 grid((p.T + tc::kRows - 1) / tc::kRows, p.Hq, p.B);
  cudaFuncSetAttribute(prefill_fwd_tc_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)FC::kSmem);
  // the whole unified L1 as shared memory, so two head_dim-64 blocks fit an SM
  cudaFuncSetAttribute(prefill_fwd_tc_kernel<T, D>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  prefill_fwd_tc_kernel<T, D><<<grid, kFThreads, FC::kSmem, stream>>>(p);
  SKV_CHECK_LAUNCH();
  if (colmass) {
    using TC = tc::TcCfg<D>;
    cudaFuncSetAttribute(prefill_colmass_tc_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)TC::kSmem);
    const dim3 g2((p.T + tc::kRows - 1) / tc::kRows, p.Hq, p.B);
    prefill_colmass_tc_kernel<T, D><<<g2, kCThreads, TC::kSmem, stream>>>(p);
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
