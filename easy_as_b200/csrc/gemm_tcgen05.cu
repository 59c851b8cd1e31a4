// gemm_tcgen05.cu — native sm_100a tensor-core GEMMs for the `mk.dot` / `mk.mma` GEMM patterns.
//
// Computes the strided batched product the DSL expresses as one `mk.dot` per
// output element (reference dot lowering: easy_as eas/codegen/msl.py:920-952,
// an f32 `fma` chain over f16 inputs):
//
//   C[b][m][n] = sum_k A[b][m][k] * B[b][k][n]        f16 x f16 -> f32
//
//   A[b][m][k] at a + b*a_bstride + m*lda + k                    (K-major)
//   B[b][k][n] at b + b*b_bstride + k*ldb + n   (b_kmajor == 0, N-major)
//            or b + b*b_bstride + n*ldb + k     (b_kmajor == 1, K-major)
//   C[b][m][n] at c + b*c_bstride + m*ldc + n                    (f32)
//
// Design (one persistent CTA per SM, 6 warps):
//   warp 0      TMA producer: 128B-swizzled A (128 x 64) and B (BN x 64) tiles
//               into a STAGES-deep shared-memory ring, mbarrier complete_tx.
//   warp 1      allocates TMEM (2 x BN f32 columns: double-buffered
//               accumulators) and issues tcgen05.mma.cta_group::1.kind::f16
//               (M=128, N=BN, K=16) from one lane; tcgen05.commit frees ring
//               slots and publishes finished accumulators.
//   warps 2..5  epilogue: tcgen05.ld 32x32b rows of the accumulator, masked
//               f32 stores to C, then release the accumulator buffer.
// K, M and N tails are zero-filled by TMA (out-of-range box elements read 0),
// so they add nothing to the sums; stores are masked to m < M, n < N.
//
// CTA-pair kernel (gemm_f16_tcgen05_2sm_kernel, cluster of 2,
// tcgen05.mma.cta_group::2 with M = 256, N = 256): each CTA loads its half of A
// and of every 256-column B half; the pair tile is 256 x 256 with two TMEM
// accumulators (NH = 1), or 256 x 512 with one 512-column accumulator that the
// epilogue frees by halves (NH = 2, taken when it adds no tile rounds).  Split-K
// (launches that leave most pairs idle) sums K parts into a zeroed C with TMA
// reduce-adds.  The same kernels run kind::tf32 on f32 operands (TF = true),
// including the 3xTF32 mode, whose producer maps k-blocks onto [hi | lo] segments.
// No TMA load uses cluster multicast: every CTA loads only what it keeps.
//
// Every mbarrier wait is bounded (clock64 budget).  On expiry the kernel sets
// a shared abort flag, every role leaves its loop, TMEM is freed, and the
// code EAS_ERR_TIMEOUT is written to the host-mapped status word.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstdlib>
#include <mutex>

#include "eas_internal.h"

namespace {

constexpr int BM = 128;
constexpr int BK = 64;                       // one 128-byte swizzle row of f16
constexpr int kThreads = 192;                // 6 warps
constexpr long long kWaitBudget = 4000000000LL;  // cycles (~2 s) before a wait is declared hung
constexpr int kGroupM = 16;                  // tile-order swizzle for L2 reuse

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: false when the budget ran out or another role aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          long long budget = kWaitBudget) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > budget) {
      *abort_flag = 1;
      return false;
    }
  }
}

// Self-test of the expiry path: a barrier that nothing ever completes, waited on with `budget`.
__global__ void wait_selftest_kernel(long long budget, int* status) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (threadIdx.x == 0 && !mbar_wait(&bar, 0, &abort_flag, budget) && status) *status = EAS_ERR_TIMEOUT;
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
               : "memory");
}

// f32 add of a shared-memory box into global memory (split-K partial tiles); same bulk group as
// the stores, so the same waits cover it
__device__ __forceinline__ void tma_reduce_add_3d(const CUtensorMap* map, const void* src, int x, int y, int z) {
  asm volatile("cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
               : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

template <bool TF>
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  if constexpr (TF)
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
  else
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Shared-memory matrix descriptor (tcgen05), 128-byte swizzle:
//   [0,14) start address >> 4, [16,30) leading byte offset >> 4,
//   [32,46) stride byte offset >> 4, [46,48) version = 1,
//   [49,52) base offset = 0 (atoms are 1024-byte aligned), [61,64) layout = 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor, kind::f16 / kind::tf32: D = f32 (bits 4-5 = 1), A and B formats at bits
// 7-9 and 10-12 (f16 = 0, tf32 = 2), A K-major (bit 15 = 0), B major per b_mn (bit 16),
// N >> 3 at bits 17-22, M >> 4 at bits 24-28.
constexpr uint32_t kFmtTF32 = (2u << 7) | (2u << 10);
__host__ __device__ constexpr uint32_t instr_desc(int n, bool b_mn_major, bool tf32 = false) {
  return (1u << 4) | (tf32 ? kFmtTF32 : 0u) | ((b_mn_major ? 1u : 0u) << 16) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

struct TileCoord {
  int b, m0, n0;
};

struct Sched {
  int mt, nt, tiles_per_batch, total, group_m = kGroupM;
  __device__ TileCoord at(int t) const {
    TileCoord c;
    c.b = t / tiles_per_batch;
    int r = t - c.b * tiles_per_batch;
    const int per_group = group_m * nt;
    const int g = r / per_group;
    const int first_m = g * group_m;
    const int gsize = min(group_m, mt - first_m);
    const int rr = r - g * per_group;
    c.m0 = (first_m + rr % gsize) * BM;
    c.n0 = rr / gsize;  // tile index along N (times BN at the call site)
    return c;
  }
};

// KS k-blocks of 64 per pipeline stage (BLOCK_K = 64 KS): stage = KS A boxes then KS B boxes.
template <int BN, int STAGES, bool B_MN, int KS = 1>
struct Smem {
  static constexpr int kA1 = BM * BK * 2;  // one k-block of A
  static constexpr int kB1 = BN * BK * 2;  // one k-block of B
  static constexpr int kABytes = KS * kA1;
  static constexpr int kBBytes = KS * kB1;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kEpiOffset = STAGES * kStageBytes;       // 4 warps x 2 x 32x32 f32 staging boxes
  static constexpr int kEpiBytes = 4 * 2 * 32 * 32 * 4;
  static constexpr int kBarOffset = kEpiOffset + kEpiBytes;
  static constexpr int kTotal = kBarOffset + (2 * STAGES + 4) * 8 + 16 + 1024;  // + alignment slack
};

// 3xTF32 k-block map: A and B rows hold [hi | lo] segments of seg_kb k-blocks each; the GEMM runs
// over 3 seg_kb k-blocks: (A_hi, B_hi), then (A_hi, B_lo), then (A_lo, B_hi).
__device__ __forceinline__ void seg_coords(int kb, int seg_kb, int& ka, int& kbk) {
  const int seg = kb / seg_kb, kin = kb - seg * seg_kb;
  ka = ((seg == 2 ? seg_kb : 0) + kin) * 32;
  kbk = ((seg == 1 ? seg_kb : 0) + kin) * 32;
}

template <int BN, int STAGES, bool B_MN, bool TMA_C, bool TF = false, int KS = 1>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_f16_tcgen05_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                            const __grid_constant__ CUtensorMap map_c, float* __restrict__ c, int M, int N, int K,
                            int batch, long long ldc, long long c_bstride, int* status, int seg_kb, int ksplit) {
  static_assert(!(TF && B_MN), "tf32 operands are K-major here");
  static_assert(KS == 1 || (KS == 2 && !TF), "two k-blocks per stage are f16 only");
  constexpr int kBKe = TF ? 32 : BK;  // elements per 128-byte K row of a k-block
  using L = Smem<BN, STAGES, B_MN, KS>;
  // split-K as in the pair kernel: unit u is K part (u % ks) of tile (u / ks), summed into a zeroed C
  const int ks = TMA_C && ksplit > 1 ? ksplit : 1;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  constexpr uint32_t kTmemCols = 2 * BN;  // power of two: 256 or 512

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);  // one arrival per epilogue warp
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  Sched sched;
  sched.mt = (M + BM - 1) / BM;
  sched.nt = (N + BN - 1) / BN;
  sched.tiles_per_batch = sched.mt * sched.nt;
  sched.total = sched.tiles_per_batch * batch;
  const int kblocks = (K + kBKe - 1) / kBKe;
  const int kstages = (kblocks + KS - 1) / KS;  // pipeline stages per tile (the last may overhang K: zeros)
  const int units = sched.total * ks;
  auto k_range = [&](int u, int& kb0, int& kb1) {  // stage range of work unit u
    const int part = u % ks;
    kb0 = (int)((long long)part * kstages / ks);
    kb1 = (int)((long long)(part + 1) * kstages / ks);
  };

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x) {
        const TileCoord tc = sched.at(u / ks);
        const int n0 = tc.n0 * BN;
        int kb_lo, kb_hi;
        k_range(u, kb_lo, kb_hi);
        for (int kb = kb_lo; kb < kb_hi; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) break;
          mbar_expect_tx(&full[s], L::kStageBytes);
#pragma unroll
          for (int sub = 0; sub < KS; ++sub) {
            uint8_t* sa = smem + s * L::kStageBytes + sub * L::kA1;
            uint8_t* sb = smem + s * L::kStageBytes + L::kABytes + sub * L::kB1;
            const int kbs = kb * KS + sub;  // k-block (of 64 f16 / 32 tf32 elements)
            int ka = kbs * kBKe, kbk = ka;
            if (TF && seg_kb) seg_coords(kbs, seg_kb, ka, kbk);
            tma_load_3d(sa, &map_a, &full[s], ka, tc.m0, tc.b);
            if (B_MN) {
#pragma unroll
              for (int j = 0; j < BN / 64; ++j)
                tma_load_3d(sb + j * (BK * 128), &map_b, &full[s], n0 + 64 * j, kbs * BK, tc.b);
            } else {
              tma_load_3d(sb, &map_b, &full[s], kbk, n0, tc.b);
            }
          }
          if (++s == STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = instr_desc(BN, B_MN, TF);
      int s = 0;
      uint32_t ph = 0;
      int local = 0;
      for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x, ++local) {
        const int buf = local & 1;
        const uint32_t acc_ph = (local >> 1) & 1;
        if (!mbar_wait(&acc_empty[buf], acc_ph ^ 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        bool ok = true;
        int kb_lo, kb_hi;
        k_range(u, kb_lo, kb_hi);
        for (int kb = kb_lo; kb < kb_hi; ++kb) {
          if (!mbar_wait(&full[s], ph, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int sub = 0; sub < KS; ++sub) {
            const uint32_t a_addr = smem_u32(smem + s * L::kStageBytes + sub * L::kA1);
            const uint32_t b_addr = smem_u32(smem + s * L::kStageBytes + L::kABytes + sub * L::kB1);
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk) {
              const uint64_t adesc = smem_desc(a_addr + kk * 32, 16, 1024);
              const uint64_t bdesc = B_MN ? smem_desc(b_addr + kk * 2048, BK * 128, 1024)
                                          : smem_desc(b_addr + kk * 32, 16, 1024);
              tc_mma<TF>(d_tmem, adesc, bdesc, idesc, (kb != kb_lo || sub != 0 || kk != 0) ? 1u : 0u);
            }
          }
          tc_commit(&empty[s]);  // slot s is free once these MMAs have read it
          if (++s == STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
        tc_commit(&acc_full[buf]);  // accumulator complete
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const bool vec_ok = ((ldc & 3) == 0) && ((c_bstride & 3) == 0) && ((reinterpret_cast<uintptr_t>(c) & 15) == 0);
    // TMA_C: this warp's 32x32 f32 box, 128B-swizzled (16-byte chunk j of row r lives at chunk j ^ (r & 7))
    uint8_t* boxes = smem + L::kEpiOffset + q * (2 * 32 * 32 * 4);
    int nbox = 0;  // boxes issued by this warp so far; box nbox & 1 is the next to fill
    int local = 0;
    for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x, ++local) {
      const int buf = local & 1;
      const uint32_t acc_ph = (local >> 1) & 1;
      if (!mbar_wait(&acc_full[buf], acc_ph, abort_flag)) break;
      tc_fence_after();
      const TileCoord tc = sched.at(u / ks);
      const int n0 = tc.n0 * BN;
      const int m = tc.m0 + q * 32 + lane;
      float* crow = c + (long long)tc.b * c_bstride + (long long)m * ldc;
#pragma unroll 1
      for (int cc = 0; cc < BN / 32; ++cc) {
        uint32_t r[32];
        tmem_ld32(tmem_base + buf * BN + cc * 32 + ((uint32_t)(q * 32) << 16), r);
        const int nb = n0 + cc * 32;
        if (TMA_C) {
          if (nb < N && tc.m0 + q * 32 < M) {  // boxes wholly outside C are skipped; partial ones are clipped
            uint8_t* box = boxes + (nbox & 1) * (32 * 32 * 4);
            if (lane == 0) bulk_wait_read1();  // the store that last used this box has read it
            __syncwarp();
            uint8_t* row = box + lane * 128;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              float4 v = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                     __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
              *reinterpret_cast<float4*>(row + ((j ^ (lane & 7)) << 4)) = v;
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) {
              if (ks > 1)
                tma_reduce_add_3d(&map_c, box, nb, tc.m0 + q * 32, tc.b);
              else
                tma_store_3d(&map_c, box, nb, tc.m0 + q * 32, tc.b);
              bulk_commit();
            }
            ++nbox;
          }
        } else if (m < M) {
          if (vec_ok && nb + 32 <= N) {
            float4* dst = reinterpret_cast<float4*>(crow + nb);
#pragma unroll
            for (int j = 0; j < 8; ++j)
              dst[j] = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                   __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (nb + j < N) crow[nb + j] = __uint_as_float(r[j]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
    if (TMA_C && lane == 0) bulk_wait_all0();  // stores complete before the CTA's shared memory goes away
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols) : "memory");
  }
  if (threadIdx.x == 0 && *abort_flag && status) *status = EAS_ERR_TIMEOUT;
}

// ---------------------------------------------------------------------------
// 2-SM variant: a cluster of two CTAs computes a 256 x 256 tile with
// tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 16).  CTA rank r of the pair
// stages rows [128r, 128r+128) of the A tile and columns [128r, 128r+128) of
// the B tile, so each SM holds half of B; the leader (rank 0) issues the MMAs
// and its accumulators span both CTAs' TMEM (each CTA holds its 128 rows).
//   * both CTAs' TMA loads complete on the leader's `full` barrier, which the
//     leader alone arms with the pair's byte count (a CTA loads a slot only
//     after the leader's commit freed it, so the peer's bytes always land in
//     the phase the leader armed);
//   * the leader's commits arrive on `empty` / `acc_full` in both CTAs
//     (multicast commit, mask 0b11);
//   * all 8 epilogue warps of the pair arrive on the leader's `acc_empty`.
// No TMA multicast is used: every CTA loads only what it keeps.
// ---------------------------------------------------------------------------


__device__ __forceinline__ uint32_t mapa_rank(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ bool mbar_try_wait_cl(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_wait_cl(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait_cl(a, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait_cl(a, parity)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > kWaitBudget) {
      *abort_flag = 1;
      return false;
    }
  }
}

__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int x, int y,
                                                 int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, "
      "%5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

template <int kStages2, bool TMA_C, int NH = 1, int KS = 1>
struct Smem2 {
  static constexpr int kA1 = 128 * BK * 2;            // one k-block of this CTA's half of the A tile
  static constexpr int kB1 = NH * 128 * BK * 2;       // one k-block of its half of each 256-column B half
  static constexpr int kABytes = KS * kA1;
  static constexpr int kBBytes = KS * kB1;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kEpiOffset = kStages2 * kStageBytes;
  static constexpr int kEpiBytes = TMA_C ? 4 * 2 * 32 * 32 * 4 : 0;
  static constexpr int kBarOffset = kEpiOffset + kEpiBytes;
  static constexpr int kTotal = kBarOffset + (2 * kStages2 + 4) * 8 + 16 + 1024;
};

template <int kStages2, bool B_MN, bool TMA_C, bool TF = false, int NH = 1, int KS = 1>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_f16_tcgen05_2sm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                                const __grid_constant__ CUtensorMap map_c, float* __restrict__ c, int M, int N, int K,
                                int batch, long long ldc, long long c_bstride, int* status, int seg_kb,
                                int ksplit) {
  static_assert(!(TF && B_MN), "tf32 operands are K-major here");
  constexpr int kBKe = TF ? 32 : BK;  // elements per 128-byte K row of a stage
  // NH = 2: 256 x 512 pair tiles (two 256-column halves, one MMA each per k step) in ONE 512-column
  // accumulator, so the epilogue no longer overlaps the next tile's main loop, but each A tile
  // feeds twice the columns (25 % fewer operand bytes per FLOP from L2)
  static_assert(NH == 1 || NH == 2, "one or two 256-column halves per pair tile");
  static_assert(!(TF && NH == 2), "wide tiles are f16 only");
  static_assert(KS == 1 || (KS == 2 && !TF), "two k-blocks per stage are f16 only");
  using L = Smem2<kStages2, TMA_C, NH, KS>;
  // split-K: work unit u is K part (u % ks) of tile (u / ks); parts after the first are summed into
  // C (zeroed by the host) with TMA reduce-adds, so only the TMA-store epilogue splits
  const int ks = TMA_C && ksplit > 1 ? ksplit : 1;
  constexpr int BN = 256 * NH;       // columns of a pair tile
  constexpr int NBUF = NH == 1 ? 2 : 1;  // TMEM accumulators (512 columns in all)
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* empty = full + kStages2;
  uint64_t* acc_full = empty + kStages2;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  uint32_t rank;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
  constexpr uint32_t kTmemCols = 512;  // NBUF accumulators of 128 lanes x BN columns per CTA

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages2; ++s) {
      mbar_init(&full[s], 1);  // armed by the leader with both CTAs' bytes (leader's copy is used)
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 8);  // 4 epilogue warps x 2 CTAs (leader's copy is used)
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // peer barriers are initialised before anyone signals them
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  Sched sched;
  sched.mt = (M + 255) / 256;
  sched.nt = (N + BN - 1) / BN;
  sched.tiles_per_batch = sched.mt * sched.nt;
  sched.total = sched.tiles_per_batch * batch;
  const int kblocks = (K + kBKe - 1) / kBKe;
  const int kstages = (kblocks + KS - 1) / KS;  // pipeline stages per tile (the last may overhang K: zeros)
  const int cid = blockIdx.x >> 1;
  const int ncl = gridDim.x >> 1;
  const int units = sched.total * ks;
  auto k_range = [&](int u, int& kb0, int& kb1) {  // stage range of work unit u
    const int part = u % ks;
    kb0 = (int)((long long)part * kstages / ks);
    kb1 = (int)((long long)(part + 1) * kstages / ks);
  };

  if (warp == 0) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      for (int u = cid; u < units && !*abort_flag; u += ncl) {
        const TileCoord tc = sched.at(u / ks);  // m0 in units of 128: pair tiles are 256 rows
        const int m0 = (tc.m0 / BM) * 256 + 128 * (int)rank;
        const int n0 = tc.n0 * BN + 128 * (int)rank;
        int kb_lo, kb_hi;
        k_range(u, kb_lo, kb_hi);
        for (int kb = kb_lo; kb < kb_hi; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) break;
          const uint32_t fl = mapa_rank(smem_u32(&full[s]), 0);
          if (rank == 0) mbar_expect_tx(&full[s], 2 * L::kStageBytes);
#pragma unroll
          for (int sub = 0; sub < KS; ++sub) {
            uint8_t* sa = smem + s * L::kStageBytes + sub * L::kA1;
            uint8_t* sb = smem + s * L::kStageBytes + L::kABytes + sub * L::kB1;
            const int kbs = kb * KS + sub;  // k-block (of 64 f16 / 32 tf32 elements)
            int ka = kbs * kBKe, kbk = ka;
            if (TF && seg_kb) seg_coords(kbs, seg_kb, ka, kbk);
            tma_load_3d_pair(sa, &map_a, fl, ka, m0, tc.b);
#pragma unroll
            for (int h = 0; h < NH; ++h) {  // this CTA's 128 columns of each 256-column half
              uint8_t* sbh = sb + h * (128 * BK * 2);
              if (B_MN) {
                tma_load_3d_pair(sbh, &map_b, fl, n0 + 256 * h, kbs * BK, tc.b);
                tma_load_3d_pair(sbh + BK * 128, &map_b, fl, n0 + 256 * h + 64, kbs * BK, tc.b);
              } else {
                tma_load_3d_pair(sbh, &map_b, fl, kbk, n0 + 256 * h, tc.b);
              }
            }
          }
          if (++s == kStages2) {
            s = 0;
            ph ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = (1u << 4) | (TF ? kFmtTF32 : 0u) | ((B_MN ? 1u : 0u) << 16) | ((uint32_t)(256 >> 3) << 17) |
                                 ((uint32_t)(256 >> 4) << 24);
      int s = 0;
      uint32_t ph = 0;
      int local = 0;
      // MMAs of halves [h0, h1) of the stage in slot st at k-block kb
      auto issue = [&](int st, int kb, int kb_lo, uint32_t d_tmem, int h0, int h1) {
#pragma unroll
        for (int sub = 0; sub < KS; ++sub) {
        const uint32_t a_addr = smem_u32(smem + st * L::kStageBytes + sub * L::kA1);
        const uint32_t b_addr = smem_u32(smem + st * L::kStageBytes + L::kABytes + sub * L::kB1);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          const uint64_t adesc = smem_desc(a_addr + kk * 32, 16, 1024);
          const uint32_t acc = (kb != kb_lo || sub != 0 || kk != 0) ? 1u : 0u;
#pragma unroll
          for (int h = 0; h < NH; ++h) {  // one N = 256 MMA per half, into its 256 accumulator columns
            if (h < h0 || h >= h1) continue;
            const uint32_t bh = b_addr + h * (128 * BK * 2);
            const uint64_t bdesc = B_MN ? smem_desc(bh + kk * 2048, BK * 128, 1024) : smem_desc(bh + kk * 32, 16, 1024);
            const uint32_t dh = d_tmem + h * 256;
            if constexpr (TF)
              asm volatile(
                  "{\n\t.reg .pred p;\n\t"
                  "setp.ne.b32 p, %4, 0;\n\t"
                  "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(dh),
                  "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
                  : "memory");
            else
              asm volatile(
                  "{\n\t.reg .pred p;\n\t"
                  "setp.ne.b32 p, %4, 0;\n\t"
                  "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(dh),
                  "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
                  : "memory");
          }
        }
        }
      };
      auto release = [&](int st) {
        asm volatile(
            "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
                smem_u32(&empty[st])),
            "h"((uint16_t)3)
            : "memory");
      };
      auto advance = [&]() {
        if (++s == kStages2) {
          s = 0;
          ph ^= 1;
        }
      };
      for (int u = cid; u < units && !*abort_flag; u += ncl, ++local) {
        const int buf = NBUF == 2 ? (local & 1) : 0;
        const uint32_t acc_ph = NBUF == 2 ? (local >> 1) & 1 : local & 1;
        if (!mbar_wait_cl(&acc_empty[buf], acc_ph ^ 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        bool ok = true;
        int kb_lo, kb_hi;
        k_range(u, kb_lo, kb_hi);
        int kb = kb_lo;
        if constexpr (NH == 2) {
          // the epilogue frees the accumulator by halves (acc_empty[0]: columns 0-255, [1]: 256-511):
          // run half 0 of the first F k-blocks while the epilogue still drains half 1, holding
          // those stages (F <= the ring depth, so the producer never waits on a held stage), then
          // half 1 of the same stages once it is free
          const int F = kb_hi - kb_lo < kStages2 ? kb_hi - kb_lo : kStages2;
          const int s0 = s;
          const uint32_t ph0 = ph;
          for (int i = 0; i < F && ok; ++i) {
            if (!mbar_wait(&full[s], ph, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue(s, kb_lo + i, kb_lo, d_tmem, 0, 1);
            advance();
          }
          if (ok && !mbar_wait_cl(&acc_empty[1], acc_ph ^ 1, abort_flag)) ok = false;
          if (!ok) break;
          tc_fence_after();
          s = s0;
          ph = ph0;
          for (int i = 0; i < F; ++i) {
            issue(s, kb_lo + i, kb_lo, d_tmem, 1, 2);
            release(s);
            advance();
          }
          kb = kb_lo + F;
        }
        for (; kb < kb_hi; ++kb) {
          if (!mbar_wait(&full[s], ph, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue(s, kb, kb_lo, d_tmem, 0, NH);
          release(s);
          advance();
        }
        if (!ok) break;
        asm volatile(
            "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
                smem_u32(&acc_full[buf])),
            "h"((uint16_t)3)
            : "memory");
      }
    }
  } else {
    const int q = warp & 3;
    uint8_t* boxes = smem + L::kEpiOffset + q * (2 * 32 * 32 * 4);
    int nbox = 0;
    const bool vec_ok = ((ldc & 3) == 0) && ((c_bstride & 3) == 0) && ((reinterpret_cast<uintptr_t>(c) & 15) == 0);
    const uint32_t acc_empty_leader[2] = {mapa_rank(smem_u32(&acc_empty[0]), 0), mapa_rank(smem_u32(&acc_empty[1]), 0)};
    int local = 0;
    for (int u = cid; u < units && !*abort_flag; u += ncl, ++local) {
      const int buf = NBUF == 2 ? (local & 1) : 0;
      const uint32_t acc_ph = NBUF == 2 ? (local >> 1) & 1 : local & 1;
      if (!mbar_wait(&acc_full[buf], acc_ph, abort_flag)) break;
      tc_fence_after();
      const TileCoord tc = sched.at(u / ks);
      const int n0 = tc.n0 * BN;
      const int mrow0 = (tc.m0 / BM) * 256 + 128 * (int)rank + q * 32;
      const int m = mrow0 + lane;
      float* crow = c + (long long)tc.b * c_bstride + (long long)m * ldc;
      const uint32_t tbase = tmem_base + buf * BN + ((uint32_t)(q * 32) << 16);
      auto release_half0 = [&]() {  // columns 0-255 are in registers: half 0 is free
        tc_fence_before();
        __syncwarp();
        if (lane == 0)
          asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(acc_empty_leader[0])
                       : "memory");
      };
      auto put = [&](const uint32_t (&r)[32], int cc) {
        const int nb = n0 + cc * 32;
        if (TMA_C) {
          if (nb < N && mrow0 < M) {
            uint8_t* box = boxes + (nbox & 1) * (32 * 32 * 4);
            if (lane == 0) bulk_wait_read1();
            __syncwarp();
            uint8_t* row = box + lane * 128;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              float4 v = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                     __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
              *reinterpret_cast<float4*>(row + ((j ^ (lane & 7)) << 4)) = v;
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) {
              if (ks > 1)
                tma_reduce_add_3d(&map_c, box, nb, mrow0, tc.b);
              else
                tma_store_3d(&map_c, box, nb, mrow0, tc.b);
              bulk_commit();
            }
            ++nbox;
          }
        } else if (m < M) {
          if (vec_ok && nb + 32 <= N) {
            float4* dst = reinterpret_cast<float4*>(crow + nb);
#pragma unroll
            for (int j = 0; j < 8; ++j)
              dst[j] = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                   __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (nb + j < N) crow[nb + j] = __uint_as_float(r[j]);
          }
        }
      };
#pragma unroll 1
      for (int cc = 0; cc < BN / 32; ++cc) {
        uint32_t r[32];
        tmem_ld32(tbase + cc * 32, r);
        if (NH == 2 && cc == 256 / 32 - 1) release_half0();
        put(r, cc);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0)  // NH == 2: half 1 (barrier 1); otherwise the whole accumulator `buf`
        asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(
                         acc_empty_leader[NH == 2 ? 1 : buf])
                     : "memory");
    }
    if (TMA_C && lane == 0) bulk_wait_all0();
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the pair leaves together: no MMA still targets the peer's TMEM
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols)
                 : "memory");
  }
  if (threadIdx.x == 0 && *abort_flag && status) *status = EAS_ERR_TIMEOUT;
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

int encode_map(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t stride1_bytes,
               uint64_t stride2_bytes, uint32_t box0, uint32_t box1,
               CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT16) {
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  const cuuint32_t box[3] = {box0, box1, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_drv.tensorMapEncodeTiled(map, dt, 3, const_cast<void*>(base), dims,
                                          strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return eas_drv_check(r, "cuTensorMapEncodeTiled", EAS_ERR_VALUE);
}

// Tile configuration of the most recent GEMM launch in this process (reporting only).
struct LastConfig {
  int bm, bn, stages, ksplit, pair, block_k;
};
LastConfig g_last_config = {0, 0, 0, 0, 0, 0};

// The dynamic shared-memory opt-in is a per-function, per-device setting: make it once per kernel
// instantiation and device instead of on every launch.
template <auto Kern>
int set_smem_once(int bytes, const char* what) {
  static bool done[64] = {false};  // one flag array per kernel instantiation
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && done[dev]) return EAS_OK;
  int rc = eas_cuda_check(cudaFuncSetAttribute(Kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes), what,
                          EAS_ERR_LAUNCH);
  if (!rc && dev >= 0 && dev < 64) done[dev] = true;
  return rc;
}

// Split-K for launches that leave most CTAs (1-SM kernel) or CTA pairs idle: with at most half as
// many tiles as resident CTAs / pairs (`slots`), each tile's K range is cut into ks parts
// (ks <= slots / tiles, at least 8 k-blocks per part) and the parts are summed into a zeroed C with
// TMA reduce-adds.  Launches with a tile per slot or more do not split: zeroing C and summing
// partial tiles through L2 cost more than the last wave's idle pairs (measured on the per-GPU
// shards of C4 at 8 GPUs, 128 tiles on 74 pairs: 1109 TFLOP/s split 4 ways vs 1215 unsplit).
//
// Reproducibility: the reduce-adds of one tile land in any order.  With two parts every element
// is (0 + p) + q or (0 + q) + p, and both are exactly p + q (0 + x is x for every x, the sign of
// zero included, and f32 addition is commutative), so ks <= 2 gives the same bits on every run.
// Three or more parts would not (f32 addition is not associative), so the default cap is 2.
// EAS_GEMM_SPLITK=0 turns splitting off; EAS_GEMM_SPLITK=4 allows up to 4 parts, which is faster
// on very small grids but may differ from run to run in the last bits.
int splitk_cap() {
  static const int cap = [] {
    const char* e = getenv("EAS_GEMM_SPLITK");
    if (!e || !e[0]) return 2;
    const int v = atoi(e);
    return v <= 1 ? 1 : (v >= 4 ? 4 : v);
  }();
  return cap;
}

int choose_ksplit(long long tiles, long long slots, int kblocks, int batch) {
  const int cap = splitk_cap();
  if (cap <= 1 || slots <= 0 || tiles <= 0 || batch > 64 || 2 * tiles > slots) return 1;
  long long ks = slots / tiles;
  if (ks > cap) ks = cap;
  while (ks > 1 && kblocks < 8 * ks) --ks;
  return (int)ks;
}

// Zero C before a split launch: its K parts are summed into it.
int zero_c_for_split(float* c, int M, int N, int batch, long long ldc, long long cbs, cudaStream_t stream) {
  for (int b = 0; b < batch; ++b) {
    int rc = eas_cuda_check(cudaMemset2DAsync(c + (long long)b * cbs, (size_t)ldc * 4, 0, (size_t)N * 4, (size_t)M,
                                              stream),
                            "gemm: zero C for split-K", EAS_ERR_LAUNCH);
    if (rc) return rc;
  }
  return EAS_OK;
}

template <int BN, int STAGES, bool B_MN, bool TMA_C, bool TF = false, int KS = 1>
int launch_variant(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, float* c, int M, int N, int K,
                   int batch, long long ldc, long long cbs, int* status, cudaStream_t stream, int num_sms, int seg_kb = 0) {
  using L = Smem<BN, STAGES, B_MN, KS>;
  static_assert(L::kTotal <= 232448, "shared memory over the 227 KB per-CTA limit");
  auto kern = gemm_f16_tcgen05_kernel<BN, STAGES, B_MN, TMA_C, TF, KS>;
  int rc = set_smem_once<gemm_f16_tcgen05_kernel<BN, STAGES, B_MN, TMA_C, TF, KS>>(L::kTotal,
                                                                               "gemm: set smem attribute");
  if (rc) return rc;
  const long long tiles = (long long)((M + BM - 1) / BM) * ((N + BN - 1) / BN) * batch;
  const int ksplit = TMA_C ? choose_ksplit(tiles, num_sms, (K + (TF ? 32 : BK) - 1) / (TF ? 32 : BK), batch) : 1;
  if (ksplit > 1) {
    rc = zero_c_for_split(c, M, N, batch, ldc, cbs, stream);
    if (rc) return rc;
  }
  const long long units = tiles * ksplit;
  const int grid = (int)(units < num_sms ? units : num_sms);
  g_last_config = {BM, BN, STAGES, ksplit, 0, KS * BK};
  kern<<<grid, kThreads, L::kTotal, stream>>>(ma, mb, mc, c, M, N, K, batch, ldc, cbs, status, seg_kb, ksplit);
  return eas_cuda_check(cudaGetLastError(), "gemm: launch", EAS_ERR_LAUNCH);
}

template <int STAGES, bool B_MN, bool TMA_C, bool TF = false, int NH = 1, int KS = 1>
int launch_2sm(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, float* c, int M, int N, int K,
               int batch, long long ldc, long long cbs, int* status, cudaStream_t stream, int num_sms, int seg_kb = 0) {
  using L = Smem2<STAGES, TMA_C, NH, KS>;
  static_assert(L::kTotal <= 232448, "shared memory over the 227 KB per-CTA limit");
  auto kern = gemm_f16_tcgen05_2sm_kernel<STAGES, B_MN, TMA_C, TF, NH, KS>;
  int rc = set_smem_once<gemm_f16_tcgen05_2sm_kernel<STAGES, B_MN, TMA_C, TF, NH, KS>>(
      L::kTotal, "gemm(2sm): set smem attribute");
  if (rc) return rc;
  const long long tiles = (long long)((M + 255) / 256) * ((N + 256 * NH - 1) / (256 * NH)) * batch;
  // persistent grid: only as many pairs as can be resident at once (GPC boundaries can leave SMs unpaired)
  static int resident_pairs[64] = {0};  // one table per kernel instantiation
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (resident_pairs[dev] == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (num_sms / 2), 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = L::kTotal;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = num_sms / 2;
    }
    resident_pairs[dev] = n;
  }
  const long long pairs = resident_pairs[dev];
  const int ksplit = TMA_C ? choose_ksplit(tiles, pairs, (K + (TF ? 32 : BK) - 1) / (TF ? 32 : BK), batch) : 1;
  if (ksplit > 1) {  // the K parts are summed into C by TMA reduce-adds: start from zeros
    rc = zero_c_for_split(c, M, N, batch, ldc, cbs, stream);
    if (rc) return rc;
  }
  const long long units = tiles * ksplit;
  const int grid = 2 * (int)(units < pairs ? units : pairs);
  g_last_config = {256, 256 * NH, STAGES, ksplit, 1, KS * BK};
  kern<<<grid, kThreads, L::kTotal, stream>>>(ma, mb, mc, c, M, N, K, batch, ldc, cbs, status, seg_kb, ksplit);
  return eas_cuda_check(cudaGetLastError(), "gemm(2sm): launch", EAS_ERR_LAUNCH);
}

// 256 x 512 pair tiles read 25 % fewer operand bytes from L2 per FLOP than 256 x 256 ones but
// keep one accumulator (no epilogue overlap) and halve the tile count.  Taken when they need no
// more tile-rounds of work over the CTA pairs: 2 * ceil(wide tiles / pairs) <= ceil(tiles / pairs)
// (C4 8192^3: 512 wide tiles = 7 rounds vs 1024 = 14; M = N = 768: 6 wide tiles pay a half-empty
// column of tiles and lose).  The exposed part of a wide tile's epilogue is a fixed cost per
// tile, so short K loops lose with them: below 64 k-blocks (K < 4096) the 256 x 256 tiles with two
// accumulators win (C5, K = 2088: 3.60 ms against 4.42 ms wide, measured by the autotuner on one
// B200; C4, K = 8192: 0.736 ms wide against 0.786 ms).  EAS_GEMM_WIDE=0 / 1 forces the choice.
bool use_wide(uint32_t M, uint32_t N, uint32_t K, uint32_t batch, int num_sms) {
  static const int forced = [] {
    const char* e = getenv("EAS_GEMM_WIDE");
    return e && (e[0] == '0' || e[0] == '1') ? e[0] - '0' : -1;
  }();
  if (forced >= 0) return forced == 1;
  if (K < 64u * BK) return false;
  const long long pairs = num_sms / 2 > 0 ? num_sms / 2 : 1;
  const long long mt = (M + 255) / 256;
  const long long t1 = mt * ((N + 255) / 256) * batch, t2 = mt * ((N + 511) / 512) * batch;
  return 2 * ((t2 + pairs - 1) / pairs) <= (t1 + pairs - 1) / pairs;
}

bool use_2sm(int block_n, uint32_t M) {
  static const bool enabled = [] {
    const char* e = getenv("EAS_GEMM_2SM");
    return !(e && e[0] == '0');
  }();
  return enabled && block_n == 256 && M > 128;
}

// The f16 kernel a launch runs.  tile_m = 0 lets the library choose (CTA pair for block_n = 256
// and M > 128, wide pair tiles by use_wide, one k-block per stage); an explicit request is the
// autotune space of the DSL's BLOCK_M / BLOCK_N / BLOCK_K:
//   tile_m  128: the 1-SM kernel, tile 128 x block_n;
//           256: the CTA pair (M = 256 per MMA), each CTA staging block_n columns of B per
//                k-block, so the pair tile is 256 x 2 block_n (256 x 512 needs a TMA-storable C;
//                without one the pair tile stays 256 x 256);
//   block_k 64 or 128: K depth of one pipeline stage (one or two 64-wide k-blocks), with half as
//                many stages at 128 (same shared memory).
struct F16Choice {
  bool pair;
  int tile_n;  // columns of the (pair) tile
  int nh;      // pair only: 256-column halves per pair tile
  int ks;      // k-blocks per stage
  int stages;
};

F16Choice choose_f16(uint32_t M, uint32_t N, uint32_t K, uint32_t batch, int block_n, int tile_m, int block_k,
                     bool tma_c, int num_sms) {
  F16Choice ch{};
  ch.ks = block_k == 128 ? 2 : 1;
  ch.pair = tile_m == 0 ? use_2sm(block_n, M) : tile_m == 256;
  if (ch.pair) {
    const bool wide = tma_c && (tile_m == 0 ? (N >= 512 && use_wide(M, N, K, batch, num_sms)) : block_n == 256);
    ch.nh = wide ? 2 : 1;
    ch.tile_n = 256 * ch.nh;
    ch.stages = wide ? 4 / ch.ks : (tma_c ? 6 / ch.ks : (ch.ks == 1 ? 7 : 3));
  } else {
    ch.nh = 0;
    ch.tile_n = block_n;
    ch.stages = (block_n == 256 ? 4 : 6) / ch.ks;
  }
  return ch;
}

// Launch the kernel of `ch` (f16 operands).  Stage counts here and in choose_f16 agree.
template <int KS>
int launch_f16_choice(const F16Choice& ch, bool b_mn, bool tma_c, const CUtensorMap& ma, const CUtensorMap& mb,
                      const CUtensorMap& mc, float* c, int M, int N, int K, int batch, long long ldc, long long cbs,
                      int* status, cudaStream_t s, int num_sms) {
  constexpr int kS1w = 4 / KS, kS1 = 6 / KS, kS1d = KS == 1 ? 7 : 3;  // pair: wide, 256-wide, direct-store C
  constexpr int kSs256 = 4 / KS, kSs128 = 6 / KS;                    // 1-SM: BN = 256, 128
#define EAS_ARGS ma, mb, mc, c, M, N, K, batch, ldc, cbs, status, s, num_sms
  if (ch.pair) {
    if (ch.nh == 2)  // TMA-storable C only
      return b_mn ? launch_2sm<kS1w, true, true, false, 2, KS>(EAS_ARGS)
                  : launch_2sm<kS1w, false, true, false, 2, KS>(EAS_ARGS);
    if (!tma_c)
      return b_mn ? launch_2sm<kS1d, true, false, false, 1, KS>(EAS_ARGS)
                  : launch_2sm<kS1d, false, false, false, 1, KS>(EAS_ARGS);
    return b_mn ? launch_2sm<kS1, true, true, false, 1, KS>(EAS_ARGS)
                : launch_2sm<kS1, false, true, false, 1, KS>(EAS_ARGS);
  }
  if (ch.tile_n == 256)
    return b_mn ? (tma_c ? launch_variant<256, kSs256, true, true, false, KS>(EAS_ARGS)
                         : launch_variant<256, kSs256, true, false, false, KS>(EAS_ARGS))
                : (tma_c ? launch_variant<256, kSs256, false, true, false, KS>(EAS_ARGS)
                         : launch_variant<256, kSs256, false, false, false, KS>(EAS_ARGS));
  return b_mn ? (tma_c ? launch_variant<128, kSs128, true, true, false, KS>(EAS_ARGS)
                       : launch_variant<128, kSs128, true, false, false, KS>(EAS_ARGS))
              : (tma_c ? launch_variant<128, kSs128, false, true, false, KS>(EAS_ARGS)
                       : launch_variant<128, kSs128, false, false, false, KS>(EAS_ARGS));
#undef EAS_ARGS
}

int* g_status_host = nullptr;  // host-mapped status words, one per device
int* g_status_dev = nullptr;
std::once_flag g_status_once;

}  // namespace

int* eas_native_status_dev(int dev) {
  std::call_once(g_status_once, [] {
    void* h = nullptr;
    if (cudaHostAlloc(&h, 64 * sizeof(int), cudaHostAllocMapped | cudaHostAllocPortable) == cudaSuccess) {
      g_status_host = static_cast<int*>(h);
      for (int i = 0; i < 64; ++i) g_status_host[i] = 0;
      void* d = nullptr;
      if (cudaHostGetDevicePointer(&d, h, 0) == cudaSuccess) g_status_dev = static_cast<int*>(d);
    }
    cudaGetLastError();
  });
  return (g_status_dev && dev >= 0 && dev < 64) ? g_status_dev + dev : nullptr;
}

extern "C" int eas_gemm_status(int dev, int* code) {
  if (!code) return eas_fail(EAS_ERR_VALUE, "eas_gemm_status: null pointer");
  *code = (g_status_host && dev >= 0 && dev < 64) ? g_status_host[dev] : 0;
  if (g_status_host && dev >= 0 && dev < 64) g_status_host[dev] = 0;
  return EAS_OK;
}

extern "C" int eas_wait_selftest(long long budget_cycles, void* stream) {
  if (budget_cycles <= 0 || budget_cycles > kWaitBudget)
    return eas_fail(EAS_ERR_VALUE, "eas_wait_selftest: budget must be in (0, %lld] cycles", kWaitBudget);
  int dev = 0;
  cudaGetDevice(&dev);
  int* status = eas_native_status_dev(dev);
  if (!status) return eas_fail(EAS_ERR_MEMORY, "eas_wait_selftest: no status word");
  wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(budget_cycles, status);
  return eas_cuda_check(cudaGetLastError(), "wait_selftest launch", EAS_ERR_LAUNCH);
}

namespace {

// Host side shared by the f16 and tf32 entries: TMA maps over 2- or 4-byte operands with 128-byte
// K rows (64 f16 or 32 tf32 elements), then the 1-SM or CTA-pair kernel.
template <bool TF>
int gemm_entry(const char* who, const void* a, const void* b, float* c, uint32_t M, uint32_t N, uint32_t K,
               uint32_t batch, uint64_t lda, uint64_t a_bstride, uint64_t ldb, uint64_t b_bstride, int b_kmajor,
               uint64_t ldc, uint64_t c_bstride, int block_n, void* stream, bool split = false, int tile_m = 0,
               int block_k = 0) {
  constexpr uint64_t kElem = TF ? 4 : 2;
  constexpr uint32_t kBoxK = TF ? 32 : BK;
  const CUtensorMapDataType dt = TF ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  int rc = eas_driver_init();
  if (rc) return rc;
  if (!a || !b || !c) return eas_fail(EAS_ERR_VALUE, "%s: null operand", who);
  if (M == 0 || N == 0 || batch == 0) return EAS_OK;
  if (K == 0) return eas_fail(EAS_ERR_VALUE, "%s: K == 0 (nothing to accumulate)", who);
  if (block_n != 128 && block_n != 256) return eas_fail(EAS_ERR_VALUE, "%s: block_n must be 128 or 256", who);
  if (tile_m != 0 && tile_m != 128 && tile_m != 256)
    return eas_fail(EAS_ERR_VALUE, "%s: tile_m must be 0 (library's choice), 128 or 256", who);
  if (block_k != 0 && block_k != 64 && block_k != 128)
    return eas_fail(EAS_ERR_VALUE, "%s: block_k must be 0 (library's choice), 64 or 128", who);
  if (M > 0x7fffffffu || N > 0x7fffffffu || K > 0x7fffffffu)
    return eas_fail(EAS_ERR_VALUE, "%s: dimension exceeds 2^31-1", who);
  if (TF && !b_kmajor) return eas_fail(EAS_ERR_VALUE, "%s: B must be K-major", who);
  // split (3xTF32): A and B rows are [hi | lo] of K elements each (K a multiple of 32); the kernel
  // runs 3 K/32 k-blocks over them
  if (split && (K % 32 || 3ull * K > 0x7fffffffull))
    return eas_fail(EAS_ERR_VALUE, "%s: segment length must be a multiple of 32 below 2^31/3", who);
  const uint64_t k_map = split ? 2ull * K : K;
  const int seg_kb = split ? (int)(K / 32) : 0;
  const int k_run = split ? (int)(3 * K) : (int)K;
  // TMA rules: 16-byte aligned bases, 16-byte multiple strides
  if ((reinterpret_cast<uintptr_t>(a) & 15) || (reinterpret_cast<uintptr_t>(b) & 15))
    return eas_fail(EAS_ERR_VALUE, "%s: A/B base must be 16-byte aligned", who);
  if ((lda * kElem) % 16 || (ldb * kElem) % 16 ||
      (batch > 1 && ((a_bstride * kElem) % 16 || (b_bstride * kElem) % 16)))
    return eas_fail(EAS_ERR_VALUE, "%s: A/B strides must be multiples of 16 bytes", who);
  int dev = 0;
  cudaGetDevice(&dev);
  int* status = eas_native_status_dev(dev);
  int num_sms = 148;
  cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev);

  const uint64_t ab = batch > 1 ? a_bstride * kElem : (uint64_t)M * lda * kElem;
  const uint64_t bb = batch > 1 ? b_bstride * kElem : (uint64_t)(b_kmajor ? N : K) * ldb * kElem;
  CUtensorMap ma, mb;
  rc = encode_map(&ma, a, k_map, M, batch, lda * kElem, ab ? ab : 16, kBoxK, BM, dt);
  if (rc) return rc;
  const bool b_mn = !b_kmajor;
  // C through TMA stores when its rows/batches are 16-byte strided and the base is aligned
  const bool tma_c = (reinterpret_cast<uintptr_t>(c) & 15) == 0 && (ldc * 4) % 16 == 0 &&
                     (batch == 1 || (c_bstride * 4) % 16 == 0) && ldc >= N;
  const F16Choice ch = choose_f16(M, N, K, batch, block_n, TF ? 0 : tile_m, TF ? 0 : block_k, tma_c, num_sms);
  const bool pair = ch.pair;
  if (b_mn)
    rc = encode_map(&mb, b, N, K, batch, ldb * kElem, bb ? bb : 16, 64, kBoxK, dt);
  else
    rc = encode_map(&mb, b, k_map, N, batch, ldb * kElem, bb ? bb : 16, kBoxK, pair ? 128u : (uint32_t)block_n, dt);
  if (rc) return rc;
  CUtensorMap mc;
  if (tma_c) {
    const uint64_t cb = batch > 1 ? c_bstride * 4 : (uint64_t)M * ldc * 4;
    rc = encode_map(&mc, c, N, M, batch, ldc * 4, cb ? cb : 16, 32, 32, CU_TENSOR_MAP_DATA_TYPE_FLOAT32);
    if (rc) return rc;
  } else {
    mc = ma;  // unused by the direct-store variant
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const long long ldc_l = (long long)ldc, cbs = (long long)c_bstride;
  if constexpr (TF) {  // K-major operands only
    if (pair)
      return tma_c ? launch_2sm<6, false, true, true>(ma, mb, mc, c, M, N, k_run, batch, ldc_l, cbs, status, s, num_sms,
                                                      seg_kb)
                   : launch_2sm<7, false, false, true>(ma, mb, mc, c, M, N, k_run, batch, ldc_l, cbs, status, s,
                                                       num_sms, seg_kb);
    return tma_c ? launch_variant<128, 6, false, true, true>(ma, mb, mc, c, M, N, k_run, batch, ldc_l, cbs, status, s,
                                                             num_sms, seg_kb)
                 : launch_variant<128, 6, false, false, true>(ma, mb, mc, c, M, N, k_run, batch, ldc_l, cbs, status, s,
                                                              num_sms, seg_kb);
  } else {
    if (ch.ks == 2)
      return launch_f16_choice<2>(ch, b_mn, tma_c, ma, mb, mc, c, M, N, K, batch, ldc_l, cbs, status, s, num_sms);
    return launch_f16_choice<1>(ch, b_mn, tma_c, ma, mb, mc, c, M, N, K, batch, ldc_l, cbs, status, s, num_sms);
  }
}

}  // namespace

extern "C" int eas_gemm_f16_plan(uint32_t M, uint32_t N, uint32_t K, uint32_t batch, int block_n, int tile_m,
                                 int block_k, int c_tma_ok, int num_sms, int resident_pairs, int* out_tile_m,
                                 int* out_tile_n, int* stages, int* ksplit, int* pair, int* out_block_k) {
  // the same helpers, in the same order, as the launch branch of gemm_entry<false> and its launchers
  if (!out_tile_m || !out_tile_n || !stages || !ksplit || !pair || !out_block_k)
    return eas_fail(EAS_ERR_VALUE, "eas_gemm_f16_plan: null");
  if (block_n != 128 && block_n != 256) return eas_fail(EAS_ERR_VALUE, "eas_gemm_f16_plan: block_n must be 128 or 256");
  if (tile_m != 0 && tile_m != 128 && tile_m != 256)
    return eas_fail(EAS_ERR_VALUE, "eas_gemm_f16_plan: tile_m must be 0, 128 or 256");
  if (block_k != 0 && block_k != 64 && block_k != 128)
    return eas_fail(EAS_ERR_VALUE, "eas_gemm_f16_plan: block_k must be 0, 64 or 128");
  if (M == 0 || N == 0 || K == 0 || batch == 0 || num_sms <= 0)
    return eas_fail(EAS_ERR_VALUE, "eas_gemm_f16_plan: empty launch");
  const int kblocks = (int)((K + BK - 1) / BK);
  const F16Choice ch = choose_f16(M, N, K, batch, block_n, tile_m, block_k, c_tma_ok != 0, num_sms);
  *pair = ch.pair ? 1 : 0;
  *out_tile_m = ch.pair ? 256 : BM;
  *out_tile_n = ch.tile_n;
  *stages = ch.stages;
  *out_block_k = BK * ch.ks;
  const long long tiles = (long long)((M + *out_tile_m - 1) / *out_tile_m) * ((N + ch.tile_n - 1) / ch.tile_n) * batch;
  *ksplit = c_tma_ok ? choose_ksplit(tiles, ch.pair ? resident_pairs : num_sms, kblocks, (int)batch) : 1;
  return EAS_OK;
}

extern "C" int eas_gemm_last_config(int* tile_m, int* tile_n, int* stages, int* ksplit, int* pair, int* block_k) {
  if (!tile_m || !tile_n || !stages || !ksplit || !pair || !block_k)
    return eas_fail(EAS_ERR_VALUE, "eas_gemm_last_config: null");
  *tile_m = g_last_config.bm;
  *tile_n = g_last_config.bn;
  *stages = g_last_config.stages;
  *ksplit = g_last_config.ksplit;
  *pair = g_last_config.pair;
  *block_k = g_last_config.block_k;
  return EAS_OK;
}

extern "C" int eas_gemm_f16(const void* a, const void* b, float* c, uint32_t M, uint32_t N, uint32_t K,
                            uint32_t batch, uint64_t lda, uint64_t a_bstride, uint64_t ldb, uint64_t b_bstride,
                            int b_kmajor, uint64_t ldc, uint64_t c_bstride, int block_n, void* stream) {
  return gemm_entry<false>("eas_gemm_f16", a, b, c, M, N, K, batch, lda, a_bstride, ldb, b_bstride, b_kmajor, ldc,
                           c_bstride, block_n, stream);
}

extern "C" int eas_gemm_f16_tile(const void* a, const void* b, float* c, uint32_t M, uint32_t N, uint32_t K,
                                 uint32_t batch, uint64_t lda, uint64_t a_bstride, uint64_t ldb, uint64_t b_bstride,
                                 int b_kmajor, uint64_t ldc, uint64_t c_bstride, int tile_m, int block_n, int block_k,
                                 void* stream) {
  return gemm_entry<false>("eas_gemm_f16_tile", a, b, c, M, N, K, batch, lda, a_bstride, ldb, b_bstride, b_kmajor,
                           ldc, c_bstride, block_n, stream, false, tile_m, block_k);
}

extern "C" int eas_gemm_tf32(const float* a, const float* b, float* c, uint32_t M, uint32_t N, uint32_t K,
                             uint32_t batch, uint64_t lda, uint64_t a_bstride, uint64_t ldb, uint64_t b_bstride,
                             uint64_t ldc, uint64_t c_bstride, int block_n, void* stream) {
  return gemm_entry<true>("eas_gemm_tf32", a, b, c, M, N, K, batch, lda, a_bstride, ldb, b_bstride, 1, ldc,
                          c_bstride, block_n, stream);
}

extern "C" int eas_gemm_3xtf32(const float* a2, const float* b2, float* c, uint32_t M, uint32_t N, uint32_t K,
                               uint32_t batch, uint64_t lda, uint64_t a_bstride, uint64_t ldb, uint64_t b_bstride,
                               uint64_t ldc, uint64_t c_bstride, int block_n, void* stream) {
  return gemm_entry<true>("eas_gemm_3xtf32", a2, b2, c, M, N, K, batch, lda, a_bstride, ldb, b_bstride, 1, ldc,
                          c_bstride, block_n, stream, true);
}

// ---------------------------------------------------------------------------
// Allocation-free variant
// ---------------------------------------------------------------------------
//
// eas_gemm_f16 keeps the kernel's status word in pinned, host-mapped memory
// that the library allocates with cudaHostAlloc on its first call.  Some
// callers cannot let a library allocate: code that owns every allocation in
// the process (a custom device allocator or a fixed memory budget), or code
// that must not trigger an allocation at an arbitrary point.  For them the
// status word lives in the array below instead, a file-scope device variable
// that every GPU loading this library holds until the process exits.
//
// Its size is fixed: one 4-byte word per device, whatever the problem size.
// In host code `g_noalloc_status` is only a stand-in symbol, not a device
// address; the real address comes from cudaGetSymbolAddress, looked up once
// per device with that device current, on the first call made on it.

namespace {
constexpr int kNoAllocStatusWords = 1;  // the whole scratch: one status word
static __device__ __align__(256) int g_noalloc_status[kNoAllocStatusWords];

int* g_noalloc_ptr[64];                    // device address of g_noalloc_status, per device
std::atomic<uint64_t> g_noalloc_ready{0};  // bit d: g_noalloc_ptr[d] is valid
std::mutex g_noalloc_mu;

int noalloc_status_ptr(int dev, int** out) {
  if (dev < 0 || dev >= 64) return eas_fail(EAS_ERR_VALUE, "eas_gemm_f16_noalloc: device %d out of range", dev);
  const uint64_t bit = 1ull << dev;
  if (!(g_noalloc_ready.load() & bit)) {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!(g_noalloc_ready.load() & bit)) {
      void* p = nullptr;
      int rc = eas_cuda_check(cudaGetSymbolAddress(&p, g_noalloc_status), "eas_gemm_f16_noalloc: cudaGetSymbolAddress",
                              EAS_ERR_UNAVAILABLE);
      if (rc) return rc;
      g_noalloc_ptr[dev] = static_cast<int*>(p);
      g_noalloc_ready.fetch_or(bit);
    }
  }
  *out = g_noalloc_ptr[dev];
  return EAS_OK;
}
}  // namespace

extern "C" int eas_gemm_f16_noalloc(const void* a, const void* b, float* c, uint32_t M, uint32_t N, uint32_t K,
                                    uint32_t batch, uint64_t lda, uint64_t a_bstride, uint64_t ldb,
                                    uint64_t b_bstride, int b_kmajor, uint64_t ldc, uint64_t c_bstride, int block_n,
                                    void* stream, int* status_out) {
  if (status_out) *status_out = 0;
  int rc = eas_driver_init();
  if (rc) return rc;
  if (!a || !b || !c) return eas_fail(EAS_ERR_VALUE, "eas_gemm_f16_noalloc: null operand");
  if (M == 0 || N == 0 || batch == 0) return EAS_OK;
  if (K == 0) return eas_fail(EAS_ERR_VALUE, "eas_gemm_f16_noalloc: K == 0 (nothing to accumulate)");
  if (block_n != 128 && block_n != 256)
    return eas_fail(EAS_ERR_VALUE, "eas_gemm_f16_noalloc: block_n must be 128 or 256");
  if (M > 0x7fffffffu || N > 0x7fffffffu || K > 0x7fffffffu || batch > 0x7fffffffu)
    return eas_fail(EAS_ERR_VALUE,
                    "eas_gemm_f16_noalloc: M, N, K and batch must each be below 2^31 (the fixed status word "
                    "covers any size within these limits)");
  if ((reinterpret_cast<uintptr_t>(a) & 15) || (reinterpret_cast<uintptr_t>(b) & 15))
    return eas_fail(EAS_ERR_VALUE, "eas_gemm_f16_noalloc: A/B base must be 16-byte aligned");
  if ((lda * 2) % 16 || (ldb * 2) % 16 || (batch > 1 && ((a_bstride * 2) % 16 || (b_bstride * 2) % 16)))
    return eas_fail(EAS_ERR_VALUE, "eas_gemm_f16_noalloc: A/B strides must be multiples of 8 elements");
  int dev = 0;
  rc = eas_cuda_check(cudaGetDevice(&dev), "eas_gemm_f16_noalloc: cudaGetDevice", EAS_ERR_UNAVAILABLE);
  if (rc) return rc;
  int* status = nullptr;
  rc = noalloc_status_ptr(dev, &status);
  if (rc) return rc;
  int num_sms = 148;
  cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev);

  const uint64_t ab = batch > 1 ? a_bstride * 2 : (uint64_t)M * lda * 2;
  const uint64_t bb = batch > 1 ? b_bstride * 2 : (uint64_t)(b_kmajor ? N : K) * ldb * 2;
  CUtensorMap ma, mb, mc;
  rc = encode_map(&ma, a, K, M, batch, lda * 2, ab ? ab : 16, BK, BM);
  if (rc) return rc;
  const bool b_mn = !b_kmajor;
  rc = b_mn ? encode_map(&mb, b, N, K, batch, ldb * 2, bb ? bb : 16, 64, BK)
            : encode_map(&mb, b, K, N, batch, ldb * 2, bb ? bb : 16, BK, (uint32_t)block_n);
  if (rc) return rc;
  const bool tma_c = (reinterpret_cast<uintptr_t>(c) & 15) == 0 && (ldc * 4) % 16 == 0 &&
                     (batch == 1 || (c_bstride * 4) % 16 == 0) && ldc >= N;
  if (tma_c) {
    const uint64_t cb = batch > 1 ? c_bstride * 4 : (uint64_t)M * ldc * 4;
    rc = encode_map(&mc, c, N, M, batch, ldc * 4, cb ? cb : 16, 32, 32, CU_TENSOR_MAP_DATA_TYPE_FLOAT32);
    if (rc) return rc;
  } else {
    mc = ma;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // the word keeps the previous call's value: clear it before this call's kernel
  rc = eas_cuda_check(cudaMemsetAsync(status, 0, sizeof(int), s), "eas_gemm_f16_noalloc: clear status",
                      EAS_ERR_LAUNCH);
  if (rc) return rc;
  const long long ldc_l = (long long)ldc, cbs = (long long)c_bstride;
  if (block_n == 256) {
    rc = b_mn ? (tma_c ? launch_variant<256, 4, true, true>(ma, mb, mc, c, M, N, K, batch, ldc_l, cbs, status, s, num_sms)
                       : launch_variant<256, 4, true, false>(ma, mb, mc, c, M, N, K, batch, ldc_l, cbs, status, s, num_sms))
              : (tma_c ? launch_variant<256, 4, false, true>(ma, mb, mc, c, M, N, K, batch, ldc_l, cbs, status, s, num_sms)
                       : launch_variant<256, 4, false, false>(ma, mb, mc, c, M, N, K, batch, ldc_l, cbs, status, s, num_sms));
  } else {
    rc = b_mn ? (tma_c ? launch_variant<128, 6, true, true>(ma, mb, mc, c, M, N, K, batch, ldc_l, cbs, status, s, num_sms)
                       : launch_variant<128, 6, true, false>(ma, mb, mc, c, M, N, K, batch, ldc_l, cbs, status, s, num_sms))
              : (tma_c ? launch_variant<128, 6, false, true>(ma, mb, mc, c, M, N, K, batch, ldc_l, cbs, status, s, num_sms)
                       : launch_variant<128, 6, false, false>(ma, mb, mc, c, M, N, K, batch, ldc_l, cbs, status, s, num_sms));
  }
  if (rc || !status_out) return rc;
  // the caller asked for the status: wait for the kernel and copy the word out
  rc = eas_cuda_check(cudaMemcpyAsync(status_out, status, sizeof(int), cudaMemcpyDeviceToHost, s),
                      "eas_gemm_f16_noalloc: read status", EAS_ERR_LAUNCH);
  if (rc) return rc;
  return eas_cuda_check(cudaStreamSynchronize(s), "eas_gemm_f16_noalloc: kernel execution", EAS_ERR_LAUNCH);
}
