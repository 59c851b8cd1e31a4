// sgemm_ffma.cu — native sm_100a kernel for the fp32 tiled-matmul pattern.
//
// The reference's fp32 tiled matmul (easy_as examples/matmul_tiled.py:134-230,
// lowered by eas/codegen/msl.py:920-952 and :1201-1359) stages A and B tiles in
// threadgroup memory and, per K tile of KT elements, computes every output as
//
//     p   = fma(A[m][k0+KT-1], B[k0+KT-1][n], ... fma(A[m][k0], B[k0][n], 0.0f))
//     acc = acc + p                     (acc starts as 0.0f + p, or as p)
//
// in true fp32 (no TF32, no reassociation).  This kernel performs exactly those
// operations for every output, in the same order, so its results are
// bit-identical; only the work split differs:
//
//   * a BM x BN output tile per CTA, a TM x TN register tile per thread (rows
//     ty + (BM/TM)*i, TN/4 column groups of 4); a warp covers 4 thread rows by
//     8 thread columns.  128 x 128 tiles with 8 x 8 per thread (256 threads,
//     1 CTA/SM) for large launches, 64 x 64 with 8 x 4 (128 threads, 3 CTAs/SM
//     for 32-deep K tiles, else 4) when there are fewer than four waves of
//     128 x 128 tiles;
//   * K staged BKS = 32, 16 or 8 deep (the largest that divides KT) through a
//     2- or 3-deep cp.async ring (16-byte copies, zero-filled outside the valid
//     bounds; 4-byte copies when a row of A, B or C is not 16-byte aligned), one
//     __syncthreads per stage;
//   * A kept k-contiguous in shared memory ([BM][BKS+4]) and read as float4
//     along k; interleaved thread rows put the 4 rows a warp reads at once in
//     different banks; B as [BKS][BN+4], 8 consecutive float4 per warp read;
//   * the FMAs are issued as packed pairs (fma.rn.f32x2, two adjacent columns of a row per
//     instruction, the A value broadcast to both lanes) and the fold as add.rn.f32x2: every
//     lane is one fma.rn.f32 / add.rn.f32, so the operations and their order are unchanged;
//   * the first k of every K tile starts the partial sums with
//     fmaf(a, b, 0.0f); the running sum starts at -0.0f (zero_init = 0, and
//     -0.0f + p == p bit for bit, NaN included) or +0.0f (zero_init = 1), so
//     the fold is a plain __fadd_rn.
//
//   C[b][m][n] at c + b*c_bs + m*ldc + n
//   A[b][m][k] at a + b*a_bs + m*lda + k
//   B[b][k][n] at b + b*b_bs + k*ldb + n
//
// A[m][k] reads as zero unless m < a_rows and k < a_k, B[k][n] unless k < b_k
// and n < b_cols (the DSL kernel's masked loads); outputs m < M, n < N are
// computed and stored.  No spin
// waits; the only synchronisation is cp.async.wait_group and __syncthreads.
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdlib>
#include <type_traits>

#include "eas_internal.h"

namespace {

// Zero-fill bounds of the operands: A[m][k] reads as 0 unless m < a_rows and k < a_k, B[k][n]
// unless k < b_k and n < b_cols (the masked loads of the DSL kernel).  Stores cover m < M, n < N.
struct SgemmValid {
  uint32_t a_rows, a_k, b_cols, b_k;
};

__device__ __forceinline__ void cp_async16(float* dst, const float* src, uint32_t bytes) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_async4(float* dst, const float* src, uint32_t bytes) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(d), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

// Packed fp32 pairs (sm_100 fma.rn.f32x2 / add.rn.f32x2): each lane is exactly one fma.rn.f32
// (add.rn.f32), so a pair computes the same two results as two scalar instructions, in one issue
// slot.  d = {a, a} * b + d.
__device__ __forceinline__ void fma2_bcast(float2& d, float a, float2 b) {
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %2};\n\t"
      "mov.b64 rb, {%3, %4};\n\t"
      "mov.b64 rd, {%0, %1};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rd;\n\t"
      "mov.b64 {%0, %1}, rd;\n\t}"
      : "+f"(d.x), "+f"(d.y)
      : "f"(a), "f"(b.x), "f"(b.y));
}
__device__ __forceinline__ void add2(float2& d, float2 p) {
  asm("{\n\t.reg .b64 rp, rd;\n\t"
      "mov.b64 rp, {%2, %3};\n\t"
      "mov.b64 rd, {%0, %1};\n\t"
      "add.rn.f32x2 rd, rd, rp;\n\t"
      "mov.b64 {%0, %1}, rd;\n\t}"
      : "+f"(d.x), "+f"(d.y)
      : "f"(p.x), "f"(p.y));
}

template <int BM, int BN, int BKS, int STAGES, int TM, int TN>
struct SgemmCfg {
  static constexpr int kTX = BN / TN, kTY = BM / TM, kThreads = kTX * kTY, kCG = TN / 4;
  static constexpr int kLdA = BKS + 4, kLdB = BN + 4;
  static constexpr int kAStage = BM * kLdA, kBStage = BKS * kLdB;
  static constexpr int kSmemFloats = STAGES * (kAStage + kBStage);
  static constexpr int kAChunks = BM * BKS / 4 / kThreads, kBChunks = BKS * BN / 4 / kThreads;
  static_assert(kTX % 8 == 0 && kTY % 4 == 0, "warp layout needs BN % 64 == 0 and BM % 32 == 0");
  static_assert(kAChunks >= 1 && kBChunks >= 1, "staging does not divide");
  static_assert(BKS % 4 == 0, "BKS must be a multiple of 4");
};

template <int BM, int BN, int BKS, int STAGES, int TM, int TN, int MINB, bool VEC, bool F2 = false>
__global__ void __launch_bounds__(SgemmCfg<BM, BN, BKS, STAGES, TM, TN>::kThreads, MINB)
sgemm_ffma_kernel(const float* __restrict__ A, const float* __restrict__ B, float* __restrict__ C, uint32_t M,
                  uint32_t N, uint32_t K, uint32_t stages_per_tile, uint64_t lda, uint64_t ldb, uint64_t ldc,
                  uint64_t a_bs, uint64_t b_bs, uint64_t c_bs, int zero_init, SgemmValid valid) {
  using Cfg = SgemmCfg<BM, BN, BKS, STAGES, TM, TN>;
  extern __shared__ __align__(16) float smem[];
  float* sA = smem;
  float* sB = smem + STAGES * Cfg::kAStage;
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  constexpr int kWarpsX = Cfg::kTX / 8;
  const int ty = (warp / kWarpsX) * 4 + (lane >> 3);
  const int tx = (warp % kWarpsX) * 8 + (lane & 7);
  const uint32_t m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  A += (uint64_t)blockIdx.z * a_bs;
  B += (uint64_t)blockIdx.z * b_bs;
  C += (uint64_t)blockIdx.z * c_bs;
  const uint32_t nstages = K / BKS;

  auto issue = [&](uint32_t st) {
    if (st < nstages && !VEC) {  // rows not 16-byte aligned: element-wise copies
      const int buf = st % STAGES;
      const uint32_t k0 = st * BKS;
#pragma unroll
      for (int q = 0; q < BM * BKS / Cfg::kThreads; ++q) {
        const int idx = tid + q * Cfg::kThreads;
        const int r = idx / BKS, kc = idx % BKS;
        const uint32_t m = m0 + r, k = k0 + kc;
        const bool live = m < valid.a_rows && k < valid.a_k;
        cp_async4(sA + buf * Cfg::kAStage + r * Cfg::kLdA + kc, live ? A + (uint64_t)m * lda + k : A, live ? 4u : 0u);
      }
#pragma unroll
      for (int q = 0; q < BKS * BN / Cfg::kThreads; ++q) {
        const int idx = tid + q * Cfg::kThreads;
        const int r = idx / BN, nc = idx % BN;
        const uint32_t n = n0 + nc, k = k0 + r;
        const bool live = n < valid.b_cols && k < valid.b_k;
        cp_async4(sB + buf * Cfg::kBStage + r * Cfg::kLdB + nc, live ? B + (uint64_t)k * ldb + n : B, live ? 4u : 0u);
      }
    } else if (st < nstages) {
      const int buf = st % STAGES;
      const uint32_t k0 = st * BKS;
#pragma unroll
      for (int q = 0; q < Cfg::kAChunks; ++q) {
        const int idx = tid + q * Cfg::kThreads;
        const int r = idx / (BKS / 4), kc = (idx % (BKS / 4)) * 4;
        const uint32_t m = m0 + r, k = k0 + kc;
        const bool live = m < valid.a_rows && k < valid.a_k;
        const uint32_t bytes = live ? (k + 4 <= valid.a_k ? 16u : 4u * (valid.a_k - k)) : 0u;
        const float* src = live ? A + (uint64_t)m * lda + k : A;
        cp_async16(sA + buf * Cfg::kAStage + r * Cfg::kLdA + kc, src, bytes);
      }
#pragma unroll
      for (int q = 0; q < Cfg::kBChunks; ++q) {
        const int idx = tid + q * Cfg::kThreads;
        const int r = idx / (BN / 4), nc = (idx % (BN / 4)) * 4;
        const uint32_t n = n0 + nc, k = k0 + r;
        const bool live = n < valid.b_cols && k < valid.b_k;
        const uint32_t bytes = live ? (n + 4 <= valid.b_cols ? 16u : 4u * (valid.b_cols - n)) : 0u;
        const float* src = live ? B + (uint64_t)k * ldb + n : B;
        cp_async16(sB + buf * Cfg::kBStage + r * Cfg::kLdB + nc, src, bytes);
      }
    }
    cp_async_commit();
  };

  static_assert(!F2 || TN % 2 == 0, "packed pairs need an even TN");
  float acc[TM][TN], p[TM][TN];
  const float init = zero_init ? 0.0f : -0.0f;
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = init;

#pragma unroll
  for (int st = 0; st < STAGES - 1; ++st) issue(st);

  auto compute = [&](int buf, auto first_tag) {
    constexpr bool kFirst = decltype(first_tag)::value;
    const float* a = sA + buf * Cfg::kAStage + ty * Cfg::kLdA;
    const float* b = sB + buf * Cfg::kBStage + tx * 4;
#pragma unroll
    for (int kb = 0; kb < BKS; kb += 4) {
      float4 af[TM];
#pragma unroll
      for (int i = 0; i < TM; ++i) af[i] = *reinterpret_cast<const float4*>(a + i * Cfg::kTY * Cfg::kLdA + kb);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        float bv[TN];
#pragma unroll
        for (int g = 0; g < Cfg::kCG; ++g) {
          const float4 bq = *reinterpret_cast<const float4*>(b + (kb + kk) * Cfg::kLdB + g * (BN / Cfg::kCG));
          bv[4 * g + 0] = bq.x;
          bv[4 * g + 1] = bq.y;
          bv[4 * g + 2] = bq.z;
          bv[4 * g + 3] = bq.w;
        }
        float av[TM];
#pragma unroll
        for (int i = 0; i < TM; ++i) av[i] = kk == 0 ? af[i].x : kk == 1 ? af[i].y : kk == 2 ? af[i].z : af[i].w;
        if constexpr (F2) {
#pragma unroll
          for (int i = 0; i < TM; ++i)
#pragma unroll
            for (int j = 0; j < TN; j += 2) {
              float2 d = (kFirst && kb == 0 && kk == 0) ? make_float2(0.0f, 0.0f) : make_float2(p[i][j], p[i][j + 1]);
              fma2_bcast(d, av[i], make_float2(bv[j], bv[j + 1]));
              p[i][j] = d.x;
              p[i][j + 1] = d.y;
            }
        } else {
#pragma unroll
          for (int i = 0; i < TM; ++i)
#pragma unroll
            for (int j = 0; j < TN; ++j)
              p[i][j] = (kFirst && kb == 0 && kk == 0) ? fmaf(av[i], bv[j], 0.0f) : fmaf(av[i], bv[j], p[i][j]);
        }
      }
    }
  };

  uint32_t in_tile = 0;
  for (uint32_t s = 0; s < nstages; ++s) {
    cp_async_wait<STAGES - 2>();
    __syncthreads();
    issue(s + STAGES - 1);
    const int buf = s % STAGES;
    if (in_tile == 0)
      compute(buf, std::true_type{});
    else
      compute(buf, std::false_type{});
    if (++in_tile == stages_per_tile) {  // end of a K tile: fold its partial sums, in order
      in_tile = 0;
      if constexpr (F2) {
#pragma unroll
        for (int i = 0; i < TM; ++i)
#pragma unroll
          for (int j = 0; j < TN; j += 2) {
            float2 d = make_float2(acc[i][j], acc[i][j + 1]);
            add2(d, make_float2(p[i][j], p[i][j + 1]));
            acc[i][j] = d.x;
            acc[i][j + 1] = d.y;
          }
      } else {
#pragma unroll
        for (int i = 0; i < TM; ++i)
#pragma unroll
          for (int j = 0; j < TN; ++j) acc[i][j] = __fadd_rn(acc[i][j], p[i][j]);
      }
    }
  }
  cp_async_wait<0>();

#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const uint32_t m = m0 + ty + Cfg::kTY * i;
    if (m >= M) continue;
    float* row = C + (uint64_t)m * ldc;
#pragma unroll
    for (int h = 0; h < Cfg::kCG; ++h) {
      const uint32_t n = n0 + h * (BN / Cfg::kCG) + tx * 4;
      const float* v = &acc[i][h * 4];
      if (VEC && n + 3 < N) {
        *reinterpret_cast<float4*>(row + n) = make_float4(v[0], v[1], v[2], v[3]);
      } else {
        for (int j = 0; j < 4; ++j)
          if (n + j < N) row[n + j] = v[j];
      }
    }
  }
}

template <int BM, int BN, int BKS, int STAGES, int TM, int TN, int MINB, bool VEC, bool F2 = false>
int launch_sgemm(const float* a, const float* b, float* c, uint32_t M, uint32_t N, uint32_t K, uint32_t k_tile,
                 uint32_t batch, uint64_t lda, uint64_t a_bs, uint64_t ldb, uint64_t b_bs, uint64_t ldc,
                 uint64_t c_bs, int zero_init, SgemmValid valid, cudaStream_t s) {
  using Cfg = SgemmCfg<BM, BN, BKS, STAGES, TM, TN>;
  const uint32_t gy = (M + BM - 1) / BM;
  if (gy > 65535) return eas_fail(EAS_ERR_VALUE, "eas_sgemm_f32_tiled: M too large");
  const size_t smem = Cfg::kSmemFloats * sizeof(float);
  auto kern = sgemm_ffma_kernel<BM, BN, BKS, STAGES, TM, TN, MINB, VEC, F2>;
  static int attr_done[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return eas_fail(EAS_ERR_VALUE, "eas_sgemm_f32_tiled: device index out of range");
  if (!attr_done[dev]) {
    int rc = eas_cuda_check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                            "sgemm_ffma smem attribute", EAS_ERR_LAUNCH);
    if (rc) return rc;
    attr_done[dev] = 1;
  }
  dim3 grid((N + BN - 1) / BN, gy, batch);
  kern<<<grid, Cfg::kThreads, smem, s>>>(a, b, c, M, N, K, k_tile / BKS, lda, ldb, ldc, a_bs, b_bs, c_bs,
                                         zero_init, valid);
  return eas_cuda_check(cudaGetLastError(), "sgemm_ffma launch", EAS_ERR_LAUNCH);
}

}  // namespace

extern "C" int eas_sgemm_f32_tiled(const float* a, const float* b, float* c, uint32_t M, uint32_t N, uint32_t K,
                                   uint32_t k_tile, uint32_t batch, uint64_t lda, uint64_t a_bstride, uint64_t ldb,
                                   uint64_t b_bstride, uint64_t ldc, uint64_t c_bstride, int zero_init,
                                   uint32_t a_rows, uint32_t a_k, uint32_t b_cols, uint32_t b_k, void* stream) {
  if (!a || !b || !c) return eas_fail(EAS_ERR_VALUE, "eas_sgemm_f32_tiled: null operand");
  if (M == 0 || N == 0 || batch == 0) return EAS_OK;
  if (K == 0 || k_tile == 0 || K % k_tile) return eas_fail(EAS_ERR_VALUE, "eas_sgemm_f32_tiled: K must be a positive multiple of k_tile");
  if (k_tile % 8) return eas_fail(EAS_ERR_VALUE, "eas_sgemm_f32_tiled: k_tile must be a multiple of 8");
  if ((reinterpret_cast<uintptr_t>(a) & 3) || (reinterpret_cast<uintptr_t>(b) & 3) ||
      (reinterpret_cast<uintptr_t>(c) & 3))
    return eas_fail(EAS_ERR_VALUE, "eas_sgemm_f32_tiled: operands must be 4-byte aligned");
  // 16-byte copies and stores when every row of A, B and C starts on a 16-byte boundary
  const bool vec = !((reinterpret_cast<uintptr_t>(a) & 15) || (reinterpret_cast<uintptr_t>(b) & 15) ||
                     (reinterpret_cast<uintptr_t>(c) & 15) || lda % 4 || ldb % 4 || ldc % 4 ||
                     (batch > 1 && (a_bstride % 4 || b_bstride % 4 || c_bstride % 4)));
  if (batch > 65535) return eas_fail(EAS_ERR_VALUE, "eas_sgemm_f32_tiled: batch exceeds 65535");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const SgemmValid valid{a_rows < M ? a_rows : M, a_k < K ? a_k : K, b_cols < N ? b_cols : N, b_k < K ? b_k : K};
  // 128 x 128 tiles (8 x 8 per thread, 1 CTA per SM) when the launch has at least four waves of
  // them; otherwise 64 x 64 tiles (8 x 4 per thread, 4 CTAs per SM), which balance small
  // problems better over the SMs (2048^3: 1024 tiles instead of 256 on 148 SMs).
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const uint64_t big_tiles = (uint64_t)((M + 127) / 128) * ((N + 127) / 128) * batch;
  const bool small = big_tiles < 4ull * (uint64_t)sms;
#define EAS_SG(BM, BN, BKS, ST, TM, TN, MINB)                                                                    \
  (vec ? (f2 ? launch_sgemm<BM, BN, BKS, ST, TM, TN, MINB, true, true>(a, b, c, M, N, K, k_tile, batch, lda,       \
                                                                       a_bstride, ldb, b_bstride, ldc, c_bstride,  \
                                                                       zero_init, valid, s)                        \
              : launch_sgemm<BM, BN, BKS, ST, TM, TN, MINB, true>(a, b, c, M, N, K, k_tile, batch, lda, a_bstride, \
                                                                  ldb, b_bstride, ldc, c_bstride, zero_init, valid, s)) \
       : launch_sgemm<BM, BN, BKS, ST, TM, TN, MINB, false>(a, b, c, M, N, K, k_tile, batch, lda, a_bstride, ldb,   \
                                                            b_bstride, ldc, c_bstride, zero_init, valid, s))
  // packed fma.rn.f32x2 pairs (the same fp32 operations, half the FMA issue slots): C3 44.6 TFLOP/s
  // against 41.6 with scalar FFMAs on one B200, bit-identical; EAS_SGEMM_F2=0 keeps scalar FFMAs
  static const bool f2 = [] {
    const char* e = getenv("EAS_SGEMM_F2");
    return !(e && e[0] == '0');
  }();
  if (small) {
    // 3 CTAs per SM (up to 168 registers; 156 used) rather than 4 at 128: 46.4 TFLOP/s against
    // 44.4 on C3 with packed pairs (the spare registers go to deeper operand prefetch)
    if (k_tile % 32 == 0) return EAS_SG(64, 64, 32, 2, 8, 4, 3);
    if (k_tile % 16 == 0) return EAS_SG(64, 64, 16, 2, 8, 4, 4);
    return EAS_SG(64, 64, 8, 3, 8, 4, 4);
  }
  if (k_tile % 32 == 0) return EAS_SG(128, 128, 32, 3, 8, 8, 1);
  if (k_tile % 16 == 0) return EAS_SG(128, 128, 16, 3, 8, 8, 1);
  return EAS_SG(128, 128, 8, 3, 8, 8, 1);
#undef EAS_SG
}
