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
// bit-identical; only the work split differs: a 128 x 128 output tile per CTA,
// an 8 x 8 register tile per thread (two 4-wide row and column groups, so the
// shared-memory reads are 128-bit and conflict-free), K staged BKS = 8 or 16
// deep through double-buffered shared memory with register prefetch, one
// __syncthreads per stage.  A is stored transposed (k-major) in shared memory.
//
//   C[b][m][n] at c + b*c_bs + m*ldc + n
//   A[b][m][k] at a + b*a_bs + m*lda + k
//   B[b][k][n] at b + b*b_bs + k*ldb + n
//
// Rows m >= M and columns n >= N are read as zero and not stored.  No spin
// waits; the only synchronisation is __syncthreads.
#include <cuda_runtime.h>
#include <stdint.h>

#include "eas_internal.h"

namespace {

constexpr int kBM = 128, kBN = 128, kThreads = 256, kPad = 4;

template <int BKS>
struct SgemmSmem {
  float a[2][BKS][kBM + kPad];  // k-major A tile
  float b[2][BKS][kBN + kPad];
};

template <int BKS>
__global__ void __launch_bounds__(kThreads, 1)
sgemm_ffma_kernel(const float* __restrict__ A, const float* __restrict__ B, float* __restrict__ C, uint32_t M,
                  uint32_t N, uint32_t K, uint32_t stages_per_tile, uint64_t lda, uint64_t ldb, uint64_t ldc,
                  uint64_t a_bs, uint64_t b_bs, uint64_t c_bs, int zero_init) {
  __shared__ __align__(16) SgemmSmem<BKS> sm;
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const uint32_t m0 = blockIdx.y * kBM, n0 = blockIdx.x * kBN;
  A += (uint64_t)blockIdx.z * a_bs;
  B += (uint64_t)blockIdx.z * b_bs;
  C += (uint64_t)blockIdx.z * c_bs;

  // global -> register staging: A rows of BKS floats (BKS/4 float4 each), B rows of 128 floats
  constexpr int kAPerRow = BKS / 4;                     // float4 per A row
  constexpr int kARowsPerPass = kThreads / kAPerRow;    // rows covered by one pass of the CTA
  constexpr int kPasses = BKS / 8;                      // passes for A (128 rows) and for B (BKS rows)
  const int a_row = tid / kAPerRow, a_kc = (tid % kAPerRow) * 4;
  const int b_row = tid >> 5, b_nc = (tid & 31) * 4;
  float4 ra[kPasses], rb[kPasses];

  auto load_stage = [&](uint32_t k0) {
#pragma unroll
    for (int q = 0; q < kPasses; ++q) {
      const uint32_t m = m0 + a_row + q * kARowsPerPass;
      ra[q] = m < M ? __ldg(reinterpret_cast<const float4*>(A + (uint64_t)m * lda + k0 + a_kc))
                    : make_float4(0.f, 0.f, 0.f, 0.f);
      const uint32_t k = k0 + b_row + q * 8;
      const uint32_t n = n0 + b_nc;
      const float* src = B + (uint64_t)k * ldb + n;
      if (n + 3 < N) {
        rb[q] = __ldg(reinterpret_cast<const float4*>(src));
      } else {
        rb[q].x = n < N ? src[0] : 0.f;
        rb[q].y = n + 1 < N ? src[1] : 0.f;
        rb[q].z = n + 2 < N ? src[2] : 0.f;
        rb[q].w = 0.f;
      }
    }
  };
  auto store_stage = [&](int buf) {
#pragma unroll
    for (int q = 0; q < kPasses; ++q) {
      const int r = a_row + q * kARowsPerPass;
      sm.a[buf][a_kc + 0][r] = ra[q].x;
      sm.a[buf][a_kc + 1][r] = ra[q].y;
      sm.a[buf][a_kc + 2][r] = ra[q].z;
      sm.a[buf][a_kc + 3][r] = ra[q].w;
      *reinterpret_cast<float4*>(&sm.b[buf][b_row + q * 8][b_nc]) = rb[q];
    }
  };

  float acc[8][8], p[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      acc[i][j] = 0.f;
      p[i][j] = 0.f;
    }
  bool first = true;

  const uint32_t nstages = K / BKS;
  load_stage(0);
  store_stage(0);
  __syncthreads();
  uint32_t in_tile = 0;
  for (uint32_t s = 0; s < nstages; ++s) {
    const int cur = s & 1;
    if (s + 1 < nstages) load_stage((s + 1) * BKS);
#pragma unroll
    for (int k = 0; k < BKS; ++k) {
      const float4 a0 = *reinterpret_cast<const float4*>(&sm.a[cur][k][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&sm.a[cur][k][64 + ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&sm.b[cur][k][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&sm.b[cur][k][64 + tx * 4]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) p[i][j] = fmaf(av[i], bv[j], p[i][j]);
    }
    if (++in_tile == stages_per_tile) {  // end of a K tile: fold its partial sums, in order
      in_tile = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          acc[i][j] = first ? (zero_init ? __fadd_rn(0.f, p[i][j]) : p[i][j]) : __fadd_rn(acc[i][j], p[i][j]);
          p[i][j] = 0.f;
        }
      first = false;
    }
    if (s + 1 < nstages) {
      store_stage(cur ^ 1);
      __syncthreads();
    }
  }

#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (m >= M) continue;
    float* row = C + (uint64_t)m * ldc;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t n = n0 + h * 64 + tx * 4;
      const float* v = &acc[i][h * 4];
      if (n + 3 < N) {
        *reinterpret_cast<float4*>(row + n) = make_float4(v[0], v[1], v[2], v[3]);
      } else {
        for (int j = 0; j < 4; ++j)
          if (n + j < N) row[n + j] = v[j];
      }
    }
  }
}

}  // namespace

extern "C" int eas_sgemm_f32_tiled(const float* a, const float* b, float* c, uint32_t M, uint32_t N, uint32_t K,
                                   uint32_t k_tile, uint32_t batch, uint64_t lda, uint64_t a_bstride, uint64_t ldb,
                                   uint64_t b_bstride, uint64_t ldc, uint64_t c_bstride, int zero_init,
                                   void* stream) {
  if (!a || !b || !c) return eas_fail(EAS_ERR_VALUE, "eas_sgemm_f32_tiled: null operand");
  if (M == 0 || N == 0 || batch == 0) return EAS_OK;
  if (K == 0 || k_tile == 0 || K % k_tile) return eas_fail(EAS_ERR_VALUE, "eas_sgemm_f32_tiled: K must be a positive multiple of k_tile");
  int bks = (k_tile % 16 == 0) ? 16 : (k_tile % 8 == 0 ? 8 : 0);
  if (!bks) return eas_fail(EAS_ERR_VALUE, "eas_sgemm_f32_tiled: k_tile must be a multiple of 8");
  if ((reinterpret_cast<uintptr_t>(a) & 15) || (reinterpret_cast<uintptr_t>(b) & 15) ||
      (reinterpret_cast<uintptr_t>(c) & 15))
    return eas_fail(EAS_ERR_VALUE, "eas_sgemm_f32_tiled: operands must be 16-byte aligned");
  if (lda % 4 || ldb % 4 || ldc % 4 || (batch > 1 && (a_bstride % 4 || b_bstride % 4 || c_bstride % 4)))
    return eas_fail(EAS_ERR_VALUE, "eas_sgemm_f32_tiled: strides must be multiples of 4 elements");
  if (batch > 65535) return eas_fail(EAS_ERR_VALUE, "eas_sgemm_f32_tiled: batch exceeds 65535");
  const uint32_t gy = (M + kBM - 1) / kBM;
  if (gy > 65535) return eas_fail(EAS_ERR_VALUE, "eas_sgemm_f32_tiled: M too large");
  dim3 grid((N + kBN - 1) / kBN, gy, batch);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (bks == 16)
    sgemm_ffma_kernel<16><<<grid, kThreads, 0, s>>>(a, b, c, M, N, K, k_tile / 16, lda, ldb, ldc, a_bstride,
                                                    b_bstride, c_bstride, zero_init);
  else
    sgemm_ffma_kernel<8><<<grid, kThreads, 0, s>>>(a, b, c, M, N, K, k_tile / 8, lda, ldb, ldc, a_bstride,
                                                   b_bstride, c_bstride, zero_init);
  return eas_cuda_check(cudaGetLastError(), "sgemm_ffma launch", EAS_ERR_LAUNCH);
}
