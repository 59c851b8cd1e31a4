// cast_f16.cu — operand staging for native GEMMs on tcgen05:
//   * f32 -> f16 for the proven simdgroup-MMA GEMM;
//   * f32 -> (hi, lo) TF32 pairs for the opt-in 3xTF32 mode of proven fp32 matmuls.
//
// The reference's matmul_simdgroup kernel (easy_as examples/matmul_simdgroup.py:29-127) casts
// its f32 A and B tiles to f16 in threadgroup memory (cast with round-to-nearest-even, the same
// cvt.rn.f16.f32 the generated kernel uses) and multiplies them on the matrix units with f32
// accumulation.  When that kernel is proven to be a GEMM, the runtime writes the f16 operands
// once with this kernel and runs the tcgen05 GEMM on them.
//
//   dst[b][r][c] = (r < rows_valid && c < cols_valid) ? f16(src[b*bs_src + r*ld_src + c]) : 0
//   for r < rows, c < cols_pad (cols_pad a multiple of 8, ld_dst >= cols_pad, dst 16-byte aligned)
//
// Each thread writes 8 halves (16 bytes); grid-stride loop.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "eas_internal.h"

namespace {

__device__ __forceinline__ uint16_t f2h_rn(float f) {
  uint16_t h;
  asm("cvt.rn.f16.f32 %0, %1;" : "=h"(h) : "f"(f));
  return h;
}

__global__ void cast_f32_f16_kernel(const float* __restrict__ src, uint16_t* __restrict__ dst, uint32_t rows,
                                    uint32_t groups, uint64_t ld_src, uint64_t ld_dst, uint32_t rows_valid,
                                    uint32_t cols_valid, uint32_t batch, uint64_t bs_src, uint64_t bs_dst) {
  const uint64_t total = (uint64_t)batch * rows * groups;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t g = i % groups;
    const uint64_t br = i / groups;
    const uint32_t r = br % rows;
    const uint32_t b = br / rows;
    const uint32_t c0 = g * 8;
    uint16_t h[8];
    const float* s = src + b * bs_src + (uint64_t)r * ld_src;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t c = c0 + j;
      h[j] = (r < rows_valid && c < cols_valid) ? f2h_rn(s[c]) : (uint16_t)0;
    }
    uint4 v;
    v.x = h[0] | ((uint32_t)h[1] << 16);
    v.y = h[2] | ((uint32_t)h[3] << 16);
    v.z = h[4] | ((uint32_t)h[5] << 16);
    v.w = h[6] | ((uint32_t)h[7] << 16);
    *reinterpret_cast<uint4*>(dst + b * bs_dst + (uint64_t)r * ld_dst + c0) = v;
  }
}

}  // namespace

namespace {

// x = hi + lo + (rest): hi = tf32(x), lo = tf32(x - hi) (x - hi is exact in f32); both have their
// 13 low mantissa bits clear, so kind::tf32 reads them exactly.
__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

__device__ __forceinline__ float tf32_part(float x, bool lo) {
  const float hi = tf32_rna(x);
  return lo ? tf32_rna(x - hi) : hi;
}

// Rows of src ([rows][k], row pitch ld_src) into dst rows of 3 segments of kp elements:
// segment s holds tf32_part(src, bit s of lo_mask), zero outside r < rows_valid, k < k_valid.
__global__ void split3_rows_kernel(const float* __restrict__ src, float* __restrict__ dst, uint32_t rows,
                                   uint32_t kp, uint64_t ld_src, uint32_t rows_valid, uint32_t k_valid,
                                   uint32_t batch, uint64_t bs_src, int lo_mask) {
  const uint64_t per = (uint64_t)rows * kp;
  const uint64_t total = (uint64_t)batch * per;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t b = i / per;
    const uint64_t rk = i % per;
    const uint32_t r = rk / kp, k = rk % kp;
    const float x = (r < rows_valid && k < k_valid) ? src[b * bs_src + (uint64_t)r * ld_src + k] : 0.0f;
    float* d = dst + b * 3 * per + (uint64_t)r * 3 * kp + k;
#pragma unroll
    for (int seg = 0; seg < 3; ++seg) d[(uint64_t)seg * kp] = tf32_part(x, (lo_mask >> seg) & 1);
  }
}

// Columns of src ([k][cols], row pitch ld_src) into dst rows (one per column) of 3 segments of kp
// elements, through a 32 x 32 shared-memory transpose: dst[n][s*kp + k] = tf32_part(src[k][n], ...).
__global__ void split3_cols_kernel(const float* __restrict__ src, float* __restrict__ dst, uint32_t cols,
                                   uint32_t kp, uint64_t ld_src, uint32_t cols_valid, uint32_t k_valid,
                                   uint64_t bs_src, int lo_mask) {
  __shared__ float tile[32][33];
  const uint32_t k0 = blockIdx.x * 32, n0 = blockIdx.y * 32, b = blockIdx.z;
  const float* s = src + (uint64_t)b * bs_src;
  float* d = dst + (uint64_t)b * 3 * (uint64_t)cols * kp;
  for (int j = threadIdx.y; j < 32; j += blockDim.y) {
    const uint32_t k = k0 + j, n = n0 + threadIdx.x;
    tile[j][threadIdx.x] = (k < k_valid && n < cols_valid) ? s[(uint64_t)k * ld_src + n] : 0.0f;
  }
  __syncthreads();
  for (int j = threadIdx.y; j < 32; j += blockDim.y) {
    const uint32_t n = n0 + j, k = k0 + threadIdx.x;
    if (n < cols && k < kp) {
      const float x = tile[threadIdx.x][j];
#pragma unroll
      for (int seg = 0; seg < 3; ++seg) d[(uint64_t)n * 3 * kp + (uint64_t)seg * kp + k] = tf32_part(x, (lo_mask >> seg) & 1);
    }
  }
}

}  // namespace

extern "C" int eas_split3_tf32(const float* src, float* dst, uint32_t rows, uint32_t kp, uint64_t ld_src,
                               uint32_t rows_valid, uint32_t k_valid, uint32_t batch, uint64_t bs_src, int lo_mask,
                               int transpose, void* stream) {
  if (!src || !dst) return eas_fail(EAS_ERR_VALUE, "eas_split3_tf32: null pointer");
  if (rows == 0 || kp == 0 || batch == 0) return EAS_OK;
  if (batch > 65535) return eas_fail(EAS_ERR_VALUE, "eas_split3_tf32: batch exceeds 65535");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (transpose) {
    dim3 grid((kp + 31) / 32, (rows + 31) / 32, batch);
    if (grid.y > 65535) return eas_fail(EAS_ERR_VALUE, "eas_split3_tf32: too many columns");
    split3_cols_kernel<<<grid, dim3(32, 8, 1), 0, s>>>(src, dst, rows, kp, ld_src, rows_valid, k_valid, bs_src,
                                                       lo_mask);
  } else {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const uint64_t total = (uint64_t)batch * rows * kp;
    const uint64_t want = (total + 255) / 256;
    const unsigned grid = (unsigned)(want < (uint64_t)sms * 16 ? want : (uint64_t)sms * 16);
    split3_rows_kernel<<<grid, 256, 0, s>>>(src, dst, rows, kp, ld_src, rows_valid, k_valid, batch, bs_src, lo_mask);
  }
  return eas_cuda_check(cudaGetLastError(), "split3_tf32 launch", EAS_ERR_LAUNCH);
}

extern "C" int eas_cast_f32_f16_2d(const float* src, void* dst, uint32_t rows, uint32_t cols_pad, uint64_t ld_src,
                                   uint64_t ld_dst, uint32_t rows_valid, uint32_t cols_valid, uint32_t batch,
                                   uint64_t bs_src, uint64_t bs_dst, void* stream) {
  if (!src || !dst) return eas_fail(EAS_ERR_VALUE, "eas_cast_f32_f16_2d: null pointer");
  if (rows == 0 || cols_pad == 0 || batch == 0) return EAS_OK;
  if (cols_pad % 8 || ld_dst % 8 || ld_dst < cols_pad || (batch > 1 && bs_dst % 8) ||
      (reinterpret_cast<uintptr_t>(dst) & 15))
    return eas_fail(EAS_ERR_VALUE, "eas_cast_f32_f16_2d: destination rows must be 16-byte aligned");
  if (cols_valid > cols_pad) return eas_fail(EAS_ERR_VALUE, "eas_cast_f32_f16_2d: cols_valid exceeds cols_pad");
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const uint64_t total = (uint64_t)batch * rows * (cols_pad / 8);
  const uint64_t want = (total + 255) / 256;
  const unsigned grid = (unsigned)(want < (uint64_t)sms * 16 ? want : (uint64_t)sms * 16);
  cast_f32_f16_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      src, static_cast<uint16_t*>(dst), rows, cols_pad / 8, ld_src, ld_dst, rows_valid, cols_valid, batch, bs_src,
      bs_dst);
  return eas_cuda_check(cudaGetLastError(), "cast_f32_f16 launch", EAS_ERR_LAUNCH);
}
