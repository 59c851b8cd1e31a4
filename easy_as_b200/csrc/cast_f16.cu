// cast_f16.cu — operand staging for native GEMMs on tcgen05:
//   * f32 -> f16 for the proven simdgroup-MMA GEMM;
//   * f16 -> f16 re-pitching for fp16 dot GEMMs whose rows TMA cannot read in place (a row
//     pitch or base that is not a multiple of 16 bytes);
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

__device__ __forceinline__ uint16_t to_f16_bits(float f) { return f2h_rn(f); }
__device__ __forceinline__ uint16_t to_f16_bits(uint16_t h) { return h; }  // f16 source: bits copied

template <typename Src>
__global__ void cast_f32_f16_kernel(const Src* __restrict__ src, uint16_t* __restrict__ dst, uint32_t rows,
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
    const Src* s = src + b * bs_src + (uint64_t)r * ld_src;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t c = c0 + j;
      h[j] = (r < rows_valid && c < cols_valid) ? to_f16_bits(s[c]) : (uint16_t)0;
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

// x = hi + lo + (rest): hi = tf32(x), lo = tf32(x - hi) (x - hi is exact in f32), both rounded to
// nearest with ties away from zero; their 13 low mantissa bits are clear, so kind::tf32 reads
// them exactly.
__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// Rows of src ([rows][k], row pitch ld_src) into dst rows [hi | lo] of kp elements each (kp a
// multiple of 4), zero outside r < rows_valid, k < k_valid.  Four k per thread, 16-byte stores.
__global__ void split_rows_kernel(const float* __restrict__ src, float* __restrict__ dst, uint32_t rows, uint32_t kp,
                                  uint64_t ld_src, uint32_t rows_valid, uint32_t k_valid, uint32_t batch,
                                  uint64_t bs_src) {
  const uint32_t k0 = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (k0 >= kp) return;
  for (uint32_t b = blockIdx.z; b < batch; b += gridDim.z) {
    for (uint32_t r = blockIdx.y; r < rows; r += gridDim.y) {
      const float* s = src + b * bs_src + (uint64_t)r * ld_src;
      float x[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) x[j] = (r < rows_valid && k0 + j < k_valid) ? s[k0 + j] : 0.0f;
      float4 hi, lo;
      hi.x = tf32_rna(x[0]); lo.x = tf32_rna(x[0] - hi.x);
      hi.y = tf32_rna(x[1]); lo.y = tf32_rna(x[1] - hi.y);
      hi.z = tf32_rna(x[2]); lo.z = tf32_rna(x[2] - hi.z);
      hi.w = tf32_rna(x[3]); lo.w = tf32_rna(x[3] - hi.w);
      float* d = dst + ((uint64_t)b * rows + r) * 2 * kp + k0;
      *reinterpret_cast<float4*>(d) = hi;
      *reinterpret_cast<float4*>(d + kp) = lo;
    }
  }
}

// Columns of src ([k][cols], row pitch ld_src) into dst rows (one per column) [hi | lo] of kp
// elements each, through a 64 (k) x 32 (column) shared-memory tile: coalesced 128-byte loads
// along columns, 8-byte stores along k.
__global__ void split_cols_kernel(const float* __restrict__ src, float* __restrict__ dst, uint32_t cols, uint32_t kp,
                                  uint64_t ld_src, uint32_t cols_valid, uint32_t k_valid, uint32_t batch,
                                  uint64_t bs_src) {
  __shared__ float tile[64][33];
  const uint32_t k0 = blockIdx.x * 64;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 8 warps
  for (uint32_t b = blockIdx.z; b < batch; b += gridDim.z) {
    for (uint32_t n0 = blockIdx.y * 32; n0 < cols; n0 += gridDim.y * 32) {
      const float* s = src + b * bs_src;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint32_t k = k0 + ty + 8 * j, n = n0 + tx;
        tile[ty + 8 * j][tx] = (k < k_valid && n < cols_valid) ? s[(uint64_t)k * ld_src + n] : 0.0f;
      }
      __syncthreads();
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t nl = ty + 8 * j, n = n0 + nl, k = k0 + 2 * tx;
        if (n < cols && k < kp) {  // kp is a multiple of 4: k and k + 1 are both inside
          const float x0 = tile[2 * tx][nl], x1 = tile[2 * tx + 1][nl];
          float2 hi, lo;
          hi.x = tf32_rna(x0); lo.x = tf32_rna(x0 - hi.x);
          hi.y = tf32_rna(x1); lo.y = tf32_rna(x1 - hi.y);
          float* d = dst + ((uint64_t)b * cols + n) * 2 * kp + k;
          *reinterpret_cast<float2*>(d) = hi;
          *reinterpret_cast<float2*>(d + kp) = lo;
        }
      }
      __syncthreads();
    }
  }
}

}  // namespace

extern "C" int eas_split_tf32(const float* src, float* dst, uint32_t rows, uint32_t kp, uint64_t ld_src,
                              uint32_t rows_valid, uint32_t k_valid, uint32_t batch, uint64_t bs_src, int transpose,
                              void* stream) {
  if (!src || !dst) return eas_fail(EAS_ERR_VALUE, "eas_split_tf32: null pointer");
  if (rows == 0 || kp == 0 || batch == 0) return EAS_OK;
  if (kp % 4 || (reinterpret_cast<uintptr_t>(dst) & 15))
    return eas_fail(EAS_ERR_VALUE, "eas_split_tf32: kp must be a multiple of 4 and dst 16-byte aligned");
  if (rows_valid > rows || k_valid > kp) return eas_fail(EAS_ERR_VALUE, "eas_split_tf32: valid extents exceed rows/kp");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const unsigned gz = batch < 65535u ? batch : 65535u;
  if (transpose) {
    const unsigned gy = (rows + 31) / 32 < 65535u ? (rows + 31) / 32 : 65535u;
    split_cols_kernel<<<dim3((kp + 63) / 64, gy, gz), 256, 0, s>>>(src, dst, rows, kp, ld_src, rows_valid, k_valid,
                                                                   batch, bs_src);
  } else {
    const unsigned gy = rows < 65535u ? rows : 65535u;
    split_rows_kernel<<<dim3((kp / 4 + 255) / 256, gy, gz), 256, 0, s>>>(src, dst, rows, kp, ld_src, rows_valid,
                                                                         k_valid, batch, bs_src);
  }
  return eas_cuda_check(cudaGetLastError(), "split_tf32 launch", EAS_ERR_LAUNCH);
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
  cast_f32_f16_kernel<float><<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      src, static_cast<uint16_t*>(dst), rows, cols_pad / 8, ld_src, ld_dst, rows_valid, cols_valid, batch, bs_src,
      bs_dst);
  return eas_cuda_check(cudaGetLastError(), "cast_f32_f16 launch", EAS_ERR_LAUNCH);
}

extern "C" int eas_pad_f16_2d(const void* src, void* dst, uint32_t rows, uint32_t cols_pad, uint64_t ld_src,
                              uint64_t ld_dst, uint32_t rows_valid, uint32_t cols_valid, uint32_t batch,
                              uint64_t bs_src, uint64_t bs_dst, void* stream) {
  if (!src || !dst) return eas_fail(EAS_ERR_VALUE, "eas_pad_f16_2d: null pointer");
  if (rows == 0 || cols_pad == 0 || batch == 0) return EAS_OK;
  if (reinterpret_cast<uintptr_t>(src) & 1) return eas_fail(EAS_ERR_VALUE, "eas_pad_f16_2d: source not 2-byte aligned");
  if (cols_pad % 8 || ld_dst % 8 || ld_dst < cols_pad || (batch > 1 && bs_dst % 8) ||
      (reinterpret_cast<uintptr_t>(dst) & 15))
    return eas_fail(EAS_ERR_VALUE, "eas_pad_f16_2d: destination rows must be 16-byte aligned");
  if (cols_valid > cols_pad) return eas_fail(EAS_ERR_VALUE, "eas_pad_f16_2d: cols_valid exceeds cols_pad");
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const uint64_t total = (uint64_t)batch * rows * (cols_pad / 8);
  const uint64_t want = (total + 255) / 256;
  const unsigned grid = (unsigned)(want < (uint64_t)sms * 16 ? want : (uint64_t)sms * 16);
  cast_f32_f16_kernel<uint16_t><<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(src), static_cast<uint16_t*>(dst), rows, cols_pad / 8, ld_src, ld_dst, rows_valid,
      cols_valid, batch, bs_src, bs_dst);
  return eas_cuda_check(cudaGetLastError(), "pad_f16 launch", EAS_ERR_LAUNCH);
}
