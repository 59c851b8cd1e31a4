// cast_f16.cu — f32 -> f16 operand staging for the proven simdgroup-MMA GEMM.
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
