/*
 * eas_cuda.h — C ABI of libeas_cuda.so, the native device layer of easy_as_b200.
 *
 * The reference binds its device layer as the CPython extension `eas._metal`
 * (easy_as eas/runtime/_metal.mm, method table at _metal.mm:1436-1461; the
 * required subset is checked by eas/runtime/metal_ext.py:22-33).  This header
 * replaces that module with plain C entry points — pointers, sizes and status
 * codes, no Python or torch types — bound from Python with ctypes
 * (easy_as_b200/runtime/cuda_ext.py).  Each entry point names the `eas._metal`
 * method it replaces.
 *
 * Conventions
 *   - Every function returns an int status (EAS_OK == 0).  On failure
 *     eas_last_error() returns a thread-local, human-readable message.
 *   - Device pointers are CUdeviceptr values carried as void*.
 *   - `stream` is a cudaStream_t / CUstream (NULL = legacy default stream,
 *     which is also torch's default stream).
 *   - Nothing here traps, asserts or spins without bound on the device.
 */
#ifndef EAS_CUDA_H
#define EAS_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define EAS_OK 0
#define EAS_ERR_UNAVAILABLE 1 /* no driver, no device, or NVRTC missing           */
#define EAS_ERR_COMPILE 2     /* NVRTC rejected the source (log in last_error)     */
#define EAS_ERR_LAUNCH 3      /* launch or asynchronous kernel failure             */
#define EAS_ERR_VALUE 4       /* bad argument (sizes, dims, alignment)             */
#define EAS_ERR_MEMORY 5      /* allocation or copy failure                        */
#define EAS_ERR_INJECTED 6    /* failure injected by eas_fault_inject()            */
#define EAS_ERR_TIMEOUT 7     /* a bounded device-side wait gave up                */

/* ---- errors / availability -------------------------------------------- */

/* Message for the last failing call on this thread ("" if none). */
const char* eas_last_error(void);

/* 1 if a CUDA driver and at least one device are usable, else 0.
 * Replaces `eas._metal.is_available` (_metal.mm:168-183). */
int eas_is_available(void);

/* Device selection has no reference counterpart: the Metal extension uses one
 * process-wide device and queue (_metal.mm:141-166); here each rank or caller
 * picks one of the box's B200s. */

/* Number of visible CUDA devices. */
int eas_device_count(int* count);

/* Make `dev` current on this thread and initialise its primary context. */
int eas_set_device(int dev);

/* Compute capability of `dev` (e.g. 10, 0 for sm_100). */
int eas_device_capability(int dev, int* major, int* minor);

/* Runtime versions: CUDA driver, NVRTC major*1000+minor*10. */
int eas_versions(int* driver_version, int* nvrtc_version);

/* ---- compile (replaces `eas._metal.compile`, _metal.mm:185-260) ------- */

/* Compile CUDA C++ `src` with NVRTC for sm_100a and return a CUBIN image
 * (never PTX).  `opts` are extra NVRTC options.  The image is malloc'd and
 * must be released with eas_free_host().  On EAS_ERR_COMPILE the NVRTC log is
 * in eas_last_error(). */
int eas_compile(const char* src, const char* name, const char* const* opts, int nopts,
                void** image, size_t* image_size);

/* Frees an image returned by eas_compile (the Metal library object needs no
 * such call, _metal.mm:185-260). */
void eas_free_host(void* p);

/* Load a CUBIN on `dev` and resolve kernel `name`.  `max_dyn_smem` > 0 raises
 * the function's dynamic shared-memory limit (needed above 48 KiB).
 * Returns an opaque pipeline handle. */
int eas_pipeline_load(int dev, const void* image, size_t image_size, const char* name,
                      int max_dyn_smem, void** pipeline);

int eas_pipeline_free(void* pipeline);

/* Registers per thread / static shared bytes of a loaded pipeline. */
int eas_pipeline_attrs(void* pipeline, int* num_regs, int* static_smem, int* max_threads);

/* ---- launch (replaces `eas._metal.launch/launch_async`, _metal.mm:1013-1395) ---- */

/* Enqueue one launch.  `params` is a block holding the kernel's parameter
 * values; parameter i starts at byte offsets[i] (nparams entries, in the
 * kernel's declaration order).  Asynchronous: pair with
 * eas_stream_synchronize / events. */
int eas_launch(void* pipeline, const uint32_t grid[3], const uint32_t block[3], uint32_t dyn_smem,
               void* stream, const void* params, const uint32_t* offsets, uint32_t nparams);
/* eas_launch with programmatic dependent launch: the grid may be scheduled
 * while the previous kernel in the stream is finishing.  For kernels that begin
 * with griddepcontrol.wait (every generated kernel does), which holds them until
 * that grid has completed and its memory is visible; same arguments and errors
 * as eas_launch (falls back to it when the driver lacks cuLaunchKernelEx). */
int eas_launch_pdl(void* pipeline, const uint32_t grid[3], const uint32_t block[3], uint32_t dyn_smem,
               void* stream, const void* params, const uint32_t* offsets, uint32_t nparams);

/* ---- memory (replaces alloc_buffer / copy_from_host / copy_to_host,
 *      _metal.mm:262-455) -------------------------------------------------- */

int eas_alloc_buffer(int dev, size_t nbytes, void** dptr);
int eas_free_buffer(void* dptr);
/* host -> device; waits until the host buffer may be reused */
int eas_copy_from_host(void* dst, const void* src, size_t nbytes, void* stream);
/* device -> host; returns when `dst` holds the data */
int eas_copy_to_host(void* dst, const void* src, size_t nbytes, void* stream);
/* device -> device (same or peer device over NVLink), asynchronous */
int eas_copy_device(void* dst, const void* src, size_t nbytes, void* stream);
int eas_memset_d8(void* dst, int value, size_t nbytes, void* stream);
/* Asynchronous host <-> device copies for page-locked host memory: they return
 * at once; the host buffer must stay untouched until the stream reaches them. */
int eas_copy_from_host_async(void* dst, const void* src, size_t nbytes, void* stream);
int eas_copy_to_host_async(void* dst, const void* src, size_t nbytes, void* stream);
/* *pinned = 1 when `ptr` lies in page-locked host memory known to CUDA. */
int eas_host_is_pinned(const void* ptr, int* pinned);
/* Page-locked host memory (cudaHostAlloc, portable), for the runtime's bounce
 * buffer of small host-array launches: one asynchronous copy each way instead
 * of a synchronous copy per array (the reference passes host arrays to Metal
 * through temporary shared MTLBuffers, eas/runtime/metal.py:209-232
 * and :335-345). */
int eas_alloc_pinned(size_t nbytes, void** out);
int eas_free_pinned(void* p);
/* Device address of memory from eas_alloc_pinned (it is mapped): kernels of
 * elementwise launches read and write the bounce buffer in place over PCIe,
 * with no copies (each element is touched once). */
int eas_pinned_device_pointer(void* host, void** dev);

/* ---- synchronisation (replaces synchronize / queue_synchronize,
 *      _metal.mm:1397-1434) ------------------------------------------------ */

int eas_stream_synchronize(void* stream);
/* *capturing = 1 while `stream` is being captured into a CUDA graph. */
int eas_stream_is_capturing(void* stream, int* capturing);
int eas_device_synchronize(int dev);
int eas_stream_create(int dev, void** stream);
int eas_stream_destroy(void* stream);
int eas_event_create(void** event);
int eas_event_destroy(void* event);
int eas_event_record(void* event, void* stream);
/* Make `stream` wait (on the device) until `event` has completed. */
int eas_stream_wait_event(void* stream, void* event);
int eas_event_synchronize(void* event);
/* 1 if complete, 0 if pending */
int eas_event_query(void* event, int* done);
int eas_event_elapsed_ms(void* start, void* end, float* ms);

/* ---- native kernels (pattern-lowered DSL kernels) --------------------- */

/* Strided batched GEMM, f16 x f16 -> f32 accumulate -> f32, on tcgen05/TMEM
 * tensor cores (sm_100a).  Replaces the launch of the generated kernel for the
 * `mk.dot` GEMM pattern (reference: dot lowering eas/codegen/msl.py:920-952,
 * dispatched through eas._metal.launch, _metal.mm:1013-1222):
 *   C[b][m][n] = sum_{k<K} A[b][m][k] * B[b][k][n]
 *   A at a + b*a_bstride + m*lda + k                       (elements)
 *   B at b + b*b_bstride + k*ldb + n  (b_kmajor = 0)  or  + n*ldb + k  (1)
 *   C at c + b*c_bstride + m*ldc + n
 * A and B must be 16-byte aligned with strides that are multiples of 8
 * elements (TMA); otherwise EAS_ERR_VALUE (the caller then runs the generic
 * kernel).  block_n is the N tile (128 or 256); the library picks the rest
 * of the tile (eas_gemm_f16_tile with tile_m = 0).  Asynchronous on `stream`.
 * A pipeline wait that exceeds its budget ends the kernel early and is
 * reported by eas_gemm_status().  Launches that leave most SMs idle split K
 * into at most 2 parts by default (see eas_gemm_f16_plan), which keeps every
 * result bit-reproducible; EAS_GEMM_SPLITK=4 allows 4 parts, whose order of
 * summation (and so the last bits) may vary from run to run. */
int eas_gemm_f16(const void* a, const void* b, float* c, uint32_t M, uint32_t N, uint32_t K, uint32_t batch,
                 uint64_t lda, uint64_t a_bstride, uint64_t ldb, uint64_t b_bstride, int b_kmajor, uint64_t ldc,
                 uint64_t c_bstride, int block_n, void* stream);

/* eas_gemm_f16 with an explicit tile configuration: the native meaning of the
 * autotune space BLOCK_M x BLOCK_N x BLOCK_K of a DSL dot GEMM (the reference
 * times each Config and keeps the fastest, eas/kernel.py:73-127; its Metal
 * kernel uses the values as threadgroup tile sizes).
 *   tile_m  0: the library's choice (as eas_gemm_f16);
 *           128: the 1-SM kernel, output tile 128 x block_n;
 *           256: a CTA pair (tcgen05 cta_group::2, M = 256), each CTA staging
 *                block_n columns of B per k-block: pair tile 256 x 2*block_n
 *                (256 x 512 only when C is TMA-storable, else 256 x 256).
 *   block_k 0 or 64: one 64-deep k-block per pipeline stage; 128: two, with
 *           half as many stages in the same shared memory.
 * Every (tile_m, block_n, block_k) in {128, 256} x {128, 256} x {64, 128}
 * launches a different kernel.  Other values: EAS_ERR_VALUE. */
int eas_gemm_f16_tile(const void* a, const void* b, float* c, uint32_t M, uint32_t N, uint32_t K, uint32_t batch,
                      uint64_t lda, uint64_t a_bstride, uint64_t ldb, uint64_t b_bstride, int b_kmajor,
                      uint64_t ldc, uint64_t c_bstride, int tile_m, int block_n, int block_k, void* stream);

/* Strided batched fp32 GEMM with per-K-tile partial sums, true fp32 FFMA on
 * the CUDA cores.  Replaces the launch of the generated kernel for the
 * reference's fp32 tiled matmul (easy_as examples/matmul_tiled.py:134-230,
 * its dot groups lowered by eas/codegen/msl.py:1201-1359 and launched through
 * eas._metal.launch_tg, _metal.mm:1013-1222):
 *   for each K tile t of k_tile elements:
 *     p = fma(A[m][k], B[k][n], p) for k ascending in the tile, p from 0.0f
 *     acc = acc + p   (first tile: acc = 0.0f + p if zero_init, else acc = p)
 *   C[b][m][n] = acc
 *   A at a + b*a_bstride + m*lda + k, B at b + b*b_bstride + k*ldb + n,
 *   C at c + b*c_bstride + m*ldc + n   (elements)
 * A[m][k] reads as 0.0f unless m < a_rows and k < a_k, B[k][n] unless
 * k < b_k and n < b_cols (the DSL kernel's masked loads, which yield 0);
 * outputs m < M, n < N are stored.
 * The same operations in the same order as the generated kernel, so the
 * results are bit-identical.  K must be a multiple of k_tile and k_tile a
 * multiple of 8, operands 4-byte aligned; otherwise EAS_ERR_VALUE (16-byte
 * aligned rows take the vector path).  Asynchronous on `stream`. */
int eas_sgemm_f32_tiled(const float* a, const float* b, float* c, uint32_t M, uint32_t N, uint32_t K,
                        uint32_t k_tile, uint32_t batch, uint64_t lda, uint64_t a_bstride, uint64_t ldb,
                        uint64_t b_bstride, uint64_t ldc, uint64_t c_bstride, int zero_init,
                        uint32_t a_rows, uint32_t a_k, uint32_t b_cols, uint32_t b_k, void* stream);

/* f32 -> f16 operand staging (round to nearest even, cvt.rn.f16.f32, the cast
 * of the generated kernels) for the proven simdgroup-MMA GEMM of the
 * reference's matmul_simdgroup kernel (easy_as examples/matmul_simdgroup.py:
 * 29-127, whose tiles are cast to f16 in threadgroup memory before
 * simdgroup_multiply_accumulate, eas/codegen/msl.py:953-1002):
 *   dst[b][r][c] = (r < rows_valid && c < cols_valid) ? f16(src[b*bs_src + r*ld_src + c]) : 0
 * for r < rows, c < cols_pad.  cols_pad and ld_dst multiples of 8, dst
 * 16-byte aligned (bs_dst a multiple of 8 when batch > 1); otherwise
 * EAS_ERR_VALUE.  Asynchronous on `stream`. */
int eas_cast_f32_f16_2d(const float* src, void* dst, uint32_t rows, uint32_t cols_pad, uint64_t ld_src,
                        uint64_t ld_dst, uint32_t rows_valid, uint32_t cols_valid, uint32_t batch, uint64_t bs_src,
                        uint64_t bs_dst, void* stream);

/* f16 -> f16 re-pitching, the same layout rules as eas_cast_f32_f16_2d with an
 * f16 source (bits copied, zero outside the valid extent; source 2-byte
 * aligned, any pitch).  The runtime stages through it the operands of an fp16
 * `mk.dot` GEMM whose row pitch or base TMA cannot read in place (not a
 * multiple of 16 bytes), so the launch still runs on eas_gemm_f16_tile (the
 * reference has no such constraint: Metal kernels read any pitch,
 * msl.py:920-952). */
int eas_pad_f16_2d(const void* src, void* dst, uint32_t rows, uint32_t cols_pad, uint64_t ld_src, uint64_t ld_dst,
                   uint32_t rows_valid, uint32_t cols_valid, uint32_t batch, uint64_t bs_src, uint64_t bs_dst,
                   void* stream);

/* Self-test of the bounded waits of the native kernels (no counterpart in
 * the reference): launches one warp that waits, with the same bounded
 * mbarrier wait the GEMM uses, on a barrier that nothing ever completes.  The
 * wait gives up after budget_cycles (1 .. the kernels' own budget of 4e9
 * cycles), the kernel sets EAS_ERR_TIMEOUT in the device's status word and
 * returns; read it with eas_gemm_status after the stream synchronised.
 * Nothing faults or hangs; the context stays usable.  Asynchronous. */
int eas_wait_selftest(long long budget_cycles, void* stream);

/* What eas_gemm_f16_tile (tile_m, block_n, block_k; tile_m = block_k = 0 is
 * eas_gemm_f16) would launch, without a device: the CTA-pair or 1-SM kernel
 * (*pair), the output tile (out_tile_m x out_tile_n per CTA pair or CTA),
 * pipeline stages, split-K parts and the K depth of a stage (out_block_k),
 * for a C that TMA can store (c_tma_ok: 16-byte aligned base and strides) on
 * a GPU with num_sms SMs of which resident_pairs CTA pairs are co-resident
 * (cudaOccupancyMaxActiveClusters).  Composes the same rules the launcher
 * applies (no reference counterpart). */
int eas_gemm_f16_plan(uint32_t M, uint32_t N, uint32_t K, uint32_t batch, int block_n, int tile_m, int block_k,
                      int c_tma_ok, int num_sms, int resident_pairs, int* out_tile_m, int* out_tile_n, int* stages,
                      int* ksplit, int* pair, int* out_block_k);

/* Tile configuration the most recent eas_gemm_* launch in this process used:
 * output tile (tile_m x tile_n per CTA, or per CTA pair when *pair is 1),
 * pipeline stages, split-K parts and K depth of a stage.  Reporting only (no
 * reference counterpart). */
int eas_gemm_last_config(int* tile_m, int* tile_n, int* stages, int* ksplit, int* pair, int* block_k);

/* Strided batched GEMM on tcgen05 with TF32 operands (kind::tf32, f32
 * accumulate): C[b][m][n] = sum_k A[b][m][k] * B[b][n][k] with A at
 * a + b*a_bstride + m*lda + k and B K-major at b + b*b_bstride + n*ldb + k
 * (f32 storage; the tensor core reads the TF32 part, the 19 high bits).  Used
 * by the opt-in 3xTF32 mode of proven fp32 matmuls (north_star: 3xTF32 where
 * it meets rtol 1e-4) over operands from eas_split3_tf32.  Alignment and
 * status as eas_gemm_f16 (strides multiples of 4 elements). */
int eas_gemm_tf32(const float* a, const float* b, float* c, uint32_t M, uint32_t N, uint32_t K, uint32_t batch,
                  uint64_t lda, uint64_t a_bstride, uint64_t ldb, uint64_t b_bstride, uint64_t ldc,
                  uint64_t c_bstride, int block_n, void* stream);

/* 3xTF32 on tcgen05: the same kernel as eas_gemm_tf32 over operands from
 * eas_split_tf32, whose rows are [hi | lo] segments of K elements each (K a
 * multiple of 32; lda, ldb >= 2K).  The kernel runs 3K/32 k-blocks:
 * C = A_hi.B_hi + A_hi.B_lo + A_lo.B_hi (f32 accumulate).  With eas_split_tf32
 * it is the opt-in alternative to eas_sgemm_f32_tiled for a launch of the
 * reference's fp32 tiled matmul (examples/matmul_tiled.py:134-230, dot groups
 * msl.py:1201-1359). */
int eas_gemm_3xtf32(const float* a2, const float* b2, float* c, uint32_t M, uint32_t N, uint32_t K, uint32_t batch,
                    uint64_t lda, uint64_t a_bstride, uint64_t ldb, uint64_t b_bstride, uint64_t ldc,
                    uint64_t c_bstride, int block_n, void* stream);

/* 3xTF32 operand staging: each value x splits into hi = tf32(x) and
 * lo = tf32(x - hi) (round to nearest, ties away from zero; x - hi is exact).
 * Row r of the source (transpose = 0: src[r][k], row pitch ld_src) or column r
 * (transpose = 1: src[k][r]) becomes dst row r = [hi | lo], each segment kp
 * elements (kp a multiple of 4; dst 16-byte aligned, dense
 * [batch][rows][2*kp]); zero outside r < rows_valid, k < k_valid. */
int eas_split_tf32(const float* src, float* dst, uint32_t rows, uint32_t kp, uint64_t ld_src, uint32_t rows_valid,
                   uint32_t k_valid, uint32_t batch, uint64_t bs_src, int transpose, void* stream);

/* Read and clear the status word of native kernels on `dev` (0 = ok,
 * EAS_ERR_TIMEOUT = a bounded wait expired).  Valid after the stream synced.
 * The nearest reference analogue is the command-buffer status check after a
 * Metal dispatch (_metal.mm:1206-1217); Metal kernels have no bounded waits. */
int eas_gemm_status(int dev, int* code);

/* Allocation-free form of eas_gemm_f16, for callers that cannot let a library
 * allocate memory: code that owns every allocation in its process (its own
 * device allocator or a fixed memory budget), or code that must not allocate
 * at the point where it launches work.  No counterpart in the reference.
 *
 * Same arguments as eas_gemm_f16, and the same sums, but it launches only the
 * 1-SM kernels (128 x block_n tiles, one k-block per stage), never the CTA-pair
 * or 256 x 512 tiles that eas_gemm_f16 takes for M > 128: slower on large
 * shapes, and the results agree with eas_gemm_f16 to f32 rounding, not bit for
 * bit (the tensor core may sum a different tile shape in another order).
 * eas_gemm_f16_plan and eas_gemm_last_config do not describe its launch
 * choice beyond that.  The kernel's only scratch, one
 * 4-byte status word, lives in a file-scope __device__ array of this library
 * (one word per GPU that loads it, held until the process exits) instead of
 * memory allocated on first use; this call never calls cudaMalloc, cudaFree
 * or cudaHostAlloc.  Any size within the limits of eas_gemm_f16 fits (M, N,
 * K and batch each below 2^31); larger values are rejected with
 * EAS_ERR_VALUE.
 *
 * The first call on a device looks the word's device address up
 * (cudaGetSymbolAddress) with that device current; make that first call
 * before any stream capture.  Every call clears the word, then runs the
 * kernel.  All calls on a device share the word, so calls that overlap on the
 * GPU race on it.  The stream must belong to the current device (the word is
 * looked up for the current device).  With status_out != NULL the call
 * copies the word out and synchronises the stream, then stores the status
 * there (0 = ok, EAS_ERR_TIMEOUT = a bounded wait expired).  With NULL it
 * returns at once and the status is lost: nothing reads the word back, and
 * the next call clears it, so a wait that expired then goes unreported and C
 * may be incomplete.  Pass status_out wherever the result matters. */
int eas_gemm_f16_noalloc(const void* a, const void* b, float* c, uint32_t M, uint32_t N, uint32_t K,
                         uint32_t batch, uint64_t lda, uint64_t a_bstride, uint64_t ldb, uint64_t b_bstride,
                         int b_kmajor, uint64_t ldc, uint64_t c_bstride, int block_n, void* stream,
                         int* status_out);

/* ---- host-side fault injection (tests; no device fault is ever made; no
 *      counterpart in the reference) ---------------------------------------- */

/* Make the `nth` (1-based) next call of kind "compile", "alloc", "launch" or
 * "copy" fail with EAS_ERR_INJECTED.  nth <= 0 clears the injection. */
int eas_fault_inject(const char* kind, int nth);

#ifdef __cplusplus
}
#endif

#endif /* EAS_CUDA_H */
