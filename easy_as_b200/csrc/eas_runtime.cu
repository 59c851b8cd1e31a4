// eas_runtime.cu — libeas_cuda.so: NVRTC compile, module cache, launch,
// memory, streams/events for easy_as_b200.  C ABI declared in include/eas_cuda.h.
//
// Design
//  * The CUDA runtime is linked statically; it loads the driver lazily, so the
//    library itself loads on a machine without a GPU (the CPU test suite
//    checks every exported symbol).
//  * Driver-API entry points (module load, cuLaunchKernel, function
//    attributes) are fetched with cudaGetDriverEntryPointByVersion, so there
//    is no link-time dependency on libcuda.
//  * NVRTC is opened with dlopen at the first compile.
//  * One primary context per device, shared with torch.
//
// Replaces the reference's ObjC++ Metal module (easy_as eas/runtime/_metal.mm).
#include <cuda.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nvrtc.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "eas_internal.h"

// ---------------------------------------------------------------------------
// errors
// ---------------------------------------------------------------------------

static thread_local std::string g_last_error;

int eas_fail(int code, const char* fmt, ...) {
  char buf[2048];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

static void set_error_string(int code, const std::string& msg) {
  (void)code;
  g_last_error = msg;
}

int eas_cuda_check(cudaError_t e, const char* what, int code) {
  if (e == cudaSuccess) return EAS_OK;
  cudaGetLastError();  // clear the sticky-free error state
  return eas_fail(code, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

extern "C" const char* eas_last_error(void) { return g_last_error.c_str(); }

// ---------------------------------------------------------------------------
// host-side fault injection
// ---------------------------------------------------------------------------

namespace {
enum FaultKind { kCompile = 0, kAlloc, kLaunch, kCopy, kNumKinds };
std::atomic<int> g_fault_countdown[kNumKinds];

int fault_kind(const char* kind) {
  if (!kind) return -1;
  if (!strcmp(kind, "compile")) return kCompile;
  if (!strcmp(kind, "alloc")) return kAlloc;
  if (!strcmp(kind, "launch")) return kLaunch;
  if (!strcmp(kind, "copy")) return kCopy;
  return -1;
}

// true when this call must fail (the countdown reaches zero)
bool fault_hit(int kind) {
  int v = g_fault_countdown[kind].load();
  while (v > 0) {
    if (g_fault_countdown[kind].compare_exchange_weak(v, v - 1)) return v == 1;
  }
  return false;
}

struct FaultEnvInit {
  // EAS_FAULT_INJECT="launch:3,alloc:1"
  FaultEnvInit() {
    const char* env = getenv("EAS_FAULT_INJECT");
    if (!env) return;
    std::string s(env);
    size_t pos = 0;
    while (pos < s.size()) {
      size_t end = s.find(',', pos);
      if (end == std::string::npos) end = s.size();
      std::string item = s.substr(pos, end - pos);
      size_t colon = item.find(':');
      if (colon != std::string::npos) {
        int k = fault_kind(item.substr(0, colon).c_str());
        if (k >= 0) g_fault_countdown[k] = atoi(item.c_str() + colon + 1);
      }
      pos = end + 1;
    }
  }
} g_fault_env_init;
}  // namespace

extern "C" int eas_fault_inject(const char* kind, int nth) {
  int k = fault_kind(kind);
  if (k < 0) return eas_fail(EAS_ERR_VALUE, "eas_fault_inject: unknown kind '%s'", kind ? kind : "(null)");
  g_fault_countdown[k] = nth > 0 ? nth : 0;
  return EAS_OK;
}

#define EAS_INJECT(kind, what)                                                  \
  do {                                                                          \
    if (fault_hit(kind)) return eas_fail(EAS_ERR_INJECTED, "%s: injected failure", what); \
  } while (0)

// ---------------------------------------------------------------------------
// driver entry points
// ---------------------------------------------------------------------------

DriverApi g_drv;
static std::once_flag g_drv_once;
static int g_drv_status = EAS_ERR_UNAVAILABLE;
static std::string g_drv_error;

template <typename F>
static bool fetch(const char* sym, F& out) {
  void* fp = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPointByVersion(sym, &fp, 12000, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || fp == nullptr) {
    cudaGetLastError();
    return false;
  }
  out = reinterpret_cast<F>(fp);
  return true;
}

int eas_driver_init() {
  std::call_once(g_drv_once, [] {
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) {
      g_drv_error = std::string("no usable CUDA driver/device: ") + cudaGetErrorString(e);
      cudaGetLastError();
      return;
    }
    if (n <= 0) {
      g_drv_error = "no CUDA device visible";
      return;
    }
    bool ok = fetch("cuModuleLoadData", g_drv.moduleLoadData) &&
              fetch("cuModuleUnload", g_drv.moduleUnload) &&
              fetch("cuModuleGetFunction", g_drv.moduleGetFunction) &&
              fetch("cuLaunchKernel", g_drv.launchKernel) &&
              fetch("cuFuncSetAttribute", g_drv.funcSetAttribute) &&
              fetch("cuFuncGetAttribute", g_drv.funcGetAttribute) &&
              fetch("cuGetErrorString", g_drv.getErrorString) &&
              fetch("cuTensorMapEncodeTiled", g_drv.tensorMapEncodeTiled);
    if (!ok) {
      g_drv_error = "could not resolve CUDA driver entry points";
      return;
    }
    fetch("cuFuncGetParamInfo", g_drv.funcGetParamInfo);
    fetch("cuLaunchKernelEx", g_drv.launchKernelEx);
    g_drv_status = EAS_OK;
  });
  if (g_drv_status != EAS_OK) return eas_fail(g_drv_status, "%s", g_drv_error.c_str());
  return EAS_OK;
}

int eas_drv_check(CUresult r, const char* what, int code) {
  if (r == CUDA_SUCCESS) return EAS_OK;
  const char* s = nullptr;
  if (g_drv.getErrorString) g_drv.getErrorString(r, &s);
  return eas_fail(code, "%s: %s (CUresult %d)", what, s ? s : "unknown error", (int)r);
}

extern "C" int eas_is_available(void) { return eas_driver_init() == EAS_OK ? 1 : 0; }

extern "C" int eas_device_count(int* count) {
  if (!count) return eas_fail(EAS_ERR_VALUE, "eas_device_count: null pointer");
  *count = 0;
  int rc = eas_driver_init();
  if (rc) return rc;
  return eas_cuda_check(cudaGetDeviceCount(count), "cudaGetDeviceCount", EAS_ERR_UNAVAILABLE);
}

static std::atomic<uint64_t> g_ctx_ready{0};  // bit d: primary context of device d initialised

extern "C" int eas_set_device(int dev) {
  int rc = eas_driver_init();
  if (rc) return rc;
  int cur = -1;
  if (cudaGetDevice(&cur) != cudaSuccess || cur != dev) {
    rc = eas_cuda_check(cudaSetDevice(dev), "cudaSetDevice", EAS_ERR_VALUE);
    if (rc) return rc;
  }
  uint64_t bit = (dev >= 0 && dev < 64) ? (1ull << dev) : 0;
  if (!bit || !(g_ctx_ready.load() & bit)) {
    rc = eas_cuda_check(cudaFree(nullptr), "primary context init", EAS_ERR_UNAVAILABLE);
    if (rc) return rc;
    g_ctx_ready.fetch_or(bit);
  }
  return EAS_OK;
}

extern "C" int eas_device_capability(int dev, int* major, int* minor) {
  int rc = eas_driver_init();
  if (rc) return rc;
  rc = eas_cuda_check(cudaDeviceGetAttribute(major, cudaDevAttrComputeCapabilityMajor, dev), "capability",
                      EAS_ERR_VALUE);
  if (rc) return rc;
  return eas_cuda_check(cudaDeviceGetAttribute(minor, cudaDevAttrComputeCapabilityMinor, dev), "capability",
                        EAS_ERR_VALUE);
}

// ---------------------------------------------------------------------------
// NVRTC
// ---------------------------------------------------------------------------

namespace {
struct Nvrtc {
  decltype(&nvrtcCreateProgram) create = nullptr;
  decltype(&nvrtcCompileProgram) compile = nullptr;
  decltype(&nvrtcGetProgramLogSize) log_size = nullptr;
  decltype(&nvrtcGetProgramLog) log = nullptr;
  decltype(&nvrtcGetCUBINSize) cubin_size = nullptr;
  decltype(&nvrtcGetCUBIN) cubin = nullptr;
  decltype(&nvrtcDestroyProgram) destroy = nullptr;
  decltype(&nvrtcVersion) version = nullptr;
  decltype(&nvrtcGetErrorString) errstr = nullptr;
};
Nvrtc g_nvrtc;
std::once_flag g_nvrtc_once;
int g_nvrtc_status = EAS_ERR_UNAVAILABLE;
std::string g_nvrtc_error;

int nvrtc_init() {
  std::call_once(g_nvrtc_once, [] {
    const char* names[] = {"libnvrtc.so.12", "libnvrtc.so"};
    void* h = nullptr;
    for (const char* n : names) {
      h = dlopen(n, RTLD_NOW | RTLD_LOCAL);
      if (h) break;
    }
    if (!h) {
      g_nvrtc_error = std::string("cannot load NVRTC (libnvrtc.so.12): ") + dlerror();
      return;
    }
#define EAS_SYM(field, sym)                                              \
  g_nvrtc.field = reinterpret_cast<decltype(g_nvrtc.field)>(dlsym(h, sym)); \
  if (!g_nvrtc.field) {                                                  \
    g_nvrtc_error = "NVRTC symbol missing: " sym;                        \
    return;                                                              \
  }
    EAS_SYM(create, "nvrtcCreateProgram");
    EAS_SYM(compile, "nvrtcCompileProgram");
    EAS_SYM(log_size, "nvrtcGetProgramLogSize");
    EAS_SYM(log, "nvrtcGetProgramLog");
    EAS_SYM(cubin_size, "nvrtcGetCUBINSize");
    EAS_SYM(cubin, "nvrtcGetCUBIN");
    EAS_SYM(destroy, "nvrtcDestroyProgram");
    EAS_SYM(version, "nvrtcVersion");
    EAS_SYM(errstr, "nvrtcGetErrorString");
#undef EAS_SYM
    g_nvrtc_status = EAS_OK;
  });
  if (g_nvrtc_status != EAS_OK) return eas_fail(g_nvrtc_status, "%s", g_nvrtc_error.c_str());
  return EAS_OK;
}
}  // namespace

extern "C" int eas_versions(int* driver_version, int* nvrtc_version) {
  if (driver_version) {
    *driver_version = 0;
    cudaDriverGetVersion(driver_version);
    cudaGetLastError();
  }
  if (nvrtc_version) {
    *nvrtc_version = 0;
    if (nvrtc_init() == EAS_OK) {
      int mj = 0, mn = 0;
      g_nvrtc.version(&mj, &mn);
      *nvrtc_version = mj * 1000 + mn * 10;
    }
  }
  return EAS_OK;
}

extern "C" int eas_compile(const char* src, const char* name, const char* const* opts, int nopts, void** image,
                           size_t* image_size) {
  if (!src || !image || !image_size) return eas_fail(EAS_ERR_VALUE, "eas_compile: null argument");
  *image = nullptr;
  *image_size = 0;
  EAS_INJECT(kCompile, "eas_compile");
  int rc = nvrtc_init();
  if (rc) return rc;
  nvrtcProgram prog;
  nvrtcResult r = g_nvrtc.create(&prog, src, name ? name : "eas_kernel.cu", 0, nullptr, nullptr);
  if (r != NVRTC_SUCCESS) return eas_fail(EAS_ERR_COMPILE, "nvrtcCreateProgram: %s", g_nvrtc.errstr(r));
  std::vector<const char*> all = {"--gpu-architecture=sm_100a", "--std=c++17", "--fmad=false",
                                  "--device-as-default-execution-space"};
  for (int i = 0; i < nopts; ++i) all.push_back(opts[i]);
  r = g_nvrtc.compile(prog, (int)all.size(), all.data());
  size_t log_n = 0;
  g_nvrtc.log_size(prog, &log_n);
  std::string log(log_n, '\0');
  if (log_n) g_nvrtc.log(prog, &log[0]);
  if (r != NVRTC_SUCCESS) {
    g_nvrtc.destroy(&prog);
    set_error_string(EAS_ERR_COMPILE, std::string("CUDA compile failed (NVRTC): ") + g_nvrtc.errstr(r) + "\n" + log);
    return EAS_ERR_COMPILE;
  }
  size_t n = 0;
  r = g_nvrtc.cubin_size(prog, &n);
  if (r != NVRTC_SUCCESS || n == 0) {
    g_nvrtc.destroy(&prog);
    return eas_fail(EAS_ERR_COMPILE, "nvrtcGetCUBINSize failed");
  }
  void* buf = malloc(n);
  if (!buf) {
    g_nvrtc.destroy(&prog);
    return eas_fail(EAS_ERR_MEMORY, "out of host memory for CUBIN");
  }
  r = g_nvrtc.cubin(prog, (char*)buf);
  g_nvrtc.destroy(&prog);
  if (r != NVRTC_SUCCESS) {
    free(buf);
    return eas_fail(EAS_ERR_COMPILE, "nvrtcGetCUBIN failed");
  }
  *image = buf;
  *image_size = n;
  return EAS_OK;
}

extern "C" void eas_free_host(void* p) { free(p); }

// ---------------------------------------------------------------------------
// pipelines
// ---------------------------------------------------------------------------

namespace {
struct Pipeline {
  int dev;
  CUmodule mod;
  CUfunction fn;
  int nparams;  // -1 when the driver cannot report it
};

int count_params(CUfunction fn) {
  if (!g_drv.funcGetParamInfo) return -1;
  for (int i = 0; i < 4096; ++i) {
    size_t off = 0, size = 0;
    if (g_drv.funcGetParamInfo(fn, (size_t)i, &off, &size) != CUDA_SUCCESS) return i;
  }
  return -1;
}
}  // namespace

extern "C" int eas_pipeline_load(int dev, const void* image, size_t image_size, const char* name, int max_dyn_smem,
                                 void** pipeline) {
  (void)image_size;
  if (!image || !name || !pipeline) return eas_fail(EAS_ERR_VALUE, "eas_pipeline_load: null argument");
  int rc = eas_set_device(dev);
  if (rc) return rc;
  CUmodule mod;
  rc = eas_drv_check(g_drv.moduleLoadData(&mod, image), "cuModuleLoadData", EAS_ERR_COMPILE);
  if (rc) return rc;
  CUfunction fn;
  rc = eas_drv_check(g_drv.moduleGetFunction(&fn, mod, name), "cuModuleGetFunction", EAS_ERR_COMPILE);
  if (rc) {
    g_drv.moduleUnload(mod);
    return rc;
  }
  if (max_dyn_smem > 0) {
    rc = eas_drv_check(g_drv.funcSetAttribute(fn, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, max_dyn_smem),
                       "cuFuncSetAttribute(max dynamic smem)", EAS_ERR_VALUE);
    if (rc) {
      g_drv.moduleUnload(mod);
      return rc;
    }
  }
  *pipeline = new Pipeline{dev, mod, fn, count_params(fn)};
  return EAS_OK;
}

extern "C" int eas_pipeline_free(void* pipeline) {
  if (!pipeline) return EAS_OK;
  Pipeline* p = static_cast<Pipeline*>(pipeline);
  if (g_drv.moduleUnload) g_drv.moduleUnload(p->mod);
  delete p;
  return EAS_OK;
}

extern "C" int eas_pipeline_attrs(void* pipeline, int* num_regs, int* static_smem, int* max_threads) {
  if (!pipeline) return eas_fail(EAS_ERR_VALUE, "eas_pipeline_attrs: null pipeline");
  Pipeline* p = static_cast<Pipeline*>(pipeline);
  int rc = EAS_OK;
  if (num_regs) rc |= eas_drv_check(g_drv.funcGetAttribute(num_regs, CU_FUNC_ATTRIBUTE_NUM_REGS, p->fn), "attr", 4);
  if (static_smem)
    rc |= eas_drv_check(g_drv.funcGetAttribute(static_smem, CU_FUNC_ATTRIBUTE_SHARED_SIZE_BYTES, p->fn), "attr", 4);
  if (max_threads)
    rc |= eas_drv_check(g_drv.funcGetAttribute(max_threads, CU_FUNC_ATTRIBUTE_MAX_THREADS_PER_BLOCK, p->fn),
                        "attr", 4);
  return rc ? EAS_ERR_VALUE : EAS_OK;
}

namespace {
int launch_impl(bool pdl, void* pipeline, const uint32_t grid[3], const uint32_t block[3], uint32_t dyn_smem,
                void* stream, const void* params, const uint32_t* offsets, uint32_t nparams) {
  if (!pipeline || !grid || !block) return eas_fail(EAS_ERR_VALUE, "eas_launch: null argument");
  if (nparams && (!params || !offsets)) return eas_fail(EAS_ERR_VALUE, "eas_launch: null parameter block");
  if (nparams > 256) return eas_fail(EAS_ERR_VALUE, "eas_launch: %u parameters (max 256)", nparams);
  EAS_INJECT(kLaunch, "eas_launch");
  Pipeline* p = static_cast<Pipeline*>(pipeline);
  if (p->nparams >= 0 && (uint32_t)p->nparams != nparams)
    return eas_fail(EAS_ERR_VALUE, "eas_launch: kernel takes %d parameters, %u given", p->nparams, nparams);
  if (block[0] * block[1] * block[2] > 1024u || block[0] == 0)
    return eas_fail(EAS_ERR_VALUE, "eas_launch: block (%u,%u,%u) exceeds 1024 threads", block[0], block[1], block[2]);
  if (grid[1] > 65535u || grid[2] > 65535u)
    return eas_fail(EAS_ERR_VALUE, "eas_launch: grid.y/z (%u,%u) exceed 65535", grid[1], grid[2]);
  if (grid[0] == 0 || grid[1] == 0 || grid[2] == 0) return EAS_OK;
  void* argv[256];
  for (uint32_t i = 0; i < nparams; ++i) argv[i] = const_cast<char*>(static_cast<const char*>(params) + offsets[i]);
  if (pdl && g_drv.launchKernelEx) {
    // programmatic stream serialisation: the grid may be scheduled while the previous kernel in the
    // stream finishes; the kernel's griddepcontrol.wait holds it until that grid has completed
    CUlaunchAttribute attr[1];
    attr[0].id = CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION;
    attr[0].value.programmaticStreamSerializationAllowed = 1;
    CUlaunchConfig cfg = {};
    cfg.gridDimX = grid[0];
    cfg.gridDimY = grid[1];
    cfg.gridDimZ = grid[2];
    cfg.blockDimX = block[0];
    cfg.blockDimY = block[1];
    cfg.blockDimZ = block[2];
    cfg.sharedMemBytes = dyn_smem;
    cfg.hStream = (CUstream)stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    CUresult r = g_drv.launchKernelEx(&cfg, p->fn, nparams ? argv : nullptr, nullptr);
    return eas_drv_check(r, "cuLaunchKernelEx", EAS_ERR_LAUNCH);
  }
  CUresult r = g_drv.launchKernel(p->fn, grid[0], grid[1], grid[2], block[0], block[1], block[2], dyn_smem,
                                  (CUstream)stream, nparams ? argv : nullptr, nullptr);
  return eas_drv_check(r, "cuLaunchKernel", EAS_ERR_LAUNCH);
}
}  // namespace

extern "C" int eas_launch(void* pipeline, const uint32_t grid[3], const uint32_t block[3], uint32_t dyn_smem,
                          void* stream, const void* params, const uint32_t* offsets, uint32_t nparams) {
  return launch_impl(false, pipeline, grid, block, dyn_smem, stream, params, offsets, nparams);
}

extern "C" int eas_launch_pdl(void* pipeline, const uint32_t grid[3], const uint32_t block[3], uint32_t dyn_smem,
                              void* stream, const void* params, const uint32_t* offsets, uint32_t nparams) {
  return launch_impl(true, pipeline, grid, block, dyn_smem, stream, params, offsets, nparams);
}

// ---------------------------------------------------------------------------
// memory
// ---------------------------------------------------------------------------

extern "C" int eas_alloc_buffer(int dev, size_t nbytes, void** dptr) {
  if (!dptr) return eas_fail(EAS_ERR_VALUE, "eas_alloc_buffer: null pointer");
  *dptr = nullptr;
  EAS_INJECT(kAlloc, "eas_alloc_buffer");
  int rc = eas_set_device(dev);
  if (rc) return rc;
  void* p = nullptr;
  rc = eas_cuda_check(cudaMalloc(&p, nbytes ? nbytes : 1), "cudaMalloc", EAS_ERR_MEMORY);
  if (rc) return rc;
  *dptr = p;
  return EAS_OK;
}

extern "C" int eas_free_buffer(void* dptr) {
  if (!dptr) return EAS_OK;
  return eas_cuda_check(cudaFree(dptr), "cudaFree", EAS_ERR_MEMORY);
}

extern "C" int eas_copy_from_host(void* dst, const void* src, size_t nbytes, void* stream) {
  EAS_INJECT(kCopy, "eas_copy_from_host");
  if (!nbytes) return EAS_OK;
  int rc = eas_cuda_check(cudaMemcpyAsync(dst, src, nbytes, cudaMemcpyHostToDevice, (cudaStream_t)stream),
                          "copy host->device", EAS_ERR_MEMORY);
  if (rc) return rc;
  // the source may be pageable host memory that the caller reuses at once
  return eas_cuda_check(cudaStreamSynchronize((cudaStream_t)stream), "copy host->device (sync)", EAS_ERR_MEMORY);
}

extern "C" int eas_copy_to_host(void* dst, const void* src, size_t nbytes, void* stream) {
  EAS_INJECT(kCopy, "eas_copy_to_host");
  if (!nbytes) return EAS_OK;
  int rc = eas_cuda_check(cudaMemcpyAsync(dst, src, nbytes, cudaMemcpyDeviceToHost, (cudaStream_t)stream),
                          "copy device->host", EAS_ERR_MEMORY);
  if (rc) return rc;
  return eas_cuda_check(cudaStreamSynchronize((cudaStream_t)stream), "copy device->host (sync)", EAS_ERR_MEMORY);
}

extern "C" int eas_copy_device(void* dst, const void* src, size_t nbytes, void* stream) {
  EAS_INJECT(kCopy, "eas_copy_device");
  if (!nbytes) return EAS_OK;
  return eas_cuda_check(cudaMemcpyAsync(dst, src, nbytes, cudaMemcpyDefault, (cudaStream_t)stream),
                        "copy device->device", EAS_ERR_MEMORY);
}

extern "C" int eas_copy_from_host_async(void* dst, const void* src, size_t nbytes, void* stream) {
  EAS_INJECT(kCopy, "eas_copy_from_host_async");
  if (!nbytes) return EAS_OK;
  return eas_cuda_check(cudaMemcpyAsync(dst, src, nbytes, cudaMemcpyHostToDevice, (cudaStream_t)stream),
                        "copy host->device (async)", EAS_ERR_MEMORY);
}

extern "C" int eas_copy_to_host_async(void* dst, const void* src, size_t nbytes, void* stream) {
  EAS_INJECT(kCopy, "eas_copy_to_host_async");
  if (!nbytes) return EAS_OK;
  return eas_cuda_check(cudaMemcpyAsync(dst, src, nbytes, cudaMemcpyDeviceToHost, (cudaStream_t)stream),
                        "copy device->host (async)", EAS_ERR_MEMORY);
}

extern "C" int eas_alloc_pinned(size_t nbytes, void** out) {
  if (!out) return eas_fail(EAS_ERR_VALUE, "eas_alloc_pinned: null out pointer");
  *out = nullptr;
  int rc = eas_driver_init();
  if (rc) return rc;
  return eas_cuda_check(cudaHostAlloc(out, nbytes ? nbytes : 1, cudaHostAllocPortable | cudaHostAllocMapped),
                        "pinned host allocation", EAS_ERR_MEMORY);
}

extern "C" int eas_pinned_device_pointer(void* host, void** dev) {
  if (!host || !dev) return eas_fail(EAS_ERR_VALUE, "eas_pinned_device_pointer: null pointer");
  *dev = nullptr;
  return eas_cuda_check(cudaHostGetDevicePointer(dev, host, 0), "device address of pinned host memory",
                        EAS_ERR_MEMORY);
}

extern "C" int eas_free_pinned(void* p) {
  if (!p) return EAS_OK;
  return eas_cuda_check(cudaFreeHost(p), "free pinned host memory", EAS_ERR_MEMORY);
}

extern "C" int eas_host_is_pinned(const void* ptr, int* pinned) {
  if (!pinned) return eas_fail(EAS_ERR_VALUE, "eas_host_is_pinned: null pointer");
  *pinned = 0;
  int rc = eas_driver_init();
  if (rc) return rc;
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, ptr) != cudaSuccess) {
    cudaGetLastError();
    return EAS_OK;
  }
  *pinned = at.type == cudaMemoryTypeHost ? 1 : 0;
  return EAS_OK;
}

extern "C" int eas_memset_d8(void* dst, int value, size_t nbytes, void* stream) {
  if (!nbytes) return EAS_OK;
  return eas_cuda_check(cudaMemsetAsync(dst, value, nbytes, (cudaStream_t)stream), "memset", EAS_ERR_MEMORY);
}

// ---------------------------------------------------------------------------
// streams / events
// ---------------------------------------------------------------------------

extern "C" int eas_stream_synchronize(void* stream) {
  return eas_cuda_check(cudaStreamSynchronize((cudaStream_t)stream), "kernel execution (stream sync)",
                        EAS_ERR_LAUNCH);
}

extern "C" int eas_stream_is_capturing(void* stream, int* capturing) {
  if (!capturing) return eas_fail(EAS_ERR_VALUE, "eas_stream_is_capturing: null pointer");
  cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
  int rc = eas_cuda_check(cudaStreamIsCapturing((cudaStream_t)stream, &st), "cudaStreamIsCapturing", EAS_ERR_VALUE);
  *capturing = (st == cudaStreamCaptureStatusActive) ? 1 : 0;
  return rc;
}

extern "C" int eas_device_synchronize(int dev) {
  int rc = eas_set_device(dev);
  if (rc) return rc;
  return eas_cuda_check(cudaDeviceSynchronize(), "kernel execution (device sync)", EAS_ERR_LAUNCH);
}

extern "C" int eas_stream_create(int dev, void** stream) {
  int rc = eas_set_device(dev);
  if (rc) return rc;
  cudaStream_t s;
  rc = eas_cuda_check(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreate", EAS_ERR_VALUE);
  if (rc) return rc;
  *stream = s;
  return EAS_OK;
}

extern "C" int eas_stream_destroy(void* stream) {
  if (!stream) return EAS_OK;
  return eas_cuda_check(cudaStreamDestroy((cudaStream_t)stream), "cudaStreamDestroy", EAS_ERR_VALUE);
}

extern "C" int eas_event_create(void** event) {
  cudaEvent_t e;
  int rc = eas_cuda_check(cudaEventCreate(&e), "cudaEventCreate", EAS_ERR_VALUE);
  if (rc) return rc;
  *event = e;
  return EAS_OK;
}

extern "C" int eas_event_destroy(void* event) {
  if (!event) return EAS_OK;
  return eas_cuda_check(cudaEventDestroy((cudaEvent_t)event), "cudaEventDestroy", EAS_ERR_VALUE);
}

extern "C" int eas_event_record(void* event, void* stream) {
  return eas_cuda_check(cudaEventRecord((cudaEvent_t)event, (cudaStream_t)stream), "cudaEventRecord",
                        EAS_ERR_LAUNCH);
}

extern "C" int eas_stream_wait_event(void* stream, void* event) {
  return eas_cuda_check(cudaStreamWaitEvent((cudaStream_t)stream, (cudaEvent_t)event, 0), "cudaStreamWaitEvent",
                        EAS_ERR_LAUNCH);
}

extern "C" int eas_event_synchronize(void* event) {
  return eas_cuda_check(cudaEventSynchronize((cudaEvent_t)event), "kernel execution (event sync)", EAS_ERR_LAUNCH);
}

extern "C" int eas_event_query(void* event, int* done) {
  cudaError_t e = cudaEventQuery((cudaEvent_t)event);
  if (e == cudaErrorNotReady) {
    cudaGetLastError();
    *done = 0;
    return EAS_OK;
  }
  *done = 1;
  return eas_cuda_check(e, "kernel execution (event query)", EAS_ERR_LAUNCH);
}

extern "C" int eas_event_elapsed_ms(void* start, void* end, float* ms) {
  return eas_cuda_check(cudaEventElapsedTime(ms, (cudaEvent_t)start, (cudaEvent_t)end), "cudaEventElapsedTime",
                        EAS_ERR_VALUE);
}
