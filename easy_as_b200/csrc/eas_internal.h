// eas_internal.h — declarations shared by the .cu files of libeas_cuda.so.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/eas_cuda.h"

// Driver-API entry points resolved at runtime (no link against libcuda).
struct DriverApi {
  decltype(&::cuModuleLoadData) moduleLoadData = nullptr;
  decltype(&::cuModuleUnload) moduleUnload = nullptr;
  decltype(&::cuModuleGetFunction) moduleGetFunction = nullptr;
  decltype(&::cuLaunchKernel) launchKernel = nullptr;
  decltype(&::cuFuncSetAttribute) funcSetAttribute = nullptr;
  decltype(&::cuFuncGetAttribute) funcGetAttribute = nullptr;
  decltype(&::cuGetErrorString) getErrorString = nullptr;
  decltype(&::cuTensorMapEncodeTiled) tensorMapEncodeTiled = nullptr;
  decltype(&::cuFuncGetParamInfo) funcGetParamInfo = nullptr;  // optional (driver >= 12.4)
  decltype(&::cuLaunchKernelEx) launchKernelEx = nullptr;      // optional: programmatic dependent launch
};
extern DriverApi g_drv;

int eas_driver_init();
int eas_fail(int code, const char* fmt, ...);
int eas_cuda_check(cudaError_t e, const char* what, int code);
int eas_drv_check(CUresult r, const char* what, int code);

// Device address of this device's native-kernel status word (host-mapped, read and cleared by
// eas_gemm_status); kernels write EAS_ERR_TIMEOUT there when a bounded wait expires.
int* eas_native_status_dev(int dev);
