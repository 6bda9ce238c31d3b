// Runtime compilation shared by the code-generating engines (fused tapes, scalar-AAD replay):
// driver entry points resolved through the runtime, and NVRTC compilation of generated CUDA C
// to an sm_100a cubin with a process-wide cache keyed by the exact source text.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include <string>
#include <vector>

namespace j4b {

// Driver entry points, resolved through the runtime so the library loads on machines without
// a driver (CPU build and planning checks). `ok` is false when any of them is missing.
struct Driver {
  PFN_cuModuleLoadData_v2000 ModuleLoadData = nullptr;
  PFN_cuModuleGetFunction_v2000 ModuleGetFunction = nullptr;
  PFN_cuModuleUnload_v2000 ModuleUnload = nullptr;
  PFN_cuFuncSetAttribute_v9000 FuncSetAttribute = nullptr;
  PFN_cuOccupancyMaxActiveBlocksPerMultiprocessor_v6050 Occupancy = nullptr;
  PFN_cuLaunchKernel_v4000 LaunchKernel = nullptr;
  PFN_cuLaunchKernelEx_v11060 LaunchKernelEx = nullptr;  // optional: programmatic dependent launch
  PFN_cuGetErrorName_v6000 GetErrorName = nullptr;
  bool ok = false;
};
const Driver& driver();

// Compiles `src` for sm_100a; `name` labels the program in compiler messages. Without
// `contract_fma` no multiply-add is fused, so generated arithmetic rounds exactly as written
// (what the fused tapes need to reproduce the reference's float results). Cached by source
// text and option.
int compile_source(const std::string& src, const char* name, std::vector<char>& cubin,
                   bool contract_fma = false);

// Sets the last error from a driver status and returns J4B_ECUDA.
int cu_error(CUresult r, const char* what);

}  // namespace j4b
