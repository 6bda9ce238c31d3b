// Runtime compilation helpers (see j4b_rtc.h).
#include <nvrtc.h>

#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "j4b_internal.h"
#include "j4b_rtc.h"

namespace j4b {

const Driver& driver() {
  static Driver d;
  static std::once_flag once;
  std::call_once(once, [] {
    auto get = [](const char* name, void** fn) {
      cudaDriverEntryPointQueryResult q;
      return cudaGetDriverEntryPointByVersion(name, fn, 12000, cudaEnableDefault, &q) == cudaSuccess &&
             q == cudaDriverEntryPointSuccess && *fn != nullptr;
    };
    d.ok = get("cuModuleLoadData", (void**)&d.ModuleLoadData) &&
           get("cuModuleGetFunction", (void**)&d.ModuleGetFunction) &&
           get("cuModuleUnload", (void**)&d.ModuleUnload) &&
           get("cuFuncSetAttribute", (void**)&d.FuncSetAttribute) &&
           get("cuOccupancyMaxActiveBlocksPerMultiprocessor", (void**)&d.Occupancy) &&
           get("cuLaunchKernel", (void**)&d.LaunchKernel) &&
           get("cuGetErrorName", (void**)&d.GetErrorName);
    if (!get("cuLaunchKernelEx", (void**)&d.LaunchKernelEx)) d.LaunchKernelEx = nullptr;
  });
  return d;
}

namespace {
std::mutex g_nvrtc_mu;
std::unordered_map<std::string, std::vector<char>>& cubin_cache() {
  static std::unordered_map<std::string, std::vector<char>> c;
  return c;
}
}  // namespace

int compile_source(const std::string& src, const char* name, std::vector<char>& cubin, bool contract_fma) {
  const std::string key = (contract_fma ? "F" : "N") + src;
  {
    std::lock_guard<std::mutex> lk(g_nvrtc_mu);
    auto it = cubin_cache().find(key);
    if (it != cubin_cache().end()) {
      cubin = it->second;
      return J4B_OK;
    }
  }
  nvrtcProgram prog;
  if (nvrtcCreateProgram(&prog, src.c_str(), name, 0, nullptr, nullptr) != NVRTC_SUCCESS)
    return set_error(J4B_ECUDA, "nvrtcCreateProgram failed");
  const char* opts[] = {"--gpu-architecture=sm_100a", "-std=c++17", contract_fma ? "--fmad=true" : "--fmad=false",
                        "-default-device", "-lineinfo"};
  nvrtcResult r = nvrtcCompileProgram(prog, 5, opts);
  if (r != NVRTC_SUCCESS) {
    size_t ls = 0;
    nvrtcGetProgramLogSize(prog, &ls);
    std::string log(ls, '\0');
    nvrtcGetProgramLog(prog, &log[0]);
    nvrtcDestroyProgram(&prog);
    return set_error(J4B_ECUDA, "%s compilation failed: %s", name, log.substr(0, 900).c_str());
  }
  size_t n = 0;
  nvrtcGetCUBINSize(prog, &n);
  cubin.resize(n);
  nvrtcGetCUBIN(prog, cubin.data());
  nvrtcDestroyProgram(&prog);
  counters().compilations++;
  std::lock_guard<std::mutex> lk(g_nvrtc_mu);
  cubin_cache()[key] = cubin;
  return J4B_OK;
}

int cu_error(CUresult r, const char* what) {
  const char* name = nullptr;
  if (driver().GetErrorName) driver().GetErrorName(r, &name);
  return set_error(J4B_ECUDA, "%s failed: %s (code %d)", what, name ? name : "?", (int)r);
}

}  // namespace j4b
