// Host-side kernel launch with programmatic stream serialization (PDL).
// Set B200_PDL=0 in the environment to launch without the attribute.
#pragma once

#include <cuda_runtime.h>

#include <cstdlib>
#include <map>
#include <mutex>
#include <stdexcept>
#include <string>

namespace b200 {

inline bool pdl_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("B200_PDL");
    v = (e != nullptr && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

// Raise a kernel's dynamic shared-memory limit on the current device, once per
// (kernel, device): the attribute belongs to each device's context, so a
// process that drives several GPUs sets it on every one. Thread-safe; a failed
// call throws instead of surfacing later as a launch error.
inline std::mutex& smem_attr_mutex() {
  static std::mutex m;
  return m;
}
inline std::map<std::pair<const void*, int>, size_t>& smem_attr_done() {
  static std::map<std::pair<const void*, int>, size_t> m;
  return m;
}
template <typename... KArgs>
inline void ensure_smem(void (*kern)(KArgs...), size_t bytes) {
  if (bytes <= 48 * 1024) return;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) throw std::runtime_error("b200: cudaGetDevice failed");
  std::lock_guard<std::mutex> lk(smem_attr_mutex());
  auto key = std::make_pair(reinterpret_cast<const void*>(kern), dev);
  auto& done = smem_attr_done();
  auto it = done.find(key);
  if (it != done.end() && it->second >= bytes) return;
  const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e != cudaSuccess)
    throw std::runtime_error(std::string("b200: cannot raise the shared-memory limit: ") + cudaGetErrorString(e));
  done[key] = bytes;
}

template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
  if (e != cudaSuccess) throw std::runtime_error(std::string("b200: kernel launch failed: ") + cudaGetErrorString(e));
}

}  // namespace b200
