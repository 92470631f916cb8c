// Library identification, error reporting and the shared launch helper.
#include <cstdarg>
#include <cstdio>
#include <map>
#include <mutex>
#include <utility>

#include "qd_host.h"

namespace qd {

static thread_local char g_msg[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return code;
}

int host_sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev >= 0 && dev < 64 && cached[dev] > 0) return cached[dev];
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  if (dev >= 0 && dev < 64) cached[dev] = n;
  return n;
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

int set_max_dynamic_smem(const void* func, int smem) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> done;  // (kernel, device) -> limit set
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(QD_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  std::lock_guard<std::mutex> lock(mu);
  int& have = done[std::make_pair(func, dev)];
  if (smem <= have) return QD_OK;
  e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return set_error(QD_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  have = smem;
  return QD_OK;
}

int launch_kernel(const void* func, dim3 grid, dim3 block, int smem, int pdl, cudaStream_t stream, void* arg) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  void* args[1] = {arg};
  cudaError_t e = cudaLaunchKernelExC(&cfg, func, args);
  if (e != cudaSuccess) return set_error(QD_ERR_CUDA, "launch: %s", cudaGetErrorString(e));
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(QD_ERR_CUDA, "launch: %s", cudaGetErrorString(e));
  return QD_OK;
}

}  // namespace qd

extern "C" const char* qd_version(void) { return "qd_decode 0.1 (sm_100a)"; }
extern "C" const char* qd_last_error(void) { return qd::g_msg; }
extern "C" int qd_sm_count(int* out) {
  if (!out) return qd::set_error(QD_ERR_ARG, "null out");
  *out = qd::host_sm_count();
  return QD_OK;
}
