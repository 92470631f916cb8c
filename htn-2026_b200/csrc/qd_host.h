// Host-side helpers shared by the C-ABI translation units.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/qd_decode.h"

namespace qd {

// Record a message for qd_last_error() (thread-local) and return `code`.
int set_error(int code, const char* fmt, ...);
// SM count of the current device (cached per device).
int host_sm_count();
// cudaLaunchKernelEx of a kernel whose only parameter is the struct at `arg`; `pdl` adds the
// programmatic-stream-serialization attribute so the kernel may start before its predecessor ends.
int launch_kernel(const void* func, dim3 grid, dim3 block, int smem, int pdl, cudaStream_t stream, void* arg);
// Raise `func`'s dynamic shared memory limit to at least `smem` bytes on the current device. The
// attribute belongs to the device's context, so the largest value set so far is remembered per
// (kernel, device) pair, under a lock: a process that drives several GPUs sets it on each of them.
int set_max_dynamic_smem(const void* func, int smem);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// cuTensorMapEncodeTiled through the runtime's driver entry point (looked up once): the library needs no
// link-time dependency on the driver library, so it loads on hosts without a GPU. Null if unavailable.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

}  // namespace qd
