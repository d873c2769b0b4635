// Host-side runtime shared by every entry point of libtorobi_b200: status
// codes and the thread-local last-error message, the per-device status word
// kernels report lost waits into, and TMA tensor-map encoding.
#pragma once

#include <cstdarg>
#include <cstdint>
#include <utility>
#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/torobi_b200.h"

namespace tq {

// Records a formatted message as this thread's last error and returns `code`.
int fail(int code, const char* fmt, ...);

// Returns TQ_OK, or TQ_ERR_CUDA with the message recorded.
int check_cuda(cudaError_t e, const char* what);

// The per-device status word kernels OR kDevTimeout into.  Resolved once per
// device (with that device current) through cudaGetSymbolAddress.
int* device_status_ptr(int* err_code);

// Encodes a 2D/3D tiled tensor map.  dims/strides innermost first; strides in
// bytes for dims 1.. (dim 0 is contiguous).  Returns TQ_OK or an error.
int encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                CUtensorMapSwizzle swizzle);

inline bool aligned(const void* p, uintptr_t a) {
  return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0;
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Number of SMs of the current device (cached per device).
int sm_count();

// Raises a kernel's dynamic shared-memory limit on the current device, once
// per (kernel, device): later calls return at once, so a launch inside a
// stream capture makes no attribute call.
int set_max_smem_once(const void* func, int bytes, const char* what);

// Whether kernels of the training step are launched with programmatic
// stream serialization (read once per process; TQ_PDL=0 turns it off).
bool pdl_enabled();

// Launches `kernel` on `stream`, in clusters of shape `cluster` when that
// holds more than one CTA, and -- when pdl_enabled() -- allowed to start before the
// previous kernel on the stream has finished: its CTAs may be scheduled once
// every CTA of that kernel has signalled (griddep_launch_dependents) or
// exited, and must call griddep_wait before touching global memory.
template <typename... KArgs, typename... Args>
int launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                  cudaStream_t stream, dim3 cluster, const char* what, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (cluster.x * cluster.y * cluster.z > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster.x;
    attr[n].val.clusterDim.y = cluster.y;
    attr[n].val.clusterDim.z = cluster.z;
    ++n;
  }
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return check_cuda(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...), what);
}

}  // namespace tq
