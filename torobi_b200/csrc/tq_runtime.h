// Host-side runtime shared by every entry point of libtorobi_b200: status
// codes and the thread-local last-error message, the per-device status word
// kernels report lost waits into, and TMA tensor-map encoding.
#pragma once

#include <cstdarg>
#include <cstdint>
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

}  // namespace tq
