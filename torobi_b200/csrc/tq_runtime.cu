// Runtime pieces shared by every entry point: error reporting, the device
// status word, tensor-map encoding.
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "tq_runtime.h"

namespace tq {

namespace {

thread_local char g_last_error[512] = "";

// Kernels OR kDevTimeout here.  One word per device (a __device__ variable
// has a separate instance on every device that loads the module).
__device__ int g_device_status = 0;

constexpr int kMaxDevices = 64;
int* g_status_ptr[kMaxDevices] = {};
int g_sm_count[kMaxDevices] = {};
std::mutex g_mu;

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

}  // namespace

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return TQ_OK;
  return fail(TQ_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int* device_status_ptr(int* err_code) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *err_code = fail(TQ_ERR_CUDA, "no current CUDA device");
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_status_ptr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_device_status);
    if (e != cudaSuccess) {
      *err_code = check_cuda(e, "cudaGetSymbolAddress(device status)");
      return nullptr;
    }
    g_status_ptr[dev] = static_cast<int*>(p);
  }
  *err_code = TQ_OK;
  return g_status_ptr[dev];
}

int set_max_smem_once(const void* func, int bytes, const char* what) {
  struct Entry {
    const void* func;
    int dev;
  };
  static Entry done[512];
  static int n_done = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(TQ_ERR_CUDA, "no current CUDA device");
  std::lock_guard<std::mutex> lock(g_mu);
  for (int i = 0; i < n_done; ++i)
    if (done[i].func == func && done[i].dev == dev) return TQ_OK;
  const int rc = check_cuda(
      cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes), what);
  if (rc) return rc;
  if (n_done < 512) done[n_done++] = Entry{func, dev};
  return TQ_OK;
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("TQ_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  if (!g_sm_count[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    g_sm_count[dev] = n;
  }
  return g_sm_count[dev];
}

static int get_encoder() {
  if (g_encode) return TQ_OK;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_encode) return TQ_OK;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
    return fail(TQ_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return TQ_OK;
}

int encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                CUtensorMapSwizzle swizzle) {
  int rc = get_encoder();
  if (rc) return rc;
  // The encoder is a driver call and needs a current context.  A host thread
  // whose first CUDA work is this call (e.g. a framework's backward worker,
  // which only selected the device) has none bound yet: binding the runtime's
  // context to the thread once is what every runtime call would do first.
  thread_local int bound_dev = -1;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(TQ_ERR_CUDA, "no current CUDA device");
  if (bound_dev != dev) {
    rc = check_cuda(cudaSetDevice(dev), "cudaSetDevice");
    if (rc) return rc;
    bound_dev = dev;
  }
  cuuint64_t gdim[5];
  cuuint64_t gstride[4];
  cuuint32_t bdim[5];
  cuuint32_t estride[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    estride[i] = 1;
  }
  for (int i = 0; i + 1 < rank; ++i) gstride[i] = strides_bytes[i];
  CUresult r = g_encode(map, dtype, static_cast<cuuint32_t>(rank), const_cast<void*>(base), gdim,
                        gstride, bdim, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(TQ_ERR_INVALID,
                "cuTensorMapEncodeTiled failed (%d): rank %d dims [%llu, %llu] box [%u, %u]",
                static_cast<int>(r), rank, (unsigned long long)dims[0],
                (unsigned long long)(rank > 1 ? dims[1] : 0), box[0], rank > 1 ? box[1] : 0);
  return TQ_OK;
}

}  // namespace tq

extern "C" {

int tq_version(void) { return 100; }

const char* tq_last_error(void) { return tq::g_last_error; }

int tq_device_status(int* status_out, int clear) {
  int rc = TQ_OK;
  int* p = tq::device_status_ptr(&rc);
  if (!p) return rc;
  int v = 0;
  rc = tq::check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  if (rc) return rc;
  rc = tq::check_cuda(cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost), "read status");
  if (rc) return rc;
  if (clear && v) {
    int zero = 0;
    rc = tq::check_cuda(cudaMemcpy(p, &zero, sizeof(int), cudaMemcpyHostToDevice), "clear status");
    if (rc) return rc;
  }
  if (status_out) *status_out = v;
  if (v & 1) return tq::fail(TQ_ERR_TIMEOUT, "a device-side wait ran out (status %d)", v);
  return TQ_OK;
}

}  // extern "C"
