// Data-parallel plumbing: one NCCL communicator per process (one process per
// GPU), and the allreduce of the flattened LoRA gradient buffer.
#include <nccl.h>

#include <cstring>

#include "tq_runtime.h"

namespace {

int check_nccl(ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return TQ_OK;
  return tq::fail(TQ_ERR_NCCL, "%s: %s", what, ncclGetErrorString(r));
}

}  // namespace

extern "C" int tq_dp_unique_id(void* id128) {
  static_assert(sizeof(ncclUniqueId) == 128, "NCCL unique id is 128 bytes");
  if (!id128) return tq::fail(TQ_ERR_INVALID, "null id buffer");
  ncclUniqueId id;
  int rc = check_nccl(ncclGetUniqueId(&id), "ncclGetUniqueId");
  if (rc) return rc;
  memcpy(id128, &id, sizeof(id));
  return TQ_OK;
}

extern "C" int tq_dp_comm_init(void** comm, const void* id128, int nranks, int rank) {
  if (!comm || !id128) return tq::fail(TQ_ERR_INVALID, "null pointer");
  if (nranks < 1 || rank < 0 || rank >= nranks)
    return tq::fail(TQ_ERR_INVALID, "rank %d of %d is not a valid rank", rank, nranks);
  ncclUniqueId id;
  memcpy(&id, id128, sizeof(id));
  ncclComm_t c = nullptr;
  int rc = check_nccl(ncclCommInitRank(&c, nranks, id, rank), "ncclCommInitRank");
  if (rc) return rc;
  *comm = c;
  return TQ_OK;
}

extern "C" int tq_dp_allreduce_sum(void* comm, void* buf, int64_t count, int dtype, void* stream) {
  if (!comm) return tq::fail(TQ_ERR_INVALID, "null communicator");
  if (count < 0) return tq::fail(TQ_ERR_INVALID, "negative count");
  if (count == 0) return TQ_OK;
  if (!buf) return tq::fail(TQ_ERR_INVALID, "null buffer");
  ncclDataType_t t;
  if (dtype == TQ_DTYPE_F32) t = ncclFloat32;
  else if (dtype == TQ_DTYPE_BF16) t = ncclBfloat16;
  else return tq::fail(TQ_ERR_UNSUPPORTED, "dtype %d is not f32 or bf16", dtype);
  return check_nccl(ncclAllReduce(buf, buf, static_cast<size_t>(count), t, ncclSum,
                                  static_cast<ncclComm_t>(comm), tq::as_stream(stream)),
                    "ncclAllReduce");
}

extern "C" int tq_dp_comm_destroy(void* comm) {
  if (!comm) return TQ_OK;
  return check_nccl(ncclCommDestroy(static_cast<ncclComm_t>(comm)), "ncclCommDestroy");
}

// After a lost rank: frees the communicator without waiting for its peers
// (ncclCommDestroy may wait on operations a dead peer never completes).
extern "C" int tq_dp_comm_abort(void* comm) {
  if (!comm) return TQ_OK;
  return check_nccl(ncclCommAbort(static_cast<ncclComm_t>(comm)), "ncclCommAbort");
}

// The communicator's asynchronous error state (ncclCommGetAsyncError): the
// host polls it, with the collective's completion, while it waits for a
// collective under a deadline.
extern "C" int tq_dp_comm_async_error(void* comm, int* nccl_result) {
  if (!comm || !nccl_result) return tq::fail(TQ_ERR_INVALID, "null pointer");
  ncclResult_t r = ncclSuccess;
  const int rc = check_nccl(ncclCommGetAsyncError(static_cast<ncclComm_t>(comm), &r),
                            "ncclCommGetAsyncError");
  if (rc) return rc;
  *nccl_result = static_cast<int>(r);
  return TQ_OK;
}
