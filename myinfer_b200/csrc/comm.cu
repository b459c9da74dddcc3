// Communicators of a multi-GPU model (tensor parallel for dense layers,
// expert parallel for MoE layers): NCCL over NVLink / NVSwitch, one
// communicator per rank, all calls stream-ordered so they can be captured in
// the decode step's CUDA graph together with the kernels.
#include <cstring>

#include "comm.cuh"

#if defined(M5_HAVE_NCCL)
#include <nccl.h>
#endif

namespace m5 {

#if defined(M5_HAVE_NCCL)
struct Comm {
  ncclComm_t nccl = nullptr;
  int nranks = 1, rank = 0;
};

static int nccl_fail(ncclResult_t r, const char* what) {
  return fail(M5_ERR_COMM, std::string(what) + ": " + ncclGetErrorString(r));
}

int comm_allreduce_f32(void* comm, float* buf, int64_t n, cudaStream_t st) {
  Comm* c = static_cast<Comm*>(comm);
  if (!c) return fail(M5_ERR_STATE, "allreduce: no communicator");
  if (n <= 0 || c->nranks == 1) return M5_OK;
  ncclResult_t r = ncclAllReduce(buf, buf, size_t(n), ncclFloat, ncclSum, c->nccl, st);
  return r == ncclSuccess ? M5_OK : nccl_fail(r, "ncclAllReduce");
}

int comm_allgather_bf16(void* comm, const bf16* send, bf16* recv, int64_t n, cudaStream_t st) {
  Comm* c = static_cast<Comm*>(comm);
  if (!c) return fail(M5_ERR_STATE, "allgather: no communicator");
  if (n <= 0) return M5_OK;
  ncclResult_t r = ncclAllGather(send, recv, size_t(n), ncclBfloat16, c->nccl, st);
  return r == ncclSuccess ? M5_OK : nccl_fail(r, "ncclAllGather");
}

int comm_size(void* comm) { return comm ? static_cast<Comm*>(comm)->nranks : 1; }
int comm_rank(void* comm) { return comm ? static_cast<Comm*>(comm)->rank : 0; }

#else
int comm_allreduce_f32(void*, float*, int64_t, cudaStream_t) {
  return fail(M5_ERR_UNSUPPORTED, "built without NCCL");
}
int comm_allgather_bf16(void*, const bf16*, bf16*, int64_t, cudaStream_t) {
  return fail(M5_ERR_UNSUPPORTED, "built without NCCL");
}
int comm_size(void*) { return 1; }
int comm_rank(void*) { return 0; }
#endif

}  // namespace m5

using namespace m5;

extern "C" int m5_comm_unique_id(void* out, size_t len) {
  M5_CHECK_ARG(out && len >= M5_COMM_ID_BYTES, "m5_comm_unique_id: buffer must hold M5_COMM_ID_BYTES");
#if defined(M5_HAVE_NCCL)
  static_assert(sizeof(ncclUniqueId) <= M5_COMM_ID_BYTES, "NCCL unique id larger than M5_COMM_ID_BYTES");
  ncclUniqueId id;
  ncclResult_t r = ncclGetUniqueId(&id);
  if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
  memset(out, 0, len);
  memcpy(out, &id, sizeof(id));
  return M5_OK;
#else
  return fail(M5_ERR_UNSUPPORTED, "m5_comm_unique_id: built without NCCL");
#endif
}

extern "C" int m5_comm_init(const void* id, size_t len, int nranks, int rank, void** comm) {
  M5_CHECK_ARG(id && comm && len >= M5_COMM_ID_BYTES, "m5_comm_init: bad argument");
  M5_CHECK_ARG(nranks >= 1 && rank >= 0 && rank < nranks, "m5_comm_init: rank out of range");
#if defined(M5_HAVE_NCCL)
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  Comm* c = new Comm();
  c->nranks = nranks;
  c->rank = rank;
  ncclResult_t r = ncclCommInitRank(&c->nccl, nranks, uid, rank);
  if (r != ncclSuccess) {
    delete c;
    return nccl_fail(r, "ncclCommInitRank");
  }
  *comm = c;
  return M5_OK;
#else
  return fail(M5_ERR_UNSUPPORTED, "m5_comm_init: built without NCCL");
#endif
}

extern "C" int m5_comm_destroy(void* comm) {
#if defined(M5_HAVE_NCCL)
  Comm* c = static_cast<Comm*>(comm);
  if (!c) return M5_OK;
  ncclResult_t r = ncclCommDestroy(c->nccl);
  delete c;
  return r == ncclSuccess ? M5_OK : nccl_fail(r, "ncclCommDestroy");
#else
  (void)comm;
  return M5_OK;
#endif
}

extern "C" int m5_allreduce_f32(void* comm, float* buf, int64_t n, void* stream) {
  M5_CHECK_ARG(comm && (buf || n == 0) && n >= 0, "m5_allreduce_f32: bad argument");
  return comm_allreduce_f32(comm, buf, n, (cudaStream_t)stream);
}
