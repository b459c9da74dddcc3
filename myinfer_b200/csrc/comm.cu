// Communicators of a multi-GPU model (tensor parallel for dense layers,
// expert parallel for MoE layers): NCCL over NVLink / NVSwitch, one
// communicator per rank, all calls stream-ordered so they can be captured in
// the decode step's CUDA graph together with the kernels.
#include <algorithm>
#include <cstring>
#include <vector>

#include "comm.cuh"
#include "ops.cuh"

#if defined(M5_HAVE_NCCL)
#include <nccl.h>
#endif

namespace m5 {

// One-shot all-reduce over NVLink peer memory for decode-sized vectors.
//
// Every rank owns a receive area [2][nranks][kArMax] fp32 plus nranks flag
// words, mapped into every other rank with CUDA IPC (plain peer loads and
// stores, no multicast).  A call pushes this rank's partial into slot `rank`
// of every rank's area (buffer epoch & 1), fences, and the last CTA to finish
// pushing raises flag[rank] = epoch on every rank; each CTA then waits for all
// flags of this epoch and sums the slots in rank order (the same order on
// every rank, so all ranks hold bit-identical sums) straight into the bf16
// residual stream.  A rank can run at most one call ahead of another (it
// waits for everybody's flag), so two buffers keep a fast rank's next push
// off the slots a slow rank is still reading.  Waits are bounded (~2 s of
// wall time); a timeout records a device error and the call completes.
constexpr int kArMaxRanks = 8;
constexpr int64_t kArMax = 1 << 17;  // floats per slot (decode and short chunks)
constexpr int kArThreads = 256;
constexpr int kArMaxCtas = 32;       // always co-resident: waits never block a pusher

struct ArPeers {
  float* recv[kArMaxRanks];      // each rank's receive area
  uint32_t* flags[kArMaxRanks];  // each rank's flag words
};

static __device__ int g_ar_err = 0;

#if defined(M5_HAVE_NCCL)
struct Comm {
  ncclComm_t nccl = nullptr;
  int nranks = 1, rank = 0;
  // peer-memory all-reduce (null when the peers are not reachable by IPC)
  char* sym = nullptr;                       // local [2][nranks][kArMax] fp32 + [nranks] u32 flags
  void* peer_base[kArMaxRanks] = {nullptr};  // opened IPC mappings (self: sym)
  ArPeers peers{};
  uint32_t* d_state = nullptr;               // epoch, arrival count, done count
};

static int nccl_fail(ncclResult_t r, const char* what) {
  return fail(M5_ERR_COMM, std::string(what) + ": " + ncclGetErrorString(r));
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint64_t ar_now() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// h[i] = bf16(h[i] + bf16(sum over ranks of partial[i])), i < n.
__global__ void __launch_bounds__(kArThreads) ar_residual_kernel(const float* __restrict__ partial, bf16* h, int n,
                                                                 int nranks, int rank, ArPeers peers,
                                                                 uint32_t* state) {
  __shared__ uint32_t s_epoch;
  __shared__ int s_last;
  const int tid = threadIdx.x;
  if (tid == 0) s_epoch = *reinterpret_cast<volatile uint32_t*>(&state[0]) + 1;
  __syncthreads();
  const uint32_t epoch = s_epoch;
  const int buf = epoch & 1;
  const int n4 = n >> 2;
  const float4* src = reinterpret_cast<const float4*>(partial);
  // push this rank's partial into slot `rank` of every rank
  for (int p = 0; p < nranks; ++p) {
    float4* dst = reinterpret_cast<float4*>(peers.recv[p] + (size_t(buf) * nranks + rank) * kArMax);
    for (int i = blockIdx.x * kArThreads + tid; i < n4; i += gridDim.x * kArThreads) dst[i] = src[i];
  }
  __threadfence_system();
  __syncthreads();
  if (tid == 0) s_last = atomicAdd(&state[1], 1u) == gridDim.x - 1;
  __syncthreads();
  if (s_last && tid < nranks) {
    if (tid == 0) state[1] = 0;
    __threadfence_system();
    st_release_sys(peers.flags[tid] + rank, epoch);  // "my slot on your side holds epoch"
  }
  // wait for every rank's slot of this epoch (bounded)
  if (tid < nranks) {
    const uint32_t* f = peers.flags[rank] + tid;
    const uint64_t t0 = ar_now();
    for (uint32_t k = 0; ld_acquire_sys(f) < epoch; ++k) {
      if ((k & 255) == 255 && ar_now() - t0 > 2000000000ull) {
        atomicExch(&g_ar_err, 1);
        break;
      }
    }
  }
  __syncthreads();
  const float* mine = peers.recv[rank] + size_t(buf) * nranks * kArMax;
  for (int i = blockIdx.x * kArThreads + tid; i < n4; i += gridDim.x * kArThreads) {
    // L2-only loads: a line of this buffer read two calls ago must not be served from L1
    float4 acc = __ldcg(reinterpret_cast<const float4*>(mine) + i);
    for (int p = 1; p < nranks; ++p) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(mine + size_t(p) * kArMax) + i);
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    __nv_bfloat162* hp = reinterpret_cast<__nv_bfloat162*>(h + 4 * size_t(i));
    const __nv_bfloat162 h0 = hp[0], h1 = hp[1];
    hp[0] = __floats2bfloat162_rn(__low2float(h0) + rbf(acc.x), __high2float(h0) + rbf(acc.y));
    hp[1] = __floats2bfloat162_rn(__low2float(h1) + rbf(acc.z), __high2float(h1) + rbf(acc.w));
  }
  __syncthreads();
  if (tid == 0 && atomicAdd(&state[2], 1u) == gridDim.x - 1) {
    state[2] = 0;
    *reinterpret_cast<volatile uint32_t*>(&state[0]) = epoch;  // the next call uses epoch + 1
  }
}

// IPC-mapped receive areas of every rank; leaves c->sym null (NCCL fallback)
// when the peers cannot be mapped.
static void ar_setup(Comm* c) {
  if (c->nranks < 2 || c->nranks > kArMaxRanks) return;
  const size_t bytes = size_t(2) * c->nranks * kArMax * sizeof(float) + 256;
  char* sym = nullptr;
  if (cudaMalloc(&sym, bytes) != cudaSuccess) return;
  cudaMemset(sym, 0, bytes);
  cudaIpcMemHandle_t mine;
  if (cudaIpcGetMemHandle(&mine, sym) != cudaSuccess) {
    cudaFree(sym);
    cudaGetLastError();
    return;
  }
  // exchange the handles (and a reachability vote) through NCCL
  char* dev = nullptr;
  const size_t hb = sizeof(cudaIpcMemHandle_t);
  if (cudaMalloc(&dev, hb * (c->nranks + 1)) != cudaSuccess) {
    cudaFree(sym);
    return;
  }
  cudaMemcpy(dev + hb * c->nranks, &mine, hb, cudaMemcpyHostToDevice);
  std::vector<cudaIpcMemHandle_t> all(c->nranks);
  bool ok = ncclAllGather(dev + hb * c->nranks, dev, hb, ncclChar, c->nccl, 0) == ncclSuccess &&
            cudaStreamSynchronize(0) == cudaSuccess &&
            cudaMemcpy(all.data(), dev, hb * c->nranks, cudaMemcpyDeviceToHost) == cudaSuccess;
  cudaFree(dev);
  for (int p = 0; ok && p < c->nranks; ++p) {
    if (p == c->rank) {
      c->peer_base[p] = sym;
      continue;
    }
    void* base = nullptr;
    if (cudaIpcOpenMemHandle(&base, all[p], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      cudaGetLastError();
      ok = false;
      break;
    }
    c->peer_base[p] = base;
  }
  // every rank must agree before any of them uses peer memory
  int vote = ok ? 1 : 0, *dvote = nullptr;
  if (cudaMalloc(&dvote, sizeof(int)) == cudaSuccess) {
    cudaMemcpy(dvote, &vote, sizeof(int), cudaMemcpyHostToDevice);
    ok = ncclAllReduce(dvote, dvote, 1, ncclInt, ncclMin, c->nccl, 0) == ncclSuccess &&
         cudaStreamSynchronize(0) == cudaSuccess && cudaMemcpy(&vote, dvote, sizeof(int), cudaMemcpyDeviceToHost) ==
                                                        cudaSuccess &&
         vote == 1;
    cudaFree(dvote);
  } else {
    ok = false;
  }
  if (ok && cudaMalloc(&c->d_state, 4 * sizeof(uint32_t)) == cudaSuccess) {
    cudaMemset(c->d_state, 0, 4 * sizeof(uint32_t));
    c->sym = sym;
    for (int p = 0; p < c->nranks; ++p) {
      c->peers.recv[p] = static_cast<float*>(c->peer_base[p]);
      c->peers.flags[p] = reinterpret_cast<uint32_t*>(static_cast<char*>(c->peer_base[p]) +
                                                      size_t(2) * c->nranks * kArMax * sizeof(float));
    }
    return;
  }
  for (int p = 0; p < c->nranks; ++p)
    if (p != c->rank && c->peer_base[p]) cudaIpcCloseMemHandle(c->peer_base[p]);
  for (int p = 0; p < kArMaxRanks; ++p) c->peer_base[p] = nullptr;
  cudaFree(sym);
  cudaGetLastError();
}

static void ar_teardown(Comm* c) {
  if (!c->sym) return;
  cudaDeviceSynchronize();
  for (int p = 0; p < c->nranks; ++p)
    if (p != c->rank && c->peer_base[p]) cudaIpcCloseMemHandle(c->peer_base[p]);
  cudaFree(c->sym);
  cudaFree(c->d_state);
  c->sym = nullptr;
}

int comm_allreduce_residual(void* comm, float* partial, bf16* h, int64_t n, cudaStream_t st) {
  Comm* c = static_cast<Comm*>(comm);
  if (!c) return fail(M5_ERR_STATE, "allreduce: no communicator");
  if (n <= 0) return M5_OK;
  const bool peer_ok = c->sym && n <= kArMax && (n % 4) == 0 &&
                       (reinterpret_cast<uintptr_t>(partial) & 15) == 0 && (reinterpret_cast<uintptr_t>(h) & 7) == 0;
  if (!peer_ok) {
    int rc = comm_allreduce_f32(comm, partial, n, st);
    if (rc) return rc;
    return residual_add_f32_launch(h, partial, n, st);
  }
  const int ctas = (int)std::min<int64_t>(kArMaxCtas, std::max<int64_t>(1, (n / 4 + kArThreads - 1) / kArThreads));
  ar_residual_kernel<<<ctas, kArThreads, 0, st>>>(partial, h, (int)n, c->nranks, c->rank, c->peers, c->d_state);
  M5_LAUNCH_CHECK("peer all-reduce launch");
  return M5_OK;
}

int comm_ar_error(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_ar_err, sizeof(int)) != cudaSuccess) return -1;
  if (reset && v) {
    const int z = 0;
    cudaMemcpyToSymbol(g_ar_err, &z, sizeof(int));
  }
  return v;
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
int comm_allreduce_residual(void*, float*, bf16*, int64_t, cudaStream_t) {
  return fail(M5_ERR_UNSUPPORTED, "built without NCCL");
}
int comm_ar_error(int) { return 0; }
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
  const char* e = getenv("M5_PEER_ALLREDUCE");
  if (!(e && e[0] == '0')) ar_setup(c);
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
  ar_teardown(c);
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
