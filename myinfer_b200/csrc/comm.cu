// Communicators of a multi-GPU model (tensor parallel for dense layers,
// expert parallel for MoE layers): NCCL over NVLink / NVSwitch, one
// communicator per rank, all calls stream-ordered so they can be captured in
// the decode step's CUDA graph together with the kernels.
#include <algorithm>
#include <chrono>
#include <cstring>
#include <thread>
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
// off the slots a slow rank is still reading.  Waits are bounded (2 s of
// wall time by default, m5_comm_set_wait_ms); a CTA whose wait runs out
// records a device error (m5_device_status), leaves its part of the residual
// stream untouched instead of adding slots that may be stale, and the call
// completes.
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
  uint64_t wait_ns = 2000000000ull;          // bound of the peer all-reduce's flag wait
  bool aborted = false;
};

static int nccl_fail(ncclResult_t r, const char* what) {
  return fail(M5_ERR_COMM, std::string(what) + ": " + ncclGetErrorString(r));
}

// The communicator is non-blocking: an NCCL call may return ncclInProgress
// while its work is still being set up.  Poll its state until it settles,
// for at most `timeout_s`; a communicator that does not settle (a rank that
// never joins, a peer that died) is aborted and reported as a timeout.
static int nccl_settle(Comm* c, ncclResult_t r, const char* what, double timeout_s) {
  if (r != ncclSuccess && r != ncclInProgress) return nccl_fail(r, what);
  if (r == ncclSuccess) return M5_OK;
  const auto t0 = std::chrono::steady_clock::now();
  ncclResult_t st = ncclInProgress;
  for (;;) {
    if (ncclCommGetAsyncError(c->nccl, &st) != ncclSuccess) return fail(M5_ERR_COMM, "ncclCommGetAsyncError failed");
    if (st != ncclInProgress) break;
    const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (el > timeout_s) {
      ncclCommAbort(c->nccl);
      c->aborted = true;
      return fail(M5_ERR_TIMEOUT, std::string(what) + ": did not complete within " + std::to_string(timeout_s) +
                                      " s (communicator aborted)");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
  return st == ncclSuccess ? M5_OK : nccl_fail(st, what);
}

static double env_seconds(const char* name, double dflt) {
  const char* e = getenv(name);
  if (!e || !*e) return dflt;
  const double v = atof(e);
  return v > 0 ? v : dflt;
}
// bound on setting up (and tearing down) a communicator, and on enqueueing a
// collective, in seconds
static double init_timeout_s() { return env_seconds("M5_COMM_INIT_TIMEOUT_S", 300.0); }
static double call_timeout_s() { return env_seconds("M5_COMM_CALL_TIMEOUT_S", 60.0); }

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
                                                                 uint32_t* state, uint64_t wait_ns) {
  __shared__ uint32_t s_epoch;
  __shared__ int s_last, s_timeout;
  const int tid = threadIdx.x;
  if (tid == 0) {
    s_epoch = *reinterpret_cast<volatile uint32_t*>(&state[0]) + 1;
    s_timeout = 0;
  }
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
      if ((k & 255) == 255 && ar_now() - t0 > wait_ns) {
        atomicExch(&g_ar_err, 1);
        s_timeout = 1;
        break;
      }
    }
  }
  __syncthreads();
  const float* mine = peers.recv[rank] + size_t(buf) * nranks * kArMax;
  const int n4_sum = s_timeout ? 0 : n4;  // a late rank's slot may hold an older partial: add nothing
  for (int i = blockIdx.x * kArThreads + tid; i < n4_sum; i += gridDim.x * kArThreads) {
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
  bool ok = nccl_settle(c, ncclAllGather(dev + hb * c->nranks, dev, hb, ncclChar, c->nccl, 0), "ncclAllGather",
                        init_timeout_s()) == M5_OK &&
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
    ok = nccl_settle(c, ncclAllReduce(dvote, dvote, 1, ncclInt, ncclMin, c->nccl, 0), "ncclAllReduce",
                     init_timeout_s()) == M5_OK &&
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
  ar_residual_kernel<<<ctas, kArThreads, 0, st>>>(partial, h, (int)n, c->nranks, c->rank, c->peers, c->d_state,
                                                  c->wait_ns);
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
  if (c->aborted) return fail(M5_ERR_STATE, "allreduce: the communicator was aborted");
  return nccl_settle(c, ncclAllReduce(buf, buf, size_t(n), ncclFloat, ncclSum, c->nccl, st), "ncclAllReduce",
                     call_timeout_s());
}

int comm_allgather_bf16(void* comm, const bf16* send, bf16* recv, int64_t n, cudaStream_t st) {
  Comm* c = static_cast<Comm*>(comm);
  if (!c) return fail(M5_ERR_STATE, "allgather: no communicator");
  if (n <= 0) return M5_OK;
  if (c->aborted) return fail(M5_ERR_STATE, "allgather: the communicator was aborted");
  return nccl_settle(c, ncclAllGather(send, recv, size_t(n), ncclBfloat16, c->nccl, st), "ncclAllGather",
                     call_timeout_s());
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
  // Non-blocking set-up, bounded: a rank that never joins ends in a timeout
  // and an aborted communicator instead of a process stuck in NCCL.
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclResult_t r = ncclCommInitRankConfig(&c->nccl, nranks, uid, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    if (c->nccl) ncclCommAbort(c->nccl);
    delete c;
    return nccl_fail(r, "ncclCommInitRankConfig");
  }
  if (int rc = nccl_settle(c, r, "ncclCommInitRankConfig", init_timeout_s())) {
    if (!c->aborted) ncclCommAbort(c->nccl);
    delete c;
    return rc;
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
  int rc = M5_OK;
  if (!c->aborted) {
    ncclResult_t r = ncclCommFinalize(c->nccl);
    rc = nccl_settle(c, r, "ncclCommFinalize", init_timeout_s());
    if (!c->aborted) {
      r = ncclCommDestroy(c->nccl);
      if (r != ncclSuccess && !rc) rc = nccl_fail(r, "ncclCommDestroy");
    }
  }
  delete c;
  return rc;
#else
  (void)comm;
  return M5_OK;
#endif
}

extern "C" int m5_allreduce_f32(void* comm, float* buf, int64_t n, void* stream) {
  M5_CHECK_ARG(comm && (buf || n == 0) && n >= 0, "m5_allreduce_f32: bad argument");
  return comm_allreduce_f32(comm, buf, n, (cudaStream_t)stream);
}

extern "C" int m5_comm_check(void* comm) {
  M5_CHECK_ARG(comm, "m5_comm_check: null communicator");
#if defined(M5_HAVE_NCCL)
  Comm* c = static_cast<Comm*>(comm);
  if (c->aborted) return fail(M5_ERR_STATE, "m5_comm_check: the communicator was aborted");
  ncclResult_t st = ncclSuccess;
  ncclResult_t r = ncclCommGetAsyncError(c->nccl, &st);
  if (r != ncclSuccess) return nccl_fail(r, "ncclCommGetAsyncError");
  if (st != ncclSuccess && st != ncclInProgress) return nccl_fail(st, "communicator error");
  return M5_OK;
#else
  return fail(M5_ERR_UNSUPPORTED, "m5_comm_check: built without NCCL");
#endif
}

extern "C" int m5_comm_abort(void* comm) {
  M5_CHECK_ARG(comm, "m5_comm_abort: null communicator");
#if defined(M5_HAVE_NCCL)
  Comm* c = static_cast<Comm*>(comm);
  if (!c->aborted) {
    ncclCommAbort(c->nccl);
    c->aborted = true;
  }
  return M5_OK;
#else
  return fail(M5_ERR_UNSUPPORTED, "m5_comm_abort: built without NCCL");
#endif
}

extern "C" int m5_comm_set_wait_ms(void* comm, int ms) {
  M5_CHECK_ARG(comm && ms > 0, "m5_comm_set_wait_ms: bad argument");
#if defined(M5_HAVE_NCCL)
  static_cast<Comm*>(comm)->wait_ns = uint64_t(ms) * 1000000ull;
  return M5_OK;
#else
  return fail(M5_ERR_UNSUPPORTED, "m5_comm_set_wait_ms: built without NCCL");
#endif
}

// The peer all-reduce on this one GPU with a stand-in for a second rank that
// never pushes its partial nor raises its flag: rank 0's areas and rank 1's
// are both local buffers, so the wait for rank 1's flag can only run out.
// Checks that the wait ends after `wait_ms`, that the device error word is
// set, and that the residual stream is left as it was.
extern "C" int m5_comm_peer_wait_selftest(int wait_ms, int* device_code, double* elapsed_ms, int* h_unchanged) {
  M5_CHECK_ARG(wait_ms > 0 && wait_ms <= 10000 && device_code && elapsed_ms && h_unchanged,
               "m5_comm_peer_wait_selftest: bad argument");
#if defined(M5_HAVE_NCCL)
  const int nranks = 2, n = 1024;
  const size_t area = size_t(2) * nranks * kArMax * sizeof(float) + 256;
  char *a0 = nullptr, *a1 = nullptr;
  float* partial = nullptr;
  bf16* h = nullptr;
  uint32_t* state = nullptr;
  int rc = M5_OK;
  if (cudaMalloc(&a0, area) != cudaSuccess || cudaMalloc(&a1, area) != cudaSuccess ||
      cudaMalloc(&partial, n * sizeof(float)) != cudaSuccess || cudaMalloc(&h, n * sizeof(bf16)) != cudaSuccess ||
      cudaMalloc(&state, 4 * sizeof(uint32_t)) != cudaSuccess) {
    rc = fail(M5_ERR_CUDA, "m5_comm_peer_wait_selftest: allocation failed");
  }
  std::vector<uint16_t> h_host(n, 0x3F80), h_back(n, 0);  // h = 1.0 everywhere
  if (!rc) {
    cudaMemset(a0, 0, area);
    cudaMemset(a1, 0, area);
    cudaMemset(partial, 0, n * sizeof(float));
    cudaMemset(state, 0, 4 * sizeof(uint32_t));
    cudaMemcpy(h, h_host.data(), n * sizeof(bf16), cudaMemcpyHostToDevice);
    comm_ar_error(1);
    ArPeers peers{};
    char* base[2] = {a0, a1};
    for (int p = 0; p < nranks; ++p) {
      peers.recv[p] = reinterpret_cast<float*>(base[p]);
      peers.flags[p] = reinterpret_cast<uint32_t*>(base[p] + size_t(2) * nranks * kArMax * sizeof(float));
    }
    const auto t0 = std::chrono::steady_clock::now();
    ar_residual_kernel<<<1, kArThreads>>>(partial, h, n, nranks, 0, peers, state, uint64_t(wait_ms) * 1000000ull);
    const cudaError_t e = cudaDeviceSynchronize();
    *elapsed_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    if (e != cudaSuccess) rc = cuda_fail(e, "m5_comm_peer_wait_selftest");
    if (!rc) {
      *device_code = comm_ar_error(1);
      cudaMemcpy(h_back.data(), h, n * sizeof(bf16), cudaMemcpyDeviceToHost);
      *h_unchanged = h_back == h_host ? 1 : 0;
    }
  }
  cudaFree(a0);
  cudaFree(a1);
  cudaFree(partial);
  cudaFree(h);
  cudaFree(state);
  return rc;
#else
  (void)wait_ms;
  return fail(M5_ERR_UNSUPPORTED, "m5_comm_peer_wait_selftest: built without NCCL");
#endif
}
