// Collectives of a multi-GPU model (comm.cu): thin, stream-ordered wrappers
// over the communicator handle the C ABI creates (m5_comm_init).
#pragma once

#include "common.cuh"

namespace m5 {

int comm_allreduce_f32(void* comm, float* buf, int64_t n, cudaStream_t st);                 // in place, sum
int comm_allgather_bf16(void* comm, const bf16* send, bf16* recv, int64_t n, cudaStream_t st);  // n per rank
// h += sum over ranks of partial (h = bf16(h + bf16(sum)), fp32 sum in rank
// order): one-shot over NVLink peer memory when set up, else NCCL + a kernel.
int comm_allreduce_residual(void* comm, float* partial, bf16* h, int64_t n, cudaStream_t st);
int comm_ar_error(int reset);  // sticky device error word of the peer all-reduce waits
int comm_size(void* comm);
int comm_rank(void* comm);

}  // namespace m5
