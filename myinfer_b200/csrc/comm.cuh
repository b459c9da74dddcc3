// Collectives of a multi-GPU model (comm.cu): thin, stream-ordered wrappers
// over the communicator handle the C ABI creates (m5_comm_init).
#pragma once

#include "common.cuh"

namespace m5 {

int comm_allreduce_f32(void* comm, float* buf, int64_t n, cudaStream_t st);                 // in place, sum
int comm_allgather_bf16(void* comm, const bf16* send, bf16* recv, int64_t n, cudaStream_t st);  // n per rank
int comm_size(void* comm);
int comm_rank(void* comm);

}  // namespace m5
