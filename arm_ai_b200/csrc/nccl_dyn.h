// nccl_dyn.h — the few NCCL calls tensor parallelism uses, resolved at run time.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

namespace armai {

int nccl_unique_id(void* out128);
int nccl_comm_init(void** comm, int nranks, const void* id128, int rank);
int nccl_allreduce_sum_f32(const float* send, float* recv, size_t n, void* comm, cudaStream_t s);
int nccl_allgather_b32(const void* send, void* recv, size_t n_per_rank, void* comm, cudaStream_t s);
void nccl_comm_destroy(void* comm);
// Ends the communicator's pending collectives (their kernels return) and frees it.
void nccl_comm_abort(void* comm);

}  // namespace armai
