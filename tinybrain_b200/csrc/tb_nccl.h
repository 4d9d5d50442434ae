// tb_nccl.h -- the NCCL calls of the tensor-parallel decode step, resolved at
// run time (dlopen of libnccl.so.2) so the library loads on hosts without
// NCCL and shares the communicator library already loaded by the process.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <string>

namespace tb {

constexpr int kNcclIdBytes = 128;

// 0 on success; otherwise `why` says what failed.
int nccl_unique_id(unsigned char* id, std::string& why);
int nccl_comm_init(void** comm, const unsigned char* id, int rank, int world, std::string& why);
void nccl_comm_destroy(void* comm);
// In-place fp32 sum over all ranks of `count` floats at `buf`, on `st`.
cudaError_t nccl_allreduce_sum_f32(void* comm, float* buf, size_t count, cudaStream_t st, std::string& why);

}  // namespace tb
