// Tensor parallelism plumbing: NCCL, loaded at run time from the library file the caller names
// (the one PyTorch ships), so that libnespec.so carries no link-time NCCL dependency. Only the
// calls below are used: one communicator per model, sum all-reduce of fp32 partial projections,
// max all-reduce of 64-bit argmax keys.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

namespace ne {

constexpr int TP_UNIQUE_ID_BYTES = 128;

int tp_load(const char* library_path);                 // dlopen + dlsym (once per path)
int tp_unique_id(void* out);                           // TP_UNIQUE_ID_BYTES bytes
int tp_comm_init(void** comm, int world, const void* unique_id, int rank);
int tp_comm_destroy(void* comm);
int tp_allreduce_sum_f32(float* buf, size_t count, void* comm, cudaStream_t stream);
int tp_allreduce_max_u64(unsigned long long* buf, size_t count, void* comm, cudaStream_t stream);

}  // namespace ne
