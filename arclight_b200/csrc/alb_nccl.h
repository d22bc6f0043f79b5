// Run-time loaded NCCL (tensor parallelism only).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>

namespace alb {
int  nccl_unique_id(void * out128);
int  nccl_init(void ** comm, int rank, int size, const void * id128);
// dtype 0 = fp32, 1 = uint64; op 0 = sum, 1 = max
int  nccl_allreduce(void * comm, const void * src, void * dst, size_t count, int dtype, int op, cudaStream_t st);
// dst [size][count] fp32: rank r's src at dst + r * count
int  nccl_allgather_f32(void * comm, const float * src, float * dst, size_t count, cudaStream_t st);
int  nccl_async_error(void * comm);
void nccl_destroy(void * comm, bool abort);
}  // namespace alb
