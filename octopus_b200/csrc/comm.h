// Launchers of comm.cu (fused compute + collective kernels over peer memory).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

namespace octo {
void rs_sum_sq(const int64_t* grad_ptrs, int world, size_t off, size_t n, float* out, float* sqnorm, cudaStream_t st);
void adamw_bcast(float* p, const float* g, float* m, float* v, const int64_t* dst_ptrs, int world, size_t off,
                 size_t n, float lr, float b1, float b2, float eps, float wd, int step, const float* sqnorm,
                 float max_norm, float grad_scale, cudaStream_t st);
void bcast_bf16(const __nv_bfloat16* src, const int64_t* dst_ptrs, int world, size_t off, size_t n, cudaStream_t st);
void peer_gather_bf16(const int64_t* src_ptrs, int world, size_t n, __nv_bfloat16* dst, cudaStream_t st);
void peer_rs_acc(const int64_t* src_ptrs, int world, size_t n, float* acc, cudaStream_t st);
// budget_ns > 0: this barrier's own time limit (else the device status word's budget)
void peer_barrier(const int64_t* flag_ptrs, int world, int me, int seq, int* status, cudaStream_t st,
                  unsigned long long budget_ns = 0);
}  // namespace octo
