// Fused compute + collective kernels over NVLink peer memory (one process per GPU).
//
// Every rank maps the other ranks' IPC buffers (cudaIpcOpenMemHandle) and the kernels
// read/write peer memory directly with 16-byte loads/stores; no TMA, no library GEMM
// touches peer memory.
//
//   rs_sum_sq:     reduce-scatter of the fp32 gradient buffers fused with the squared
//                  norm of the reduced shard:  g[i] = sum_r grad_r[off + i]  (P2P loads),
//                  sq += sum g[i]^2.  Each rank reduces only the shard it owns.
//   adamw_bcast:   AdamW on the owned fp32 master shard (clip factor from the global
//                  squared norm in device memory) fused with the all-gather of the new
//                  bf16 weights: each updated bf16 value is stored into the compute
//                  buffer of every rank (P2P stores), which is also the rollout engine's
//                  weight buffer — the trainer -> rollout weight sync.
//   bcast_bf16:    plain shard broadcast (initial weight replication).
//   peer_gather_bf16 / peer_rs_acc:  the full-shard (FSDP) actor's per-layer all-gather of
//                  bf16 weight shards and reduce-scatter (accumulate) of fp32 gradients.
//   peer_barrier:  bounded flag barrier across ranks (sequence-numbered flags in peer
//                  memory, each wait limited by a time budget; on timeout the kernel
//                  records kErrPeerTimeout and returns).
#include <cuda_bf16.h>

#include "comm.h"
#include "common.cuh"

namespace octo {

constexpr int kMaxRanks = 8;

struct PeerPtrs {
  const void* p[kMaxRanks];
};

__global__ void rs_sum_sq_kernel(PeerPtrs grads, int world, size_t off, size_t n, float* __restrict__ out,
                                 float* __restrict__ sqnorm) {
  float acc = 0.f;
  const size_t n4 = n / 4;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r) {
      if (r < world) {
        const float4 v = reinterpret_cast<const float4*>(static_cast<const float*>(grads.p[r]) + off)[i];
        s.x += v.x;
        s.y += v.y;
        s.z += v.z;
        s.w += v.w;
      }
    }
    reinterpret_cast<float4*>(out)[i] = s;
    acc += s.x * s.x + s.y * s.y + s.z * s.z + s.w * s.w;
  }
  for (size_t i = n4 * 4 + blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    float s = 0.f;
    for (int r = 0; r < world; ++r) s += static_cast<const float*>(grads.p[r])[off + i];
    out[i] = s;
    acc += s * s;
  }
  acc = warp_sum(acc);
  __shared__ float sh[32];
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0 && sqnorm != nullptr) atomicAdd(sqnorm, v);
  }
}

__global__ void adamw_bcast_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                                   float* __restrict__ v, PeerPtrs dst16, int world, size_t off, size_t n, float lr,
                                   float b1, float b2, float eps, float wd, float bc1, float bc2,
                                   const float* __restrict__ sqnorm, float max_norm, float grad_scale) {
  float clip = grad_scale;
  if (sqnorm != nullptr && max_norm > 0.f) {
    const float nrm = sqrtf(*sqnorm) * grad_scale;
    if (nrm > max_norm) clip *= max_norm / (nrm + 1e-6f);
  }
  const size_t n8 = n / 8;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n8;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    float pv[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const size_t k = i * 8 + e;
      const float gi = g[k] * clip;
      const float mi = b1 * m[k] + (1.f - b1) * gi;
      const float vi = b2 * v[k] + (1.f - b2) * gi * gi;
      m[k] = mi;
      v[k] = vi;
      float x = p[k];
      x -= lr * wd * x;
      x -= lr * (mi / bc1) / (sqrtf(vi / bc2) + eps);
      p[k] = x;
      pv[e] = x;
    }
    uint4 u;
    u.x = pack_bf16x2(pv[0], pv[1]);
    u.y = pack_bf16x2(pv[2], pv[3]);
    u.z = pack_bf16x2(pv[4], pv[5]);
    u.w = pack_bf16x2(pv[6], pv[7]);
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r) {
      if (r < world) {
        __nv_bfloat16* d = const_cast<__nv_bfloat16*>(static_cast<const __nv_bfloat16*>(dst16.p[r]));
        *reinterpret_cast<uint4*>(d + off + i * 8) = u;
      }
    }
  }
}

__global__ void bcast_bf16_kernel(const __nv_bfloat16* __restrict__ src, PeerPtrs dst16, int world, size_t off,
                                  size_t n) {
  const size_t n8 = n / 8;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n8;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const uint4 u = reinterpret_cast<const uint4*>(src)[i];
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r) {
      if (r < world) {
        __nv_bfloat16* d = const_cast<__nv_bfloat16*>(static_cast<const __nv_bfloat16*>(dst16.p[r]));
        *reinterpret_cast<uint4*>(d + off + i * 8) = u;
      }
    }
  }
}

// flags: each rank's flag array (int32[kMaxRanks]) in its own IPC buffer.  Rank `me`
// writes `seq` into slot `me` of every rank's array, then waits (bounded) until its own
// array holds `seq` in every slot.
__global__ void peer_barrier_kernel(PeerPtrs flags, int world, int me, int seq, int* status,
                                    unsigned long long budget_ns) {
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int r = 0; r < world; ++r) {
      volatile int* f = const_cast<volatile int*>(static_cast<const volatile int*>(flags.p[r]));
      f[me] = seq;
    }
    __threadfence_system();
    volatile int* mine = const_cast<volatile int*>(static_cast<const volatile int*>(flags.p[me]));
    const uint64_t t0 = globaltimer_ns();
    const uint64_t budget = budget_ns ? budget_ns : wait_budget_ns(status);
    for (int r = 0; r < world; ++r) {
      while (mine[r] < seq) {
        if (globaltimer_ns() - t0 > budget) {
          record_error(status, kErrPeerTimeout, 900 + r);
          return;
        }
      }
    }
    __threadfence_system();
  }
}

// FSDP all-gather of one unit: dst[r * n + j] = shard_r[j] (16-byte peer loads; n % 8 == 0).
__global__ void peer_gather_bf16_kernel(PeerPtrs src, int world, size_t n, __nv_bfloat16* __restrict__ dst) {
  const size_t n8 = n / 8;
  const size_t total = n8 * static_cast<size_t>(world);
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i / n8);
    const size_t j = i - static_cast<size_t>(r) * n8;
    const uint4 u = reinterpret_cast<const uint4*>(src.p[r])[j];
    reinterpret_cast<uint4*>(dst)[i] = u;
  }
}

// FSDP reduce-scatter of one unit's gradient: acc[j] += sum_r part_r[j] in rank order
// (part_r = this rank's slice of rank r's gradient slot; 16-byte peer loads; n % 4 == 0).
__global__ void peer_rs_acc_kernel(PeerPtrs src, int world, size_t n, float* __restrict__ acc) {
  const size_t n4 = n / 4;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    float4 s = reinterpret_cast<const float4*>(acc)[i];
    float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r) {
      if (r < world) {
        const float4 v = reinterpret_cast<const float4*>(src.p[r])[i];
        t.x += v.x;
        t.y += v.y;
        t.z += v.z;
        t.w += v.w;
      }
    }
    s.x += t.x;
    s.y += t.y;
    s.z += t.z;
    s.w += t.w;
    reinterpret_cast<float4*>(acc)[i] = s;
  }
}

static PeerPtrs to_peers(const int64_t* ptrs, int world) {
  PeerPtrs pp{};
  for (int r = 0; r < world && r < kMaxRanks; ++r) pp.p[r] = reinterpret_cast<const void*>(ptrs[r]);
  return pp;
}

static int grid_for(size_t n, int per_thread) {
  const size_t threads = (n / per_thread + 255) / 256 + 1;
  return static_cast<int>(threads < 148 * 16 ? threads : 148 * 16);
}

void rs_sum_sq(const int64_t* grad_ptrs, int world, size_t off, size_t n, float* out, float* sqnorm,
               cudaStream_t st) {
  if (n == 0) return;
  rs_sum_sq_kernel<<<grid_for(n, 4), 256, 0, st>>>(to_peers(grad_ptrs, world), world, off, n, out, sqnorm);
}

void adamw_bcast(float* p, const float* g, float* m, float* v, const int64_t* dst_ptrs, int world, size_t off,
                 size_t n, float lr, float b1, float b2, float eps, float wd, int step, const float* sqnorm,
                 float max_norm, float grad_scale, cudaStream_t st) {
  if (n == 0) return;
  const float bc1 = 1.f - powf(b1, static_cast<float>(step));
  const float bc2 = 1.f - powf(b2, static_cast<float>(step));
  adamw_bcast_kernel<<<grid_for(n, 8), 256, 0, st>>>(p, g, m, v, to_peers(dst_ptrs, world), world, off, n, lr, b1,
                                                       b2, eps, wd, bc1, bc2, sqnorm, max_norm, grad_scale);
}

void bcast_bf16(const __nv_bfloat16* src, const int64_t* dst_ptrs, int world, size_t off, size_t n,
                cudaStream_t st) {
  if (n == 0) return;
  bcast_bf16_kernel<<<grid_for(n, 8), 256, 0, st>>>(src, to_peers(dst_ptrs, world), world, off, n);
}

void peer_gather_bf16(const int64_t* src_ptrs, int world, size_t n, __nv_bfloat16* dst, cudaStream_t st) {
  if (n == 0) return;
  peer_gather_bf16_kernel<<<grid_for(n * world, 8), 256, 0, st>>>(to_peers(src_ptrs, world), world, n, dst);
}

void peer_rs_acc(const int64_t* src_ptrs, int world, size_t n, float* acc, cudaStream_t st) {
  if (n == 0) return;
  peer_rs_acc_kernel<<<grid_for(n, 4), 256, 0, st>>>(to_peers(src_ptrs, world), world, n, acc);
}

void peer_barrier(const int64_t* flag_ptrs, int world, int me, int seq, int* status, cudaStream_t st,
                  unsigned long long budget_ns) {
  peer_barrier_kernel<<<1, 32, 0, st>>>(to_peers(flag_ptrs, world), world, me, seq, status, budget_ns);
}

}  // namespace octo
