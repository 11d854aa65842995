// Fused split-K finishes of the decode layer (CUDA graphs of the rollout engine).
//
// A decode-sized projection (M <= 256 rows) runs as a split-K tcgen05 GEMM whose fp32
// partials land in a workspace; the kernel that sums them also does the element-wise
// work that follows the projection in the layer, so those steps cost no launch and no
// extra pass over the activations:
//   splitk_finish_norm  x = sum + bias + residual (bf16: the residual stream), then
//                       h = RMSNorm(x) * w of the next sub-layer (one CTA per row, so the
//                       row's sum of squares is a block reduction)
//   splitk_finish_qkv   qkv = sum + bias (rounded to bf16 as the unfused GEMM output is),
//                       rotary embedding of the q and k heads (rope_sincos, as the rotary
//                       kernel), q rows to the attention input, k / v rows to the KV cache
//                       slots of their rows
#include <cuda_bf16.h>

#include "common.cuh"
#include "elementwise.h"

namespace octo {

using bf16 = __nv_bfloat16;

namespace {

__device__ __forceinline__ float round_bf16(float v) { return __bfloat162float(__float2bfloat16(v)); }

__device__ __forceinline__ void sum_splits8(const float* __restrict__ p, int splits, size_t plane, float (&a)[8]) {
#pragma unroll
  for (int e = 0; e < 8; ++e) a[e] = 0.f;
  for (int s = 0; s < splits; ++s) {
    const float4 x = *reinterpret_cast<const float4*>(p + s * plane);
    const float4 y = *reinterpret_cast<const float4*>(p + s * plane + 4);
    a[0] += x.x; a[1] += x.y; a[2] += x.z; a[3] += x.w;
    a[4] += y.x; a[5] += y.y; a[6] += y.z; a[7] += y.w;
  }
}

}  // namespace

__global__ void splitk_finish_norm_kernel(const float* __restrict__ ws, int splits, int M, int N,
                                          const bf16* __restrict__ bias, const bf16* __restrict__ res, int ldr,
                                          bf16* __restrict__ x, int ldx, const bf16* __restrict__ w, float eps,
                                          int plus_one, bf16* __restrict__ h, int ldh) {
  grid_dep_launch();
  __shared__ float red[32];
  const int row = blockIdx.x;
  const int c = threadIdx.x * 8;
  const bool active = c < N;
  const size_t plane = static_cast<size_t>(M) * N;
  float a[8];
  float ss = 0.f;
  if (active) {
    sum_splits8(ws + static_cast<size_t>(row) * N + c, splits, plane, a);
    if (bias != nullptr) {
      float b[8];
      load8(bias + c, b);
#pragma unroll
      for (int e = 0; e < 8; ++e) a[e] += b[e];
    }
    if (res != nullptr) {
      float r[8];
      load8(res + static_cast<size_t>(row) * ldr + c, r);
#pragma unroll
      for (int e = 0; e < 8; ++e) a[e] += r[e];
    }
    store8(x + static_cast<size_t>(row) * ldx + c, a);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      a[e] = round_bf16(a[e]);  // the norm reads the stored (bf16) residual stream
      ss += a[e] * a[e];
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  ss = warp_sum(ss);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  if (warp == 0) {
    float v = lane < static_cast<int>((blockDim.x + 31) >> 5) ? red[lane] : 0.f;
    v = warp_sum(v);
    if (lane == 0) red[0] = v;
  }
  __syncthreads();
  const float r = rsqrtf(red[0] / N + eps);
  if (active) {
    float g[8];
    load8(w + c, g);
#pragma unroll
    for (int e = 0; e < 8; ++e) a[e] = a[e] * r * (plus_one ? 1.f + g[e] : g[e]);
    store8(h + static_cast<size_t>(row) * ldh + c, a);
  }
}

__global__ void splitk_finish_qkv_kernel(const float* __restrict__ ws, int splits, int M, int Hq, int Hkv, int D,
                                         const bf16* __restrict__ bias, const int32_t* __restrict__ pos,
                                         float log2_theta, bf16* __restrict__ q, int ldq,
                                         const int64_t* __restrict__ slots, bf16* __restrict__ kc,
                                         bf16* __restrict__ vc, long long n_slots, int* status) {
  grid_dep_launch();
  const int row = blockIdx.x;
  const int half = D / 2, per_head = half / 8;
  const int hd = threadIdx.x / per_head;
  const int i0 = (threadIdx.x - hd * per_head) * 8;
  if (hd >= Hq + 2 * Hkv) return;
  const int N = (Hq + 2 * Hkv) * D;
  const size_t plane = static_cast<size_t>(M) * N;
  const float* p = ws + static_cast<size_t>(row) * N + static_cast<size_t>(hd) * D;
  float lo[8], hi[8];
  sum_splits8(p + i0, splits, plane, lo);
  sum_splits8(p + i0 + half, splits, plane, hi);
  if (bias != nullptr) {
    float b0[8], b1[8];
    load8(bias + static_cast<size_t>(hd) * D + i0, b0);
    load8(bias + static_cast<size_t>(hd) * D + i0 + half, b1);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      lo[e] += b0[e];
      hi[e] += b1[e];
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) {  // the GEMM's bf16 output, which the rotary kernel would read
    lo[e] = round_bf16(lo[e]);
    hi[e] = round_bf16(hi[e]);
  }
  if (hd < Hq + Hkv) {
    const int ps = pos[row];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float sn, cs;
      rope_sincos(ps, i0 + e, D, log2_theta, sn, cs);
      const float a = lo[e], b = hi[e];
      lo[e] = a * cs - b * sn;
      hi[e] = b * cs + a * sn;
    }
  }
  if (hd < Hq) {
    bf16* dst = q + static_cast<size_t>(row) * ldq + static_cast<size_t>(hd) * D;
    store8(dst + i0, lo);
    store8(dst + i0 + half, hi);
    return;
  }
  const int64_t slot = slots[row];
  if (slot < 0 || !index_ok(slot, n_slots, status, 720)) return;  // negative: not written
  const bool is_k = hd < Hq + Hkv;
  const int kh = is_k ? hd - Hq : hd - Hq - Hkv;
  bf16* dst = (is_k ? kc : vc) + slot * static_cast<int64_t>(Hkv) * D + static_cast<size_t>(kh) * D;
  store8(dst + i0, lo);
  store8(dst + i0 + half, hi);
}

void splitk_finish_norm(const float* ws, int splits, int M, int N, const bf16* bias, const bf16* res, int ldr,
                        bf16* x, int ldx, const bf16* w, float eps, bool plus_one, bf16* h, int ldh, cudaStream_t st) {
  if (M == 0) return;
  const int threads = ((N / 8) + 31) / 32 * 32;
  splitk_finish_norm_kernel<<<M, threads, 0, st>>>(ws, splits, M, N, bias, res, ldr, x, ldx, w, eps,
                                                   plus_one ? 1 : 0, h, ldh);
}

void splitk_finish_qkv(const float* ws, int splits, int M, int Hq, int Hkv, int D, const bf16* bias,
                       const int32_t* pos, float theta, bf16* q, int ldq, const int64_t* slots, bf16* kc, bf16* vc,
                       long long n_slots, int* status, cudaStream_t st) {
  if (M == 0) return;
  const int threads = ((Hq + 2 * Hkv) * (D / 16) + 31) / 32 * 32;
  splitk_finish_qkv_kernel<<<M, threads, 0, st>>>(ws, splits, M, Hq, Hkv, D, bias, pos, log2f(theta), q, ldq, slots,
                                                  kc, vc, n_slots, status);
}

}  // namespace octo
