// Memory-bound kernels of the decoder: RMSNorm fwd/bwd, rotary embedding, SwiGLU,
// embedding gather/scatter, paged-KV writes, head / sampling combines, grad-norm and
// the fused AdamW update.  All are vectorised (16-byte accesses) and fp32 inside.
#include <cuda_bf16.h>

#include "common.cuh"
#include "elementwise.h"
#include "head_epilogue.cuh"

namespace octo {

using bf16 = __nv_bfloat16;


// ----------------------------------------------------------------- head combine
__global__ void head_combine_kernel(const float* __restrict__ part, int M, int T, const int32_t* __restrict__ labels,
                                    float* logp, float* ent, float* lse_out) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const float4* p = reinterpret_cast<const float4*>(part) + static_cast<size_t>(row) * T;
  float gm = -INFINITY;
  for (int i = lane; i < T; i += 32) gm = fmaxf(gm, p[i].x);
  gm = warp_max(gm);
  float S = 0.f, Tt = 0.f, zl = 0.f;
  for (int i = lane; i < T; i += 32) {
    const float4 q = p[i];
    if (q.x != -INFINITY) {
      const float sc = __expf(q.x - gm);
      S += q.y * sc;
      Tt += q.z * sc;
    }
    zl += q.w;
  }
  S = warp_sum(S);
  Tt = warp_sum(Tt);
  zl = warp_sum(zl);
  if (lane == 0) {
    const float L = gm + logf(S);
    lse_out[row] = L;
    ent[row] = L - Tt / S;
    logp[row] = labels[row] >= 0 ? zl - L : 0.f;
  }
}

void head_combine(const float* part, int M, int T, const int32_t* labels, float* logp, float* ent, float* lse,
                  cudaStream_t st) {
  if (M == 0) return;
  head_combine_kernel<<<(M + 7) / 8, 256, 0, st>>>(part, M, T, labels, logp, ent, lse);
}

// ----------------------------------------------------------------- sample combine
__global__ void sample_combine_kernel(const float* __restrict__ part, int M, int T, uint64_t seed,
                                      const int64_t* __restrict__ row_stream, int64_t* tokens, float* logprob) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const float4* p = reinterpret_cast<const float4*>(part) + static_cast<size_t>(row) * T;
  float gm = -INFINITY, best = -INFINITY;
  int best_col = -1;
  for (int i = lane; i < T; i += 32) {
    const float4 q = p[i];
    gm = fmaxf(gm, q.x);
    const int c = __float_as_int(q.w);
    if (c >= 0 && (q.z > best || (q.z == best && c < best_col))) {
      best = q.z;
      best_col = c;
    }
  }
  gm = warp_max(gm);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oc = __shfl_xor_sync(0xffffffffu, best_col, o);
    if (oc >= 0 && (ob > best || (ob == best && oc < best_col) || best_col < 0)) {
      best = ob;
      best_col = oc;
    }
  }
  float S = 0.f;
  for (int i = lane; i < T; i += 32) {
    const float4 q = p[i];
    if (q.x != -INFINITY) S += q.y * __expf(q.x - gm);
  }
  S = warp_sum(S);
  if (lane == 0) {
    const uint64_t stream = row_stream != nullptr ? static_cast<uint64_t>(row_stream[row]) : static_cast<uint64_t>(row);
    const float z = best - gumbel_noise(row_key(seed, stream), static_cast<uint32_t>(best_col));
    tokens[row] = best_col;
    logprob[row] = z - (gm + logf(S));
  }
}

void sample_combine(const float* part, int M, int T, uint64_t seed, const int64_t* row_stream, int64_t* tokens,
                    float* logprob, cudaStream_t st) {
  if (M == 0) return;
  sample_combine_kernel<<<(M + 7) / 8, 256, 0, st>>>(part, M, T, seed, row_stream, tokens, logprob);
}

// ----------------------------------------------------------------- RMSNorm
// y = x * rsqrt(mean(x^2) + eps) * (w or 1 + w).  One warp per row, H % 256 == 0 or H % 8 == 0.
__global__ void rmsnorm_fwd_kernel(const bf16* __restrict__ x, int ldx, const bf16* __restrict__ w, bf16* y,
                                   int ldy, float* rstd_out, int T, int H, float eps, int plus_one) {
  grid_dep_launch();  // a dependent GEMM may start its prologue and weight prefetch
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= T) return;
  const bf16* xr = x + static_cast<size_t>(row) * ldx;
  float ss = 0.f;
  for (int c = lane * 8; c < H; c += 256) {
    float f[8];
    load8(xr + c, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += f[i] * f[i];
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / H + eps);
  if (lane == 0 && rstd_out != nullptr) rstd_out[row] = r;
  bf16* yr = y + static_cast<size_t>(row) * ldy;
  for (int c = lane * 8; c < H; c += 256) {
    float f[8], g[8];
    load8(xr + c, f);
    load8(w + c, g);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = f[i] * r * (plus_one ? 1.f + g[i] : g[i]);
    store8(yr + c, f);
  }
}

void rmsnorm_fwd(const bf16* x, int ldx, const bf16* w, bf16* y, int ldy, float* rstd, int T, int H, float eps,
                 int plus_one, cudaStream_t st) {
  if (T == 0) return;
  rmsnorm_fwd_kernel<<<(T + 7) / 8, 256, 0, st>>>(x, ldx, w, y, ldy, rstd, T, H, eps, plus_one);
}

// dx = r * (gw - xh * mean(xh * gw)) (+ dres),  gw = dy * weff,  xh = x * r
// dw += sum_rows dy * xh   (fp32 accumulation; block partials then atomics)
__global__ void rmsnorm_bwd_kernel(const bf16* __restrict__ dy, const bf16* __restrict__ x, int ldx,
                                   const bf16* __restrict__ w, const float* __restrict__ rstd,
                                   const bf16* __restrict__ dres, bf16* dx, float* dw, int T, int H, int plus_one,
                                   int rows_per_block) {
  extern __shared__ float sdw[];  // [H]
  for (int c = threadIdx.x; c < H; c += blockDim.x) sdw[c] = 0.f;
  __syncthreads();
  const int warps = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r0 = blockIdx.x * rows_per_block;
  const int r1 = min(T, r0 + rows_per_block);
  for (int row = r0 + warp; row < r1; row += warps) {
    const bf16* xr = x + static_cast<size_t>(row) * ldx;
    const bf16* dyr = dy + static_cast<size_t>(row) * H;
    const float r = rstd[row];
    float dot = 0.f;
    for (int c = lane * 8; c < H; c += 256) {
      float fx[8], fd[8], fw[8];
      load8(xr + c, fx);
      load8(dyr + c, fd);
      load8(w + c, fw);
#pragma unroll
      for (int i = 0; i < 8; ++i) dot += fd[i] * (plus_one ? 1.f + fw[i] : fw[i]) * fx[i] * r;
    }
    dot = warp_sum(dot) / H;
    for (int c = lane * 8; c < H; c += 256) {
      float fx[8], fd[8], fw[8], o[8];
      load8(xr + c, fx);
      load8(dyr + c, fd);
      load8(w + c, fw);
      float fr[8];
      if (dres != nullptr) load8(dres + static_cast<size_t>(row) * H + c, fr);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float xh = fx[i] * r;
        const float gw = fd[i] * (plus_one ? 1.f + fw[i] : fw[i]);
        o[i] = r * (gw - xh * dot) + (dres != nullptr ? fr[i] : 0.f);
        atomicAdd(&sdw[c + i], fd[i] * xh);
      }
      store8(dx + static_cast<size_t>(row) * H + c, o);
    }
  }
  __syncthreads();
  if (dw != nullptr)
    for (int c = threadIdx.x; c < H; c += blockDim.x) atomicAdd(&dw[c], sdw[c]);
}

void rmsnorm_bwd(const bf16* dy, const bf16* x, int ldx, const bf16* w, const float* rstd, const bf16* dres,
                 bf16* dx, float* dw, int T, int H, int plus_one, cudaStream_t st) {
  if (T == 0) return;
  const int rows_per_block = 64;
  const int blocks = (T + rows_per_block - 1) / rows_per_block;
  rmsnorm_bwd_kernel<<<blocks, 256, H * sizeof(float), st>>>(dy, x, ldx, w, rstd, dres, dx, dw, T, H, plus_one,
                                                              rows_per_block);
}

// ----------------------------------------------------------------- rotary (neox, rotate-half)
// In place on the q heads [0, Hq) and k heads [Hq, Hq+Hkv) of a fused qkv row.
// angle = pos * theta^(-2i/D); sign = -1 applies the inverse rotation (backward).
__global__ void rope_kernel(bf16* qkv, int ld, const int32_t* __restrict__ pos, int T, int Hq, int Hkv, int D,
                            float log2_theta, float sign) {
  const int half = D / 2;
  const int heads = Hq + Hkv;
  const long total = static_cast<long>(T) * heads * half;
  for (long idx = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<long>(gridDim.x) * blockDim.x) {
    const int i = idx % half;
    const long th = idx / half;
    const int h = th % heads;
    const int t = th / heads;
    float sn, cs;
    rope_sincos(pos[t], i, D, log2_theta, sn, cs);
    sn *= sign;
    bf16* base = qkv + static_cast<size_t>(t) * ld + static_cast<size_t>(h) * D;
    const float a = __bfloat162float(base[i]);
    const float b = __bfloat162float(base[i + half]);
    base[i] = __float2bfloat16(a * cs - b * sn);
    base[i + half] = __float2bfloat16(b * cs + a * sn);
  }
}

void rope_apply(bf16* qkv, int ld, const int32_t* pos, int T, int Hq, int Hkv, int D, float theta, bool inverse,
                cudaStream_t st) {
  if (T == 0) return;
  const long total = static_cast<long>(T) * (Hq + Hkv) * (D / 2);
  const int blocks = static_cast<int>(std::min<long>((total + 255) / 256, 148L * 32));
  rope_kernel<<<blocks, 256, 0, st>>>(qkv, ld, pos, T, Hq, Hkv, D, log2f(theta), inverse ? -1.f : 1.f);
}

// ----------------------------------------------------------------- SwiGLU
// gu = [gate | up] along features (each F wide); out = silu(gate) * up
__global__ void swiglu_fwd_kernel(const bf16* __restrict__ gu, bf16* out, int T, int F) {
  grid_dep_launch();  // a dependent GEMM may start its prologue and weight prefetch
  const long total = static_cast<long>(T) * F / 8;
  for (long v = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; v < total;
       v += static_cast<long>(gridDim.x) * blockDim.x) {
    const long e = v * 8;
    const int t = e / F, c = e % F;
    float g[8], u[8], o[8];
    load8(gu + static_cast<size_t>(t) * 2 * F + c, g);
    load8(gu + static_cast<size_t>(t) * 2 * F + F + c, u);
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = g[i] / (1.f + __expf(-g[i])) * u[i];
    store8(out + static_cast<size_t>(t) * F + c, o);
  }
}

__global__ void swiglu_bwd_kernel(const bf16* __restrict__ gu, const bf16* __restrict__ dout, bf16* dgu, int T,
                                  int F) {
  const long total = static_cast<long>(T) * F / 8;
  for (long v = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; v < total;
       v += static_cast<long>(gridDim.x) * blockDim.x) {
    const long e = v * 8;
    const int t = e / F, c = e % F;
    float g[8], u[8], d[8], dg[8], du[8];
    load8(gu + static_cast<size_t>(t) * 2 * F + c, g);
    load8(gu + static_cast<size_t>(t) * 2 * F + F + c, u);
    load8(dout + static_cast<size_t>(t) * F + c, d);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float s = 1.f / (1.f + __expf(-g[i]));
      du[i] = d[i] * g[i] * s;
      dg[i] = d[i] * u[i] * s * (1.f + g[i] * (1.f - s));
    }
    store8(dgu + static_cast<size_t>(t) * 2 * F + c, dg);
    store8(dgu + static_cast<size_t>(t) * 2 * F + F + c, du);
  }
}

static int ew_blocks(long vecs) { return static_cast<int>(std::min<long>((vecs + 255) / 256, 148L * 16)); }

void swiglu_fwd(const bf16* gu, bf16* out, int T, int F, cudaStream_t st) {
  if (T == 0) return;
  swiglu_fwd_kernel<<<ew_blocks(static_cast<long>(T) * F / 8), 256, 0, st>>>(gu, out, T, F);
}
void swiglu_bwd(const bf16* gu, const bf16* dout, bf16* dgu, int T, int F, cudaStream_t st) {
  if (T == 0) return;
  swiglu_bwd_kernel<<<ew_blocks(static_cast<long>(T) * F / 8), 256, 0, st>>>(gu, dout, dgu, T, F);
}

// ----------------------------------------------------------------- embedding
// A token id outside [0, V) is reported (kErrBadIndex, site 700, the id) and its row is
// written as zeros instead of reading outside the table.
__global__ void embed_fwd_kernel(const int64_t* __restrict__ ids, const bf16* __restrict__ W, bf16* out, int T, int H,
                                 int V, int* status) {
  const int row = blockIdx.x;
  if (row >= T) return;
  const int64_t id = ids[row];
  uint4* dst = reinterpret_cast<uint4*>(out + static_cast<size_t>(row) * H);
  if (!index_ok(id, V, status, 700)) {
    for (int c = threadIdx.x; c < H / 8; c += blockDim.x) dst[c] = make_uint4(0u, 0u, 0u, 0u);
    return;
  }
  const uint4* src = reinterpret_cast<const uint4*>(W + static_cast<size_t>(id) * H);
  for (int c = threadIdx.x; c < H / 8; c += blockDim.x) dst[c] = src[c];
}
__global__ void embed_bwd_kernel(const int64_t* __restrict__ ids, const bf16* __restrict__ dout, float* dW, int T,
                                 int H, int V, int* status) {
  const int row = blockIdx.x;
  if (row >= T) return;
  const int64_t id = ids[row];
  if (!index_ok(id, V, status, 701)) return;
  for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
    float f[8];
    load8(dout + static_cast<size_t>(row) * H + c, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) atomicAdd(&dW[static_cast<size_t>(id) * H + c + i], f[i]);
  }
}
void embed_fwd(const int64_t* ids, const bf16* W, bf16* out, int T, int H, int V, int* status, cudaStream_t st) {
  if (T == 0) return;
  embed_fwd_kernel<<<T, 128, 0, st>>>(ids, W, out, T, H, V, status);
}
void embed_bwd(const int64_t* ids, const bf16* dout, float* dW, int T, int H, int V, int* status, cudaStream_t st) {
  if (T == 0) return;
  embed_bwd_kernel<<<T, 128, 0, st>>>(ids, dout, dW, T, H, V, status);
}

// ----------------------------------------------------------------- paged KV write
// cache[slot[t], h, :] = src[t, h, :] for the k and v heads of a fused qkv row.  A
// negative slot means "no write"; a slot >= n_slots is reported (kErrBadIndex, site 710)
// and skipped.
__global__ void kv_write_kernel(const bf16* __restrict__ qkv, int ld, int Hq, int Hkv, int D,
                                const int64_t* __restrict__ slots, bf16* kc, bf16* vc, int T, long long n_slots,
                                int* status) {
  const int t = blockIdx.x;
  if (t >= T) return;
  const int64_t slot = slots[t];
  if (slot < 0 || !index_ok(slot, n_slots, status, 710)) return;
  const int width = Hkv * D;
  const bf16* k = qkv + static_cast<size_t>(t) * ld + static_cast<size_t>(Hq) * D;
  const bf16* v = k + width;
  for (int c = threadIdx.x * 8; c < width; c += blockDim.x * 8) {
    *reinterpret_cast<uint4*>(kc + slot * width + c) = *reinterpret_cast<const uint4*>(k + c);
    *reinterpret_cast<uint4*>(vc + slot * width + c) = *reinterpret_cast<const uint4*>(v + c);
  }
}
void kv_write(const bf16* qkv, int ld, int Hq, int Hkv, int D, const int64_t* slots, bf16* kc, bf16* vc, int T,
              long long n_slots, int* status, cudaStream_t st) {
  if (T == 0) return;
  kv_write_kernel<<<T, 64, 0, st>>>(qkv, ld, Hq, Hkv, D, slots, kc, vc, T, n_slots, status);
}

// ----------------------------------------------------------------- optimizer
// Sum of squares of an fp32 buffer into out[0] (fp32 atomics over block partials).
__global__ void sqnorm_kernel(const float* __restrict__ g, long n, float* out) {
  float acc = 0.f;
  const long n4 = n / 4;
  for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const float4 v = reinterpret_cast<const float4*>(g)[i];
    acc += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  for (long i = n4 * 4 + blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long>(gridDim.x) * blockDim.x)
    acc += g[i] * g[i];
  acc = warp_sum(acc);
  __shared__ float sh[32];
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) atomicAdd(out, v);
  }
}
void sqnorm_accum(const float* g, long n, float* out, cudaStream_t st) {
  if (n == 0) return;
  const int blocks = static_cast<int>(std::min<long>((n / 4 + 255) / 256 + 1, 148L * 8));
  sqnorm_kernel<<<blocks, 256, 0, st>>>(g, n, out);
}

// AdamW on fp32 master weights with the gradient scaled by min(1, max_norm / ||g||)
// (the squared norm is read from device memory, so no host sync is needed), writing
// the bf16 compute copy in the same pass.
__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, bf16* __restrict__ p16, long n, float lr, float b1, float b2,
                             float eps, float wd, float bc1, float bc2, const float* __restrict__ sqnorm,
                             float max_norm, float grad_scale) {
  float clip = grad_scale;
  if (sqnorm != nullptr && max_norm > 0.f) {
    const float nrm = sqrtf(*sqnorm) * grad_scale;
    if (nrm > max_norm) clip *= max_norm / (nrm + 1e-6f);
  }
  for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const float gi = g[i] * clip;
    const float mi = b1 * m[i] + (1.f - b1) * gi;
    const float vi = b2 * v[i] + (1.f - b2) * gi * gi;
    m[i] = mi;
    v[i] = vi;
    float pi = p[i];
    pi -= lr * wd * pi;
    pi -= lr * (mi / bc1) / (sqrtf(vi / bc2) + eps);
    p[i] = pi;
    if (p16 != nullptr) p16[i] = __float2bfloat16(pi);
  }
}
void adamw_step(float* p, const float* g, float* m, float* v, bf16* p16, long n, float lr, float b1, float b2,
                float eps, float wd, int step, const float* sqnorm, float max_norm, float grad_scale,
                cudaStream_t st) {
  if (n == 0) return;
  const float bc1 = 1.f - powf(b1, static_cast<float>(step));
  const float bc2 = 1.f - powf(b2, static_cast<float>(step));
  const int blocks = static_cast<int>(std::min<long>((n + 255) / 256, 148L * 16));
  adamw_kernel<<<blocks, 256, 0, st>>>(p, g, m, v, p16, n, lr, b1, b2, eps, wd, bc1, bc2, sqnorm, max_norm,
                                       grad_scale);
}

}  // namespace octo
