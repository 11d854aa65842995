// Linear recurrences of hybrid models (sm_100a): gated delta rule (GDN) and simple
// gated linear attention (the Mamba-2 SSD form), over variable-length segments with
// initial and final states, forward and backward; and a causal depthwise conv1d with
// per-segment context rows.
//
// Recurrences, per segment and head, state S [dv, dk] (fp32), scalar gate a_t = exp(g_t):
//   GDN:  S_t = a_t S_{t-1} + d_t k_t^T,  d_t = beta_t (v_t - a_t S_{t-1} k_t)
//   GLA:  S_t = a_t S_{t-1} + v_t k_t^T          (beta ignored)
//   o_t = scale * S_t q_t
// Rows of S evolve independently given (k, a, beta), so a CTA of dv threads runs one
// (segment, head) with thread j holding row j of S in registers; the token vectors are
// staged in shared memory one token ahead.  The forward writes S every kChunk tokens;
// the backward replays each chunk from its checkpoint into a per-CTA scratch of the
// chunk's states (transposed so every access is coalesced), then walks it in reverse.
// Cross-row reductions (dq, dk, da, dbeta) go through shared memory.
//
// This is the token-serial formulation (work O(T dk dv) per head, no tensor cores); the
// chunked WY form on tcgen05 is the planned fast path.  dk = dv = 128 or 64.
#include <cuda_bf16.h>

#include "common.cuh"
#include "recurrence.h"

namespace octo {

namespace {

constexpr int kChunk = 16;  // checkpoint interval (tokens)

template <int DK>
__device__ __forceinline__ float row_dot(const float (&s)[DK], const float* v) {
  float a = 0.f;
#pragma unroll
  for (int i = 0; i < DK; ++i) a += s[i] * v[i];
  return a;
}

__device__ __forceinline__ float to_f(const __nv_bfloat16* p) { return __bfloat162float(*p); }

}  // namespace

// ------------------------------------------------------------------ forward
template <int DK>
__global__ void __launch_bounds__(DK) recur_fwd_kernel(RecurParams p) {
  const int seg = blockIdx.x, h = blockIdx.y, j = threadIdx.x;  // j: value row
  const int t0 = p.seg_start[seg], T = p.seg_len[seg];
  __shared__ float sk[2][DK], sq[2][DK], sv[2][DK], sab[2][2];
  float S[DK];
  const float* s0 = p.init_state != nullptr && p.init_idx[seg] >= 0
                        ? p.init_state + ((static_cast<size_t>(p.init_idx[seg]) * p.H + h) * DK + j) * DK
                        : nullptr;
#pragma unroll
  for (int i = 0; i < DK; ++i) S[i] = s0 != nullptr ? s0[i] : 0.f;
  auto stage = [&](int t, int b) {
    const size_t r = static_cast<size_t>(t0 + t);
    sk[b][j] = to_f(p.k + r * p.ldk + h * DK + j);
    sq[b][j] = to_f(p.q + r * p.ldq + h * DK + j);
    sv[b][j] = to_f(p.v + r * p.ldv + h * DK + j);
    if (j == 0) {
      sab[b][0] = __expf(p.g[r * p.H + h]);
      sab[b][1] = p.beta != nullptr ? p.beta[r * p.H + h] : 0.f;
    }
  };
  if (T > 0) stage(0, 0);
  __syncthreads();
  for (int t = 0; t < T; ++t) {
    const int b = t & 1;
    if (p.ckpt != nullptr && t % kChunk == 0) {
      float* c = p.ckpt + ((static_cast<size_t>(p.ckpt_off[seg] + t / kChunk) * p.H + h) * DK + j) * DK;
#pragma unroll
      for (int i = 0; i < DK; ++i) c[i] = S[i];
    }
    if (t + 1 < T) stage(t + 1, b ^ 1);
    const float a = sab[b][0];
    if (p.delta) {
      const float d = sab[b][1] * (sv[b][j] - a * row_dot<DK>(S, sk[b]));
#pragma unroll
      for (int i = 0; i < DK; ++i) S[i] = a * S[i] + d * sk[b][i];
    } else {
      const float vj = sv[b][j];
#pragma unroll
      for (int i = 0; i < DK; ++i) S[i] = a * S[i] + vj * sk[b][i];
    }
    const float o = p.scale * row_dot<DK>(S, sq[b]);
    p.o[static_cast<size_t>(t0 + t) * p.ldo + h * DK + j] = __float2bfloat16(o);
    __syncthreads();
  }
  if (p.final_state != nullptr) {
    float* f = p.final_state + ((static_cast<size_t>(seg) * p.H + h) * DK + j) * DK;
#pragma unroll
    for (int i = 0; i < DK; ++i) f[i] = S[i];
  }
}

// ------------------------------------------------------------------ backward
// dS row j in registers; per token (reverse): dS += scale do_j q;  dq_i = scale sum_j S_t[j,i] do_j
// GDN: ddelta_j = dS_j . k; dk_i += sum_j dS[j,i] d_j; da += sum_j dS_j . S-_j;
//      dv_j = beta ddelta_j; dbeta += ddelta_j (v_j - a u_j); du_j = -beta a ddelta_j;
//      da += -beta ddelta_j u_j; dS- = a dS + du_j k (row); dk_i += sum_j du_j S-[j,i]
// GLA: dv_j = dS_j . k; dk_i += sum_j dS[j,i] v_j; da += sum_j dS_j . S-_j; dS- = a dS
template <int DK>
__global__ void __launch_bounds__(DK) recur_bwd_kernel(RecurParams p, RecurGrads gr) {
  const int seg = blockIdx.x, h = blockIdx.y, j = threadIdx.x;
  const int t0 = p.seg_start[seg], T = p.seg_len[seg];
  extern __shared__ float sh[];
  float* red = sh;                    // [DK][DK + 1] cross-row reduction pad
  float* sm = red + DK * (DK + 1);    // S_{t-1} of the current token, [i][j]
  float* vec = sm + DK * DK;          // k, q of the current token + per-warp scalars
  float* sk = vec, *sq = vec + DK;
  float* scratch = p.scratch + (static_cast<size_t>(blockIdx.y) * gridDim.x + blockIdx.x) *
                                   static_cast<size_t>(kChunk + 1) * DK * DK;  // [t][i][j]
  float dS[DK];
  const float* dfin = gr.d_final != nullptr ? gr.d_final + ((static_cast<size_t>(seg) * p.H + h) * DK + j) * DK
                                            : nullptr;
#pragma unroll
  for (int i = 0; i < DK; ++i) dS[i] = dfin != nullptr ? dfin[i] : 0.f;
  const int nch = (T + kChunk - 1) / kChunk;
  for (int c = nch - 1; c >= 0; --c) {
    const int a0 = c * kChunk, a1 = min(T, a0 + kChunk);
    // replay the chunk from its checkpoint: scratch[t - a0] = S_{t-1} (row j at [i][j]);
    // the replayed state lives in shared memory (dS already occupies the registers)
    {
      const float* ck = p.ckpt + ((static_cast<size_t>(p.ckpt_off[seg] + c) * p.H + h) * DK + j) * DK;
      for (int i = 0; i < DK; ++i) sm[i * DK + j] = ck[i];
      for (int t = a0; t < a1; ++t) {
        float* dst = scratch + static_cast<size_t>(t - a0) * DK * DK;
        for (int i = 0; i < DK; ++i) dst[i * DK + j] = sm[i * DK + j];
        const size_t r = static_cast<size_t>(t0 + t);
        sk[j] = to_f(p.k + r * p.ldk + h * DK + j);
        __syncthreads();
        const float a = __expf(p.g[r * p.H + h]);
        const float vj = to_f(p.v + r * p.ldv + h * DK + j);
        float d = vj;
        if (p.delta) {
          float u = 0.f;
          for (int i = 0; i < DK; ++i) u += sm[i * DK + j] * sk[i];
          d = p.beta[r * p.H + h] * (vj - a * u);
        }
        for (int i = 0; i < DK; ++i) sm[i * DK + j] = a * sm[i * DK + j] + d * sk[i];
        __syncthreads();
      }
    }
    __syncthreads();
    for (int t = a1 - 1; t >= a0; --t) {
      const size_t r = static_cast<size_t>(t0 + t);
      const float* prev = scratch + static_cast<size_t>(t - a0) * DK * DK;  // S_{t-1}, [i][j]
      // S_{t-1} into shared memory ([i][j]: thread j reads column entries conflict-free)
      for (int i = 0; i < DK; ++i) sm[i * DK + j] = prev[i * DK + j];
      sk[j] = to_f(p.k + r * p.ldk + h * DK + j);
      sq[j] = to_f(p.q + r * p.ldq + h * DK + j);
      __syncthreads();
      const float a = __expf(p.g[r * p.H + h]);
      const float beta = p.delta ? p.beta[r * p.H + h] : 0.f;
      const float vj = to_f(p.v + r * p.ldv + h * DK + j);
      const float doj = p.scale * to_f(gr.d_o + r * p.ldo + h * DK + j);
      float u = 0.f;
      if (p.delta) {
        for (int i = 0; i < DK; ++i) u += sm[i * DK + j] * sk[i];
      }
      const float d = p.delta ? beta * (vj - a * u) : vj;
      // S_t row j (for dq) and dS += do_j q
#pragma unroll
      for (int i = 0; i < DK; ++i) {
        const float st = a * sm[i * DK + j] + d * sk[i];
        red[i * (DK + 1) + j] = st * doj;  // dq_i contributions (summed over rows j)
        dS[i] += doj * sq[i];
      }
      __syncthreads();
      {
        float s2 = 0.f;
        for (int jj = 0; jj < DK; ++jj) s2 += red[j * (DK + 1) + jj];
        gr.dq[r * p.ldq + h * DK + j] = __float2bfloat16(s2);
      }
      __syncthreads();
      float dd = 0.f, da = 0.f;  // d(loss)/d d_j, and the gate gradient part <dS_j, S-_j>
#pragma unroll
      for (int i = 0; i < DK; ++i) {
        dd += dS[i] * sk[i];
        da += dS[i] * sm[i * DK + j];
      }
      float du = 0.f, dbeta = 0.f, dvj;
      if (p.delta) {
        dvj = beta * dd;
        dbeta = dd * (vj - a * u);
        du = -beta * a * dd;
        da += -beta * dd * u;
      } else {
        dvj = dd;
      }
      gr.dv[r * p.ldv + h * DK + j] = __float2bfloat16(dvj);
      // dk_i = sum_j (dS[j,i] d_j + du_j S-[j,i]);  then dS <- dS_{t-1} = a dS + du_j k
#pragma unroll
      for (int i = 0; i < DK; ++i) {
        red[i * (DK + 1) + j] = dS[i] * d + du * sm[i * DK + j];
        dS[i] = a * dS[i] + du * sk[i];
      }
      float* sc = vec + 2 * DK;
      const float wda = warp_sum(da), wdb = warp_sum(dbeta);
      if ((j & 31) == 0) {
        sc[(j >> 5) * 2] = wda;
        sc[(j >> 5) * 2 + 1] = wdb;
      }
      __syncthreads();
      {
        float s2 = 0.f;
        for (int jj = 0; jj < DK; ++jj) s2 += red[j * (DK + 1) + jj];
        gr.dk[r * p.ldk + h * DK + j] = __float2bfloat16(s2);
      }
      if (j == 0) {
        float ta = 0.f, tb = 0.f;
        for (int w = 0; w < DK / 32; ++w) {
          ta += sc[2 * w];
          tb += sc[2 * w + 1];
        }
        gr.dg[r * p.H + h] = ta * a;  // a = exp(g)
        if (gr.dbeta != nullptr) gr.dbeta[r * p.H + h] = tb;
      }
      __syncthreads();
    }
  }
  if (gr.d_init != nullptr) {
    float* di = gr.d_init + ((static_cast<size_t>(seg) * p.H + h) * DK + j) * DK;
#pragma unroll
    for (int i = 0; i < DK; ++i) di[i] = dS[i];
  }
}

int recur_chunk() { return kChunk; }

size_t recur_scratch_floats(int n_seg, int H, int dk) {
  return static_cast<size_t>(n_seg) * H * (kChunk + 1) * dk * dk;
}

void recur_fwd(const RecurParams& p, int n_seg, int dk, cudaStream_t st) {
  if (n_seg == 0) return;
  if (dk == 128) recur_fwd_kernel<128><<<dim3(n_seg, p.H), 128, 0, st>>>(p);
  else recur_fwd_kernel<64><<<dim3(n_seg, p.H), 64, 0, st>>>(p);
}

void recur_bwd(const RecurParams& p, const RecurGrads& g, int n_seg, int dk, cudaStream_t st) {
  if (n_seg == 0) return;
  const size_t smem = (static_cast<size_t>(dk) * (dk + 1) + static_cast<size_t>(dk) * dk + 2 * dk + 16) * sizeof(float);
  if (dk == 128) {
    cudaFuncSetAttribute(recur_bwd_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    recur_bwd_kernel<128><<<dim3(n_seg, p.H), 128, smem, st>>>(p, g);
  } else {
    cudaFuncSetAttribute(recur_bwd_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    recur_bwd_kernel<64><<<dim3(n_seg, p.H), 64, smem, st>>>(p, g);
  }
}

// ------------------------------------------------------------------ causal depthwise conv1d
// y[t, c] = bias[c] + sum_{w < W} x[t - (W - 1) + w, c] * wt[c, w], rows before a segment's
// start taken from its context ctx[seg][W - 1][C] (zeros when ctx_idx < 0); optional SiLU.
__global__ void conv_fwd_kernel(ConvParams p) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const int seg = blockIdx.y;
  if (c >= p.C) return;
  const int t0 = p.cu[seg], T = p.cu[seg + 1] - t0;
  const int W = p.W;
  float hist[8];
  const float* ctx = p.ctx != nullptr && p.ctx_idx[seg] >= 0 ? p.ctx + static_cast<size_t>(p.ctx_idx[seg]) * (W - 1) * p.C
                                                              : nullptr;
  for (int w = 0; w < W - 1; ++w) hist[w] = ctx != nullptr ? ctx[static_cast<size_t>(w) * p.C + c] : 0.f;
  float wt[8];
  for (int w = 0; w < W; ++w) wt[w] = p.w[c * W + w];
  const float b = p.bias != nullptr ? p.bias[c] : 0.f;
  for (int t = 0; t < T; ++t) {
    const float x = to_f(p.x + static_cast<size_t>(t0 + t) * p.ldx + c);
    float y = b + wt[W - 1] * x;
    for (int w = 0; w < W - 1; ++w) y += wt[w] * hist[w];
    for (int w = 0; w + 1 < W - 1; ++w) hist[w] = hist[w + 1];
    if (W > 1) hist[W - 2] = x;
    if (p.silu) y = y / (1.f + __expf(-y));
    p.y[static_cast<size_t>(t0 + t) * p.ldy + c] = __float2bfloat16(y);
  }
}

// backward: dpre = dy * silu'(pre) (pre recomputed); dx[t] = sum_w dpre[t + (W-1) - w] wt[w];
// dw[c, w] += sum_t dpre[t] x[t - (W-1) + w]; dbias[c] += sum_t dpre[t]; dctx for context rows.
__global__ void conv_bwd_kernel(ConvParams p, const __nv_bfloat16* __restrict__ dy, __nv_bfloat16* dx, float* dw,
                                float* dbias, float* dctx) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const int seg = blockIdx.y;
  if (c >= p.C) return;
  const int t0 = p.cu[seg], T = p.cu[seg + 1] - t0;
  const int W = p.W;
  const float* ctx = p.ctx != nullptr && p.ctx_idx[seg] >= 0 ? p.ctx + static_cast<size_t>(p.ctx_idx[seg]) * (W - 1) * p.C
                                                              : nullptr;
  float wt[8];
  for (int w = 0; w < W; ++w) wt[w] = p.w[c * W + w];
  const float b = p.bias != nullptr ? p.bias[c] : 0.f;
  auto xat = [&](int t) -> float {  // input row t of the segment (t < 0: context)
    if (t >= 0) return to_f(p.x + static_cast<size_t>(t0 + t) * p.ldx + c);
    const int w = t + (W - 1);
    return ctx != nullptr && w >= 0 ? ctx[static_cast<size_t>(w) * p.C + c] : 0.f;
  };
  auto dpre_at = [&](int t) -> float {
    float y = b;
    for (int w = 0; w < W; ++w) y += wt[w] * xat(t - (W - 1) + w);
    float g = to_f(dy + static_cast<size_t>(t0 + t) * p.ldy + c);
    if (p.silu) {
      const float s = 1.f / (1.f + __expf(-y));
      g *= s * (1.f + y * (1.f - s));
    }
    return g;
  };
  float gw[8] = {0, 0, 0, 0, 0, 0, 0, 0}, gb = 0.f;
  float dctx_acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  float dp[8];  // dpre[t .. t + W - 1] window
  for (int w = 0; w < W; ++w) dp[w] = (w < T) ? dpre_at(w) : 0.f;
  for (int t = 0; t < T; ++t) {
    // dx[t] = sum_w dpre[t + (W - 1) - w] wt[w]
    float g = 0.f;
    for (int w = 0; w < W; ++w) {
      const int u = t + (W - 1) - w;
      if (u < T) g += dp[u - t] * wt[w];
    }
    dx[static_cast<size_t>(t0 + t) * p.ldx + c] = __float2bfloat16(g);
    const float d0 = dp[0];
    gb += d0;
    for (int w = 0; w < W; ++w) gw[w] += d0 * xat(t - (W - 1) + w);
    for (int w = 0; w + 1 < W; ++w) dp[w] = dp[w + 1];
    dp[W - 1] = (t + W < T) ? dpre_at(t + W) : 0.f;
  }
  // context rows feed the first W - 1 outputs
  for (int t = 0; t < min(T, W - 1); ++t) {
    const float d = dpre_at(t);
    for (int w = 0; w < W; ++w) {
      const int src = t - (W - 1) + w;  // < 0: context row src + (W - 1)
      if (src < 0) dctx_acc[src + (W - 1)] += d * wt[w];
    }
  }
  for (int w = 0; w < W; ++w) atomicAdd(&dw[c * W + w], gw[w]);
  if (dbias != nullptr) atomicAdd(&dbias[c], gb);
  if (dctx != nullptr)
    for (int w = 0; w < W - 1; ++w) dctx[(static_cast<size_t>(seg) * (W - 1) + w) * p.C + c] = dctx_acc[w];
}

void conv_fwd(const ConvParams& p, int n_seg, cudaStream_t st) {
  if (n_seg == 0) return;
  conv_fwd_kernel<<<dim3((p.C + 127) / 128, n_seg), 128, 0, st>>>(p);
}

void conv_bwd(const ConvParams& p, int n_seg, const void* dy, void* dx, float* dw, float* dbias, float* dctx,
              cudaStream_t st) {
  if (n_seg == 0) return;
  conv_bwd_kernel<<<dim3((p.C + 127) / 128, n_seg), 128, 0, st>>>(
      p, static_cast<const __nv_bfloat16*>(dy), static_cast<__nv_bfloat16*>(dx), dw, dbias, dctx);
}

}  // namespace octo
