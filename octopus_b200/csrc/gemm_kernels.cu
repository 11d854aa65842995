// Instantiations and launcher of the tcgen05 GEMM (no torch headers in this unit).
#include <algorithm>

#include "gemm_sm100.cuh"
#include "head_epilogue.cuh"

namespace octo {

int gemm_smem_bytes(int bn, int mt) {
  if (mt == 2) return bn == 256 ? GemmCfg<256, 2>::kSmemBytes : GemmCfg<128, 2>::kSmemBytes;
  return bn == 256 ? GemmCfg<256>::kSmemBytes : (bn == 128 ? GemmCfg<128>::kSmemBytes : GemmCfg<64>::kSmemBytes);
}

template <int BN, bool A_MN, bool B_MN, class Epi, int MT = 1>
static void launch_one(const GemmLaunch& g, const Epi& epi) {
  using Cfg = GemmCfg<BN, MT>;
  auto kern = gemm_tcgen05_kernel<BN, A_MN, B_MN, Epi, ALocal<A_MN>, MT>;
  static SmemOptIn opt;  // the attribute is set per device context
  opt.ensure(kern, Cfg::kSmemBytes);
  if (!g.s.pdl) {
    kern<<<g.grid, kGemmThreads, Cfg::kSmemBytes, g.stream>>>(ALocal<A_MN>{g.ta}, g.tb, g.s, epi, g.status);
    return;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(g.grid);
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cfg.stream = g.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kern, ALocal<A_MN>{g.ta}, g.tb, g.s, epi, g.status);
}

template <int BN, class Epi>
static void by_major(const GemmLaunch& g, const Epi& epi) {
  if (!g.a_mn && !g.b_mn) launch_one<BN, false, false>(g, epi);
  else if (!g.a_mn && g.b_mn) launch_one<BN, false, true>(g, epi);
  else if (g.a_mn && !g.b_mn) launch_one<BN, true, false>(g, epi);
  else launch_one<BN, true, true>(g, epi);
}

template <class Epi>
static void by_bn(const GemmLaunch& g, const Epi& epi) {
  if (g.mt == 2) {  // decode-sized M, K-major operands (chosen by the host)
    if (g.bn == 256) launch_one<256, false, false, Epi, 2>(g, epi);
    else launch_one<128, false, false, Epi, 2>(g, epi);
    return;
  }
  if (g.bn == 256) by_major<256>(g, epi);
  else if (g.bn == 128) by_major<128>(g, epi);
  else by_major<64>(g, epi);
}

void gemm_launch(const GemmLaunch& g) {
  if (g.epi == kEpiBF16) {
    EpiBF16 e{reinterpret_cast<__nv_bfloat16*>(g.C), g.ldc, reinterpret_cast<const __nv_bfloat16*>(g.R), g.ldr,
              g.alpha, reinterpret_cast<const __nv_bfloat16*>(g.bias)};
    by_bn(g, e);
  } else if (g.epi == kEpiF32) {
    EpiF32 e{reinterpret_cast<float*>(g.C), g.ldc, g.alpha, g.accumulate};
    by_bn(g, e);
  } else if (g.epi == kEpiHeadLse) {
    EpiHeadLse e{g.labels, g.partial, g.s.n_tiles, g.bn, g.alpha, g.vocab_limit};
    // head GEMMs are always K-major x K-major (hidden rows x vocab rows)
    if (g.bn == 256) launch_one<256, false, false>(g, e);
    else launch_one<128, false, false>(g, e);
  } else if (g.epi == kEpiHeadGrad) {
    EpiHeadGrad e{reinterpret_cast<__nv_bfloat16*>(g.C), g.ldc, g.labels, g.lse, g.ent, g.g_lp, g.g_ent, g.alpha,
                  g.vocab_limit};
    if (g.bn == 256) launch_one<256, false, false>(g, e);
    else launch_one<128, false, false>(g, e);
  } else if (g.epi == kEpiSplitK) {
    EpiSplitK e{reinterpret_cast<float*>(g.C), g.s.M, g.s.N, nullptr};
    by_bn(g, e);
  } else if (g.epi == kEpiSwiGLU) {
    EpiSwiGLU e{reinterpret_cast<__nv_bfloat16*>(g.C), g.ldc};
    if (g.mt == 2) launch_one<256, false, false, EpiSwiGLU, 2>(g, e);
    else launch_one<256, false, false>(g, e);
  } else if (g.epi == kEpiQKVRope) {
    EpiQKVRope e{reinterpret_cast<__nv_bfloat16*>(g.C), g.ldc, reinterpret_cast<const __nv_bfloat16*>(g.bias), g.pos,
                 g.rope_log2_theta, g.rope_heads, g.bn};
    if (g.bn == 128) launch_one<128, false, false>(g, e);
    else launch_one<64, false, false>(g, e);
  } else if (g.epi == kEpiSample) {
    EpiSample e{g.partial, g.s.n_tiles, g.bn, g.alpha, g.vocab_limit, g.seed, g.row_offset, g.col_base};
    if (g.bn == 256) launch_one<256, false, false>(g, e);
    else if (g.bn == 128) launch_one<128, false, false>(g, e);
    else launch_one<64, false, false>(g, e);
  }
}

// out = sum of the split partials (+ bias) (+ residual), 8 columns per thread
__global__ void splitk_finish_kernel(const float* __restrict__ ws, int splits, int M, int N,
                                     const __nv_bfloat16* __restrict__ bias, const __nv_bfloat16* __restrict__ res,
                                     int ldr, __nv_bfloat16* __restrict__ out, int ldc) {
  grid_dep_launch();
  const int n8 = N / 8;
  const size_t total = static_cast<size_t>(M) * n8;
  const size_t plane = static_cast<size_t>(M) * N;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int row = static_cast<int>(i / n8), c = static_cast<int>(i - static_cast<size_t>(row) * n8) * 8;
    float a[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) a[e] = 0.f;
    const float* p = ws + static_cast<size_t>(row) * N + c;
    for (int s = 0; s < splits; ++s) {
      const float4 x = *reinterpret_cast<const float4*>(p + s * plane);
      const float4 y = *reinterpret_cast<const float4*>(p + s * plane + 4);
      a[0] += x.x; a[1] += x.y; a[2] += x.z; a[3] += x.w;
      a[4] += y.x; a[5] += y.y; a[6] += y.z; a[7] += y.w;
    }
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
    store8(out + static_cast<size_t>(row) * ldc + c, a);
  }
}

void splitk_finish(const float* ws, int splits, int M, int N, const void* bias, const void* residual, int ldr,
                   void* out, int ldc, cudaStream_t st) {
  const size_t total = static_cast<size_t>(M) * (N / 8);
  if (total == 0) return;
  const int grid = static_cast<int>(std::min<size_t>((total + 255) / 256, 148 * 8));
  splitk_finish_kernel<<<grid, 256, 0, st>>>(ws, splits, M, N, static_cast<const __nv_bfloat16*>(bias),
                                             static_cast<const __nv_bfloat16*>(residual), ldr,
                                             static_cast<__nv_bfloat16*>(out), ldc);
}

}  // namespace octo
