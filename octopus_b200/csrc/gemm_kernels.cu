// Instantiations and launcher of the tcgen05 GEMM (no torch headers in this unit).
#include "gemm_sm100.cuh"
#include "head_epilogue.cuh"

namespace octo {

int gemm_smem_bytes(int bn) {
  return bn == 256 ? GemmCfg<256>::kSmemBytes : (bn == 128 ? GemmCfg<128>::kSmemBytes : GemmCfg<64>::kSmemBytes);
}

template <int BN, bool A_MN, bool B_MN, class Epi>
static void launch_one(const GemmLaunch& g, const Epi& epi) {
  using Cfg = GemmCfg<BN>;
  auto kern = gemm_tcgen05_kernel<BN, A_MN, B_MN, Epi>;
  static bool configured = false;  // attribute is per function, not per device context
  if (!configured) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
    configured = true;
  }
  kern<<<g.grid, kGemmThreads, Cfg::kSmemBytes, g.stream>>>(ALocal<A_MN>{g.ta}, g.tb, g.s, epi, g.status);
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
  } else if (g.epi == kEpiSample) {
    EpiSample e{g.partial, g.s.n_tiles, g.bn, g.alpha, g.vocab_limit, g.seed, g.row_offset, g.col_base};
    if (g.bn == 256) launch_one<256, false, false>(g, e);
    else if (g.bn == 128) launch_one<128, false, false>(g, e);
    else launch_one<64, false, false>(g, e);
  }
}

}  // namespace octo
