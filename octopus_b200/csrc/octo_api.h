// Plain C++ interface between the torch-facing host glue (*.cpp, g++) and the CUDA
// kernel translation units (*.cu, nvcc, no torch headers).  Only POD structs and
// launch functions live here.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace octo {

// Per-device status word (int32): [0] error code, [1] site, [2] runtime wait budget in
// microseconds (0: the compiled default), [3] index rejected by a debug bounds check.
constexpr int kStatusWordsHost = 4;

struct GemmShape {
  int M, N, K;
  int m_tiles, n_tiles, k_blocks, num_tiles;
  int m_shift;  // M-block rotation of the tile order (tensor-parallel: own rows first)
  int k_splits; // split-K factor (0 or 1: none); tiles = k_splits x m_tiles x n_tiles
  int pdl;      // launched as a programmatic dependent: prefetch weights to L2, then wait for the predecessor
  int b_prefetch;  // > 0: the producer keeps L2 prefetches of B this many K-blocks ahead of its loads
  int b_pair;      // > 0: paired B tiles (gated MLP): B rows [nb*BN/2, +BN/2) and [b_pair + nb*BN/2, +BN/2)
                   // form tile nb; the epilogue gets each output chunk's two halves together
};

enum GemmEpiKind : int {
  kEpiBF16 = 0,     // C bf16 = alpha*acc (+ residual)
  kEpiF32 = 1,      // C fp32 = alpha*acc (+ C if accumulate)
  kEpiHeadLse = 2,  // per (row, n-tile) partial (max, sumexp, sum z*exp, label logit)
  kEpiSample = 3,   // per (row, n-tile) partial (max, sumexp, best gumbel score, argmax)
  kEpiHeadGrad = 4, // C bf16 = d(loss)/d(logit) of the logprob head, recomputed from lse/entropy
  kEpiSplitK = 5,   // fp32 partial of one K split -> workspace[split][M][N] (then splitk_finish)
  kEpiSwiGLU = 6,   // C bf16 [M, N] = silu(gate) * up from paired B tiles (b_pair = N)
  kEpiQKVRope = 7,  // C bf16 = acc + bias with the rotary embedding on the q / k heads (BN = head dim)
};

struct GemmLaunch {
  CUtensorMap ta, tb;
  GemmShape s;
  int bn;
  int mt;                  // M-tiles per CTA (1, or 2 for decode-sized M with K-major operands)
  bool a_mn, b_mn;
  int epi;
  void* C;
  int ldc;
  const void* R;
  int ldr;
  float alpha;
  int accumulate;
  // head / sampling epilogue extras
  const int32_t* labels;   // [M] label per row (head) or unused
  float* partial;          // [M, n_tiles, 4] fp32 partials
  uint64_t seed;           // sampling RNG seed
  const int64_t* row_offset;  // sampling: per-row RNG stream id (may be null)
  int vocab_limit;         // columns >= vocab_limit are masked (padding)
  int col_base;            // sampling: global vocabulary index of local column 0
  const void* bias;        // bf16 [N] bias added in the bf16 epilogue (may be null)
  const float* lse;        // head grad: per-row log-normaliser
  const float* ent;        // head grad: per-row entropy
  const float* g_lp;       // head grad: d loss / d logp per row
  const float* g_ent;      // head grad: d loss / d entropy per row
  const int32_t* pos;      // rope epilogue: per-row position
  float rope_log2_theta;   // rope epilogue: log2(rope theta)
  int rope_heads;          // rope epilogue: rotated heads (q + k); later heads are stored unrotated
  int* status;
  int grid;
  cudaStream_t stream;
};

void gemm_launch(const GemmLaunch& g);
// out[M, N] bf16 = sum_s ws[s][M][N] (+ bias[N]) (+ residual[M, N], row stride ldr)
void splitk_finish(const float* ws, int splits, int M, int N, const void* bias, const void* residual, int ldr,
                   void* out, int ldc, cudaStream_t st);
int gemm_smem_bytes(int bn, int mt = 1);

}  // namespace octo
