// Tensor-parallel fused kernels over NVLink peer memory (plain C++ interface).
//
// Sync buffer of one TP group member (cudaMalloc'd, IPC-mapped into every rank):
//   int32 flags[kTpSlots][kMaxTp]   flags[s][r] counts signals rank r sent for purpose s
//   int32 done [kTpSlots]           CTA completion counter of the waiting kernel
// A signal is a system-scope release add of 1 into the receiver's flags[s][sender].
// The waiting kernel's last CTA subtracts the number of signals one call delivers, so
// the counters return to zero without host-side sequence numbers (CUDA-graph safe).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "octo_api.h"

namespace octo {

constexpr int kMaxTp = 8;
constexpr int kTpSlots = 16;
constexpr int kTpSyncBytes = (kTpSlots * kMaxTp + kTpSlots) * 4;

// One purpose's counters as seen by rank `me`.
struct TpSlot {
  int* flags;                // local flags[s][*]
  int* peer_flags[kMaxTp];   // rank r's flags[s][*]
  int* done;                 // local done[s]
  int tp, me;
};

// AG -> GEMM: C[M = tp * rows_s, N] = concat_r(X_r)[M, K] @ W[N, K]^T (+ bias), with X_r
// rank r's activation shard.  Every remote row crosses NVLink once: the epilogue warps of all CTAs first copy the
// peers' shards (P2P loads) into a local staging buffer, chunk by chunk from a shared
// work counter, and count finished chunks per M-block; the TMA producer loads an
// M-block holding remote rows once its count is complete.  Tiles of the rank's own
// rows are scheduled first (m_shift) and need no copy.
struct AgLaunch {
  GemmLaunch g;               // B map, shape, bf16 epilogue, bn, grid, stream, status
  CUtensorMap a[kMaxTp];      // rank r's rows [rows_s, K] (own: the shard; peers: staging) box 64 x box_rows
  const void* peer_x[kMaxTp]; // rank r's shard (peer pointers)
  int ldx;                    // shard row stride (elements)
  void* stage;                // local staging [tp * rows_s, K] bf16 (row stride K)
  int* work;                  // local counters: [0] chunk work counter, [1 + mb] chunks staged of M-block mb
  int rows_s, box_rows;
  TpSlot slot;
  int peer_grid;              // signals one call of a peer delivers (its grid)
};
void ag_gemm_launch(const AgLaunch& a);

// GEMM -> RS: partial C = A[M, K_loc] @ W[N, K_loc]^T; rows of rank p's shard are stored
// (bf16) into p's receive buffer at [split * tp + me][row - p * rows_s][:] by peer stores
// (split-K for decode-sized M: every split's partial goes to its own slot).
struct RsLaunch {
  GemmLaunch g;
  void* recv[kMaxTp];         // rank r's receive buffer [tp][rows_s][ldc] bf16
  int ldc, rows_s;
  TpSlot slot;
};
void gemm_rs_launch(const RsLaunch& r);

// h[rows_s, N] += sum_r recv[r][rows_s, N] (fixed rank order), optionally
// x = rmsnorm(h) * (w or 1 + w).  Waits for every peer's RS signals first.
// recv holds `parts` = splits * tp partial slices [parts][rows_s][N].
int tp_reduce(const void* recv, int parts, void* h, int ldh, int N, int rows_s, const void* w, void* x, int ldx,
              float eps, int plus_one, const TpSlot& slot, int peer_grid, int* status, cudaStream_t st);

// Vocab-parallel sampling: local combine of the sampling partials, exchange of
// (max, sum, best score, best column) per row with every rank, then the final merge.
int tp_sample_local(const float* part, int M, int T, void* const* xch, const TpSlot& slot, cudaStream_t st);
void tp_sample_final(const void* xch_local, int M, uint64_t seed, const int64_t* row_stream, int64_t* tokens,
                     float* logprob, const TpSlot& slot, int peer_grid, int* status, cudaStream_t st);

// Bounded all-rank barrier on one slot (single CTA).
void tp_barrier(const TpSlot& slot, int* status, cudaStream_t st);

// Strided 2D copies (weight reshard: trainer layout -> TP shard layout); sources may be
// peer pointers.  Segments live in device memory; `first` is the segment's first
// 16-byte chunk in the flattened chunk space.
struct ReshardSeg {
  const void* src;
  void* dst;
  int64_t lds, ldd;   // row strides in elements (bf16)
  int rows, cols;     // cols a multiple of 8
  int64_t first;
};
void reshard_copy(const ReshardSeg* segs, int nseg, int64_t total_chunks, cudaStream_t st);

}  // namespace octo
