// Parameter blocks and launchers of attention.cu (no torch types).
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace octo {

struct AttnParams {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  __nv_bfloat16* o;
  float* lse;          // [Hq, Tq] natural-log normaliser (may be null)
  const int32_t* cu_q;     // [nseq + 1] query row ranges
  const int32_t* cu_k;     // [nseq + 1] ranges into key_idx
  const int32_t* key_idx;  // gathered key rows
  const int32_t* tiles;    // [n_tiles, 2] (seq, q0) with q0 a multiple of the CTA's row tile
  int ldq, ldk, ldo;       // row strides (elements)
  int Tq, Hq, Hkv;
  float scale;
  int causal;
  unsigned long long* trace;  // optional per-CTA event timestamps (tcgen05 kernel, debugging)
};

struct AttnBwdParams {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  const __nv_bfloat16* dO;
  const float* lse;    // [Hq, Tq]
  const float* delta;  // [Hq, Tq]
  __nv_bfloat16* dq;   // [Tq, Hq, D]
  float* dk_acc;       // [rows, Hkv, D] fp32 accumulators (row stride ld_acc)
  float* dv_acc;
  const int32_t* cu_q;
  const int32_t* cu_k;
  const int32_t* key_idx;
  const int32_t* tiles;   // [n_qtiles, 2] (seq, q0), q0 multiple of 64
  const int32_t* ktiles;  // [n_ktiles, 2] (seq, k0), k0 multiple of 64
  int ldq, ldk, lddo, lddq;
  long ld_acc;
  int Tq, Hq, Hkv;
  float scale;
  int causal;
};

struct DecodeParams {
  const __nv_bfloat16* q;  // [B, Hq, D] (row stride ldq)
  const __nv_bfloat16* k_cache;  // [slots, Hkv, D]
  const __nv_bfloat16* v_cache;
  __nv_bfloat16* o;        // [B, Hq, D] (row stride ldo)
  const int32_t* kv_start;    // [B] first entry of request b in kv_indices
  const int32_t* kv_len;      // [B] number of keys of request b
  const int32_t* kv_indices;  // slot ids
  float* part_o;    // [B, Hq, splits, D] scratch (splits > 1)
  float* part_lse;  // [B, Hq, splits]
  int ldq, ldk, ldo;
  int Hq, Hkv;
  int num_splits;
  float scale;
};

void attn_fwd(const AttnParams& p, int n_tiles, int D, cudaStream_t st);
void attn_bwd_delta(const __nv_bfloat16* o, int ldo, const __nv_bfloat16* dO, int lddo, float* delta, int Tq, int Hq,
                    int D, cudaStream_t st);
void attn_bwd(const AttnBwdParams& p, int n_qtiles, int n_ktiles, int D, cudaStream_t st);
cudaError_t attn_decode(const DecodeParams& p, int B, int D, cudaStream_t st);  // this call's launch error
// tcgen05/TMEM forward (head_dim 128), same contract as attn_fwd with 128-row query tiles

// TMA maps of the two-query-tile forward: q [Tq, Hq*D] box 64 x 128; k, v [rows, Hkv*D]
// box 64 x 64 (one producer warp's rows), all 128-byte swizzled.
struct AttnMaps {
  CUtensorMap q, k, v;
};
// head_dim 128; tiles [n_tiles, 2] (seq, q0) with q0 a multiple of 256
void attn_fwd_pp(const AttnParams& p, const AttnMaps& maps, int n_tiles, int* status, cudaStream_t st);

// TMA maps of the tcgen05 backward: q, dO [Tq, Hq*D]; k, v [rows, Hkv*D]; all boxes 64 x 64,
// 128-byte swizzled.
struct AttnBwdMaps {
  CUtensorMap q, dO, k, v;
};
// head_dim 128; p.tiles: (seq, q0) with q0 a multiple of 128; p.ktiles: (seq, k0), k0 a
// multiple of 128 (sequences with queries only).  dk_acc / dv_acc are added to.
void attn_bwd_tc(const AttnBwdParams& p, const AttnBwdMaps& maps, int n_qtiles, int n_ktiles, int* status,
                 cudaStream_t st);

}  // namespace octo
